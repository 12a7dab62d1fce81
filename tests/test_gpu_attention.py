"""GPU parity of the attention launch (ee_attention) against an fp32
reference -- F.scaled_dot_product_attention on the same bf16 / fp16 inputs
upcast to fp32 -- and against the bf16 / fp16 SDPA call it replaces on the
layer-by-layer path (kernel/flow_expert.py:86, :91): self-attention read in
place from a fused [q | k | v] projection and cross-attention to a
[batch, P, 2d] prefix K/V."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
TOL = 2e-2  # max |out - ref| / max |ref| (bf16 probabilities in P V, as flash attention)


def _split(x, h):
    b, t, d = x.shape
    return x.view(b, t, h, d // h).transpose(1, 2)


def _merge(x):
    b, h, t, hd = x.shape
    return x.transpose(1, 2).reshape(b, t, h * hd)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("b,n,h,hd,p", [(256, 50, 16, 64, 256), (3, 50, 8, 128, 100), (5, 17, 4, 64, 33),
                                         (41, 64, 16, 64, 64), (7, 50, 16, 64, 700), (300, 50, 8, 128, 50),
                                         (9, 33, 16, 64, 100), (150, 50, 16, 64, 200)])
def test_matches_sdpa(cuda, dtype, b, n, h, hd, p):
    from embodied_efficiency_b200.expert import _attention
    g = torch.Generator(device="cpu").manual_seed(b * 7 + p)
    d = h * hd
    qkv = torch.randn(b, n, 3 * d, generator=g).to(cuda, dtype)
    a = _attention(qkv, 3 * d, qkv[..., d:], 3 * d, qkv[..., 2 * d:], 3 * d, b, h, hd, n, n, n, n)
    q, k, v = qkv.chunk(3, dim=-1)
    _check(a, _split(q, h), _split(k, h), _split(v, h))
    kv = torch.randn(b, p, 2 * d, generator=g).to(cuda, dtype)
    qc = torch.randn(b, n, d, generator=g).to(cuda, dtype)
    kk, vv = _split(kv[..., :d], h), _split(kv[..., d:], h)
    a = _attention(qc, d, kk, 2 * d, vv, 2 * d, b, h, hd, n, p, n, p)
    _check(a, _split(qc, h), kk, vv)


def _check(a, q, k, v):
    """max |a - ref| / max |ref| <= TOL against the fp32 reference and against
    the same-dtype SDPA."""
    ref32 = _merge(F.scaled_dot_product_attention(q.float(), k.float(), v.float()))
    ref = _merge(F.scaled_dot_product_attention(q, k, v)).float()
    torch.cuda.synchronize()
    af = a.float()
    assert float((af - ref32).abs().max()) <= TOL * float(ref32.abs().max())
    assert float((af - ref).abs().max()) <= TOL * float(ref.abs().max())


def test_rejects_long_query_blocks(cuda):
    from embodied_efficiency_b200.expert import _attention
    x = torch.randn(1, 65, 3 * 256, device=cuda, dtype=torch.bfloat16)
    assert _attention(x, 768, x[..., 256:], 768, x[..., 512:], 768, 1, 4, 64, 65, 65, 65, 65) is None
