"""GPU parity of the int4 packing and the dequant-GEMM (ee_pack_int4 /
ee_unpack_int4 / ee_wq_gemm) against the CPU oracle and the reference's
golden outputs. Tolerance (the path's bf16 gate): max|Y - Y_ref| / max|Y_ref| <= 2e-2."""
import numpy as np
import pytest
import torch

from conftest import bits_to_f32, golden
from oracle import quant as OQ

pytestmark = pytest.mark.gpu
TOL = 2e-2


def rel_err(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30)


def test_pack_unpack_bit_exact(cuda):
    from embodied_efficiency_b200 import _pack_int4, _unpack_int4
    g = golden("pack")
    for qk, pk in (("q", "packed"), ("q_all", "packed_all")):
        q = torch.from_numpy(g[qk]).to(cuda)
        p = _pack_int4(q)
        np.testing.assert_array_equal(p.cpu().numpy(), g[pk])
        np.testing.assert_array_equal(_unpack_int4(p).cpu().numpy(), g[qk])
    rng = np.random.default_rng(3)
    q = rng.integers(-8, 8, size=(4096, 4096), dtype=np.int8)
    p = _pack_int4(torch.from_numpy(q).to(cuda))
    np.testing.assert_array_equal(p.cpu().numpy(), OQ.pack_int4(q))
    np.testing.assert_array_equal(_unpack_int4(p).cpu().numpy(), q)
    # empty and odd-K inputs
    assert _pack_int4(torch.empty(0, 8, dtype=torch.int8, device=cuda)).shape == (0, 4)
    with pytest.raises(ValueError):
        _pack_int4(torch.zeros(2, 3, dtype=torch.int8, device=cuda))


def _quant(w, kind, group):
    """(kernel tensors, oracle-dequantised fp32 weight) for one weight format."""
    n, k = w.shape
    if kind == "bf16":
        return dict(weight=torch.from_numpy(w).bfloat16(), bits=16, scales=None, zeros=None,
                    group=0), OQ.round_bf16(w)
    if kind == "int4z":
        u, s16, z16, gs = OQ.quantize_weight_asym4(w, group)
        return dict(weight=torch.from_numpy(OQ.pack_uint4(u)), bits=4, scales=torch.from_numpy(s16),
                    zeros=torch.from_numpy(z16), group=gs), \
            OQ.dequant_asym4(OQ.pack_uint4(u), s16, z16, gs)
    bits = 8 if kind.startswith("int8") else 4
    q, s, gs = OQ.quantize_weight(w, bits, group)
    q2 = q.reshape(n, k)
    wt = OQ.pack_int4(q2) if bits == 4 else q2
    return dict(weight=torch.from_numpy(wt), bits=bits, scales=torch.from_numpy(s.reshape(n, -1)),
                zeros=None, group=gs), OQ.dequantize_weight(q, s, gs)


def _run(cuda, x, w, kind, group, bias=None, act=torch.bfloat16, scale_f16=False, gelu=False,
         residual=None):
    from embodied_efficiency_b200 import wq_linear
    kt, wd = _quant(w, kind, group)
    sc = kt["scales"]
    if sc is not None and scale_f16:
        sc = sc.half()
    xt = torch.from_numpy(x).to(act).to(cuda)
    y = wq_linear(xt, kt["weight"].to(cuda), None if sc is None else sc.to(cuda),
                  None if bias is None else torch.from_numpy(bias).to(act).to(cuda), kt["group"],
                  kt["bits"], zeros=None if kt["zeros"] is None else kt["zeros"].to(cuda), gelu=gelu,
                  residual=None if residual is None else torch.from_numpy(residual).to(act).to(cuda))
    rnd = OQ.round_bf16 if act == torch.bfloat16 else OQ.round_f16
    if scale_f16 and sc is not None and kind != "int4z":
        n = w.shape[0]
        q, s, gs = OQ.quantize_weight(w, 8 if kind.startswith("int8") else 4, group)
        wd = OQ.dequantize_weight(q, s.astype(np.float16).astype(np.float32), gs)
    xr = rnd(x)
    ref = OQ.linear_ref(xr, wd, None if bias is None else rnd(bias), act_round=rnd)
    if gelu:
        import math
        ref = rnd(np.vectorize(lambda v: 0.5 * v * (1 + math.erf(v / math.sqrt(2))))(ref).astype(np.float32))
    if residual is not None:
        ref = rnd(rnd(residual) + ref)
    return y.float().cpu().numpy(), ref


def test_golden_config1_int8_per_channel(cuda):
    g = golden("gemm")
    torch.manual_seed(0)
    x = torch.randn(50, 1024).bfloat16().float().numpy()
    w = (torch.randn(1024, 1024) * 0.02).numpy()
    y, ref = _run(cuda, x, w, "int8", 1024)
    gold = bits_to_f32(g["c1_y"])
    assert rel_err(y, gold) <= TOL
    assert rel_err(y, ref) <= TOL
    # fp16 scales = max|W_row|/127 stored in half (the single int8 per-channel GEMM workload)
    y16, ref16 = _run(cuda, x, w, "int8", 1024, scale_f16=True)
    assert rel_err(y16, ref16) <= TOL and rel_err(y16, gold) <= TOL


def test_golden_small_shapes_with_bias(cuda):
    g = golden("gemm")
    gc = torch.Generator().manual_seed(7)
    for (m, n, k) in ((1, 256, 256), (16, 384, 512), (50, 256, 1024)):
        xs = torch.randn(m, k, generator=gc).bfloat16()
        ws = (torch.randn(n, k, generator=gc) * 0.02).numpy()
        bs = bits_to_f32(g[f"b_{m}_{n}_{k}"])
        torch.randn(n, generator=gc)
        for bits in (8, 4):
            y, ref = _run(cuda, xs.float().numpy(), ws, f"int{bits}", 128, bias=bs)
            gold = bits_to_f32(g[f"y_{m}_{n}_{k}_b{bits}"]).reshape(m, n)
            assert rel_err(y, gold) <= TOL, (m, n, k, bits)
            assert rel_err(y, ref) <= TOL, (m, n, k, bits)


SWEEP_M = [1, 16, 50, 128, 512]
SWEEP_K = [512, 1024, 2048, 4096]
KINDS = [("int8", "pc"), ("int8", 128), ("int4", 128), ("int4z", 128), ("bf16", 0)]


@pytest.mark.parametrize("k", SWEEP_K)
@pytest.mark.parametrize("kind,group", KINDS)
def test_config2_sweep(cuda, k, kind, group):
    """The M x (K=N) x format sweep, against the oracle (fp32-accumulated reference)."""
    rng = np.random.default_rng(k)
    w = (rng.standard_normal((k, k)) * 0.02).astype(np.float32)
    grp = k if group == "pc" else group
    for m in SWEEP_M:
        x = rng.standard_normal((m, k)).astype(np.float32)
        y, ref = _run(cuda, x, w, kind, grp)
        assert rel_err(y, ref) <= TOL, (m, k, kind, group, rel_err(y, ref))


@pytest.mark.parametrize("n,k", [(8192, 8192), (6144, 2048), (8192, 2048), (2048, 8192), (1024, 16384)])
@pytest.mark.parametrize("kind,group", [("int4", 128), ("int8", 128), ("int8", "pc"), ("int4z", 128), ("bf16", 0)])
def test_large_weights_few_tokens(cuda, n, k, kind, group):
    """Weights larger than a streaming CTA's old 16-k-block limit (K / split
    up to 64 k-blocks per CTA, deep stage rings) at the batch-1 token counts,
    against the oracle; the Pi0-scale expert's GEMM shapes among them."""
    rng = np.random.default_rng(n + k)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    grp = k if group == "pc" else group
    for m in (1, 7, 16, 32, 50, 64):
        x = rng.standard_normal((m, k)).astype(np.float32)
        y, ref = _run(cuda, x, w, kind, grp)
        assert rel_err(y, ref) <= TOL, (m, n, k, kind, group, rel_err(y, ref))
    from embodied_efficiency_b200 import wq_gemm
    assert wq_gemm.gemm_status() == 0


@pytest.mark.parametrize("m,n,k", [(3, 200, 128), (77, 130, 384), (65, 1000, 640), (1, 8, 256),
                                   (129, 4096, 1024), (700, 96, 2048)])
@pytest.mark.parametrize("kind", ["int8", "int4", "int4z", "bf16"])
def test_ragged_shapes(cuda, m, n, k, kind):
    rng = np.random.default_rng(m * 7 + n)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    x = rng.standard_normal((m, k)).astype(np.float32)
    b = (rng.standard_normal(n) * 0.1).astype(np.float32)
    y, ref = _run(cuda, x, w, kind, 128 if kind != "bf16" else 0, bias=b)
    assert rel_err(y, ref) <= TOL


@pytest.mark.parametrize("m", [33, 50, 64])
@pytest.mark.parametrize("n,k", [(1000, 128), (136, 384), (4096, 1024), (200, 2048)])
@pytest.mark.parametrize("kind,group", [("int8", 128), ("int8", "pc"), ("int4", 128), ("int4", 256),
                                        ("int4z", 128), ("bf16", 0)])
def test_few_tokens_tensor_core_path(cuda, m, n, k, kind, group):
    """33-64 tokens (the sampler's 50-token batch among them) run the tcgen05
    tile kernel with one token tile: one CTA per unit (K = 128, 384: no split)
    and cluster split-K (K = 1024, 2048), ragged N, per-channel and 256-wide
    groups, every weight kind, bias + GELU and bias + residual epilogues (f16
    activations at 33 tokens), against the oracle."""
    rng = np.random.default_rng(m * 131 + n + k)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    x = rng.standard_normal((m, k)).astype(np.float32)
    b = (rng.standard_normal(n) * 0.1).astype(np.float32)
    grp = k if group == "pc" or (group and k % group) else group  # 256-wide groups where K allows
    y, ref = _run(cuda, x, w, kind, grp, bias=b, gelu=True)
    assert rel_err(y, ref) <= TOL, (m, n, k, kind, group, rel_err(y, ref))
    r = rng.standard_normal((m, n)).astype(np.float32)
    y, ref = _run(cuda, x, w, kind, grp, bias=b, residual=r, act=torch.float16 if m == 33 else torch.bfloat16)
    assert rel_err(y, ref) <= TOL, (m, n, k, kind, group, rel_err(y, ref))
    from embodied_efficiency_b200 import wq_gemm
    assert wq_gemm.gemm_status() == 0


@pytest.mark.parametrize("kind", ["int8", "int4", "bf16"])
def test_epilogues_and_fp16(cuda, kind):
    rng = np.random.default_rng(11)
    m, n, k = 50, 512, 1024
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    x = rng.standard_normal((m, k)).astype(np.float32)
    b = (rng.standard_normal(n) * 0.1).astype(np.float32)
    r = rng.standard_normal((m, n)).astype(np.float32)
    grp = 128 if kind != "bf16" else 0
    y, ref = _run(cuda, x, w, kind, grp, bias=b, gelu=True)
    assert rel_err(y, ref) <= TOL
    y, ref = _run(cuda, x, w, kind, grp, bias=b, residual=r)
    assert rel_err(y, ref) <= TOL
    y, ref = _run(cuda, x, w, kind, grp, bias=b, act=torch.float16)
    assert rel_err(y, ref) <= TOL


@pytest.mark.parametrize("kind", ["int8", "int4", "int4z", "bf16"])
def test_more_tiles_than_sms(cuda, kind):
    """M=2600, N=2048, K=256: 11 x 16 tiles of 256 tokens, more than the SMs,
    so the persistent form of the tensor-core GEMM runs (tiles looped per CTA,
    epilogue overlapped, a ragged last token tile) -- bias, GELU and residual
    epilogues against the oracle."""
    rng = np.random.default_rng(29)
    m, n, k = 2600, 2048, 256
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    x = rng.standard_normal((m, k)).astype(np.float32)
    b = (rng.standard_normal(n) * 0.1).astype(np.float32)
    grp = 128 if kind != "bf16" else 0
    y, ref = _run(cuda, x, w, kind, grp, bias=b)
    assert rel_err(y, ref) <= TOL
    r = rng.standard_normal((m, n)).astype(np.float32)
    y, ref = _run(cuda, x, w, kind, grp, bias=b, residual=r)
    assert rel_err(y, ref) <= TOL
    if kind == "int4":
        y, ref = _run(cuda, x, w, kind, grp, bias=b, gelu=True)
        assert rel_err(y, ref) <= TOL


def test_fp32_activations_and_errors(cuda):
    from embodied_efficiency_b200 import wq_linear
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((256, 512)) * 0.02).astype(np.float32)
    x = rng.standard_normal((10, 512)).astype(np.float32)
    kt, wd = _quant(w, "int8", 128)
    y = wq_linear(torch.from_numpy(x).to(cuda), kt["weight"].to(cuda), kt["scales"].to(cuda), None,
                  128, 8)
    assert y.dtype == torch.float32
    assert rel_err(y.cpu().numpy(), x @ wd.T) <= TOL
    with pytest.raises(RuntimeError):  # K not a multiple of 128
        wq_linear(torch.zeros(2, 96, device=cuda, dtype=torch.bfloat16),
                  torch.zeros(8, 96, dtype=torch.int8, device=cuda),
                  torch.ones(8, 1, device=cuda), None, 96, 8)
    with pytest.raises(RuntimeError):  # CPU tensors: no CPU path
        wq_linear(torch.zeros(2, 128), torch.zeros(8, 128, dtype=torch.int8),
                  torch.ones(8, 1), None, 128, 8)


def test_reference_correctness_check(cuda):
    """kernel/triton_gemm.py:198-210 on our kernels (published T4 error 1.95e-3)."""
    from embodied_efficiency_b200 import correctness_check
    errs = correctness_check()
    assert all(e < 5e-1 for e in errs.values())


def test_quant_linear_module(cuda):
    from embodied_efficiency_b200 import TritonQuantLinear, quantize_weight
    torch.manual_seed(2)
    lin = torch.nn.Linear(1024, 768).to(cuda).bfloat16()
    x = torch.randn(4, 50, 1024, device=cuda, dtype=torch.bfloat16)
    for bits in (8, 4):
        ql = TritonQuantLinear(lin, bits).to(cuda)
        q, s, gs = quantize_weight(lin.weight.detach().float().cpu(), bits, 128)
        wd = (q.float() * s).reshape(768, 1024)
        ref = torch.nn.functional.linear(x.float().cpu(), wd.bfloat16().float(),
                                         lin.bias.detach().float().cpu())
        with torch.no_grad():
            y = ql(x)
        assert y.shape == (4, 50, 768) and y.dtype == torch.bfloat16
        assert rel_err(y.float().cpu().numpy(), ref.numpy()) <= TOL
        assert ql.weight.dtype == (torch.uint8 if bits == 4 else torch.int8)
        assert ql.scales.dtype == torch.float32 and ql.scales.shape == (768, 8)


@pytest.mark.parametrize("act", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("kind,group", [("int8", 1024), ("int8", 128), ("int4", 128), ("int4z", 128)])
def test_dequant_weight_bit_exact(cuda, kind, group, act):
    """ee_dequant_weight against the oracle's dequantisation with the GEMM's
    rounding: the exact integer times the scale rounded to the activation
    type, one rounding (zero-point form: v - z, exact, then times the scale)."""
    from embodied_efficiency_b200.wq_gemm import dequant_weight
    rng = np.random.default_rng(7)
    n, k = 384, 1024
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    kt, _ = _quant(w, kind, group)
    z = None if kt["zeros"] is None else kt["zeros"].to(cuda)
    got = dequant_weight(kt["weight"].to(cuda), kt["scales"].to(cuda), kt["group"], kt["bits"], act, zeros=z)
    assert got.shape == (n, k) and got.dtype == act
    rnd = OQ.round_bf16 if act == torch.bfloat16 else OQ.round_f16
    gs = kt["group"]
    ng = k // gs
    s = rnd(kt["scales"].numpy().astype(np.float32)).reshape(n, ng, 1)
    if kind == "int4z":
        v = OQ.unpack_uint4(kt["weight"].numpy()).astype(np.float32)
        v = v.reshape(n, ng, gs) - kt["zeros"].numpy().astype(np.float32).reshape(n, ng, 1)
    else:
        wt = kt["weight"].numpy()
        v = (OQ.unpack_int4(wt) if kt["bits"] == 4 else wt).astype(np.float32).reshape(n, ng, gs)
    ref = rnd(v * s).reshape(n, k)
    assert np.array_equal(got.float().cpu().numpy(), ref)


def test_quant_linear_dense_copy_for_many_tokens(cuda):
    """From DENSE_MIN_TOKENS tokens on, TritonQuantLinear runs on a cached
    dense copy of its weight: the same result within the GEMM tolerance, one
    copy reused across calls, rebuilt when the weight changes, and kept out
    of state_dict."""
    from embodied_efficiency_b200 import TritonQuantLinear
    from embodied_efficiency_b200.wq_gemm import DENSE_MIN_TOKENS
    torch.manual_seed(3)
    lin = torch.nn.Linear(1024, 1024).to(cuda).bfloat16()
    x = torch.randn(DENSE_MIN_TOKENS + 77, 1024, device=cuda, dtype=torch.bfloat16)
    for bits in (8, 4):
        ql = TritonQuantLinear(lin, bits).to(cuda)
        with torch.no_grad():
            y = ql(x)
            dense = ql.__dict__["_dense"][1]
            y2 = ql(x)
        assert ql.__dict__["_dense"][1] is dense
        assert torch.equal(y, y2)
        packed = ql.linear(x[:DENSE_MIN_TOKENS - 1])  # below the threshold: the packed weights
        assert rel_err(y[:DENSE_MIN_TOKENS - 1].float().cpu().numpy(), packed.float().cpu().numpy()) <= TOL
        ref = torch.nn.functional.linear(x.float(), dense.float(), lin.bias.detach().float())
        assert rel_err(y.float().cpu().numpy(), ref.cpu().numpy()) <= TOL
        assert set(ql.state_dict()) == {"weight", "scales", "bias"}
        with torch.no_grad():
            ql.scales.mul_(2)
            y3 = ql(x)
        assert ql.__dict__["_dense"][1] is not dense
        assert rel_err(y3.float().cpu().numpy(), (2 * ref - lin.bias.detach().float()).cpu().numpy()) <= TOL


def test_zz_gemm_status_clean(cuda):
    """No launch of this module's tests recorded an in-kernel timeout or a
    launch-shape error."""
    from embodied_efficiency_b200.wq_gemm import gemm_status
    assert gemm_status(reset=True) == 0
