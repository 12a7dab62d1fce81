"""GPU parity of the LayerNorm row kernel (ee_layer_norm) against an fp32
reference (F.layer_norm of the same inputs upcast to fp32) and against
torch's bf16 / fp16 nn.LayerNorm, the op it replaces on the layer-by-layer
path."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _ln(x, w, b, eps):
    from embodied_efficiency_b200 import _lib
    from embodied_efficiency_b200.expert import _apply_norm
    m = torch.nn.LayerNorm(x.shape[-1], eps=eps).to(x.device, x.dtype)
    with torch.no_grad():
        m.weight.copy_(w)
        m.bias.copy_(b)
    with torch.no_grad():
        return _apply_norm(m, x), m(x)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,cols", [(12800, 1024), (3, 256), (1001, 2048), (50, 8), (40000, 512), (777, 1000)])
def test_matches_torch_layer_norm(cuda, dtype, rows, cols):
    g = torch.Generator(device="cpu").manual_seed(rows + cols)
    x = (torch.randn(rows, cols, generator=g) * 3 + 0.5).to(cuda, dtype)
    w = (torch.randn(cols, generator=g) * 0.5 + 1).to(cuda, dtype)
    b = (torch.randn(cols, generator=g) * 0.1).to(cuda, dtype)
    y, ref = _ln(x, w, b, 1e-5)
    ref32 = F.layer_norm(x.float(), (cols,), w.float(), b.float(), 1e-5)
    torch.cuda.synchronize()
    ulp = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10
    # fp32 statistics, one rounding of the fp32 result: within half a unit
    # in the last place of the fp32 reference (plus summation-order noise)
    d32 = (y.float() - ref32).abs()
    assert bool((d32 <= 0.5 * ulp * ref32.abs() * 1.01 + 1e-5).all())
    # fp32 statistics differ from torch's only in summation order: at most one
    # rounding step of the output apart, and almost everywhere identical
    diff = (y.float() - ref.detach().float()).abs()
    assert float((diff / ref.float().abs().clamp_min(1.0)).max()) <= 2 * ulp
    assert float((diff > 0).float().mean()) < 0.01


def test_batched_shape_and_fallbacks(cuda):
    from embodied_efficiency_b200 import _lib
    x = torch.randn(4, 50, 512, device=cuda, dtype=torch.bfloat16)
    w = torch.ones(512, device=cuda, dtype=torch.bfloat16)
    b = torch.zeros(512, device=cuda, dtype=torch.bfloat16)
    y, ref = _ln(x, w, b, 1e-5)
    assert y.shape == x.shape and float((y.float() - ref.float()).abs().max()) <= 2 ** -6
    lib = _lib.load()
    shape_err = 2  # EE_ERR_SHAPE: cols not a multiple of 8, or above 2048
    assert lib.ee_layer_norm(x.data_ptr(), None, None, x.data_ptr(), 4, 12, 12, 12, 1e-5, _lib.EE_BF16,
                             _lib.stream_ptr(cuda)) == shape_err
    assert lib.ee_layer_norm(x.data_ptr(), None, None, x.data_ptr(), 4, 4096, 4096, 4096, 1e-5, _lib.EE_BF16,
                             _lib.stream_ptr(cuda)) == shape_err
