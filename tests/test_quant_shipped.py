"""The shipped quantiser (``embodied_efficiency_b200.quant.quantize_weight``,
the function ``TritonQuantLinear`` runs at load time, on the GPU when the
module lives there) against the reference's own outputs in
``tests/golden/quant.npz`` (kernel/quant.py:22-30): bit-exact ``q``, ``scale``
and group size, for int8 / int4, group 128 and the per-row fallback, on the
CPU and on a CUDA device."""
import numpy as np
import pytest
import torch

from conftest import golden

CASES = [("a", 128), ("a", 256), ("b", 128), ("b", 96), ("c", 128), ("c", 1024)]


def _check(device):
    from embodied_efficiency_b200.quant import quantize_weight
    g = golden("quant")
    for case, gsz in CASES:
        w = torch.from_numpy(g[f"{case}_w"]).to(device)
        for bits in (8, 4):
            q, s, gs = quantize_weight(w, bits, gsz)
            key = f"{case}_b{bits}_g{gsz}"
            assert q.dtype == torch.int8 and s.dtype == torch.float32
            np.testing.assert_array_equal(q.cpu().numpy(), g[f"{key}_q"], err_msg=key)
            np.testing.assert_array_equal(s.cpu().numpy(), g[f"{key}_s"], err_msg=key)
            assert gs == int(g[f"{key}_gs"]), key


def test_shipped_quantize_weight_bit_exact_cpu():
    _check("cpu")


@pytest.mark.gpu
def test_shipped_quantize_weight_bit_exact_gpu(cuda):
    _check(cuda)


@pytest.mark.gpu
def test_quantized_module_buffers_match_reference_quantiser(cuda):
    """TritonQuantLinear built on the GPU holds exactly the reference
    quantiser's integers (int8 as stored, int4 after unpacking) and scales."""
    from embodied_efficiency_b200 import TritonQuantLinear
    from embodied_efficiency_b200.wq_gemm import _unpack_int4
    from oracle import quant as OQ
    g = torch.Generator().manual_seed(3)
    lin = torch.nn.Linear(512, 384)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(384, 512, generator=g) * 0.02)
    for bits in (8, 4):
        ql = TritonQuantLinear(lin.to(cuda), bits)
        q_ref, s_ref, _ = OQ.quantize_weight(lin.weight.detach().float().cpu().numpy(), bits, 128)
        q = ql.weight if bits == 8 else _unpack_int4(ql.weight)
        np.testing.assert_array_equal(q.cpu().numpy(), q_ref.reshape(384, 512))
        np.testing.assert_array_equal(ql.scales.cpu().numpy(), s_ref.reshape(384, 4))
