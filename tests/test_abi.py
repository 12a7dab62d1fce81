"""The C ABI library loads on a machine without a GPU, exports every symbol
include/ee_b200.h declares, agrees with the ctypes records, and rejects bad
arguments with error codes (no compute is launched)."""
import ctypes
import os
import re

import pytest
import torch

from conftest import ROOT


@pytest.fixture(scope="module")
def lib():
    from embodied_efficiency_b200 import _lib, build
    build.build()
    return _lib.load()


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "ee_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return set(re.findall(r"\b(ee_[a-z0-9_]+)\s*\(", src))


def test_exports_every_declared_symbol(lib):
    from embodied_efficiency_b200 import _lib
    names = declared_symbols()
    assert "ee_wq_gemm" in names and "ee_flow_sample" in names
    for n in names:
        assert hasattr(lib, n), n
    assert names == set(_lib.SIGNATURES), names ^ set(_lib.SIGNATURES)


def test_struct_layout_matches(lib):
    from embodied_efficiency_b200 import _lib
    for i, cls in enumerate((_lib.Linear, _lib.Norm, _lib.Block, _lib.Expert)):
        assert lib.ee_struct_size(i) == ctypes.sizeof(cls)
    assert lib.ee_struct_size(99) == 0


def test_strerror_and_version(lib):
    from embodied_efficiency_b200 import _lib
    assert lib.ee_version() >= 1
    assert "timed out" in _lib.strerror(_lib.EE_ERR_TIMEOUT)
    assert _lib.strerror(12345) == "unknown error"


def test_argument_errors_without_launch(lib):
    from embodied_efficiency_b200 import _lib
    # null pointers / bad enums / shapes are rejected before any device call
    assert lib.ee_pack_int4(None, None, 4, 4, None) == 1
    assert lib.ee_pack_int4(1, 1, 4, 3, None) == 2
    args = [16, 16, 0, 0, 0, 0, 16, 50, 64, 1024, _lib.EE_W_INT4, 128, _lib.EE_BF16, _lib.EE_F32, 0, None]
    a = list(args)
    a[10] = 9
    assert lib.ee_wq_gemm(*a) == 1                    # bad weight kind
    a = list(args)
    a[9] = 96
    assert lib.ee_wq_gemm(*a) == 2                    # K % 128
    a = list(args)
    a[12] = 7
    assert lib.ee_wq_gemm(*a) == 4                    # bad act dtype
    a = list(args)
    a[2] = 0
    assert lib.ee_wq_gemm(*a) == 1                    # int4 needs scales
    a = list(args)
    a[2] = 16
    a[0] = 8
    assert lib.ee_wq_gemm(*a) == 3                    # misaligned x
    a = list(args)
    a[2] = 16
    a[11] = 96
    assert lib.ee_wq_gemm(*a) == 2                    # group does not divide K
    # ee_dequant_weight(weight, scales, zeros, out, n, k, wkind, group, act, scale_dtype, stream)
    dq = [16, 16, 0, 16, 64, 1024, _lib.EE_W_INT4, 128, _lib.EE_BF16, _lib.EE_F32, None]
    for i, v, rc in ((0, 0, 1),                       # no weight
                     (8, 7, 4),                       # bad act dtype
                     (6, _lib.EE_W_DENSE, 1),         # nothing to dequantise
                     (5, 96, 2),                      # K % 128
                     (1, 0, 1),                       # int4 needs scales
                     (3, 8, 3),                       # misaligned output
                     (7, 96, 2),                      # group does not divide K
                     (6, _lib.EE_W_UINT4Z, 1)):       # zero-point form needs zeros
        a = list(dq)
        a[i] = v
        assert lib.ee_dequant_weight(*a) == rc, (i, v)
    # ee_attention(q, ldq, k, ldk, v, ldv, out, ldo, batch, heads, hd, n_q, n_k, q_rows, k_rows, act, stream)
    at = [16, 1024, 16, 2048, 16, 2048, 16, 1024, 1, 16, 64, 50, 256, 50, 256, _lib.EE_BF16, None]
    for i, v, rc in ((0, 0, 1),                       # no q
                     (10, 96, 9),                     # head size 96
                     (11, 65, 9),                     # more than 64 queries
                     (13, 49, 2),                     # fewer q rows per item than queries
                     (13, 1 << 31, 2),                # q rows per item beyond 32 bits
                     (14, 1 << 31, 2),                # k rows per item beyond 32 bits
                     (1, 8, 2)):                      # row stride below the heads' width
        a = list(at)
        a[i] = v
        assert lib.ee_attention(*a) == rc, (i, v)
    assert lib.ee_flow_sample(None, 0, 0, 0, 10, 0, 0, 0, None) == 1
    assert lib.ee_barrier_selftest(None, 1000, None) == 1
    assert lib.ee_barrier_selftest(16, 0, None) == 1


def test_expert_validation(lib):
    """ee_check_expert on a host description: shape and pointer rules."""
    from embodied_efficiency_b200 import _lib
    ex = _lib.Expert()
    ex.d_model, ex.n_layers, ex.n_heads, ex.horizon = 1024, 1, 16, 50
    ex.action_dim, ex.prefix_len, ex.hidden, ex.batch = 32, 256, 4096, 1
    ex.act_dtype, ex.eps = _lib.EE_BF16, 1e-5
    ex.freqs = ex.blocks = 16
    ex.out_norm.weight = ex.out_norm.bias = 16
    ex.in_proj = _lib.Linear(weight=16, n=1024, k=32, wkind=_lib.EE_W_DENSE)
    ex.out_proj = _lib.Linear(weight=16, n=32, k=1024, wkind=_lib.EE_W_DENSE)
    ex.t_proj = _lib.Linear(weight=16, scales=16, n=1024, k=1024, wkind=_lib.EE_W_INT4, group=128,
                          scale_dtype=_lib.EE_F32)
    blk = (_lib.Block * 1)()
    b = blk[0]
    for nm in ("n1", "nx", "n2"):
        setattr(b, nm, _lib.Norm(weight=16, bias=16))
    shapes = {"qkv": (3072, 1024), "proj": (1024, 1024), "q_c": (1024, 1024), "out_c": (1024, 1024),
              "mlp0": (4096, 1024), "mlp2": (1024, 4096)}
    for nm, (n, k) in shapes.items():
        setattr(b, nm, _lib.Linear(weight=16, scales=16, n=n, k=k, wkind=_lib.EE_W_INT4, group=128,
                                   scale_dtype=_lib.EE_F32))
    b.kv = 16
    assert lib.ee_check_expert(ctypes.byref(ex), blk, 10, 0) == 0
    assert lib.ee_flow_sample_workspace_bytes(ctypes.byref(ex), 10) > 0
    b.mlp2.k = 2048
    assert lib.ee_check_expert(ctypes.byref(ex), blk, 10, 0) == 2
    b.mlp2.k = 4096
    ex.n_heads = 4                                    # head size 256: unsupported
    assert lib.ee_check_expert(ctypes.byref(ex), blk, 10, 0) == 9
    ex.n_heads = 16
    assert lib.ee_check_expert(ctypes.byref(ex), blk, 2, _lib.EE_MODE_VELOCITY) == 1


def test_cpu_tensors_fail_loudly():
    from embodied_efficiency_b200 import _pack_int4, wq_linear
    with pytest.raises(RuntimeError, match="no CPU path"):
        _pack_int4(torch.zeros(4, 8, dtype=torch.int8))
    with pytest.raises(RuntimeError, match="no CPU path"):
        wq_linear(torch.zeros(2, 128), torch.zeros(8, 128, dtype=torch.int8), torch.ones(8, 1),
                  None, 128, 8)


def test_quant_operand_shapes_checked_before_any_call():
    """The C ABI sees raw pointers and cannot check that scales / zero points
    are [N, K / group]; the Python entry points do, before the device is
    touched (a mismatch would otherwise read past the scales on the GPU)."""
    from embodied_efficiency_b200 import wq_linear
    from embodied_efficiency_b200.wq_gemm import dequant_weight
    x = torch.zeros(2, 256)
    w8 = torch.zeros(8, 256, dtype=torch.int8)
    w4 = torch.zeros(8, 128, dtype=torch.uint8)
    with pytest.raises(ValueError, match="scales have shape"):
        wq_linear(x, w8, torch.ones(8, 1), None, 128, 8)          # group 128 needs [8, 2]
    with pytest.raises(ValueError, match="scales have shape"):
        wq_linear(x, w4, torch.ones(8, 4), None, 128, 4)
    with pytest.raises(ValueError, match="does not divide"):
        wq_linear(x, w8, torch.ones(8, 3), None, 96, 8)
    with pytest.raises(ValueError, match="need scales"):
        wq_linear(x, w8, None, None, 128, 8)
    with pytest.raises(ValueError, match="float32 or float16"):
        wq_linear(x, w8, torch.ones(8, 2, dtype=torch.float64), None, 128, 8)
    with pytest.raises(ValueError, match="zeros have shape"):
        wq_linear(x, w4, torch.ones(8, 2), None, 128, 4, zeros=torch.zeros(8, 1))
    with pytest.raises(ValueError, match="int8 weights"):
        wq_linear(x, w8.to(torch.uint8), torch.ones(8, 2), None, 128, 8)
    with pytest.raises(ValueError, match="scales have shape"):
        dequant_weight(w4, torch.ones(2, 8), 128, 4, torch.bfloat16)
    with pytest.raises(ValueError, match="bits must be"):
        wq_linear(x, w8, torch.ones(8, 2), None, 128, 3)
    # well-formed operands get as far as the device check
    with pytest.raises(RuntimeError, match="no CPU path"):
        wq_linear(x, w8, torch.ones(8, 2), None, 128, 8)
