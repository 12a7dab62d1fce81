"""Weight-only int8 / int4 dequant-GEMM: drop-in for the reference's
``kernel/triton_gemm.py`` surface, backed by the sm_100a kernels of
``libee_b200.so`` (no Triton, no CPU path).

Layouts are the reference's: int8 weights [N, K]; int4 packed two per byte
[N, K/2] with the even k in the low nibble; fp32 scales [N, K/group].
"""
from __future__ import annotations

import ctypes

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from .quant import quantize_weight


# ---------------------------------------------------------------------------
# packing (bit-exact with kernel/triton_gemm.py:37-48), on the GPU
# ---------------------------------------------------------------------------
def _pack_int4(q2d: torch.Tensor) -> torch.Tensor:
    """kernel/triton_gemm.py:37-39: int8 [N, K] in -8..7 -> uint8 [N, K/2]."""
    _lib.require_cuda(q2d)
    if q2d.dim() != 2 or q2d.shape[1] % 2:
        raise ValueError("_pack_int4 expects [N, K] with K even")
    q = q2d.to(torch.int8).contiguous()
    out = torch.empty(q.shape[0], q.shape[1] // 2, dtype=torch.uint8, device=q.device)
    _lib.check(_lib.load().ee_pack_int4(q.data_ptr(), out.data_ptr(), q.shape[0], q.shape[1],
                                        _lib.stream_ptr(q.device)), "ee_pack_int4")
    return out


def _unpack_int4(packed: torch.Tensor) -> torch.Tensor:
    """kernel/triton_gemm.py:42-48: uint8 [N, K/2] -> int8 [N, K] (sign-extended nibbles)."""
    _lib.require_cuda(packed)
    p = packed.to(torch.uint8).contiguous()
    n, kh = p.shape
    out = torch.empty(n, 2 * kh, dtype=torch.int8, device=p.device)
    _lib.check(_lib.load().ee_unpack_int4(p.data_ptr(), out.data_ptr(), n, 2 * kh,
                                          _lib.stream_ptr(p.device)), "ee_unpack_int4")
    return out


def _dequant_int8(q, scale, gs):
    """kernel/triton_gemm.py:51-55 (reference helper, used only to check kernels)."""
    n, k = q.shape
    ng = scale.shape[1]
    return (q.float().view(n, ng, gs) * scale.float().view(n, ng, 1)).view(n, k)


def _dequant_int4(packed, scale, gs):
    """kernel/triton_gemm.py:57-58."""
    return _dequant_int8(_unpack_int4(packed), scale, gs)


# ---------------------------------------------------------------------------
# the fused dequant-GEMM
# ---------------------------------------------------------------------------
def wkind_for(bits: int, zeros=None) -> int:
    if bits == 4:
        return _lib.EE_W_UINT4Z if zeros is not None else _lib.EE_W_INT4
    if bits == 8:
        return _lib.EE_W_INT8
    if bits == 16:
        return _lib.EE_W_DENSE
    raise ValueError(f"bits must be 4, 8 or 16, got {bits}")


def _check_quant_operands(weight, scales, zeros, n, k, group_size, bits):
    """Shape / dtype / device checks the C ABI cannot make (it sees raw
    pointers): scales (and zero points) must be [n, k / group_size] on the
    weight's device, or the kernels would read past their end."""
    if bits == 16:
        return
    if scales is None:
        raise ValueError(f"int{bits} weights need scales")
    g = int(group_size)
    if g <= 0 or k % g:
        raise ValueError(f"group_size {group_size} does not divide K={k}")
    if tuple(scales.shape) != (n, k // g):
        raise ValueError(f"scales have shape {tuple(scales.shape)}, expected {(n, k // g)} "
                         f"for a [{n}, {k}] weight with group_size {g}")
    if scales.dtype not in (torch.float32, torch.float16):
        raise ValueError(f"scales must be float32 or float16, not {scales.dtype}")
    if scales.device != weight.device:
        raise ValueError("scales and weight are on different devices")
    if zeros is not None:
        if tuple(zeros.shape) != (n, k // g):
            raise ValueError(f"zeros have shape {tuple(zeros.shape)}, expected {(n, k // g)}")
        if zeros.device != weight.device:
            raise ValueError("zeros and weight are on different devices")
        if bits != 4:
            raise ValueError("zero points apply to int4 weights only")
    ok = (torch.uint8, torch.int8) if bits == 4 else (torch.int8,)
    if weight.dtype not in ok:
        raise ValueError(f"int{bits} weights are {' or '.join(map(str, ok))}, not {weight.dtype}")


def wq_linear(x, weight, scales, bias, group_size, bits, zeros=None, gelu=False, residual=None):
    """kernel/triton_gemm.py:141-164: ``x @ dequant(weight).T + bias`` in x.dtype.

    Runs ``ee_wq_gemm``: dequantisation in registers, fp32 accumulation, bias
    in fp32, one rounding to the activation dtype. bf16 / fp16 activations are
    used as they are; fp32 activations are computed in bf16 and the result is
    returned as fp32. Optional fused epilogues: ``gelu`` (exact erf GELU) or
    ``residual`` (+ residual, both rounded as separate torch ops would).
    ``bits=16`` means ``weight`` is a dense [N, K] matrix in the activation dtype.
    """
    if bits not in (4, 8, 16):
        raise ValueError(f"bits must be 4, 8 or 16, got {bits}")
    *lead, k_in = x.shape
    n = weight.shape[0]
    k = weight.shape[1] * 2 if bits == 4 else weight.shape[1]
    if k_in != k:
        raise ValueError(f"x has K={k_in}, weight has K={k}")
    _check_quant_operands(weight, scales, zeros, n, k, group_size, bits)
    _lib.require_cuda(x, weight)
    out_dtype = x.dtype
    act = x.dtype if x.dtype in (torch.bfloat16, torch.float16) else torch.bfloat16
    xf = x.reshape(-1, k).to(act).contiguous()
    m = xf.shape[0]
    if bits == 16:
        weight = weight.to(act)
    w = weight.contiguous()
    s = None if scales is None else scales.contiguous()
    z = None if zeros is None else zeros.to(torch.float16).contiguous()
    b = None if bias is None else bias.to(act).contiguous()
    r = None if residual is None else residual.reshape(m, n).to(act).contiguous()
    y = torch.empty(m, n, dtype=act, device=x.device)
    if m == 0:
        return y.reshape(*lead, n).to(out_dtype)
    epi = (_lib.EE_EPI_BIAS if b is not None else 0) | (_lib.EE_EPI_GELU if gelu else 0) | \
        (_lib.EE_EPI_RESIDUAL if r is not None else 0)
    rc = _lib.load().ee_wq_gemm(
        xf.data_ptr(), w.data_ptr(), _lib.ptr(s), _lib.ptr(z), _lib.ptr(b), _lib.ptr(r), y.data_ptr(),
        m, n, k, wkind_for(bits, z), int(group_size) if bits != 16 else 0, _lib.act_code(act),
        _lib.scale_code(s.dtype) if s is not None else _lib.EE_F32, epi, _lib.stream_ptr(x.device))
    _lib.check(rc, "ee_wq_gemm")
    return y.reshape(*lead, n).to(out_dtype)


def dequant_weight(weight, scales, group_size, bits, dtype, zeros=None):
    """[N, K] ``dtype`` (bf16 / fp16) copy of a packed weight, the values the
    dequant-GEMM multiplies (``ee_dequant_weight``: the exact integer times
    the scale rounded to ``dtype``, one rounding; kernel/quant.py:33-35)."""
    if dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"dequantised weights are bf16 or fp16, not {dtype}")
    if bits not in (4, 8):
        raise ValueError(f"bits must be 4 or 8, got {bits}")
    n = weight.shape[0]
    k = weight.shape[1] * 2 if bits == 4 else weight.shape[1]
    _check_quant_operands(weight, scales, zeros, n, k, group_size, bits)
    _lib.require_cuda(weight, scales)
    w = weight.contiguous()
    s = scales.contiguous()
    z = None if zeros is None else zeros.to(torch.float16).contiguous()
    out = torch.empty(n, k, dtype=dtype, device=weight.device)
    _lib.check(_lib.load().ee_dequant_weight(w.data_ptr(), s.data_ptr(), _lib.ptr(z), out.data_ptr(), n, k,
                                             wkind_for(bits, z), int(group_size), _lib.act_code(dtype),
                                             _lib.scale_code(s.dtype), _lib.stream_ptr(weight.device)),
               "ee_dequant_weight")
    return out


# Tokens from which a quantized linear runs on a cached dense copy of its
# weight: there the GEMM is bound by the tensor cores, and the tcgen05 kernel
# with the dense weight brought by TMA straight into the MMA's tiles beats
# dequantising a weight tile again for every token tile (12800 tokens,
# K = N = 1024: 40 vs 49 us; K = 4096, N = 1024: 102 vs 137 us). The copy
# costs device memory for as long as the module lives: 2 bytes per weight
# (4x the packed int4 bytes, 2x int8), about 2.2 GB for a 1.1 B-weight
# model. None turns the copy off (every call then runs on the packed weight).
DENSE_MIN_TOKENS = 1024


def gemm_status(reset: bool = False) -> int:
    """Device status word of the dequant-GEMM kernels on the current device
    (0, or the first error a launch recorded: a bounded in-kernel wait that
    gave up, or a launch without its planned cluster shape). Synchronises."""
    st = ctypes.c_int32(0)
    _lib.check(_lib.load().ee_wq_gemm_status(ctypes.byref(st), 1 if reset else 0), "ee_wq_gemm_status")
    return int(st.value)


class TritonQuantLinear(nn.Module):
    """kernel/triton_gemm.py:167-184: weight-only int8 / int4 linear.

    Same buffers and attributes as the reference (``weight``, ``scales``,
    ``bias``, ``bits``, ``group_size``, ``in_features``, ``out_features``) so
    that callers such as ``compiler._weight_mb`` see the same module; the
    forward runs the sm_100a dequant-GEMM.
    """

    def __init__(self, lin: nn.Linear, bits: int = 8, group_size: int = 128):
        super().__init__()
        assert bits in (4, 8)
        q3, scale3, gs = quantize_weight(lin.weight.data.float(), bits, group_size)
        out, ng, g = q3.shape
        q2d = q3.reshape(out, ng * g).to(torch.int8)
        if bits == 4:
            dev = q2d.device
            if not q2d.is_cuda:
                if not torch.cuda.is_available():
                    raise RuntimeError("int4 packing runs on the GPU; no CUDA device is visible")
                q2d = q2d.cuda()
            weight = _pack_int4(q2d).to(dev)
        else:
            weight = q2d.contiguous()
        self.register_buffer("weight", weight)
        self.register_buffer("scales", scale3.reshape(out, ng).contiguous().float())
        self.bias = lin.bias
        self.bits, self.group_size = bits, gs
        self.out_features, self.in_features = out, ng * g

    def _dense_key(self, dtype):
        return (dtype, self.weight.data_ptr(), self.weight._version, self.scales.data_ptr(), self.scales._version)

    def dense_weight(self, dtype):
        """The weight dequantised into ``dtype`` (``dequant_weight``), made on
        first use and kept until the weight or scales change; a plain
        attribute, not a buffer, so ``state_dict`` holds only the packed form."""
        cached = self.__dict__.get("_dense")
        if cached is None or cached[0] != self._dense_key(dtype):
            cached = (self._dense_key(dtype), dequant_weight(self.weight, self.scales, self.group_size, self.bits,
                                                             dtype))
            self.__dict__["_dense"] = cached
        return cached[1]

    def linear(self, x, gelu=False, residual=None):
        """``wq_linear`` with this module's buffers (and the fused epilogues);
        from ``DENSE_MIN_TOKENS`` bf16 / fp16 tokens on, on the dense copy of
        the weight -- the same products, so the same results up to the
        GEMM's accumulation order. Never builds the copy during stream capture."""
        m = x.numel() // self.in_features if self.in_features else 0
        if (DENSE_MIN_TOKENS is not None and x.is_cuda and x.dtype in (torch.bfloat16, torch.float16)
                and m >= DENSE_MIN_TOKENS
                and (not torch.cuda.is_current_stream_capturing()
                     or self.__dict__.get("_dense", (None,))[0] == self._dense_key(x.dtype))):
            return wq_linear(x, self.dense_weight(x.dtype), None, self.bias, 0, 16, gelu=gelu, residual=residual)
        return wq_linear(x, self.weight, self.scales, self.bias, self.group_size, self.bits, gelu=gelu,
                         residual=residual)

    def forward(self, x):
        return self.linear(x)

    def weight_bytes(self) -> float:
        """kernel/quant.py:58-59: int weights + scales counted as fp16."""
        return self.out_features * self.in_features * self.bits / 8.0 + self.scales.numel() * 2

    def extra_repr(self):
        return f"in={self.in_features}, out={self.out_features}, bits={self.bits}, group={self.group_size}"


def quantize_model_triton(model, bits=8, group_size=128, skip=("in_proj", "out_proj")):
    """kernel/triton_gemm.py:187-195: swap every nn.Linear except ``skip`` for
    ``TritonQuantLinear``, recursively; returns the mutated model."""
    for name, mod in list(model.named_children()):
        if name in skip:
            continue
        if isinstance(mod, nn.Linear):
            setattr(model, name, TritonQuantLinear(mod, bits, group_size))
        else:
            quantize_model_triton(mod, bits, group_size, skip)
    return model


def correctness_check():
    """kernel/triton_gemm.py:198-210 on the sm_100a kernels: fp16 X [50, 512],
    nn.Linear(512, 1536), kernel vs torch dequant + F.linear, max abs < 0.5."""
    torch.manual_seed(1)
    x = torch.randn(50, 512, device="cuda", dtype=torch.float16)
    errs = {}
    for bits in (8, 4):
        lin = nn.Linear(512, 1536).cuda().half()
        ql = TritonQuantLinear(lin, bits).cuda()
        y = wq_linear(x, ql.weight, ql.scales, ql.bias, ql.group_size, bits)
        deq = (_dequant_int4 if bits == 4 else _dequant_int8)(ql.weight, ql.scales, ql.group_size)
        err = (y - F.linear(x, deq.to(x.dtype), ql.bias)).abs().max().item()
        print(f"  int{bits}: sm_100a kernel vs torch-dequant max abs err = {err:.4e}")
        assert err < 5e-1, f"int{bits} kernel disagrees with reference"
        errs[bits] = err
    print("sm_100a dequant-GEMM correctness ok")
    return errs
