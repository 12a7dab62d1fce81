"""numpy restatement of the reference's weight quantisation and int4 packing.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the checker for the
CUDA pack / unpack / dequant-GEMM kernels, never shipped or measured.

Every function names the reference lines it restates. All arithmetic is the
reference's: fp32 amax, fp32 division, round-half-to-even, clamp, int8
storage, two nibbles per byte with the even k in the low nibble.
"""
from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------------------
# bf16 / fp16 helpers (numpy has no bfloat16)
# ---------------------------------------------------------------------------


def f32_to_bf16_bits(x) -> np.ndarray:
    """fp32 -> bf16 bit pattern, round to nearest even (torch's ``.to(bfloat16)``)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[np.isnan(x)] = 0x7FC0
    return r


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_bf16(x) -> np.ndarray:
    """Round fp32 values to the nearest bf16 value, returned as fp32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def round_f16(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


# ---------------------------------------------------------------------------
# symmetric group quantisation (the reference scheme)
# ---------------------------------------------------------------------------


def group_size_for(k: int, group_size: int = 128) -> int:
    """kernel/quant.py:25 -- per-row fallback when K is not a multiple of the group."""
    return group_size if k % group_size == 0 else k


def quantize_weight(w, bits: int, group_size: int = 128):
    """kernel/quant.py:22-30.

    w: fp32 [out, in]. Returns (q int8 [out, in/gs, gs], scale fp32
    [out, in/gs, 1], gs) with ``scale = max(amax/qmax, 1e-8)`` and
    ``q = clamp(round_half_even(w/scale), -qmax-1, qmax)``.
    """
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    gs = group_size_for(k, group_size)
    wg = w.reshape(n, k // gs, gs)
    qmax = np.float32(2 ** (bits - 1) - 1)
    amax = np.abs(wg).max(axis=-1, keepdims=True)
    scale = np.maximum(amax / qmax, np.float32(1e-8)).astype(np.float32)
    q = np.clip(np.rint(wg / scale), -qmax - 1, qmax).astype(np.int8)
    return q, scale, gs


def dequantize_weight(q, scale, gs: int) -> np.ndarray:
    """kernel/quant.py:33-35: ``(q.float() * scale).view(out, in)`` in fp32."""
    out, ng, _ = q.shape
    return (q.astype(np.float32) * scale.astype(np.float32)).reshape(out, ng * gs)


def pack_int4(q2d) -> np.ndarray:
    """kernel/triton_gemm.py:37-39: two's-complement nibbles, even k in the low nibble."""
    q2d = np.asarray(q2d)
    nib = (q2d.astype(np.int16) & 0xF).astype(np.uint8)
    return ((nib[:, 1::2] << 4) | nib[:, 0::2]).astype(np.uint8)


def unpack_int4(packed) -> np.ndarray:
    """kernel/triton_gemm.py:42-48: split nibbles, interleave, sign-extend (v >= 8 -> v - 16)."""
    packed = np.asarray(packed, dtype=np.uint8)
    n, kh = packed.shape
    out = np.empty((n, 2 * kh), dtype=np.int16)
    out[:, 0::2] = packed & 0xF
    out[:, 1::2] = (packed >> 4) & 0xF
    return np.where(out >= 8, out - 16, out).astype(np.int8)


def dequant_int8(q2d, scales2d, gs: int) -> np.ndarray:
    """kernel/triton_gemm.py:51-55: per-group fp32 dequantisation of an [N, K] int8 matrix."""
    n, k = q2d.shape
    ng = scales2d.shape[1]
    return (q2d.astype(np.float32).reshape(n, ng, gs)
            * np.asarray(scales2d, np.float32).reshape(n, ng, 1)).reshape(n, k)


def dequant_int4(packed, scales2d, gs: int) -> np.ndarray:
    """kernel/triton_gemm.py:57-58."""
    return dequant_int8(unpack_int4(packed), scales2d, gs)


# ---------------------------------------------------------------------------
# asymmetric int4 (no reference code: this restatement is its only oracle)
# ---------------------------------------------------------------------------

F16_MIN_NORMAL = np.float32(2.0 ** -14)


def quantize_weight_asym4(w, group_size: int = 128):
    """Asymmetric 4-bit group quantisation with fp16 scale and fp16 zero per group.

    Definition used by this project (the reference has only the symmetric
    scheme): per group ``scale = fp16(max((max-min)/15, 2^-14))``,
    ``zero = clamp(round(-min/scale), 0, 15)`` (an integer stored as fp16),
    ``q = clamp(round(w/scale) + zero, 0, 15)``; dequantised ``(q - zero) * scale``.
    Returns (q uint8 [N, K] in 0..15, scale fp16 [N, K/gs], zero fp16 [N, K/gs], gs).
    """
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    gs = group_size_for(k, group_size)
    wg = w.reshape(n, k // gs, gs)
    wmin = wg.min(axis=-1, keepdims=True)
    wmax = wg.max(axis=-1, keepdims=True)
    scale = np.maximum((wmax - wmin) / np.float32(15.0), F16_MIN_NORMAL)
    scale = scale.astype(np.float16).astype(np.float32)
    zero = np.clip(np.rint(-wmin / scale), 0, 15).astype(np.float32)
    q = np.clip(np.rint(wg / scale) + zero, 0, 15).astype(np.uint8)
    return (q.reshape(n, k), scale.reshape(n, k // gs).astype(np.float16),
            zero.reshape(n, k // gs).astype(np.float16), gs)


def pack_uint4(u2d) -> np.ndarray:
    """Pack unsigned nibbles (0..15) two per byte, even k in the low nibble."""
    u2d = np.asarray(u2d, dtype=np.uint8)
    return ((u2d[:, 1::2] << 4) | (u2d[:, 0::2] & 0xF)).astype(np.uint8)


def unpack_uint4(packed) -> np.ndarray:
    packed = np.asarray(packed, dtype=np.uint8)
    n, kh = packed.shape
    out = np.empty((n, 2 * kh), dtype=np.uint8)
    out[:, 0::2] = packed & 0xF
    out[:, 1::2] = packed >> 4
    return out


def dequant_asym4(packed, scales16, zeros16, gs: int) -> np.ndarray:
    u = unpack_uint4(packed).astype(np.float32)
    n, k = u.shape
    ng = k // gs
    s = np.asarray(scales16, np.float16).astype(np.float32).reshape(n, ng, 1)
    z = np.asarray(zeros16, np.float16).astype(np.float32).reshape(n, ng, 1)
    return ((u.reshape(n, ng, gs) - z) * s).reshape(n, k)


# ---------------------------------------------------------------------------
# dequantise-then-matmul GEMM (kernel/quant.py:54-56 QuantLinear.forward)
# ---------------------------------------------------------------------------


def linear_ref(x, w_deq, bias=None, act_round=round_bf16):
    """``F.linear(x, dequant(W).to(x.dtype), bias)``: the weight is rounded to the
    activation dtype first (kernel/quant.py:55), the product is formed in float64
    here (a tighter reference than any fp32-accumulating GEMM) and the result is
    rounded to the activation dtype.
    """
    x = np.asarray(x, np.float32)
    w = act_round(np.asarray(w_deq, np.float32))
    y = x.astype(np.float64) @ w.astype(np.float64).T
    if bias is not None:
        y = y + np.asarray(bias, np.float64)[None, :]
    return act_round(y.astype(np.float32))
