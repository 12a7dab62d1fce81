"""Host-side weight quantisation (load time, not the timed path).

Same names, signatures and arithmetic as the reference's ``kernel/quant.py``:
fp32 amax, fp32 division, round-half-to-even, clamp, int8 storage, so the
integers are bit-identical to the reference's on any device. The packed
weights these produce are consumed by the sm_100a kernels in ``csrc/``.
"""
from __future__ import annotations

import torch
import torch.nn as nn


def quantize_weight(w: torch.Tensor, bits: int, group_size: int = 128):
    """kernel/quant.py:22-30 -- symmetric per-group quantisation along the input dim.

    w: [out, in] float. Returns (q int8 [out, in/gs, gs], scale fp32
    [out, in/gs, 1], gs) with gs = group_size if in % group_size == 0 else in.
    """
    out, inf = w.shape
    gs = group_size if inf % group_size == 0 else inf
    wg = w.float().reshape(out, inf // gs, gs)
    qmax = 2 ** (bits - 1) - 1
    amax = wg.abs().amax(dim=-1, keepdim=True)
    # a tensor divisor, not the Python number: on CUDA, torch divides by a
    # scalar as a multiplication by its reciprocal, which differs from the
    # true quotient (what the reference computes on the CPU) in the last bit
    # of some scales; tensor / tensor is a true division on either device
    scale = (amax / torch.full_like(amax, qmax)).clamp_min(1e-8)
    q = torch.clamp(torch.round(wg / scale), -qmax - 1, qmax)
    return q.to(torch.int8), scale, gs


def dequantize_weight(q: torch.Tensor, scale: torch.Tensor, gs: int) -> torch.Tensor:
    """kernel/quant.py:33-35."""
    out, ng, _ = q.shape
    return (q.float() * scale).view(out, ng * gs)


def quantize_weight_asym4(w: torch.Tensor, group_size: int = 128):
    """Asymmetric int4 with an fp16 scale and an fp16 (integer-valued) zero per group.

    No reference counterpart (the reference quantises symmetrically only).
    Per group: ``scale = fp16(max((max - min) / 15, 2^-14))``,
    ``zero = clamp(round(-min / scale), 0, 15)``,
    ``q = clamp(round(w / scale) + zero, 0, 15)``; dequantised ``(q - zero) * scale``.
    Returns (q uint8 [out, in] in 0..15, scale fp16 [out, in/gs],
    zero fp16 [out, in/gs], gs).
    """
    out, inf = w.shape
    gs = group_size if inf % group_size == 0 else inf
    wg = w.float().reshape(out, inf // gs, gs)
    wmin = wg.amin(dim=-1, keepdim=True)
    wmax = wg.amax(dim=-1, keepdim=True)
    rng = wmax - wmin
    scale = (rng / torch.full_like(rng, 15.0)).clamp_min(2.0 ** -14).half().float()  # true division (see above)
    zero = torch.clamp(torch.round(-wmin / scale), 0, 15)
    q = torch.clamp(torch.round(wg / scale) + zero, 0, 15).to(torch.uint8)
    return (q.reshape(out, inf), scale.reshape(out, -1).half(), zero.reshape(out, -1).half(), gs)


class QuantLinear(nn.Module):
    """kernel/quant.py:36-59: drop-in for nn.Linear holding int weights and fp32
    scales in the reference's buffers -- ``q`` int8 [out, in/gs, gs] and
    ``scale`` fp32 [out, in/gs, 1] -- so state dicts interchange. Where the
    reference dequantises a full fp weight on every forward, this forward runs
    the sm_100a dequant-GEMM on the integers directly (the kernel operands --
    the [out, in] int8 view, or the packed int4 bytes -- are derived on first
    use and re-derived only when ``q`` or ``scale`` changes). CUDA only."""

    def __init__(self, lin: nn.Linear, bits: int, group_size: int = 128):
        super().__init__()
        q, scale, gs = quantize_weight(lin.weight.data.float(), bits, group_size)
        self.register_buffer("q", q)
        self.register_buffer("scale", scale)
        self.gs, self.bits = gs, bits
        self.bias = lin.bias
        self.out_features, self.in_features = lin.weight.shape
        self._ops = None  # (key, kernel weight, kernel scales)

    def _operands(self):
        key = (self.q.data_ptr(), self.q._version, self.scale.data_ptr(), self.scale._version)
        if self._ops is None or self._ops[0] != key:
            from .wq_gemm import _pack_int4
            w2 = self.q.reshape(self.out_features, self.in_features)
            if self.bits == 4:
                w2 = _pack_int4(w2.contiguous())
            self._ops = (key, w2.contiguous(), self.scale.reshape(self.out_features, -1).float().contiguous())
        return self._ops[1], self._ops[2]

    def forward(self, x):
        from .wq_gemm import wq_linear
        w, s = self._operands()
        return wq_linear(x, w, s, self.bias, self.gs, self.bits)

    def weight_bytes(self) -> float:
        """kernel/quant.py:58-59: int weights plus fp16-counted scales."""
        return self.q.numel() * self.bits / 8.0 + self.scale.numel() * 2


def quantize_model(model: nn.Module, bits: int, group_size: int = 128,
                   skip=("in_proj", "out_proj")) -> nn.Module:
    """kernel/quant.py:62-73: swap the transformer linears for ``QuantLinear``
    (IO projections stay dense); mutates and returns ``model``."""
    for name, mod in list(model.named_children()):
        if name in skip:
            continue
        if isinstance(mod, nn.Linear):
            setattr(model, name, QuantLinear(mod, bits, group_size))
        else:
            quantize_model(mod, bits, group_size, skip)
    return model


def linear_bytes(model: nn.Module, dtype_bytes: int = 2) -> float:
    """kernel/quant.py:76-77: dense linear weight bytes at ``dtype_bytes`` each."""
    return sum(m.weight.numel() * dtype_bytes for m in model.modules() if isinstance(m, nn.Linear))


def quant_linear_bytes(model: nn.Module) -> float:
    """kernel/quant.py:58-59,80-81: int weights plus fp16-counted scales of every
    quantised linear."""
    tot = 0.0
    for m in model.modules():
        if hasattr(m, "weight_bytes") and callable(m.weight_bytes):
            tot += m.weight_bytes()
    return tot
