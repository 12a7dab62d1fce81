"""torch-CPU restatement of the reference action expert and its Euler sampler.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the checker for the
fused CUDA sampler and the timed CPU baseline, never shipped or measured on
the GPU.

The model is described by a flat parameter dict whose keys are the
reference's ``state_dict`` names (``in_proj.weight``, ``blocks.0.qkv.bias``,
...), so the same weights can be loaded into the reference module, into this
oracle and into the CUDA path. Quantised linears follow the reference's
dequantise-then-matmul ``QuantLinear`` (kernel/quant.py:38-56): the int
weight is dequantised in fp32, rounded to the activation dtype and fed to
``F.linear``. Every function cites the reference lines it restates.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import quant as Q

QUANT_SKIP = ("in_proj", "out_proj")  # kernel/quant.py:63 / triton_gemm.py:187


@dataclass
class Cfg:
    """Model shape (kernel/flow_expert.py:28-35) plus two variant flags.

    ``norm`` ("layernorm" as in the reference, or "rmsnorm") and ``self_attn``
    (False drops the action-token self-attention sub-block) describe the
    pre-RMSNorm / cross-attention-only block variant; the reference has only
    ``norm="layernorm", self_attn=True``.
    """

    d_model: int = 512
    n_layers: int = 6
    n_heads: int = 8
    horizon: int = 50
    action_dim: int = 32
    prefix_len: int = 256
    mlp_ratio: float = 4.0
    norm: str = "layernorm"
    self_attn: bool = True
    eps: float = 1e-5


def linear_names(cfg) -> list:
    names = ["in_proj", "t_proj"]
    for i in range(cfg.n_layers):
        p = f"blocks.{i}."
        if getattr(cfg, "self_attn", True):
            names += [p + "qkv", p + "proj"]
        names += [p + "q_c", p + "kv_c", p + "out_c", p + "mlp.0", p + "mlp.2"]
    names.append("out_proj")
    return names


def quantize_params(params: dict, cfg, bits: int, group_size: int = 128) -> dict:
    """kernel/quant.py:62-73 + :45-52: every linear except in/out_proj gets
    ``quantize_weight(weight.float(), bits, group_size)``."""
    qp = {}
    for name in linear_names(cfg):
        if name.split(".")[-1] in QUANT_SKIP:
            continue
        w = params[name + ".weight"].float().numpy()
        q, s, gs = Q.quantize_weight(w, bits, group_size)
        qp[name] = (torch.from_numpy(q), torch.from_numpy(s), gs)
    return qp


def _linear(x, params, qp, name):
    bias = params.get(name + ".bias")
    if qp is not None and name in qp:
        q, s, gs = qp[name]
        # kernel/quant.py:33-35,55: fp32 dequant, then round to the activation dtype
        w = (q.float() * s).view(q.shape[0], -1).to(x.dtype)
    else:
        w = params[name + ".weight"]
    return F.linear(x, w, bias)


def _norm(x, params, name, cfg):
    w = params[name + ".weight"]
    if getattr(cfg, "norm", "layernorm") == "rmsnorm":
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + cfg.eps)
        return y.to(x.dtype) * w
    return F.layer_norm(x, (x.shape[-1],), w, params.get(name + ".bias"), cfg.eps)


def timestep_embedding(t, dim: int, max_period: float = 10000.0):
    """kernel/flow_expert.py:38-48: fp32 frequencies, args = t*freqs*1000, [cos, sin]."""
    half = dim // 2
    freqs = torch.exp(-math.log(max_period)
                      * torch.arange(half, device=t.device, dtype=torch.float32) / half)
    args = t.float()[:, None] * freqs[None] * 1000.0
    emb = torch.cat([torch.cos(args), torch.sin(args)], dim=-1)
    if dim % 2 == 1:
        emb = torch.cat([emb, torch.zeros_like(emb[:, :1])], dim=-1)
    return emb


def _heads(x, h):  # kernel/flow_expert.py:70-72
    b, t, d = x.shape
    return x.view(b, t, h, d // h).transpose(1, 2)


def _merge(x):  # kernel/flow_expert.py:74-76
    b, h, t, hd = x.shape
    return x.transpose(1, 2).contiguous().view(b, t, h * hd)


def encode_prefix(params, cfg, prefix, qp=None):
    """kernel/flow_expert.py:78-81,112-115: per block ``kv_c(prefix)`` split into K, V heads."""
    out = []
    for i in range(cfg.n_layers):
        k, v = _linear(prefix, params, qp, f"blocks.{i}.kv_c").chunk(2, dim=-1)
        out.append((_heads(k, cfg.n_heads), _heads(v, cfg.n_heads)))
    return out


def block_forward(x, params, qp, cfg, i, kv):
    """kernel/flow_expert.py:83-95."""
    p = f"blocks.{i}."
    h = cfg.n_heads
    if getattr(cfg, "self_attn", True):
        q, k, v = _linear(_norm(x, params, p + "n1", cfg), params, qp, p + "qkv").chunk(3, dim=-1)
        a = F.scaled_dot_product_attention(_heads(q, h), _heads(k, h), _heads(v, h))
        x = x + _linear(_merge(a), params, qp, p + "proj")
    q = _heads(_linear(_norm(x, params, p + "nx", cfg), params, qp, p + "q_c"), h)
    a = F.scaled_dot_product_attention(q, kv[0], kv[1])
    x = x + _linear(_merge(a), params, qp, p + "out_c")
    u = F.gelu(_linear(_norm(x, params, p + "n2", cfg), params, qp, p + "mlp.0"))
    x = x + _linear(u, params, qp, p + "mlp.2")
    return x


def expert_forward(params, cfg, x_act, t, prefix_kv, qp=None):
    """kernel/flow_expert.py:117-124: velocity for actions x_act [B,H,A] at times t [B]."""
    x = _linear(x_act, params, qp, "in_proj")
    temb = _linear(timestep_embedding(t, cfg.d_model).to(x.dtype), params, qp, "t_proj")
    x = x + temb[:, None, :]
    for i in range(cfg.n_layers):
        x = block_forward(x, params, qp, cfg, i, prefix_kv[i])
    return _linear(_norm(x, params, "out_norm", cfg), params, qp, "out_proj")


@torch.no_grad()
def flow_sample(params, cfg, x_init, n_steps: int, prefix_kv, qp=None):
    """kernel/flow_expert.py:127-137: Euler steps, ``t`` kept in x.dtype."""
    x = x_init
    dt = 1.0 / n_steps
    t = torch.zeros(x.shape[0], device=x.device, dtype=x.dtype)
    for _ in range(n_steps):
        v = expert_forward(params, cfg, x, t, prefix_kv, qp)
        x = x + v * dt
        t = t + dt
    return x


@torch.no_grad()
def run(params, cfg, x0, prefix, n_steps: int = 10, bits=None, group_size: int = 128,
        dtype=torch.bfloat16, qp=None):
    """One full sampler call as the reference performs it: cast the model to
    ``dtype``, quantise (``bits`` 8/4) from the cast weights, encode the prefix
    once, run ``n_steps`` Euler steps."""
    p = {k: v.to(dtype) for k, v in params.items()}
    if bits is not None and qp is None:
        qp = quantize_params(p, cfg, bits, group_size)
    kv = encode_prefix(p, cfg, prefix.to(dtype), qp)
    return flow_sample(p, cfg, x0.to(dtype), n_steps, kv, qp)


def action_error(out, ref) -> float:
    """kernel/quant.py:104-105: rMSE / mean|ref| (the reference's fidelity metric)."""
    out = out.float()
    ref = ref.float()
    return (out - ref).pow(2).mean().sqrt().item() / (ref.abs().mean().item() + 1e-9)
