"""Seeded synthetic weights and inputs for the sampler workloads.

The reference ships no checkpoints or datasets for this path; every workload
is random-init weights plus N(0, 1) noise and prefix. These helpers fix one
reproducible definition, keyed by the reference's ``state_dict`` names:

* ``init_params(cfg, gen)``: every Linear weight and bias ~ N(0, 0.02),
  every norm weight 1 and bias 0, drawn in the reference's
  ``named_parameters()`` order from ``gen``.
* ``make_request(cfg, batch, gen)``: x0 [batch, horizon, action_dim] ~ N(0, 1)
  and prefix [batch, prefix_len, d_model] ~ N(0, 1) (bf16), drawn after the
  weights from the same generator when ``gen`` is shared.
"""
from __future__ import annotations

from collections import OrderedDict

import torch


def param_shapes(cfg) -> "OrderedDict[str, tuple]":
    """Parameter names and shapes in kernel/flow_expert.py:98-107 registration order."""
    d, a = cfg.d_model, cfg.action_dim
    hid = int(d * cfg.mlp_ratio)
    rms = getattr(cfg, "norm", "layernorm") == "rmsnorm"
    sa = getattr(cfg, "self_attn", True)
    shapes = OrderedDict()
    shapes["in_proj.weight"] = (d, a)
    shapes["in_proj.bias"] = (d,)
    shapes["t_proj.weight"] = (d, d)
    shapes["t_proj.bias"] = (d,)

    def norm(name):
        shapes[name + ".weight"] = (d,)
        if not rms:
            shapes[name + ".bias"] = (d,)

    for i in range(cfg.n_layers):
        p = f"blocks.{i}."
        if sa:
            norm(p + "n1")
            shapes[p + "qkv.weight"] = (3 * d, d)
            shapes[p + "qkv.bias"] = (3 * d,)
            shapes[p + "proj.weight"] = (d, d)
            shapes[p + "proj.bias"] = (d,)
        norm(p + "nx")
        shapes[p + "q_c.weight"] = (d, d)
        shapes[p + "q_c.bias"] = (d,)
        shapes[p + "kv_c.weight"] = (2 * d, d)
        shapes[p + "kv_c.bias"] = (2 * d,)
        shapes[p + "out_c.weight"] = (d, d)
        shapes[p + "out_c.bias"] = (d,)
        norm(p + "n2")
        shapes[p + "mlp.0.weight"] = (hid, d)
        shapes[p + "mlp.0.bias"] = (hid,)
        shapes[p + "mlp.2.weight"] = (d, hid)
        shapes[p + "mlp.2.bias"] = (d,)
    norm("out_norm")
    shapes["out_proj.weight"] = (a, d)
    shapes["out_proj.bias"] = (a,)
    return shapes


def _is_norm(name: str) -> bool:
    parts = name.split(".")
    return len(parts) >= 2 and parts[-2] in ("n1", "nx", "n2", "out_norm")


def init_params(cfg, gen: torch.Generator, std: float = 0.02) -> "OrderedDict[str, torch.Tensor]":
    out = OrderedDict()
    for name, shape in param_shapes(cfg).items():
        if _is_norm(name):
            out[name] = torch.ones(shape) if name.endswith("weight") else torch.zeros(shape)
        else:
            out[name] = torch.randn(shape, generator=gen) * std
    return out


def make_request(cfg, batch: int, gen: torch.Generator):
    x0 = torch.randn(batch, cfg.horizon, cfg.action_dim, generator=gen)
    prefix = torch.randn(batch, cfg.prefix_len, cfg.d_model, generator=gen).to(torch.bfloat16)
    return x0, prefix


def workload(cfg, seed: int = 0, batch: int = 1):
    """(params, x0, prefix) for one seeded workload: one generator, weights first."""
    g = torch.Generator().manual_seed(seed)
    params = init_params(cfg, g)
    x0, prefix = make_request(cfg, batch, g)
    return params, x0, prefix


def fleet_request(cfg, r: int):
    """Request r of the fleet: (prefix [1, P, d] bf16, x0 [1, H, A]) drawn from
    ``torch.Generator().manual_seed(r)`` (noise first)."""
    x0, pre = make_request(cfg, 1, torch.Generator().manual_seed(r))
    return pre, x0


def fleet_requests(cfg, n_requests: int, first: int = 0):
    """Fleet-mode inputs: request r draws its own x0 [1, H, A] and prefix [1, P, d]
    from ``torch.Generator().manual_seed(r)``."""
    xs, ps = [], []
    for r in range(first, first + n_requests):
        g = torch.Generator().manual_seed(r)
        x0, pre = make_request(cfg, 1, g)
        xs.append(x0)
        ps.append(pre)
    return torch.cat(xs), torch.cat(ps)
