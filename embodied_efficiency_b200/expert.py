"""Flow-matching action expert and sampler: drop-in for the reference's
``kernel/flow_expert.py`` surface.

The module tree (names, registration order, shapes) is the reference's, so
``state_dict``s interchange and ``torch.manual_seed(s); ActionExpert(cfg)``
draws the same default-initialised weights. On CUDA, ``flow_sample`` /
``ActionExpert.forward`` run the whole computation as one fused sm_100a launch
(``ee_flow_sample``); configurations that launch does not cover run an eager
GPU composition whose linears still go through ``ee_wq_gemm``. There is no
CPU path.
"""
from __future__ import annotations

import math
import weakref
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from . import fused as _fused
from .wq_gemm import wq_linear


@dataclass
class ActionExpertConfig:
    """kernel/flow_expert.py:28-35 plus two variant flags.

    ``norm`` ("layernorm", the reference's, or "rmsnorm") and ``self_attn``
    (False drops the action-token self-attention sub-block) describe the
    pre-RMSNorm, cross-attention-only block variant; ``eps`` is the RMSNorm
    epsilon (LayerNorm keeps nn.LayerNorm's 1e-5).
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


def timestep_embedding(t: torch.Tensor, dim: int, max_period: float = 10000.0) -> torch.Tensor:
    """kernel/flow_expert.py:38-48: [cos, sin] of t * freqs * 1000, fp32. The fused
    launch computes the same values in-kernel; this is the module-level helper."""
    half = dim // 2
    freqs = torch.exp(-math.log(max_period)
                      * torch.arange(half, device=t.device, dtype=torch.float32) / half)
    args = t.float()[:, None] * freqs[None] * 1000.0
    emb = torch.cat([torch.cos(args), torch.sin(args)], dim=-1)
    if dim % 2 == 1:
        emb = torch.cat([emb, torch.zeros_like(emb[:, :1])], dim=-1)
    return emb


class RMSNorm(nn.Module):
    """``(x * rsqrt(mean(x^2) + eps))`` rounded to x.dtype, times ``weight``."""

    def __init__(self, d: int, eps: float = 1e-5):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))
        self.eps = eps

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).to(x.dtype) * self.weight


def _norm(cfg):
    return RMSNorm(cfg.d_model, cfg.eps) if getattr(cfg, "norm", "layernorm") == "rmsnorm" \
        else nn.LayerNorm(cfg.d_model)


def _apply_norm(mod, x):
    """The blocks' norm on the layer-by-layer path: nn.LayerNorm of bf16 / fp16
    CUDA activations on the sm_100a row kernel (``ee_layer_norm``: fp32
    statistics, nn.LayerNorm's formula and one rounding); other norms and
    shapes run the module itself."""
    d = x.shape[-1]
    if (isinstance(mod, nn.LayerNorm) and x.is_cuda and x.dtype in (torch.bfloat16, torch.float16)
            and d % 8 == 0 and d <= 2048 and mod.weight is not None and mod.weight.dtype == x.dtype
            and (mod.bias is None or mod.bias.dtype == x.dtype)):
        xf = x.reshape(-1, d)
        if not xf.is_contiguous() or xf.data_ptr() % 16:
            xf = xf.contiguous()
        y = torch.empty_like(xf)
        _lib.check(_lib.load().ee_layer_norm(xf.data_ptr(), mod.weight.data_ptr(), _lib.ptr(mod.bias),
                                             y.data_ptr(), xf.shape[0], d, d, d, float(mod.eps),
                                             _lib.act_code(x.dtype), _lib.stream_ptr(x.device)),
                   "ee_layer_norm")
        return y.reshape(x.shape)
    return mod(x)


def _attention(q, ldq, k, ldk, v, ldv, b: int, h: int, hd: int, n_q: int, n_k: int, q_rows: int, k_rows: int):
    """Non-causal attention on the sm_100a attention units (``ee_attention``)
    from row-major q / k / v (head j at column j * hd, row strides in elements,
    the tensors give pointer, dtype and device); returns the merged-head
    output [b, n_q, h * hd], or None where the kernel does not apply."""
    if (q.dtype not in (torch.bfloat16, torch.float16) or not q.is_cuda or hd not in (64, 128) or n_q > 64
            or any(t.data_ptr() % 16 for t in (q, k, v))):
        return None
    out = torch.empty(b, n_q, h * hd, device=q.device, dtype=q.dtype)
    _lib.check(_lib.load().ee_attention(q.data_ptr(), ldq, k.data_ptr(), ldk, v.data_ptr(), ldv, out.data_ptr(),
                                        h * hd, b, h, hd, n_q, n_k, q_rows, k_rows, _lib.act_code(q.dtype),
                                        _lib.stream_ptr(q.device)), "ee_attention")
    return out


_FREQS: dict = {}


def _row_kernels_ok(x: torch.Tensor) -> bool:
    return x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and x.is_contiguous() and x.data_ptr() % 16 == 0


def _time_embedding_act(t: torch.Tensor, d: int, dtype) -> torch.Tensor:
    """timestep_embedding(t, d).to(dtype) (kernel/flow_expert.py:38-48, :120) on
    the row kernel ``ee_time_embed`` (the fused launch's frequencies and
    arithmetic) for CUDA bf16 / fp16; other inputs take the torch helper."""
    if not (t.is_cuda and dtype in (torch.bfloat16, torch.float16) and t.dtype == dtype and d % 2 == 0):
        return timestep_embedding(t, d).to(dtype)
    key = (t.device, d)
    freqs = _FREQS.get(key)
    if freqs is None:
        freqs = _FREQS[key] = _fused.time_freqs(d, t.device)
    tc = t.contiguous()
    emb = torch.empty(t.shape[0], d, device=t.device, dtype=dtype)
    _lib.check(_lib.load().ee_time_embed(tc.data_ptr(), freqs.data_ptr(), emb.data_ptr(), t.shape[0], d,
                                         _lib.act_code(dtype), _lib.stream_ptr(t.device)), "ee_time_embed")
    return emb


def _expert_head(expert, x_act: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
    """x = in_proj(x_act) + t_proj(temb(t))[:, None] (kernel/flow_expert.py:119-121):
    t_proj on the dequant-GEMM, then ``ee_expert_head`` for the K = action_dim
    in_proj, its bias and the broadcast add in one pass (bf16 / fp16 CUDA);
    other inputs run the torch ops."""
    cfg = expert.cfg
    d, a = cfg.d_model, x_act.shape[-1]
    ip = expert.in_proj
    temb = _apply_linear(expert.t_proj, _time_embedding_act(t, d, x_act.dtype))
    if not (_row_kernels_ok(x_act) and isinstance(ip, nn.Linear) and ip.weight.dtype == x_act.dtype
            and (ip.bias is None or ip.bias.dtype == x_act.dtype) and a % 8 == 0 and a <= 64
            and ip.weight.is_contiguous() and ip.weight.data_ptr() % 16 == 0 and temb.is_contiguous()):
        return _apply_linear(ip, x_act) + temb[:, None, :]
    b, h = x_act.shape[0], x_act.shape[1]
    x = torch.empty(b, h, d, device=x_act.device, dtype=x_act.dtype)
    _lib.check(_lib.load().ee_expert_head(x_act.data_ptr(), ip.weight.data_ptr(), _lib.ptr(ip.bias), temb.data_ptr(),
                                          x.data_ptr(), b * h, a, d, h, d, _lib.act_code(x_act.dtype),
                                          _lib.stream_ptr(x_act.device)), "ee_expert_head")
    return x


def _euler_step(x: torch.Tensor, v: torch.Tensor, t: torch.Tensor, dt: float):
    """x = x + v * dt; t = t + dt (kernel/flow_expert.py:133-136) in place with
    ``ee_euler_step`` (bf16 / fp16 CUDA), else as the torch ops; returns (x, t)."""
    if (_row_kernels_ok(x) and _row_kernels_ok(t) and v.dtype == x.dtype and v.is_contiguous()
            and v.shape == x.shape and t.dtype == x.dtype):
        _lib.check(_lib.load().ee_euler_step(x.data_ptr(), v.data_ptr(), t.data_ptr(), x.numel(), t.shape[0],
                                             float(dt), _lib.act_code(x.dtype), _lib.stream_ptr(x.device)),
                   "ee_euler_step")
        return x, t
    return x + v * dt, t + dt


def _apply_linear(mod, x, gelu: bool = False, residual=None):
    """A linear of the eager path on the sm_100a GEMM (cuBLAS only for K % 128 != 0),
    with GELU or ``residual +`` fused into the GEMM epilogue (the same roundings
    as the separate torch ops: bias add, round, then GELU or residual add, round)."""
    fast = x.dtype in (torch.bfloat16, torch.float16)
    if isinstance(mod, nn.Linear) and mod.in_features % 128 == 0 and fast:
        return wq_linear(x, mod.weight, None, mod.bias, 0, 16, gelu=gelu, residual=residual)
    if type(mod).__name__ == "TritonQuantLinear" and fast:
        return mod.linear(x, gelu=gelu, residual=residual)
    y = F.linear(x, mod.weight, mod.bias) if isinstance(mod, nn.Linear) else mod(x)
    if gelu:
        y = F.gelu(y)
    return y if residual is None else residual + y


class Block(nn.Module):
    """kernel/flow_expert.py:51-95: pre-norm self-attention over the action chunk
    (optional), cross-attention to the cached prefix, GELU MLP."""

    def __init__(self, cfg: ActionExpertConfig):
        super().__init__()
        d, h = cfg.d_model, cfg.n_heads
        assert d % h == 0
        self.h, self.hd = h, d // h
        if getattr(cfg, "self_attn", True):
            self.n1 = _norm(cfg)
            self.qkv = nn.Linear(d, 3 * d)
            self.proj = nn.Linear(d, d)
        else:
            self.n1 = self.qkv = self.proj = None
        self.nx = _norm(cfg)
        self.q_c = nn.Linear(d, d)
        self.kv_c = nn.Linear(d, 2 * d)
        self.out_c = nn.Linear(d, d)
        self.n2 = _norm(cfg)
        hidden = int(d * cfg.mlp_ratio)
        self.mlp = nn.Sequential(nn.Linear(d, hidden), nn.GELU(), nn.Linear(hidden, d))

    def _split(self, x):
        b, t, _ = x.shape
        return x.view(b, t, self.h, self.hd).transpose(1, 2)

    def _merge(self, x):
        b, _, t, _ = x.shape
        return x.transpose(1, 2).contiguous().view(b, t, self.h * self.hd)

    def precompute_kv(self, prefix: torch.Tensor):
        """kernel/flow_expert.py:78-81: prefix [B,P,D] -> (K, V) [B,h,P,hd], views of
        one kv_c output."""
        _lib.require_cuda(prefix)
        k, v = _apply_linear(self.kv_c, prefix).chunk(2, dim=-1)
        return self._split(k), self._split(v)

    def forward(self, x: torch.Tensor, kv_c):
        """Eager GPU composition (used only where the fused launch does not apply)."""
        _lib.require_cuda(x)
        b, n, d = x.shape
        hd = d // self.h
        if self.qkv is not None:
            qkv = _apply_linear(self.qkv, _apply_norm(self.n1, x))
            a = None
            if qkv.is_contiguous():
                a = _attention(qkv, 3 * d, qkv[..., d:], 3 * d, qkv[..., 2 * d:], 3 * d, b, self.h, hd, n, n, n, n)
            if a is None:
                q, k, v = qkv.chunk(3, dim=-1)
                a = self._merge(F.scaled_dot_product_attention(self._split(q), self._split(k), self._split(v)))
            x = _apply_linear(self.proj, a, residual=x)
        qc = _apply_linear(self.q_c, _apply_norm(self.nx, x))
        k, v = kv_c
        a = None
        p = k.shape[2]
        es = k.element_size()
        if (qc.is_contiguous() and k.dtype == qc.dtype and v.dtype == qc.dtype and k.stride() == (p * 2 * d, hd, 2 * d, 1)
                and v.stride() == k.stride() and v.data_ptr() - k.data_ptr() == d * es):
            # the prefix K/V views share one [b, P, 2d] projection output
            a = _attention(qc, d, k, 2 * d, v, 2 * d, b, self.h, hd, n, p, n, p)
        if a is None:
            a = self._merge(F.scaled_dot_product_attention(self._split(qc), k, v))
        x = _apply_linear(self.out_c, a, residual=x)
        return _apply_linear(self.mlp[2], _apply_linear(self.mlp[0], _apply_norm(self.n2, x), gelu=True), residual=x)


class ActionExpert(nn.Module):
    """kernel/flow_expert.py:98-124."""

    def __init__(self, cfg: ActionExpertConfig):
        super().__init__()
        self.cfg = cfg
        d = cfg.d_model
        self.in_proj = nn.Linear(cfg.action_dim, d)
        self.t_proj = nn.Linear(d, d)
        self.blocks = nn.ModuleList([Block(cfg) for _ in range(cfg.n_layers)])
        self.out_norm = _norm(cfg)
        self.out_proj = nn.Linear(d, cfg.action_dim)
        # stand-in for the VLM prefix embedding (kernel/flow_expert.py:108-110)
        self.register_buffer("_prefix", torch.randn(1, cfg.prefix_len, d) * 0.02, persistent=False)

    def encode_prefix(self, batch: int):
        """kernel/flow_expert.py:112-115: per-layer prefix K/V for a batch, computed once."""
        prefix = self._prefix.to(self.out_norm.weight.dtype).expand(batch, -1, -1)
        return [blk.precompute_kv(prefix) for blk in self.blocks]

    def encode(self, prefix: torch.Tensor):
        """Per-layer K/V of an explicit prefix [B, P, d] (one per request)."""
        prefix = prefix.to(self.out_norm.weight.dtype)
        return [blk.precompute_kv(prefix) for blk in self.blocks]

    def plan(self, batch: int, prefix_kv):
        """The fused-launch plan for this batch and prefix K/V (built once, cached)."""
        return get_plan(self, batch, prefix_kv)

    def forward(self, x_act: torch.Tensor, t: torch.Tensor, prefix_kv):
        """kernel/flow_expert.py:117-124: velocity for x_act [B,H,A] at times t [B]."""
        _lib.require_cuda(x_act)
        b = x_act.shape[0]
        if _fused.preferred(self, b, FUSED_MAX_TOKENS):
            v = self.plan(b, prefix_kv).run(x_act, 1, t0=t, mode=_lib.EE_MODE_VELOCITY)
            return v.to(x_act.dtype)
        return self.forward_layers(x_act, t, prefix_kv)

    def forward_layers(self, x_act: torch.Tensor, t: torch.Tensor, prefix_kv):
        """The same velocity computed layer by layer (sm_100a GEMMs with fused
        GELU / residual epilogues, the LayerNorm row kernel and the attention
        launch between them)."""
        x = _expert_head(self, x_act, t)
        for blk, kv in zip(self.blocks, prefix_kv):
            x = blk(x, kv)
        return _apply_linear(self.out_proj, _apply_norm(self.out_norm, x))

    @torch.no_grad()
    def sample(self, prefix: torch.Tensor, steps: int = 10, x0: torch.Tensor | None = None):
        """One sampler call from a raw prefix [B, P, d]: encode the prefix, then
        ``steps`` Euler steps from x0 (N(0,1) noise when not given)."""
        b = prefix.shape[0]
        if x0 is None:
            x0 = torch.randn(b, self.cfg.horizon, self.cfg.action_dim, device=prefix.device,
                             dtype=self.out_norm.weight.dtype)
        return flow_sample(self, x0, steps, self.encode(prefix))


# plans per expert module, outside the module (so deepcopy / state_dict never see them)
_PLANS: "weakref.WeakKeyDictionary" = weakref.WeakKeyDictionary()


def get_plan(expert, batch: int, prefix_kv):
    """Fused-launch plan of any action-expert module (this package's or the
    reference's) for a batch and prefix K/V, cached on the module and rebuilt
    when a parameter or buffer is replaced or modified in place (quantised
    linears keep their integers and scales in buffers, and a plan packs
    private copies of them, so ``load_state_dict`` into a quantised model
    must retire the plan)."""
    key = (batch, tuple(kv[0].data_ptr() for kv in prefix_kv),
           tuple((p.data_ptr(), p._version) for p in expert.parameters()),
           tuple((b.data_ptr(), b._version) for b in expert.buffers()))
    cache = _PLANS.setdefault(expert, {})
    pl = cache.get(key)
    if pl is None:
        if len(cache) > 8:
            cache.clear()
        pl = _fused.FusedPlan(expert, batch, prefix_kv)
        cache[key] = pl
    return pl


# Token count (batch x horizon) up to which a sampler call runs as the single
# fused launch; larger batches are GEMM-throughput work and run layer by layer
# with the tcgen05 dequant-GEMM (GELU / residual in its epilogues).
FUSED_MAX_TOKENS = 600


@torch.no_grad()
def flow_sample(expert, x_init: torch.Tensor, n_steps: int, prefix_kv, path: str = "auto") -> torch.Tensor:
    """kernel/flow_expert.py:127-137: Euler integration over n_steps, t in x.dtype.

    On the fused path all n_steps run in one ``ee_flow_sample`` launch. ``path``:
    "auto" (fused up to FUSED_MAX_TOKENS tokens, else layer by layer), "fused"
    or "layers".
    """
    _lib.require_cuda(x_init)
    b = x_init.shape[0]
    fused_ok = _fused.supports(expert, b)
    if path == "fused" and not fused_ok:
        raise ValueError("the fused launch does not cover this expert / batch")
    use_fused = fused_ok and (path == "fused" or (path == "auto" and _fused.preferred(expert, b, FUSED_MAX_TOKENS)))
    if use_fused:
        return get_plan(expert, b, prefix_kv).run(x_init, n_steps).to(x_init.dtype)
    x = x_init.contiguous().clone()  # updated in place below
    dt = 1.0 / n_steps
    t = torch.zeros(x.shape[0], device=x.device, dtype=x.dtype)
    for _ in range(n_steps):
        v = expert.forward_layers(x, t, prefix_kv) if hasattr(expert, "forward_layers") else expert(x, t, prefix_kv)
        x, t = _euler_step(x, v, t, dt)
    return x


def sample(expert, prefix: torch.Tensor, steps: int = 10, x0: torch.Tensor | None = None):
    """Function form of ``ActionExpert.sample``."""
    return expert.sample(prefix, steps, x0)
