"""Host plan for the fused sampler launch (``ee_flow_sample``).

A plan binds one action-expert module (this package's ``ActionExpert`` or the
reference's, with dense ``nn.Linear`` or quantised linears) and one set of
cached prefix K/V to the C ABI: it gathers device pointers into the
``ee_expert`` / ``ee_block`` records, uploads the block table, computes the
time-embedding frequencies exactly as kernel/flow_expert.py:41-43 does, and
owns the workspace. Building a plan is host work done once; ``run`` is one
asynchronous launch on the current stream (capturable in a CUDA graph).
"""
from __future__ import annotations

import ctypes
import math

import torch
import torch.nn as nn

from . import _lib
from .wq_gemm import _pack_int4


def _is_quant_linear(m) -> bool:
    return type(m).__name__ == "TritonQuantLinear" and hasattr(m, "scales") and hasattr(m, "bits")


def _is_ref_quantlinear(m) -> bool:  # the reference's dequantise-then-matmul module
    return type(m).__name__ == "QuantLinear" and hasattr(m, "q") and hasattr(m, "scale")


def supports(expert, batch: int) -> bool:
    """Whether the fused launch covers this expert (else callers run the eager path)."""
    try:
        cfg = expert.cfg
        d, h = cfg.d_model, cfg.n_heads
        hid = int(d * cfg.mlp_ratio)
        if d % 256 or d > 2048 or d % h or (d // h) not in (64, 128):
            return False
        if cfg.horizon > 64 or cfg.action_dim % 8 or not (8 <= cfg.action_dim <= 32):
            return False
        if hid % 128:
            return False
        # one CTA stages at most a 512-wide K slice (K split over a cluster of 8,
        # or of 16 where the width splits into 16 k-block slices and the device
        # can hold such clusters): the MLP down-projection's K bounds the launch
        if max(hid, d) > 8 * 512:
            if max(hid, d) > 16 * 512 or (d // 128) % 16:
                return False
            if not _wide_geometry_ok(cfg, batch, expert.out_norm.weight.dtype):
                return False
        for blk in expert.blocks:
            mods = [blk.q_c, blk.out_c, blk.mlp[0], blk.mlp[2]]
            if getattr(blk, "qkv", None) is not None:
                mods += [blk.qkv, blk.proj]
            for m in mods:
                if not (isinstance(m, nn.Linear) or _is_quant_linear(m) or _is_ref_quantlinear(m)):
                    return False
        return isinstance(expert.in_proj, nn.Linear) and isinstance(expert.out_proj, nn.Linear)
    except AttributeError:
        return False


def preferred(expert, batch: int, max_tokens: int) -> bool:
    """Whether ``flow_sample(path="auto")`` should take the fused launch:
    supported, at most ``max_tokens`` tokens, and a model whose widest K
    slice fits an 8-CTA cluster. Wider models (the 8192-wide MLP at
    d_model 2048) run in the fused launch only on request: there every phase
    streams megabytes of weights from HBM with a small prefetch area per CTA,
    and the layer-by-layer path measured faster (Pi0-scale expert, batch 1,
    int4: 30.1 vs 32.2 ms per 10-step call; bf16 28.2 vs 50.5 ms)."""
    cfg = expert.cfg
    if max(int(cfg.d_model * cfg.mlp_ratio), cfg.d_model) > 8 * 512:
        return False
    return batch * cfg.horizon <= max_tokens and supports(expert, batch)


_GEOMETRY_OK: dict = {}


def _wide_geometry_ok(cfg, batch: int, dtype) -> bool:
    """Whether the current device can launch the fused sampler for a model
    whose MLP needs 16-CTA clusters (non-portable): asks
    ``ee_flow_sample_geometry`` once per shape and device."""
    if not torch.cuda.is_available():
        return False
    dev = torch.cuda.current_device()
    d = cfg.d_model
    key = (dev, d, cfg.n_layers, cfg.n_heads, int(d * cfg.mlp_ratio), cfg.horizon, batch, str(dtype))
    if key not in _GEOMETRY_OK:
        ex = _lib.Expert()
        ex.d_model, ex.n_layers, ex.n_heads = d, cfg.n_layers, cfg.n_heads
        ex.horizon, ex.action_dim, ex.prefix_len = cfg.horizon, cfg.action_dim, cfg.prefix_len
        ex.hidden, ex.batch = int(d * cfg.mlp_ratio), batch
        ex.act_dtype = _lib.act_code(dtype if dtype in (torch.bfloat16, torch.float16) else torch.bfloat16)
        ex.self_attn = 1 if getattr(cfg, "self_attn", True) else 0
        g, c, sm = ctypes.c_int32(0), ctypes.c_int32(0), ctypes.c_size_t(0)
        rc = _lib.load().ee_flow_sample_geometry(ctypes.byref(ex), ctypes.byref(g), ctypes.byref(c),
                                                 ctypes.byref(sm))
        _GEOMETRY_OK[key] = rc == 0 and g.value > 0
    return _GEOMETRY_OK[key]


def time_freqs(d: int, device) -> torch.Tensor:
    """kernel/flow_expert.py:41-43, computed on the host with the same torch ops."""
    half = d // 2
    f = torch.exp(-math.log(10000.0) * torch.arange(half, dtype=torch.float32) / half)
    return f.to(device)


class FusedPlan:
    def __init__(self, expert, batch: int, prefix_kv, device=None):
        cfg = expert.cfg
        self.cfg = cfg
        self.batch = int(batch)
        self.device = torch.device(device) if device is not None else next(expert.parameters()).device
        if self.device.type != "cuda":
            raise RuntimeError("the fused sampler needs the expert on a CUDA device")
        pdtype = expert.out_norm.weight.dtype
        self.act = pdtype if pdtype in (torch.bfloat16, torch.float16) else torch.bfloat16
        self._keep = []  # tensors whose pointers the plan holds
        d = cfg.d_model
        self.d = d
        self.hidden = int(d * cfg.mlp_ratio)
        self.rms = getattr(cfg, "norm", "layernorm") == "rmsnorm"
        self.self_attn = bool(getattr(cfg, "self_attn", True))

        ex = _lib.Expert()
        ex.d_model, ex.n_layers, ex.n_heads = d, cfg.n_layers, cfg.n_heads
        ex.horizon, ex.action_dim, ex.prefix_len = cfg.horizon, cfg.action_dim, cfg.prefix_len
        ex.hidden, ex.batch = self.hidden, self.batch
        ex.act_dtype = _lib.act_code(self.act)
        ex.norm_kind = _lib.EE_NORM_RMS if self.rms else _lib.EE_NORM_LAYER
        ex.self_attn = 1 if self.self_attn else 0
        ex.eps = float(getattr(cfg, "eps", 1e-5)) if self.rms else float(expert.out_norm.eps)
        freqs = time_freqs(d, self.device)
        self._keep.append(freqs)
        ex.freqs = freqs.data_ptr()
        ex.in_proj = self._linear(expert.in_proj)
        ex.t_proj = self._linear(expert.t_proj)
        ex.out_proj = self._linear(expert.out_proj)
        ex.out_norm = self._norm(expert.out_norm)

        blocks = (_lib.Block * cfg.n_layers)()
        for i, blk in enumerate(expert.blocks):
            b = blocks[i]
            if self.self_attn:
                b.n1 = self._norm(blk.n1)
                b.qkv = self._linear(blk.qkv)
                b.proj = self._linear(blk.proj)
            b.nx = self._norm(blk.nx)
            b.q_c = self._linear(blk.q_c)
            b.out_c = self._linear(blk.out_c)
            b.n2 = self._norm(blk.n2)
            b.mlp0 = self._linear(blk.mlp[0])
            b.mlp2 = self._linear(blk.mlp[2])
            b.kv = self._kv(prefix_kv[i]).data_ptr()
        raw = torch.frombuffer(bytearray(ctypes.string_at(blocks, ctypes.sizeof(blocks))),
                               dtype=torch.uint8)
        dev_blocks = raw.to(self.device)
        self._keep.append(dev_blocks)
        ex.blocks = dev_blocks.data_ptr()
        self.ex = ex
        self.host_blocks = blocks
        lib = _lib.load()
        _lib.check(lib.ee_check_expert(ctypes.byref(ex), blocks, 1, _lib.EE_MODE_EULER),
                   "ee_check_expert")
        # TMA descriptors of the cached prefix K/V (head size 64): the
        # cross-attention then loads K/V tiles with TMA instead of cp.async
        self.kv_maps = None
        if d // cfg.n_heads == 64:
            maps = torch.empty(cfg.n_layers * 128, dtype=torch.uint8, device=self.device)
            rc = lib.ee_encode_kv_maps(ctypes.byref(ex), blocks, maps.data_ptr(), maps.numel(),
                                       _lib.stream_ptr(self.device))
            if rc == 0:
                self.kv_maps = maps
                ex.kv_maps = maps.data_ptr()
        self._ws = {}

    # -- record builders ---------------------------------------------------
    def _own(self, t):
        t = t.to(self.device)
        self._keep.append(t)
        return t

    def _act_tensor(self, t):
        if t is None:
            return None
        if t.dtype != self.act or not t.is_contiguous() or t.device != self.device:
            t = t.to(device=self.device, dtype=self.act).contiguous()
        self._keep.append(t)
        return t

    def _norm(self, m) -> _lib.Norm:
        r = _lib.Norm()
        r.weight = self._act_tensor(m.weight.detach()).data_ptr()
        b = getattr(m, "bias", None)
        r.bias = self._act_tensor(b.detach()).data_ptr() if b is not None else 0
        return r

    def _linear(self, m) -> _lib.Linear:
        r = _lib.Linear()
        bias = getattr(m, "bias", None)
        r.bias = self._act_tensor(bias.detach()).data_ptr() if bias is not None else 0
        if _is_quant_linear(m):
            r.weight = self._own(m.weight.contiguous()).data_ptr()
            r.scales = self._own(m.scales.float().contiguous()).data_ptr()
            r.n, r.k = m.out_features, m.in_features
            r.wkind = _lib.EE_W_INT4 if m.bits == 4 else _lib.EE_W_INT8
            r.group = m.group_size
            r.scale_dtype = _lib.EE_F32
        elif _is_ref_quantlinear(m):
            n, ng, gs = m.q.shape
            q2d = m.q.reshape(n, ng * gs).to(self.device)
            w = _pack_int4(q2d) if m.bits == 4 else q2d.contiguous()
            r.weight = self._own(w).data_ptr()
            r.scales = self._own(m.scale.reshape(n, ng).float().contiguous()).data_ptr()
            r.n, r.k = n, ng * gs
            r.wkind = _lib.EE_W_INT4 if m.bits == 4 else _lib.EE_W_INT8
            r.group = gs
            r.scale_dtype = _lib.EE_F32
        else:
            w = self._act_tensor(m.weight.detach())
            r.weight = w.data_ptr()
            r.n, r.k = w.shape
            r.wkind = _lib.EE_W_DENSE
        return r

    def _kv(self, kv):
        """Prefix K/V of one block as the [batch, P, 2d] kv_c output it is a view of."""
        k, v = kv
        b, h, p, hd = k.shape
        d = h * hd
        es = k.element_size()
        if (k.dtype == self.act and v.dtype == self.act and k.stride() == (p * 2 * d, hd, 2 * d, 1)
                and v.stride() == k.stride() and v.data_ptr() - k.data_ptr() == d * es
                and k.device == self.device):
            base = k.as_strided((b, p, 2 * d), (p * 2 * d, 2 * d, 1))
        else:
            base = torch.cat([k.transpose(1, 2).reshape(b, p, d), v.transpose(1, 2).reshape(b, p, d)],
                             dim=-1).to(device=self.device, dtype=self.act).contiguous()
        if b != self.batch or p != self.cfg.prefix_len:
            raise ValueError(f"prefix K/V has batch {b}, length {p}; plan expects "
                             f"{self.batch}, {self.cfg.prefix_len}")
        self._keep.append(base)
        return base

    # -- launch ------------------------------------------------------------
    def workspace(self, n_steps: int) -> torch.Tensor:
        ws = self._ws.get(n_steps)
        if ws is None:
            nbytes = _lib.load().ee_flow_sample_workspace_bytes(ctypes.byref(self.ex), n_steps)
            ws = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
            self._ws[n_steps] = ws
        return ws

    def run(self, x, n_steps: int, t0=None, mode: int = _lib.EE_MODE_EULER, out=None):
        """x [batch, horizon, action_dim] on the plan's device -> new tensor (or ``out``)."""
        if x.shape != (self.batch, self.cfg.horizon, self.cfg.action_dim):
            raise ValueError(f"x has shape {tuple(x.shape)}")
        xin = x if (x.dtype == self.act and x.is_contiguous()) else x.to(self.act).contiguous()
        if out is None:
            out = torch.empty_like(xin)
        tt = None
        if t0 is not None:
            tt = t0.to(device=self.device, dtype=self.act).reshape(self.batch).contiguous()
        ws = self.workspace(n_steps)
        rc = _lib.load().ee_flow_sample(ctypes.byref(self.ex), xin.data_ptr(), _lib.ptr(tt),
                                        out.data_ptr(), n_steps, mode, ws.data_ptr(), ws.numel(),
                                        _lib.stream_ptr(self.device))
        _lib.check(rc, "ee_flow_sample")
        return out

    def trace(self, x, n_steps: int):
        """Run one call with the device phase timeline on; returns (phase kinds,
        int64 tensor [n_phases, grid, 2] of globaltimer ns: work done, barrier left)."""
        lib = _lib.load()
        grid, _, _ = self.geometry()
        nph = lib.ee_flow_sample_phases(ctypes.byref(self.ex), n_steps)
        tr = torch.zeros(nph, grid, 2, dtype=torch.int64, device=self.device)
        xin = x.to(self.act).contiguous()
        out = torch.empty_like(xin)
        ws = self.workspace(n_steps)
        _lib.check(lib.ee_flow_sample_traced(ctypes.byref(self.ex), xin.data_ptr(), None,
                                             out.data_ptr(), n_steps, _lib.EE_MODE_EULER,
                                             ws.data_ptr(), ws.numel(), tr.data_ptr(),
                                             _lib.stream_ptr(self.device)), "ee_flow_sample_traced")
        torch.cuda.synchronize(self.device)
        per_block = ["qkv", "self_attn", "proj", "q_c", "cross_attn", "out_c", "mlp0", "mlp2"]
        if not self.self_attn:
            per_block = per_block[3:]
        kinds = ["emb", "t_proj", "head"]
        for _ in range(n_steps):
            kinds += per_block * self.cfg.n_layers + ["tail"]
        return kinds, tr.cpu()

    def geometry(self):
        """(grid CTAs, CTAs per cluster, dynamic shared memory bytes) of the launch."""
        g, c, sm = ctypes.c_int32(0), ctypes.c_int32(0), ctypes.c_size_t(0)
        _lib.check(_lib.load().ee_flow_sample_geometry(ctypes.byref(self.ex), ctypes.byref(g),
                                                       ctypes.byref(c), ctypes.byref(sm)),
                   "ee_flow_sample_geometry")
        return g.value, c.value, sm.value

    def status(self, n_steps: int) -> int:
        """Device status word of the last launch with ``n_steps`` (synchronises)."""
        st = ctypes.c_int32(0)
        ws = self.workspace(n_steps)
        _lib.check(_lib.load().ee_read_status(ws.data_ptr(), ctypes.byref(st),
                                              _lib.stream_ptr(self.device)), "ee_read_status")
        return st.value
