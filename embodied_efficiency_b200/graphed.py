"""CUDA-graph sampler: drop-in for the reference's ``kernel/cudagraph.py``.

``GraphedSampler(expert, x_template, n_steps)`` builds the fused-launch plan,
warms it up on a side stream, captures one sampler call (copy-in + the single
``ee_flow_sample`` launch) into a CUDA graph, and ``run(x)`` replays it:
static input ``copy_``, ``replay``, ``clone`` of the static output -- the
reference's contract (kernel/cudagraph.py:29-57), including its stale-input
and output-aliasing defences.
"""
from __future__ import annotations

import torch

from . import _lib
from . import fused as _fused
from . import expert as _expert
from .expert import flow_sample, get_plan


class GraphedSampler:
    """Captures ``flow_sample(expert, x, n_steps)`` into a CUDA graph with a static input."""

    def __init__(self, expert, x_template, n_steps, warmup=5, prefix_kv=None):
        """``prefix_kv`` (not in the reference, whose sampler always encodes
        the module's own prefix) bakes given per-layer K/V -- requests' own
        prefixes, as fleet mode has them -- into the graph instead of
        ``expert.encode_prefix(batch)``."""
        _lib.require_cuda(x_template)
        self.expert, self.n = expert, n_steps
        self.cuda = True
        # constant, baked into the graph
        self.prefix_kv = prefix_kv if prefix_kv is not None else expert.encode_prefix(x_template.shape[0])
        self.static_in = x_template.clone()
        b = x_template.shape[0]
        # the same choice flow_sample makes: the single fused launch up to
        # FUSED_MAX_TOKENS tokens, else the layer-by-layer path (captured too)
        self.fused = _fused.preferred(expert, b, _expert.FUSED_MAX_TOKENS)
        self.plan = get_plan(expert, b, self.prefix_kv) if self.fused else None
        if self.fused:
            self.static_out = torch.empty_like(self.static_in, dtype=self.plan.act)
            self.plan.workspace(n_steps)  # allocate before capture
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self._body()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            out = self._body()
        if not self.fused:
            self.static_out = out

    def _body(self):
        if self.fused:
            return self.plan.run(self.static_in, self.n, out=self.static_out)
        return flow_sample(self.expert, self.static_in, self.n, self.prefix_kv)

    def run(self, x):
        self.static_in.copy_(x)          # never trust the new tensor's address, copy in
        self.graph.replay()
        return self.static_out.to(x.dtype).clone()  # storage is reused on next replay

    def replay(self):
        """Replay on the input already in ``static_in``; returns ``static_out``
        itself (overwritten by the next replay, no copy)."""
        self.graph.replay()
        return self.static_out

    def status(self) -> int:
        """Device status word of the last replay (synchronises); 0 = ok."""
        return self.plan.status(self.n) if self.fused else 0


def _build(bits=None, device="cuda", seed=0, cfg=None, dtype=torch.bfloat16):
    """kernel/cudagraph.py:60-71: seeded expert, optionally quantised."""
    from .expert import ActionExpert, ActionExpertConfig
    from .wq_gemm import quantize_model_triton
    torch.manual_seed(seed)
    m = ActionExpert(cfg or ActionExpertConfig()).to(device).to(dtype).eval()
    if bits:
        quantize_model_triton(m, bits=bits)
    return m


def eval_all(n=10, B=1, tol=2e-1, cfg=None, dtype=torch.bfloat16):
    """kernel/cudagraph.py:73-108 GPU evals: graph vs eager on two distinct inputs
    (stale-input check) and no memory growth over 50 replays. Returns per-precision
    (max_err, leaked_bytes)."""
    res = {}
    for label, bits in [("bf16" if dtype == torch.bfloat16 else "fp16", None), ("int8", 8), ("int4", 4)]:
        m = _build(bits=bits, cfg=cfg, dtype=dtype)
        xt = torch.randn(B, m.cfg.horizon, m.cfg.action_dim, device="cuda", dtype=dtype)
        gs = GraphedSampler(m, xt, n)
        pkv = gs.prefix_kv
        max_err = 0.0
        for _ in range(2):
            x = torch.randn_like(xt)
            max_err = max(max_err, (gs.run(x) - flow_sample(m, x, n, pkv)).abs().max().item())
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        m0 = torch.cuda.memory_allocated()
        for _ in range(50):
            gs.run(xt)
        torch.cuda.synchronize()
        leaked = torch.cuda.memory_allocated() - m0
        ok = max_err < tol and leaked <= 4096
        print(f"  {label:5s} graph: max_err={max_err:.3e}  leaked={leaked}B  -> {'OK' if ok else 'FAIL'}")
        res[label] = (max_err, leaked)
    return res
