#!/usr/bin/env python
"""Benchmark of the fused flow-matching sampler (one JSON line on rank 0).

Headline metric: ms per 10-step sampler call at batch 1, on the action expert
with d_model 1024, 4 blocks, 16 heads x 64, MLP 4096, prefix 256, horizon 50,
action dim 32 (synthetic seeded weights and inputs), int4 group-128 weights,
bf16 activations. A "step" of this benchmark is one sampler call (10 Euler
steps). ``value`` is device time per call with inputs resident in HBM and the
L2 flushed between calls; ``e2e`` is the same call through ``GraphedSampler``
with the input in pinned host memory and the result copied back to the host
inside the timed region. bf16 and int8 weights are reported beside int4; at
N=1 also the standalone dequant-GEMM's HBM throughput (``gemm``), the prefix
encoder's kv_c GEMM (``kv_prefix_gemm``), the reference-default expert
(``config3_ref``) and the Pi0-scale expert (``config5``).

Multi-GPU (torchrun, one rank per GPU): independent replicas of the batch-1
call (the call does not shard); ``value`` is the latency of one call, the
max over ranks of each rank's mean device time per call, ``scaling`` "weak".
The sharded workload is fleet mode (``fleet``): 256 independent requests
split over the ranks, aggregate actions/s, measured at every N.

``--impl reference`` times the CPU restatement of the reference's own path
(the oracle: dequantise-then-matmul + eager Euler loop in torch on the host
cores, all threads) on the same workload and prints the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

WORKLOAD = dict(d_model=1024, n_layers=4, n_heads=16, horizon=50, action_dim=32, prefix_len=256,
                mlp_ratio=4.0)
METRIC = "ms per 10-step sampler call (batch 1)"
# the reference's default expert (kernel/flow_expert.py:28-35), the shape of its published numbers
CONFIG3_REF = dict(d_model=512, n_layers=6, n_heads=8, horizon=50, action_dim=32, prefix_len=256, mlp_ratio=4.0)
# the Pi0-scale expert: 18 blocks of width 2048, MLP 8192, 16 heads x 128, prefix 816
CONFIG5 = dict(d_model=2048, n_layers=18, n_heads=16, horizon=50, action_dim=32, prefix_len=816, mlp_ratio=4.0)
N_STEPS = 10
L2_FLUSH_BYTES = 256 << 20
# DRAM bytes (read + write) of one sampler_kernel launch of WORKLOAD at int4,
# from one ncu capture (36.46 MB read + 0.37 MB written): the weights come
# from HBM once per call and from L2 for the other nine steps.
SAMPLER_DRAM_BYTES = 36829696


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def linear_bytes(n, k, bits, group=128):
    """Algorithmic bytes of one linear: weights + fp16-counted scales + bias
    (the reference's accounting, kernel/quant.py:58-59)."""
    if bits == 16:
        return n * k * 2 + n * 2
    return n * k * bits // 8 + n * (k // group) * 2 + n * 2


def step_bytes(cfg, bits, batch=1):
    """Bytes one Euler step must read: every per-step linear (t_proj, the six
    block linears, dense in/out projections), norm parameters; plus the cached
    prefix K/V separately."""
    d, hid, a = cfg["d_model"], int(cfg["d_model"] * cfg["mlp_ratio"]), cfg["action_dim"]
    w = linear_bytes(d, d, bits) + linear_bytes(d, a, 16) + linear_bytes(a, d, 16)
    per_block = (linear_bytes(3 * d, d, bits) + linear_bytes(d, d, bits) * 3
                 + linear_bytes(hid, d, bits) + linear_bytes(d, hid, bits) + 3 * 2 * d * 2)
    w += cfg["n_layers"] * per_block + 2 * d * 2
    kv = cfg["n_layers"] * 2 * batch * cfg["prefix_len"] * d * 2
    return w, kv


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms while running.
    Entering waits (up to 5 s) for the first sample, so a short timed region
    that starts afterwards is covered by samples."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        import threading
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return self
        first = threading.Event()

        def reader():
            for ln in self.proc.stdout:
                if ln.strip():
                    self.lines.append(ln.strip())
                    first.set()
            first.set()

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()
        first.wait(5.0)
        self.t_start = len(self.lines)  # samples taken before the timed region are not counted
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.thread.join(timeout=5)
            self.lines = self.lines[max(0, getattr(self, "t_start", 0) - 1):]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(backend):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        kw = {"device_id": torch.device("cuda", local)} if backend == "nccl" else {}
        torch.distributed.init_process_group(backend, timeout=datetime.timedelta(seconds=120), **kw)
    return rank, world, local


def build_expert(bits, device):
    from embodied_efficiency_b200 import ActionExpert, ActionExpertConfig, quantize_model_triton, synth
    cfg = ActionExpertConfig(**WORKLOAD)
    params, x0, prefix = synth.workload(cfg, seed=0, batch=1)
    torch.manual_seed(0)  # the module's stand-in prefix buffer (used by GraphedSampler)
    m = ActionExpert(cfg)
    m.load_state_dict(params)
    m = m.to(device).bfloat16().eval()
    if bits != 16:
        quantize_model_triton(m, bits=bits)
    return m, x0, prefix


def time_calls(fn, steps, warmup, flush):
    """Per-call device time (CUDA events on the launching stream), L2 flushed
    between calls; returns the list of per-call ms."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    for i in range(steps):
        flush.zero_()
        ev[i][0].record()
        fn()
        ev[i][1].record()
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in ev]


def _weight_copies(n, k, bits, device, copies, g):
    """`copies` independent [n, k] weights (packed int4 / int8 + fp32 scales,
    or bf16), quantised from N(0, 0.02) draws."""
    from embodied_efficiency_b200.quant import quantize_weight
    from embodied_efficiency_b200.wq_gemm import _pack_int4
    out = []
    for _ in range(copies):
        w = torch.randn(n, k, generator=g, device=device) * 0.02
        if bits == 16:
            out.append((w.bfloat16(), None))
        else:
            q, sc, _ = quantize_weight(w, bits, 128)
            q2 = q.reshape(n, k)
            out.append((_pack_int4(q2) if bits == 4 else q2, sc.reshape(n, -1)))
        del w
    return out


def gemm_sweep(device, shapes=((4096, 4096), (8192, 8192), (6144, 2048), (8192, 2048), (2048, 8192)),
               ms=(1, 16, 50), bits_list=(4, 8, 16), reps=20):
    """Standalone dequant-GEMM (``wq_linear``), N x K weights, M tokens:
    back-to-back launches replayed from one CUDA graph that cycles through
    enough independent weight copies to exceed twice the L2 (each launch
    reads its weights from HBM); per-launch time = graph time / launches.
    Reports algorithmic HBM GB/s (weights + fp16-counted scales +
    activations + output) and TFLOP/s."""
    from embodied_efficiency_b200 import wq_linear
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    g = torch.Generator(device=device).manual_seed(0)
    out = {}
    for (n, k) in shapes:
        for bits in bits_list:
            wbytes = linear_bytes(n, k, bits) - n * 2
            copies = max(2, min(64, -(-2 * l2 // wbytes)))
            mats = _weight_copies(n, k, bits, device, copies, g)
            for m in ms:
                x = torch.randn(m, k, generator=g, device=device).bfloat16()
                for wt, sc in mats[:2]:
                    wq_linear(x, wt, sc, None, 128, bits)
                torch.cuda.synchronize()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    for wt, sc in mats:
                        wq_linear(x, wt, sc, None, 128, bits)
                graph.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(reps):
                    graph.replay()
                e1.record()
                torch.cuda.synchronize()
                t = e0.elapsed_time(e1) / (reps * copies)
                nbytes = wbytes + m * k * 2 + m * n * 2
                out[f"n{n}_k{k}_m{m}_{'bf16' if bits == 16 else f'int{bits}'}"] = {
                    "us": round(t * 1e3, 2), "GBps": round(nbytes / (t * 1e-3) / 1e9, 1),
                    "TFLOPs": round(2.0 * m * n * k / (t * 1e-3) / 1e12, 1)}
                del graph
            del mats
            torch.cuda.empty_cache()
    return out


def sampler_variants(cfg_kw, device, flush, bits_list=(16, 8, 4), calls=20, warmup=5, batch=1):
    """ms per 10-step call (device time, L2 flushed between calls) of an
    expert of the given shape at bf16 / int8 / int4 weights, batch ``batch``;
    weights drawn on the device (not the oracle's seeded set)."""
    from embodied_efficiency_b200 import ActionExpert, ActionExpertConfig, GraphedSampler, quantize_model_triton
    cfg = ActionExpertConfig(**cfg_kw)
    out = {}
    for bits in bits_list:
        torch.manual_seed(0)
        with torch.device(device):
            m = ActionExpert(cfg)
        with torch.no_grad():
            for name, prm in m.named_parameters():
                if "n1" in name or "nx" in name or "n2" in name or "out_norm" in name:
                    continue
                prm.normal_(0.0, 0.02)
        m = m.bfloat16().eval()
        if bits != 16:
            quantize_model_triton(m, bits=bits)
        g = torch.Generator(device=device).manual_seed(1)
        x = torch.randn(batch, cfg.horizon, cfg.action_dim, generator=g, device=device).bfloat16()
        prefix = torch.randn(batch, cfg.prefix_len, cfg.d_model, generator=g, device=device).bfloat16()
        gs = GraphedSampler(m, x, N_STEPS, warmup=2, prefix_kv=m.encode(prefix))
        ms = time_calls(gs.replay, calls, warmup, flush)
        w_b, kv_b = step_bytes(cfg_kw, bits, batch)
        t = statistics.median(ms)
        out["bf16" if bits == 16 else f"int{bits}"] = {
            "ms_per_call": round(t, 4), "weight_MB_per_step": round(w_b / 1e6, 2),
            "weight_GBps": round(w_b * N_STEPS / (t * 1e-3) / 1e9, 1),
            "path": "fused launch" if gs.fused else "layer by layer (CUDA graph)"}
        del gs, m
        torch.cuda.empty_cache()
    return out


def kv_prefix_gemm(device, flush):
    """The prefix encoder's kv_c GEMM (kernel/flow_expert.py:78-81, once per
    call): M = P * batch tokens, N = 2 d, K = d, int4 group-128; device time
    per launch (L2 flushed), TFLOP/s and algorithmic GB/s."""
    from embodied_efficiency_b200 import wq_linear
    g = torch.Generator(device=device).manual_seed(0)
    out = {}
    for tag, d, p, b in (("c3_P256_B1", 1024, 256, 1), ("c5_P816_B1", 2048, 816, 1),
                         ("c5_P816_B8", 2048, 816, 8), ("fleet_P256_B256", 1024, 256, 256)):
        (wt, sc), = _weight_copies(2 * d, d, 4, device, 1, g)
        x = torch.randn(p * b, d, generator=g, device=device).bfloat16()
        ms = time_calls(lambda: wq_linear(x, wt, sc, None, 128, 4), 20, 3, flush)
        t = statistics.median(ms)
        m = p * b
        nbytes = linear_bytes(2 * d, d, 4) + m * d * 2 + m * 2 * d * 2
        out[tag] = {"M": m, "N": 2 * d, "K": d, "us": round(t * 1e3, 2),
                    "TFLOPs": round(2.0 * m * 2 * d * d / (t * 1e-3) / 1e12, 1),
                    "GBps": round(nbytes / (t * 1e-3) / 1e9, 1)}
        del wt, sc, x
    return out


def fleet_run(expert, rank, world, dev, n_requests=256, chunk=256, steps=5, warmup=3):
    """Fleet mode: n_requests independent int4 sampler requests (request r
    seeded with r) sharded in contiguous blocks over the ranks, no collective;
    device time of one fleet step (every chunk of this rank), max over ranks."""
    from embodied_efficiency_b200 import synth
    from embodied_efficiency_b200.fleet import FleetSampler
    cfg = expert.cfg
    fs = FleetSampler(n_requests, rank, world, chunk=chunk, expert=expert, device=dev)
    fs.stage(lambda i: synth.fleet_request(cfg, i))
    for _ in range(warmup):
        fs.run_device()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fs.run_device()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / steps], device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = t.item()
    return {"metric": "actions/s", "value": round(n_requests * cfg.horizon / (ms * 1e-3), 1),
            "unit": "actions/s", "requests": n_requests, "requests_per_gpu": fs.hi - fs.lo,
            "chunk": chunk, "ms_per_fleet_step": round(ms, 3), "n_gpus": world,
            "workload": "256 requests x (10-step int4 group-128 sampler, d1024 L4, own prefix and noise)",
            "scaling": "strong (fixed 256 requests split over the GPUs)", "collectives": "none on the data path"}


def fleet_share_run(expert, world, dev, n_requests=256, chunk=256, steps=5, warmup=3):
    """Rank 0's share of the fleet for a world of `world` GPUs, timed on this
    one GPU. Fleet mode has no collective, so a rank's fleet step is its own
    work; the aggregate it projects for `world` GPUs is n_requests * horizon /
    (rank 0's step time), rank 0 holding the largest share."""
    from embodied_efficiency_b200 import synth
    from embodied_efficiency_b200.fleet import FleetSampler
    cfg = expert.cfg
    fs = FleetSampler(n_requests, 0, world, chunk=chunk, expert=expert, device=dev)
    fs.stage(lambda i: synth.fleet_request(cfg, i))
    for _ in range(warmup):
        fs.run_device()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fs.run_device()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    return {"world": world, "requests_per_gpu": fs.hi - fs.lo, "ms_per_fleet_step": round(ms, 3),
            "projected_actions_per_s": round(n_requests * cfg.horizon / (ms * 1e-3), 1)}


def cpu_baseline_run(budget_s=15.0, bits=4):
    """The oracle (CPU restatement of the reference path) on the host cores."""
    from embodied_efficiency_b200 import synth
    from oracle import sampler as OS
    cfg = OS.Cfg(**WORKLOAD)
    params, x0, prefix = synth.workload(cfg, seed=0, batch=1)
    p = {k: v.bfloat16() for k, v in params.items()}
    qp = OS.quantize_params(p, cfg, bits) if bits != 16 else None
    kv = OS.encode_prefix(p, cfg, prefix.bfloat16(), qp)
    xb = x0.bfloat16()
    OS.flow_sample(p, cfg, xb, N_STEPS, kv, qp)  # warm-up
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 2:
        t0 = time.perf_counter()
        OS.flow_sample(p, cfg, xb, N_STEPS, kv, qp)
        times.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(times), len(times)


def run_reference(args):
    rank, world, _ = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), 0
    if rank != 0:
        return
    from embodied_efficiency_b200 import synth
    from oracle import sampler as OS
    torch.set_num_threads(os.cpu_count() or 1)
    cfg = OS.Cfg(**WORKLOAD)
    params, x0, prefix = synth.workload(cfg, seed=0, batch=1)
    p = {k: v.bfloat16() for k, v in params.items()}
    qp = OS.quantize_params(p, cfg, 4)
    kv = OS.encode_prefix(p, cfg, prefix.bfloat16(), qp)
    xb = x0.bfloat16()
    for _ in range(max(args.warmup, 1)):
        OS.flow_sample(p, cfg, xb, N_STEPS, kv, qp)
    times = []
    t_start = time.perf_counter()
    for i in range(args.steps):
        t0 = time.perf_counter()
        OS.flow_sample(p, cfg, xb, N_STEPS, kv, qp)
        times.append((time.perf_counter() - t0) * 1e3)
        if time.perf_counter() - t_start > 150 and i >= 2:
            break
    v = statistics.mean(times)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "ms",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(v, 3),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": "action-expert sampler d1024 L4 h16x64 mlp4096 P256 H50 A32, "
                               "batch 1, 10 Euler steps, int4 group-128", "weights": "int4",
                   "batch": 1, "n_steps": N_STEPS},
        "cpu_baseline": {"value": round(v, 3), "unit": "ms", "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": f"{len(times)} full sampler calls (oracle restatement of the "
                                   "reference's dequantise-then-matmul eager loop, torch CPU)"},
        "e2e": {"value": round(v, 3), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def profile_case(spec, launches):
    """A few launches of one kernel for a profiler (no timing, no JSON):
    ``gemm:M:K:BITS[:N[:gelu]]`` runs the standalone dequant-GEMM on a K x N
    weight (N = K unless given; BITS 16 = dense bf16), with the GELU epilogue
    when asked,
    ``sampler:BITS`` replays the captured sampler call (a plain cluster launch
    inside a CUDA graph), ``norm:ROWS:COLS`` runs the LayerNorm row kernel and
    ``attn:BATCH:P`` the layer path's cross-attention of BATCH requests (50
    queries, 16 heads of 64, P prefix keys), ``selfattn:BATCH`` its
    self-attention over the 50 action tokens (q / k / v read in place from the
    fused projection) and ``dequant:N:K:BITS`` the weight dequantisation
    kernel on an [N, K] weight (group 128), ``fleet:WORLD`` rank 0's share of
    the 256-request int4 fleet for WORLD GPUs (its fleet steps after two
    warm-up steps)."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    kind, *rest = spec.split(":")
    if kind == "gemm":
        from embodied_efficiency_b200 import wq_linear
        from embodied_efficiency_b200.quant import quantize_weight
        from embodied_efficiency_b200.wq_gemm import _pack_int4
        m, k, bits = (int(v) for v in rest[:3])
        n = int(rest[3]) if len(rest) > 3 else k
        gelu = len(rest) > 4 and rest[4] == "gelu"
        g = torch.Generator(device="cpu").manual_seed(0)
        w = torch.randn(n, k, generator=g) * 0.02
        if bits == 16:
            wt, sc = w.bfloat16().to(dev), None
        else:
            q, s, _ = quantize_weight(w, bits, 128)
            q2 = q.reshape(n, k).to(dev)
            wt, sc = (_pack_int4(q2) if bits == 4 else q2), s.reshape(n, -1).to(dev)
        x = torch.randn(m, k, generator=g).bfloat16().to(dev)
        flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
        for _ in range(launches):
            flush.zero_()
            y = wq_linear(x, wt, sc, None, 128, bits, gelu=gelu)
        torch.cuda.synchronize()
        print(f"gemm m={m} k={k} n={n} bits={bits} gelu={gelu} mean|y|={float(y.float().abs().mean()):.5f}")
    elif kind == "sampler":
        from embodied_efficiency_b200 import GraphedSampler
        bits = int(rest[0]) if rest else 4
        m, x0, prefix = build_expert(bits, dev)
        x = x0.to(dev).bfloat16()
        gs = GraphedSampler(m, x, N_STEPS, warmup=1)
        for _ in range(launches):
            y = gs.run(x)
        torch.cuda.synchronize()
        if gs.status() != 0:
            raise RuntimeError(f"sampler status {gs.status()}")
        print(f"sampler bits={bits} mean|x|={float(y.float().abs().mean()):.5f}")
    elif kind == "norm":
        from embodied_efficiency_b200.expert import _apply_norm
        rows, cols = (int(v) for v in rest)
        g = torch.Generator(device="cpu").manual_seed(0)
        x = torch.randn(rows, cols, generator=g).bfloat16().to(dev)
        ln = torch.nn.LayerNorm(cols).to(dev).bfloat16()
        flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
        with torch.no_grad():
            for _ in range(launches):
                flush.zero_()
                y = _apply_norm(ln, x)
        torch.cuda.synchronize()
        print(f"norm rows={rows} cols={cols} mean|y|={float(y.float().abs().mean()):.5f}")
    elif kind == "attn":
        from embodied_efficiency_b200.expert import _attention
        b, p = (int(v) for v in rest)
        h, hd, n = 16, 64, 50
        d = h * hd
        g = torch.Generator(device="cpu").manual_seed(0)
        q = torch.randn(b, n, d, generator=g).bfloat16().to(dev)
        kv = torch.randn(b, p, 2 * d, generator=g).bfloat16().to(dev)
        flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
        for _ in range(launches):
            flush.zero_()
            y = _attention(q, d, kv, 2 * d, kv[..., d:], 2 * d, b, h, hd, n, p, n, p)
        torch.cuda.synchronize()
        print(f"attn batch={b} P={p} mean|y|={float(y.float().abs().mean()):.5f}")
    elif kind == "selfattn":
        from embodied_efficiency_b200.expert import _attention
        b = int(rest[0])
        h, hd, n = 16, 64, 50
        d = h * hd
        g = torch.Generator(device="cpu").manual_seed(0)
        qkv = torch.randn(b, n, 3 * d, generator=g).bfloat16().to(dev)
        flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
        for _ in range(launches):
            flush.zero_()
            y = _attention(qkv, 3 * d, qkv[..., d:], 3 * d, qkv[..., 2 * d:], 3 * d, b, h, hd, n, n, n, n)
        torch.cuda.synchronize()
        print(f"selfattn batch={b} mean|y|={float(y.float().abs().mean()):.5f}")
    elif kind == "dequant":
        from embodied_efficiency_b200.quant import quantize_weight
        from embodied_efficiency_b200.wq_gemm import _pack_int4, dequant_weight
        n, k, bits = (int(v) for v in rest)
        g = torch.Generator(device="cpu").manual_seed(0)
        q, s, _ = quantize_weight(torch.randn(n, k, generator=g) * 0.02, bits, 128)
        q2 = q.reshape(n, k).to(dev)
        wt, sc = (_pack_int4(q2) if bits == 4 else q2), s.reshape(n, -1).to(dev)
        flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
        for _ in range(launches):
            flush.zero_()
            y = dequant_weight(wt, sc, 128, bits, torch.bfloat16)
        torch.cuda.synchronize()
        print(f"dequant n={n} k={k} bits={bits} mean|w|={float(y.float().abs().mean()):.6f}")
    elif kind == "fleet":
        from embodied_efficiency_b200 import synth
        from embodied_efficiency_b200.fleet import FleetSampler
        world = int(rest[0]) if rest else 8
        m, x0, prefix = build_expert(4, dev)
        fs = FleetSampler(256, 0, world, chunk=256, expert=m, device=dev)
        fs.stage(lambda i: synth.fleet_request(m.cfg, i))
        for _ in range(2 + launches):
            fs.run_device()
        torch.cuda.synchronize()
        print(f"fleet world={world} requests={fs.hi - fs.lo}")
    else:
        raise SystemExit(f"unknown --profile case {spec!r}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-fleet", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the config 3-ref and config 5 sampler lines")
    ap.add_argument("--fleet-chunk", type=int, default=256)
    ap.add_argument("--fleet-share", default=None,
                    help="comma-separated world sizes: time rank 0's fleet share for each on this GPU and print "
                         "the projected aggregate (one JSON line), nothing else")
    ap.add_argument("--profile", default=None,
                    help="gemm:M:K:BITS[:N[:gelu]], sampler:BITS, norm:ROWS:COLS, attn:BATCH:P, selfattn:BATCH or dequant:N:K:BITS -- a few launches for a profiler")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.profile:
        return profile_case(args.profile, max(args.steps if args.steps != 200 else 4, 1))
    if args.fleet_share:
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        m, _, _ = build_expert(4, dev)
        shares = [fleet_share_run(m, int(w), dev) for w in args.fleet_share.split(",")]
        print(json.dumps({"metric": "projected fleet actions/s (rank 0's share timed on one GPU)",
                          "workload": "256 requests x (10-step int4 group-128 sampler, d1024 L4, own prefix and noise)",
                          "shares": shares}))
        return
    if args.impl == "reference":
        return run_reference(args)

    rank, world, local = dist_setup("nccl")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from embodied_efficiency_b200 import GraphedSampler, flow_sample

    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    results = {}
    experts = {}
    for bits in (16, 8, 4):
        m, x0, prefix = build_expert(bits, dev)
        kv = m.encode(prefix.to(dev))
        x = x0.to(dev).bfloat16()
        plan = m.plan(1, kv)
        out = torch.empty_like(x)
        fn = lambda: plan.run(x, N_STEPS, out=out)  # noqa: E731
        results[bits] = time_calls(fn, 20, args.warmup, flush)
        experts[bits] = (m, x, kv, plan, out)

    m, x, kv, plan, out = experts[4]
    fn = lambda: plan.run(x, N_STEPS, out=out)  # noqa: E731
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        per_call = time_calls(fn, args.steps, args.warmup, flush)
    total_ms = sum(per_call)
    t_max = torch.tensor([total_ms], device=dev)
    if world > 1:
        torch.distributed.all_reduce(t_max, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.barrier()
    value = t_max.item() / args.steps  # one call's latency (max over the replicas)
    status = plan.status(N_STEPS)
    if status != 0:
        raise RuntimeError(f"sampler status {status}")

    # e2e: GraphedSampler.run with a pinned host input, result copied back to the host
    gs = GraphedSampler(m, x, N_STEPS)
    xh = x.cpu().pin_memory()
    yh = torch.empty_like(xh).pin_memory()

    def e2e_call():
        y = gs.run(xh)
        yh.copy_(y, non_blocking=True)

    e2e_ms = time_calls(e2e_call, args.steps, args.warmup, flush)
    e2e_total = torch.tensor([sum(e2e_ms)], device=dev)
    if world > 1:
        torch.distributed.all_reduce(e2e_total, op=torch.distributed.ReduceOp.MAX)
    e2e_value = e2e_total.item() / args.steps

    fleet = None if args.no_fleet else fleet_run(m, rank, world, dev, chunk=args.fleet_chunk)

    # every rank's GPU work is done; the other ranks leave before rank 0
    # times the CPU baseline, so no rank spins on the host cores meanwhile
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return

    hbm, peak_kind = peaks()
    wb, kvb = step_bytes(WORKLOAD, 4)
    kernel_ms = statistics.mean(per_call)
    achieved = wb * N_STEPS / (kernel_ms * 1e-3) / 1e9
    variants = {}
    for bits, ms in results.items():
        w_b, _ = step_bytes(WORKLOAD, bits)
        t = statistics.median(ms)
        variants["bf16" if bits == 16 else f"int{bits}"] = {
            "ms_per_call": round(t, 4), "weight_MB_per_step": round(w_b / 1e6, 2),
            "weight_GBps": round(w_b * N_STEPS / (t * 1e-3) / 1e9, 1)}
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": "ms", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(value, 4),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": "action-expert sampler d1024 L4 h16x64 mlp4096 P256 H50 A32, "
                               "batch 1, 10 Euler steps, int4 group-128",
                   "weights": "int4", "batch": 1, "n_steps": N_STEPS,
                   "parallelism": f"replicas x{world}",
                   "l2": f"flushed between calls ({L2_FLUSH_BYTES >> 20} MiB write)"},
        "e2e": {"value": round(e2e_value, 4), "unit": "ms", "h2d_bytes_per_step": xh.numel() * 2,
                "d2h_bytes_per_step": yh.numel() * 2,
                "path": "GraphedSampler.run(pinned host x) + copy of the result to pinned host"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": SAMPLER_DRAM_BYTES,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                                       "sampler_kernel launch of this workload",
                     "peak_kind": peak_kind,
                     "kernel": "sampler_kernel (one launch per call)",
                     "algorithmic_bytes_per_launch": wb * N_STEPS,
                     "kv_bytes_per_launch": kvb * N_STEPS},
        "variants": variants,
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    if fleet is not None:
        line["fleet"] = fleet
    if world == 1 and not args.no_sweep:
        line["gemm"] = gemm_sweep(dev)
        line["gemm_method"] = ("wq_linear back to back in one CUDA graph over weight copies totalling "
                               ">= 2x L2 (weights from HBM every launch); time per launch")
        line["kv_prefix_gemm"] = kv_prefix_gemm(dev, flush)
    if world == 1 and not args.no_extra:
        line["config3_ref"] = sampler_variants(CONFIG3_REF, dev, flush)
        line["config3_ref"]["workload"] = ("reference default expert d512 L6 h8x64 mlp2048 P256 H50 A32, "
                                           "batch 1, 10 steps, CUDA graph; L4 published 4.4709 / 5.9973 / "
                                           "12.3748 ms bf16 / int8 / int4 (space/app/pareto.py:34-36)")
        c5 = sampler_variants(CONFIG5, dev, flush, calls=10, warmup=3)
        for b in (8, 64):
            c5.update({f"{k}_B{b}": v for k, v in
                       sampler_variants(CONFIG5, dev, flush, bits_list=(4,), calls=5, warmup=2, batch=b).items()})
        c5["workload"] = "Pi0-scale expert d2048 L18 h16x128 mlp8192 P816 H50 A32, 10 steps, CUDA graph"
        line["config5"] = c5
    if not args.no_cpu_baseline:
        torch.set_num_threads(os.cpu_count() or 1)
        v, n = cpu_baseline_run()
        line["cpu_baseline"] = {"value": round(v, 2), "unit": "ms", "cores": torch.get_num_threads(),
                                "kind": "port",
                                "sample": f"{n} full sampler calls of the same workload (oracle "
                                          "restatement of the reference path, torch CPU, bf16)"}
    print(json.dumps(line))


if __name__ == "__main__":
    main()
