"""Deploy-compiler search on the B200 sampler.

The reference's deploy compiler (kernel/compiler.py:97-154) searches the
efficiency levers of a flow-matching sampler and scores every configuration on
four axes -- latency per executed action, weight footprint, action fidelity
and staleness -- then keeps the Pareto frontier and picks the best
configuration under a budget; kernel/measure_table.py:35-61 runs that search
over several model widths and tags every row with the GPU it ran on. This
module is that search on this package's kernels (the fused sampler, its CUDA
graph, the int8 / int4 dequant-GEMM), with the reference's levers, row schema
and Pareto / budget rules:

* precision  bf16 / int8 / int4 (``quantize_model_triton`` of a deep copy);
* steps      max_steps, max_steps // 2, max_steps // 4 (at least 2);
* graph      the call captured as a CUDA graph (``GraphedSampler.run``) or
             dispatched directly (``flow_sample``);
* exec_horizon  1, horizon // 4, horizon actions executed per call:
             ms_per_action = call_ms / k, staleness = k - 1;
* speculative  a draft of the fewest steps proposes the chunk, the full-step
             sampler verifies it; expected latency = draft + (1 - accept) * full
             with the accept rate measured against the full-step output
             (relative rMSE below ``accept_tol``).

Fidelity is the reference's action error: rMSE against the bf16, full-step
output divided by its mean absolute value (kernel/quant.py:104-105).
Latency is wall time per call around ``iters`` back-to-back calls with a
device synchronisation on both sides, as the reference measures it
(kernel/compiler.py:72-88).

Run on a GPU:  python -m embodied_efficiency_b200.deploy --sizes 256,512,1024,2048 --out rows.json
"""
from __future__ import annotations

import argparse
import copy
import json
import re
import time

import torch
import torch.nn as nn

OBJECTIVES = ("ms_per_action", "weight_mb", "rmse", "staleness")


def weight_mb(model) -> float:
    """Stored weight bytes in MB (kernel/compiler.py:58-69): dense linears'
    weight and bias, quantised linears' packed weight, scales and bias."""
    tot = 0
    for m in model.modules():
        if isinstance(m, nn.Linear):
            tot += m.weight.numel() * m.weight.element_size()
            if m.bias is not None:
                tot += m.bias.numel() * m.bias.element_size()
        elif type(m).__name__ == "TritonQuantLinear":
            tot += m.weight.numel() * m.weight.element_size() + m.scales.numel() * m.scales.element_size()
            if m.bias is not None:
                tot += m.bias.numel() * m.bias.element_size()
    return tot / 1e6


def call_ms(model, x, steps: int, graph: bool, iters: int) -> float:
    """Wall time of one sampler call (a whole action chunk) in ms."""
    from .expert import flow_sample
    from .graphed import GraphedSampler
    if graph:
        gs = GraphedSampler(model, x, steps)
        fn = lambda: gs.run(x)  # noqa: E731
    else:
        pkv = model.encode_prefix(x.shape[0])
        fn = lambda: flow_sample(model, x, steps, pkv)  # noqa: E731
    for _ in range(max(2, iters // 4)):
        fn()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(iters):
        fn()
    torch.cuda.synchronize()
    return (time.perf_counter() - t0) / iters * 1e3


def make_row(precision, steps, graph, exec_h, ms, mb, rmse, mode) -> dict:
    """One configuration in the reference's row schema (kernel/compiler.py:91-94)."""
    return {"precision": precision, "steps": steps, "graph": graph, "exec_horizon": exec_h,
            "mode": mode, "call_ms": round(ms, 4), "ms_per_action": round(ms / exec_h, 4),
            "weight_mb": round(mb, 2), "rmse": round(rmse, 4), "staleness": exec_h - 1}


def _rel_rmse(out, ref, scale) -> float:
    return (out.float() - ref).pow(2).mean().sqrt().item() / scale


def search(d_model: int = 512, batch: int = 1, max_steps: int = 10, accept_tol: float = 0.05,
           iters: int = 20, seed: int = 0, cfg=None) -> dict:
    """The lever search for one expert width (default-initialised
    ``ActionExpert`` drawn after ``torch.manual_seed(seed)``, bf16, CUDA)."""
    from .expert import ActionExpert, ActionExpertConfig, flow_sample
    from .wq_gemm import quantize_model_triton
    dev = "cuda"
    cfg = cfg or ActionExpertConfig()
    cfg.d_model = d_model
    horizon = cfg.horizon
    torch.manual_seed(seed)
    base = ActionExpert(cfg).to(dev).to(torch.bfloat16).eval()
    x = torch.randn(batch, horizon, cfg.action_dim, device=dev, dtype=torch.bfloat16)
    ref = flow_sample(base, x, max_steps, base.encode_prefix(batch)).float()
    rscale = ref.abs().mean().item() + 1e-9

    steps_opts = sorted({max_steps, max(2, max_steps // 2), max(2, max_steps // 4)}, reverse=True)
    exec_opts = sorted({1, max(1, horizon // 4), horizon})
    models = {"bf16": base,
              "int8": quantize_model_triton(copy.deepcopy(base), bits=8),
              "int4": quantize_model_triton(copy.deepcopy(base), bits=4)}
    rows = []
    for precision, m in models.items():
        mb = weight_mb(m)
        for s in steps_opts:
            rmse = _rel_rmse(flow_sample(m, x, s, m.encode_prefix(batch)), ref, rscale)
            for graph in (True, False):
                ms = call_ms(m, x, s, graph, iters)
                for k in exec_opts:
                    rows.append(make_row(precision, s, graph, k, ms, mb, rmse, "plain"))

    # speculative draft / verify on the bf16 expert (kernel/compiler.py:130-151)
    draft_steps, full_steps = min(steps_opts), max_steps
    draft_ms = call_ms(base, x, draft_steps, True, iters)
    full_ms = call_ms(base, x, full_steps, True, iters)
    pkv = base.encode_prefix(batch)
    trials, accepts = 6, 0
    for _ in range(trials):
        xi = torch.randn_like(x)
        d = flow_sample(base, xi, draft_steps, pkv).float()
        f = flow_sample(base, xi, full_steps, pkv).float()
        if (d - f).pow(2).mean().sqrt().item() / (f.abs().mean().item() + 1e-9) < accept_tol:
            accepts += 1
    accept = accepts / trials
    rmse_full = _rel_rmse(flow_sample(base, x, full_steps, pkv), ref, rscale)
    for k in exec_opts:
        rows.append(make_row("bf16", full_steps, True, k, draft_ms + (1 - accept) * full_ms, weight_mb(base),
                             rmse_full, f"spec(draft={draft_steps},accept={accept:.2f})"))
    return {"device": "cuda", "base_dtype": "bfloat16", "d_model": d_model, "batch": batch,
            "horizon": horizon, "latency_real": True, "rows": rows}


def _dominates(a: dict, b: dict, objs) -> bool:
    return all(a[o] <= b[o] for o in objs) and any(a[o] < b[o] for o in objs)


def pareto(rows, objs=OBJECTIVES):
    """Rows no other row beats on every objective (kernel/compiler.py:157-162)."""
    return [r for r in rows if not any(_dominates(o, r, objs) for o in rows if o is not r)]


def pick_config(rows, budget: dict):
    """Best row under a budget (max_ms_per_action, max_weight_mb, max_rmse,
    max_staleness) by ``budget["objective"]`` (default ms_per_action); None
    when nothing fits (kernel/compiler.py:165-172)."""
    obj = budget.get("objective", "ms_per_action")
    feas = [r for r in rows
            if r["ms_per_action"] <= budget.get("max_ms_per_action", float("inf"))
            and r["weight_mb"] <= budget.get("max_weight_mb", float("inf"))
            and r["rmse"] <= budget.get("max_rmse", float("inf"))
            and r["staleness"] <= budget.get("max_staleness", float("inf"))]
    return min(feas, key=lambda r: r[obj]) if feas else None


def gpu_slug() -> str:
    name = torch.cuda.get_device_name(0) if torch.cuda.is_available() else "cpu"
    return re.sub(r"[^a-z0-9]+", "-", name.lower()).strip("-")


def measure_table(sizes=(256, 512, 1024, 2048), max_steps: int = 10, iters: int = 20) -> dict:
    """The search over several widths, every row tagged with the GPU
    (kernel/measure_table.py:35-61 schema)."""
    dev_name = torch.cuda.get_device_name(0)
    rows = []
    for d in sizes:
        res = search(d_model=d, max_steps=max_steps, iters=iters)
        for r in res["rows"]:
            rows.append({"gpu": dev_name, "d_model": d, "latency_real": res["latency_real"], **r})
    return {"gpu": dev_name, "gpu_slug": gpu_slug(), "sizes": list(sizes), "latency_real": True, "rows": rows}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--sizes", default="256,512,1024,2048")
    ap.add_argument("--max-steps", type=int, default=10)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--out", default=None, help="JSON file for the rows (default <gpu-slug>.json)")
    args = ap.parse_args()
    sizes = [int(s) for s in args.sizes.split(",") if s.strip()]
    table = measure_table(sizes, args.max_steps, args.iters)
    out = args.out or f"{table['gpu_slug']}.json"
    with open(out, "w") as f:
        json.dump(table, f, indent=2)
    for d in sizes:
        rows = [r for r in table["rows"] if r["d_model"] == d]
        best = min((r for r in rows if r["mode"] == "plain"), key=lambda r: r["ms_per_action"])
        fast = pick_config(rows, {"objective": "ms_per_action", "max_rmse": 0.05, "max_staleness": 0})
        print(f"d_model={d}: {len(rows)} configs; fastest plain {best['precision']} {best['steps']} steps "
              f"graph={best['graph']} exec={best['exec_horizon']} -> {best['ms_per_action']} ms/action; "
              f"fastest at rMSE<=0.05, no staleness: {fast and (fast['precision'], fast['steps'], fast['call_ms'])}")
    print(f"wrote {out} ({len(table['rows'])} rows)")


if __name__ == "__main__":
    main()
