"""Run the reference's own scripts on this package.

The reference's scripts (``kernel/bench.py``, ``kernel/compiler.py``,
``kernel/measure_table.py``, ``kernel/sweep.py``, ``kernel/cudagraph.py`` ...)
import their hot-path modules by bare name: ``flow_expert``, ``triton_gemm``,
``cudagraph`` and ``quant``. ``install()`` registers this package's modules
under those names, so a reference script then runs unmodified on the sm_100a
kernels:

    python -m embodied_efficiency_b200.dropin path/to/kernel/compiler.py
    python -m embodied_efficiency_b200.dropin path/to/kernel/bench.py --quant int4 --graph

The script's own directory stays on ``sys.path`` for its other imports;
the registered names take precedence over same-named files there.
"""
from __future__ import annotations

import importlib
import os
import runpy
import sys

# reference module name -> this package's module with the same surface
ALIASES = {
    "flow_expert": "embodied_efficiency_b200.expert",   # kernel/flow_expert.py
    "triton_gemm": "embodied_efficiency_b200.wq_gemm",  # kernel/triton_gemm.py
    "cudagraph": "embodied_efficiency_b200.graphed",    # kernel/cudagraph.py
    "quant": "embodied_efficiency_b200.quant",          # kernel/quant.py
}

# names the reference's scripts import from each module
EXPECTED = {
    "flow_expert": ("ActionExpertConfig", "ActionExpert", "flow_sample", "timestep_embedding", "Block"),
    "triton_gemm": ("quantize_model_triton", "TritonQuantLinear", "wq_linear", "_pack_int4", "_unpack_int4"),
    "cudagraph": ("GraphedSampler",),
    "quant": ("quantize_weight", "dequantize_weight", "QuantLinear", "quantize_model"),
}


def install() -> dict:
    """Register the aliases in ``sys.modules``; returns {alias: module}."""
    mods = {}
    for alias, target in ALIASES.items():
        mod = importlib.import_module(target)
        sys.modules[alias] = mod
        mods[alias] = mod
    return mods


def run(script: str, argv=()) -> dict:
    """Run ``script`` as ``__main__`` with ``argv`` after ``install()``."""
    install()
    script = os.path.abspath(script)
    sys.path.insert(0, os.path.dirname(script))
    old_argv = sys.argv
    sys.argv = [script, *argv]
    try:
        return runpy.run_path(script, run_name="__main__")
    finally:
        sys.argv = old_argv


if __name__ == "__main__":
    if len(sys.argv) < 2:
        raise SystemExit("usage: python -m embodied_efficiency_b200.dropin SCRIPT [ARGS...]")
    run(sys.argv[1], sys.argv[2:])
