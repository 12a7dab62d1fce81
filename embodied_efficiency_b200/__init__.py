"""embodied_efficiency_b200 -- B200 (sm_100a) weight-only dequant-GEMM and fused
flow-matching sampler, with the reference's Python operator surface.

Modules (reference counterpart in brackets):
  quant      quantize_weight, dequantize_weight, byte counters   [kernel/quant.py]
  wq_gemm    _pack_int4, _unpack_int4, wq_linear, TritonQuantLinear,
             quantize_model_triton, correctness_check            [kernel/triton_gemm.py]
  expert     ActionExpertConfig, Block, ActionExpert, timestep_embedding,
             flow_sample, sample                                 [kernel/flow_expert.py]
  graphed    GraphedSampler, eval_all                            [kernel/cudagraph.py]
  fused      plan of the single-launch sampler (ee_flow_sample)
  fleet      batch-of-robots mode over several GPUs
  dropin     runs the reference's scripts on top of this package
The compute lives in lib/libee_b200.so (C ABI: include/ee_b200.h).
"""
from .quant import dequantize_weight, quantize_weight, quantize_weight_asym4
from .wq_gemm import (TritonQuantLinear, _pack_int4, _unpack_int4, correctness_check,
                      quantize_model_triton, wq_linear)
from .expert import ActionExpert, ActionExpertConfig, Block, flow_sample, sample, timestep_embedding
from .graphed import GraphedSampler

__all__ = ["quantize_weight", "dequantize_weight", "quantize_weight_asym4", "TritonQuantLinear",
           "_pack_int4", "_unpack_int4", "wq_linear", "quantize_model_triton", "correctness_check",
           "ActionExpert", "ActionExpertConfig", "Block", "flow_sample", "sample",
           "timestep_embedding", "GraphedSampler"]
