"""CPU oracle for the weight-only dequant-GEMM and flow-matching sampler path.

TEST INFRASTRUCTURE ONLY. Nothing in the shipped package imports this
directory: only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
legs of ``bench.py`` may use it, and only as the checker / the timed CPU
baseline, never as the thing measured on the GPU.

Contents
--------
``quant``    numpy restatement of the reference's integer work: symmetric
             group quantisation, int4 packing and unpacking, dequantisation
             and fp32 -> bf16 round-to-nearest-even (reference
             ``kernel/quant.py`` and ``kernel/triton_gemm.py``), plus the
             asymmetric int4 variant, which has no reference code.
``sampler``  torch-CPU restatement of the reference's action expert, its
             dequantise-then-matmul ``QuantLinear`` forward and the Euler
             ``flow_sample`` loop (reference ``kernel/flow_expert.py``,
             ``kernel/quant.py``).

Parity pinning: ``tests/golden/make_golden.py`` imports the reference in a
container where it is mounted and writes the fixtures under ``tests/golden``;
``tests/test_oracle.py`` checks this oracle against every one of them and
against the reference's published fidelity figures.
"""
