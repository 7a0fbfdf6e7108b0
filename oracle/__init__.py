"""CPU oracle for the decode-step hot path (TEST INFRASTRUCTURE ONLY).

This package restates, in NumPy float64, the arithmetic of the reference's Metal decode
kernels (ios_kernels/kernels/unsloth__Llama-3.2-1B-Instruct/kernel_metal_f16_20261024-1620/
kernels.metal and main.swift) plus the extensions that BASELINE.json names (32-block int8/4-bit
weights, paged KV, ragged batches, tensor parallelism).  It is the checker, never the thing
measured or shipped: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import it.  The product path (the CUDA library) never calls into it.

Pinning: the reference's kernels are Metal and cannot run here, and its own tests hold no
op-level golden vectors.  The oracle is pinned instead against HF transformers' Llama modules,
the third-party implementation the reference itself treats as ground truth
(ios_kernels/benchmarking/reference.py:64-70), through fixtures under tests/golden/ made by
tests/golden/make_golden.py.
"""

from . import ops, step  # noqa: F401
