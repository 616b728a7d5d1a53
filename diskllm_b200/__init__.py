"""diskllm_b200 -- DiskLLM's sampler hot path (sampler.c + the grammar logit mask) for B200.

The compute runs in libdiskllm_cuda.so (hand-written sm_100a kernels behind a C ABI, see
include/diskllm_cuda.h and include/sampler.h).  This package is the Python host side:
`capi` binds the C ABI (drop-in sampler API + batched device entry point), `workloads`
generates the seeded benchmark inputs, `build` compiles the library in-tree.
"""
from . import capi  # noqa: F401
from .capi import (  # noqa: F401
    DllmError,
    Sampler,
    apply_presence_penalty,
    apply_repetition_penalty,
    greedy_sample,
    load_library,
    make_params,
    sample_batch,
    version,
)

__all__ = [
    "capi", "DllmError", "Sampler", "apply_presence_penalty", "apply_repetition_penalty",
    "greedy_sample", "load_library", "make_params", "sample_batch", "version",
]
