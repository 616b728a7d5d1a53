"""Builds libdiskllm_cuda.so in-tree (diskllm_b200/libdiskllm_cuda.so) with nvcc for sm_100a.

    python -m diskllm_b200.build [--force]

The library is self-contained (static CUDA runtime) so plain C callers can link it.  The
kernels are compiled once per sub-chunk length, in parallel.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libdiskllm_cuda.so")

SUB_LENGTHS = [4, 12, 20, 28, 36, 44, 52, 60]
UNITS = [("dllm_launch.cu", []), ("dllm_capi.cu", []), ("dllm_noalloc.cu", []), ("dllm_shard.cu", []), ("dllm_grammar.cu", []), ("dllm_lmhead.cu", []), ("dllm_sorted.cu", []), ("dllm_largek.cu", [])] + [
    ("dllm_kernel_inst.cu", [f"-DDLLM_SUB={s}"]) for s in SUB_LENGTHS
]
SOURCES = sorted({u[0] for u in UNITS})
HEADERS = ["dllm_internal.h", "dllm_kernel.cuh", "dllm_chunk.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    # bit-exact penalised logits: no contraction into FMA; FTZ like the reference build
    "-fmad=false", "-ftz=true", "-prec-div=true", "-prec-sqrt=true",
    "-Xcompiler", "-fPIC,-O2,-fvisibility=hidden",
    "-cudart=static",
]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, s) for s in SOURCES + HEADERS]
    deps += [os.path.join(ROOT, "include", h) for h in ("diskllm_cuda.h", "sampler.h", "grammar.h")]
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    nvcc = _nvcc()
    tmp = os.path.join(HERE, "_build")
    os.makedirs(tmp, exist_ok=True)
    jobs = []
    for src, defs in UNITS:
        tag = "".join(d.split("=")[-1] for d in defs)
        o = os.path.join(tmp, src.replace(".cu", f"{tag}.o"))
        cmd = [nvcc, *NVCC_FLAGS, *defs, "-I", os.path.join(ROOT, "include"), "-I", CSRC,
               "-c", os.path.join(CSRC, src), "-o", o]
        jobs.append((cmd, o))
    if verbose:
        for cmd, _ in jobs:
            print(" ".join(cmd))
    with ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
        for f in [ex.submit(subprocess.run, cmd, check=True) for cmd, _ in jobs]:
            f.result()
    out_tmp = LIB + ".tmp"
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart=static",
           *[o for _, o in jobs], "-o", out_tmp, "-lpthread"]
    subprocess.run(cmd, check=True)
    os.replace(out_tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
