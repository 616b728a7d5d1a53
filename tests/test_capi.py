"""The C-ABI library loads and exports every entry point its public headers declare; argument
validation runs without touching a GPU."""
import ctypes as C
import os
import re

from diskllm_b200 import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for h in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not h.endswith(".h"):
            continue
        src = open(os.path.join(ROOT, "include", h)).read()
        for m in re.finditer(r"DLLM_API\s+[\w\s\*]+?\b(\w+)\s*\(", src):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol():
    lib = capi.load_library()
    declared = _declared()
    assert declared == set(capi.EXPORTS)
    for name in declared:
        assert hasattr(lib, name), name


def test_version_string():
    assert "sm_100a" in capi.version()


def test_invalid_arguments_rejected_without_gpu():
    lib = capi.load_library()
    assert lib.dllm_cuda_sample_batch(None, None) == 1
    d = capi.BatchDesc()
    d.rows, d.vocab = -1, 10
    assert lib.dllm_cuda_sample_batch(C.byref(d), None) == 1
    d.rows, d.vocab, d.row_stride = 2, 10, 10
    assert lib.dllm_cuda_sample_batch(C.byref(d), None) == 1   # null pointers
    d.logits = d.uniforms = d.token = 16
    d.row_stride = 5                                          # stride < vocab
    assert lib.dllm_cuda_sample_batch(C.byref(d), None) == 1
    d.row_stride = 10
    d.dtype = 7
    assert lib.dllm_cuda_sample_batch(C.byref(d), None) == 1
    d.dtype = 0
    d.flags = 0x8                                             # unknown mode bit
    assert lib.dllm_cuda_sample_batch(C.byref(d), None) == 6
    d.flags = capi.MODE_TOPP_SORTED                           # sorted mode beyond 2^21 ids
    d.vocab = d.row_stride = (1 << 21) + 1
    assert lib.dllm_cuda_sample_batch(C.byref(d), None) == 6
    d.vocab = d.row_stride = 10
    d.flags = 0
    d.rows = 0                                                # empty batch: no launch
    assert lib.dllm_cuda_sample_batch(C.byref(d), None) == 0


def test_struct_layouts_match_headers():
    assert C.sizeof(capi.SamplerParams) == 28
    assert C.sizeof(capi.SamplerConfig) == 24
