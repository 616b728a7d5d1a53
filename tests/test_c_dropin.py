"""The drop-in at the C level: C programs written against DiskLLM's own headers, linked against
libdiskllm_cuda.so in place of src/sampler.c and src/core/grammar.c.

  * the reference's tools/test_grammar_unit.c, unchanged, linked with libdiskllm_cuda.so
    (oracle/_ref/test_grammar_unit_cuda);
  * tests/c/dropin_driver.c with the reference's unchanged src/core/sampler_api.c, built once
    with the reference's sampler.c + grammar.c (oracle/_ref/dropin_ref) and once with
    libdiskllm_cuda.so (oracle/_ref/dropin_cuda): decode loops with top-k, index-order top-p,
    the JSON grammar, top-k above the fused kernel's list and greedy; the sampled ids must agree.

oracle/Makefile builds the binaries where the reference sources are; they travel prebuilt.
"""
from __future__ import annotations

import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "oracle", "_ref")


def _bin(name):
    p = os.path.join(REF_DIR, name)
    if not os.path.exists(p):
        pytest.skip(f"{p} not built (make -C oracle ref where the reference sources are)")
    return p


def test_reference_grammar_unit_test_against_the_library():
    res = subprocess.run([_bin("test_grammar_unit_cuda")], capture_output=True, text=True, timeout=60)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "PASSED" in res.stdout


def test_driver_links_the_library_not_the_reference_sampler():
    res = subprocess.run(["ldd", _bin("dropin_cuda")], capture_output=True, text=True, timeout=60)
    assert "libdiskllm_cuda.so" in res.stdout and "not found" not in res.stdout, res.stdout
    syms = subprocess.run(["nm", "--defined-only", _bin("dropin_cuda")], capture_output=True, text=True)
    assert " sampler_sample" not in syms.stdout


@pytest.mark.gpu
def test_sampler_api_decode_loops_match_the_reference():
    ref = subprocess.run([_bin("dropin_ref")], capture_output=True, text=True, timeout=300)
    cud = subprocess.run([_bin("dropin_cuda")], capture_output=True, text=True, timeout=300)
    assert ref.returncode == 0 and cud.returncode == 0, cud.stderr[-2000:]
    a, b = ref.stdout.splitlines(), cud.stdout.splitlines()
    assert len(a) == len(b) == 98
    diff = [(x, y) for x, y in zip(a, b) if x != y]
    assert not diff, diff[:5]
