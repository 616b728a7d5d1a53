"""Sorted-nucleus mode (DLLM_MODE_TOPP_SORTED) and relative min-p (DLLM_MODE_MINP_RELATIVE) on
the GPU against the CPU restatement's definition of the same modes (dllm_oracle.c,
sample_row_sorted; checked against a numpy statement in test_sorted_oracle.py).

Bars as for the reference mode: penalised logits bit-exact, probabilities within 1e-6, ids
identical except where r lies within 1e-6 of a CDF boundary.  The cases reach every path of the
radix descent: collected candidates, refinement histograms, and keys shared by more entries
than the candidate list holds (per-chunk counts, then an ordered scan)."""
from __future__ import annotations

import zlib

import numpy as np
import pytest
import torch

import oracle as O
from diskllm_b200 import capi
from test_gpu_parity import check
from util import ids_match, pack_mask, u24

pytestmark = pytest.mark.gpu

S = O.TOPP_SORTED

PARAMS = {
    "cfg3": dict(temperature=1.0, top_p=0.95),
    "cfg4": dict(temperature=1.0, top_p=0.99, repetition=1.05),
    "cold": dict(temperature=0.6, top_p=0.9, presence=0.3, frequency=0.1),
    "plain": dict(temperature=1.0, top_p=1.0),
    "minp": dict(temperature=0.8, top_p=0.7, min_p=2e-5),
    "minp_only": dict(temperature=1.3, top_p=1.0, min_p=1e-5),
    "topp_tiny": dict(temperature=1.0, top_p=0.02),
    "topp_zero": dict(temperature=1.0, top_p=0.0),
}


def _hist(rng, rows, V):
    return [np.concatenate([rng.integers(0, V, 64), rng.integers(0, 20, 40), [-3, V + 7]]) for _ in range(rows)]


@pytest.mark.parametrize("V", [1000, 32000, 128256])
@pytest.mark.parametrize("name", list(PARAMS))
def test_sorted_random_rows(V, name):
    rng = np.random.default_rng(zlib.crc32(f"s-{V}-{name}".encode()))
    rows = 8
    lg = (rng.standard_normal((rows, V)) * rng.choice([0.5, 2.0, 4.0], (rows, 1))).astype(np.float32)
    u = u24(rng, rows)
    check(lg, PARAMS[name], u, hist=_hist(rng, rows, V), flags=S)


def test_sorted_with_mask_and_bf16():
    rng = np.random.default_rng(3)
    rows, V = 6, 50000
    lg = (rng.standard_normal((rows, V)) * 2.0).astype(np.float32)
    allow = rng.random((rows, V)) < 0.3
    allow[5] = False  # fully masked row
    u = u24(rng, rows)
    check(lg, PARAMS["cfg4"], u, mask=pack_mask(allow), hist=_hist(rng, rows, V), flags=S)
    check(lg, PARAMS["cold"], u, hist=_hist(rng, rows, V), flags=S, dtype="bf16")


@pytest.mark.parametrize("kind", ["flat", "integers", "two_levels", "peaked"])
def test_sorted_ties_beyond_candidate_capacity(kind):
    """keys held by more entries than the collected list holds (32768)"""
    rng = np.random.default_rng(zlib.crc32(kind.encode()))
    rows, V = 4, 256000
    if kind == "flat":
        lg = np.zeros((rows, V), np.float32)
    elif kind == "integers":
        lg = rng.integers(-3, 4, (rows, V)).astype(np.float32)
    elif kind == "two_levels":
        lg = np.where(rng.random((rows, V)) < 0.5, 1.0, 1.0 - 2.0 ** -20).astype(np.float32)
    else:
        lg = np.zeros((rows, V), np.float32)
        lg[:, rng.integers(0, V, 5)] = 9.0
    u = u24(rng, rows)
    for params in (PARAMS["cfg3"], PARAMS["plain"], PARAMS["minp"]):
        check(lg, params, u, flags=S)


def test_sorted_config4_rows():
    """config 4's shape (vocab 256000, top-p 0.99, repetition 1.05, 256-id history), 48 rows"""
    rng = np.random.default_rng(44)
    rows, V = 48, 256000
    lg = (rng.standard_normal((rows, V)) * rng.uniform(0.5, 4.0, (rows, 1))).astype(np.float32)
    hist = [rng.integers(0, V, 256) for _ in range(rows)]
    u = u24(rng, rows)
    check(lg, PARAMS["cfg4"], u, hist=hist, flags=S)


def test_sorted_known_answer_probe():
    """1000 tokens, logits 0 except id 999 = 10, top-p 0.02: the reference never returns 999
    (index-order prefix); the sorted mode always does"""
    V, rows = 1000, 64
    lg = np.zeros((rows, V), np.float32)
    lg[:, 999] = 10.0
    u = u24(np.random.default_rng(1), rows)
    dev = torch.device("cuda", 0)
    x = torch.from_numpy(lg).to(dev)
    ut = torch.from_numpy(u).to(dev)
    srt = capi.sample_batch(x, ut, dict(temperature=1.0, top_p=0.02), flags=S).cpu().numpy()
    ref = capi.sample_batch(x, ut, dict(temperature=1.0, top_p=0.02)).cpu().numpy()
    assert np.all(srt == 999)
    assert not np.any(ref == 999)


@pytest.mark.parametrize("sorted_mode", [False, True])
def test_relative_min_p(sorted_mode):
    rng = np.random.default_rng(9)
    rows, V = 8, 32000
    lg = (rng.standard_normal((rows, V)) * 3.0).astype(np.float32)
    u = u24(rng, rows)
    flags = O.MINP_RELATIVE | (S if sorted_mode else 0)
    check(lg, dict(temperature=1.0, top_p=0.95, min_p=0.05), u, flags=flags)
    check(lg, dict(temperature=0.7, top_k=50, top_p=0.9, min_p=0.1), u, flags=flags)


def _row_params(lst):
    arr = (capi.SamplerParams * len(lst))()
    for i, d in enumerate(lst):
        arr[i] = capi.make_params(**d)
    raw = np.frombuffer(bytes(arr), dtype=np.uint8).copy()
    return torch.from_numpy(raw).cuda()


def test_sorted_per_row_params_mixes_modes():
    """per-row parameters: rows with top-k, greedy rows and sorted rows in one batch"""
    rng = np.random.default_rng(21)
    V = 20000
    plist = [PARAMS["cfg3"], dict(temperature=0.8, top_k=40, top_p=0.95), dict(temperature=0.0),
             PARAMS["minp"], dict(temperature=1.2, top_k=V + 5, top_p=0.8), PARAMS["plain"]]
    rows = len(plist)
    lg = (rng.standard_normal((rows, V)) * 2.5).astype(np.float32)
    u = u24(rng, rows)
    dev = torch.device("cuda", 0)
    status = torch.full((rows,), -1, dtype=torch.int32, device=dev)
    tok = capi.sample_batch(torch.from_numpy(lg).to(dev), torch.from_numpy(u).to(dev), None,
                            row_params=_row_params(plist), topk_max=40, flags=S, status=status)
    tok = tok.cpu().numpy()
    assert np.all(status.cpu().numpy() == 0)
    ora = O.sample_restated(lg, plist, u, flags=S, kept_cap=V)
    for i in range(rows):
        assert ids_match(int(tok[i]), ora, u, i), (i, tok[i], ora.token[i])


def test_sorted_workspace_and_static_entry():
    rng = np.random.default_rng(5)
    rows, V = 3, 40000
    lg = torch.from_numpy((rng.standard_normal((rows, V)) * 2).astype(np.float32)).cuda()
    u = torch.from_numpy(u24(rng, rows)).cuda()
    p = PARAMS["cfg3"]
    nb = capi.workspace_bytes(lg, u, p, flags=S)
    assert nb > 0
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    a = capi.sample_batch(lg, u, p, flags=S, workspace=ws).cpu().numpy()
    b = capi.sample_batch(lg, u, p, flags=S).cpu().numpy()
    c, rc = capi.sample_batch_static(lg, u, p, flags=S)
    np.testing.assert_array_equal(a, b)
    assert rc == 0
    np.testing.assert_array_equal(c.cpu().numpy(), a)
