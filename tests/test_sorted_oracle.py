"""The sorted-nucleus mode and the relative min-p mode of the CPU restatement (modes that are not
the reference's; the GPU is checked against them).  The restatement is compared with a separate
numpy statement of the same definition, and with the known-answer probe that shows the
reference's index-order top-p: 1000 tokens, all logits 0 except id 999 = 10 (p ~ 0.96),
top-p 0.02 -- the reference never returns 999 with top-k off, the sorted mode always does."""
from __future__ import annotations

import ctypes as C
import ctypes.util
import math

import numpy as np
import pytest

import oracle as O
from util import u24

_libm = C.CDLL(ctypes.util.find_library("m"))
_libm.expf.restype = C.c_float
_libm.expf.argtypes = [C.c_float]


def _sorted_numpy(x, p, r, relative=False):
    """the definition, step by step, in numpy / Python integers"""
    x = np.asarray(x, np.float32)
    m = x.max()
    inv_temp = np.float32(1.0) / np.float32(p.get("temperature", 1.0))
    t = ((x - m).astype(np.float32) * inv_temp).astype(np.float32)
    order = np.lexsort((np.arange(len(x)), -t.astype(np.float64)))
    e = np.array([_libm.expf(float(v)) for v in t[order]], np.float32)
    E = [int(np.rint(float(v) * 2.0 ** 42)) for v in e]
    npos = max(i + 1 for i, v in enumerate(E) if v > 0)
    nk = npos
    if p.get("min_p", 0.0) > 0:
        inv_sum = np.float32(1.0 / (sum(E) * 2.0 ** -42))
        thr = np.float32(p["min_p"]) * inv_sum if relative else np.float32(p["min_p"])
        n = 0
        while n < npos and np.float32(e[n] * inv_sum) >= thr:
            n += 1
        nk = n or nk
    s2 = sum(E[:nk])
    kc, s3 = nk, s2
    if p.get("top_p", 1.0) < 1.0:
        T = max(math.ceil(float(np.float32(p["top_p"])) * float(s2)), 1) - 1
        cum = 0
        for i in range(nk):
            cum += E[i]
            if cum > T:
                kc = i + 1
                break
        s3 = sum(E[:kc])
    T = math.floor(float(r) * float(s3))
    cum = 0
    for i in range(kc):
        cum += E[i]
        if cum > T:
            return int(order[i])
    return int(order[kc - 1])


@pytest.mark.parametrize("params", [
    dict(temperature=1.0, top_p=0.9),
    dict(temperature=0.7, top_p=0.99, min_p=0.0005),
    dict(temperature=1.3, top_p=1.0),
    dict(temperature=1.0, top_p=0.5, min_p=0.05),
])
def test_sorted_mode_matches_numpy_definition(params):
    rng = np.random.default_rng(11)
    rows, V = 6, 3000
    x = (rng.standard_normal((rows, V)) * 2.0).astype(np.float32)
    x[1, :50] = x[1, 0]          # ties
    x[2] = np.round(x[2])        # many ties
    u = u24(rng, rows)
    ora = O.sample_restated(x, params, u, flags=O.TOPP_SORTED, kept_cap=V)
    for r in range(rows):
        assert ora.token[r] == _sorted_numpy(x[r], params, u[r]), r
        n = int(ora.kept_n[r])
        assert abs(float(ora.kept_cdf[r, n - 1]) - 1.0) < 1e-6
        assert np.all(np.diff(ora.kept_cdf[r, :n]) >= 0)


def test_relative_min_p_matches_numpy_definition():
    rng = np.random.default_rng(12)
    rows, V = 4, 2000
    x = (rng.standard_normal((rows, V)) * 3.0).astype(np.float32)
    u = u24(rng, rows)
    params = dict(temperature=1.0, top_p=0.95, min_p=0.02)
    ora = O.sample_restated(x, params, u, flags=O.TOPP_SORTED | O.MINP_RELATIVE, kept_cap=V)
    for r in range(rows):
        assert ora.token[r] == _sorted_numpy(x[r], params, u[r], relative=True)
    # relative min-p in the reference mode keeps p >= min_p * p_max
    ref = O.sample_restated(x, dict(temperature=1.0, min_p=0.5), u, flags=O.MINP_RELATIVE, kept_cap=V)
    for r in range(rows):
        n = int(ref.kept_n[r])
        p = ref.kept_prob[r, :n]
        assert n >= 1 and p.max() > 0


def test_index_order_probe_and_sorted_mode():
    V = 1000
    x = np.zeros((200, V), np.float32)
    x[:, 999] = 10.0
    rng = np.random.default_rng(1)
    u = u24(rng, 200)
    params = dict(temperature=1.0, top_p=0.02)
    ref = O.sample_restated(x, params, u)
    assert not np.any(ref.token == 999) and ref.token.max() <= 460
    srt = O.sample_restated(x, params, u, flags=O.TOPP_SORTED)
    assert np.all(srt.token == 999)
    if O.have_reference():
        asb, _ = O.sample_reference(x, params, u)
        np.testing.assert_array_equal(asb.token, ref.token)
