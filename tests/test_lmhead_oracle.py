"""The LM-head tail's CPU restatement (oracle.lmhead_restated) pinned to the reference: the
final norm against src/rmsnorm.c compiled from the reference sources
(oracle/_ref/librmsnorm_asbuilt.so), with and without the weight, with the Gemma (w + 1) form.
src/matvec.c cannot be built here (it includes vulkan/vulkan.h), so the matvec restatement is
checked against an exact rational-free bound instead: the double dot product rounded once."""
from __future__ import annotations

import os

import numpy as np
import pytest

import oracle as O


def _have_rmsnorm():
    return os.path.exists(O.RMSNORM_SO)


@pytest.mark.parametrize("hidden,weighted,add_one", [(4096, True, False), (2304, True, True), (1000, False, False),
                                                     (8, True, False)])
def test_rmsnorm_restatement_matches_reference(hidden, weighted, add_one):
    if not _have_rmsnorm():
        pytest.skip("oracle/_ref/librmsnorm_asbuilt.so not built (reference sources unavailable)")
    rng = np.random.default_rng(hidden + add_one)
    x = (rng.standard_normal((6, hidden)) * rng.uniform(0.01, 30.0, (6, 1))).astype(np.float32)
    x[0, : hidden // 3] = 0.0
    w = (rng.standard_normal(hidden) * 0.3).astype(np.float32) if weighted else None
    ref = O.rmsnorm_reference(x, w, 1e-6, add_one)
    ours = O.rmsnorm_restated(x, w, 1e-6, add_one)
    np.testing.assert_array_equal(ours, ref)


def test_lmhead_restatement_is_the_rounded_double_dot_product():
    rng = np.random.default_rng(3)
    hidden, vocab = 512, 300
    h = rng.standard_normal((2, hidden)).astype(np.float32)
    w = (rng.standard_normal((vocab, hidden)) * 0.05).astype(np.float32)
    out = O.lmhead_restated(h, w)
    hn = O.rmsnorm_restated(h, None, 1e-6, False).astype(np.float64)
    for r in range(2):
        for v in (0, 7, 299):
            exact = sum(float(w[v, i]) * float(hn[r, i]) for i in range(hidden))
            assert abs(float(out[r, v]) - exact) <= abs(exact) * 2.0 ** -23 + 1e-30
    capped = O.lmhead_restated(h, w, softcap=30.0)
    assert np.all(np.abs(capped) < 30.0)
    np.testing.assert_allclose(capped, 30.0 * np.tanh(out / 30.0), rtol=1e-6, atol=1e-6)
