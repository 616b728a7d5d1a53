"""The restated oracle against golden outputs of DiskLLM's own sampler (tests/golden/
sampler_golden.json, written by tests/golden/make_golden.py from the reference compiled from its
sources).  These pin the oracle without the reference sources: tokens for eight injected
uniforms per row, penalised logits bit for bit (by digest) and the reference's fp32 CDF
boundaries.  The GPU check runs the CUDA path on the same rows."""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np
import pytest

import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_golden as G  # noqa: E402

with open(os.path.join(HERE, "golden", "sampler_golden.json")) as f:
    GOLD = json.load(f)
CASES = {c["name"]: c for c in GOLD["cases"]}


def _inputs(c):
    lg, mask, hist, u = G.case_inputs(c["seed"], c["rows"], c["vocab"], c["sigma"], c["mask"], c["history"])
    assert G.inputs_digest(lg, mask, hist, u) == c["inputs_sha256"], "input generator changed"
    return lg, mask, hist, u


@pytest.mark.parametrize("name", list(CASES))
def test_oracle_reproduces_reference_tokens_and_penalties(name):
    c = CASES[name]
    lg, mask, hist, u = _inputs(c)
    want = np.array(c["tokens"])
    for j in range(u.shape[1]):
        res = O.sample_restated(lg, c["params"], u[:, j].copy(), mask=mask, hist=hist, want_pen=(j == 0))
        np.testing.assert_array_equal(res.token, want[:, j], err_msg=f"{name} uniform column {j}")
        if j == 0:
            assert hashlib.sha256(res.pen_logits.tobytes()).hexdigest() == c["pen_logits_sha256"]


@pytest.mark.parametrize("name", [n for n, c in CASES.items() if "cdf_ids" in c])
def test_oracle_reproduces_reference_cdf(name):
    c = CASES[name]
    lg, mask, hist, _ = _inputs(c)
    r = c["cdf_row"]
    o = O.sample_restated(lg[r:r + 1], c["params"], np.zeros(1, np.float32),
                          mask=None if mask is None else mask[r:r + 1], hist=[hist[r]], kept_cap=c["vocab"])
    n = int(o.kept_n[0])
    oid, ocdf, opr = o.kept_idx[0, :n], o.kept_cdf[0, :n], o.kept_prob[0, :n]
    # positions that no uniform can reach (zero probability, or a running sum that did not move)
    keep = (opr > 0) & np.concatenate([[True], np.diff(ocdf.astype(np.float64)) > 0])
    oid, ocdf = oid[keep], ocdf[keep]
    ids, bits = c["cdf_ids"], c["cdf_bits"]
    m = min(len(ids), len(oid))
    assert m >= 2
    np.testing.assert_array_equal(np.array(ids[:m]), oid[:m])
    for i in range(m - 1):
        if bits[i] is not None:
            assert int(ocdf[i].view(np.uint32)) == bits[i], f"{name} boundary {i}"


@pytest.mark.parametrize("name", [n for n, c in CASES.items() if "around_id" in c])
def test_oracle_reproduces_reference_cdf_at_full_vocabulary(name):
    """at the benchmark vocabularies (up to 262144 entries of sequential fp32 drift) the oracle's
    running sum equals the reference's on both boundaries around the drawn entry, bit for bit"""
    c = CASES[name]
    lg, mask, hist, u = _inputs(c)
    r = c["around_row"]
    o = O.sample_restated(lg[r:r + 1], c["params"], u[r:r + 1, 0].copy(),
                          mask=None if mask is None else mask[r:r + 1], hist=[hist[r]], kept_cap=c["vocab"])
    assert int(o.token[0]) == c["around_id"]
    n = int(o.kept_n[0])
    ids = o.kept_idx[0, :n]
    j = int(np.nonzero(ids == c["around_id"])[0][0])
    lo_bits, hi_bits = c["around_bits"]
    assert int(o.kept_cdf[0, j].view(np.uint32)) == hi_bits
    if j > 0:
        # the reference's lowest uniform drawing this id is the running sum before its entry
        assert int(o.kept_cdf[0, j - 1].view(np.uint32)) == lo_bits


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(CASES))
def test_cuda_path_on_golden_rows(name):
    import torch

    from diskllm_b200 import capi
    from util import ids_match

    c = CASES[name]
    lg, mask, hist, u = _inputs(c)
    want = np.array(c["tokens"])
    dev = torch.device("cuda", 0)
    from util import csr
    hid, hoff = (torch.from_numpy(a).to(dev) for a in csr(hist))
    kw = dict(hist_ids=hid, hist_off=hoff)
    if mask is not None:
        kw["mask"] = torch.from_numpy(mask.view(np.int32)).to(dev)
    x = torch.from_numpy(lg).to(dev)
    for j in range(u.shape[1]):
        uj = u[:, j].copy()
        tok = capi.sample_batch(x, torch.from_numpy(uj).to(dev), c["params"], **kw).cpu().numpy()
        ora = O.sample_restated(lg, c["params"], uj, mask=mask, hist=hist, kept_cap=c["vocab"])
        np.testing.assert_array_equal(ora.token, want[:, j])
        for r in range(c["rows"]):
            assert ids_match(int(tok[r]), ora, uj, r), f"{name} row {r} uniform {j}: {tok[r]} vs {want[r, j]}"
