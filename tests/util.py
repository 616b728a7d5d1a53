"""Shared helpers for the parity tests (test infrastructure)."""
from __future__ import annotations

import numpy as np

TOL_PROB = 1e-6      # probabilities: absolute tolerance
TOL_BOUNDARY = 1e-6  # ids may differ only where r lies this close to a CDF boundary


def u24(rng, n):
    """uniforms on the 2^-24 grid (every such value is an exact reference rand_f32 output)."""
    return ((rng.integers(0, 2 ** 32, n, dtype=np.uint64) >> 8).astype(np.float64)
            * 2.0 ** -24).astype(np.float32)


def pack_mask(allow: np.ndarray) -> np.ndarray:
    rows, V = allow.shape
    W = (V + 31) // 32
    pad = np.zeros((rows, W * 32), dtype=bool)
    pad[:, :V] = allow
    bits = pad.reshape(rows, W, 32).astype(np.uint64) << np.arange(32, dtype=np.uint64)
    return bits.sum(-1).astype(np.uint32)


def csr(hist):
    off = np.zeros(len(hist) + 1, dtype=np.int64)
    for i, h in enumerate(hist):
        off[i + 1] = off[i] + len(h)
    ids = np.concatenate([np.asarray(h, dtype=np.int32) for h in hist]) if off[-1] else \
        np.zeros(1, dtype=np.int32)
    return ids, off


def ids_match(gpu_tok, ora, uniforms, row):
    """True if the GPU id equals the oracle id, or r lies within TOL_BOUNDARY of one of the
    oracle's CDF boundaries (the allowance for differently rounded probabilities)."""
    if gpu_tok == ora.token[row]:
        return True
    if ora.kept_cdf is None:
        return False
    n = int(ora.kept_n[row])
    cdf = ora.kept_cdf[row, :min(n, ora.kept_cdf.shape[1])].astype(np.float64)
    r = float(uniforms[row])
    return bool(np.any(np.abs(cdf - r) <= TOL_BOUNDARY))


def dense_probs(ora, row, vocab):
    out = np.zeros(vocab, dtype=np.float32)
    n = int(ora.kept_n[row])
    if n:
        out[ora.kept_idx[row, :n]] = ora.kept_prob[row, :n]
    return out


TOL_CUT = 5e-7  # a top-p prefix this close to the threshold is a knife-edge cut


def knife_edge_rescue(bad, gpu_tok, lg, params, u, mask=None, hist=None, flags=0):
    """Rows of `bad` whose GPU id is explained by a knife-edge index-order top-p cut.

    The reference cuts where (float)(double prefix of p) first reaches top_p
    (src/sampler.c:204-222), with p = expf(t) * (float)(1/sum).  The reference's own vector
    expf is up to 3 ulp from the scalar one, and the GPU's exponential differs from both by a
    few ulp, so the two sums can round (float)(1/sum) one ulp apart: every prefix then moves by
    up to ~1.2e-7 relative.  When the prefix at the cut lies that close to the threshold the cut
    legitimately moves by one entry, which renormalises the nucleus by ~p_cut and shifts the CDF
    near r ~ top_p by more than the 1e-6 draw tolerance.  A row is rescued only if (a) the
    prefix at the oracle's cut, or just before it, lies within TOL_CUT of the threshold, and
    (b) the GPU id is the oracle's draw (with the usual 1e-6 boundary tolerance) for the cut one
    entry earlier or later.  Returns the rows that stay unexplained."""
    import oracle as O

    if not bad or params.get("top_p", 1.0) >= 1.0 or 0 < params.get("top_k", 0) < lg.shape[1]:
        return bad
    rows = np.asarray(bad)
    sub = lambda a: None if a is None else a[rows]
    hsub = None if hist is None else [hist[i] for i in rows]
    usub = u[rows]
    base = O.sample_restated(lg[rows], params, usub, mask=sub(mask), hist=hsub, flags=flags, want_pen=True,
                             kept_cap=lg.shape[1], topk_cap=1)
    alts = [O.sample_restated(lg[rows], params, usub, mask=sub(mask), hist=hsub, flags=flags | f,
                              kept_cap=lg.shape[1], topk_cap=1) for f in (O.CUT_EARLIER, O.CUT_LATER)]
    tp = np.float32(params["top_p"])
    thr = (float(np.nextafter(tp, np.float32(0))) + float(tp)) / 2.0  # (float)x >= tp  <=>  x >= thr
    left = []
    for j, i in enumerate(rows):
        x = base.pen_logits[j].astype(np.float64)
        t = ((x - x.max()) * (1.0 / params.get("temperature", 1.0)))
        e = np.exp(t)
        pref = np.cumsum(e / e.sum())
        n = int(base.kept_n[j])
        near = abs(pref[n - 1] - thr) <= TOL_CUT or (n >= 2 and abs(pref[n - 2] - thr) <= TOL_CUT)
        ok = near and any(ids_match(int(gpu_tok[i]), a, usub, j) for a in alts)
        if not ok:
            left.append(int(i))
    return left
