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
