"""Generates tests/golden/sampler_golden.json from DiskLLM's own sampler, compiled from the
reference sources by oracle/Makefile (oracle/_ref/libref_asbuilt.so: src/sampler.c and
src/core/grammar.c at the reference's Makefile:10 flags).

Every case is rebuilt from its seed by `case_inputs` (numpy PCG64 streams); the file stores a
SHA-256 of the inputs so that a generator change is caught instead of silently comparing other
rows.  Stored outputs, all from the reference:
  * tokens for eight injected uniforms per row (the harness seeds the reference's xorshift so
    that rand_f32 returns the wanted value);
  * SHA-256 of the penalised, masked logits (mask -> presence -> repetition, bit for bit);
  * for the small rows, the first fp32 CDF boundaries recovered by bisection on the uniform;
  * for the full-vocabulary rows, the two CDF boundaries that enclose row 1's first uniform.

    python tests/golden/make_golden.py      # needs oracle/_ref (make -C oracle ref)
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

CASES = [
    # name, seed, rows, V, sigma, mask, history length, params
    ("cfg1_like", 101, 4, 4099, 2.5, False, 64, dict(temperature=0.8, top_k=40, top_p=0.95, repetition=1.1)),
    ("cfg2_like", 102, 4, 3000, 3.0, False, 96, dict(temperature=0.7, top_k=50, top_p=0.9, repetition=1.1,
                                                      presence=0.2)),
    ("cfg3_like_mask", 103, 4, 4099, 2.0, True, 0, dict(temperature=1.0, top_k=0, top_p=0.95)),
    ("cfg4_like", 104, 4, 4096, 0.5, False, 256, dict(temperature=1.0, top_k=0, top_p=0.99, repetition=1.05)),
    ("cfg5_like_mask", 105, 4, 4096, 2.0, True, 128, dict(temperature=0.9, top_k=64, top_p=0.9, repetition=1.1)),
    ("greedy_negative_presence", 106, 4, 1000, 1.0, False, 32, dict(temperature=0.0, repetition=1.3,
                                                                     presence=-0.5)),
    ("min_p_server", 107, 4, 2048, 2.0, False, 16, dict(temperature=0.7, top_k=40, top_p=0.9, min_p=0.05)),
    ("min_p_only", 108, 4, 1500, 1.5, False, 0, dict(temperature=1.3, top_k=0, top_p=1.0, min_p=1e-4)),
    ("top_p_tiny", 109, 4, 700, 2.0, False, 0, dict(temperature=1.0, top_k=0, top_p=0.02)),
    ("top_k_3", 110, 4, 300, 2.0, False, 8, dict(temperature=0.5, top_k=3, top_p=1.0)),
    ("top_k_ge_V", 111, 4, 257, 2.0, True, 8, dict(temperature=2.0, top_k=999999, top_p=0.5)),
    ("tiny_vocab", 112, 4, 5, 2.0, False, 3, dict(temperature=1.0, top_k=0, top_p=0.9)),
    # the benchmark configurations' full vocabularies, where the
    # reference's sequential fp32 running sum drifts furthest from the exact prefix
    ("cfg1_V128256", 121, 2, 128256, 2.5, False, 64, dict(temperature=0.8, top_k=40, top_p=0.95, repetition=1.1)),
    ("cfg2_V151936", 122, 2, 151936, 3.0, False, 512, dict(temperature=0.7, top_k=50, top_p=0.9, repetition=1.1,
                                                            presence=0.2)),
    ("cfg3_V151936_mask", 123, 2, 151936, 2.0, 0.02, 0, dict(temperature=1.0, top_k=0, top_p=0.95)),
    ("cfg4_V256000", 124, 2, 256000, 0.5, False, 256, dict(temperature=1.0, top_k=0, top_p=0.99, repetition=1.05)),
    ("cfg5_V262144_mask", 125, 2, 262144, 2.0, 0.10, 128, dict(temperature=0.9, top_k=64, top_p=0.9,
                                                                 repetition=1.1)),
]
UNIFORMS_PER_ROW = 8
CDF_BOUNDARIES = 24


def case_inputs(seed, rows, V, sigma, with_mask, hlen):
    """(logits, mask or None, history lists, uniforms [rows][UNIFORMS_PER_ROW]) of one case.
    with_mask: False, True (30 % of ids allowed) or the allowed fraction."""
    rng = np.random.default_rng(seed)
    lg = (rng.standard_normal((rows, V)) * sigma).astype(np.float32)
    lg[0, V // 3] = lg[0].max()  # a tie for the maximum in the first row
    mask = None
    if with_mask:
        allow = rng.random((rows, V)) < (0.3 if with_mask is True else float(with_mask))
        allow[:, 0] = True
        W = (V + 31) // 32
        pad = np.zeros((rows, W * 32), dtype=bool)
        pad[:, :V] = allow
        mask = (pad.reshape(rows, W, 32).astype(np.uint64) << np.arange(32, dtype=np.uint64)).sum(-1)
        mask = mask.astype(np.uint32)
    hist = [np.concatenate([rng.integers(0, V, hlen), [-3, V + 7]]).astype(np.int32) if hlen else
            np.zeros(0, dtype=np.int32) for _ in range(rows)]
    u = ((rng.integers(0, 2 ** 32, (rows, UNIFORMS_PER_ROW), dtype=np.uint64) >> 8).astype(np.float64)
         * 2.0 ** -24).astype(np.float32)
    return lg, mask, hist, u


def inputs_digest(lg, mask, hist, u) -> str:
    h = hashlib.sha256()
    h.update(lg.tobytes())
    if mask is not None:
        h.update(mask.tobytes())
    for x in hist:
        h.update(np.asarray(x, dtype=np.int32).tobytes())
        h.update(b"|")
    h.update(u.tobytes())
    return h.hexdigest()


def main():
    import oracle as O

    if not O.have_reference():
        raise SystemExit("oracle/_ref is not built: run `make -C oracle ref` where the reference sources are")
    out = {"generator": "tests/golden/make_golden.py", "reference": "src/sampler.c + src/core/grammar.c, "
           "Makefile:10 flags (oracle/_ref/libref_asbuilt.so)", "uniforms_per_row": UNIFORMS_PER_ROW,
           "cases": []}
    for name, seed, rows, V, sigma, with_mask, hlen, params in CASES:
        lg, mask, hist, u = case_inputs(seed, rows, V, sigma, with_mask, hlen)
        tokens = np.zeros((rows, UNIFORMS_PER_ROW), dtype=np.int64)
        pen = None
        for j in range(UNIFORMS_PER_ROW):
            res, _ = O.sample_reference(lg, params, u[:, j].copy(), mask=mask, hist=hist, want_pen=(j == 0),
                                        threads=1)
            tokens[:, j] = res.token
            if j == 0:
                pen = res.pen_logits
        case = {"name": name, "seed": seed, "rows": rows, "vocab": V, "sigma": sigma, "mask": with_mask,
                "history": hlen, "params": params, "inputs_sha256": inputs_digest(lg, mask, hist, u),
                "tokens": tokens.tolist(), "pen_logits_sha256": hashlib.sha256(pen.tobytes()).hexdigest()}
        if V >= 100000 and params.get("temperature", 1.0) > 0:
            # the reference's CDF boundaries on both sides of row 1's first uniform
            lo, hi, tid = O.reference_cdf_around(lg[1], params, float(u[1, 0]), None if mask is None else mask[1],
                                                 hist[1])
            case["around_row"] = 1
            case["around_id"] = tid
            case["around_bits"] = [int(np.float32(lo).view(np.uint32)), int(np.float32(hi).view(np.uint32))]
        if V <= 1500 and params.get("temperature", 1.0) > 0:
            ids, cdf = O.reference_cdf(lg[1], params, None if mask is None else mask[1], hist[1],
                                       n_boundaries=CDF_BOUNDARIES)
            case["cdf_row"] = 1
            case["cdf_ids"] = ids.tolist()
            case["cdf_bits"] = [int(np.float32(c).view(np.uint32)) if np.isfinite(c) else None for c in cdf]
        out["cases"].append(case)
    with open(os.path.join(HERE, "sampler_golden.json"), "w") as f:
        json.dump(out, f, indent=1)
    print(f"wrote {len(out['cases'])} cases")


if __name__ == "__main__":
    main()
