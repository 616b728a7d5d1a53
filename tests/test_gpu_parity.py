"""Parity of the CUDA sampler (through the C ABI) with the restated oracle, which is itself
pinned bit-for-bit to DiskLLM's compiled sampler.c (test_oracle_vs_reference.py).

Bars:
  * penalised / masked logits: bit-exact
  * top-k id lists: bit-exact
  * probabilities: within 1e-6 absolute
  * sampled ids: identical, except where the uniform lies within 1e-6 of a CDF boundary
"""
import zlib

import numpy as np
import pytest

import oracle as O
from util import TOL_PROB, csr, dense_probs, ids_match, pack_mask, u24

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def gpu_run(lg, params, u, mask=None, hist=None, flags=0, dtype="f32"):
    from diskllm_b200 import capi

    dev = "cuda"
    rows, V = lg.shape
    x = torch.from_numpy(lg).to(dev)
    if dtype == "bf16":
        x = x.to(torch.bfloat16)
    ut = torch.from_numpy(np.ascontiguousarray(u, np.float32)).to(dev)
    kw = {}
    if mask is not None:
        kw["mask"] = torch.from_numpy(mask.view(np.int32)).to(dev)
    if hist is not None:
        ids, off = csr(hist)
        kw["hist_ids"] = torch.from_numpy(ids).to(dev)
        kw["hist_off"] = torch.from_numpy(off).to(dev)
    probs = torch.full((rows, V), -1.0, device=dev)
    pen = torch.empty((rows, V), device=dev)
    status = torch.full((rows,), -1, dtype=torch.int32, device=dev)
    tk = None
    k = params.get("top_k", 0)
    if 0 < k < V:
        tk = torch.full((rows, k), -1, dtype=torch.int32, device=dev)
    tok = capi.sample_batch(x, ut, params, flags=flags, probs=probs, pen_logits=pen,
                            status=status, topk_ids=tk, **kw)
    torch.cuda.synchronize()
    return (tok.cpu().numpy(), probs.cpu().numpy(), pen.cpu().numpy(), status.cpu().numpy(),
            None if tk is None else tk.cpu().numpy())


def _any_allowed(mrow, V):
    bits = np.unpackbits(mrow.view(np.uint8), bitorder="little")[:V]
    return bits.any()


def check(lg, params, u, mask=None, hist=None, flags=0, dtype="f32", check_probs=True, stats=None):
    """GPU against the oracle on every row (see compare)."""
    out = gpu_run(lg, params, u, mask, hist, flags, dtype)
    return compare(lg, params, u, *out, mask=mask, hist=hist, flags=flags, dtype=dtype,
                   check_probs=check_probs, stats=stats)


def compare(lg, params, u, tok, probs, pen, status, tk, mask=None, hist=None, flags=0, dtype="f32",
            check_probs=True, stats=None):
    """GPU outputs against the oracle on every row.  A row the GPU flags ROW_TOPP_EDGE (its
    index-order top-p prefix lies within the reference's rounding reach of the threshold) is held
    to the same bars against the oracle as it stands or with its cut moved one entry earlier or
    later, whichever the GPU's id and probabilities follow; every other row against the oracle as
    it stands.  `stats` (a dict) accumulates rows, flagged rows and rows whose cut moved."""
    from diskllm_b200 import capi

    rows, V = lg.shape
    ref_lg = lg
    if dtype == "bf16":
        ref_lg = torch.from_numpy(lg).to(torch.bfloat16).float().numpy()
    k = params.get("top_k", 0)
    ora = O.sample_restated(ref_lg, params, u, mask=mask, hist=hist, flags=flags, want_pen=True,
                            kept_cap=V, topk_cap=k if 0 < k < V else 1)
    assert np.all((status & ~capi.ROW_TOPP_EDGE) == 0), status
    edge = (status & capi.ROW_TOPP_EDGE) != 0
    assert np.array_equal(pen.view(np.uint32), ora.pen_logits.view(np.uint32))
    variants = [ora]
    if edge.any():
        variants += [O.sample_restated(ref_lg, params, u, mask=mask, hist=hist, flags=flags | f, kept_cap=V,
                                       topk_cap=k if 0 < k < V else 1) for f in (O.CUT_EARLIER, O.CUT_LATER)]

    def probs_close(i, o):
        g, d = probs[i].astype(np.float64), dense_probs(o, i, V).astype(np.float64)
        if not np.array_equal(np.isnan(g), np.isnan(d)):
            return False, np.inf
        diff = np.abs(np.nan_to_num(g) - np.nan_to_num(d))
        return diff.max() <= TOL_PROB, diff.max()

    sampling = params.get("temperature", 1.0) != 0.0
    moved = 0
    for i in range(rows):
        cands = variants if edge[i] else variants[:1]
        skip_probs = (not check_probs or not sampling or ref_lg[i].max() == -np.inf
                      or (mask is not None and not _any_allowed(mask[i], V)))
        ok, worst = False, None
        for j, o in enumerate(cands):
            if not ids_match(int(tok[i]), o, u, i):
                continue
            if not skip_probs:
                good, d = probs_close(i, o)
                worst = d if worst is None else min(worst, d)
                if not good:
                    continue
            ok = True
            moved += j > 0
            break
        assert ok, (f"row {i} (edge flag {bool(edge[i])}): gpu id {tok[i]} oracle id {ora.token[i]}, "
                    f"closest probability distance {worst}")
    if stats is not None:
        stats["rows"] = stats.get("rows", 0) + rows
        stats["flagged"] = stats.get("flagged", 0) + int(edge.sum())
        stats["cut_moved"] = stats.get("cut_moved", 0) + moved
    if sampling and tk is not None:
        for i in range(rows):
            assert np.array_equal(tk[i], ora.topk_idx[i, :k]), i
    return tok, ora


PARAM_SETS = {
    "cfg1": dict(temperature=0.8, top_k=40, top_p=0.95, repetition=1.1),
    "cfg2": dict(temperature=0.7, top_k=50, top_p=0.9, repetition=1.1, frequency=0.3, presence=0.2),
    "cfg3": dict(temperature=1.0, top_k=0, top_p=0.95),
    "cfg4": dict(temperature=1.0, top_k=0, top_p=0.99, repetition=1.05),
    "cfg5": dict(temperature=0.9, top_k=64, top_p=0.9, repetition=1.1),
    "greedy": dict(temperature=0.0, repetition=1.3, presence=-0.5),
    "server": dict(temperature=0.7, top_k=40, top_p=0.9, min_p=0.05, repetition=1.1),
    "minp_only": dict(temperature=1.3, top_k=0, top_p=1.0, min_p=1e-5),
    "minp_topp": dict(temperature=0.8, top_k=0, top_p=0.7, min_p=2e-5),
    "plain": dict(temperature=1.0, top_k=0, top_p=1.0),
    "topp_tiny": dict(temperature=1.0, top_k=0, top_p=0.02),
    "topp_zero": dict(temperature=1.0, top_k=0, top_p=0.0),
    "k3": dict(temperature=0.5, top_k=3, top_p=1.0),
    "k_big": dict(temperature=1.1, top_k=700, top_p=0.97),
    "k_huge": dict(temperature=0.9, top_k=3000, top_p=0.95, min_p=1e-5),  # above the fused list
    "k_ge_V": dict(temperature=2.0, top_k=10 ** 7, top_p=0.5),
    "hot": dict(temperature=3.0, top_k=0, top_p=0.999, presence=0.4, frequency=0.1),
}


@pytest.mark.parametrize("V", [1000, 4099, 32000])
@pytest.mark.parametrize("name", list(PARAM_SETS))
@pytest.mark.parametrize("with_mask", [False, True])
def test_parity_random_rows(V, name, with_mask):
    p = PARAM_SETS[name]
    if p.get("top_k", 0) > V and name != "k_ge_V":
        pytest.skip("k > V")
    rng = np.random.default_rng(zlib.crc32(f"{V}-{name}-{with_mask}".encode()))
    rows = 12
    sigma = {1000: 2.5, 4099: 0.5, 32000: 3.0}[V]
    lg = (rng.standard_normal((rows, V)) * sigma).astype(np.float32)
    hist = [np.concatenate([rng.integers(0, V, 64), rng.integers(0, 20, 40), [-3, V + 7]])
            for _ in range(rows)]
    mask = None
    if with_mask:
        allow = rng.random((rows, V)) < 0.3
        allow[0, :] = False                # fully masked row
        allow[1, :] = False
        allow[1, V // 3] = True            # exactly one allowed id
        mask = pack_mask(allow)
    u = u24(rng, rows)
    tok, ora = check(lg, p, u, mask=mask, hist=hist)
    # a single allowed token is returned, except when top_p <= 0 cuts the index-order list
    # at its first entry (token 0), which is what the reference does too
    if with_mask and p.get("temperature", 1.0) != 0.0 and p.get("top_p", 1.0) > 0.0:
        assert tok[1] == V // 3


@pytest.mark.parametrize("V,name", [(5003, n) for n in ("cfg3", "cfg4", "plain", "server", "cfg1")] +
                         [(256000, n) for n in ("cfg4", "cfg3", "minp_topp", "cfg1")])
def test_parity_degenerate_rows(V, name):
    """all-equal rows (the largest linear fp32 drift: at V = 256000 far beyond the draw window,
    so the walk recomputes unslotted ranges), a dominant spike, a ramp, pairwise ties, very
    peaked and tiny values"""
    rng = np.random.default_rng(5)
    rows = [np.zeros(V, np.float32)]                                       # all ties (linear drift)
    r = np.full(V, -5.0, np.float32); r[300] = 40.0; rows.append(r)        # p ~ 1 spike
    rows.append(np.linspace(-3, 3, V).astype(np.float32))                  # ramp
    r = rng.standard_normal(V).astype(np.float32); r[1::2] = r[:-1:2]; rows.append(r)  # ties
    rows.append((rng.standard_normal(V) * 30).astype(np.float32))          # very peaked
    rows.append(np.full(V, 1e-30, np.float32))                              # tiny values
    lg = np.stack(rows)
    for seed in range(4 if V < 100000 else 2):
        u = u24(np.random.default_rng(seed), len(rows))
        check(lg, PARAM_SETS[name], u)


def test_parity_uniform_extremes():
    V = 2048
    rng = np.random.default_rng(9)
    lg = (rng.standard_normal((6, V)) * 0.5).astype(np.float32)
    u = np.array([0.0, 2.0 ** -24, 0.5, 1.0 - 2.0 ** -24, 0.999999, 0.25], np.float32)
    for name in ("cfg4", "plain", "cfg1", "minp_topp"):
        check(lg, PARAM_SETS[name], u)


@pytest.mark.parametrize("name", ["cfg5", "cfg3", "greedy"])
def test_parity_bf16(name):
    V = 32768
    rng = np.random.default_rng(21)
    lg = (rng.standard_normal((8, V)) * 2).astype(np.float32)
    hist = [rng.integers(0, V, 128) for _ in range(8)]
    allow = rng.random((8, V)) < 0.1
    u = u24(rng, 8)
    check(lg, PARAM_SETS[name], u, mask=pack_mask(allow), hist=hist, dtype="bf16")


def test_true_division_mode():
    from diskllm_b200 import capi

    V = 4000
    rng = np.random.default_rng(4)
    lg = (rng.standard_normal((6, V)) * 4).astype(np.float32)
    hist = [rng.integers(0, V, 300) for _ in range(6)]
    u = u24(rng, 6)
    p = dict(temperature=0.9, top_k=20, top_p=0.9, repetition=1.1, presence=0.3)
    tok, probs, pen, status, tk = gpu_run(lg, p, u, hist=hist, flags=capi.MODE_PEN_TRUE_DIV)
    ora = O.sample_restated(lg, p, u, hist=hist, want_pen=True, flags=O.PEN_TRUE_DIV)
    assert np.array_equal(pen.view(np.uint32), ora.pen_logits.view(np.uint32))


@pytest.mark.parametrize("cfg", [2, 3, 4])
def test_config_shaped_rows(cfg):
    """full vocabulary of the benchmark configurations on a few rows"""
    from diskllm_b200 import workloads as W

    w = W.CONFIGS[cfg](device="cuda", rows=8)
    lg = w.logits.float().cpu().numpy()
    mask = None if w.mask is None else w.mask.cpu().numpy().view(np.uint32)
    u = w.uniforms.cpu().numpy()
    check(lg, w.params, u, mask=mask, hist=W.hist_lists(w))


def test_full_config4_batch_properties():
    """config 4 at full size: deterministic, statuses clean, and a sample of rows against the
    oracle."""
    from diskllm_b200 import capi
    from diskllm_b200 import workloads as W

    w = W.config4(device="cuda")
    st = torch.full((w.rows,), -1, dtype=torch.int32, device="cuda")
    t1 = capi.sample_batch(w.logits, w.uniforms, w.params, hist_ids=w.hist_ids,
                           hist_off=w.hist_off, hist_max=w.hist_max, status=st)
    t2 = capi.sample_batch(w.logits, w.uniforms, w.params, hist_ids=w.hist_ids,
                           hist_off=w.hist_off, hist_max=w.hist_max)
    torch.cuda.synchronize()
    assert torch.equal(t1, t2)
    assert int((st & ~capi.ROW_TOPP_EDGE).abs().sum()) == 0
    sel = list(range(0, w.rows, 64))
    lg = w.logits[sel].cpu().numpy()
    hist = [W.hist_lists(w)[i] for i in sel]
    u = w.uniforms.cpu().numpy()[sel]
    ora = O.sample_restated(lg, w.params, u, hist=hist, kept_cap=w.vocab)
    tok = t1.cpu().numpy()[sel]
    for i in range(len(sel)):
        assert ids_match(int(tok[i]), ora, u, i), (sel[i], tok[i], ora.token[i])


def test_drop_in_sampler_matches_reference_stream():
    """sampler_create / sampler_sample through the C ABI against the oracle driven by the same
    xorshift64 stream (seeded like src/sampler.c:83-89)."""
    from diskllm_b200 import capi

    rng = np.random.default_rng(12)
    V = 20000
    s = capi.Sampler(temperature=0.8, top_k=40, top_p=0.95, seed=1234)
    us = O.xorshift_uniforms(1234, 20)
    for i in range(20):
        row = (rng.standard_normal(V) * 2.5).astype(np.float32)
        tok = s.sample(row)
        ora = O.sample_restated(row[None], dict(temperature=0.8, top_k=40, top_p=0.95),
                                us[i:i + 1], kept_cap=40)
        assert ids_match(tok, ora, us[i:i + 1], 0)
    g = capi.Sampler(temperature=0.0, seed=5)      # greedy does not advance the stream
    st0 = g.rng_state
    row = rng.standard_normal(V).astype(np.float32)
    assert g.sample(row) == int(np.argmax(row))
    assert g.rng_state == st0
    assert capi.greedy_sample(row) == int(np.argmax(row))


def test_drop_in_penalties_in_place():
    from diskllm_b200 import capi

    rng = np.random.default_rng(13)
    V = 5000
    row = (rng.standard_normal(V) * 3).astype(np.float32)
    seen = np.concatenate([rng.integers(0, V, 200), [-1, V, V + 5], rng.integers(0, 10, 50)])
    a = row.copy()
    capi.apply_presence_penalty(a, seen, 0.25)
    capi.apply_repetition_penalty(a, seen, 1.15)
    ora = O.sample_restated(row[None], dict(temperature=0.0, presence=0.25, repetition=1.15),
                            np.zeros(1, np.float32), hist=[seen], want_pen=True)
    assert np.array_equal(a.view(np.uint32), ora.pen_logits[0].view(np.uint32))


def test_parity_config4_shape_256_rows():
    """config 4's shape (vocab 256000, flat N(0, 0.5^2), top-p 0.99, repetition 1.05 over 256
    uniform ids) on 256 rows: enough rows that about one has a knife-edge top-p cut (accepted
    only as util.knife_edge_rescue describes)"""
    rng = np.random.default_rng(44)
    rows, V = 256, 256000
    lg = (rng.standard_normal((rows, V)) * 0.5).astype(np.float32)
    hist = [rng.integers(0, V, 256) for _ in range(rows)]
    u = u24(rng, rows)
    stats = {}
    check(lg, PARAM_SETS["cfg4"], u, hist=hist, stats=stats)
    print(f"config-4 shape, 256 rows: {stats}")


def _full_batch(cfg):
    """one launch over a whole benchmark batch, every output on"""
    from diskllm_b200 import capi
    from diskllm_b200 import workloads as W

    w = W.CONFIGS[cfg](device="cuda")
    V = w.vocab
    probs = torch.full((w.rows, V), -1.0, device="cuda")
    pen = torch.empty((w.rows, V), device="cuda")
    status = torch.full((w.rows,), -1, dtype=torch.int32, device="cuda")
    k = w.params.get("top_k", 0)
    tk = torch.full((w.rows, k), -1, dtype=torch.int32, device="cuda") if 0 < k < V else None
    kw = dict(probs=probs, pen_logits=pen, status=status, topk_ids=tk)
    if w.hist_ids is not None:
        kw.update(hist_ids=w.hist_ids, hist_off=w.hist_off, hist_max=w.hist_max)
    if w.mask is not None:
        kw["mask"] = w.mask
    tok = capi.sample_batch(w.logits, w.uniforms, w.params, **kw)
    torch.cuda.synchronize()
    out = dict(tok=tok.cpu().numpy(), probs=probs.cpu().numpy(), pen=pen.cpu().numpy(),
               status=status.cpu().numpy(), tk=None if tk is None else tk.cpu().numpy())
    del probs, pen
    return w, out


@pytest.mark.parametrize("cfg", [2, 3, 4])
def test_every_row_of_benchmark_batch(cfg):
    """configs 2, 3 and 4 at full size (64 x 151936, 256 x 151936 with its JSON mask, 1024 x
    256000): every row against the oracle, probabilities included, in blocks of rows"""
    from diskllm_b200 import workloads as W

    w, out = _full_batch(cfg)
    lg = w.logits.float().cpu().numpy()
    w.logits = None
    torch.cuda.empty_cache()
    mask = None if w.mask is None else w.mask.cpu().numpy().view(np.uint32)
    hist = W.hist_lists(w)
    u = w.uniforms.cpu().numpy()
    stats = {}
    blk = 128
    for r0 in range(0, w.rows, blk):
        sl = slice(r0, min(w.rows, r0 + blk))
        sub = lambda a: None if a is None else a[sl]
        compare(lg[sl], w.params, u[sl], out["tok"][sl], out["probs"][sl], out["pen"][sl], out["status"][sl],
                sub(out["tk"]), mask=sub(mask), hist=None if hist is None else hist[sl], stats=stats)
    if cfg == 3:
        for r in w.notes["single_allowed_rows"]:
            bits = np.unpackbits(mask[r].view(np.uint8), bitorder="little")[:w.vocab]
            assert out["tok"][r] == int(np.nonzero(bits)[0][0]), r
    print(f"config {cfg} full batch: {stats}")


@pytest.mark.parametrize("k", [0, 40, 2000])
def test_nonfinite_rows_follow_the_reference(k):
    """+inf logits (one or several, or alone among -inf), all-NaN rows and NaN rows with top-k
    off: the reference's sums turn NaN and its draw returns its list's last entry (the oracle is
    pinned to that on CPU)"""
    from diskllm_b200 import capi

    rng = np.random.default_rng(33)
    rows, V = 6, 6000
    lg = (rng.standard_normal((rows, V))).astype(np.float32)
    lg[0, 17] = np.inf
    lg[1, [5, 4000]] = np.inf
    lg[2, 123] = np.nan
    lg[3, :] = -np.inf
    lg[3, 9] = np.inf
    lg[5, :] = np.nan
    u = u24(rng, rows)
    p = dict(temperature=0.8, top_k=k, top_p=0.9)
    tok, _, _, st, _ = gpu_run(lg, p, u)
    ora = O.sample_restated(lg, p, u)
    for i in range(rows):
        if i == 2 and k:
            # a NaN among top-k candidates: the reference's insertion-sort order of NaNs is not
            # defined by its -ffast-math build; the row is flagged instead
            assert st[i] & capi.ROW_ERR_NONFINITE, st
            continue
        assert tok[i] == ora.token[i], (i, tok[i], ora.token[i])
        assert st[i] & ~capi.ROW_TOPP_EDGE == 0, (i, st[i])


def test_per_row_top_k_above_and_below_the_fused_list():
    """per-row parameters mixing top-k off, small k, and k above the fused kernel's list
    capacity (those rows take the large-k pass after the fused kernel)"""
    from diskllm_b200 import capi

    rng = np.random.default_rng(31)
    rows, V = 8, 9000
    lg = (rng.standard_normal((rows, V)) * 1.5).astype(np.float32)
    hist = [rng.integers(0, V, 50) for _ in range(rows)]
    u = u24(rng, rows)
    ks = [3, 1500, 0, 40, 5000, 8999, 1025, 0]
    per_row = [dict(temperature=0.8 + 0.05 * i, top_k=k, top_p=0.93, repetition=1.1) for i, k in enumerate(ks)]
    dev = "cuda"
    ids, off = csr(hist)
    st = torch.full((rows,), -1, dtype=torch.int32, device=dev)
    probs = torch.full((rows, V), -1.0, device=dev)
    tok = capi.sample_batch(torch.from_numpy(lg).to(dev), torch.from_numpy(u).to(dev), per_row[0],
                            row_params=capi.params_array(per_row, dev), topk_max=max(ks),
                            hist_ids=torch.from_numpy(ids).to(dev), hist_off=torch.from_numpy(off).to(dev),
                            status=st, probs=probs)
    torch.cuda.synchronize()
    tok, st, probs = tok.cpu().numpy(), st.cpu().numpy(), probs.cpu().numpy()
    assert np.all((st & ~capi.ROW_TOPP_EDGE) == 0), st
    for i in range(rows):
        ora = O.sample_restated(lg[i:i + 1], per_row[i], u[i:i + 1], hist=[hist[i]], kept_cap=V)
        assert ids_match(int(tok[i]), ora, u[i:i + 1], 0), (i, ks[i], tok[i], ora.token[0])
        if ks[i] > 0:
            d = np.abs(probs[i].astype(np.float64) - dense_probs(ora, 0, V))
            assert d.max() <= TOL_PROB, (i, d.max())


def test_drop_in_sampler_with_top_k_above_the_fused_list():
    """the reference accepts any 0 < top_k < vocab (src/sampler.c:165-170); so does the drop-in"""
    from diskllm_b200 import capi

    rng = np.random.default_rng(32)
    V = 20000
    s = capi.Sampler(temperature=0.9, top_k=4000, top_p=0.9, seed=77)
    us = O.xorshift_uniforms(77, 4)
    for i in range(4):
        row = (rng.standard_normal(V) * 1.2).astype(np.float32)
        tok = s.sample(row)
        ora = O.sample_restated(row[None], dict(temperature=0.9, top_k=4000, top_p=0.9), us[i:i + 1], kept_cap=V)
        assert ids_match(tok, ora, us[i:i + 1], 0)
