"""ctypes front end for the parity checkers (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs import
this module.  The product (diskllm_b200 + libdiskllm_cuda.so) never does.

Two checkers, same call shape:
  * ``restated``  -- oracle/libdllm_oracle.so, this repo's C restatement of DiskLLM's
                     sampler chain (src/sampler.c:9-234, src/core/sampler_api.c:48-63,
                     grammar mask src/core/grammar.c:275-308) with injectable uniforms,
                     the frequency-penalty and sorted-nucleus extensions and internals
                     (penalised row, top-k list, final probabilities and fp32 CDF).
  * ``reference`` -- oracle/_ref/libref_asbuilt.so, DiskLLM's own src/sampler.c compiled
                     with its Makefile:10 flags, driven row by row by oracle/ref_harness.c.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
RESTATED_SO = os.path.join(HERE, "libdllm_oracle.so")
REF_ASBUILT_SO = os.path.join(HERE, "_ref", "libref_asbuilt.so")
REF_STRICT_SO = os.path.join(HERE, "_ref", "libref_strict.so")

TOPP_SORTED = 0x1
MINP_RELATIVE = 0x4
PEN_TRUE_DIV = 0x2
CUT_EARLIER = 0x200  # oracle only: index-order top-p cut one entry earlier
CUT_LATER = 0x400    # oracle only: index-order top-p cut one entry later


class Params(C.Structure):
    _fields_ = [
        ("temperature", C.c_float),
        ("top_p", C.c_float),
        ("min_p", C.c_float),
        ("top_k", C.c_int),
        ("repetition", C.c_float),
        ("presence", C.c_float),
        ("frequency", C.c_float),
    ]


class _OracleBatch(C.Structure):
    _fields_ = [
        ("rows", C.c_int),
        ("vocab", C.c_int),
        ("logits", C.c_void_p),
        ("mask", C.c_void_p),
        ("hist_ids", C.c_void_p),
        ("hist_off", C.c_void_p),
        ("uniforms", C.c_void_p),
        ("params", C.c_void_p),
        ("params_per_row", C.c_int),
        ("flags", C.c_uint),
        ("token", C.c_void_p),
        ("pen_logits", C.c_void_p),
        ("kept_n", C.c_void_p),
        ("kept_idx", C.c_void_p),
        ("kept_prob", C.c_void_p),
        ("kept_cdf", C.c_void_p),
        ("kept_cap", C.c_int),
        ("topk_idx", C.c_void_p),
        ("topk_cap", C.c_int),
    ]


class _RefBatch(C.Structure):
    _fields_ = [
        ("rows", C.c_int),
        ("vocab", C.c_int),
        ("logits", C.c_void_p),
        ("mask", C.c_void_p),
        ("hist_ids", C.c_void_p),
        ("hist_off", C.c_void_p),
        ("uniforms", C.c_void_p),
        ("params", C.c_void_p),
        ("params_per_row", C.c_int),
        ("token", C.c_void_p),
        ("pen_logits", C.c_void_p),
    ]


_libs: dict[str, C.CDLL] = {}


def _lib(path: str) -> C.CDLL:
    if path not in _libs:
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (run `make -C oracle`)")
        _libs[path] = C.CDLL(path)
    return _libs[path]


def have_reference() -> bool:
    return os.path.exists(REF_ASBUILT_SO)


def _ptr(a):
    return None if a is None else a.ctypes.data


def make_params(rows_or_one):
    """dict or list of dicts -> (ctypes array, per_row flag)."""
    if isinstance(rows_or_one, dict):
        lst, per_row = [rows_or_one], 0
    else:
        lst, per_row = list(rows_or_one), 1
    arr = (Params * len(lst))()
    for i, d in enumerate(lst):
        arr[i] = Params(
            float(d.get("temperature", 1.0)),
            float(d.get("top_p", 1.0)),
            float(d.get("min_p", 0.0)),
            int(d.get("top_k", 0)),
            float(d.get("repetition", 1.0)),
            float(d.get("presence", 0.0)),
            float(d.get("frequency", 0.0)),
        )
    return arr, per_row


@dataclass
class OracleResult:
    token: np.ndarray
    pen_logits: np.ndarray | None = None
    kept_n: np.ndarray | None = None
    kept_idx: np.ndarray | None = None
    kept_prob: np.ndarray | None = None
    kept_cdf: np.ndarray | None = None
    topk_idx: np.ndarray | None = None


def _csr(hist):
    """list of int sequences (or None) -> (ids int32, offsets int64)"""
    if hist is None:
        return None, None
    off = np.zeros(len(hist) + 1, dtype=np.int64)
    for i, h in enumerate(hist):
        off[i + 1] = off[i] + len(h)
    ids = np.zeros(max(int(off[-1]), 1), dtype=np.int32)
    for i, h in enumerate(hist):
        ids[off[i]:off[i + 1]] = np.asarray(h, dtype=np.int32)
    return ids, off


def sample_restated(logits, params, uniforms, mask=None, hist=None, hist_ids=None,
                    hist_off=None, flags=0, want_pen=False, kept_cap=0, topk_cap=0,
                    ftz=True, threads=8) -> OracleResult:
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    rows, vocab = logits.shape
    uniforms = np.ascontiguousarray(uniforms, dtype=np.float32)
    assert uniforms.shape == (rows,)
    if hist is not None:
        hist_ids, hist_off = _csr(hist)
    if mask is not None:
        mask = np.ascontiguousarray(mask, dtype=np.uint32)
        assert mask.shape == (rows, (vocab + 31) // 32)
    parr, per_row = make_params(params)
    res = OracleResult(token=np.zeros(rows, dtype=np.int32))
    if want_pen:
        res.pen_logits = np.zeros((rows, vocab), dtype=np.float32)
    if kept_cap:
        res.kept_n = np.zeros(rows, dtype=np.int32)
        res.kept_idx = np.full((rows, kept_cap), -1, dtype=np.int32)
        res.kept_prob = np.zeros((rows, kept_cap), dtype=np.float32)
        res.kept_cdf = np.zeros((rows, kept_cap), dtype=np.float32)
    if topk_cap:
        res.topk_idx = np.full((rows, topk_cap), -1, dtype=np.int32)
    b = _OracleBatch(
        rows, vocab, _ptr(logits), _ptr(mask), _ptr(hist_ids), _ptr(hist_off),
        _ptr(uniforms), C.addressof(parr), per_row, flags, _ptr(res.token),
        _ptr(res.pen_logits), _ptr(res.kept_n), _ptr(res.kept_idx), _ptr(res.kept_prob),
        _ptr(res.kept_cdf), kept_cap, _ptr(res.topk_idx), topk_cap,
    )
    lib = _lib(RESTATED_SO)
    lib.dllm_oracle_sample_batch.restype = C.c_int
    rc = lib.dllm_oracle_sample_batch(C.byref(b), int(ftz), int(threads))
    if rc != 0:
        raise RuntimeError(f"dllm_oracle_sample_batch failed: {rc}")
    return res


def sample_reference(logits, params, uniforms=None, mask=None, hist=None, hist_ids=None,
                     hist_off=None, want_pen=False, strict=False, threads=8, stream=False):
    """Runs DiskLLM's compiled sampler.  Returns (OracleResult, seconds)."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    rows, vocab = logits.shape
    if uniforms is not None:
        uniforms = np.ascontiguousarray(uniforms, dtype=np.float32)
    if hist is not None:
        hist_ids, hist_off = _csr(hist)
    if mask is not None:
        mask = np.ascontiguousarray(mask, dtype=np.uint32)
    parr, per_row = make_params(params)
    res = OracleResult(token=np.zeros(rows, dtype=np.int32))
    if want_pen:
        res.pen_logits = np.zeros((rows, vocab), dtype=np.float32)
    b = _RefBatch(rows, vocab, _ptr(logits), _ptr(mask), _ptr(hist_ids), _ptr(hist_off),
                  _ptr(uniforms), C.addressof(parr), per_row, _ptr(res.token),
                  _ptr(res.pen_logits))
    lib = _lib(REF_STRICT_SO if strict else REF_ASBUILT_SO)
    lib.ref_sample_batch.restype = C.c_int
    secs = C.c_double(0.0)
    rc = lib.ref_sample_batch(C.byref(b), int(threads), int(stream), C.byref(secs))
    if rc != 0:
        raise RuntimeError(f"ref_sample_batch failed: {rc}")
    return res, secs.value


def reference_greedy(row) -> int:
    row = np.ascontiguousarray(row, dtype=np.float32)
    lib = _lib(REF_ASBUILT_SO)
    lib.ref_greedy.restype = C.c_int
    return int(lib.ref_greedy(C.c_void_p(row.ctypes.data), C.c_int(row.shape[0])))


def reference_seed_for_uniform(r: float) -> int:
    lib = _lib(REF_ASBUILT_SO)
    lib.ref_seed_for_uniform.restype = C.c_uint64
    lib.ref_seed_for_uniform.argtypes = [C.c_float]
    return int(lib.ref_seed_for_uniform(r))


def xorshift_uniforms(seed: int, n: int) -> np.ndarray:
    """n successive rand_f32() values of a reference sampler created with `seed`."""
    lib = _lib(RESTATED_SO)
    lib.dllm_oracle_xorshift_uniform.restype = C.c_float
    st = C.c_uint64(seed if seed else 0xDEADBEEF12345678)
    out = np.empty(n, dtype=np.float32)
    for i in range(n):
        out[i] = lib.dllm_oracle_xorshift_uniform(C.byref(st))
    return out


def reference_cdf(logits_row, params, mask_row=None, hist_row=None, n_boundaries=None):
    """Recovers the reference's own fp32 running-sum CDF for one row by bisection on the
    uniform: the reference returns the candidate at position i iff cdf[i-1] <= r < cdf[i].
    Returns (ids in draw order, cdf) for the first n_boundaries positions."""
    row = np.ascontiguousarray(logits_row, dtype=np.float32)[None, :]
    mask = None if mask_row is None else np.asarray(mask_row, dtype=np.uint32)[None, :]
    hist = None if hist_row is None else [hist_row]

    def draw(bits):
        r = np.array([np.uint32(bits)], dtype=np.uint32).view(np.float32)
        res, _ = sample_reference(row, params, r, mask=mask, hist=hist, threads=1)
        return int(res.token[0])

    # uniforms are float bit patterns in [0, 1); rand_f32 can emit any float >= 2^-30
    lo_bits = int(np.array([2.0 ** -30], dtype=np.float32).view(np.uint32)[0])
    hi_bits = int(np.array([1.0], dtype=np.float32).view(np.uint32)[0]) - 1
    ids, cdf = [], []
    cur_bits = lo_bits
    cur_id = draw(cur_bits)
    while cur_bits <= hi_bits and (n_boundaries is None or len(ids) < n_boundaries):
        last_id = draw(hi_bits)
        if last_id == cur_id:
            ids.append(cur_id)
            cdf.append(np.inf)
            break
        a, z = cur_bits, hi_bits  # draw(a) == cur_id, draw(z) != cur_id
        while z - a > 1:
            mid = (a + z) // 2
            if draw(mid) == cur_id:
                a = mid
            else:
                z = mid
        ids.append(cur_id)
        cdf.append(float(np.array([np.uint32(z)], dtype=np.uint32).view(np.float32)[0]))
        cur_bits = z
        cur_id = draw(z)
    return np.array(ids, dtype=np.int64), np.array(cdf, dtype=np.float64)


def reference_cdf_around(logits_row, params, r, mask_row=None, hist_row=None):
    """The reference's fp32 CDF boundaries that enclose the uniform r: returns (lo, hi, id) with
    lo <= r < hi, where the reference returns `id` for every uniform in [lo, hi) (lo = the
    running sum before id's entry, hi = the one after it; hi = inf when id is the list's last
    entry and r reaches the total).  Found by bisection on the uniform's bit pattern."""
    row = np.ascontiguousarray(logits_row, dtype=np.float32)[None, :]
    mask = None if mask_row is None else np.asarray(mask_row, dtype=np.uint32)[None, :]
    hist = None if hist_row is None else [hist_row]

    def draw(bits):
        x = np.array([np.uint32(bits)], dtype=np.uint32).view(np.float32)
        res, _ = sample_reference(row, params, x, mask=mask, hist=hist, threads=1)
        return int(res.token[0])

    f2b = lambda x: int(np.array([x], dtype=np.float32).view(np.uint32)[0])
    b2f = lambda b: float(np.array([np.uint32(b)], dtype=np.uint32).view(np.float32)[0])
    rb = f2b(r)
    tid = draw(rb)
    # rand_f32 can emit every float in [2^-30, 1) and nothing smaller but 0
    lo_lim, hi_lim = f2b(2.0 ** -30), f2b(1.0) - 1
    if draw(hi_lim) == tid:
        hi = np.inf
    else:
        a, z = rb, hi_lim
        while z - a > 1:
            m = (a + z) // 2
            if draw(m) == tid:
                a = m
            else:
                z = m
        hi = b2f(z)
    if draw(lo_lim) == tid:
        lo = 0.0
    else:
        a, z = lo_lim, rb  # draw(a) != tid, draw(z) == tid
        while z - a > 1:
            m = (a + z) // 2
            if draw(m) == tid:
                z = m
            else:
                a = m
        lo = b2f(z)
    return lo, hi, tid


# ---- LM-head tail (the step before the sampler) ----------------------------------------------

RMSNORM_SO = os.path.join(HERE, "_ref", "librmsnorm_asbuilt.so")


def rmsnorm_restated(x: np.ndarray, w, eps: float, add_one: bool) -> np.ndarray:
    """src/rmsnorm.c:4-27 for each row: sum of squares in double, mean, + eps,
    scale = (float)(1 / sqrt(.)), then in fp32 the products as the reference compiles them at
    -O3 -ffast-math (measured against oracle/_ref/librmsnorm_asbuilt.so): x * scale without a
    weight, (x * scale) * (w + 1) with add_one, and (x * w) * scale with a plain weight (the
    compiler reassociates the source's x * scale * w)."""
    x = np.asarray(x, dtype=np.float32)
    out = np.empty_like(x)
    for r in range(x.shape[0]):
        ss = float(np.sum(x[r].astype(np.float64) ** 2)) / x.shape[1] + float(np.float32(eps))
        scale = np.float32(1.0 / np.sqrt(ss))
        if w is None:
            v = x[r] * scale
        elif add_one:
            ww = (np.asarray(w, dtype=np.float32) + np.float32(1.0)).astype(np.float32)
            v = (x[r] * scale).astype(np.float32) * ww
        else:
            v = (x[r] * np.asarray(w, dtype=np.float32)).astype(np.float32) * scale
        out[r] = v.astype(np.float32)
    return out


def rmsnorm_reference(x: np.ndarray, w, eps: float, add_one: bool) -> np.ndarray:
    """The reference's own rmsnorm_ext (oracle/_ref/librmsnorm_asbuilt.so) on each row."""
    lib = _lib(RMSNORM_SO)
    lib.rmsnorm_ext.restype = None
    lib.rmsnorm_ext.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_float, C.c_int]
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    ww = None if w is None else np.ascontiguousarray(w, dtype=np.float32)
    for r in range(x.shape[0]):
        lib.rmsnorm_ext(out[r].ctypes.data, x[r].ctypes.data, None if ww is None else ww.ctypes.data,
                        x.shape[1], float(eps), int(add_one))
    return out


def lmhead_restated(h: np.ndarray, w_f32: np.ndarray, norm_w=None, eps=1e-6, add_one=False,
                    softcap=0.0) -> np.ndarray:
    """src/core/context.c:854-876 for unquantised output weights: rmsnorm_ext, then per output
    row the double-precision dot product of src/matvec.c:251-366 (products of the fp32-upcast
    weights and inputs, summed in double, rounded to float once), then the softcap
    cap * tanhf(x / cap).  w_f32 holds the weights upcast exactly to fp32."""
    hn = rmsnorm_restated(h, norm_w, eps, add_one).astype(np.float64)
    out = (hn @ np.asarray(w_f32, dtype=np.float64).T).astype(np.float32)
    if softcap > 0:
        cap = np.float32(softcap)
        out = (cap * np.tanh((out / cap).astype(np.float32)).astype(np.float32)).astype(np.float32)
    return out
