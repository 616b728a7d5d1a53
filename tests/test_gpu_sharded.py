"""Vocabulary-sharded sampling on the GPU against the whole-row oracle.

On one GPU the N shards run one after another (dllm_cuda_shard_candidates per column range),
their candidates are stacked as the all-gather would stack them, and dllm_cuda_merge_sample
draws.  Checked: every shard's candidates (values and ids) bit for bit against the oracle's
penalised row, and the tokens against the oracle's tokens (src/sampler.c:136-234 on whole rows).
With 2, 4 or 8 GPUs the same runs through NCCL, one process per GPU.  Every test runs on both candidate
kernels (the per-row streaming kernel and the per-chunk kernels).
"""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import oracle as O
from diskllm_b200 import capi, sharded
from util import csr, ids_match, pack_mask, u24

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(autouse=True, params=["stream", "chunked"])
def shard_path(request, monkeypatch):
    """both candidate kernels: one streaming CTA per row (the default when k + the history bound
    fits its exact select) and the per-chunk kernels with the row merge (DLLM_SHARD_CHUNKED)"""
    if request.param == "chunked":
        monkeypatch.setenv("DLLM_SHARD_CHUNKED", "1")
    else:
        monkeypatch.delenv("DLLM_SHARD_CHUNKED", raising=False)
    return request.param


def _shard_np(pen, s, e, k):
    vals = np.zeros((pen.shape[0], k), dtype=np.float32)
    ids = np.zeros((pen.shape[0], k), dtype=np.int32)
    for r in range(pen.shape[0]):
        seg = pen[r, s:e]
        order = np.lexsort((np.arange(s, e), -seg.astype(np.float64)))[:k]
        vals[r] = seg[order]
        ids[r] = order + s
    return vals, ids


def _run(x, allow, hist, params, nsh, k, dtype=torch.bfloat16, seed=0):
    rows, V = x.shape
    rng = np.random.default_rng(seed)
    uni = u24(rng, rows)
    mask = pack_mask(allow) if allow is not None else None
    ora = O.sample_restated(x, params, uni, mask=mask, hist=hist, want_pen=True, kept_cap=k, topk_cap=k)
    dev = torch.device("cuda", 0)
    xt = torch.from_numpy(x).to(dev).to(dtype)
    mt = torch.from_numpy(mask.view(np.int32)).to(dev) if mask is not None else None
    hid, hoff = (torch.from_numpy(a).to(dev) for a in csr(hist)) if hist is not None else (None, None)
    ut = torch.from_numpy(uni).to(dev)
    vs, is_ = [], []
    for r in range(nsh):
        s, e = sharded.shard_range(V, r, nsh)
        kw = dict(hist_ids=hid, hist_off=hoff)
        if mt is not None:
            kw["mask"] = mt[:, s // 32:(e + 31) // 32].contiguous()
        v, i = capi.shard_candidates(xt[:, s:e], s, V, k, params, **kw)
        vs.append(v)
        is_.append(i)
        ev, ei = _shard_np(ora.pen_logits, s, e, k)
        np.testing.assert_array_equal(i.cpu().numpy(), ei, err_msg=f"shard {r} candidate ids")
        np.testing.assert_array_equal(v.cpu().numpy().view(np.uint32), ev.view(np.uint32),
                                      err_msg=f"shard {r} candidate values")
    tok = capi.merge_sample(torch.stack(vs).contiguous(), torch.stack(is_).contiguous(), ut, params)
    torch.cuda.synchronize()
    tok = tok.cpu().numpy()
    bad = [r for r in range(rows) if not ids_match(int(tok[r]), ora, uni, r)]
    assert not bad, f"rows {bad[:8]}: gpu {tok[bad[:8]]} oracle {ora.token[bad[:8]]}"
    return tok, ora


def _bf16_grid(a):
    """values exactly representable in bf16 (so the oracle sees what the GPU reads)"""
    return torch.from_numpy(a).to(torch.bfloat16).float().numpy()


@pytest.mark.parametrize("nsh", [2, 4, 8])
def test_config5_shape_bf16(nsh):
    rng = np.random.default_rng(505 + nsh)
    rows, V = 24, 262144
    x = _bf16_grid((rng.standard_normal((rows, V)) * 2.0).astype(np.float32))
    allow = rng.random((rows, V)) < 0.10
    hist = [rng.integers(0, V, 128) for _ in range(rows)]
    params = dict(temperature=0.9, top_k=64, top_p=0.9, repetition=1.1)
    _run(x, allow, hist, params, nsh, 64, seed=nsh)


# shard counts whose merges rank nsh * k <= 256 candidates by search and more than 256 by a sort
@pytest.mark.parametrize("nsh", [3, 6])
def test_f32_penalties_minp_odd_vocab(nsh):
    rng = np.random.default_rng(11)
    rows, V = 16, 5000
    x = (rng.standard_normal((rows, V)) * 3.0).astype(np.float32)
    hist = [rng.integers(0, V, 40) for _ in range(rows)]
    params = dict(temperature=0.7, top_k=50, top_p=0.95, min_p=0.01, repetition=1.2, presence=0.3)
    _run(x, None, hist, params, nsh, 64, dtype=torch.float32)


@pytest.mark.parametrize("nsh", [4, 8])
def test_ties_take_lowest_ids(nsh):
    rng = np.random.default_rng(12)
    rows, V = 8, 8192
    x = rng.integers(-3, 3, (rows, V)).astype(np.float32)  # thousands of equal values
    params = dict(temperature=1.0, top_k=40, top_p=0.8)
    _run(x, None, None, params, nsh, 40, dtype=torch.float32)


@pytest.mark.parametrize("nsh", [2, 9])
def test_fewer_allowed_than_k_and_fully_masked_rows(nsh):
    rng = np.random.default_rng(13)
    rows, V = 8, 4096
    x = (rng.standard_normal((rows, V))).astype(np.float32)
    allow = np.zeros((rows, V), dtype=bool)
    for r in range(1, rows):
        allow[r, rng.choice(V, size=r * 3, replace=False)] = True  # 3 .. 21 allowed, k = 32
    params = dict(temperature=1.0, top_k=32, top_p=0.9)
    tok, ora = _run(x, allow, None, params, nsh, 32, dtype=torch.float32)
    assert tok[0] == ora.token[0] == 31  # fully masked: the reference returns its list's last id


def test_greedy():
    rng = np.random.default_rng(14)
    rows, V = 8, 20000
    x = _bf16_grid((rng.standard_normal((rows, V)) * 2.0).astype(np.float32))
    x[:, 777] = x.max()  # ties for the maximum: the first id wins
    params = dict(temperature=0.0, top_k=8, repetition=1.1)
    hist = [rng.integers(0, V, 16) for _ in range(rows)]
    _run(x, None, hist, params, 4, 8)


@pytest.mark.parametrize("exchange", ["nccl", "peer"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_nccl_ranks(world, exchange, shard_path):
    """world ranks, one per GPU, each sampling from its own columns; candidates all-gathered by NCCL
    or stored into every rank's buffer over NVLink (three steps each)"""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    if exchange == "peer" and shard_path == "chunked":
        pytest.skip("the peer exchange is written by the streaming candidate kernel")
    script = os.path.join(ROOT, "tests", "sharded_nccl_worker.py")
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([ROOT, os.path.join(ROOT, "tests"),
                                                      os.path.join(ROOT, "oracle")]), DLLM_TEST_EXCHANGE=exchange)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr=127.0.0.1", f"--master-port={29613 + world + (8 if exchange == 'peer' else 0)}", script]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
    assert "SHARDED_NCCL_OK" in res.stdout


def test_merge_rejects_rows_the_candidates_cannot_serve():
    """per-row top_k above the gathered k, or top-k off, at temperature > 0: greedy token plus
    DLLM_ROW_ERR_TOPK_LARGE; the other rows sample normally"""
    rng = np.random.default_rng(15)
    rows, V, k = 6, 4096, 16
    x = (rng.standard_normal((rows, V)) * 2.0).astype(np.float32)
    uni = u24(rng, rows)
    good = dict(temperature=0.8, top_k=12, top_p=0.9)
    per_row = [good, dict(good, top_k=k + 1), dict(good, top_k=0), good, dict(good, top_k=-3),
               dict(good, top_k=k)]
    dev = torch.device("cuda", 0)
    xt = torch.from_numpy(x).to(dev)
    vs, is_ = [], []
    for r in range(2):
        s, e = sharded.shard_range(V, r, 2)
        v, i = capi.shard_candidates(xt[:, s:e], s, V, k, good)
        vs.append(v)
        is_.append(i)
    rp = capi.params_array(per_row, dev)
    status = torch.full((rows,), -1, dtype=torch.int32, device=dev)
    tok = capi.merge_sample(torch.stack(vs).contiguous(), torch.stack(is_).contiguous(),
                            torch.from_numpy(uni).to(dev), good, row_params=rp, status=status)
    torch.cuda.synchronize()
    tok, status = tok.cpu().numpy(), status.cpu().numpy()
    for r, p in enumerate(per_row):
        if 1 <= p["top_k"] <= k:
            assert status[r] == 0
            ora = O.sample_restated(x[r:r + 1], p, uni[r:r + 1], kept_cap=k)
            assert ids_match(int(tok[r]), ora, uni[r:r + 1], 0)
        else:
            assert status[r] == capi.ROW_ERR_TOPK_LARGE
            assert tok[r] == int(np.argmax(x[r]))
    with pytest.raises(capi.DllmError):
        capi.merge_sample(torch.stack(vs).contiguous(), torch.stack(is_).contiguous(),
                          torch.from_numpy(uni).to(dev), dict(good, top_k=k + 1))



def _peer_single(world, rows, k):
    buf, _ = capi.peer_exchange_create(rows, k, world)
    return buf


def test_peer_exchange_on_one_gpu_matches_oracle(shard_path):
    """world 1: the candidate kernel stores into this GPU's exchange buffer and the merge reads it,
    for two steps (both slots)"""
    if shard_path == "chunked":
        pytest.skip("the peer exchange is written by the streaming candidate kernel")
    rng = np.random.default_rng(17)
    rows, V, k = 8, 20000, 40
    x = _bf16_grid((rng.standard_normal((rows, V)) * 2.0).astype(np.float32))
    hist = [rng.integers(0, V, 64) for _ in range(rows)]
    params = dict(temperature=0.9, top_k=32, top_p=0.9, repetition=1.1)
    dev = torch.device("cuda", 0)
    xt = torch.from_numpy(x).to(dev).to(torch.bfloat16)
    hid, hoff = (torch.from_numpy(a).to(dev) for a in csr(hist))
    buf = _peer_single(1, rows, k)
    peers = torch.tensor([buf], dtype=torch.int64, device=dev)
    try:
        for epoch in (1, 2):
            uni = u24(rng, rows)
            capi.shard_candidates_peer(xt, 0, V, k, params, peers, 0, 1, epoch, hist_ids=hid, hist_off=hoff,
                                       hist_max=64)
            st = torch.full((rows,), -1, dtype=torch.int32, device=dev)
            tok = capi.merge_sample_peer(rows, 1, k, buf, epoch, torch.from_numpy(uni).to(dev), params, status=st)
            torch.cuda.synchronize()
            ora = O.sample_restated(x, params, uni, hist=hist, kept_cap=k, topk_cap=k)
            t = tok.cpu().numpy()
            assert np.all(st.cpu().numpy() == 0)
            assert all(ids_match(int(t[r]), ora, uni, r) for r in range(rows)), (t, ora.token)
    finally:
        capi.load_library().dllm_cuda_peer_exchange_free(buf)


def test_peer_merge_times_out_when_a_rank_never_arrives(shard_path):
    """a two-rank exchange in which nothing is ever stored: the merge's bounded wait gives up
    (about 2 s), every row gets DLLM_ROW_ERR_TIMEOUT, and the context stays usable"""
    import time

    if shard_path == "chunked":
        pytest.skip("one run is enough")
    rows, k = 4, 16
    dev = torch.device("cuda", 0)
    buf = _peer_single(2, rows, k)
    try:
        st = torch.full((rows,), -1, dtype=torch.int32, device=dev)
        t0 = time.time()
        capi.merge_sample_peer(rows, 2, k, buf, 1, torch.zeros(rows, device=dev), dict(temperature=1.0, top_k=8),
                               status=st)
        torch.cuda.synchronize()
        assert time.time() - t0 < 30
        assert np.all(st.cpu().numpy() == capi.ROW_ERR_TIMEOUT)
    finally:
        capi.load_library().dllm_cuda_peer_exchange_free(buf)
    x = torch.randn(2, 1000, device=dev)
    capi.sample_batch(x, torch.full((2,), 0.5, device=dev), dict(temperature=1.0, top_k=5))
    torch.cuda.synchronize()
