"""Vocabulary-sharded sampling: the host side on CPU with two gloo ranks.

Each rank selects its shard's candidates with a numpy restatement of the selection rule
(k best by (value desc, id asc) after mask and penalties), exchanges them through the product's
`sharded.gather_candidates`, and rank 0 merges them like the merge kernel (row max, t = (v-M)/T,
k best by (t desc, id asc)).  The merged list must equal the top-k list of the whole-row oracle
(src/sampler.c:109-170), which is what the GPU merge then samples from.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from diskllm_b200 import sharded
import oracle as O
from util import pack_mask


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(seed=7, rows=6, V=4096):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((rows, V)) * 2.0).astype(np.float32)
    allow = rng.random((rows, V)) < 0.3
    allow[0, :] = True
    hist = [rng.integers(0, V, 24) for _ in range(rows)]
    params = dict(temperature=0.9, top_k=16, top_p=0.9, repetition=1.1, presence=0.2)
    return x, allow, hist, params


def _shard_candidates_np(pen: np.ndarray, s: int, e: int, k: int):
    """k best of columns [s, e) by (value desc, id asc) for every row: (values, global ids)."""
    vals = np.zeros((pen.shape[0], k), dtype=np.float32)
    ids = np.zeros((pen.shape[0], k), dtype=np.int32)
    for r in range(pen.shape[0]):
        seg = pen[r, s:e]
        order = np.lexsort((np.arange(s, e), -seg.astype(np.float64)))[:k]
        vals[r] = seg[order]
        ids[r] = order + s
    return vals, ids


def _merge_np(all_v: np.ndarray, all_i: np.ndarray, temperature: float, k: int):
    nsh, rows, kk = all_v.shape
    out = np.zeros((rows, k), dtype=np.int32)
    for r in range(rows):
        v = all_v[:, r, :].reshape(-1)
        i = all_i[:, r, :].reshape(-1)
        M = np.float32(v.max())
        inv = np.float32(1.0) / np.float32(temperature)
        t = ((v - M).astype(np.float32) * inv).astype(np.float32)
        order = np.lexsort((i, -t.astype(np.float64)))[:k]
        out[r] = i[order]
    return out


def _worker(rank, world, port, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, allow, hist, params = _case()
        rows, V = x.shape
        k = params["top_k"]
        ora = O.sample_restated(x, params, np.zeros(rows, np.float32), mask=pack_mask(allow), hist=hist,
                                want_pen=True, topk_cap=k)
        s, e = sharded.shard_range(V, rank, world)
        v, i = _shard_candidates_np(ora.pen_logits, s, e, k)
        all_v, all_i = sharded.gather_candidates(torch.from_numpy(v), torch.from_numpy(i))
        # the single-collective layout sample_vocab_sharded uses: values and ids in one buffer
        buf, bv, bi = sharded.candidate_buffer(rows, k, "cpu")
        bv.copy_(torch.from_numpy(v))
        bi.copy_(torch.from_numpy(i))
        pv, pi = sharded.gather_packed(buf, rows, k)
        if rank == 0:
            result["packed_equal"] = bool(torch.equal(pv.view(torch.int32), all_v.view(torch.int32)) and
                                          torch.equal(pi, all_i))
            merged = _merge_np(all_v.numpy(), all_i.numpy(), params["temperature"], k)
            result["ok"] = bool(np.array_equal(merged, ora.topk_idx))
            result["shapes"] = tuple(all_v.shape)
    finally:
        dist.destroy_process_group()


def test_shard_range_partitions_on_mask_words():
    for V, world in [(262144, 8), (151936, 3), (4096, 2), (1000, 4)]:
        spans = [sharded.shard_range(V, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == V
        for (s0, e0), (s1, e1) in zip(spans, spans[1:]):
            assert e0 == s1
        assert all(s % 32 == 0 for s, _ in spans)


def test_two_gloo_ranks_merge_to_the_whole_row_topk():
    port = _free_port()
    with mp.Manager() as mgr:
        result = mgr.dict()
        mp.spawn(_worker, args=(2, port, result), nprocs=2, join=True)
        assert result.get("shapes") == (2, 6, 16)
        assert result.get("ok"), "merged shard candidates differ from the whole-row top-k"
        assert result.get("packed_equal"), "one-buffer all-gather differs from the two-tensor gather"
