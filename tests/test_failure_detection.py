"""Failure detection without a GPU fault.

GPU (test hooks of the library, off by default):
  * a bounded mbarrier wait that nothing completes runs out after a few thousand polls; the
    kernel goes on, the launch succeeds, the row's status carries DLLM_ROW_ERR_TIMEOUT, and the
    next launch on the same context samples correctly.  The waited barrier has no copy or store
    in flight to it: the hook waits for the phase after the one that completed.
  * a device allocation that fails as if out of memory makes the call return DLLM_ERR_OOM, and
    the next call succeeds (the reference returns NULL from sampler_create on OOM,
    src/sampler.c:83-85).
CPU (gloo ranks):
  * a rank that dies before the candidate all-gather of vocabulary-sharded sampling makes the
    other rank's gather raise an error within the process group's timeout instead of hanging.
"""
from __future__ import annotations

import datetime
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle as O
from util import csr, ids_match, u24


def _rows(V=32000, rows=3, seed=0):
    rng = np.random.default_rng(seed)
    lg = (rng.standard_normal((rows, V)) * 0.7).astype(np.float32)
    hist = [rng.integers(0, V, 64) for _ in range(rows)]
    return lg, hist, u24(rng, rows)


def _sample(lg, hist, u, params, stream=None):
    from diskllm_b200 import capi

    dev = torch.device("cuda", 0)
    ids, off = csr(hist)
    st = torch.full((lg.shape[0],), -1, dtype=torch.int32, device=dev)
    tok = capi.sample_batch(torch.from_numpy(lg).to(dev), torch.from_numpy(u).to(dev), params,
                            hist_ids=torch.from_numpy(ids).to(dev), hist_off=torch.from_numpy(off).to(dev),
                            status=st, stream=stream)
    torch.cuda.synchronize()
    return tok.cpu().numpy(), st.cpu().numpy()


PARAMS = {
    "index_order": dict(temperature=1.0, top_k=0, top_p=0.99, repetition=1.05),
    "top_k": dict(temperature=0.8, top_k=40, top_p=0.95, repetition=1.1),
}


@pytest.mark.gpu
@pytest.mark.parametrize("site", ["copy", "exchange"])
@pytest.mark.parametrize("name", list(PARAMS))
def test_bounded_wait_runs_out_and_is_reported(site, name):
    from diskllm_b200 import capi

    lg, hist, u = _rows()
    p = PARAMS[name]
    s = capi.FAULT_COPY_WAIT if site == "copy" else capi.FAULT_EXCHANGE_WAIT
    capi.inject_wait_timeout(s, 4096)
    try:
        t0 = time.time()
        _, st = _sample(lg, hist, u, p)
        elapsed = time.time() - t0
    finally:
        capi.inject_wait_timeout(capi.FAULT_NONE)
    # three rows fit three clusters, so every row is its cluster's first and carries the timeout
    assert np.all(st & capi.ROW_ERR_TIMEOUT), st
    assert elapsed < 30.0
    # the context is intact: the same rows sample correctly with the hook off
    tok, st = _sample(lg, hist, u, p)
    assert np.all(st & ~capi.ROW_TOPP_EDGE == 0), st
    ora = O.sample_restated(lg, p, u, hist=hist, kept_cap=lg.shape[1])
    for i in range(lg.shape[0]):
        assert ids_match(int(tok[i]), ora, u, i) or st[i] & capi.ROW_TOPP_EDGE, (i, tok[i], ora.token[i])


@pytest.mark.gpu
def test_allocation_failure_returns_oom():
    from diskllm_b200 import capi

    lg, hist, u = _rows(rows=2)
    p = PARAMS["index_order"]
    side = torch.cuda.Stream()  # a stream the library holds no workspace for yet
    capi.fail_allocations(1)
    try:
        with pytest.raises(capi.DllmError, match="OOM"):
            _sample(lg, hist, u, p, stream=side.cuda_stream)
    finally:
        capi.fail_allocations(0)
    tok, st = _sample(lg, hist, u, p, stream=side.cuda_stream)
    assert np.all(st & ~capi.ROW_TOPP_EDGE == 0)


def test_hooks_validate_arguments_without_gpu():
    from diskllm_b200 import capi

    lib = capi.load_library()
    assert lib.dllm_cuda_debug_inject_wait_timeout(3, 10) == capi.DLLM_ERR_INVALID_ARG
    assert lib.dllm_cuda_debug_inject_wait_timeout(1, 0) == capi.DLLM_ERR_INVALID_ARG
    assert lib.dllm_cuda_debug_inject_wait_timeout(0, 0) == capi.DLLM_OK
    assert lib.dllm_cuda_debug_fail_allocations(-1) == capi.DLLM_ERR_INVALID_ARG
    assert lib.dllm_cuda_debug_fail_allocations(0) == capi.DLLM_OK


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, result):
    import torch.distributed as dist

    from diskllm_b200 import capi, sharded

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        # this rank fails between steps, before its candidates are exchanged
        os._exit(3)
    buf, v, i = sharded.candidate_buffer(4, 8, "cpu")
    v.fill_(1.0)
    i.fill_(7)
    t0 = time.time()
    try:
        sharded.gather_packed(buf, 4, 8)
        result["outcome"] = "returned"
    except capi.DllmError as e:
        result["outcome"] = "error"
        result["message"] = str(e)
    result["seconds"] = time.time() - t0


def test_dead_rank_surfaces_as_error_not_hang():
    port = _free_port()
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, result)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        alive = [p.is_alive() for p in procs]
        for p in procs:
            if p.is_alive():
                p.kill()
        assert not any(alive), "a rank hung"
        assert procs[1].exitcode == 3
        assert result.get("outcome") == "error", dict(result)
        assert "all-gather" in result.get("message", "")
        assert result["seconds"] < 60
