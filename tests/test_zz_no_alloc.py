"""dllm_cuda_sample_batch_static: the allocation-free entry point, for callers that cannot call
cudaMalloc (an embedder whose device memory belongs to its own allocator, or a decode loop that
must not stall on cudaMalloc's device-wide synchronisation).  It must sample exactly like the
regular entry point while using only the library's fixed scratch array.

This file is collected last on purpose (tests/test_zz_*), so a run that stops at the first
failure has already run every other test.  It passes both alone in a fresh process and after the
other tests."""
import ctypes as C

import numpy as np
import pytest

from util import csr, u24

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _inputs(rows, V, seed):
    rng = np.random.default_rng(seed)
    lg = (rng.standard_normal((rows, V)) * 0.5).astype(np.float32)
    hist = [rng.integers(0, V, 256) for _ in range(rows)]
    ids, off = csr(hist)
    dev = "cuda"
    return (torch.from_numpy(lg).to(dev), torch.from_numpy(u24(rng, rows)).to(dev),
            torch.from_numpy(ids).to(dev), torch.from_numpy(off).to(dev))


@pytest.mark.parametrize("params", [
    dict(temperature=1.0, top_k=0, top_p=0.99, repetition=1.05),   # index-order path (uses scratch)
    dict(temperature=0.8, top_k=40, top_p=0.95, repetition=1.1),    # top-k path
])
def test_static_entry_matches_regular_entry_twice(params):
    from diskllm_b200 import capi

    rows, V = 96, 64000
    x, u, ids, off = _inputs(rows, V, 7)
    p_ref = torch.full((rows, V), -1.0, device="cuda")
    t_ref = capi.sample_batch(x, u, params, hist_ids=ids, hist_off=off, probs=p_ref)
    torch.cuda.synchronize()
    for _ in range(2):   # two calls in a row share and reuse the static scratch
        p_s = torch.full((rows, V), -1.0, device="cuda")
        t_s, rc = capi.sample_batch_static(x, u, params, hist_ids=ids, hist_off=off, probs=p_s)
        torch.cuda.synchronize()
        assert rc == capi.DLLM_OK
        assert torch.equal(t_s, t_ref)
        assert float((p_s - p_ref).abs().max()) <= 1e-6


def test_static_entry_rejects_batches_beyond_its_scratch():
    from diskllm_b200 import capi

    x, u, ids, off = _inputs(4, 1024, 1)
    d, tok = capi.fill_desc(x, u, dict(temperature=1.0, top_p=0.99))
    d.rows, d.vocab, d.row_stride = 8192, 256000, 256000   # needs far more than 16 MiB; no launch
    lib = capi.load_library()
    assert lib.dllm_cuda_workspace_bytes(C.byref(d)) > (16 << 20)
    rc = lib.dllm_cuda_sample_batch_static(C.byref(d), None)
    assert rc == 6
    assert b"static scratch" in lib.dllm_cuda_last_error()
