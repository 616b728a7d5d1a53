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


PARAMS = {
    "index_order": dict(temperature=1.0, top_k=0, top_p=0.99, repetition=1.05),  # records, stash, wide slots
    "top_k": dict(temperature=0.8, top_k=40, top_p=0.95, repetition=1.1),
    "sorted_nucleus": dict(temperature=0.9, top_k=0, top_p=0.9),                  # sorted-mode scratch
}


def _outputs(x):
    rows, V = x.shape
    return (torch.empty(rows, dtype=torch.int32, device="cuda"), torch.full((rows, V), -1.0, device="cuda"),
            torch.full((rows,), -1, dtype=torch.int32, device="cuda"))


def _run(fn, x, u, ids, off, params, flags, outs=None, **kw):
    from diskllm_b200 import capi

    tok, probs, status = outs if outs is not None else _outputs(x)
    out = fn(x, u, params, hist_ids=ids, hist_off=off, token=tok, probs=probs, status=status, flags=flags, **kw)
    rc = out[1] if isinstance(out, tuple) else capi.DLLM_OK
    torch.cuda.synchronize()
    return tok, probs, status, rc


@pytest.mark.parametrize("name", list(PARAMS))
def test_static_entry_matches_regular_entry_twice(name):
    """two static calls in a row on DIFFERENT batches, each identical bit for bit to the regular
    entry point on the same batch, so leftover scratch from the first call cannot leak into the
    second.  The second call runs on a new stream while every library allocation is made to fail,
    and the device's free memory does not change: the static entry allocates nothing."""
    from diskllm_b200 import capi

    params = PARAMS[name]
    flags = capi.MODE_TOPP_SORTED if name == "sorted_nucleus" else 0
    rows, V = (32 if name == "sorted_nucleus" else 96), 64000  # within the 16 MiB scratch
    batches = [_inputs(rows, V, 7), _inputs(rows, V, 8)]
    want = [_run(capi.sample_batch, *b, params, flags) for b in batches]
    _run(capi.sample_batch_static, *batches[1], params, flags)  # set-up: symbol address, launch configuration
    side = torch.cuda.Stream()
    for i, b in enumerate(batches):
        outs = _outputs(b[0])
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        if i == 1:
            capi.fail_allocations(1 << 20)
        try:
            tok, probs, status, rc = _run(capi.sample_batch_static, *b, params, flags, outs=outs,
                                          stream=side.cuda_stream if i == 1 else None)
        finally:
            capi.fail_allocations(0)
        assert rc == capi.DLLM_OK
        assert torch.cuda.mem_get_info()[0] == free0
        t_ref, p_ref, s_ref, _ = want[i]
        assert torch.equal(tok, t_ref), i
        assert torch.equal(status, s_ref), i
        assert torch.equal(probs.view(torch.int32), p_ref.view(torch.int32)), i
    assert not torch.equal(want[0][0], want[1][0])  # the two batches really differ


def test_static_entry_rejects_batches_beyond_its_scratch():
    from diskllm_b200 import capi

    x, u, ids, off = _inputs(4, 1024, 1)
    d, tok = capi.fill_desc(x, u, dict(temperature=1.0, top_p=0.99))
    d.rows, d.vocab, d.row_stride = 8192, 256000, 256000   # needs far more than 16 MiB; no launch
    lib = capi.load_library()
    assert lib.dllm_cuda_workspace_bytes(C.byref(d)) > (16 << 20)
    rc = lib.dllm_cuda_sample_batch_static(C.byref(d), None)
    assert rc == capi.DLLM_ERR_UNSUPPORTED
    assert b"static scratch" in lib.dllm_cuda_last_error()
