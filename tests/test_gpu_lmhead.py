"""The LM-head tail on the GPU (dllm_cuda_lmhead_logits: final RMSNorm, logits matvec, softcap;
src/core/context.c:854-876) against the CPU restatement oracle.lmhead_restated on the same
inputs.  Tolerances: the matvec sums its products in double in a different order from the
reference's sequential loop, so the rounded float agrees to within one ulp; tanhf on the
device differs from the host's by at most two ulp, so with a softcap the bound is 4 ulp."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from diskllm_b200 import capi

pytestmark = pytest.mark.gpu


def _weights(rng, vocab, hidden, dtype):
    w32 = (rng.standard_normal((vocab, hidden)) * 0.04).astype(np.float32)
    wt = torch.from_numpy(w32).to(dtype)
    return wt, wt.float().numpy()  # weights as stored, and their exact fp32 upcast


@pytest.mark.parametrize("rows,hidden,vocab,dtype,norm,add_one,softcap", [
    (1, 4096, 32000, torch.bfloat16, True, False, 0.0),
    (3, 2304, 5003, torch.bfloat16, True, True, 30.0),       # Gemma-style (w + 1) norm and softcap
    (8, 1024, 4099, torch.float16, True, False, 0.0),
    (11, 512, 1000, torch.float32, False, False, 0.0),       # more rows than one launch's group
    (2, 264, 77, torch.float32, True, False, 0.0),           # hidden not a multiple of 256
])
def test_lmhead_matches_restatement(rows, hidden, vocab, dtype, norm, add_one, softcap):
    rng = np.random.default_rng(rows * 1000 + hidden)
    h = (rng.standard_normal((rows, hidden)) * 3.0).astype(np.float32)
    nw = (rng.standard_normal(hidden) * 0.2 + (0.0 if add_one else 1.0)).astype(np.float32) if norm else None
    wt, w32 = _weights(rng, vocab, hidden, dtype)
    dev = torch.device("cuda", 0)
    got = capi.lmhead_logits(torch.from_numpy(h).to(dev), wt.to(dev).contiguous(),
                             norm_w=None if nw is None else torch.from_numpy(nw).to(dev), add_one=add_one,
                             softcap=softcap).cpu().numpy()
    torch.cuda.synchronize()
    ref = O.lmhead_restated(h, w32, nw, 1e-6, add_one, softcap)
    np.testing.assert_array_max_ulp(got, ref, maxulp=4 if softcap > 0 else 1)
    if softcap == 0:
        assert np.mean(got == ref) > 0.99


def test_lmhead_feeds_the_sampler():
    """logits from the tail sampled greedily equal the arg-max of the restated logits"""
    rng = np.random.default_rng(5)
    rows, hidden, vocab = 4, 2048, 50000
    h = rng.standard_normal((rows, hidden)).astype(np.float32)
    wt, w32 = _weights(rng, vocab, hidden, torch.bfloat16)
    dev = torch.device("cuda", 0)
    lg = capi.lmhead_logits(torch.from_numpy(h).to(dev), wt.to(dev))
    u = torch.zeros(rows, dtype=torch.float32, device=dev)
    tok = capi.sample_batch(lg, u, dict(temperature=0.0)).cpu().numpy()
    ref = O.lmhead_restated(h, w32)
    np.testing.assert_array_equal(tok, np.argmax(ref, axis=1))


def test_lmhead_rejects_bad_arguments():
    dev = torch.device("cuda", 0)
    h = torch.zeros(1, 12, device=dev)
    w = torch.zeros(10, 12, device=dev)
    with pytest.raises(capi.DllmError):
        capi.lmhead_logits(h, w)  # hidden not a multiple of 8
