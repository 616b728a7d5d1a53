"""Decode loop (sample, append to the device history, next step) against the reference's step
sequence run on the host by the oracle, with the history growing by the sampled ids
(src/core/sampler_api.c:48-73 per step).  The graph replay and the eager launches agree."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from diskllm_b200.decode import DecodeLoop
from util import ids_match, u24

pytestmark = pytest.mark.gpu


def _case(seed, R, V, steps):
    rng = np.random.default_rng(seed)
    ring = (rng.standard_normal((R, V)) * 2.5).astype(np.float32)
    for r in range(R):
        ring[r, rng.choice(V, 20, replace=False)] += 8.0
    hist0 = rng.integers(0, V, 64).astype(np.int32)
    u = u24(rng, steps)
    return ring, hist0, u


@pytest.mark.parametrize("params", [
    dict(temperature=0.8, top_k=40, top_p=0.95, repetition=1.1),        # config 1
    dict(temperature=1.0, top_k=0, top_p=0.9, repetition=1.3, presence=0.4),
])
def test_decode_loop_matches_host_step_sequence(params):
    R, V, steps = 4, 128256, 48
    ring, hist0, u = _case(7, R, V, steps)
    dev = torch.device("cuda", 0)
    loop = DecodeLoop(torch.from_numpy(ring).to(dev), torch.from_numpy(u).to(dev), params,
                      torch.from_numpy(hist0).to(dev))
    eager = loop.run_eager().cpu().numpy().copy()
    graph = loop.replay().cpu().numpy().copy()
    np.testing.assert_array_equal(graph, eager)
    hist = list(hist0)
    for i in range(steps):
        ora = O.sample_restated(ring[i % R:i % R + 1], params, u[i:i + 1], hist=[np.array(hist, np.int32)],
                                kept_cap=V)
        if graph[i] != ora.token[0]:
            # only a uniform within the tolerance of a CDF boundary may differ; the sequences
            # then legitimately diverge, so the comparison ends there
            assert ids_match(int(graph[i]), ora, u[i:i + 1], 0), f"step {i}: {graph[i]} vs {ora.token[0]}"
            break
        hist.append(int(graph[i]))
    gh = loop.hist_ids[: loop.hist_off[1]].cpu().numpy()
    np.testing.assert_array_equal(gh, np.concatenate([hist0, graph]).astype(np.int32))


def test_history_window_slides_when_full():
    R, V, steps = 2, 5000, 12
    ring, hist0, u = _case(8, R, V, steps)
    dev = torch.device("cuda", 0)
    params = dict(temperature=1.0, top_k=20, repetition=1.2)
    loop = DecodeLoop(torch.from_numpy(ring).to(dev), torch.from_numpy(u).to(dev), params,
                      torch.from_numpy(hist0).to(dev), cap=70)
    tok = loop.replay().cpu().numpy()
    full = np.concatenate([hist0, tok]).astype(np.int32)
    np.testing.assert_array_equal(loop.hist_ids[:70].cpu().numpy(), full[-70:])
    assert int(loop.hist_off[1]) == 70
