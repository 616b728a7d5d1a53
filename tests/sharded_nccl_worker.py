"""Multi-GPU run (2, 4 or 8 ranks; DLLM_TEST_EXCHANGE=peer for the NVLink peer exchange instead of
the NCCL all-gather) of vocabulary-sharded sampling through NCCL (launched by test_gpu_sharded.py with
torch.distributed.run).  Every rank builds the same seeded rows, samples from its own columns
with sharded.sample_vocab_sharded, and checks that all ranks drew the same tokens; rank 0 checks
them against the whole-row oracle."""
from __future__ import annotations

import os

import numpy as np
import torch
import torch.distributed as dist

import oracle as O
from diskllm_b200 import sharded
from util import csr, ids_match, pack_mask, u24


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev)
    rng = np.random.default_rng(2024)
    rows, V = 32, 262144
    x = torch.from_numpy((rng.standard_normal((rows, V)) * 2.0).astype(np.float32)).to(torch.bfloat16)
    allow = rng.random((rows, V)) < 0.10
    hist = [rng.integers(0, V, 128) for _ in range(rows)]
    uni = u24(rng, rows)
    params = dict(temperature=0.9, top_k=64, top_p=0.9, repetition=1.1)
    mask = pack_mask(allow)
    s, e = sharded.shard_range(V, rank, world)
    hid, hoff = (torch.from_numpy(a).to(dev) for a in csr(hist))
    xs = x[:, s:e].contiguous().to(dev)
    ms = torch.from_numpy(mask[:, s // 32:(e + 31) // 32].copy().view(np.int32)).to(dev)
    peer = os.environ.get("DLLM_TEST_EXCHANGE") == "peer"
    px = sharded.PeerExchange(rows, 64, dev) if peer else None
    ok = True
    # three steps with different uniforms (the peer exchange alternates its two slots)
    for step in range(3):
        us = np.roll(uni, step).copy()
        ut = torch.from_numpy(us).to(dev)
        if peer:
            st = torch.full((rows,), -1, dtype=torch.int32, device=dev)
            tok = px.sample(xs, s, V, ut, params, mask_shard=ms, hist_ids=hid, hist_off=hoff, hist_max=128, status=st)
            ok &= bool((st == 0).all().item())
        else:
            tok = sharded.sample_vocab_sharded(xs, s, V, ut, params, k=64, mask_shard=ms, hist_ids=hid, hist_off=hoff)
        allt = [torch.empty_like(tok) for _ in range(world)]
        dist.all_gather(allt, tok)
        same = all(torch.equal(allt[0], t) for t in allt)
        if rank == 0:
            ora = O.sample_restated(x.float().numpy(), params, us, mask=mask, hist=hist, kept_cap=64, topk_cap=64)
            t = tok.cpu().numpy()
            bad = [r for r in range(rows) if not ids_match(int(t[r]), ora, us, r)]
            if not (same and not bad):
                ok = False
                print("MISMATCH step", step, "same-on-all-ranks", same, "bad rows", bad[:8], flush=True)
    if px is not None:
        px.close()
    if rank == 0 and ok:
        print("SHARDED_NCCL_OK", flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
