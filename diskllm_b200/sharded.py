"""Vocabulary-sharded sampling across GPUs (the tensor-parallel LM-head layout): each rank holds
columns [rank * Vs, (rank + 1) * Vs) of every row.  One exchange step:

    local candidates (k best per row on this shard, after mask and penalties)
      -> all-gather over the process group (NCCL over NVLink on B200 nodes)
      -> merge on every rank (global max, t = (v - M) / T, top-k by (t desc, id asc), softmax,
         min-p, top-p, fp32 draw with the row's uniform)

The reference sampler (src/sampler.c:136-234) sees whole rows; these tokens equal its tokens for
rows with 0 < top_k <= k.  Every rank computes the same tokens.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import capi


def _all_gather(out: torch.Tensor, inp: torch.Tensor, group) -> None:
    """all_gather_into_tensor that reports a failed exchange (a rank that died, a timed-out or
    aborted communicator) as a DllmError instead of the backend's exception type."""
    try:
        dist.all_gather_into_tensor(out, inp, group=group)
    except Exception as e:  # the backends raise RuntimeError / DistBackendError subclasses
        raise capi.DllmError(f"all-gather of shard candidates failed: {e}") from e


def gather_candidates(vals: torch.Tensor, ids: torch.Tensor, group=None) -> tuple[torch.Tensor, torch.Tensor]:
    """All-gathers this rank's [rows][k] candidates into [world][rows][k] (rank order)."""
    world = dist.get_world_size(group)
    rows, k = vals.shape
    # concatenated along rows (the layout every backend accepts), viewed as [world][rows][k]
    out_v = torch.empty((world * rows, k), dtype=vals.dtype, device=vals.device)
    out_i = torch.empty((world * rows, k), dtype=ids.dtype, device=ids.device)
    _all_gather(out_v, vals.contiguous(), group)
    _all_gather(out_i, ids.contiguous(), group)
    return out_v.view(world, rows, k), out_i.view(world, rows, k)


def candidate_buffer(rows: int, k: int, device) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """One int32 buffer [2][rows][k] holding a rank's candidate values (float32 bits) then ids, so
    one all-gather moves both.  Returns (buffer, values view, ids view)."""
    buf = torch.empty(2 * rows * k, dtype=torch.int32, device=device)
    return buf, buf[:rows * k].view(torch.float32).view(rows, k), buf[rows * k:].view(rows, k)


def gather_packed(buf: torch.Tensor, rows: int, k: int, group=None) -> tuple[torch.Tensor, torch.Tensor]:
    """All-gathers every rank's candidate_buffer with one collective and returns the values
    [world][rows][k] float32 and ids [world][rows][k] int32, contiguous, in rank order."""
    world = dist.get_world_size(group)
    allb = torch.empty(world * 2 * rows * k, dtype=torch.int32, device=buf.device)
    _all_gather(allb, buf, group)
    allb = allb.view(world, 2, rows, k)
    return allb[:, 0].contiguous().view(torch.float32), allb[:, 1].contiguous()


def shard_range(vocab_total: int, rank: int, world: int) -> tuple[int, int]:
    """Columns [start, end) of `rank` when vocab_total is split into `world` equal shards whose
    boundaries fall on mask words (multiples of 32)."""
    per = -(-vocab_total // world)
    per = -(-per // 32) * 32
    start = min(vocab_total, rank * per)
    return start, min(vocab_total, start + per)


def sample_vocab_sharded(logits_shard: torch.Tensor, vocab_offset: int, vocab_total: int,
                         uniforms: torch.Tensor, params: dict, *, k: int | None = None, mask_shard=None,
                         hist_ids=None, hist_off=None, hist_max=None, group=None) -> torch.Tensor:
    """Samples one token per row; call on every rank of `group` with that rank's shard.  `mask_shard`
    holds the mask words of this shard's columns ([rows][ceil(Vs/32)] int32, bit i&31 of word i>>5
    allows local column i); history ids are global.  Returns int32 [rows] (identical on all ranks)."""
    k = int(k if k is not None else params.get("top_k", 0))
    if not (0 < int(params.get("top_k", 0)) <= k):
        raise ValueError("vocabulary-sharded sampling needs 0 < top_k <= k")
    rows = logits_shard.shape[0]
    distributed = group is not None or (dist.is_available() and dist.is_initialized())
    if distributed:
        buf, vals, ids = candidate_buffer(rows, k, logits_shard.device)
        capi.shard_candidates(logits_shard, vocab_offset, vocab_total, k, params, mask=mask_shard,
                              hist_ids=hist_ids, hist_off=hist_off, hist_max=hist_max, out=(vals, ids))
        all_v, all_i = gather_packed(buf, rows, k, group)
        return capi.merge_sample(all_v, all_i, uniforms, params)
    vals, ids = capi.shard_candidates(logits_shard, vocab_offset, vocab_total, k, params, mask=mask_shard,
                                      hist_ids=hist_ids, hist_off=hist_off, hist_max=hist_max)
    return capi.merge_sample(vals.unsqueeze(0), ids.unsqueeze(0), uniforms, params)


class PeerExchange:
    """The NVLink peer exchange for vocabulary-sharded sampling, one per (rows, k) on every rank of
    `group`: each rank's candidate kernel stores its rows' candidates straight into every rank's
    buffer (CUDA IPC mappings exchanged once through the process group), so no collective runs on
    the data path.  Steps must run on every rank, in the same order."""

    def __init__(self, rows: int, k: int, device, group=None):
        self.rows, self.k, self.group = int(rows), int(k), group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.local, handle = capi.peer_exchange_create(self.rows, self.k, self.world)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self.mapped = []
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(self.local)
            else:
                p = capi.peer_exchange_open(h)
                self.mapped.append(p)
                ptrs.append(p)
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=device)
        self.epoch = 0
        self._key = self._desc = self._prm = None
        dist.barrier(group=group)  # every rank has mapped every buffer before any store

    def sample(self, logits_shard, vocab_offset, vocab_total, uniforms, params, *, mask_shard=None, hist_ids=None,
               hist_off=None, hist_max=None, token=None, status=None):
        """One step: this rank's candidates into every buffer, then the merge on this rank.  The
        batch descriptor and the parameters are built once and kept while the tensors and settings
        of later steps are the same (a decode loop over fixed buffers), so a step costs two
        library calls on the host."""
        ptr = lambda t: 0 if t is None else t.data_ptr()
        pkey = tuple(sorted(params.items())) if isinstance(params, dict) else id(params)
        key = (ptr(logits_shard), tuple(logits_shard.shape), tuple(logits_shard.stride()), logits_shard.dtype,
               int(vocab_offset), int(vocab_total), ptr(mask_shard), ptr(hist_ids), ptr(hist_off), hist_max,
               ptr(uniforms), pkey)
        if key != self._key:
            prm = capi.make_params(**params) if isinstance(params, dict) else params
            desc, _ = capi.fill_desc(logits_shard, uniforms, prm, mask=mask_shard, hist_ids=hist_ids,
                                     hist_off=hist_off, hist_max=hist_max)
            self._key, self._desc, self._prm = key, desc, prm
        if token is None:
            token = torch.empty(self.rows, dtype=torch.int32, device=uniforms.device)
        stream = torch.cuda.current_stream(uniforms.device).cuda_stream
        self.epoch += 1
        capi.shard_candidates_peer_desc(self._desc, vocab_offset, vocab_total, self.k, self.peers, self.rank,
                                        self.world, self.epoch, stream)
        return capi.merge_sample_peer(self.rows, self.world, self.k, self.local, self.epoch, uniforms, self._prm,
                                      token=token, status=status, stream=stream)

    def close(self):
        torch.cuda.synchronize()
        dist.barrier(group=self.group)  # no rank stores into a buffer being unmapped
        lib = capi.load_library()
        for p in self.mapped:
            lib.dllm_cuda_peer_exchange_close(p)
        lib.dllm_cuda_peer_exchange_free(self.local)
        self.mapped = []
