"""Seeded synthetic inputs for the five sampler configurations.

No public dataset exists for this path: the inputs ARE the synthetic rows described by the
benchmark configurations (shapes, value distributions, history and mask statistics), with a
fixed seed per configuration.  Uniforms come from Philox4x32-10 (Salmon et al., "Parallel
random numbers: as easy as 1, 2, 3", SC'11), implemented here from the paper: 10 rounds of
two 32x32->64-bit multiplies with the published round multipliers and Weyl key increments;
a uniform is (x0 >> 8) * 2^-24 of the first output word.

Logits and histories are drawn with torch generators on the target device (the same
generator seed gives the same rows on any B200); `scale` shrinks the vocabulary / batch for
CPU-sized parity tests while keeping the distributions.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

PHILOX_M0 = np.uint64(0xD2511F53)
PHILOX_M1 = np.uint64(0xCD9E8D57)
PHILOX_W0 = np.uint32(0x9E3779B9)
PHILOX_W1 = np.uint32(0xBB67AE85)
_MASK32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(counter: np.ndarray, key: tuple[int, int]) -> np.ndarray:
    """counter: uint32 [n, 4]; returns uint32 [n, 4]."""
    c = counter.astype(np.uint32).copy()
    k0 = np.uint32(key[0] & 0xFFFFFFFF)
    k1 = np.uint32(key[1] & 0xFFFFFFFF)
    with np.errstate(over="ignore"):
        for _ in range(10):
            p0 = c[:, 0].astype(np.uint64) * PHILOX_M0
            p1 = c[:, 2].astype(np.uint64) * PHILOX_M1
            hi0 = (p0 >> np.uint64(32)).astype(np.uint32)
            lo0 = (p0 & _MASK32).astype(np.uint32)
            hi1 = (p1 >> np.uint64(32)).astype(np.uint32)
            lo1 = (p1 & _MASK32).astype(np.uint32)
            c = np.stack([hi1 ^ c[:, 1] ^ k0, lo1, hi0 ^ c[:, 3] ^ k1, lo0], axis=1)
            k0 = np.uint32(k0 + PHILOX_W0)
            k1 = np.uint32(k1 + PHILOX_W1)
    return c


def philox_uniforms(seed: int, n: int, step: int = 0) -> np.ndarray:
    """n uniforms in [0, 1) (multiples of 2^-24): counter (i, step, 0, 0), key (seed lo, hi)."""
    ctr = np.zeros((n, 4), dtype=np.uint32)
    ctr[:, 0] = np.arange(n, dtype=np.uint64).astype(np.uint32)
    ctr[:, 1] = np.uint32(step)
    out = philox4x32_10(ctr, (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF))
    return ((out[:, 0] >> np.uint32(8)).astype(np.float64) * 2.0 ** -24).astype(np.float32)


@dataclass
class Workload:
    name: str
    rows: int
    vocab: int
    dtype: str                      # "f32" | "bf16"
    params: dict
    logits: object                  # torch tensor [rows, vocab]
    uniforms: object                # torch float32 [rows]
    hist_ids: object = None         # torch int32
    hist_off: object = None         # torch int64 [rows+1]
    hist_max: int = 0
    mask: object = None             # torch int32 [rows, (vocab+31)//32]
    steps: int = 1
    algo_bytes_per_row: int = 0
    notes: dict = field(default_factory=dict)


def _gen(device, seed):
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _hist_uniform(rows, hlen, vocab, device, g):
    import torch

    ids = torch.randint(0, vocab, (rows * hlen,), generator=g, device=device, dtype=torch.int64)
    off = torch.arange(0, rows + 1, device=device, dtype=torch.int64) * hlen
    return ids.to(torch.int32), off


def _zipf_ranks(n, s, vmax, g, device):
    """ranks in [0, vmax) with P(rank=k) ~ 1/(k+1)^s (inverse CDF on the truncated law)."""
    import torch

    k = torch.arange(1, vmax + 1, device=device, dtype=torch.float64)
    cdf = torch.cumsum(k.pow(-s), 0)
    cdf = cdf / cdf[-1]
    u = torch.rand(n, generator=g, device=device, dtype=torch.float64)
    return torch.searchsorted(cdf, u).clamp_(max=vmax - 1)


def _algo_bytes(vocab, elem, mask_words, hlen):
    return vocab * elem + mask_words * 4 + hlen * 4


def _pack_bits(allow):
    import torch

    rows, n = allow.shape
    W = n // 32
    bits = allow.reshape(rows, W, 32).to(torch.int64)
    weights = torch.ones(32, dtype=torch.int64, device=allow.device) << torch.arange(32, device=allow.device)
    words = (bits * weights).sum(-1)
    return torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32)


def config1(device="cuda", scale=1.0, seed=101):
    """Single row, vocab 128256, N(0, 2.5^2) + 20 ids boosted by +8; 64-id history,
    repetition 1.1, T 0.8, top-k 40, top-p 0.95; 1000 sequential steps."""
    import torch

    V = max(256, int(128256 * scale))
    g = _gen(device, seed)
    x = torch.randn(1, V, generator=g, device=device) * 2.5
    boost = torch.randperm(V, generator=g, device=device)[:20]
    x[0, boost] += 8.0
    hid, hoff = _hist_uniform(1, 64, V, device, g)
    u = torch.from_numpy(philox_uniforms(seed, 1)).to(device)
    return Workload("cfg1_single_row_v128256", 1, V, "f32",
                    dict(temperature=0.8, top_k=40, top_p=0.95, repetition=1.1),
                    x, u, hid, hoff, 64, steps=1000, algo_bytes_per_row=_algo_bytes(V, 4, 0, 64))


def config2(device="cuda", scale=1.0, seed=202, rows=64):
    """Batch 64 x vocab 151936 N(0, 3^2) + per-row Zipf(1.1) spike profile over a random
    permutation; 512-id Zipf(1.2) histories; rep 1.1, freq 0.3, pres 0.2, T 0.7, k 50, p 0.9."""
    import torch

    V = max(256, int(151936 * scale))
    B = rows
    g = _gen(device, seed)
    x = torch.randn(B, V, generator=g, device=device) * 3.0
    ranks = torch.arange(1, V + 1, device=device, dtype=torch.float32)
    profile = 12.0 * ranks.pow(-1.1)
    for b in range(B):
        perm = torch.randperm(V, generator=g, device=device)
        x[b, perm] += profile
    H = 512
    ids = []
    for b in range(B):
        perm = torch.randperm(V, generator=g, device=device)
        ids.append(perm[_zipf_ranks(H, 1.2, V, g, device)])
    hid = torch.stack(ids).reshape(-1).to(torch.int32)
    hoff = torch.arange(0, B + 1, device=device, dtype=torch.int64) * H
    u = torch.from_numpy(philox_uniforms(seed, B)).to(device)
    return Workload("cfg2_qwen_b64_v151936", B, V, "f32",
                    dict(temperature=0.7, top_k=50, top_p=0.9, repetition=1.1, frequency=0.3,
                         presence=0.2),
                    x, u, hid, hoff, H, algo_bytes_per_row=_algo_bytes(V, 4, 0, H))


def json_mask(rows, V, g, device, frac=0.02, ranges=8, single_rows=()):
    """allow-bitmask with ~frac allowed: `ranges` random contiguous id ranges plus uniform
    scatter; rows listed in single_rows allow exactly one id."""
    import torch

    W = (V + 31) // 32
    allow = torch.zeros(rows, W * 32, dtype=torch.bool, device=device)
    per_range = max(1, int(V * frac * 0.5 / ranges))
    for b in range(rows):
        starts = torch.randint(0, max(1, V - per_range), (ranges,), generator=g, device=device)
        for s in starts.tolist():
            allow[b, s:s + per_range] = True
    allow[:, :V] |= torch.rand(rows, V, generator=g, device=device) < frac * 0.5
    for b in single_rows:
        allow[b] = False
        allow[b, int(torch.randint(0, V, (1,), generator=g, device=device))] = True
    allow[:, V:] = False
    return _pack_bits(allow)


def config3(device="cuda", scale=1.0, seed=303, rows=256):
    """JSON mode: batch 256 x vocab 151936 N(0, 2^2), ~2% allowed (8 ranges + scatter), some
    rows with exactly one allowed id; T 1.0, top-k off, top-p 0.95."""
    import torch

    V = max(256, int(151936 * scale))
    B = rows
    g = _gen(device, seed)
    x = torch.randn(B, V, generator=g, device=device) * 2.0
    singles = tuple(range(0, B, 37))
    m = json_mask(B, V, g, device, single_rows=singles)
    u = torch.from_numpy(philox_uniforms(seed, B)).to(device)
    return Workload("cfg3_json_mask_b256_v151936", B, V, "f32",
                    dict(temperature=1.0, top_k=0, top_p=0.95),
                    x, u, mask=m, algo_bytes_per_row=_algo_bytes(V, 4, (V + 31) // 32, 0),
                    notes={"single_allowed_rows": list(singles)})


def config4(device="cuda", scale=1.0, seed=404, rows=1024):
    """Worst-case nucleus: batch 1024 x vocab 256000 flat N(0, 0.5^2), top-k 0, top-p 0.99,
    repetition 1.05 over 256 uniform ids; T 1.0."""
    import torch

    V = max(256, int(256000 * scale))
    B = rows
    g = _gen(device, seed)
    x = torch.randn(B, V, generator=g, device=device) * 0.5
    hid, hoff = _hist_uniform(B, 256, V, device, g)
    u = torch.from_numpy(philox_uniforms(seed, B)).to(device)
    return Workload("cfg4_nucleus_b1024_v256000", B, V, "f32",
                    dict(temperature=1.0, top_k=0, top_p=0.99, repetition=1.05),
                    x, u, hid, hoff, 256, algo_bytes_per_row=_algo_bytes(V, 4, 0, 256))


def config5(device="cuda", scale=1.0, seed=505, rows=512):
    """Vocab-parallel: batch 512 x vocab 262144 bf16 N(0, 2^2), 10% uniformly allowed,
    repetition 1.1 over 128 ids; T 0.9, top-k 64 per shard + global merge, top-p 0.9."""
    import torch

    V = max(1024, int(262144 * scale))
    B = rows
    g = _gen(device, seed)
    x = (torch.randn(B, V, generator=g, device=device) * 2.0).to(torch.bfloat16)
    W = (V + 31) // 32
    allow = torch.rand(B, W * 32, generator=g, device=device) < 0.10
    allow[:, V:] = False
    words = _pack_bits(allow)
    hid, hoff = _hist_uniform(B, 128, V, device, g)
    u = torch.from_numpy(philox_uniforms(seed, B)).to(device)
    return Workload("cfg5_vocab_parallel_b512_v262144_bf16", B, V, "bf16",
                    dict(temperature=0.9, top_k=64, top_p=0.9, repetition=1.1),
                    x, u, hid, hoff, 128, mask=words,
                    algo_bytes_per_row=_algo_bytes(V, 2, W, 128))


CONFIGS = {1: config1, 2: config2, 3: config3, 4: config4, 5: config5}


def hist_lists(w: Workload):
    """history as a list of numpy arrays (for the CPU checkers)."""
    if w.hist_ids is None:
        return None
    ids = w.hist_ids.cpu().numpy()
    off = w.hist_off.cpu().numpy()
    return [ids[off[i]:off[i + 1]] for i in range(w.rows)]
