// dllm_shard.cu -- vocabulary-sharded sampling (a row's logits split over N GPUs, the
// tensor-parallel LM-head layout).  The path has one exchange step:
//
//   1. dllm_cuda_shard_candidates: on each GPU, one CTA per (8192-column chunk, row) applies the
//      grammar mask and the history penalties to its columns, stages them as order-preserving
//      keys in shared memory and selects the chunk's k best by (value desc, id asc) with a 4-pass
//      radix select; a second kernel selects each row's k best of its chunks' candidates.
//      Output (value, global id), sorted, [rows][k].
//   2. The caller all-gathers the candidates ([N][rows][k], NCCL over NVLink).
//   3. dllm_cuda_merge_sample: one CTA per row takes the row maximum over the N*k candidates,
//      forms t = (v - M) * (1/T) like the reference (src/sampler.c:144-162), keeps the k best by
//      (t desc, id asc) (src/sampler.c:109-134) and draws from that sorted list with the same
//      softmax / min-p / top-p / fp32 draw code as the fused kernel (src/sampler.c:172-233).
//
// Every GPU that runs the merge on the gathered candidates gets the same tokens.
//
// Selecting on v inside a shard equals selecting on t whenever distinct values keep distinct t;
// for temperature 1 and row maxima within a binade of the values that holds, and the parity tests
// compare against the whole-row reference to catch any difference.
#include <cuda_runtime.h>
#include <stdlib.h>

#include <mutex>
#include <vector>

#include "dllm_chunk.cuh"

namespace dllm {
namespace {

constexpr int SH_T = 256;        // threads per CTA
constexpr int SH_CHUNK = 8192;   // columns per CTA (keys staged in shared memory)
constexpr int SH_KMAX = 256;     // largest k per shard

struct ShardArgs {
    const void *logits;
    int64_t row_stride;
    int dtype;
    const uint32_t *mask;
    int64_t mask_stride;
    const int32_t *hist_ids;
    const int64_t *hist_off;
    dllm_sampler_params bparams;
    const dllm_sampler_params *rparams;
    int rows, vlocal, k, nchunks;
    int64_t voff, vtotal;
    unsigned flags;
    float *cand_val;       // final [rows][k]
    int32_t *cand_id;
    uint32_t *part_key;    // per-chunk candidates [rows][nchunks][k] when nchunks > 1
    int32_t *part_id;
    int32_t *status;
    unsigned long long *dbg;  // diagnostic counters (shard_stream_kernel phase cycles) or null
    // peer exchange (null: write cand_val / cand_id): every rank's exchange buffer, mapped here
    unsigned char *const *peers;
    int p_rank, p_world, p_slot;
};

// Peer exchange buffer, one per rank (allocated by dllm_cuda_peer_exchange_create):
//   [0, 256)            arrival counters, uint64 [world]: rank r's candidate CTAs add 1 per row
//   then two slots      values float [world][rows][k], then ids int32 [world][rows][k]
// Step e uses slot e & 1 and is complete on a rank when every counter reaches e * rows.
constexpr size_t PX_HDR = 256;
constexpr int PX_MAX_WORLD = 32;
__host__ __device__ inline size_t px_slot_bytes(int world, int rows, int k) { return (size_t)world * rows * k * 8; }
__host__ __device__ inline float *px_vals(unsigned char *base, int slot, int world, int rows, int k) {
    return reinterpret_cast<float *>(base + PX_HDR + (size_t)slot * px_slot_bytes(world, rows, k));
}
__host__ __device__ inline int32_t *px_ids(unsigned char *base, int slot, int world, int rows, int k) {
    return reinterpret_cast<int32_t *>(base + PX_HDR + (size_t)slot * px_slot_bytes(world, rows, k) +
                                       (size_t)world * rows * k * 4);
}

// diagnostic counter slots of shard_stream_kernel (thread 0 of each row CTA adds its cycles)
enum : int { SDBG_ROWS = 0, SDBG_LOOP = 1, SDBG_CUT = 2, SDBG_NCUT = 3, SDBG_FINAL = 4, SDBG_UNION = 5 };
// and of merge_sample_kernel: rows, cycles to the transformed candidates, ranking, draw, and rows
// that compared every pair
enum : int { MDBG_ROWS = 8, MDBG_LOAD = 9, MDBG_RANK = 10, MDBG_DRAW = 11, MDBG_PAIRWISE = 12 };

constexpr int SH_SURV = 1024;    // survivors of the threshold pre-filter kept for the exact select

struct SelScratch {
    unsigned hist[256];
    uint32_t ck[SH_KMAX];
    int cid[SH_KMAX];
    int wsum[SH_T / 32];
    uint32_t wv[SH_T / 32];
    int bin, above, ncand;
    uint32_t thr;
    int nsurv;
    int ntie;
};

// Appends to s.ck / s.cid (from s.ncand) the `need` entries equal to `target` with the lowest ids.
// Without ids (ids grow with position) each warp scans a contiguous segment with ballots, twice:
// once to count, once to rank against the earlier segments' counts.  With ids, ranks by counting.
__device__ void select_ties(const uint32_t *keys, const int *ids, int id0, int n, uint32_t target, int need, int cap,
                            SelScratch &s) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, NT = blockDim.x, NW = NT >> 5;
    if (need <= 0) return;
    if (ids) {
        // the tied entries' ids in a short list (s.hist is free once the radix passes are done),
        // then each ranked among the tied ones only
        if (tid == 0) s.ntie = 0;
        __syncthreads();
        for (int i = tid; i < n; i += NT)
            if (keys[i] == target) {
                const int at = atomicAdd(&s.ntie, 1);
                if (at < 256) s.hist[at] = (unsigned)ids[i];
            }
        __syncthreads();
        const int nt = s.ntie;
        if (nt <= 256) {
            for (int j = tid; j < nt; j += NT) {
                const int idj = (int)s.hist[j];
                int r = 0;
                for (int q = 0; q < nt; q++) r += (int)s.hist[q] < idj;
                if (r < need) {
                    const int pos = atomicAdd(&s.ncand, 1);
                    if (pos < cap) {
                        s.ck[pos] = target;
                        s.cid[pos] = idj;
                    }
                }
            }
            __syncthreads();
            return;
        }
        for (int i = tid; i < n; i += NT) {
            if (keys[i] != target) continue;
            int r = 0;
            for (int j = 0; j < n; j++) r += keys[j] == target && ids[j] < ids[i];
            if (r < need) {
                const int pos = atomicAdd(&s.ncand, 1);
                if (pos < cap) {
                    s.ck[pos] = target;
                    s.cid[pos] = ids[i];
                }
            }
        }
        __syncthreads();
        return;
    }
    const int seg = ((n + NW - 1) / NW + 31) & ~31;
    const int b0 = min(n, wid * seg), b1 = min(n, b0 + seg);
    int cnt = 0;
    for (int base = b0; base < b1; base += 32) {
        const int i = base + lane;
        cnt += __popc(__ballot_sync(0xffffffffu, i < b1 && keys[i] == target));
    }
    if (lane == 0) s.wsum[wid] = cnt;
    __syncthreads();
    int running = 0;
    for (int w = 0; w < wid; w++) running += s.wsum[w];
    for (int base = b0; base < b1 && running < need; base += 32) {
        const int i = base + lane;
        const bool eq = i < b1 && keys[i] == target;
        const unsigned bm = __ballot_sync(0xffffffffu, eq);
        const int rank = running + __popc(bm & ((1u << lane) - 1u));
        if (eq && rank < need) {
            const int pos = atomicAdd(&s.ncand, 1);
            if (pos < cap) {
                s.ck[pos] = target;
                s.cid[pos] = id0 + i;
            }
        }
        running += __popc(bm);
    }
    __syncthreads();
}

// Order keys of bf16 values (exact fp32 upcasts) have their low 16 bits fixed by the sign: 0 for
// a positive value, 0xffff for a negative one (the key of a negative float is its complement), so
// a radix select over them needs only the two high bytes.  Completes a key from its high half.
__device__ __forceinline__ uint32_t bf16_key_low(uint32_t hi_prefix) {
    return hi_prefix | ((hi_prefix & 0x80000000u) ? 0u : 0xffffu);
}

// The K-th largest of the finite (above -inf) keys among n in shared memory, by four 8-bit radix
// passes (the same passes block_select runs); 0 when fewer than K keys are finite.  Ends with a
// barrier; every thread gets the result.
__device__ uint32_t radix_kth(const uint32_t *keys, int n, int K, SelScratch &s, bool bf16_keys) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, NT = blockDim.x, NW = NT >> 5;
    const uint32_t KNEG = okey(-INFINITY);
    int nf = 0;
    for (int base = 0; base < n; base += NT) {
        const int i = base + tid;
        nf += __popc(__ballot_sync(0xffffffffu, i < n && keys[i] > KNEG));
    }
    if (lane == 0) s.wsum[wid] = nf;
    __syncthreads();
    nf = 0;
    for (int w = 0; w < NW; w++) nf += s.wsum[w];
    if (nf < K || K <= 0) {
        __syncthreads();
        return 0u;
    }
    uint32_t prefix = 0u, pmask = 0u;
    int remaining = K;
    for (int pass = 3; pass >= (bf16_keys ? 2 : 0); pass--) {
        for (int i = tid; i < 256; i += NT) s.hist[i] = 0u;
        __syncthreads();
        const int sh = 8 * pass;
        for (int i = tid; i < n; i += NT) {
            const uint32_t key = keys[i];
            if (key > KNEG && (key & pmask) == prefix) atomicAdd(&s.hist[(key >> sh) & 255u], 1u);
        }
        __syncthreads();
        if (wid == 0) {
            unsigned c[8], tot = 0u;
#pragma unroll
            for (int b = 0; b < 8; b++) {
                c[b] = s.hist[255 - 8 * lane - b];
                tot += c[b];
            }
            unsigned incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const unsigned excl = incl - tot;
            if (excl < (unsigned)remaining && incl >= (unsigned)remaining) {
                unsigned acc = excl;
#pragma unroll
                for (int b = 0; b < 8; b++) {
                    if (acc + c[b] >= (unsigned)remaining) {
                        s.bin = 255 - 8 * lane - b;
                        s.above = (int)acc;
                        break;
                    }
                    acc += c[b];
                }
            }
        }
        __syncthreads();
        prefix |= (uint32_t)s.bin << sh;
        pmask |= 255u << sh;
        remaining -= s.above;
        __syncthreads();
    }
    return bf16_keys ? bf16_key_low(prefix) : prefix;
}

// The K best of n keys in shared memory by (key desc, id asc), written sorted to out_key / out_id
// (K entries; positions past n, when n < K, get key 0 and id INT_MAX, which rank last).
// Masked entries (-inf) are left out of the radix select of the K-th key (8 bits per pass from
// the top) and taken, lowest ids first, only when fewer than K entries are finite.  Ids: ids[i],
// or id0 + i when ids is null (then ids grow with position).
__device__ void block_select(const uint32_t *keys, const int *ids, int id0, int n, int K, SelScratch &s,
                             uint32_t *out_key, int *out_id, bool bf16_keys = false) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, NT = blockDim.x, NW = NT >> 5;
    const uint32_t KNEG = okey(-INFINITY);
    const int Kn = min(K, n);
    // entries above -inf
    int nf = 0;
    for (int base = 0; base < n; base += NT) {
        const int i = base + tid;
        nf += __popc(__ballot_sync(0xffffffffu, i < n && keys[i] > KNEG));
    }
    if (lane == 0) s.wsum[wid] = nf;
    __syncthreads();
    nf = 0;
    for (int w = 0; w < NW; w++) nf += s.wsum[w];
    if (tid == 0) s.ncand = 0;
    __syncthreads();
    const int Kf = min(Kn, nf);
    uint32_t prefix = 0u, pmask = 0u;
    int remaining = Kf;
    unsigned cnt_eq = 0u;
    for (int pass = 3; pass >= (bf16_keys ? 2 : 0) && Kf > 0; pass--) {
        for (int i = tid; i < 256; i += NT) s.hist[i] = 0u;
        __syncthreads();
        const int sh = 8 * pass;
        for (int i = tid; i < n; i += NT) {
            const uint32_t key = keys[i];
            if (key > KNEG && (key & pmask) == prefix) atomicAdd(&s.hist[(key >> sh) & 255u], 1u);
        }
        __syncthreads();
        if (wid == 0) {
            // lane l holds bins 255-8l .. 248-8l, scanned from the top
            unsigned c[8], tot = 0u;
#pragma unroll
            for (int b = 0; b < 8; b++) {
                c[b] = s.hist[255 - 8 * lane - b];
                tot += c[b];
            }
            unsigned incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const unsigned excl = incl - tot;
            if (excl < (unsigned)remaining && incl >= (unsigned)remaining) {
                unsigned acc = excl;
#pragma unroll
                for (int b = 0; b < 8; b++) {
                    if (acc + c[b] >= (unsigned)remaining) {
                        s.bin = 255 - 8 * lane - b;
                        s.above = (int)acc;
                        break;
                    }
                    acc += c[b];
                }
            }
        }
        __syncthreads();
        prefix |= (uint32_t)s.bin << sh;
        pmask |= 255u << sh;
        remaining -= s.above;
        cnt_eq = s.hist[s.bin];
        __syncthreads();
    }
    if (Kf > 0) {
        const uint32_t kstar = bf16_keys ? bf16_key_low(prefix) : prefix;
        const bool all_eq = cnt_eq == (unsigned)remaining;
        for (int i = tid; i < n; i += NT) {
            const uint32_t key = keys[i];
            if (key > kstar || (key == kstar && all_eq)) {
                const int pos = atomicAdd(&s.ncand, 1);
                if (pos < Kn) {
                    s.ck[pos] = key;
                    s.cid[pos] = ids ? ids[i] : id0 + i;
                }
            }
        }
        __syncthreads();
        if (!all_eq) select_ties(keys, ids, id0, n, kstar, remaining, Kn, s);
    }
    // fewer finite entries than K: the lowest-id masked ones
    if (Kn > nf) select_ties(keys, ids, id0, n, KNEG, Kn - nf, Kn, s);
    __syncthreads();
    for (int i = tid; i < K; i += NT) {
        if (i >= Kn) {
            out_key[i] = 0u;
            out_id[i] = INT_MAX;
            continue;
        }
        const uint32_t ki = s.ck[i];
        const int ii = s.cid[i];
        int r = 0;
        for (int j = 0; j < Kn; j++) r += s.ck[j] > ki || (s.ck[j] == ki && s.cid[j] < ii);
        out_key[r] = ki;
        out_id[r] = ii;
    }
    __syncthreads();
}

// block_select behind a pre-filter.  The threads form Kp groups (Kp = K rounded up to a power of
// two, Kp <= blockDim.x); each group's largest key is a real entry, so at least Kp >= K entries
// hold a key >= thr = the smallest group maximum, and the K best entries by (key desc, id asc),
// ties at the K-th key included, all do.  Those survivors (typically a few hundred of 8192) are
// gathered into sk / sid and block_select runs on them alone.  When thr is the masked key (some
// group saw only masked or no entries) or more than `cap` entries survive, block_select runs on
// all n.  `tmax` is the largest key among the entries this thread produced (0 if none).
__device__ void thresh_select(const uint32_t *keys, const int *ids, int id0, int n, int K, uint32_t tmax,
                              SelScratch &s, uint32_t *sk, int *sid, int cap, uint32_t *out_key, int *out_id) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, NT = blockDim.x, NW = NT >> 5;
    int Kp = 1;
    while (Kp < K) Kp <<= 1;
    const int gs = NT / Kp;  // threads per group
    uint32_t g = tmax;
    for (int o = 1; o < gs && o < 32; o <<= 1) g = max(g, __shfl_xor_sync(0xffffffffu, g, o));
    uint32_t wmin = g;
    for (int o = 16; o; o >>= 1) wmin = min(wmin, __shfl_xor_sync(0xffffffffu, wmin, o));
    if (lane == 0) s.wv[wid] = gs <= 32 ? wmin : g;
    if (tid == 0) s.nsurv = 0;
    __syncthreads();
    if (tid == 0) {
        uint32_t thr = 0xffffffffu;
        if (gs <= 32) {
            for (int w = 0; w < NW; w++) thr = min(thr, s.wv[w]);
        } else {
            const int gw = gs / 32;  // warps per group
            for (int w0 = 0; w0 < NW; w0 += gw) {
                uint32_t gm = 0u;
                for (int w = w0; w < w0 + gw; w++) gm = max(gm, s.wv[w]);
                thr = min(thr, gm);
            }
        }
        s.thr = thr;
    }
    __syncthreads();
    const uint32_t thr = s.thr;
    if (thr > okey(-INFINITY) && K <= NT) {
        for (int base = 0; base < n; base += NT) {
            const int i = base + tid;
            const bool keep = i < n && keys[i] >= thr;
            const unsigned bm = __ballot_sync(0xffffffffu, keep);
            int pos0 = 0;
            if (lane == 0 && bm) pos0 = atomicAdd(&s.nsurv, __popc(bm));
            pos0 = __shfl_sync(0xffffffffu, pos0, 0);
            const int pos = pos0 + __popc(bm & ((1u << lane) - 1u));
            if (keep && pos < cap) {
                sk[pos] = keys[i];
                sid[pos] = ids ? ids[i] : id0 + i;
            }
        }
        __syncthreads();
        const int ns = s.nsurv;
        if (ns <= cap) {
            block_select(sk, sid, 0, ns, K, s, out_key, out_id);
            return;
        }
    }
    block_select(keys, ids, id0, n, K, s, out_key, out_id);
}

// One CTA per (chunk of up to SH_CHUNK columns, row): mask, penalties, keys in shared memory, the
// chunk's k best.  With one chunk per row they are the shard's final candidates.
template <int DT>
__global__ void __launch_bounds__(SH_T) shard_chunk_kernel(const ShardArgs a) {
    extern __shared__ __align__(16) uint32_t keys[];  // SH_CHUNK keys
    __shared__ int hkeys[CH_HTAB];
    __shared__ int hcnt[CH_HTAB];
    __shared__ uint32_t penbits[SH_CHUNK / 32];
    __shared__ SelScratch sel;
    __shared__ uint32_t okey_s[SH_KMAX];
    __shared__ int oid_s[SH_KMAX];
    __shared__ int s_flags;
    const int row = blockIdx.y, ch = blockIdx.x, tid = threadIdx.x, NT = blockDim.x;
    const int c0 = ch * SH_CHUNK, n = min(SH_CHUNK, a.vlocal - c0);
    const dllm_sampler_params p = a.rparams ? a.rparams[row] : a.bparams;

    if (tid == 0) s_flags = 0;
    // mask (grammar.c:275-308) and history penalties (sampler.c:21-52), as order-preserving keys
    ChunkPen cp{hkeys, hcnt, penbits, &s_flags, pen_active(a.hist_ids, a.hist_off, p)};
    const HistPre hp = hist_prefetch(a.hist_ids, a.hist_off, row, cp.active);
    chunk_pen_build(cp, a.hist_ids, hp, a.voff, a.vtotal, c0, n, SH_CHUNK / 32);
    const uint32_t *mrow = a.mask ? a.mask + (int64_t)row * a.mask_stride : nullptr;
    const size_t esz = DT == DLLM_DTYPE_BF16 ? 2 : 4;
    const unsigned char *src = (const unsigned char *)a.logits + ((int64_t)row * a.row_stride + c0) * esz;
    const bool vec = ((uintptr_t)src & 15u) == 0;
    uint32_t tmax = 0u;
    chunk_visit<DT>(src, vec, mrow, c0, n, cp, p, a.flags, [&](int li, float v) {
        const uint32_t key = okey(v);
        keys[li] = key;
        tmax = max(tmax, key);
    });
    __syncthreads();
    uint32_t *sk = keys + SH_CHUNK;
    int *sid = reinterpret_cast<int *>(sk + SH_SURV);
    thresh_select(keys, nullptr, c0, n, a.k, tmax, sel, sk, sid, SH_SURV, okey_s, oid_s);
    if (a.nchunks == 1) {
        for (int i = tid; i < a.k; i += NT) {
            a.cand_val[(int64_t)row * a.k + i] = okey_inv(okey_s[i]);
            a.cand_id[(int64_t)row * a.k + i] = (int32_t)(oid_s[i] + a.voff);
        }
    } else {
        const int64_t o = ((int64_t)row * a.nchunks + ch) * a.k;
        for (int i = tid; i < a.k; i += NT) {
            a.part_key[o + i] = okey_s[i];
            a.part_id[o + i] = oid_s[i];
        }
    }
    if (a.status && tid == 0 && s_flags) atomicOr(&a.status[row], s_flags);
}

// One CTA per row: the k best of the row's chunk candidates, as the shard's final candidates.
__global__ void __launch_bounds__(SH_T) shard_rowmerge_kernel(const ShardArgs a) {
    extern __shared__ __align__(16) unsigned char rdyn[];
    __shared__ SelScratch sel;
    __shared__ uint32_t okey_s[SH_KMAX];
    __shared__ int oid_s[SH_KMAX];
    const int row = blockIdx.x, tid = threadIdx.x, NT = blockDim.x;
    const int n = a.nchunks * a.k;
    uint32_t *keys = reinterpret_cast<uint32_t *>(rdyn);
    int *ids = reinterpret_cast<int *>(keys + n);
    uint32_t *sk = reinterpret_cast<uint32_t *>(ids + n);
    int *sid = reinterpret_cast<int *>(sk + SH_SURV);
    uint32_t tmax = 0u;
    for (int i = tid; i < n; i += NT) {
        const uint32_t key = a.part_key[(int64_t)row * n + i];
        keys[i] = key;
        ids[i] = a.part_id[(int64_t)row * n + i];
        tmax = max(tmax, key);
    }
    __syncthreads();
    thresh_select(keys, ids, 0, n, a.k, tmax, sel, sk, sid, SH_SURV, okey_s, oid_s);
    for (int i = tid; i < a.k; i += NT) {
        a.cand_val[(int64_t)row * a.k + i] = okey_inv(okey_s[i]);
        a.cand_id[(int64_t)row * a.k + i] = (int32_t)(oid_s[i] + a.voff);
    }
}

// One CTA per row streams all of the shard's columns once and keeps a running top-K' (K' = k + the
// history bound) of the raw masked values, by (value desc, id asc):
//  * candidates go to a shared-memory buffer; once the buffer has been cut to the best K' entries,
//    only keys strictly above the K'-th (thr) can enter (an equal key arrives with a larger id and
//    loses the tie), so after the first few tiles almost nothing is appended;
//  * the first tile's threshold comes from group maxima (at least K' entries reach it);
//  * one barrier per tile decides whether the buffer must be cut (to the entries at or above its
//    K'-th key);
// History penalties are applied afterwards, exactly: the true top-k is contained in (the K' best
// raw entries that are not history ids) united with (every history id of this shard, with its
// penalised value), because at most H of the K' best raw entries are history ids.  The buffer
// holds the K' best raw entries, so the union may take all of it when it fits.  The union is
// selected by (key desc, id asc) once more.  Used when k + the history bound <= SH_KMAX.
constexpr int ST_T = 256;          // threads per row CTA
constexpr int ST_U = 2;            // 16-byte vectors per thread per tile
constexpr int ST_PD = 6;           // tiles pulled into L2 ahead of the loads
constexpr int ST_CAP = 4608;       // candidate buffer entries
constexpr int ST_FIN = 2 * SH_KMAX;  // final union entries
static_assert(ST_FIN <= 2 * ST_T, "union_select sorts 2 * ST_T entries, two per thread");
// A cut leaves at most SH_KMAX entries and a tile appends at most one per column (8 per bf16
// vector), so the buffer never overflows when a tile starts at or below ST_CAP - E.
static_assert(ST_CAP >= ST_T * ST_U * 8 + SH_KMAX, "candidate buffer smaller than a tile plus a cut");

// Sorts 2 * blockDim.x (= 512) 64-bit values held two per thread (thread t holds positions 2t
// and 2t + 1) into descending order, and writes them to tmp[0, 512) as well.  Bitonic network:
// pairs closer than 64 apart are in one warp and are exchanged by shuffles, the stages with pairs
// 64 or more apart go through `tmp`.  Every thread of a 256-thread block must call it.
__device__ void sort_desc_2x(unsigned long long (&v)[2], unsigned long long *tmp) {
    const int tid = threadIdx.x, e0 = 2 * tid, NT2 = 2 * blockDim.x;
    auto reg_stages = [&](int k, int jtop) {
        for (int j = jtop; j >= 2; j >>= 1) {
#pragma unroll
            for (int r = 0; r < 2; r++) {
                const int e = e0 + r;
                const unsigned long long o = __shfl_xor_sync(0xffffffffu, v[r], j >> 1);
                const bool desc = ((e & ~j) & k) == 0;  // descending runs where bit k of the pair is clear
                const bool keep_max = ((e & j) == 0) == desc;
                v[r] = keep_max ? (v[r] > o ? v[r] : o) : (v[r] < o ? v[r] : o);
            }
        }
        const bool desc = (e0 & k) == 0;
        if ((v[0] < v[1]) == desc) {
            const unsigned long long t = v[0];
            v[0] = v[1];
            v[1] = t;
        }
    };
    for (int k = 2; k <= 64; k <<= 1) reg_stages(k, k >> 1);
    for (int k = 128; k <= NT2; k <<= 1) {
        tmp[e0] = v[0];
        tmp[e0 + 1] = v[1];
        __syncthreads();
        for (int j = k >> 1; j >= 64; j >>= 1) {
            const int i = tid;  // one pair per thread
            const int lo = ((i & ~(j - 1)) << 1) | (i & (j - 1)), hi = lo + j;
            const unsigned long long x = tmp[lo], y = tmp[hi];
            if (((lo & k) == 0) == (x < y)) {
                tmp[lo] = y;
                tmp[hi] = x;
            }
            __syncthreads();
        }
        v[0] = tmp[e0];
        v[1] = tmp[e0 + 1];
        reg_stages(k, 32);
        __syncthreads();  // every thread has read tmp before the next stores
    }
    tmp[e0] = v[0];
    tmp[e0 + 1] = v[1];
    __syncthreads();
}

// The K best of n <= ST_FIN entries by (key desc, id asc), written sorted to out_key / out_id
// like block_select: a bitonic sort in shared memory (`tmp`, ST_FIN entries of 8 bytes) of the
// composites key << 32 | ~id, whose descending order is exactly that ranking.  Keys below the
// -inf key (negative NaN) are never taken by block_select, which runs instead when one is present.
__device__ void union_select(const uint32_t *keys, const int *ids, int n, int K, unsigned long long *tmp,
                             SelScratch &s, uint32_t *out_key, int *out_id) {
    const int tid = threadIdx.x, NT = blockDim.x;
    const uint32_t KNEG = okey(-INFINITY);
    bool odd = false;
    for (int i = tid; i < n; i += NT) odd |= keys[i] < KNEG;
    if (__syncthreads_or(odd) || n > ST_FIN) {
        block_select(keys, ids, 0, n, K, s, out_key, out_id);
        return;
    }
    // 2 * ST_T composites (zero padding, which sorts last), two per thread
    const int e0 = 2 * tid;
    unsigned long long v[2];
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const int i = e0 + r;
        v[r] = i < n ? ((unsigned long long)keys[i] << 32) | (uint32_t)~(uint32_t)ids[i] : 0ull;
    }
    sort_desc_2x(v, tmp);
    // a real composite is never 0 (its low word ~id has the top bit set), so positions past n
    // are the padding, written as block_select writes them
    for (int i = tid; i < K; i += NT) {
        const unsigned long long c = i < n ? tmp[i] : 0ull;
        out_key[i] = i < n ? (uint32_t)(c >> 32) : 0u;
        out_id[i] = i < n ? (int)~(uint32_t)c : INT_MAX;
    }
    __syncthreads();
}

template <int DT>
__global__ void __launch_bounds__(ST_T, 4) shard_stream_kernel(const ShardArgs a, int kprime) {
    extern __shared__ __align__(16) unsigned char sdyn[];
    uint32_t *bk = reinterpret_cast<uint32_t *>(sdyn);   // [ST_CAP]
    int *bid = reinterpret_cast<int *>(bk + ST_CAP);      // [ST_CAP]
    uint32_t *fk = reinterpret_cast<uint32_t *>(bid + ST_CAP);  // [ST_FIN]
    int *fid = reinterpret_cast<int *>(fk + ST_FIN);             // [ST_FIN]
    int *hl = fid + ST_FIN;                                      // [SH_KMAX] history local ids
    int *hall = hl + SH_KMAX;                                    // [SH_KMAX] the row's history ids
    __shared__ SelScratch sel;
    __shared__ uint32_t okey_s[SH_KMAX];
    __shared__ int oid_s[SH_KMAX];
    __shared__ int s_nb, s_strict, s_nh;
    __shared__ uint32_t s_thr;
    constexpr int VEC = DT == DLLM_DTYPE_BF16 ? 8 : 4;
    constexpr int E = ST_T * ST_U * VEC;  // columns per tile
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, NT = blockDim.x;
    const int n = a.vlocal;
    const dllm_sampler_params p = a.rparams ? a.rparams[row] : a.bparams;
    const uint32_t *mrow = a.mask ? a.mask + (int64_t)row * a.mask_stride : nullptr;
    const size_t esz = DT == DLLM_DTYPE_BF16 ? 2 : 4;
    const unsigned char *src = (const unsigned char *)a.logits + (int64_t)row * a.row_stride * esz;
    const bool vec = ((uintptr_t)src & 15u) == 0;
    const int nv = vec ? (n & ~(VEC - 1)) : 0;
    const uint32_t KNEG = okey(-INFINITY);
    const bool pen = pen_active(a.hist_ids, a.hist_off, p);
    int64_t h0 = 0, h1 = 0;
    if (pen) {
        h0 = a.hist_off[row];
        h1 = a.hist_off[row + 1];
    }
    if (tid == 0) {
        s_nb = 0;
        s_strict = 0;
        s_thr = 0u;
    }
    // the row's history (at most SH_KMAX - k ids: the host checks k + the bound <= SH_KMAX)
    const int nhist = pen ? (int)(h1 - h0 < (int64_t)SH_KMAX ? h1 - h0 : (int64_t)SH_KMAX) : 0;
    for (int j = tid; j < nhist; j += NT) hall[j] = a.hist_ids[h0 + j];
    auto raw_at = [&](int li) -> float {
        const bool al = !mrow || ((mrow[li >> 5] >> (li & 31)) & 1u);
        return al ? chunk_raw(src, DT, li) : -INFINITY;
    };
    // the 16-byte vector at column i -> VEC keys (masked columns get the -inf key)
    auto vec_keys = [&](int i, const uint4 raw, uint32_t mword, uint32_t (&key)[VEC]) {
        const uint32_t mw = mword >> (i & 31);
        float x[VEC];
        if (DT == DLLM_DTYPE_BF16) {
            const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                x[2 * j] = bitsf(w4[j] << 16);
                x[2 * j + 1] = bitsf(w4[j] & 0xffff0000u);
            }
        } else {
            x[0] = bitsf(raw.x);
            x[1] = bitsf(raw.y);
            x[2] = bitsf(raw.z);
            x[3] = bitsf(raw.w);
        }
#pragma unroll
        for (int j = 0; j < VEC; j++) key[j] = ((mw >> j) & 1u) ? okey(x[j]) : KNEG;
    };
    // appends this thread's passing keys (bit j of m) of the vector at column i
    auto append = [&](int i, const uint32_t (&key)[VEC], unsigned m) {
        const int c = __popc(m);
        int incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        int base = 0;
        if (lane == 31 && incl) base = atomicAdd(&s_nb, incl);
        base = __shfl_sync(0xffffffffu, base, 31) + incl - c;
#pragma unroll
        for (int j = 0; j < VEC; j++)
            if ((m >> j) & 1u) {
                if (base < ST_CAP) {
                    bk[base] = key[j];
                    bid[base] = i + j;
                }
                base++;
            }
    };
    // cuts the buffer to its best kprime entries (sorted); later keys must beat the K'-th
    long long t_cut = 0;
    auto cut = [&]() {
        const long long tc0 = a.dbg ? clock64() : 0;
        const int nb = min(s_nb, ST_CAP);
        // Fast cut: the K'-th largest key kstar, and every entry with key >= kstar kept, in any
        // order.  At least K' entries remain at or above kstar, so a later key equal to kstar
        // (larger id) can no longer reach the K' best: later keys must beat kstar strictly.  The
        // final union select orders what is kept.  The full select (below) handles buffers with
        // fewer than K' finite keys, or more ties at kstar than the compaction area holds.
        const uint32_t kstar = radix_kth(bk, nb, kprime, sel, DT == DLLM_DTYPE_BF16);
        if (kstar != 0u) {
            if (tid == 0) sel.ncand = 0;
            __syncthreads();
            for (int base = 0; base < nb; base += NT) {
                const int i = base + tid;
                const bool keep = i < nb && bk[i] >= kstar;
                const unsigned m = __ballot_sync(0xffffffffu, keep);
                int pos = 0;
                if (lane == 0 && m) pos = atomicAdd(&sel.ncand, __popc(m));
                pos = __shfl_sync(0xffffffffu, pos, 0) + __popc(m & ((1u << lane) - 1u));
                if (keep && pos < ST_FIN) {
                    fk[pos] = bk[i];
                    fid[pos] = bid[i];
                }
            }
            __syncthreads();
            const int kept = sel.ncand;
            // at most SH_KMAX kept, so that the final union (kept raw entries plus at most
            // SH_KMAX - k history entries) fits the ST_FIN union area
            if (kept <= ST_FIN - SH_KMAX) {
                for (int i = tid; i < kept; i += NT) {
                    bk[i] = fk[i];
                    bid[i] = fid[i];
                }
                __syncthreads();
                if (tid == 0) {
                    s_nb = kept;
                    s_thr = kstar;
                    s_strict = 1;
                }
                __syncthreads();
                if (a.dbg && tid == 0) {
                    t_cut += clock64() - tc0;
                    atomicAdd(a.dbg + SDBG_NCUT, 1ull);
                }
                return;
            }
        }
        block_select(bk, bid, 0, nb, kprime, sel, okey_s, oid_s, DT == DLLM_DTYPE_BF16);
        const int kk = min(nb, kprime);
        for (int i = tid; i < kk; i += NT) {
            bk[i] = okey_s[i];
            bid[i] = oid_s[i];
        }
        __syncthreads();
        if (tid == 0) {
            s_nb = kk;
            if (kk == kprime) {
                s_thr = okey_s[kprime - 1];
                s_strict = 1;
            }
        }
        __syncthreads();
        if (a.dbg && tid == 0) {
            t_cut += clock64() - tc0;
            atomicAdd(a.dbg + SDBG_NCUT, 1ull);
        }
    };

    // Tiles of E columns, ST_U 16-byte vectors per thread.  Two register sets take turns (the loop
    // is unrolled by two, so a set is reloaded only after it has been processed and no register
    // move waits on a load in flight), and thread 0 pulls the tile ST_PD tiles ahead into L2.
    const uint4 *src4 = reinterpret_cast<const uint4 *>(src);
    auto load_tile = [&](int b, uint4 (&dst)[ST_U], uint32_t (&mdst)[ST_U]) {
#pragma unroll
        for (int u = 0; u < ST_U; u++) {
            const int i = b + VEC * (tid + u * NT);
            dst[u] = i < nv ? src4[i / VEC] : make_uint4(0u, 0u, 0u, 0u);
            mdst[u] = (mrow && i < nv) ? mrow[i >> 5] : 0xffffffffu;
        }
    };
    auto prefetch_tile = [&](int b) {
        if (tid != 0 || b >= nv) return;
        const int cols = min(E, nv - b) & ~(VEC - 1);
        const unsigned char *p0 = src + (size_t)b * esz;
        if (cols > 0 && ((uintptr_t)p0 & 15u) == 0 && ((cols * esz) & 15u) == 0) prefetch_l2(p0, (uint32_t)(cols * esz));
        if (mrow) {
            const uint32_t *m0 = mrow + (b >> 5);
            const int words = (cols + 31) >> 5;
            if (((uintptr_t)m0 & 15u) == 0 && ((words * 4) & 15) == 0) prefetch_l2(m0, (uint32_t)(words * 4));
        }
    };
    bool first = true;
    // one tile: every column keyed while the threshold is not finite (the exact path); after that
    // only vectors whose largest masked value reaches it (a packed maximum and one compare each;
    // the mask only lowers values, NaN propagates to the exact path)
    auto process = [&](int b, const uint4 (&r)[ST_U], const uint32_t (&mr)[ST_U]) {
        prefetch_tile(b + ST_PD * E);
        if (s_thr <= KNEG) {
            uint32_t key[ST_U][VEC];
#pragma unroll
            for (int u = 0; u < ST_U; u++) {
                const int i = b + VEC * (tid + u * NT);
                if (i < nv) vec_keys(i, r[u], mr[u], key[u]);
                else
#pragma unroll
                    for (int j = 0; j < VEC; j++) key[u][j] = 0u;
            }
            if (first) {
                // group maxima of the first tile: at least kprime keys reach their minimum
                uint32_t tmax = 0u;
#pragma unroll
                for (int u = 0; u < ST_U; u++)
#pragma unroll
                    for (int j = 0; j < VEC; j++) tmax = max(tmax, key[u][j]);
                int Kp = 1;
                while (Kp < kprime) Kp <<= 1;
                const int gs = NT / Kp;
                uint32_t g = tmax;
                for (int o = 1; o < gs && o < 32; o <<= 1) g = max(g, __shfl_xor_sync(0xffffffffu, g, o));
                if (gs > 32) g = 0u;  // groups wider than a warp: no pre-filter
                uint32_t wmin = g;
                for (int o = 16; o; o >>= 1) wmin = min(wmin, __shfl_xor_sync(0xffffffffu, wmin, o));
                if (lane == 0) sel.wv[tid >> 5] = wmin;
                __syncthreads();
                if (tid == 0) {
                    uint32_t t = 0xffffffffu;
                    for (int w = 0; w < NT / 32; w++) t = min(t, sel.wv[w]);
                    s_thr = t == 0xffffffffu ? 0u : t;
                }
                __syncthreads();
                first = false;
            }
            const uint32_t thr = s_thr;
            const bool strict = s_strict != 0;
#pragma unroll
            for (int u = 0; u < ST_U; u++) {
                unsigned m = 0u;
#pragma unroll
                for (int j = 0; j < VEC; j++) m |= (strict ? key[u][j] > thr : key[u][j] >= thr) ? (1u << j) : 0u;
                if (__any_sync(0xffffffffu, m != 0u)) append(b + VEC * (tid + u * NT), key[u], m);
            }
        } else {
            const uint32_t thr = s_thr;
            const bool strict = s_strict != 0;
            const float tf = okey_inv(thr);
            // lane-local: a bit per column whose masked value reaches tf (or is NaN), then each
            // set bit is checked exactly on its key and appended with one shared atomic
            auto add = [&](int col, float x) {
                const uint32_t key = okey(x);
                if (strict ? key > thr : key >= thr) {
                    const int pos = atomicAdd(&s_nb, 1);
                    if (pos < ST_CAP) {
                        bk[pos] = key;
                        bid[pos] = col;
                    }
                }
            };
#pragma unroll
            for (int u = 0; u < ST_U; u++) {
                const int i = b + VEC * (tid + u * NT);
                if (i >= nv) continue;
                const uint32_t mb = mr[u] >> (i & 31);  // this vector's mask bits (all ones: no mask)
                unsigned bits;
                if (DT == DLLM_DTYPE_BF16) {
                    const __nv_bfloat162 t2 = __floats2bfloat162_rn(tf, tf);  // tf is a bf16 value
                    const uint32_t w[4] = {r[u].x, r[u].y, r[u].z, r[u].w};
                    bits = 0u;
                    __nv_bfloat162 mx = *reinterpret_cast<const __nv_bfloat162 *>(&w[0]);
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const __nv_bfloat162 a2 = *reinterpret_cast<const __nv_bfloat162 *>(&w[q]);
                        const unsigned m2 = __hge2_mask(a2, t2);
                        bits |= ((m2 & 1u) | ((m2 >> 15) & 2u)) << (2 * q);
                        if (q) mx = __hmax2_nan(mx, a2);
                    }
                    const float lo = __low2float(mx), hi = __high2float(mx);
                    if (lo != lo || hi != hi) bits = 0xffu;
                    bits &= mb & 0xffu;
                    while (bits) {
                        const int q = __ffs(bits) - 1;
                        bits &= bits - 1u;
                        const uint32_t ww = w[q >> 1];
                        add(i + q, bitsf((q & 1) ? (ww & 0xffff0000u) : (ww << 16)));
                    }
                } else {
                    const float x[4] = {bitsf(r[u].x), bitsf(r[u].y), bitsf(r[u].z), bitsf(r[u].w)};
                    bits = 0u;
#pragma unroll
                    for (int q = 0; q < 4; q++) bits |= (!(x[q] < tf)) ? (1u << q) : 0u;  // >= tf or NaN
                    bits &= mb & 0xfu;
                    while (bits) {
                        const int q = __ffs(bits) - 1;
                        bits &= bits - 1u;
                        add(i + q, x[q]);
                    }
                }
            }
        }
        __syncthreads();
        if (s_nb > ST_CAP - E) cut();
    };
    const long long t_start = a.dbg ? clock64() : 0;
    for (int d = 0; d < ST_PD; d++) prefetch_tile(d * E);
    {
        uint4 ra[ST_U], rb[ST_U];
        uint32_t ma[ST_U], mb2[ST_U];
        load_tile(0, ra, ma);
        load_tile(E, rb, mb2);
        int base = 0;
        while (base < nv) {
            process(base, ra, ma);
            if (base + 2 * E < nv) load_tile(base + 2 * E, ra, ma);
            base += E;
            if (base >= nv) break;
            process(base, rb, mb2);
            if (base + 2 * E < nv) load_tile(base + 2 * E, rb, mb2);
            base += E;
        }
    }
    // unaligned tail, one column per thread per round
    for (int i0 = nv; i0 < n; i0 += NT) {
        const int i = i0 + tid;
        uint32_t key[VEC];
#pragma unroll
        for (int j = 0; j < VEC; j++) key[j] = 0u;
        unsigned m = 0u;
        if (i < n) {
            const float v = raw_at(i);
            key[0] = okey(v);
            const uint32_t thr = s_thr;
            m = (s_strict ? key[0] > thr : key[0] >= thr) ? 1u : 0u;
        }
        if (__any_sync(0xffffffffu, m != 0u)) append(i, key, m);
        __syncthreads();
        if (s_nb > ST_CAP - NT) cut();
    }
    __syncthreads();
    const long long t_loop = a.dbg ? clock64() : 0;
    const long long t_cut_loop = t_cut;
    // The buffer holds the K' best raw entries (and others that beat the threshold of their
    // time), so the union below may take all of it: a final cut is needed only when the buffer
    // and the history entries would not fit the union area.
    if (s_nb + nhist > ST_FIN) cut();
    const long long t_fcut = a.dbg ? clock64() : 0;
    // the union: the K' best raw entries that are not history ids, and each history id of this
    // shard once, with its penalised value (src/sampler.c:21-52, after the mask).  The shard's
    // history ids go into an open-addressing set of local ids (HT_SLOTS slots, at most SH_KMAX
    // used) over sel.hist and sel.ck, which are free here; the set also drops repeated ids.
    constexpr int HT_SLOTS = 512;
    static_assert(sizeof(sel.hist) + sizeof(sel.ck) >= HT_SLOTS * sizeof(int), "history set");
    int *htab = reinterpret_cast<int *>(sel.hist);
    auto hslot = [](int li) { return (int)(((uint32_t)li * 2654435761u) >> 23); };  // 9 bits
    const int nraw = s_nb;
    if (tid == 0) s_nh = 0;
    if (pen) {
        for (int i = tid; i < HT_SLOTS; i += NT) htab[i] = -1;
        __syncthreads();
        for (int j = tid; j < nhist; j += NT) {
            const int id = hall[j];
            if (id < 0 || id >= a.vtotal) continue;
            const int64_t li64 = (int64_t)id - a.voff;
            if (li64 < 0 || li64 >= n) continue;
            const int li = (int)li64;
            for (int h = hslot(li);; h = (h + 1) & (HT_SLOTS - 1)) {
                const int prev = atomicCAS(&htab[h], -1, li);
                if (prev == -1) {  // first occurrence: it stands for all of them
                    hl[atomicAdd(&s_nh, 1)] = li;
                    break;
                }
                if (prev == li) break;
            }
        }
    }
    __syncthreads();
    const int nh = s_nh;
    // the raw entries that are not history ids (their order does not matter: the select ranks
    // by key and id)
    if (tid == 0) s_nb = 0;
    __syncthreads();
    for (int i = tid; i < nraw; i += NT) {
        bool inhist = false;
        if (nh > 0) {
            const int li = bid[i];
            for (int h = hslot(li);; h = (h + 1) & (HT_SLOTS - 1)) {
                const int t = htab[h];
                if (t == -1) break;
                if (t == li) {
                    inhist = true;
                    break;
                }
            }
        }
        if (!inhist) {
            const int at = atomicAdd(&s_nb, 1);
            fk[at] = bk[i];
            fid[at] = bid[i];
        }
    }
    __syncthreads();
    const int nr = s_nb;
    if (nh > 0) {
        const float inv_rep = __fdiv_rn(1.0f, p.repetition);
        const bool true_div = (a.flags & DLLM_MODE_PEN_TRUE_DIV) != 0;
        for (int q = tid; q < nh; q += NT) {
            const int li = hl[q];
            const int64_t gid = (int64_t)li + a.voff;
            int c = 0;
            for (int j = 0; j < nhist; j++) c += hall[j] == gid;
            fk[nr + q] = okey(penalise(raw_at(li), c, p, true_div, inv_rep));
            fid[nr + q] = li;
        }
    }
    __syncthreads();
    const long long t_union = a.dbg ? clock64() : 0;
    union_select(fk, fid, nr + nh, a.k, reinterpret_cast<unsigned long long *>(bk), sel, okey_s, oid_s);
    if (a.peers) {
        // this row's candidates straight into every rank's exchange buffer (NVLink stores to the
        // peers, no collective), then one arrival per rank, released after the stores
        for (int i = tid; i < a.p_world * a.k; i += NT) {
            const int pr = i / a.k, j = i - pr * a.k;
            unsigned char *base = a.peers[pr];
            const size_t o = ((size_t)a.p_rank * a.rows + row) * a.k + j;
            px_vals(base, a.p_slot, a.p_world, a.rows, a.k)[o] = okey_inv(okey_s[j]);
            px_ids(base, a.p_slot, a.p_world, a.rows, a.k)[o] = (int32_t)(oid_s[j] + a.voff);
        }
        __threadfence_system();
        __syncthreads();
        if (tid < a.p_world) {
            unsigned long long *ctr = reinterpret_cast<unsigned long long *>(a.peers[tid]) + a.p_rank;
            asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(ctr) : "memory");
        }
    } else {
        for (int i = tid; i < a.k; i += NT) {
            a.cand_val[(int64_t)row * a.k + i] = okey_inv(okey_s[i]);
            a.cand_id[(int64_t)row * a.k + i] = (int32_t)(oid_s[i] + a.voff);
        }
    }
    if (a.dbg && tid == 0) {
        const long long t_end = clock64();
        atomicAdd(a.dbg + SDBG_ROWS, 1ull);
        atomicAdd(a.dbg + SDBG_LOOP, (unsigned long long)(t_loop - t_start - t_cut_loop));
        atomicAdd(a.dbg + SDBG_CUT, (unsigned long long)t_cut_loop);
        atomicAdd(a.dbg + SDBG_UNION, (unsigned long long)(t_union - t_loop));  // final cut + union build
        atomicAdd(a.dbg + SDBG_FINAL, (unsigned long long)(t_end - t_union));
    }
}

struct MergeArgs {
    int rows, nsh, k;
    const float *vals;     // [nsh][rows][k]
    const int32_t *ids;
    dllm_sampler_params bparams;
    const dllm_sampler_params *rparams;
    const float *uniforms;
    int32_t *token;
    int32_t *status;       // [rows] or null
    // peer exchange: wait until every rank's arrival counter here reaches `target` (bounded)
    const unsigned long long *arrive;
    unsigned long long target;
    long long wait_ns;
    unsigned long long *dbg;  // diagnostic counters (MDBG_*) or null
};

constexpr int MG_THREADS = 256;
constexpr int MG_MAX = 16 * SH_KMAX;  // candidates per row (shards x k)

// 32-bit words of the merge kernel's shared memory before its top-k lists: the candidates' values
// and ids, or the sort's staging area when the sort ranks them
__host__ __device__ constexpr int merge_lists_words(int n) { return n <= 2 * MG_THREADS ? 4 * MG_THREADS : 2 * n; }

__global__ void __launch_bounds__(MG_THREADS) merge_sample_kernel(const MergeArgs a) {
    extern __shared__ __align__(16) unsigned char mdyn[];
    const int n = a.nsh * a.k;
    float *v = reinterpret_cast<float *>(mdyn);
    int *id = reinterpret_cast<int *>(v + n);
    // up to 2 * MG_THREADS candidates are ranked by a sort whose staging area (8 bytes per
    // position) overlays v and id, so the top-k lists start past it
    float *tl = reinterpret_cast<float *>(mdyn) + merge_lists_words(n);
    int *il = reinterpret_cast<int *>(tl + a.k);
    __shared__ float red_f[MG_THREADS / 32];
    __shared__ int red_i[MG_THREADS / 32];
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, NT = blockDim.x;
    const long long t0c = a.dbg ? clock64() : 0;
    if (a.arrive) {
        // every rank's candidates for this step have landed here once its counter reaches the
        // target; the wait is bounded (a rank that never arrives makes the row DLLM_ROW_ERR_TIMEOUT)
        __shared__ int s_late;
        if (tid == 0) {
            int late = 0;
            unsigned long long t0;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
            for (int r = 0; r < a.nsh && !late; r++) {
                for (;;) {
                    unsigned long long c;
                    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(c) : "l"(a.arrive + r) : "memory");
                    if (c >= a.target) break;
                    unsigned long long t;
                    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
                    if ((long long)(t - t0) > a.wait_ns) {
                        late = 1;
                        break;
                    }
                    __nanosleep(200);
                }
            }
            __threadfence();
            s_late = late;
        }
        __syncthreads();
        if (s_late) {
            if (tid == 0) {
                a.token[row] = 0;
                if (a.status) a.status[row] = ROW_ERR_TIMEOUT;
            }
            return;
        }
    }
    const dllm_sampler_params p = a.rparams ? a.rparams[row] : a.bparams;
    // Sampling rows need 1 <= top_k <= k: the gathered lists hold each shard's k best, so a
    // larger top_k (or top-k off) cannot be served from them.  Such a row gets the greedy token
    // (always correct to take from the candidates) and DLLM_ROW_ERR_TOPK_LARGE.
    const bool bad_k = p.temperature != 0.0f && (p.top_k < 1 || p.top_k > a.k);
    const int k = bad_k ? 1 : p.top_k;
    if (a.status && tid == 0) a.status[row] = bad_k ? ROW_ERR_TOPK_LARGE : 0;
    for (int i = tid; i < n; i += NT) {
        const int s = i / a.k, j = i % a.k;
        v[i] = a.vals[((int64_t)s * a.rows + row) * a.k + j];
        id[i] = a.ids[((int64_t)s * a.rows + row) * a.k + j];
    }
    __syncthreads();
    // row maximum, and the lowest id holding it (greedy, src/sampler.c:9-19)
    float m = -INFINITY;
    for (int i = tid; i < n; i += NT) m = fmaxf(m, v[i]);
    m = warp_allreduce(m, [](float x, float y) { return fmaxf(x, y); });
    if (lane == 0) red_f[wid] = m;
    __syncthreads();
    float M = -INFINITY;
    for (int w = 0; w < NT / 32; w++) M = fmaxf(M, red_f[w]);
    if (p.temperature == 0.0f || bad_k) {
        int best = INT_MAX;
        for (int i = tid; i < n; i += NT)
            if (v[i] == M) best = min(best, id[i]);
        best = warp_allreduce(best, [](int x, int y) { return min(x, y); });
        if (lane == 0) red_i[wid] = best;
        __syncthreads();
        if (tid == 0) {
            int b = INT_MAX;
            for (int w = 0; w < NT / 32; w++) b = min(b, red_i[w]);
            a.token[row] = b == INT_MAX ? 0 : b;
        }
        return;
    }
    if (M == -INFINITY || M == INFINITY) {
        // every t is -inf or NaN: the reference's list keeps id order and returns its last entry
        if (tid == 0) a.token[row] = k - 1;
        return;
    }
    const float inv_temp = __fdiv_rn(1.0f, p.temperature);
    for (int i = tid; i < n; i += NT) v[i] = __fmul_rn(__fsub_rn(v[i], M), inv_temp);
    __syncthreads();
    const long long t1c = a.dbg ? clock64() : 0;
    bool pairwise = false;
    if (n > MG_THREADS && n <= 2 * MG_THREADS) {
        // more than one candidate per thread: a sort of the composites okey(t) << 32 | ~(id ^ 0x80000000), whose descending order is
        // (t desc, id asc) with ids compared as signed integers
        unsigned long long c[2];
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const int i = 2 * tid + r;
            c[r] = i < n ? ((unsigned long long)okey(v[i]) << 32) | (uint32_t)~((uint32_t)id[i] ^ 0x80000000u) : 0ull;
        }
        __syncthreads();  // the sort's staging area overlays v and id
        unsigned long long *srt = reinterpret_cast<unsigned long long *>(mdyn);
        sort_desc_2x(c, srt);
        for (int i = tid; i < k; i += NT) {
            const unsigned long long x = srt[i];
            tl[i] = okey_inv((uint32_t)(x >> 32));
            il[i] = (int)(~(uint32_t)x ^ 0x80000000u);
        }
    } else {
        // at most one candidate per thread (or more than two): the k best by (t desc, id asc).
        // Each shard's list is sorted by (value desc, id asc), and t
        // is a non-decreasing function of the value, so t never increases along a list; only two
        // distinct values that round to the same t can leave a run of equal t with its ids out of
        // order.  A candidate's rank is therefore, over every list, the number of entries with a
        // larger t (a binary search) plus the entries of the equal-t run with a smaller id (a scan of
        // the run, usually empty); the count stops once it reaches k.  A list whose t increases
        // somewhere (not expected) makes the row compare every pair.
        __shared__ int s_unsorted;
        if (tid == 0) s_unsorted = 0;
        __syncthreads();
        for (int i = tid; i < n; i += NT) {
            const int j = i % a.k;
            if (j + 1 < a.k && okey(v[i]) < okey(v[i + 1])) s_unsorted = 1;
        }
        __syncthreads();
        const bool sorted_lists = s_unsorted == 0;
        pairwise = !sorted_lists;
        for (int i = tid; i < n; i += NT) {
            const uint32_t ki = okey(v[i]);
            const int ii = id[i];
            int r = 0;
            if (sorted_lists) {
                // its own list first; a count that reaches k already rules the candidate out
                const int own = i / a.k;
                for (int q = 0; q < a.nsh && r < k; q++) {
                    const int sh = own + q < a.nsh ? own + q : own + q - a.nsh;
                    const float *vl = v + sh * a.k;
                    const int *il2 = id + sh * a.k;
                    int lo = 0, hi = a.k;  // the first position whose t is not above ki
                    while (lo < hi) {
                        const int mid = (lo + hi) >> 1;
                        if (okey(vl[mid]) > ki) lo = mid + 1;
                        else hi = mid;
                    }
                    r += lo;
                    for (int t = lo; t < a.k && okey(vl[t]) == ki; t++) r += il2[t] < ii;
                }
            } else {
                for (int j = 0; j < n; j++) {
                    const uint32_t kj = okey(v[j]);
                    r += kj > ki || (kj == ki && id[j] < ii);
                }
            }
            if (r < k) {
                tl[r] = v[i];
                il[r] = ii;
            }
        }
    }
    __syncthreads();
    const long long t2c = a.dbg ? clock64() : 0;
    if (wid == 0) {
        const int tok = sample_sorted_list(tl, il, k, p, a.uniforms[row], nullptr, false);
        if (lane == 0) a.token[row] = tok;
        if (a.dbg && lane == 0) {
            atomicAdd(a.dbg + MDBG_ROWS, 1ull);
            atomicAdd(a.dbg + MDBG_LOAD, (unsigned long long)(t1c - t0c));
            atomicAdd(a.dbg + MDBG_RANK, (unsigned long long)(t2c - t1c));
            atomicAdd(a.dbg + MDBG_DRAW, (unsigned long long)(clock64() - t2c));
            if (pairwise) atomicAdd(a.dbg + MDBG_PAIRWISE, 1ull);
        }
    }
}

}  // namespace

size_t shard_part_bytes(int rows, int vlocal, int k) {
    const int nch = (vlocal + SH_CHUNK - 1) / SH_CHUNK;
    return nch > 1 ? (size_t)rows * nch * k * 8 : 0;
}


// The dynamic shared memory limit of a shard kernel, raised once per (device, kernel) to the
// largest size asked so far (a launch then costs no attribute call), and the DLLM_SHARD_CHUNKED
// switch, read once per process.
namespace {
std::mutex g_shard_attr_mu;
struct ShardAttr {
    int dev;
    const void *fn;
    size_t smem;
};
std::vector<ShardAttr> g_shard_attr;
}  // namespace

static cudaError_t shard_smem_attr(const void *fn, size_t smem) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(g_shard_attr_mu);
    ShardAttr *hit = nullptr;
    for (auto &r : g_shard_attr)
        if (r.dev == dev && r.fn == fn) hit = &r;
    if (hit && hit->smem >= smem) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    if (hit) hit->smem = smem;
    else g_shard_attr.push_back({dev, fn, smem});
    return cudaSuccess;
}

static bool shard_chunked_env() {
    static const bool on = getenv("DLLM_SHARD_CHUNKED") != nullptr;
    return on;
}

dllm_status launch_shard_candidates(const dllm_batch_desc *d, int64_t voff, int64_t vtotal, int k, float *cand_val,
                                    int32_t *cand_id, void *part, cudaStream_t stream, const PeerArgs *px) {
    if (k < 1 || k > SH_KMAX || k > d->vocab) return DLLM_ERR_UNSUPPORTED;
    ShardArgs a = {};
    a.logits = d->logits;
    a.row_stride = d->row_stride;
    a.dtype = d->dtype;
    a.mask = d->mask;
    a.mask_stride = d->mask_stride;
    a.hist_ids = d->hist_ids;
    a.hist_off = d->hist_off;
    a.bparams = d->params;
    a.rparams = d->row_params;
    a.rows = d->rows;
    a.vlocal = d->vocab;
    a.k = k;
    a.nchunks = (d->vocab + SH_CHUNK - 1) / SH_CHUNK;
    a.voff = voff;
    a.vtotal = vtotal;
    a.flags = d->flags;
    a.cand_val = cand_val;
    a.cand_id = cand_id;
    a.status = d->status;
    a.dbg = debug_counters();
    if (px) {
        a.peers = reinterpret_cast<unsigned char *const *>(px->peers);
        a.p_rank = px->rank;
        a.p_world = px->world;
        a.p_slot = (int)(px->epoch & 1u);
    }
    if (a.rows == 0) return DLLM_OK;
    // the peer exchange is written by the streaming kernel only
    const int hb0 = (d->hist_ids && d->hist_off) ? (d->hist_max > 0 ? d->hist_max : 0) : 0;
    if (px && (k + hb0 > SH_KMAX || shard_chunked_env())) return DLLM_ERR_UNSUPPORTED;
    if (a.nchunks > 1 && !px) {
        if (!part) return DLLM_ERR_OOM;
        a.part_key = reinterpret_cast<uint32_t *>(part);
        a.part_id = reinterpret_cast<int32_t *>(a.part_key + (size_t)a.rows * a.nchunks * k);
        const size_t rs = (size_t)a.nchunks * k * 8 + (size_t)SH_SURV * 8;
        if (rs > 200 * 1024) return DLLM_ERR_UNSUPPORTED;
        if (shard_smem_attr((const void *)shard_rowmerge_kernel, rs) != cudaSuccess)
            return DLLM_ERR_CUDA;
    }
    if (a.status) cudaMemsetAsync(a.status, 0, (size_t)a.rows * sizeof(int32_t), stream);
    // one streaming CTA per row when the union of K' = k + history bound raw candidates and the
    // history entries fits the exact select
    const int hb = (d->hist_ids && d->hist_off) ? (d->hist_max > 0 ? d->hist_max : 0) : 0;
    if (k + hb <= SH_KMAX && !shard_chunked_env()) {
        const size_t ss = (size_t)ST_CAP * 8 + (size_t)ST_FIN * 8 + (size_t)SH_KMAX * 8;
        const void *fs = d->dtype == DLLM_DTYPE_BF16 ? (const void *)shard_stream_kernel<DLLM_DTYPE_BF16>
                                                     : (const void *)shard_stream_kernel<DLLM_DTYPE_F32>;
        if (shard_smem_attr(fs, ss) != cudaSuccess)
            return DLLM_ERR_CUDA;
        if (d->dtype == DLLM_DTYPE_BF16)
            shard_stream_kernel<DLLM_DTYPE_BF16><<<a.rows, ST_T, ss, stream>>>(a, k + hb);
        else
            shard_stream_kernel<DLLM_DTYPE_F32><<<a.rows, ST_T, ss, stream>>>(a, k + hb);
        return cudaGetLastError() == cudaSuccess ? DLLM_OK : DLLM_ERR_CUDA;
    }
    const dim3 grid(a.nchunks, a.rows);
    const size_t ks = (size_t)SH_CHUNK * 4 + (size_t)SH_SURV * 8;  // keys, then the survivors
    const void *fn = d->dtype == DLLM_DTYPE_BF16 ? (const void *)shard_chunk_kernel<DLLM_DTYPE_BF16>
                                                 : (const void *)shard_chunk_kernel<DLLM_DTYPE_F32>;
    if (shard_smem_attr(fn, ks) != cudaSuccess)
        return DLLM_ERR_CUDA;
    if (d->dtype == DLLM_DTYPE_BF16)
        shard_chunk_kernel<DLLM_DTYPE_BF16><<<grid, SH_T, ks, stream>>>(a);
    else
        shard_chunk_kernel<DLLM_DTYPE_F32><<<grid, SH_T, ks, stream>>>(a);
    if (a.nchunks > 1)
        shard_rowmerge_kernel<<<a.rows, SH_T, (size_t)a.nchunks * k * 8 + (size_t)SH_SURV * 8, stream>>>(a);
    return cudaGetLastError() == cudaSuccess ? DLLM_OK : DLLM_ERR_CUDA;
}

dllm_status launch_merge_sample(int rows, int nsh, int k, const float *vals, const int32_t *ids,
                                const dllm_sampler_params *params, const dllm_sampler_params *row_params,
                                const float *uniforms, int32_t *token, int32_t *status, cudaStream_t stream,
                                const unsigned long long *arrive, unsigned long long target, long long wait_ns) {
    if (nsh < 1 || k < 1 || k > SH_KMAX || nsh * k > MG_MAX) return DLLM_ERR_UNSUPPORTED;
    MergeArgs a = {};
    a.rows = rows;
    a.nsh = nsh;
    a.k = k;
    a.vals = vals;
    a.ids = ids;
    a.bparams = *params;
    a.rparams = row_params;
    a.uniforms = uniforms;
    a.token = token;
    a.status = status;
    a.arrive = arrive;
    a.target = target;
    a.wait_ns = wait_ns;
    a.dbg = debug_counters();
    if (rows == 0) return DLLM_OK;
    const size_t smem = (size_t)merge_lists_words(nsh * k) * 4 + (size_t)k * 8;
    if (shard_smem_attr((const void *)merge_sample_kernel, smem) != cudaSuccess)
        return DLLM_ERR_CUDA;
    merge_sample_kernel<<<rows, MG_THREADS, smem, stream>>>(a);
    return cudaGetLastError() == cudaSuccess ? DLLM_OK : DLLM_ERR_CUDA;
}

size_t peer_exchange_bytes(int rows, int k, int world) {
    if (rows < 1 || k < 1 || world < 1 || world > PX_MAX_WORLD) return 0;
    return PX_HDR + 2 * px_slot_bytes(world, rows, k);
}

dllm_status launch_merge_sample_peer(int rows, int world, int k, const void *local_buf, unsigned long long epoch,
                                     const dllm_sampler_params *params, const dllm_sampler_params *row_params,
                                     const float *uniforms, int32_t *token, int32_t *status, long long wait_ns,
                                     cudaStream_t stream) {
    unsigned char *base = reinterpret_cast<unsigned char *>(const_cast<void *>(local_buf));
    const int slot = (int)(epoch & 1u);
    return launch_merge_sample(rows, world, k, px_vals(base, slot, world, rows, k), px_ids(base, slot, world, rows, k),
                               params, row_params, uniforms, token, status, stream,
                               reinterpret_cast<const unsigned long long *>(base), epoch * (unsigned long long)rows,
                               wait_ns);
}

}  // namespace dllm
