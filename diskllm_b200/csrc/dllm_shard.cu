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
};

struct SelScratch {
    unsigned hist[256];
    uint32_t ck[SH_KMAX];
    int cid[SH_KMAX];
    int wsum[SH_T / 32];
    int bin, above, ncand;
};

// Appends to s.ck / s.cid (from s.ncand) the `need` entries equal to `target` with the lowest ids.
// Without ids (ids grow with position) each warp scans a contiguous segment with ballots, twice:
// once to count, once to rank against the earlier segments' counts.  With ids, ranks by counting.
__device__ void select_ties(const uint32_t *keys, const int *ids, int id0, int n, uint32_t target, int need, int cap,
                            SelScratch &s) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, NT = blockDim.x, NW = NT >> 5;
    if (need <= 0) return;
    if (ids) {
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

// The K best of n keys in shared memory by (key desc, id asc), written sorted to out_key / out_id
// (K entries; positions past n, when n < K, get key 0 and id INT_MAX, which rank last).
// Masked entries (-inf) are left out of the radix select of the K-th key (8 bits per pass from
// the top) and taken, lowest ids first, only when fewer than K entries are finite.  Ids: ids[i],
// or id0 + i when ids is null (then ids grow with position).
__device__ void block_select(const uint32_t *keys, const int *ids, int id0, int n, int K, SelScratch &s,
                             uint32_t *out_key, int *out_id) {
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
    for (int pass = 3; pass >= 0 && Kf > 0; pass--) {
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
        const uint32_t kstar = prefix;
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
    chunk_visit<DT>(src, vec, mrow, c0, n, cp, p, a.flags, [&](int li, float v) { keys[li] = okey(v); });
    __syncthreads();
    block_select(keys, nullptr, c0, n, a.k, sel, okey_s, oid_s);
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
    for (int i = tid; i < n; i += NT) {
        keys[i] = a.part_key[(int64_t)row * n + i];
        ids[i] = a.part_id[(int64_t)row * n + i];
    }
    __syncthreads();
    block_select(keys, ids, 0, n, a.k, sel, okey_s, oid_s);
    for (int i = tid; i < a.k; i += NT) {
        a.cand_val[(int64_t)row * a.k + i] = okey_inv(okey_s[i]);
        a.cand_id[(int64_t)row * a.k + i] = (int32_t)(oid_s[i] + a.voff);
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
};

constexpr int MG_THREADS = 256;
constexpr int MG_MAX = 16 * SH_KMAX;  // candidates per row (shards x k)

__global__ void __launch_bounds__(MG_THREADS) merge_sample_kernel(const MergeArgs a) {
    extern __shared__ __align__(16) unsigned char mdyn[];
    const int n = a.nsh * a.k;
    float *v = reinterpret_cast<float *>(mdyn);
    int *id = reinterpret_cast<int *>(v + n);
    float *tl = reinterpret_cast<float *>(id + n);
    int *il = reinterpret_cast<int *>(tl + a.k);
    __shared__ float red_f[MG_THREADS / 32];
    __shared__ int red_i[MG_THREADS / 32];
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, NT = blockDim.x;
    const dllm_sampler_params p = a.rparams ? a.rparams[row] : a.bparams;
    const int k = min(p.top_k, a.k);
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
    if (p.temperature == 0.0f) {
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
    if (M == -INFINITY) {
        // every t is NaN: the reference's list keeps id order and returns its last entry
        if (tid == 0) a.token[row] = k - 1;
        return;
    }
    const float inv_temp = __fdiv_rn(1.0f, p.temperature);
    for (int i = tid; i < n; i += NT) v[i] = __fmul_rn(__fsub_rn(v[i], M), inv_temp);
    __syncthreads();
    // the k best by (t desc, id asc)
    for (int i = tid; i < n; i += NT) {
        const uint32_t ki = okey(v[i]);
        const int ii = id[i];
        int r = 0;
        for (int j = 0; j < n; j++) {
            const uint32_t kj = okey(v[j]);
            r += kj > ki || (kj == ki && id[j] < ii);
        }
        if (r < k) {
            tl[r] = v[i];
            il[r] = ii;
        }
    }
    __syncthreads();
    if (wid == 0) {
        const int tok = sample_sorted_list(tl, il, k, p, a.uniforms[row], nullptr, false);
        if (lane == 0) a.token[row] = tok;
    }
}

}  // namespace

size_t shard_part_bytes(int rows, int vlocal, int k) {
    const int nch = (vlocal + SH_CHUNK - 1) / SH_CHUNK;
    return nch > 1 ? (size_t)rows * nch * k * 8 : 0;
}

dllm_status launch_shard_candidates(const dllm_batch_desc *d, int64_t voff, int64_t vtotal, int k, float *cand_val,
                                    int32_t *cand_id, void *part, cudaStream_t stream) {
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
    if (a.rows == 0) return DLLM_OK;
    if (a.nchunks > 1) {
        if (!part) return DLLM_ERR_OOM;
        a.part_key = reinterpret_cast<uint32_t *>(part);
        a.part_id = reinterpret_cast<int32_t *>(a.part_key + (size_t)a.rows * a.nchunks * k);
        const size_t rs = (size_t)a.nchunks * k * 8;
        if (rs > 200 * 1024) return DLLM_ERR_UNSUPPORTED;
        if (cudaFuncSetAttribute((const void *)shard_rowmerge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)rs) != cudaSuccess)
            return DLLM_ERR_CUDA;
    }
    if (a.status) cudaMemsetAsync(a.status, 0, (size_t)a.rows * sizeof(int32_t), stream);
    const dim3 grid(a.nchunks, a.rows);
    const size_t ks = (size_t)SH_CHUNK * 4;
    const void *fn = d->dtype == DLLM_DTYPE_BF16 ? (const void *)shard_chunk_kernel<DLLM_DTYPE_BF16>
                                                 : (const void *)shard_chunk_kernel<DLLM_DTYPE_F32>;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ks) != cudaSuccess)
        return DLLM_ERR_CUDA;
    if (d->dtype == DLLM_DTYPE_BF16)
        shard_chunk_kernel<DLLM_DTYPE_BF16><<<grid, SH_T, ks, stream>>>(a);
    else
        shard_chunk_kernel<DLLM_DTYPE_F32><<<grid, SH_T, ks, stream>>>(a);
    if (a.nchunks > 1) shard_rowmerge_kernel<<<a.rows, SH_T, (size_t)a.nchunks * k * 8, stream>>>(a);
    return cudaGetLastError() == cudaSuccess ? DLLM_OK : DLLM_ERR_CUDA;
}

dllm_status launch_merge_sample(int rows, int nsh, int k, const float *vals, const int32_t *ids,
                                const dllm_sampler_params *params, const dllm_sampler_params *row_params,
                                const float *uniforms, int32_t *token, cudaStream_t stream) {
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
    if (rows == 0) return DLLM_OK;
    const size_t smem = (size_t)nsh * k * 8 + (size_t)k * 8;
    if (cudaFuncSetAttribute((const void *)merge_sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
        return DLLM_ERR_CUDA;
    merge_sample_kernel<<<rows, MG_THREADS, smem, stream>>>(a);
    return cudaGetLastError() == cudaSuccess ? DLLM_OK : DLLM_ERR_CUDA;
}

}  // namespace dllm
