// dllm_shard.cu -- vocabulary-sharded sampling (a row's logits split over N GPUs, the
// tensor-parallel LM-head layout).  The path has one exchange step:
//
//   1. dllm_cuda_shard_candidates: on each GPU, one CTA per row applies the grammar mask and the
//      history penalties to the GPU's id range and selects its k best entries by (value desc,
//      id asc) with a 4-pass radix select on order-preserving keys.  Output (value, global id),
//      sorted, [rows][k].
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

#include "dllm_kernel.cuh"

namespace dllm {
namespace {

constexpr int SH_THREADS = 512;
constexpr int SH_HTAB = 1024;  // history hash entries per row (power of two)
constexpr int SH_KMAX = 256;   // largest k per shard

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
    int rows, vlocal, k;
    int64_t voff, vtotal;
    unsigned flags;
    float *cand_val;
    int32_t *cand_id;
    int32_t *status;
};

template <int DT>
__global__ void __launch_bounds__(SH_THREADS) shard_topk_kernel(const ShardArgs a) {
    __shared__ int hkeys[SH_HTAB];
    __shared__ int hcnt[SH_HTAB];
    __shared__ unsigned hist[256];
    __shared__ float cv[SH_KMAX];
    __shared__ int ci[SH_KMAX];
    __shared__ int wsum[SH_THREADS / 32];
    __shared__ int s_bin, s_above, s_ncand, s_flags;
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, NT = blockDim.x;
    const int NW = NT >> 5;
    const dllm_sampler_params p = a.rparams ? a.rparams[row] : a.bparams;
    const int Vs = a.vlocal, K = a.k;

    // history ids of this shard: local index -> occurrence count (src/sampler.c:21-52)
    for (int i = tid; i < SH_HTAB; i += NT) {
        hkeys[i] = -1;
        hcnt[i] = 0;
    }
    if (tid == 0) {
        s_ncand = 0;
        s_flags = 0;
    }
    __syncthreads();
    const bool use_hist = a.hist_ids && a.hist_off && (p.repetition > 1.0f || p.presence != 0.0f || p.frequency != 0.0f);
    if (use_hist) {
        const int64_t h0 = a.hist_off[row], h1 = a.hist_off[row + 1];
        for (int64_t j = h0 + tid; j < h1; j += NT) {
            const int id = a.hist_ids[j];
            if (id < 0 || id >= a.vtotal) continue;
            const int64_t li = (int64_t)id - a.voff;
            if (li < 0 || li >= Vs) continue;
            uint32_t h = hash_id((uint32_t)li) & (SH_HTAB - 1);
            bool placed = false;
            for (int probe = 0; probe < SH_HTAB; probe++) {
                const int old = atomicCAS(&hkeys[h], -1, (int)li);
                if (old == -1 || old == (int)li) {
                    atomicAdd(&hcnt[h], 1);
                    placed = true;
                    break;
                }
                h = (h + 1u) & (SH_HTAB - 1);
            }
            if (!placed) atomicOr(&s_flags, ROW_ERR_HIST_TABLE);
        }
    }
    __syncthreads();
    const float inv_rep = __fdiv_rn(1.0f, p.repetition);
    const bool true_div = (a.flags & DLLM_MODE_PEN_TRUE_DIV) != 0;
    const uint32_t *mrow = a.mask ? a.mask + (int64_t)row * a.mask_stride : nullptr;

    // masked, penalised logit of local element li (grammar.c:275-308, then sampler.c:35-52, 21-33)
    auto value = [&](int li) -> float {
        float v;
        if (DT == DLLM_DTYPE_F32)
            v = ((const float *)a.logits)[(int64_t)row * a.row_stride + li];
        else
            v = bitsf((uint32_t)((const unsigned short *)a.logits)[(int64_t)row * a.row_stride + li] << 16);
        if (mrow && !((mrow[li >> 5] >> (li & 31)) & 1u)) v = -INFINITY;
        if (use_hist) {
            uint32_t h = hash_id((uint32_t)li) & (SH_HTAB - 1);
            for (int probe = 0; probe < SH_HTAB; probe++) {
                const int kk = hkeys[h];
                if (kk == -1) break;
                if (kk == li) {
                    const int c = hcnt[h];
                    if (p.presence != 0.0f) v = __fsub_rn(v, p.presence);
                    if (p.frequency != 0.0f) v = __fsub_rn(v, __fmul_rn(__int2float_rn(c), p.frequency));
                    if (p.repetition > 1.0f)
                        for (int r = 0; r < c; r++) {
                            if (v < 0.0f) v = __fmul_rn(v, p.repetition);
                            else v = true_div ? __fdiv_rn(v, p.repetition) : __fmul_rn(v, inv_rep);
                        }
                    break;
                }
                h = (h + 1u) & (SH_HTAB - 1);
            }
        }
        return v;
    };

    // radix select of the K-th largest key, 8 bits per pass from the top
    uint32_t prefix = 0u, pmask = 0u;
    int remaining = K;
    unsigned cnt_eq = 0u;
    for (int pass = 3; pass >= 0; pass--) {
        for (int i = tid; i < 256; i += NT) hist[i] = 0u;
        __syncthreads();
        const int sh = 8 * pass;
        for (int li = tid; li < Vs; li += NT) {
            const uint32_t key = okey(value(li));
            if ((key & pmask) == prefix) atomicAdd(&hist[(key >> sh) & 255u], 1u);
        }
        __syncthreads();
        if (wid == 0) {
            // lane l holds bins 255-8l .. 248-8l, scanned from the top
            unsigned c[8], tot = 0u;
#pragma unroll
            for (int b = 0; b < 8; b++) {
                c[b] = hist[255 - 8 * lane - b];
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
                        s_bin = 255 - 8 * lane - b;
                        s_above = (int)acc;
                        break;
                    }
                    acc += c[b];
                }
            }
        }
        __syncthreads();
        prefix |= (uint32_t)s_bin << sh;
        pmask |= 255u << sh;
        remaining -= s_above;
        cnt_eq = hist[s_bin];
        __syncthreads();
    }
    const uint32_t kstar = prefix;  // key of the K-th best entry; `remaining` entries equal to it are kept

    // entries above the threshold, then the lowest-index entries equal to it
    for (int li = tid; li < Vs; li += NT) {
        const float v = value(li);
        const uint32_t key = okey(v);
        const bool take = key > kstar || (key == kstar && cnt_eq == (unsigned)remaining);
        if (take) {
            const int pos = atomicAdd(&s_ncand, 1);
            if (pos < K) {
                cv[pos] = v;
                ci[pos] = li;
            }
        }
    }
    __syncthreads();
    if (cnt_eq != (unsigned)remaining) {
        int taken = 0;
        for (int base = 0; base < Vs && taken < remaining; base += NT) {
            const int li = base + tid;
            float v = 0.0f;
            bool eq = false;
            if (li < Vs) {
                v = value(li);
                eq = okey(v) == kstar;
            }
            const unsigned bm = __ballot_sync(0xffffffffu, eq);
            if (lane == 0) wsum[wid] = __popc(bm);
            __syncthreads();
            int before = 0, total = 0;
            for (int w = 0; w < NW; w++) {
                if (w < wid) before += wsum[w];
                total += wsum[w];
            }
            const int rank = taken + before + __popc(bm & ((1u << lane) - 1u));
            if (eq && rank < remaining) {
                const int pos = atomicAdd(&s_ncand, 1);
                if (pos < K) {
                    cv[pos] = v;
                    ci[pos] = li;
                }
            }
            taken += total;
            __syncthreads();
        }
    }
    __syncthreads();
    // sorted by (value desc, id asc): each entry's rank among the K
    for (int i = tid; i < K; i += NT) {
        const float vi = cv[i];
        const uint32_t ki = okey(vi);
        const int ii = ci[i];
        int r = 0;
        for (int j = 0; j < K; j++) {
            const uint32_t kj = okey(cv[j]);
            r += kj > ki || (kj == ki && ci[j] < ii);
        }
        a.cand_val[(int64_t)row * K + r] = vi;
        a.cand_id[(int64_t)row * K + r] = (int32_t)(ci[i] + a.voff);
    }
    if (tid == 0 && a.status) a.status[row] = s_flags;
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
constexpr int MG_MAX = 8 * SH_KMAX;  // candidates per row (shards x k)

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
        const int tok = sample_sorted_list(tl, il, k, p, a.uniforms[row], nullptr);
        if (lane == 0) a.token[row] = tok;
    }
}

}  // namespace

dllm_status launch_shard_candidates(const dllm_batch_desc *d, int64_t voff, int64_t vtotal, int k, float *cand_val,
                                    int32_t *cand_id, cudaStream_t stream) {
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
    a.voff = voff;
    a.vtotal = vtotal;
    a.flags = d->flags;
    a.cand_val = cand_val;
    a.cand_id = cand_id;
    a.status = d->status;
    if (a.rows == 0) return DLLM_OK;
    if (d->dtype == DLLM_DTYPE_BF16)
        shard_topk_kernel<DLLM_DTYPE_BF16><<<a.rows, SH_THREADS, 0, stream>>>(a);
    else
        shard_topk_kernel<DLLM_DTYPE_F32><<<a.rows, SH_THREADS, 0, stream>>>(a);
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
