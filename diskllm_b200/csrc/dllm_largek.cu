// dllm_largek.cu -- rows whose top-k exceeds the fused kernel's list capacity (top_k > KMAX).
//
// The reference accepts any 0 < top_k < vocab (src/sampler.c:165-170): partial_sort_top_k leaves
// the k best entries in work_buf[0..k) ordered by t descending, ties by lower id
// (src/sampler.c:109-134), and softmax / min-p / top-p / the fp32 draw then run over those k
// entries (src/sampler.c:172-233).  For k above the fused kernel's list capacity the rows take
// this pass instead, in chunks of rows:
//
//   largek_prep_kernel  one CTA per row: the masked, penalised row (src/core/sampler_api.c:48-61),
//                       its maximum, and one 64-bit key per entry, (~orderkey(t) << 32) | id, so
//                       that an ascending sort gives (t desc, id asc) with no equal keys
//   segmented radix sort of the keys (CUB, one segment per row)
//   largek_sample_kernel one warp per row: the sorted list's first k entries through the same
//                       softmax / min-p / top-p / draw code as the fused kernel's top-k rows
//
// Rows with top_k <= KMAX (per-row parameters) get empty segments and are left to the fused
// kernel.  This path serves a case the fused kernel cannot; it is not tuned.
#include <cuda_runtime.h>

#include <cub/device/device_segmented_radix_sort.cuh>

#include "dllm_chunk.cuh"

namespace dllm {
namespace {

constexpr int LK_THREADS = 1024;

struct LargeArgs {
    const void *logits;
    int64_t row_stride;
    int dtype;
    const uint32_t *mask;
    int64_t mask_stride;
    const int32_t *hist_ids;
    const int64_t *hist_off;
    const float *uniforms;
    dllm_sampler_params bparams;
    const dllm_sampler_params *rparams;
    int vocab;
    unsigned flags;
    int after_fused;       // the fused kernel ran first (status and penalised rows written)
    int row0;              // first batch row of this chunk
    int nrows;             // rows in this chunk
    unsigned long long *keys_in;   // [nrows][vocab]
    unsigned long long *keys_out;  // [nrows][vocab]
    int *seg_begin;        // [nrows]
    int *seg_end;          // [nrows]
    float *row_max;        // [nrows]
    int32_t *token;
    float *probs;
    int64_t probs_stride;
    float *pen_out;
    int64_t pen_stride;
    int32_t *status;
    int32_t *topk_ids;
    int64_t topk_stride;
};

__device__ __forceinline__ bool is_large(const dllm_sampler_params &p, int vocab) {
    return p.temperature > 0.0f && p.top_k > KMAX && p.top_k < vocab;
}

__global__ void __launch_bounds__(LK_THREADS) largek_prep_kernel(const LargeArgs a) {
    __shared__ float red[LK_THREADS / 32];
    const int b = blockIdx.x, row = a.row0 + b, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int V = a.vocab;
    const dllm_sampler_params p = a.rparams ? a.rparams[row] : a.bparams;
    const int seg0 = b * V;
    if (!is_large(p, V)) {
        if (tid == 0) {
            a.seg_begin[b] = seg0;
            a.seg_end[b] = seg0;
        }
        return;
    }
    // masked row into scratch (the output key area, unused until the sort)
    float *v = reinterpret_cast<float *>(a.keys_out + (size_t)seg0);
    const unsigned char *src = reinterpret_cast<const unsigned char *>(a.logits) +
                               (size_t)row * a.row_stride * (a.dtype == DLLM_DTYPE_BF16 ? 2 : 4);
    const uint32_t *mrow = a.mask ? a.mask + (int64_t)row * a.mask_stride : nullptr;
    for (int i = tid; i < V; i += LK_THREADS) {
        const float x = chunk_raw(src, a.dtype, i);
        v[i] = (!mrow || ((mrow[i >> 5] >> (i & 31)) & 1u)) ? x : -INFINITY;
    }
    __syncthreads();
    // history penalties: the first occurrence of each in-range id applies them once, with its
    // number of occurrences (presence and frequency once per id, repetition per occurrence)
    if (pen_active(a.hist_ids, a.hist_off, p)) {
        const int64_t h0 = a.hist_off[row], h1 = a.hist_off[row + 1];
        const bool true_div = (a.flags & DLLM_MODE_PEN_TRUE_DIV) != 0;
        const float inv_rep = __fdiv_rn(1.0f, p.repetition);
        for (int64_t j = h0 + tid; j < h1; j += LK_THREADS) {
            const int id = a.hist_ids[j];
            if (id < 0 || id >= V) continue;
            bool first = true;
            for (int64_t q = h0; q < j && first; q++) first = a.hist_ids[q] != id;
            if (!first) continue;
            int c = 0;
            for (int64_t q = j; q < h1; q++) c += a.hist_ids[q] == id;
            v[id] = penalise(v[id], c, p, true_div, inv_rep);
        }
        __syncthreads();
    }
    if (a.pen_out && !a.after_fused) {
        float *po = a.pen_out + (int64_t)row * a.pen_stride;
        for (int i = tid; i < V; i += LK_THREADS) po[i] = v[i];
    }
    float m = -INFINITY;
    bool nanf = false;
    for (int i = tid; i < V; i += LK_THREADS) {
        m = fmaxf(m, v[i]);
        nanf |= isnan(v[i]);
    }
    m = warp_allreduce(m, [](float x, float y) { return fmaxf(x, y); });
    if (lane == 0) red[wid] = m;
    nanf = __syncthreads_or(nanf);
    float M = -INFINITY;
    for (int w = 0; w < LK_THREADS / 32; w++) M = fmaxf(M, red[w]);
    const float inv_temp = __fdiv_rn(1.0f, p.temperature);
    unsigned long long *kin = a.keys_in + (size_t)seg0;
    for (int i = tid; i < V; i += LK_THREADS) {
        const float t = __fmul_rn(__fsub_rn(v[i], M), inv_temp);
        kin[i] = ((unsigned long long)(~okey(t)) << 32) | (uint32_t)i;
    }
    if (a.probs) {
        float *pr = a.probs + (int64_t)row * a.probs_stride;
        for (int i = tid; i < V; i += LK_THREADS) pr[i] = 0.0f;
    }
    if (tid == 0) {
        a.seg_begin[b] = seg0;
        a.seg_end[b] = seg0 + V;
        // a NaN logit is reported through the row maximum's slot as NaN
        a.row_max[b] = nanf && M != INFINITY && M != -INFINITY ? __int_as_float(0x7fffffff) : M;
    }
}

__global__ void __launch_bounds__(32) largek_sample_kernel(const LargeArgs a) {
    const int b = blockIdx.x, row = a.row0 + b, lane = threadIdx.x;
    const int V = a.vocab;
    const dllm_sampler_params p = a.rparams ? a.rparams[row] : a.bparams;
    if (!is_large(p, V)) return;
    const int k = p.top_k;
    const unsigned long long *ks = a.keys_out + (size_t)b * V;
    // list in the input key area: values, then ids
    float *tl = reinterpret_cast<float *>(a.keys_in + (size_t)b * V);
    int *il = reinterpret_cast<int *>(tl + V);
    const float M = a.row_max[b];
    int flags = a.status && a.after_fused ? (a.status[row] & ~ROW_ERR_TOPK_LARGE) : 0;
    int token;
    if (M == -INFINITY || M == INFINITY) {
        // fully masked, or +inf present: every t is -inf or NaN, the reference's list stays in id
        // order and its draw returns the list's last entry
        for (int i = lane; i < k; i += 32) {
            tl[i] = 0.0f;
            il[i] = i;
        }
        token = k - 1;
    } else {
        if (isnan(M)) flags |= ROW_ERR_NONFINITE;
        for (int i = lane; i < k; i += 32) {
            const unsigned long long key = ks[i];
            tl[i] = okey_inv(~(uint32_t)(key >> 32));
            il[i] = (int)(uint32_t)key;
        }
        __syncwarp();
        float *pr = a.probs ? a.probs + (int64_t)row * a.probs_stride : nullptr;
        token = sample_sorted_list(tl, il, k, p, a.uniforms[row], pr, (a.flags & DLLM_MODE_MINP_RELATIVE) != 0);
    }
    __syncwarp();
    if (a.topk_ids)
        for (int i = lane; i < k; i += 32) a.topk_ids[(int64_t)row * a.topk_stride + i] = il[i];
    if (lane == 0) {
        a.token[row] = token;
        if (a.status) a.status[row] = flags;
    }
}

// rows per chunk: keys of at most 8 MiB per buffer, and at least one row
int chunk_rows(int rows, int vocab) {
    size_t r = ((size_t)8 << 20) / ((size_t)vocab * 8);
    if (r < 1) r = 1;
    if (r > (size_t)rows) r = (size_t)rows;
    return (int)r;
}

size_t cub_temp_bytes(int nrows, int vocab) {
    size_t temp = 0;
    cub::DeviceSegmentedRadixSort::SortKeys(nullptr, temp, (const unsigned long long *)nullptr,
                                            (unsigned long long *)nullptr, nrows * vocab, nrows, (const int *)nullptr,
                                            (const int *)nullptr, 0, 64, (cudaStream_t)0);
    return temp;
}

size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace

size_t largek_ws_bytes(int rows, int vocab) {
    if (rows <= 0) return 0;
    const int R = chunk_rows(rows, vocab);
    const size_t keys = al256((size_t)R * vocab * 8);
    return 2 * keys + 3 * al256((size_t)R * 4) + al256(cub_temp_bytes(R, vocab));
}

dllm_status launch_largek(const dllm_batch_desc *d, bool after_fused, void *ws, cudaStream_t stream) {
    const int V = d->vocab;
    const int R = chunk_rows(d->rows, V);
    unsigned char *w = reinterpret_cast<unsigned char *>(ws);
    const size_t keys = al256((size_t)R * V * 8);
    LargeArgs a = {};
    a.logits = d->logits;
    a.row_stride = d->row_stride;
    a.dtype = d->dtype;
    a.mask = d->mask;
    a.mask_stride = d->mask_stride;
    a.hist_ids = d->hist_ids;
    a.hist_off = d->hist_off;
    a.uniforms = d->uniforms;
    a.bparams = d->params;
    a.rparams = d->row_params;
    a.vocab = V;
    a.flags = d->flags;
    a.after_fused = after_fused;
    a.keys_in = reinterpret_cast<unsigned long long *>(w);
    a.keys_out = reinterpret_cast<unsigned long long *>(w + keys);
    a.seg_begin = reinterpret_cast<int *>(w + 2 * keys);
    a.seg_end = reinterpret_cast<int *>(w + 2 * keys + al256((size_t)R * 4));
    a.row_max = reinterpret_cast<float *>(w + 2 * keys + 2 * al256((size_t)R * 4));
    void *temp = w + 2 * keys + 3 * al256((size_t)R * 4);
    a.token = d->token;
    a.probs = d->probs;
    a.probs_stride = d->probs_stride;
    a.pen_out = d->pen_logits;
    a.pen_stride = d->pen_stride;
    a.status = d->status;
    a.topk_ids = d->topk_ids;
    a.topk_stride = d->topk_stride;
    for (int r0 = 0; r0 < d->rows; r0 += R) {
        a.row0 = r0;
        a.nrows = d->rows - r0 < R ? d->rows - r0 : R;
        largek_prep_kernel<<<a.nrows, LK_THREADS, 0, stream>>>(a);
        if (cudaGetLastError() != cudaSuccess) return DLLM_ERR_CUDA;
        size_t temp_bytes = cub_temp_bytes(a.nrows, V);
        if (cub::DeviceSegmentedRadixSort::SortKeys(temp, temp_bytes, a.keys_in, a.keys_out, a.nrows * V, a.nrows,
                                                    a.seg_begin, a.seg_end, 0, 64, stream) != cudaSuccess)
            return DLLM_ERR_CUDA;
        largek_sample_kernel<<<a.nrows, 32, 0, stream>>>(a);
        if (cudaGetLastError() != cudaSuccess) return DLLM_ERR_CUDA;
    }
    return DLLM_OK;
}

}  // namespace dllm
