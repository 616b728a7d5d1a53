// dllm_chunk.cuh -- one CTA's view of a column chunk of a logits row: the grammar mask and the
// history penalties applied on the fly, every element visited once with its penalised value.
// Shared by the vocabulary-sharded candidate kernel and the sorted-nucleus passes.
//
// Penalties follow the reference: presence (src/sampler.c:35-52) and the frequency extension
// once per distinct id, repetition (src/sampler.c:21-33) once per occurrence, after the mask
// (src/core/sampler_api.c:48-61).  The chunk's history ids are counted in a shared-memory hash
// table; a bitmap marks their columns, so the streaming loop skips them and a second loop visits
// each of them once with its penalised value.
#pragma once

#include "dllm_kernel.cuh"

namespace dllm {
namespace {

constexpr int CH_HTAB = 512;  // history hash entries per chunk (power of two)

struct ChunkPen {
    int *hkeys;         // [CH_HTAB] local column or -1
    int *hcnt;          // [CH_HTAB] occurrences
    uint32_t *penbits;  // [chunk / 32] columns with a table entry
    int *flags;         // ROW_ERR_* (shared)
    bool active;
};

__device__ __forceinline__ bool pen_active(const int32_t *hist_ids, const int64_t *hist_off,
                                           const dllm_sampler_params &p) {
    return hist_ids && hist_off && (p.repetition > 1.0f || p.presence != 0.0f || p.frequency != 0.0f);
}

// The row's history range and this thread's first id, loaded early so that their latency overlaps
// the logits loads.
struct HistPre {
    int64_t h0, h1;
    int first;
};
__device__ __forceinline__ HistPre hist_prefetch(const int32_t *hist_ids, const int64_t *hist_off, int row, bool active) {
    HistPre h{0, 0, -1};
    if (!active) return h;
    h.h0 = hist_off[row];
    h.h1 = hist_off[row + 1];
    if (h.h0 + threadIdx.x < h.h1) h.first = hist_ids[h.h0 + threadIdx.x];
    return h;
}

// Fills the table for columns [c0, c0 + n) of the row whose history hp describes (global ids
// voff + c0 + local).  Ends with a barrier.  `nwords` = bitmap words to clear (chunk / 32).
__device__ void chunk_pen_build(ChunkPen &cp, const int32_t *hist_ids, const HistPre &hp, int64_t voff, int64_t vtotal,
                                int c0, int n, int nwords) {
    const int tid = threadIdx.x, NT = blockDim.x;
    for (int i = tid; i < CH_HTAB; i += NT) {
        cp.hkeys[i] = -1;
        cp.hcnt[i] = 0;
    }
    for (int i = tid; i < nwords; i += NT) cp.penbits[i] = 0u;
    __syncthreads();
    if (cp.active) {
        for (int64_t j = hp.h0 + tid; j < hp.h1; j += NT) {
            const int id = j == hp.h0 + tid ? hp.first : hist_ids[j];
            if (id < 0 || id >= vtotal) continue;
            const int64_t li = (int64_t)id - voff - c0;
            if (li < 0 || li >= n) continue;
            uint32_t h = hash_id((uint32_t)li) & (CH_HTAB - 1);
            bool placed = false;
            for (int probe = 0; probe < CH_HTAB; probe++) {
                const int old = atomicCAS(&cp.hkeys[h], -1, (int)li);
                if (old == -1 || old == (int)li) {
                    atomicAdd(&cp.hcnt[h], 1);
                    placed = true;
                    break;
                }
                h = (h + 1u) & (CH_HTAB - 1);
            }
            if (placed) atomicOr(&cp.penbits[li >> 5], 1u << (li & 31));
            else atomicOr(cp.flags, ROW_ERR_HIST_TABLE);
        }
    }
    __syncthreads();
}

__device__ __forceinline__ float penalise(float v, int c, const dllm_sampler_params &p, bool true_div, float inv_rep) {
    if (p.presence != 0.0f) v = __fsub_rn(v, p.presence);
    if (p.frequency != 0.0f) v = __fsub_rn(v, __fmul_rn(__int2float_rn(c), p.frequency));
    if (p.repetition > 1.0f)
        for (int r = 0; r < c; r++) {
            if (v < 0.0f) v = __fmul_rn(v, p.repetition);
            else v = true_div ? __fdiv_rn(v, p.repetition) : __fmul_rn(v, inv_rep);
        }
    return v;
}

__device__ __forceinline__ float chunk_raw(const void *src, int dt, int i) {
    return dt == DLLM_DTYPE_BF16 ? bitsf((uint32_t)((const unsigned short *)src)[i] << 16) : ((const float *)src)[i];
}

// Calls f(local column, value) once for each of the n columns: the masked logit, penalised
// where the column is in the history.  `src` points at column c0 of the row; `mrow` is the
// row's mask (word 0 = columns 0..31 of the row) or null.  The order of the calls is not the
// column order.  No barrier.
template <int DT, class F>
__device__ __forceinline__ void chunk_visit(const void *src, bool vec_ok, const uint32_t *mrow, int c0, int n,
                                            const ChunkPen &cp, const dllm_sampler_params &p, unsigned flags, F &&f) {
    const int tid = threadIdx.x, NT = blockDim.x;
    auto allowed = [&](int li) -> bool { return !mrow || ((mrow[(c0 + li) >> 5] >> ((c0 + li) & 31)) & 1u); };
    constexpr int VEC = DT == DLLM_DTYPE_BF16 ? 8 : 4;
    constexpr int UNR = 4;  // vector loads in flight per thread
    const int nv = vec_ok ? (n & ~(VEC - 1)) : 0;
    auto visit_vec = [&](int i, const uint4 raw) {
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
        // c0 and i are multiples of VEC (<= 32), so the VEC columns share one mask / bitmap word
        const uint32_t mw = mrow ? mrow[(c0 + i) >> 5] >> ((c0 + i) & 31) : 0xffffffffu;
        const uint32_t pw = cp.active ? cp.penbits[i >> 5] >> (i & 31) : 0u;
#pragma unroll
        for (int j = 0; j < VEC; j++)
            if (!((pw >> j) & 1u)) f(i + j, ((mw >> j) & 1u) ? x[j] : -INFINITY);
    };
    const uint4 *src4 = reinterpret_cast<const uint4 *>(src);
    const int step = VEC * NT;
    int i0 = VEC * tid;
    for (; i0 + (UNR - 1) * step < nv; i0 += UNR * step) {
        uint4 r[UNR];
#pragma unroll
        for (int u = 0; u < UNR; u++) r[u] = src4[(i0 + u * step) / VEC];
#pragma unroll
        for (int u = 0; u < UNR; u++) visit_vec(i0 + u * step, r[u]);
    }
    for (; i0 < nv; i0 += step) visit_vec(i0, src4[i0 / VEC]);
    for (int i = nv + tid; i < n; i += NT) {
        if (cp.active && ((cp.penbits[i >> 5] >> (i & 31)) & 1u)) continue;
        f(i, allowed(i) ? chunk_raw(src, DT, i) : -INFINITY);
    }
    if (cp.active) {
        const float inv_rep = __fdiv_rn(1.0f, p.repetition);
        const bool true_div = (flags & DLLM_MODE_PEN_TRUE_DIV) != 0;
        for (int sl = tid; sl < CH_HTAB; sl += NT) {
            const int li = cp.hkeys[sl];
            if (li < 0) continue;
            const float raw = allowed(li) ? chunk_raw(src, DT, li) : -INFINITY;
            f(li, penalise(raw, cp.hcnt[sl], p, true_div, inv_rep));
        }
    }
}

// Register-resident chunk: thread t holds vectors t, t + NT, ... (KV of them) of the chunk's first
// nv columns, loaded before anything else so the loads overlap the history-table build.
template <int DT, int KV>
__device__ __forceinline__ int chunk_load(const void *src, bool vec_ok, int n, uint4 (&r)[KV]) {
    constexpr int VEC = DT == DLLM_DTYPE_BF16 ? 8 : 4;
    const int nv = vec_ok ? (n & ~(VEC - 1)) : 0;
    const uint4 *src4 = reinterpret_cast<const uint4 *>(src);
#pragma unroll
    for (int u = 0; u < KV; u++) {
        const int i = VEC * (threadIdx.x + u * blockDim.x);
        r[u] = i < nv ? src4[i / VEC] : make_uint4(0u, 0u, 0u, 0u);
    }
    return nv;
}

// chunk_visit over a register-resident chunk (chunk_load); the columns past KV vectors per thread
// and the unaligned tail are read from memory.  Calls f(local column, value); no barrier.
template <int DT, int KV, class F>
__device__ __forceinline__ void chunk_visit_regs(const uint4 (&r)[KV], int nv, const void *src, const uint32_t *mrow,
                                                 int c0, int n, const ChunkPen &cp, const dllm_sampler_params &p,
                                                 unsigned flags, F &&f) {
    constexpr int VEC = DT == DLLM_DTYPE_BF16 ? 8 : 4;
    const int tid = threadIdx.x, NT = blockDim.x;
#pragma unroll
    for (int u = 0; u < KV; u++) {
        const int i = VEC * (tid + u * NT);
        if (i >= nv) continue;
        float x[VEC];
        if (DT == DLLM_DTYPE_BF16) {
            const uint32_t w4[4] = {r[u].x, r[u].y, r[u].z, r[u].w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                x[2 * j] = bitsf(w4[j] << 16);
                x[2 * j + 1] = bitsf(w4[j] & 0xffff0000u);
            }
        } else {
            x[0] = bitsf(r[u].x);
            x[1] = bitsf(r[u].y);
            x[2] = bitsf(r[u].z);
            x[3] = bitsf(r[u].w);
        }
        const uint32_t mw = mrow ? mrow[(c0 + i) >> 5] >> ((c0 + i) & 31) : 0xffffffffu;
        const uint32_t pw = cp.active ? cp.penbits[i >> 5] >> (i & 31) : 0u;
#pragma unroll
        for (int j = 0; j < VEC; j++)
            if (!((pw >> j) & 1u)) f(i + j, ((mw >> j) & 1u) ? x[j] : -INFINITY);
    }
    auto allowed = [&](int li) -> bool { return !mrow || ((mrow[(c0 + li) >> 5] >> ((c0 + li) & 31)) & 1u); };
    // columns past the registers: the unaligned tail, or all of a chunk longer than KV vectors a thread
    for (int i = min(nv, VEC * KV * NT) + tid; i < n; i += NT) {
        if (cp.active && ((cp.penbits[i >> 5] >> (i & 31)) & 1u)) continue;
        f(i, allowed(i) ? chunk_raw(src, DT, i) : -INFINITY);
    }
    if (cp.active) {
        const float inv_rep = __fdiv_rn(1.0f, p.repetition);
        const bool true_div = (flags & DLLM_MODE_PEN_TRUE_DIV) != 0;
        for (int sl = tid; sl < CH_HTAB; sl += NT) {
            const int li = cp.hkeys[sl];
            if (li < 0) continue;
            const float raw = allowed(li) ? chunk_raw(src, DT, li) : -INFINITY;
            f(li, penalise(raw, cp.hcnt[sl], p, true_div, inv_rep));
        }
    }
}

// The value of one column (for scans in column order).
template <int DT>
__device__ __forceinline__ float chunk_value(const void *src, const uint32_t *mrow, int c0, int li, const ChunkPen &cp,
                                             const dllm_sampler_params &p, unsigned flags) {
    const float raw = (!mrow || ((mrow[(c0 + li) >> 5] >> ((c0 + li) & 31)) & 1u)) ? chunk_raw(src, DT, li) : -INFINITY;
    if (!cp.active || !((cp.penbits[li >> 5] >> (li & 31)) & 1u)) return raw;
    uint32_t h = hash_id((uint32_t)li) & (CH_HTAB - 1);
    for (int probe = 0; probe < CH_HTAB; probe++) {
        if (cp.hkeys[h] == li)
            return penalise(raw, cp.hcnt[h], p, (flags & DLLM_MODE_PEN_TRUE_DIV) != 0, __fdiv_rn(1.0f, p.repetition));
        h = (h + 1u) & (CH_HTAB - 1);
    }
    return raw;
}

}  // namespace
}  // namespace dllm
