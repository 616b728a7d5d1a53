// dllm_sorted.cu -- sorted-nucleus mode (DLLM_MODE_TOPP_SORTED), which is not the reference's
// behaviour but the sampler its comments describe.
//
// With top-k off the reference keeps a top-p prefix in token-id order (src/sampler.c:165-170 sort
// only under top-k; the loop at 204-222 walks work_buf as it stands) and draws with a float
// running sum that drifts by ~1e-5 over 256000 entries (224-233).  This mode samples from the
// true nucleus, defined exactly:
//   order by (t desc, id asc), t = (x - max) * (1/temp) as src/sampler.c:153-162;
//   mass E = rint(expf(t) * 2^42), an integer, so every prefix sum is exact;
//   min-p: the sorted prefix with (float)(expf(t) * inv_sum) >= threshold (absolute min_p as
//   src/sampler.c:188-196, or min_p * p_max with DLLM_MODE_MINP_RELATIVE);
//   top-p: the shortest prefix whose mass reaches top_p * (kept mass); draw: the first entry
//   whose inclusive prefix mass exceeds floor(r * S3), S3 the mass of the nucleus.
//
// The row is never sorted.  Each selection -- "the first entry, in sorted order, whose
// inclusive prefix mass exceeds T" -- is a radix descent over the keys okey(t): histograms of
// mass per digit (12, 12 and 8 bits from the top), built by a pass over the row's 8192-column
// chunks, give the digit where the prefix mass crosses T.  Once a digit holds at most SO_CAP
// entries they are collected and the descent finishes in shared memory; entries with equal keys
// have equal mass and are ranked by id (the id order within a key is the column order, so a
// per-chunk count and one ordered scan find the m-th when too many entries tie).
//
// Kernels (stream-ordered, no host synchronisation, so a call can be graph-captured):
//   sorted_init_kernel     per-row state, the first work list
//   sorted_pass_kernel     CTAs over (chunk, listed row): MAX / SUM / HIST / COLLECT /
//                          TIECOUNT / LOCATE / PROBS, as the row's state asks
//   sorted_resolve_kernel  CTAs over listed rows: reads what the pass produced, advances the
//                          row's selections as far as the data allows, lists the row again when
//                          it needs another pass
//   sorted_finish_kernel   tokens of rows that ended early, status bits
// A fixed number of pass/resolve rounds is launched (enough for the deepest case); rounds with
// no listed rows cost two near-empty launches.
#include <cuda_runtime.h>
#include <stdlib.h>

#include "dllm_chunk.cuh"

namespace dllm {
namespace {

constexpr int SO_T = 256;         // threads per pass CTA
constexpr int SO_CHUNK = 8192;    // columns per pass CTA
constexpr int SO_BINS = 4096;     // 12-bit digits
constexpr int SO_CAP = 32768;     // collected candidates per row
constexpr int SO_RT = 1024;       // threads per resolve CTA
constexpr int SO_ROUNDS = 12;     // pass/resolve rounds (MAX + SUM + H0 + 2 x 4 descents + PROBS)
constexpr float SO_FX = 4398046511104.0f;  // 2^42

enum : int { OP_NONE = 0, OP_MAX, OP_SUM, OP_HIST, OP_COLLECT, OP_TIECOUNT, OP_LOCATE, OP_PROBS };
enum : int { PH_DONE = 0, PH_MAX, PH_SUM, PH_H0, PH_SEL, PH_PROBS };

typedef unsigned long long u64;

struct __align__(16) SortedRow {
    // written by passes
    uint32_t max_key;  // atomicMax of okey(x)
    int flags;         // ROW_ERR_* (atomicOr)
    int ncand;         // COLLECT appends
    int found_id;      // LOCATE result
    u64 sall;          // SUM: mass of every entry
    // what the next pass does
    int op;
    uint32_t op_key;   // HIST / COLLECT: region prefix; TIECOUNT / LOCATE: the key
    int op_bits;       // region bits resolved (0, 12, 24)
    int op_chunk, op_rank;
    uint32_t kmin;     // min-p: smallest kept key (0 = no min-p cut)
    float M, inv_temp;
    // selection state
    int phase, sel;    // sel 0: top-p cut, 1: draw
    uint32_t prefix;
    int bits;
    u64 T, above, cnt, m;
    u64 S2, S3;
    uint32_t cut_key;
    int cut_id, has_cut;
    uint32_t cand_prefix;
    int cand_bits;     // region of the collected list, -1 none
    uint32_t hr_prefix;
    int hr_bits;       // region of the refinement histogram, -1 none
    int tie_state;     // 0 none, 1 counts of op_key per chunk ready, 2 located
    int token;
};

struct SortedArgs {
    const void *logits;
    int64_t row_stride;
    int dtype, vec_ok;
    const uint32_t *mask;
    int64_t mask_stride;
    const int32_t *hist_ids;
    const int64_t *hist_off;
    const float *uniforms;
    dllm_sampler_params bparams;
    const dllm_sampler_params *rparams;
    int rows, vocab, nchunks;
    unsigned flags;
    int zero_status;   // no other kernel writes status for these rows
    int32_t *token;
    float *probs;
    int64_t probs_stride;
    float *pen_out;
    int64_t pen_stride;
    int32_t *status;
    SortedRow *st;
    u64 *h0m;          // [rows][SO_BINS] mass per top digit
    uint32_t *h0c;     // [rows][SO_BINS] entries per top digit
    u64 *hrm;          // [rows][SO_BINS] refinement histogram
    uint32_t *hrc;
    uint32_t *ckey;    // [rows][SO_CAP]
    int32_t *cid;
    uint32_t *tiecnt;  // [rows][nchunks]
    int *list;         // [2][rows]
    int *count;        // [2]
};

__device__ __forceinline__ uint32_t tkey_of(float x, float M, float inv_temp) {
    return okey(__fmul_rn(__fsub_rn(x, M), inv_temp));
}
__device__ __forceinline__ u64 mass_of(uint32_t tk) { return __float2ull_rn(__fmul_rn(expf(okey_inv(tk)), SO_FX)); }
__device__ __forceinline__ bool in_region(uint32_t tk, uint32_t prefix, int bits) {
    return bits == 0 || (tk >> (32 - bits)) == prefix;
}
__device__ __forceinline__ uint32_t digit_of(uint32_t tk, int bits) {
    return bits == 0 ? tk >> 20 : bits == 12 ? (tk >> 8) & 4095u : tk & 255u;
}
__device__ __forceinline__ int digit_width(int bits) { return bits == 24 ? 8 : 12; }

__device__ __forceinline__ bool eligible(const dllm_sampler_params &p, int V) {
    return p.temperature > 0.0f && !(p.top_k > 0 && p.top_k < V);
}

__global__ void sorted_init_kernel(const SortedArgs a) {
    const int row = blockIdx.x, tid = threadIdx.x;
    const dllm_sampler_params p = a.rparams ? a.rparams[row] : a.bparams;
    if (!eligible(p, a.vocab)) return;
    for (int i = tid; i < SO_BINS; i += blockDim.x) {
        a.h0m[(int64_t)row * SO_BINS + i] = 0ull;
        a.h0c[(int64_t)row * SO_BINS + i] = 0u;
    }
    if (tid == 0) {
        SortedRow s = {};
        s.op = OP_MAX;
        s.phase = PH_MAX;
        s.cand_bits = -1;
        s.hr_bits = -1;
        s.token = 0;
        a.st[row] = s;
        if (a.zero_status && a.status) a.status[row] = 0;
        const int pos = atomicAdd(&a.count[0], 1);
        a.list[pos] = row;
    }
}

// ---------------------------------------------------------------------------------------------
// passes

template <class T, class Op>
__device__ __forceinline__ T block_reduce_so(T v, T *scratch, Op op, T ident) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_allreduce(v, op);
    if (lane == 0) scratch[wid] = v;
    __syncthreads();
    T r = ident;
    for (int w = 0; w < nw; w++) r = op(r, scratch[w]);
    __syncthreads();
    return r;
}

template <int DT>
__global__ void __launch_bounds__(SO_T, 3) sorted_pass_kernel(const SortedArgs a, int par) {
    extern __shared__ __align__(16) unsigned char so_dyn[];
    __shared__ int hkeys[CH_HTAB];
    __shared__ int hcnt[CH_HTAB];
    __shared__ uint32_t penbits[SO_CHUNK / 32];
    __shared__ u64 red_u[SO_T / 32];
    __shared__ uint32_t red_k[SO_T / 32];
    __shared__ int s_flags, s_found, s_base;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, NT = blockDim.x;
    const int ch = blockIdx.x;
    if (ch == 0 && blockIdx.y == 0 && tid == 0) a.count[par ^ 1] = 0;  // the list this round's resolve fills
    const int items = a.count[par];
    const int *lst = a.list + (size_t)par * a.rows;
    const int c0 = ch * SO_CHUNK, n = min(SO_CHUNK, a.vocab - c0);
    const size_t esz = DT == DLLM_DTYPE_BF16 ? 2 : 4;
    constexpr int KV = SO_CHUNK / ((DT == DLLM_DTYPE_BF16 ? 8 : 4) * SO_T);  // 16-byte vectors per thread

    // the next item's row and operation are fetched while the current one is processed
    int row_n = blockIdx.y < items ? lst[blockIdx.y] : 0;
    int op_n = blockIdx.y < items ? a.st[row_n].op : OP_NONE;
    for (int j = blockIdx.y; j < items; j += gridDim.y) {
        const int row = row_n, op = op_n;
        SortedRow *st = a.st + row;
        const int jn = j + gridDim.y;
        row_n = jn < items ? lst[jn] : 0;
        if (op == OP_NONE || (op == OP_LOCATE && ch != st->op_chunk)) {
            op_n = jn < items ? a.st[row_n].op : OP_NONE;
            continue;
        }
        const dllm_sampler_params p = a.rparams ? a.rparams[row] : a.bparams;
        const float M = st->M, inv_temp = st->inv_temp;
        const uint32_t kmin = st->kmin, key = st->op_key;
        const int bits = st->op_bits;
        const uint32_t *mrow = a.mask ? a.mask + (int64_t)row * a.mask_stride : nullptr;
        const unsigned char *src = (const unsigned char *)a.logits + ((int64_t)row * a.row_stride + c0) * esz;
        uint4 r[KV];
        const int nv = chunk_load<DT, KV>(src, a.vec_ok && op != OP_LOCATE, n, r);
        ChunkPen cp{hkeys, hcnt, penbits, &s_flags, pen_active(a.hist_ids, a.hist_off, p)};
        const HistPre hp = hist_prefetch(a.hist_ids, a.hist_off, row, cp.active);
        if (tid == 0) {
            s_flags = 0;
            s_found = -1;
        }
        op_n = jn < items ? a.st[row_n].op : OP_NONE;
        chunk_pen_build(cp, a.hist_ids, hp, 0, a.vocab, c0, n, SO_CHUNK / 32);

        if (op == OP_MAX) {
            uint32_t km = 0u;
            float *pen = a.pen_out ? a.pen_out + (int64_t)row * a.pen_stride + c0 : nullptr;
            chunk_visit_regs<DT, KV>(r, nv, src, mrow, c0, n, cp, p, a.flags, [&](int li, float x) {
                km = max(km, okey(x));
                if (pen) pen[li] = x;
            });
            km = block_reduce_so(km, red_k, [](uint32_t x, uint32_t y) { return max(x, y); }, 0u);
            if (tid == 0) {
                atomicMax(&st->max_key, km);
                if (s_flags) atomicOr(&st->flags, s_flags);
            }
        } else if (op == OP_SUM) {
            u64 acc = 0ull;
            chunk_visit_regs<DT, KV>(r, nv, src, mrow, c0, n, cp, p, a.flags,
                            [&](int, float x) { acc += mass_of(tkey_of(x, M, inv_temp)); });
            acc = block_reduce_so(acc, red_u, [](u64 x, u64 y) { return x + y; }, 0ull);
            if (tid == 0 && acc) atomicAdd(&st->sall, acc);
        } else if (op == OP_HIST) {
            u64 *gm = (bits == 0 ? a.h0m : a.hrm) + (int64_t)row * SO_BINS;
            uint32_t *gc = (bits == 0 ? a.h0c : a.hrc) + (int64_t)row * SO_BINS;
            {
                // exact masses (< 2^43) as three 16-bit limbs: a chunk's limb sums stay below 2^32
                uint32_t *l0 = reinterpret_cast<uint32_t *>(so_dyn), *l1 = l0 + SO_BINS, *l2 = l1 + SO_BINS;
                uint32_t *cn = l2 + SO_BINS;
                for (int i = tid; i < 4 * SO_BINS; i += NT) l0[i] = 0u;
                __syncthreads();
                chunk_visit_regs<DT, KV>(r, nv, src, mrow, c0, n, cp, p, a.flags, [&](int, float x) {
                    const uint32_t tk = tkey_of(x, M, inv_temp);
                    if (tk < kmin || !in_region(tk, key, bits)) return;
                    const u64 e = mass_of(tk);
                    if (!e) return;
                    const uint32_t d = digit_of(tk, bits);
                    atomicAdd(&l0[d], (uint32_t)e & 0xffffu);
                    atomicAdd(&l1[d], (uint32_t)(e >> 16) & 0xffffu);
                    atomicAdd(&l2[d], (uint32_t)(e >> 32));
                    atomicAdd(&cn[d], 1u);
                });
                __syncthreads();
                for (int i = tid; i < SO_BINS; i += NT)
                    if (cn[i]) {
                        atomicAdd(&gm[i], (u64)l0[i] + ((u64)l1[i] << 16) + ((u64)l2[i] << 32));
                        atomicAdd(&gc[i], cn[i]);
                    }
            }
        } else if (op == OP_COLLECT) {
            uint32_t *ck = a.ckey + (int64_t)row * SO_CAP;
            int32_t *ci = a.cid + (int64_t)row * SO_CAP;
            chunk_visit_regs<DT, KV>(r, nv, src, mrow, c0, n, cp, p, a.flags, [&](int li, float x) {
                const uint32_t tk = tkey_of(x, M, inv_temp);
                if (tk < kmin || !in_region(tk, key, bits) || !mass_of(tk)) return;
                const int pos = atomicAdd(&st->ncand, 1);
                if (pos < SO_CAP) {
                    ck[pos] = tk;
                    ci[pos] = c0 + li;
                }
            });
        } else if (op == OP_TIECOUNT) {
            uint32_t cnt = 0u;
            chunk_visit_regs<DT, KV>(r, nv, src, mrow, c0, n, cp, p, a.flags,
                            [&](int, float x) { cnt += tkey_of(x, M, inv_temp) == key; });
            cnt = block_reduce_so(cnt, red_k, [](uint32_t x, uint32_t y) { return x + y; }, 0u);
            if (tid == 0) a.tiecnt[(int64_t)row * a.nchunks + ch] = cnt;
        } else if (op == OP_LOCATE) {
            // the op_rank-th column (0-based, column order) of this chunk whose key is op_key
            const int rank = st->op_rank;
            if (tid == 0) s_base = 0;
            __syncthreads();
            for (int base = 0; base < n; base += NT) {
                const int li = base + tid;
                const bool eq = li < n && tkey_of(chunk_value<DT>(src, mrow, c0, li, cp, p, a.flags), M, inv_temp) == key;
                const unsigned bm = __ballot_sync(0xffffffffu, eq);
                if (lane == 0) red_k[wid] = __popc(bm);
                __syncthreads();
                int before = s_base;
                for (int w = 0; w < wid; w++) before += red_k[w];
                const int r = before + __popc(bm & ((1u << lane) - 1u));
                if (eq && r == rank) s_found = c0 + li;
                __syncthreads();
                if (tid == 0) {
                    int tot = 0;
                    for (int w = 0; w < NT / 32; w++) tot += red_k[w];
                    s_base += tot;
                }
                __syncthreads();
                if (s_found >= 0 || s_base > rank) break;
            }
            if (tid == 0) st->found_id = s_found;
        } else if (op == OP_PROBS) {
            float *pr = a.probs + (int64_t)row * a.probs_stride + c0;
            const int has_cut = st->has_cut, cut_id = st->cut_id;
            const uint32_t cut_key = st->cut_key;
            const double inv3 = 1.0 / (double)st->S3;
            chunk_visit_regs<DT, KV>(r, nv, src, mrow, c0, n, cp, p, a.flags, [&](int li, float x) {
                const uint32_t tk = tkey_of(x, M, inv_temp);
                const bool kept = tk >= kmin && (!has_cut || tk > cut_key || (tk == cut_key && c0 + li <= cut_id));
                pr[li] = kept ? __double2float_rn((double)mass_of(tk) * inv3) : 0.0f;
            });
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------------------------
// resolve

// Block scan over the digits of a histogram, from the highest digit down: the digit where the
// inclusive mass first exceeds R, and the mass of the digits above it.
__device__ void scan_desc(const u64 *hm, int D, u64 R, u64 *red, int *s_digit, u64 *s_excl) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;
    const int per = (D + blockDim.x - 1) / blockDim.x;  // 4 for 4096 bins, 1 for 256
    u64 mine = 0ull;
    for (int k = 0; k < per; k++) {
        const int d = D - 1 - (tid * per + k);
        if (d >= 0) mine += hm[d];
    }
    u64 incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const u64 y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) red[wid] = incl;
    __syncthreads();
    u64 woff = 0ull;
    for (int w = 0; w < wid; w++) woff += red[w];
    (void)nw;
    const u64 excl = woff + incl - mine;
    if (excl <= R && R < excl + mine) {
        u64 run = excl;
        for (int k = 0; k < per; k++) {
            const int d = D - 1 - (tid * per + k);
            if (d < 0) break;
            if (run + hm[d] > R) {
                *s_digit = d;
                *s_excl = run;
                break;
            }
            run += hm[d];
        }
    }
    __syncthreads();
}

// Ascending counterpart over counts: the digit where the inclusive count first exceeds m.
__device__ void scan_asc_count(const uint32_t *hc, int D, u64 m, u64 *red, int *s_digit, u64 *s_excl) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int per = (D + blockDim.x - 1) / blockDim.x;
    u64 mine = 0ull;
    for (int k = 0; k < per; k++) {
        const int d = tid * per + k;
        if (d < D) mine += hc[d];
    }
    u64 incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const u64 y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) red[wid] = incl;
    __syncthreads();
    u64 woff = 0ull;
    for (int w = 0; w < wid; w++) woff += red[w];
    const u64 excl = woff + incl - mine;
    if (excl <= m && m < excl + mine) {
        u64 run = excl;
        for (int k = 0; k < per; k++) {
            const int d = tid * per + k;
            if (d >= D) break;
            if (run + hc[d] > m) {
                *s_digit = d;
                *s_excl = run;
                break;
            }
            run += hc[d];
        }
    }
    __syncthreads();
}

// Copies the row's collected keys into shared memory once per resolve of the row.  Ends with a barrier.
__device__ void load_cands(uint32_t *ck, const uint32_t *gck, int nc, int *s_cands) {
    const int have = *s_cands;
    __syncthreads();
    if (!have)
        for (int i = threadIdx.x; i < nc; i += blockDim.x) ck[i] = gck[i];
    __syncthreads();
    if (threadIdx.x == 0) *s_cands = 1;
}

__global__ void __launch_bounds__(SO_RT) sorted_resolve_kernel(const SortedArgs a, int par) {
    extern __shared__ __align__(16) unsigned char rs_dyn[];
    u64 *hm = reinterpret_cast<u64 *>(rs_dyn);                  // SO_BINS
    uint32_t *hc = reinterpret_cast<uint32_t *>(hm + SO_BINS);  // SO_BINS
    uint32_t *ck = hc + SO_BINS;                                // SO_CAP candidate keys
    __shared__ SortedRow s;
    __shared__ u64 red[SO_RT / 32];
    __shared__ int s_digit, s_cands, s_ld_bits;
    __shared__ uint32_t s_ld_prefix;
    __shared__ u64 s_excl;
    const int tid = threadIdx.x, NT = blockDim.x;
    const int items = a.count[par];
    const int *lst = a.list + (size_t)par * a.rows;
    int *out = a.list + (size_t)(par ^ 1) * a.rows;

    for (int j = blockIdx.x; j < items; j += gridDim.x) {
        const int row = lst[j];
        if (tid == 0) {
            s = a.st[row];
            s.op = OP_NONE;
            s_cands = 0;
            s_ld_bits = -1;
        }
        __syncthreads();
        const dllm_sampler_params p = a.rparams ? a.rparams[row] : a.bparams;
        const float r = a.uniforms[row];
        const u64 *g0m = a.h0m + (int64_t)row * SO_BINS, *grm = a.hrm + (int64_t)row * SO_BINS;
        const uint32_t *g0c = a.h0c + (int64_t)row * SO_BINS, *grc = a.hrc + (int64_t)row * SO_BINS;
        const uint32_t *gck = a.ckey + (int64_t)row * SO_CAP;
        const int32_t *gci = a.cid + (int64_t)row * SO_CAP;

        for (int guard = 0; guard < 64; guard++) {
            __syncthreads();
            if (s.phase == PH_DONE || s.op != OP_NONE) break;
            const int phase = s.phase;
            if (phase == PH_MAX || phase == PH_SUM || phase == PH_PROBS) {
                if (tid == 0) {
                    if (phase == PH_PROBS) {
                        s.phase = PH_DONE;
                    } else if (phase == PH_MAX) {
                        const float M = okey_inv(s.max_key);
                        if (M == -INFINITY) {
                            // fully masked row: every t is NaN in the reference, whose list stays
                            // in id order and returns its last entry
                            s.token = a.vocab - 1;
                            s.phase = PH_DONE;
                        } else if (!(M < INFINITY) || M != M) {
                            s.flags |= ROW_ERR_NONFINITE;
                            s.token = 0;
                            s.phase = PH_DONE;
                        } else {
                            s.M = M;
                            s.inv_temp = __fdiv_rn(1.0f, p.temperature);
                            s.kmin = 0u;
                            if (p.min_p > 0.0f) {
                                s.sall = 0ull;
                                s.op = OP_SUM;
                                s.phase = PH_SUM;
                            } else {
                                s.op = OP_HIST;
                                s.op_key = 0u;
                                s.op_bits = 0;
                                s.phase = PH_H0;
                            }
                        }
                    } else {  // PH_SUM: the min-p threshold as a key (the kept entries are a prefix)
                        const float inv_sum = __double2float_rn(1.0 / ((double)s.sall * 0x1p-42));
                        const float thr = (a.flags & DLLM_MODE_MINP_RELATIVE) ? __fmul_rn(p.min_p, inv_sum) : p.min_p;
                        auto keep = [&](uint32_t k) { return __fmul_rn(expf(okey_inv(k)), inv_sum) >= thr; };
                        const uint32_t ktop = okey(0.0f);
                        if (!keep(ktop)) {
                            s.kmin = 0u;  // nothing passes: the reference keeps the whole list
                        } else {
                            uint32_t lo = 0u, hi = ktop;  // keep(hi) holds; find the smallest such key
                            while (lo < hi) {
                                const uint32_t mid = lo + (hi - lo) / 2u;
                                if (keep(mid)) hi = mid;
                                else lo = mid + 1u;
                            }
                            s.kmin = hi;
                        }
                        s.op = OP_HIST;
                        s.op_key = 0u;
                        s.op_bits = 0;
                        s.phase = PH_H0;
                    }
                }
                continue;
            }
            if (phase == PH_H0) {
                for (int i = tid; i < SO_BINS; i += NT) {
                    hm[i] = g0m[i];
                    hc[i] = g0c[i];
                }
                u64 part = 0ull;
                for (int i = tid; i < SO_BINS; i += NT) part += g0m[i];
                const u64 S2 = block_reduce_so(part, red, [](u64 x, u64 y) { return x + y; }, 0ull);
                if (tid == 0) {
                    s_ld_bits = 0;
                    s_ld_prefix = 0u;
                    s.S2 = S2;
                    s.phase = PH_SEL;
                    s.above = 0ull;
                    s.prefix = 0u;
                    s.bits = 0;
                    s.tie_state = 0;
                    if (p.top_p < 1.0f) {
                        const double x = ceil((double)p.top_p * (double)S2);
                        s.sel = 0;
                        s.T = (x < 1.0 ? 1ull : (u64)x) - 1ull;
                    } else {
                        s.sel = 1;
                        s.has_cut = 0;
                        s.S3 = S2;
                        s.T = (u64)floor((double)r * (double)S2);
                    }
                }
                continue;
            }
            // ---- PH_SEL
            if (s.bits == 32) {
                const uint32_t K = s.prefix;
                bool found = false;
                int fid = 0;
                const bool covered = s.cand_bits >= 0 && (s.cand_bits == 0 || (K >> (32 - s.cand_bits)) == s.cand_prefix);
                if (tid == 0) s.m = (s.T - s.above) / mass_of(K);
                __syncthreads();
                if (s.tie_state == 2) {
                    found = true;
                    fid = s.found_id;
                } else if (covered) {
                    // the m-th smallest id among the collected entries with key K (ids < 2^24)
                    const int nc = min(s.ncand, SO_CAP);
                    load_cands(ck, gck, nc, &s_cands);
                    for (int i = tid; i < SO_BINS; i += NT) hc[i] = 0u;
                    if (tid == 0) s_digit = -1;
                    __syncthreads();
                    for (int i = tid; i < nc; i += NT)
                        if (ck[i] == K) atomicAdd(&hc[(uint32_t)gci[i] >> 12], 1u);
                    __syncthreads();
                    scan_asc_count(hc, SO_BINS, s.m, red, &s_digit, &s_excl);
                    const int hi_d = s_digit;
                    const u64 m2 = s.m - s_excl;
                    __syncthreads();
                    for (int i = tid; i < SO_BINS; i += NT) hc[i] = 0u;
                    if (tid == 0) s_digit = -1;
                    __syncthreads();
                    if (hi_d >= 0)
                        for (int i = tid; i < nc; i += NT)
                            if (ck[i] == K && ((uint32_t)gci[i] >> 12) == (uint32_t)hi_d)
                                atomicAdd(&hc[(uint32_t)gci[i] & 4095u], 1u);
                    __syncthreads();
                    scan_asc_count(hc, SO_BINS, m2, red, &s_digit, &s_excl);
                    found = true;
                    fid = (hi_d < 0 || s_digit < 0) ? -1 : (hi_d << 12) | s_digit;
                    if (tid == 0) s_ld_bits = -1;  // hm / hc were reused
                } else if (s.tie_state == 1 && s.op_key == K) {
                    if (tid == 0) {
                        u64 before = 0ull;
                        int c = 0;
                        for (; c < a.nchunks; c++) {
                            const uint32_t t = a.tiecnt[(int64_t)row * a.nchunks + c];
                            if (before + t > s.m) break;
                            before += t;
                        }
                        if (c == a.nchunks) {  // inconsistent counts: give up on this row
                            s.flags |= ROW_ERR_WALK;
                            s.token = 0;
                            s.phase = PH_DONE;
                        } else {
                            s.op = OP_LOCATE;
                            s.op_chunk = c;
                            s.op_rank = (int)(s.m - before);
                            s.tie_state = 2;
                        }
                    }
                    continue;
                } else {
                    if (tid == 0) {
                        s.op = OP_TIECOUNT;
                        s.op_key = K;
                        s.tie_state = 1;
                    }
                    continue;
                }
                if (found && tid == 0) {
                    const u64 cum = s.above + (s.m + 1ull) * mass_of(K);
                    s.tie_state = 0;
                    if (fid < 0) {
                        s.flags |= ROW_ERR_WALK;
                        s.token = 0;
                        s.phase = PH_DONE;
                    } else if (s.sel == 0) {
                        s.has_cut = 1;
                        s.cut_key = K;
                        s.cut_id = fid;
                        s.S3 = cum;
                        s.sel = 1;
                        s.T = (u64)floor((double)r * (double)cum);
                        s.above = 0ull;
                        s.prefix = 0u;
                        s.bits = 0;
                    } else {
                        s.token = fid;
                        if (a.probs) {
                            s.op = OP_PROBS;
                            s.phase = PH_PROBS;
                        } else {
                            s.phase = PH_DONE;
                        }
                    }
                }
                continue;
            }
            // region (prefix, bits) with bits < 32: its histogram over the next digit
            const uint32_t P = s.prefix;
            const int B = s.bits;
            if (!(s_ld_bits == B && s_ld_prefix == P)) {
                const bool covered = s.cand_bits >= 0 && s.cand_bits <= B &&
                                     (s.cand_bits == 0 || (P >> (B - s.cand_bits)) == s.cand_prefix);
                if (B == 0 || (s.hr_bits == B && s.hr_prefix == P)) {
                    const u64 *gm = B == 0 ? g0m : grm;
                    const uint32_t *gc = B == 0 ? g0c : grc;
                    for (int i = tid; i < SO_BINS; i += NT) {
                        hm[i] = gm[i];
                        hc[i] = gc[i];
                    }
                } else if (covered) {
                    const int nc = min(s.ncand, SO_CAP);
                    load_cands(ck, gck, nc, &s_cands);
                    for (int i = tid; i < SO_BINS; i += NT) {
                        hm[i] = 0ull;
                        hc[i] = 0u;
                    }
                    __syncthreads();
                    for (int i = tid; i < nc; i += NT) {
                        const uint32_t tk = ck[i];
                        if ((tk >> (32 - B)) != P) continue;
                        const uint32_t d = digit_of(tk, B);
                        atomicAdd(&hm[d], mass_of(tk));
                        atomicAdd(&hc[d], 1u);
                    }
                } else if (s.cnt <= (u64)SO_CAP) {
                    if (tid == 0) {
                        s.op = OP_COLLECT;
                        s.op_key = P;
                        s.op_bits = B;
                        s.ncand = 0;
                        s.cand_prefix = P;
                        s.cand_bits = B;
                        s_cands = 0;
                    }
                    continue;
                } else {
                    u64 *wm = a.hrm + (int64_t)row * SO_BINS;
                    uint32_t *wc = a.hrc + (int64_t)row * SO_BINS;
                    for (int i = tid; i < SO_BINS; i += NT) {
                        wm[i] = 0ull;
                        wc[i] = 0u;
                    }
                    if (tid == 0) {
                        s.op = OP_HIST;
                        s.op_key = P;
                        s.op_bits = B;
                        s.hr_prefix = P;
                        s.hr_bits = B;
                    }
                    continue;
                }
                __syncthreads();
                if (tid == 0) {
                    s_ld_bits = B;
                    s_ld_prefix = P;
                }
            }
            const int w = digit_width(B);
            if (tid == 0) s_digit = -1;
            __syncthreads();
            scan_desc(hm, 1 << w, s.T - s.above, red, &s_digit, &s_excl);
            if (tid == 0) {
                if (s_digit < 0) {  // the region's mass does not reach T: inconsistent state
                    s.flags |= ROW_ERR_WALK;
                    s.token = 0;
                    s.phase = PH_DONE;
                } else {
                    s.above += s_excl;
                    s.prefix = (P << w) | (uint32_t)s_digit;
                    s.bits = B + w;
                    s.cnt = hc[s_digit];
                }
            }
        }
        __syncthreads();
        if (tid == 0) {
            if (s.phase != PH_DONE && s.op == OP_NONE) {  // ran out of steps
                s.flags |= ROW_ERR_WALK;
                s.phase = PH_DONE;
            }
            if (s.phase == PH_DONE) s.op = OP_NONE;
            a.st[row] = s;
            if (s.op != OP_NONE) {
                const int pos = atomicAdd(&a.count[par ^ 1], 1);
                out[pos] = row;
            }
        }
        __syncthreads();
    }
}

__global__ void sorted_finish_kernel(const SortedArgs a) {
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= a.rows) return;
    const dllm_sampler_params p = a.rparams ? a.rparams[row] : a.bparams;
    if (!eligible(p, a.vocab)) return;
    SortedRow *s = a.st + row;
    int flags = s->flags;
    if (s->phase != PH_DONE) flags |= ROW_ERR_WALK;
    a.token[row] = s->phase == PH_DONE ? s->token : 0;
    if (a.status && flags) atomicOr(&a.status[row], flags);
}

}  // namespace

size_t sorted_ws_bytes(int rows, int vocab) {
    const size_t nch = (size_t)(vocab + SO_CHUNK - 1) / SO_CHUNK;
    const size_t per = sizeof(SortedRow) + (size_t)SO_BINS * (8 + 4) * 2 + (size_t)SO_CAP * 8 + nch * 4 + 2 * 4;
    return 256 + (size_t)rows * ((per + 255) & ~(size_t)255);
}

dllm_status launch_sorted(const dllm_batch_desc *d, bool after_fused, void *ws, cudaStream_t stream) {
    if (d->vocab > (1 << 21)) return DLLM_ERR_UNSUPPORTED;  // 2^42-scaled masses of 2^21 entries fit 64 bits
    SortedArgs a = {};
    a.logits = d->logits;
    a.row_stride = d->row_stride;
    a.dtype = d->dtype;
    const int vec = d->dtype == DLLM_DTYPE_F32 ? 4 : 8;
    a.vec_ok = ((uintptr_t)d->logits % 16 == 0) && (d->row_stride % vec == 0);
    a.mask = d->mask;
    a.mask_stride = d->mask_stride;
    a.hist_ids = d->hist_ids;
    a.hist_off = d->hist_off;
    a.uniforms = d->uniforms;
    a.bparams = d->params;
    a.rparams = d->row_params;
    a.rows = d->rows;
    a.vocab = d->vocab;
    a.nchunks = (d->vocab + SO_CHUNK - 1) / SO_CHUNK;
    a.flags = d->flags;
    a.zero_status = !after_fused;
    a.token = d->token;
    a.probs = d->probs;
    a.probs_stride = d->probs_stride;
    a.pen_out = after_fused ? nullptr : d->pen_logits;  // the fused kernel wrote them already
    a.pen_stride = d->pen_stride;
    a.status = d->status;
    // workspace carve-up
    unsigned char *w = (unsigned char *)ws;
    const size_t R = (size_t)d->rows;
    a.count = reinterpret_cast<int *>(w);
    w += 256;
    a.st = reinterpret_cast<SortedRow *>(w);
    w += R * sizeof(SortedRow);
    a.h0m = reinterpret_cast<u64 *>(w);
    w += R * SO_BINS * 8;
    a.hrm = reinterpret_cast<u64 *>(w);
    w += R * SO_BINS * 8;
    a.h0c = reinterpret_cast<uint32_t *>(w);
    w += R * SO_BINS * 4;
    a.hrc = reinterpret_cast<uint32_t *>(w);
    w += R * SO_BINS * 4;
    a.ckey = reinterpret_cast<uint32_t *>(w);
    w += R * SO_CAP * 4;
    a.cid = reinterpret_cast<int32_t *>(w);
    w += R * SO_CAP * 4;
    a.tiecnt = reinterpret_cast<uint32_t *>(w);
    w += R * a.nchunks * 4;
    a.list = reinterpret_cast<int *>(w);

    const void *pass = d->dtype == DLLM_DTYPE_BF16 ? (const void *)sorted_pass_kernel<DLLM_DTYPE_BF16>
                                                   : (const void *)sorted_pass_kernel<DLLM_DTYPE_F32>;
    const int pass_smem = SO_BINS * 16;
    const int res_smem = SO_BINS * (8 + 4) + SO_CAP * 4;
    if (cudaFuncSetAttribute(pass, cudaFuncAttributeMaxDynamicSharedMemorySize, pass_smem) != cudaSuccess ||
        cudaFuncSetAttribute((const void *)sorted_resolve_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             res_smem) != cudaSuccess)
        return DLLM_ERR_CUDA;
    int dev = 0, sms = 148, per_sm = 1;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, pass, SO_T, pass_smem);
    const int gy = min(a.rows, max(1, (8 * sms * max(per_sm, 1) + a.nchunks - 1) / a.nchunks));
    const int gr = min(a.rows, sms);

    if (cudaMemsetAsync(a.count, 0, 2 * sizeof(int), stream) != cudaSuccess) return DLLM_ERR_CUDA;
    sorted_init_kernel<<<a.rows, 256, 0, stream>>>(a);
    for (int round = 0; round < SO_ROUNDS; round++) {
        const int par = round & 1;
        if (d->dtype == DLLM_DTYPE_BF16)
            sorted_pass_kernel<DLLM_DTYPE_BF16><<<dim3(a.nchunks, gy), SO_T, pass_smem, stream>>>(a, par);
        else
            sorted_pass_kernel<DLLM_DTYPE_F32><<<dim3(a.nchunks, gy), SO_T, pass_smem, stream>>>(a, par);
        sorted_resolve_kernel<<<gr, SO_RT, res_smem, stream>>>(a, par);
    }
    sorted_finish_kernel<<<(a.rows + 255) / 256, 256, 0, stream>>>(a);
    return cudaGetLastError() == cudaSuccess ? DLLM_OK : DLLM_ERR_CUDA;
}

}  // namespace dllm
