// dllm_kernel.cuh -- fused batched sampler for B200 (sm_100a): device code.
// Included by dllm_kernel_inst.cu, which is compiled once per sub-chunk length.
//
// Two kernels per batch.
//
// Kernel A (sample_rows_kernel): one thread-block cluster samples one row at a time (persistent
// over rows).  The row is split into C contiguous slices, one per CTA; each slice is copied from
// HBM once into shared memory with a bulk (TMA) copy while the next row's slice is prefetched
// into L2, and every later pass reads shared memory.  A slice is 4 * NT sub-chunks of SUB
// elements (SUB compile-time, SUB % 8 == 4 so 16-byte shared loads of a warp are free of bank
// conflicts), in index order; thread t owns sub-chunks t, NT + t, 2NT + t, 3NT + t (one per
// quarter of the slice), which gives each thread four independent dependency chains.  Per row:
//
//   P1  bulk copy, grammar mask -> -inf, history penalties from an in-shared-memory hash table
//       (presence / frequency once per id, repetition once per occurrence), slice maximum
//                                                                         -> cluster max M
//   greedy (temperature 0): first index holding M                        -> token
//   top-k (0 < k < V): per-thread maxima give a threshold with >= k elements at or above it;
//       the survivors are gathered into CTA 0, sorted by (t desc, id asc), the first k kept,
//       and softmax / min-p / top-p / draw run on that short list (a 4-pass radix select is
//       the fallback when too many elements survive the threshold)
//   otherwise (top-k off: the reference's index-order list):
//   P2  t = (x - M) * (1/T), e = exp(t - max_t) in place, fp32 sub-chunk sums -> cluster sum
//   P2b min-p (absolute threshold) kept count / renormalisation sum      -> cluster sums
//   P3  sub-chunk sums of the list probabilities, exclusive scan over the cluster; the one warp
//       holding the sub-chunk where (float)cumsum first reaches top_p finds the cut element
//                                                                          -> cluster
//   P4  records for the exact emulation of the reference's sequential fp32 draw
//       (src/sampler.c:226-231).  Within one binade [2^e, 2^(e+1)) of the running sum c,
//       fl(c + q) = c + n*ulp(c), where n depends only on q and on the parity of c/ulp
//       (ties-to-even), so a run of adds is a function of one parity bit: (n_even, n_odd).  Each
//       thread computes that pair for its four sub-chunks (real fp32 chains started at 2^e and
//       2^e + ulp, e predicted from the exact double prefix), each warp composes its 32
//       sub-chunks of a quarter into a record (prefix run / one boundary sub-chunk / suffix run),
//       and the records, the boundary sub-chunks' probabilities and the row's scalars go to the
//       workspace.
//
// Kernel B (walk_rows_kernel): one warp per row composes the warp records in order on the exact
// running sum, checking every step's validity, replaying boundary sub-chunks in plain fp32
// (cooperatively, a few elements per lane), and descending into the region where the uniform
// falls, whose probabilities it recomputes from the row's inputs with the row's scalars.  The
// first id with r < c is the sample (or the list's last id when r reaches the total).
//
// Bit-exactness: the translation unit is built with -fmad=false and -ftz=true (the reference
// executables run with FTZ|DAZ); every operation that must round like the reference is an
// explicit __f*_rn intrinsic.
#pragma once
#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda/std/type_traits>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "dllm_internal.h"

#ifndef DLLM_TMA_PIECE
#define DLLM_TMA_PIECE (1 << 20)  // one bulk copy per slice (the mbarrier transaction count allows < 2^20 bytes)
#endif

namespace cg = cooperative_groups;

namespace dllm {

typedef void (*KernelFn)(const KernelArgs);

constexpr int MAXC_HDR = 16;  // = MAXC, the most CTAs per cluster
// Row scalars kept in the workspace for the walk kernel (128 bytes).
struct RowHdr {
    float M, inv_temp, mv, inv_sum, min_p, inv_s2, inv_s3, r;
    int cut_idx, last_idx, flags, done, minp, nokept, topp;
    int rank_flags[MAXC_HDR];  // status bits each CTA of the row's cluster saw (timeouts after #1)
    int pad[1];
};
static_assert(sizeof(RowHdr) == 128, "row_ws_bytes assumes a 128-byte row header");
// Warp-level draw record (24 bytes).  meta: type (bits 0-1), boundary sub-chunk (2-7, 63 =
// none), first suffix sub-chunk (8-13), prefix binade (16-23), suffix binade (24-31).
struct WRec {
    uint32_t meta;
    uint32_t p0, p1, s0, s1;
    int16_t nslot;  // PBS: stash slot holding the boundary sub-chunk's probabilities, or -1
    int16_t wslot;  // wide slot holding all 32 sub-chunks' probabilities, or -1
};

// everything below has internal linkage: this header is compiled into several units
namespace {

constexpr int MAXW = 16;          // warps per CTA (blockDim <= 512)
constexpr int MAXC = 16;          // CTAs per cluster
constexpr int CAND_CAP = 2048;    // top-k survivors gathered in CTA 0
constexpr int TMA_PIECE = DLLM_TMA_PIECE;  // bytes per bulk copy instruction
constexpr int WALK_WARPS = 4;     // rows per CTA of the walk kernel
constexpr int HLIST = 256;        // per-warp history ids kept for a recomputed region
constexpr float DRAW_WINDOW = 1.0f / 16384.0f;
// Relative difference of this kernel's exponential sums from the reference's (glibc's scalar and
// 4-wide vector expf), measured on B200 at most 4e-8 over the benchmark row distributions; with
// margin.  Used to flag top-p cuts the reference may place one entry away (ROW_TOPP_EDGE).
constexpr double TOPP_EXP_DIFF = 6e-8;
// one ulp of x relative to x (x a positive normal float)
__device__ __forceinline__ double ulp_rel(float x) {
    const uint32_t m = __float_as_uint(x) & 0x7fffffu;
    return 1.0 / (double)(0x800000u + m);
}  // bound assumed on |fp32 running sum - exact prefix|

enum : int { REC_IDENT = 0, REC_CLEAN = 1, REC_MIXED = 2, REC_PBS = 3 };

// Diagnostic counters: per-phase cycles of cluster rank 0 and walk statistics.  Thread 0 of
// every CTA stores KernelArgs::dbg here at kernel start (all store the same value).
__device__ unsigned long long *g_dbg = nullptr;
enum : int {
    DBG_P1 = 0, DBG_W1 = 1, DBG_P2 = 2, DBG_W2 = 3, DBG_P3 = 4, DBG_W3 = 5, DBG_CUT = 6,
    DBG_P4 = 7, DBG_WEND = 10, DBG_TOPK = 11, DBG_LOADWAIT = 12,
    DBG_ROWS = 16, DBG_REPLAY = 17, DBG_EXPAND = 18, DBG_STEPS = 19, DBG_REPLAY_IT = 20,
    DBG_PBS = 21, DBG_STASH_MISS = 22, DBG_TOPK_FALLBACK = 23, DBG_RECOMP = 24, DBG_WALK_CYC = 25,
    DBG_P2L = 13, DBG_P3L = 14, DBG_P3S = 15, DBG_P4L = 26, DBG_MAXP = 27, DBG_HBUILD = 30,
    DBG_COPY_EARLY = 31,
    DBG_B_PRE = 8, DBG_B_EXP = 9, DBG_B_REPL = 28, DBG_B_RECOMP = 29,
};
__device__ __forceinline__ void dbg_add(int k, unsigned long long v) {
    if (g_dbg) atomicAdd(g_dbg + k, v);
}

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

__device__ __forceinline__ RowHdr *row_hdr(const KernelArgs &a, int row) {
    return reinterpret_cast<RowHdr *>(a.ws + (size_t)row * row_ws_bytes(a.nrec, a.SUB));
}
__device__ __forceinline__ WRec *row_recs(const KernelArgs &a, int row) {
    return reinterpret_cast<WRec *>(reinterpret_cast<unsigned char *>(row_hdr(a, row)) + sizeof(RowHdr));
}
__device__ __forceinline__ float *row_stash(const KernelArgs &a, int row) {
    const size_t recb = ((size_t)a.nrec * sizeof(WRec) + 127) & ~(size_t)127;
    return reinterpret_cast<float *>(reinterpret_cast<unsigned char *>(row_hdr(a, row)) + sizeof(RowHdr) + recb);
}
// wide slots: the draw probabilities of all 32 sub-chunks of a MIXED warp record
__device__ __forceinline__ float *row_wide(const KernelArgs &a, int row) {
    return row_stash(a, row) + STASH_SLOTS * STASH_STRIDE;
}

// Values each CTA publishes to its cluster.  Every field is written at most once per row and
// read only after the cluster barrier that follows the write.
struct Xch {
    float m;
    float mt;
    double dsum;
    double s2;
    double s2all;
    int nkept;
    double tot;
    int first_member;
    float first_w;
    float first_e;    // exponential of the slice's first element
    int last_member;
    int cut_idx;
    int cut_flags;
    double cut_s3;
    int gidx;
    int flags;
    uint32_t theta;
    int cnt_gt, cnt_eq;
    int ncand;        // CTA 0: survivors gathered
    unsigned hist[2][256];
};

// Values pushed into every CTA of the cluster (st.async with mbarrier completion), one slot per
// source rank and row parity: #1 the penalised maximum, #2 the exponential sum, #4 the cut.
// (aligned to their size: st.async .v2 / .v4 destinations must be 8- / 16-byte aligned)
struct __align__(8) Push1 {
    float m;
    int flags;
};
struct __align__(16) Push2 {
    double dsum;
    float first_e;
    int pad;
};
struct __align__(16) Push4 {
    int cut_idx;
    int cut_flags;  // ROW_TOPP_EDGE when the prefix at the cut lies near the threshold
    double cut_s3;
};

struct Shared {
    Xch xs;
    unsigned long long tma_bar[2];
    unsigned long long xbar[3][2];  // push exchanges #1, #2, #4 by row parity
    Push1 in1[2][MAXC];
    Push2 in2[2][MAXC];
    Push4 in4[2][MAXC];
    static_assert(sizeof(Push1) == 8 && sizeof(Push2) == 16 && sizeof(Push4) == 16, "push payload sizes");
    int slots[2];                   // CTA 0: stash / wide slot claims by row parity
    double red_d[4 * MAXW];
    float red_f[MAXW];
    int red_i[4 * MAXW];
    int red_i2[MAXW];
    int bcast_i[4];
};

// Exponential of the index-order path, from the identity e^t = 2^(t * log2(e)) on the hardware
// base-2 exponential (PTX ex2.approx.ftz.f32, relative error about 2^-22): two instructions.  For
// t <= 0 the result is within about 2.5e-7 of e^t relative (the product's rounding adds
// |t| * 2^-24 * ln 2, which only matters where e^t is already tiny); -inf gives +0.  The
// reference's own softmax mixes glibc's scalar and 4-wide vector expf, which differ by up to
// 3 ulp, so agreement is to the sampler's probability tolerance, not to the bit.  The cluster
// kernel and the walk kernel both use this function, so they agree with each other exactly.
__device__ __forceinline__ float exp_t(float t) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(__fmul_rn(t, 1.44269504088896341f)));
    return r;
}

// Packed fp32 pairs (sm_100 f32x2): each lane rounds exactly like the scalar .rn.ftz operation,
// one instruction per pair.
__device__ __forceinline__ float2 fsub2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "sub.rn.ftz.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.ftz.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mul.rn.ftz.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
// 2^x (hardware base-2 exponential), the second step of exp_t
__device__ __forceinline__ float ex2(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// Compensated fp32 sum of values in [0, 4] (single probabilities, or sums of four): the running
// sum starts at CSUM_BASE (8.0), so it is never below the next addend and Fast2Sum (t = s + x;
// err = x - (t - s)) recovers each rounding error exactly; s + c - CSUM_BASE carries ~44 bits.
constexpr float CSUM_BASE = 8.0f;
struct CSum {
    float s, c;
};
__device__ __forceinline__ CSum csum_zero() { return CSum{CSUM_BASE, 0.0f}; }
__device__ __forceinline__ void csum_add(CSum &a, float x) {
    const float t = __fadd_rn(a.s, x);
    const float err = __fsub_rn(x, __fsub_rn(t, a.s));
    a.s = t;
    a.c = __fadd_rn(a.c, err);
}
__device__ __forceinline__ double csum_val(const CSum &a) {
    return ((double)a.s - (double)CSUM_BASE) + (double)a.c;
}

__device__ __forceinline__ uint32_t fbits(float x) { return __float_as_uint(x); }
__device__ __forceinline__ float bitsf(uint32_t b) { return __uint_as_float(b); }

// ----------------------------------------------------------------------------------------
// PTX: shared-memory barrier, bulk copies (no multicast), L2 prefetch

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(unsigned long long *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(unsigned long long *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(unsigned long long *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase of `bar` with the given parity: true when it completed within
// `limit` polls, false when the wait gave up (the caller records ROW_ERR_TIMEOUT and goes on).
template <bool CLUSTER>
__device__ __noinline__ bool bounded_wait_slow(unsigned long long *bar, uint32_t parity, long long limit);

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, unsigned long long *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ uint32_t mapa_rank(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
// 8- / 16-byte asynchronous store into CTA `rank`'s copy of `slot`, completing on its copy of `bar`
__device__ __forceinline__ void push8(void *slot, unsigned long long *bar, uint32_t rank, uint32_t x, uint32_t y) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.b32 [%0], {%1, %2}, [%3];" ::"r"(
                     mapa_rank(smem_u32(slot), rank)),
                 "r"(x), "r"(y), "r"(mapa_rank(smem_u32(bar), rank))
                 : "memory");
}
__device__ __forceinline__ void push16(void *slot, unsigned long long *bar, uint32_t rank, uint32_t x, uint32_t y,
                                       uint32_t z, uint32_t w) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                     mapa_rank(smem_u32(slot), rank)),
                 "r"(x), "r"(y), "r"(z), "r"(w), "r"(mapa_rank(smem_u32(bar), rank))
                 : "memory");
}
// acquire at cluster scope: the completing st.async writes came from other CTAs
__device__ __forceinline__ bool mbar_try_wait_cluster(unsigned long long *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

template <bool CLUSTER>
__device__ __noinline__ bool bounded_wait_slow(unsigned long long *bar, uint32_t parity, long long limit) {
    for (long long it = 0;;) {
        if (CLUSTER ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity)) return true;
        if (++it > limit) return false;
    }
}
// the first poll inline (the common case: the phase is already complete), the loop out of line
template <bool CLUSTER>
__device__ __forceinline__ bool bounded_wait(unsigned long long *bar, uint32_t parity, long long limit) {
    if (CLUSTER ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity)) return true;
    return bounded_wait_slow<CLUSTER>(bar, parity, limit);
}

// Cluster barrier without release/acquire semantics: execution ordering only, so it does not wait
// for this thread's outstanding global stores.  Used where the barrier only separates reads of a
// peer's shared memory (already consumed before the arrive) from later writes to it.
__device__ __forceinline__ void cluster_sync_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}

// ----------------------------------------------------------------------------------------
// block / warp helpers (deterministic: every thread computes identical results)

template <class T, class Op>
__device__ __forceinline__ T warp_allreduce(T v, Op op) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

template <class T, class Op>
__device__ __forceinline__ T block_allreduce(T v, T *scratch, Op op, T ident) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_allreduce(v, op);
    __syncthreads();
    if (lane == 0) scratch[w] = v;
    __syncthreads();
    // per-warp values folded by a shuffle tree in every warp; lane 0's result is broadcast so
    // all threads hold the same bits
    T x = lane < nw ? scratch[lane] : ident;
#pragma unroll
    for (int o = 16; o; o >>= 1) x = op(x, __shfl_down_sync(0xffffffffu, x, o));
    return __shfl_sync(0xffffffffu, x, 0);
}

// Exclusive / inclusive scan of doubles in thread order.  excl(t+1) is bit-identical to
// incl(t), and the returned total is bit-identical to incl(last).
__device__ __forceinline__ void block_scan_d(double v, double *scratch, double &excl, double &incl, double &total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    double x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        double y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x = y + x;
    }
    double prev = __shfl_up_sync(0xffffffffu, x, 1);
    __syncthreads();
    if (lane == 31) scratch[w] = x;
    __syncthreads();
    double off = 0.0;
    for (int i = 0; i < w; i++) off = off + scratch[i];
    double tot = off;
    for (int i = w; i < nw; i++) tot = tot + scratch[i];
    excl = lane == 0 ? off : off + prev;
    incl = off + x;
    total = tot;
}

__device__ __forceinline__ void block_scan_i(int v, int *scratch, int &excl, int &total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    __syncthreads();
    if (lane == 31) scratch[w] = x;
    __syncthreads();
    int off = 0, tot = 0;
    for (int i = 0; i < nw; i++) {
        if (i < w) off += scratch[i];
        tot += scratch[i];
    }
    excl = off + x - v;
    total = tot;
}

// ----------------------------------------------------------------------------------------
// probability chain of one element (index-order path)

struct Chain {
    float inv_sum;
    float min_p;
    float inv_s2;
    float inv_s3;
    int cut_idx;   // last index inside the top-p prefix (INT_MAX when no cut)
    int minp;      // min-p active
    int nokept;    // min-p active but no element reached it: all stay (sampler.c:196)
    int topp;      // top-p renormalisation active
};

// probability after softmax and min-p (0 for elements min-p removed)
__device__ __forceinline__ float w_of(const Chain &ch, float e) {
    float p = __fmul_rn(e, ch.inv_sum);
    if (ch.minp) p = (ch.nokept || p >= ch.min_p) ? __fmul_rn(p, ch.inv_s2) : 0.0f;
    return p;
}
__device__ __forceinline__ bool member_of(const Chain &ch, float e) {
    if (!ch.minp || ch.nokept) return true;
    return __fmul_rn(e, ch.inv_sum) >= ch.min_p;
}
// final draw probability
__device__ __forceinline__ float q_of(const Chain &ch, float e, int gi) {
    float w = w_of(ch, e);
    if (ch.topp) w = gi <= ch.cut_idx ? __fmul_rn(w, ch.inv_s3) : 0.0f;
    return w;
}

// ----------------------------------------------------------------------------------------
// exact fp32 running-sum walk
//
// REC_CLEAN(e, n0, n1): starting from any c in binade e (exponent field e) whose bit pattern
// has parity s, the run ends at bits(c) + n_s, provided the result stays below 2^(e+1).
// REC_IDENT adds only zeros.  REC_MIXED must be expanded.

// Composition scan over lanes: (a0, a1) of lane l becomes the composition of lanes <= l.
__device__ __forceinline__ void compose_scan(uint32_t &a0, uint32_t &a1) {
    const int lane = threadIdx.x & 31;
    if (__ballot_sync(0xffffffffu, a0 != a1) == 0u) {
        // no run depends on the parity: composition is a plain sum
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            uint32_t p = __shfl_up_sync(0xffffffffu, a0, d);
            if (lane >= d) a0 += p;
        }
        a1 = a0;
        return;
    }
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        uint32_t p0 = __shfl_up_sync(0xffffffffu, a0, d);
        uint32_t p1 = __shfl_up_sync(0xffffffffu, a1, d);
        if (lane >= d) {
            uint32_t x0 = a0, x1 = a1;
            a0 = p0 + ((p0 & 1u) ? x1 : x0);
            a1 = p1 + (((1u + p1) & 1u) ? x1 : x0);
        }
    }
}

// Four independent composition scans side by side (general parity form).
__device__ __forceinline__ void compose_scan4(uint32_t (&a0)[4], uint32_t (&a1)[4]) {
    const int lane = threadIdx.x & 31;
    if (__ballot_sync(0xffffffffu, a0[0] != a1[0] || a0[1] != a1[1] || a0[2] != a1[2] || a0[3] != a1[3]) == 0u) {
        // no run depends on the parity: plain prefix sums
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const uint32_t p0 = __shfl_up_sync(0xffffffffu, a0[q], d);
                if (lane >= d) a0[q] += p0;
            }
        }
#pragma unroll
        for (int q = 0; q < 4; q++) a1[q] = a0[q];
        return;
    }
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const uint32_t p0 = __shfl_up_sync(0xffffffffu, a0[q], d);
            const uint32_t p1 = __shfl_up_sync(0xffffffffu, a1[q], d);
            if (lane >= d) {
                const uint32_t x0 = a0[q], x1 = a1[q];
                a0[q] = p0 + ((p0 & 1u) ? x1 : x0);
                a1[q] = p1 + (((1u + p1) & 1u) ? x1 : x0);
            }
        }
    }
}

// Applies one CLEAN run (e, n0, n1) to cb when valid; returns false (cb unchanged) when the run
// cannot be applied to this cb (wrong binade, or the result would leave it).
__device__ __forceinline__ bool apply_run(uint32_t &cb, int e, uint32_t n0, uint32_t n1) {
    if (n0 == 0u && n1 == 0u) return true;
    if (cb == 0u || (cb >> 23) != (uint32_t)e) return false;
    const uint32_t out = cb + ((cb & 1u) ? n1 : n0);
    if (out >= ((uint32_t)(e + 1) << 23)) return false;
    cb = out;
    return true;
}

// One step of the walk over up to 32 records held one per lane (lanes >= n invalid), from
// record `pos`.  Either applies a run of valid CLEAN/IDENT records, or asks the caller to expand
// one record: returns WALK_EXPAND with *xj = that record and cb set to the running sum at its
// start (*must_hit: the draw lies in it).  Returns -1 to continue (pos advanced).
constexpr int WALK_EXPAND = -3;
__device__ __forceinline__ int walk_step(int n, int &pos, int type, int e, uint32_t n0, uint32_t n1, uint32_t &cb,
                                         float r, int *xj, bool *must_hit) {
    const int lane = threadIdx.x & 31;
    if (lane == 0) dbg_add(DBG_STEPS, 1);
    const unsigned live = __ballot_sync(0xffffffffu, lane >= pos && lane < n && type != REC_IDENT);
    if (!live) {
        pos = n;
        return -1;
    }
    const int f = __ffs(live) - 1;
    const int tf = __shfl_sync(0xffffffffu, type, f);
    const int ef = __shfl_sync(0xffffffffu, e, f);
    const bool inbin = cb != 0u && (cb >> 23) == (uint32_t)ef;
    *must_hit = false;
    if (tf != REC_CLEAN || !inbin) {
        *xj = f;
        return WALK_EXPAND;
    }
    const unsigned runm = __ballot_sync(0xffffffffu, lane >= f && lane < n &&
                                                         (type == REC_IDENT || (type == REC_CLEAN && e == ef)));
    const unsigned notrun = ~runm & (0xffffffffu << f);
    int run_end = notrun ? __ffs(notrun) - 1 : 32;
    if (run_end > n) run_end = n;
    const bool inrun = lane >= f && lane < run_end;
    uint32_t a0 = (inrun && type == REC_CLEAN) ? n0 : 0u;
    uint32_t a1 = (inrun && type == REC_CLEAN) ? n1 : 0u;
    compose_scan(a0, a1);
    const uint32_t inc = (cb & 1u) ? a1 : a0;
    const uint32_t cout = cb + inc;
    const uint32_t lim = (uint32_t)(ef + 1) << 23;
    const unsigned bad = __ballot_sync(0xffffffffu, inrun && !(cout < lim));
    const int good_end = bad ? __ffs(bad) - 1 : run_end;
    const unsigned hit = __ballot_sync(0xffffffffu, lane >= f && lane < good_end && r < bitsf(cout));
    const uint32_t prev = __shfl_up_sync(0xffffffffu, cout, 1);
    if (hit) {
        const int l = __ffs(hit) - 1;
        const uint32_t prevl = __shfl_sync(0xffffffffu, prev, l);
        cb = (l == f) ? cb : prevl;
        *xj = l;
        *must_hit = true;
        return WALK_EXPAND;
    }
    const uint32_t last = __shfl_sync(0xffffffffu, cout, good_end > f ? good_end - 1 : f);
    if (good_end > f) cb = last;
    pos = good_end;
    if (pos < run_end) {
        *xj = pos;
        return WALK_EXPAND;
    }
    return -1;
}

// Runs walk steps over the 32 lane records until the draw is found (>= 0), the records are
// exhausted (-1) or an error (-2); `expand(j, cb)` expands record j.
template <class Expand>
__device__ __forceinline__ int walk_records(int n, int type, int e, uint32_t n0, uint32_t n1, uint32_t &cb, float r,
                                            int guard_max, Expand &&expand) {
    int pos = 0, res = -1;
    for (int guard = 0; pos < n && res == -1 && guard < guard_max; guard++) {
        int xj = 0;
        bool must_hit = false;
        res = walk_step(n, pos, type, e, n0, n1, cb, r, &xj, &must_hit);
        if (res == WALK_EXPAND) {
            const long long t0 = g_dbg ? clock64() : 0;
            res = expand(xj, cb);
            if (g_dbg && (threadIdx.x & 31) == 0) dbg_add(DBG_B_EXP, (unsigned long long)(clock64() - t0));
            if (must_hit) {
                pos = n;
                if (res < 0) res = -2;
            } else {
                pos = xj + 1;
            }
        }
    }
    return pos < n && res == -1 ? -2 : res;
}

// Replays n consecutive draw probabilities src[0..n) (shared memory) on the exact running sum
// cb.  Warp-cooperative: lane l owns the sub-range [l*s, l*s + s), s = ceil(n/32), summarised
// as a run record; runs that stay in one binade are composed in parallel, the others are
// replayed serially by their lane.  `gbase + j` is the index of element j.  Returns the drawn
// index, -1 (not in this range; cb advanced past it) or -2.
__device__ __noinline__ int replay_elems_impl(int n, int gbase, uint32_t &cb, float r, const float *src) {
    const int lane = threadIdx.x & 31;
    const int s = (n + 31) >> 5;
    const int j0 = lane * s;
    const int cnt = max(0, min(s, n - j0));
    const float *my = src + j0;
    bool anyq = false;
    for (int k = 0; k < cnt; k++) anyq |= my[k] != 0.0f;
    if (lane == 0) dbg_add(DBG_REPLAY, 1);
    // serial replay of one lane's sub-range on the exact running sum
    auto serial = [&](int jl, uint32_t &cbx) -> int {
        int found = -1;
        uint32_t nb = 0;
        if (lane == jl) {
            float c = bitsf(cbx);
            for (int k = 0; k < cnt; k++) {
                c = __fadd_rn(c, my[k]);
                if (found < 0 && r < c) found = gbase + j0 + k;
            }
            nb = fbits(c);
        }
        found = __shfl_sync(0xffffffffu, found, jl);
        cbx = __shfl_sync(0xffffffffu, nb, jl);
        return found;
    };
    int pos = 0;
    for (int guard = 0; pos < 32 && guard < 96; guard++) {
        if (lane == 0) dbg_add(DBG_REPLAY_IT, 1);
        if (cb == 0u) {
            const unsigned m = __ballot_sync(0xffffffffu, lane >= pos && anyq);
            if (!m) return -1;
            const int fl = __ffs(m) - 1;
            int found = serial(fl, cb);
            pos = fl + 1;
            if (found >= 0) return found;
            continue;
        }
        const uint32_t eb = cb >> 23;
        const uint32_t gb = eb << 23, lim = (eb + 1u) << 23;
        float g0 = bitsf(gb), g1 = bitsf(gb | 1u);
        for (int k = 0; k < cnt; k++) {
            const float x = my[k];
            g0 = __fadd_rn(g0, x);
            g1 = __fadd_rn(g1, x);
        }
        const int type = !anyq ? REC_IDENT : ((fbits(g0) < lim && fbits(g1) < lim) ? REC_CLEAN : REC_MIXED);
        const uint32_t n0 = fbits(g0) - gb, n1 = fbits(g1) - (gb | 1u);
        int xj = 0;
        bool must_hit = false;
        int res = walk_step(32, pos, type, (int)eb, n0, n1, cb, r, &xj, &must_hit);
        if (res == WALK_EXPAND) {
            res = serial(xj, cb);
            if (must_hit) return res >= 0 ? res : -2;
            pos = xj + 1;
        }
        if (res != -1) return res;
    }
    return pos < 32 ? -2 : -1;
}

// replay_elems_impl with each lane's elements held in registers: they are loaded once (all loads
// in flight together), and a lane's run for the running sum's binade is computed once per binade
// instead of once per walk step.  Needs ceil(n / 32) <= SUBT.
template <int SUBT>
__device__ __noinline__ int replay_elems_reg(int n, int gbase, uint32_t &cb, float r, const float *src) {
    const int lane = threadIdx.x & 31;
    const int s = (n + 31) >> 5;
    const int j0 = lane * s;
    const int cnt = max(0, min(s, n - j0));
    float v[SUBT];
#pragma unroll
    for (int k = 0; k < SUBT; k++) v[k] = k < cnt ? src[j0 + k] : 0.0f;
    bool anyq = false;
#pragma unroll
    for (int k = 0; k < SUBT; k++) anyq |= v[k] != 0.0f;
    if (lane == 0) dbg_add(DBG_REPLAY, 1);
    // serial replay of one lane's sub-range on the exact running sum (the zeros past cnt leave
    // a nonnegative sum unchanged)
    auto serial = [&](int jl, uint32_t &cbx) -> int {
        int found = -1;
        uint32_t nb = 0;
        if (lane == jl) {
            float c = bitsf(cbx);
#pragma unroll
            for (int k = 0; k < SUBT; k++) {
                c = __fadd_rn(c, v[k]);
                if (found < 0 && k < cnt && r < c) found = gbase + j0 + k;
            }
            nb = fbits(c);
        }
        found = __shfl_sync(0xffffffffu, found, jl);
        cbx = __shfl_sync(0xffffffffu, nb, jl);
        return found;
    };
    int type = REC_IDENT;
    uint32_t n0 = 0u, n1 = 0u, eb_c = 0xffffffffu;
    int pos = 0;
    for (int guard = 0; pos < 32 && guard < 96; guard++) {
        if (lane == 0) dbg_add(DBG_REPLAY_IT, 1);
        if (cb == 0u) {
            const unsigned m = __ballot_sync(0xffffffffu, lane >= pos && anyq);
            if (!m) return -1;
            const int fl = __ffs(m) - 1;
            const int found = serial(fl, cb);
            pos = fl + 1;
            if (found >= 0) return found;
            continue;
        }
        const uint32_t eb = cb >> 23;  // the same in every lane
        if (eb != eb_c) {
            eb_c = eb;
            const uint32_t gb = eb << 23, lim = (eb + 1u) << 23;
            float g0 = bitsf(gb), g1 = bitsf(gb | 1u);
#pragma unroll
            for (int k = 0; k < SUBT; k++) {
                g0 = __fadd_rn(g0, v[k]);
                g1 = __fadd_rn(g1, v[k]);
            }
            type = !anyq ? REC_IDENT : ((fbits(g0) < lim && fbits(g1) < lim) ? REC_CLEAN : REC_MIXED);
            n0 = fbits(g0) - gb;
            n1 = fbits(g1) - (gb | 1u);
        }
        int xj = 0;
        bool must_hit = false;
        int res = walk_step(32, pos, type, (int)eb, n0, n1, cb, r, &xj, &must_hit);
        if (res == WALK_EXPAND) {
            res = serial(xj, cb);
            if (must_hit) return res >= 0 ? res : -2;
            pos = xj + 1;
        }
        if (res != -1) return res;
    }
    return pos < 32 ? -2 : -1;
}

// replay of n consecutive draw probabilities, with its cycles counted in the diagnostic counters
// when they are on
template <int SUBT>
__device__ __forceinline__ int replay_elems(int n, int gbase, uint32_t &cb, float r, const float *src) {
    const long long t0 = g_dbg ? clock64() : 0;
    const int res = ((n + 31) >> 5) <= SUBT ? replay_elems_reg<SUBT>(n, gbase, cb, r, src)
                                            : replay_elems_impl(n, gbase, cb, r, src);
    if (g_dbg && (threadIdx.x & 31) == 0) dbg_add(DBG_B_REPL, (unsigned long long)(clock64() - t0));
    return res;
}

// ----------------------------------------------------------------------------------------
// short sorted list: softmax, min-p, top-p, draw (src/sampler.c:172-233) by one warp.
// t[i] sorted best-first with ids id[i]; k entries.  Probabilities are written over t[].
// The double sums run in a different order than the reference's loops; they agree to ~1e-16
// relative, so (float)(1.0 / sum) is identical except at measure-zero rounding ties.

__device__ double warp_sum_list(const float *v, int k) {
    const int lane = threadIdx.x & 31;
    double s = 0.0;
    for (int i = lane; i < k; i += 32) s = s + (double)v[i];
    return warp_allreduce(s, [](double x, double y) { return x + y; });
}

__device__ int sample_sorted_list(float *t, int *id, int k, const dllm_sampler_params &p, float r,
                                  float *probs_row, bool minp_relative) {
    const int lane = threadIdx.x & 31;
    const float mv = t[0];
    for (int i = lane; i < k; i += 32) t[i] = expf(__fsub_rn(t[i], mv));
    __syncwarp();
    const double sum = warp_sum_list(t, k);
    const float inv_sum = __double2float_rn(1.0 / sum);
    for (int i = lane; i < k; i += 32) t[i] = __fmul_rn(t[i], inv_sum);
    __syncwarp();
    int kk = k;
    if (p.min_p > 0.0f) {
        // stable compaction of the entries with p >= min_p (relative: min_p * p_max, p_max = t[0])
        const float thr = minp_relative ? __fmul_rn(p.min_p, t[0]) : p.min_p;
        int nk = 0;
        for (int base = 0; base < kk; base += 32) {
            const int i = base + lane;
            const float v = i < kk ? t[i] : 0.0f;
            const int vid = i < kk ? id[i] : 0;
            const bool keep = i < kk && v >= thr;
            const unsigned m = __ballot_sync(0xffffffffu, keep);
            __syncwarp();
            if (keep) {
                const int o = nk + __popc(m & ((1u << lane) - 1u));
                t[o] = v;
                id[o] = vid;
            }
            nk += __popc(m);
            __syncwarp();
        }
        if (nk > 0) kk = nk;
        const double s2 = warp_sum_list(t, kk);
        const float inv2 = __double2float_rn(1.0 / s2);
        for (int i = lane; i < kk; i += 32) t[i] = __fmul_rn(t[i], inv2);
        __syncwarp();
    }
    if (p.top_p < 1.0f) {
        int nk = kk;
        double carry = 0.0, s3 = 0.0;
        bool found = false;
        for (int base = 0; base < kk && !found; base += 32) {
            const int i = base + lane;
            double x = i < kk ? (double)t[i] : 0.0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                double y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x = y + x;
            }
            const double cum = carry + x;
            const unsigned hit = __ballot_sync(0xffffffffu, i < kk && __double2float_rn(cum) >= p.top_p);
            if (hit) {
                const int l = __ffs(hit) - 1;
                nk = base + l + 1;
                s3 = __shfl_sync(0xffffffffu, cum, l);
                found = true;
            } else {
                carry = __shfl_sync(0xffffffffu, cum, 31);
            }
        }
        if (!found) s3 = carry;
        kk = nk;
        const float inv3 = __double2float_rn(1.0 / s3);
        for (int i = lane; i < kk; i += 32) t[i] = __fmul_rn(t[i], inv3);
        __syncwarp();
    }
    int tok = 0;
    if (lane == 0) {
        float c = 0.0f;
        tok = id[kk - 1];
        for (int i = 0; i < kk; i++) {
            c = __fadd_rn(c, t[i]);
            if (r < c) {
                tok = id[i];
                break;
            }
        }
    }
    if (probs_row)
        for (int i = lane; i < kk; i += 32) probs_row[id[i]] = t[i];
    return __shfl_sync(0xffffffffu, tok, 0);
}

// ----------------------------------------------------------------------------------------

__device__ __forceinline__ uint32_t okey(float t) {
    const uint32_t u = fbits(t);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float okey_inv(uint32_t k) {
    return bitsf((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__device__ __forceinline__ uint32_t hash_id(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    return x;
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4 raw, float *d) {
    const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
    float4 *d4 = reinterpret_cast<float4 *>(d);
    d4[0] = make_float4(bitsf(wv[0] << 16), bitsf(wv[0] & 0xffff0000u), bitsf(wv[1] << 16),
                        bitsf(wv[1] & 0xffff0000u));
    d4[1] = make_float4(bitsf(wv[2] << 16), bitsf(wv[2] & 0xffff0000u), bitsf(wv[3] << 16),
                        bitsf(wv[3] & 0xffff0000u));
}

// bf16 slices: 16-byte streaming loads (four in flight per thread), upcast exactly
__device__ void load_slice_bf16(const KernelArgs &a, int row, int slice0, int slen, float *vals) {
    const int NT = blockDim.x, tid = threadIdx.x;
    const __nv_bfloat16 *src = (const __nv_bfloat16 *)a.logits + (int64_t)row * a.row_stride + slice0;
    int done = 0;
    if (a.vec_ok) {
        const int n8 = slen >> 3;
        const uint4 *s8 = (const uint4 *)src;
        int i = tid;
        for (; i + 3 * NT < n8; i += 4 * NT) {
            uint4 raw[4];
#pragma unroll
            for (int u = 0; u < 4; u++) raw[u] = __ldcs(s8 + i + u * NT);
#pragma unroll
            for (int u = 0; u < 4; u++) bf16x8_to_f32(raw[u], vals + 8 * (i + u * NT));
        }
        for (; i < n8; i += NT) bf16x8_to_f32(__ldcs(s8 + i), vals + 8 * i);
        done = n8 * 8;
    }
    const unsigned short *s16 = (const unsigned short *)src;
    for (int i = done + tid; i < slen; i += NT) vals[i] = bitsf((uint32_t)s16[i] << 16);
}


// Exclusive / inclusive scan of four doubles per thread (one per quarter), in thread order;
// same bit-consistency as block_scan_d for each of the four.
__device__ __forceinline__ void block_scan4_d(const double v[4], double *scratch, double excl[4], double incl[4], double tot[4]) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    double x[4], prev[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
        x[q] = v[q];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            double y = __shfl_up_sync(0xffffffffu, x[q], o);
            if (lane >= o) x[q] = y + x[q];
        }
        prev[q] = __shfl_up_sync(0xffffffffu, x[q], 1);
    }
    __syncthreads();
    if (lane == 31)
#pragma unroll
        for (int q = 0; q < 4; q++) scratch[q * MAXW + w] = x[q];
    __syncthreads();
    // warp totals scanned by shuffles (lane i holds warp i's total); every warp computes the same
    // sums in the same order, so all threads agree on the offsets and totals bit for bit
#pragma unroll
    for (int q = 0; q < 4; q++) {
        double y = lane < nw ? scratch[q * MAXW + lane] : 0.0;
#pragma unroll
        for (int o = 1; o < MAXW; o <<= 1) {
            const double z = __shfl_up_sync(0xffffffffu, y, o);
            if (lane >= o) y = z + y;
        }
        const double ex = __shfl_up_sync(0xffffffffu, y, 1);
        const double off = __shfl_sync(0xffffffffu, lane == 0 ? 0.0 : ex, w);
        tot[q] = __shfl_sync(0xffffffffu, y, nw - 1);
        excl[q] = lane == 0 ? off : off + prev[q];
        incl[q] = off + x[q];
    }
}

// Exclusive scan of four ints per thread in (quarter, thread) order; returns per-quarter
// offsets already including the totals of earlier quarters.
__device__ __forceinline__ void block_scan4_i(const int v[4], int *scratch, int excl[4], int &total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int x[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
        x[q] = v[q];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, x[q], o);
            if (lane >= o) x[q] += y;
        }
    }
    __syncthreads();
    if (lane == 31)
#pragma unroll
        for (int q = 0; q < 4; q++) scratch[q * MAXW + w] = x[q];
    __syncthreads();
    int base = 0;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        int off = 0, t = 0;
        for (int i = 0; i < nw; i++) {
            if (i < w) off += scratch[q * MAXW + i];
            t += scratch[q * MAXW + i];
        }
        excl[q] = base + off + x[q] - v[q];
        base += t;
    }
    total = base;
}

__device__ __forceinline__ uint32_t pack_meta(int type, int bchunk, int sfrom, int e_pre, int e_suf) {
    return (uint32_t)type | ((uint32_t)(bchunk < 0 ? 63 : bchunk) << 2) | ((uint32_t)sfrom << 8) |
           ((uint32_t)(e_pre & 255) << 16) | ((uint32_t)(e_suf & 255) << 24);
}

// P4 element loop: the draw probability of every element of the four sub-chunks, added into
// two fp32 chains per sub-chunk (started at 2^e and 2^e + ulp); qmax[q] > 0 iff any is nonzero
template <class T>
__device__ __forceinline__ T pick4(const T (&v)[4], int q) {
    return q == 0 ? v[0] : q == 1 ? v[1] : q == 2 ? v[2] : v[3];
}

// P2 body: exponentials of this thread's four sub-chunks, written back in place, and their fp32
// sums.  Sub-chunks past the slice (the shared zero sub-chunk) are skipped.
template <int NV4>
__device__ __forceinline__ void p2_scan(float *vals, const int (&kb)[4], int S, float M, float inv_temp, float mv,
                                        double (&sube)[4]) {
    CSum sub[4];
    bool real[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
        // a plain sum from 0 in .s; .c holds the base so that csum_val returns .s exactly
        sub[q] = CSum{0.0f, CSUM_BASE};
        real[q] = kb[q] < S;
    }
    // temperature 1 (and no shift): ((x - M) * 1) - 0 == x - M exactly, so skip the two no-ops
    const bool plain = inv_temp == 1.0f && mv == 0.0f;
    const float2 M2 = make_float2(M, M), IT2 = make_float2(inv_temp, inv_temp), MV2 = make_float2(mv, mv);
    const float2 L2E2 = make_float2(1.44269504088896341f, 1.44269504088896341f);
#pragma unroll 2
    for (int j = 0; j < NV4; j++) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
            if (real[q]) {
                float4 *p = reinterpret_cast<float4 *>(vals + kb[q] + 4 * j);
                float4 x = *p;
                // t = ((x - M) * (1/T)) - mv, then e = 2^(t * log2 e), two elements per instruction
                float2 t01 = fsub2(make_float2(x.x, x.y), M2), t23 = fsub2(make_float2(x.z, x.w), M2);
                if (!plain) {
                    t01 = fsub2(fmul2(t01, IT2), MV2);
                    t23 = fsub2(fmul2(t23, IT2), MV2);
                }
                t01 = fmul2(t01, L2E2);
                t23 = fmul2(t23, L2E2);
                x = make_float4(ex2(t01.x), ex2(t01.y), ex2(t23.x), ex2(t23.y));
                *p = x;
                // plain fp32 sums: a sub-chunk of SUB elements carries a relative error of about
                // SUB/4 * 2^-24, which moves the row sum by ~1e-9 relative (random signs), far
                // below the one-ulp spread of (float)(1/sum) that the probability tolerance covers
                const float2 s2 = fadd2(make_float2(x.x, x.y), make_float2(x.z, x.w));
                sub[q].s = __fadd_rn(sub[q].s, __fadd_rn(s2.x, s2.y));
            }
        }
    }
#pragma unroll
    for (int q = 0; q < 4; q++) sube[q] = csum_val(sub[q]);
}

// P3 body: compensated sums of the list probabilities over the four sub-chunks; TRACK also
// records the first and last min-p member of this thread's sub-chunks.
template <bool TRACK, bool MINP, int NV4>
__device__ __forceinline__ void p3_scan(const float *vals, const int (&kb)[4], int slen, int slice0, const Chain &ch,
                                        double (&subd)[4], int &fmem, int &lmem, float &fw) {
    CSum sub[4];
#pragma unroll
    for (int q = 0; q < 4; q++) sub[q] = csum_zero();
#pragma unroll 2
    for (int j = 0; j < NV4; j++) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float4 x = *reinterpret_cast<const float4 *>(vals + kb[q] + 4 * j);
            const float e4[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int c = 0; c < 4; c++) {
                // w_of with the min-p branch resolved at compile time (TRACK: min-p filters,
                // MINP && !TRACK: min-p kept everything and only rescales)
                float w = __fmul_rn(e4[c], ch.inv_sum);
                if (MINP) w = (!TRACK || w >= ch.min_p) ? __fmul_rn(w, ch.inv_s2) : 0.0f;
                csum_add(sub[q], w);
                if (TRACK) {
                    const int li = kb[q] + 4 * j + c;
                    if (li < slen && member_of(ch, e4[c])) {
                        if (slice0 + li < fmem) {
                            fmem = slice0 + li;
                            fw = w;
                        }
                        lmem = max(lmem, slice0 + li);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int q = 0; q < 4; q++) subd[q] = csum_val(sub[q]);
}

template <bool MINP, int NV4>
__device__ __forceinline__ void p4_scan(const float *vals, const int (&kb)[4], const Chain &ch, const float (&s3q)[4],
                                        float (&g0)[4], float (&g1)[4], float (&qmax)[4]) {
    const float2 IS2 = make_float2(ch.inv_sum, ch.inv_sum);
#pragma unroll 2
    for (int j = 0; j < NV4; j++) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float4 x = *reinterpret_cast<const float4 *>(vals + kb[q] + 4 * j);
            // w = e * inv_sum (then min-p), q = w * scale3, two elements per multiply; the scale is
            // 0 for a sub-chunk wholly past the top-p cut, and the crossing sub-chunk's entries
            // past the cut were zeroed, so no per-element cut test is needed
            float2 w01 = fmul2(make_float2(x.x, x.y), IS2), w23 = fmul2(make_float2(x.z, x.w), IS2);
            if (MINP) {
                w01.x = (ch.nokept || w01.x >= ch.min_p) ? __fmul_rn(w01.x, ch.inv_s2) : 0.0f;
                w01.y = (ch.nokept || w01.y >= ch.min_p) ? __fmul_rn(w01.y, ch.inv_s2) : 0.0f;
                w23.x = (ch.nokept || w23.x >= ch.min_p) ? __fmul_rn(w23.x, ch.inv_s2) : 0.0f;
                w23.y = (ch.nokept || w23.y >= ch.min_p) ? __fmul_rn(w23.y, ch.inv_s2) : 0.0f;
            }
            const float2 S2 = make_float2(s3q[q], s3q[q]);
            const float2 q01 = fmul2(w01, S2), q23 = fmul2(w23, S2);
            if (MINP) qmax[q] = fmaxf(fmaxf(qmax[q], fmaxf(q01.x, q01.y)), fmaxf(q23.x, q23.y));
            g0[q] = __fadd_rn(g0[q], q01.x);
            g1[q] = __fadd_rn(g1[q], q01.x);
            g0[q] = __fadd_rn(g0[q], q01.y);
            g1[q] = __fadd_rn(g1[q], q01.y);
            g0[q] = __fadd_rn(g0[q], q23.x);
            g1[q] = __fadd_rn(g1[q], q23.x);
            g0[q] = __fadd_rn(g0[q], q23.y);
            g1[q] = __fadd_rn(g1[q], q23.y);
        }
    }
}

// ----------------------------------------------------------------------------------------
// kernel A

// IDX: the index-order path only (every row has temperature > 0, top-k off, no min-p; the host
// checks), so the greedy, top-k and min-p code is compiled out and the hot code is smaller
template <int DT, int SUBT, bool IDX = false>
__global__ void __launch_bounds__(512, 1) sample_rows_kernel(const KernelArgs a) {
    static_assert(SUBT % 8 == 4 && SUBT <= MAX_SUB, "sub-chunk length");
    constexpr int NV4 = SUBT / 4;   // float4 per sub-chunk
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ __align__(16) unsigned char dsm[];
    __shared__ Shared sh;

    const int NT = blockDim.x, NW = NT >> 5;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int C = a.cluster;
    const int rank = (int)cluster.block_rank();
    const int cid = blockIdx.x / C, ncl = gridDim.x / C;
    const int S = a.S, V = a.vocab;
    const int slice0 = rank * S;
    const int slen = max(0, min(S, V - slice0));
    int kb[4];  // slice-relative start of this thread's four sub-chunks
#pragma unroll
    for (int q = 0; q < 4; q++) {
        // sub-chunks past the slice (S need not fill 4 * NT sub-chunks) read a shared all-zero
        // sub-chunk stored right after the slice: they add nothing to sums or records
        const int sc = q * NT + tid;
        kb[q] = sc * SUBT < S ? sc * SUBT : S;
    }

    // slice buffers: with nbuf == 2 the copy of this CTA's next row lands in the other buffer
    // while the current row is processed
    float *const vbuf0 = reinterpret_cast<float *>(dsm);
    float *const vbuf1 = a.nbuf == 2 ? vbuf0 + S + SUBT : vbuf0;
    unsigned char *uni = dsm + (size_t)a.nbuf * (S + SUBT) * sizeof(float);
    for (int i = tid; i < SUBT; i += NT) {
        vbuf0[S + i] = 0.0f;
        vbuf1[S + i] = 0.0f;
    }
    // union area: history table | top-k survivors + list
    int *hkeys = reinterpret_cast<int *>(uni);
    int *hcnt = hkeys + a.htab;
    unsigned long long *cand = reinterpret_cast<unsigned long long *>(uni);

    auto remote_xs = [&](int r) -> Xch * { return cluster.map_shared_rank(&sh.xs, r); };

    if (tid == 0) {
        g_dbg = a.dbg;
        mbar_init(&sh.tma_bar[0], 1);
        mbar_init(&sh.tma_bar[1], 1);
        for (int k = 0; k < 3; k++)
            for (int b = 0; b < 2; b++) mbar_init(&sh.xbar[k][b], 1);
        sh.slots[0] = sh.slots[1] = 0;
        fence_proxy_async();
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // every CTA's exchange barriers exist before any peer pushes into them
    cluster.sync();
    uint32_t xph = 0u;  // phase bit per exchange barrier (bit 2k + parity)
    // Push exchange k of the row with parity par: threads 0..C-1 push this CTA's payload to rank
    // tid, then every thread waits (bounded) for the C payloads addressed to this CTA.
    auto xwait = [&](int k, int par) -> bool {
        const uint32_t bit = 1u << (2 * k + par);
        const bool ok = bounded_wait<true>(&sh.xbar[k][par], (xph & bit) ? 1u : 0u, a.wait_limit);
        xph ^= bit;
        return ok;
    };

    const bool timing = a.dbg != nullptr && rank == a.dbg_rank && tid == 0;
    long long tmark = clock64();
    auto mark = [&](int k) {
        if (timing) {
            const long long t = clock64();
            dbg_add(k, (unsigned long long)(t - tmark));
            tmark = t;
        }
    };

    // bulk copy of this CTA's slice of `row` (fp32 rows with 16-byte aligned slices)
    const bool use_tma = DT == DLLM_DTYPE_F32 && a.vec_ok;
    const int tma_elems = slen & ~3;
    auto issue_row_copy = [&](int row, int b) {
        const unsigned char *src = reinterpret_cast<const unsigned char *>(
            (const float *)a.logits + (int64_t)row * a.row_stride + slice0);
        unsigned char *dst = reinterpret_cast<unsigned char *>(b ? vbuf1 : vbuf0);
        const uint32_t bytes = (uint32_t)tma_elems * 4u;
        mbar_arrive_expect_tx(&sh.tma_bar[b], bytes);
        for (uint32_t off = 0; off < bytes; off += TMA_PIECE) {
            const uint32_t nb = bytes - off < (uint32_t)TMA_PIECE ? bytes - off : (uint32_t)TMA_PIECE;
            bulk_g2s(dst + off, src + off, nb, &sh.tma_bar[b]);
        }
    };
    auto prefetch_row = [&](int row) {
        const unsigned char *src = reinterpret_cast<const unsigned char *>(
            (const float *)a.logits + (int64_t)row * a.row_stride + slice0);
        const uint32_t bytes = (uint32_t)tma_elems * 4u;
        for (uint32_t off = 0; off < bytes; off += TMA_PIECE) {
            const uint32_t nb = bytes - off < (uint32_t)TMA_PIECE ? bytes - off : (uint32_t)TMA_PIECE;
            prefetch_l2(src + off, nb);
        }
    };

    const bool dbuf = a.nbuf == 2;
    if (tid == 0 && use_tma) {
        if (cid < a.rows) issue_row_copy(cid, 0);
        if (dbuf && cid + ncl < a.rows) issue_row_copy(cid + ncl, 1);
    }
    // history of the rows ahead, loaded early so the latency of these dependent global loads
    // (offsets, then ids) stays off each row's chain: the offsets two rows ahead and the first
    // HPF ids per thread one row ahead
    constexpr int HPF = 2;
    const bool have_hist = a.hist_ids && a.hist_off;
    int64_t cur_h0 = 0, cur_h1 = 0, nxt_h0 = 0, nxt_h1 = 0;
    int cur_id[HPF];
    auto load_ids = [&](int64_t h0, int64_t h1, int (&dst)[HPF]) {
#pragma unroll
        for (int k = 0; k < HPF; k++) {
            const int64_t j = h0 + tid + (int64_t)k * NT;
            dst[k] = j < h1 ? a.hist_ids[j] : -1;
        }
    };
    if (have_hist && cid < a.rows) {
        cur_h0 = a.hist_off[cid];
        cur_h1 = a.hist_off[cid + 1];
        load_ids(cur_h0, cur_h1, cur_id);
        if (cid + ncl < a.rows) {
            nxt_h0 = a.hist_off[cid + ncl];
            nxt_h1 = a.hist_off[cid + ncl + 1];
        }
    }
    // History hash table of the row about to be sampled (ids cur_h0..cur_h1, the first HPF per
    // thread already in cur_id): cleared, then every in-slice id inserted with its count.  No
    // trailing barrier.  Returns ROW_ERR_HIST_TABLE when an id found no free entry.
    auto build_table = [&](bool use_hist) -> int {
        int fl = 0;
        for (int i = tid; i < a.htab; i += NT) {
            hkeys[i] = -1;
            hcnt[i] = 0;
        }
        __syncthreads();
        if (!use_hist) return 0;
        const int64_t h0 = cur_h0, h1 = cur_h1;
        const uint32_t hm = (uint32_t)a.htab - 1u;
        int k = 0;
        for (int64_t j = h0 + tid; j < h1; j += NT, k++) {
            const int id = k == 0 ? cur_id[0] : (k == 1 ? cur_id[1] : a.hist_ids[j]);
            if (id < 0 || id >= a.vocab_total) continue;
            const int li = id - a.vocab_offset - slice0;
            if (li < 0 || li >= slen) continue;
            uint32_t h = hash_id((uint32_t)li) & hm;
            bool placed = false;
            for (int probe = 0; probe < a.htab; probe++) {
                const int old = atomicCAS(&hkeys[h], -1, li);
                if (old == -1 || old == li) {
                    atomicAdd(&hcnt[h], 1);
                    placed = true;
                    break;
                }
                h = (h + 1u) & hm;
            }
            if (!placed) fl |= ROW_ERR_HIST_TABLE;
        }
        return fl;
    };
    // Index-order-only variant: the next row's table is built while this row waits for its
    // top-p cut (exchange #4), after this row's penalties have been applied and the table is
    // no longer read; the next row then skips the build.
    bool prebuilt = false;
    int pre_flags = 0;
    int it = 0;
    for (int row = cid; row < a.rows; row += ncl, it++) {
        if (timing) dbg_add(DBG_ROWS, 1);
        const int buf = dbuf ? (it & 1) : 0;
        const uint32_t phase = dbuf ? (uint32_t)((it >> 1) & 1) : (uint32_t)(it & 1);
        float *const vals = buf ? vbuf1 : vbuf0;
        const dllm_sampler_params p = a.rparams ? a.rparams[row] : a.bparams;
        const float r = a.uniforms[row];
        RowHdr *hdr = row_hdr(a, row);
        int flags = 0;

        // ---------------- P1: bulk copy in flight while the history table is built ---------------
        if (tid == 0) {
            // the slice of this CTA's next row is copied in from the end of this row on; the one
            // after it is pulled into L2 now
            if (use_tma && !dbuf && row + 2 * ncl < a.rows) prefetch_row(row + 2 * ncl);
            // CTA 0's slot counter of the next row (its last claims, two rows back, are done)
            if (rank == 0) sh.slots[(it + 1) & 1] = 0;
            sh.bcast_i[2] = 0;  // the CTA's row status bits
            sh.xs.cut_idx = -1;
            sh.xs.cut_flags = 0;
        }
        const bool use_hist = a.hist_ids && a.hist_off &&
                              (p.repetition > 1.0f || p.presence != 0.0f || p.frequency != 0.0f);
        if (prebuilt) {
            flags |= pre_flags;  // the table was built during the previous row
            prebuilt = false;
        } else {
            flags |= build_table(use_hist);
        }
        if (have_hist && row + ncl < a.rows) {
            // this row's ids are in the table: load the next row's ids from its offsets (loaded a
            // row ago) and the offsets of the row after it; they land while this row is sampled
            cur_h0 = nxt_h0;
            cur_h1 = nxt_h1;
            load_ids(cur_h0, cur_h1, cur_id);
            if (row + 2 * ncl < a.rows) {
                nxt_h0 = a.hist_off[row + 2 * ncl];
                nxt_h1 = a.hist_off[row + 2 * ncl + 1];
            }
        }
        if (use_tma) {
            const float *src = (const float *)a.logits + (int64_t)row * a.row_stride + slice0;
            for (int i = tma_elems + tid; i < slen; i += NT) vals[i] = __ldcs(src + i);
        } else if (DT == DLLM_DTYPE_F32) {
            const float *src = (const float *)a.logits + (int64_t)row * a.row_stride + slice0;
            for (int i = tid; i < slen; i += NT) vals[i] = __ldcs(src + i);
        } else {
            load_slice_bf16(a, row, slice0, slen, vals);
        }
        for (int i = slen + tid; i < S; i += NT) vals[i] = -INFINITY;
        if (use_tma) {
            if (timing) {
                // diagnostics: the part of P1 before the wait, and whether the copy had landed
                mark(DBG_HBUILD);
                if (mbar_try_wait(&sh.tma_bar[buf], phase)) dbg_add(DBG_COPY_EARLY, 1);
            }
            if (!bounded_wait<false>(&sh.tma_bar[buf], phase, a.wait_limit)) flags |= ROW_ERR_TIMEOUT;
            // test hook (off unless a test asks): on the cluster's first row, CTA 0 also waits for
            // the barrier's next phase, which nothing completes, so the wait runs out with no
            // copy in flight
            if (a.fault_site == FAULT_COPY_WAIT && it == 0 && rank == 0 &&
                !bounded_wait<false>(&sh.tma_bar[buf], phase ^ 1u, a.wait_limit))
                flags |= ROW_ERR_TIMEOUT;
        }
        if (flags) atomicOr(&sh.bcast_i[2], flags);
        __syncthreads();
        mark(DBG_LOADWAIT);

        // ---------------- P1: penalties on the raw logits (sparse), then mask + maximum ---------
        // Penalising before masking gives the reference's values (mask -> presence ->
        // repetition): a masked entry ends at -inf either way, and the others are not masked.
        if (use_hist) {
            const float inv_rep = __fdiv_rn(1.0f, p.repetition);
            const bool true_div = (a.flags & DLLM_MODE_PEN_TRUE_DIV) != 0;
            for (int s = tid; s < a.htab; s += NT) {
                const int li = hkeys[s];
                if (li < 0) continue;
                const int c = hcnt[s];
                float v = vals[li];
                if (p.presence != 0.0f) v = __fsub_rn(v, p.presence);
                if (p.frequency != 0.0f) v = __fsub_rn(v, __fmul_rn(__int2float_rn(c), p.frequency));
                if (p.repetition > 1.0f) {
                    for (int k = 0; k < c; k++) {
                        if (v < 0.0f) v = __fmul_rn(v, p.repetition);
                        else v = true_div ? __fdiv_rn(v, p.repetition) : __fmul_rn(v, inv_rep);
                    }
                }
                vals[li] = v;
            }
            __syncthreads();
        }
        // mask + maximum (strided float4 pass over the slice)
        float lmax = -INFINITY;
        {
            float4 *v4 = reinterpret_cast<float4 *>(vals);
            const uint32_t *mrow = a.mask ? a.mask + (int64_t)row * a.mask_stride : nullptr;
            if (mrow) {
                for (int i = tid; i < S / 4; i += NT) {
                    const int li = slice0 + 4 * i;
                    float4 x = v4[i];
                    const uint32_t w = li < V ? (mrow[li >> 5] >> (li & 31)) : 0u;
                    x.x = (w & 1u) ? x.x : -INFINITY;
                    x.y = (w & 2u) ? x.y : -INFINITY;
                    x.z = (w & 4u) ? x.z : -INFINITY;
                    x.w = (w & 8u) ? x.w : -INFINITY;
                    v4[i] = x;
                    lmax = fmaxf(lmax, fmaxf(fmaxf(x.x, x.y), fmaxf(x.z, x.w)));
                }
            } else {
                // four independent maxima, so four shared loads are in flight per thread
                float m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
                int i = tid;
                for (; i + 3 * NT < S / 4; i += 4 * NT) {
                    const float4 x0 = v4[i], x1 = v4[i + NT], x2 = v4[i + 2 * NT], x3 = v4[i + 3 * NT];
                    lmax = fmaxf(lmax, fmaxf(fmaxf(x0.x, x0.y), fmaxf(x0.z, x0.w)));
                    m1 = fmaxf(m1, fmaxf(fmaxf(x1.x, x1.y), fmaxf(x1.z, x1.w)));
                    m2 = fmaxf(m2, fmaxf(fmaxf(x2.x, x2.y), fmaxf(x2.z, x2.w)));
                    m3 = fmaxf(m3, fmaxf(fmaxf(x3.x, x3.y), fmaxf(x3.z, x3.w)));
                }
                for (; i < S / 4; i += NT) {
                    const float4 x = v4[i];
                    lmax = fmaxf(lmax, fmaxf(fmaxf(x.x, x.y), fmaxf(x.z, x.w)));
                }
                lmax = fmaxf(fmaxf(lmax, m1), fmaxf(m2, m3));
            }
        }
        mark(DBG_MAXP);
        const float lm = block_allreduce(lmax, sh.red_f, [](float x, float y) { return fmaxf(x, y); }, -INFINITY);
        flags = sh.bcast_i[2];
        if (a.pen_out) {
            float *po = a.pen_out + (int64_t)row * a.pen_stride + slice0;
            for (int i = tid; i < slen; i += NT) po[i] = vals[i];
        }
        const int par = it & 1;
        if (tid == 0) {
            sh.xs.m = lm;
            sh.xs.flags = flags;
            mbar_arrive_expect_tx(&sh.xbar[0][par], (uint32_t)(C * sizeof(Push1)));
        }
        if (tid < C) push8(&sh.in1[par][rank], &sh.xbar[0][par], tid, __float_as_uint(lm), (uint32_t)flags);
        mark(DBG_P1);
        bool to1 = !xwait(0, par);  // ---- #1
        // test hook (off unless a test asks): on the cluster's first row, the last CTA also waits
        // for exchange #1's next phase, which nothing completes before this CTA moves on
        if (a.fault_site == FAULT_EXCHANGE_WAIT && it == 0 && rank == C - 1 &&
            !bounded_wait<true>(&sh.xbar[0][par], (xph & (1u << par)) ? 1u : 0u, a.wait_limit))
            to1 = true;
        mark(DBG_W1);
        float M = -INFINITY;
        int rowflags = 0;
        {
            float mv = -INFINITY;
            int fv = 0;
            if (lane < C) {
                mv = sh.in1[par][lane].m;
                fv = sh.in1[par][lane].flags;
            }
            M = warp_allreduce(mv, [](float x, float y) { return fmaxf(x, y); });
            rowflags = warp_allreduce(fv, [](int x, int y) { return x | y; });
            if (to1) rowflags |= ROW_ERR_TIMEOUT;
        }

        const bool greedy = !IDX && p.temperature == 0.0f;
        const bool topk = !IDX && p.top_k > 0 && p.top_k < a.vocab_total;
        int token = -1;
        bool done = true;   // token decided here (else the walk kernel draws it)
        bool copy_issued = false;  // the next row's bulk copy was issued early (index-order path)

        if (greedy) {
            // ---------------- greedy: first index holding M ----------------------------------
            int first = INT_MAX;
            for (int i = tid; i < slen; i += NT)
                if (vals[i] == M) {
                    first = i;
                    break;
                }
            if (first != INT_MAX) first += slice0;
            const int bf = block_allreduce(first, sh.red_i, [](int x, int y) { return min(x, y); }, INT_MAX);
            if (tid == 0) sh.xs.gidx = bf;
            cluster.sync();  // ---- greedy
            int gv = INT_MAX;
            if (lane < C) gv = remote_xs(lane)->gidx;
            token = warp_allreduce(gv, [](int x, int y) { return min(x, y); });
            if (token == INT_MAX) token = 0;
        } else if (M == -INFINITY || M == INFINITY) {
            // fully masked row (M = -inf) or a row holding +inf: every t is -inf or NaN
            // ((x - M) * inv_temp), comparisons fail, so the reference's list stays in id order
            // and, with its sum NaN, its draw returns the last entry (src/sampler.c:153-233)
            token = topk ? p.top_k - 1 : a.vocab_total - 1;
            if (topk && a.topk_ids && rank == 0)
                for (int i = tid; i < p.top_k; i += NT) a.topk_ids[(int64_t)row * a.topk_stride + i] = i + a.vocab_offset;
        } else if (topk) {
            // ---------------- top-k ----------------------------------------------------------
            {
                // a NaN logit: the reference's -ffast-math build leaves its place in the sorted
                // list undefined, so the row is flagged (each CTA for its slice; the walk kernel
                // ORs the CTAs' bits into the status)
                bool nanf = false;
                for (int i = tid; i < slen; i += NT) nanf |= isnan(vals[i]);
                if (__syncthreads_or(nanf)) rowflags |= ROW_ERR_NONFINITE;
            }
            const int k = p.top_k;
            int kp2 = 1;
            while (kp2 < k) kp2 <<= 1;
            const float inv_temp = __fdiv_rn(1.0f, p.temperature);
            auto key_of = [&](float v) -> uint32_t { return okey(__fmul_rn(__fsub_rn(v, M), inv_temp)); };
            if (k > KMAX || 8 * kp2 + 8 * k > a.uni_bytes) {
                rowflags |= ROW_ERR_TOPK_LARGE;
                token = 0;
                goto row_done;
            }
            {
            // survivor capacity: a power of two whose sort buffer and the final list both fit
            int cap = CAND_CAP;
            while (cap > kp2 && 8 * cap + 8 * k > a.uni_bytes) cap >>= 1;
            bool use_threshold = k <= NT && cap >= kp2 && 8 * cap + 8 * k <= a.uni_bytes;
            if (use_threshold) {
                // threshold: the k-th largest per-thread maximum (>= k elements at or above it)
                uint32_t tmax = 0u;
                for (int i = tid; i < slen; i += NT) tmax = max(tmax, key_of(vals[i]));
                // the k-th largest of the NT maxima, found by one warp bit by bit with ballots
                // (the CTA's candidate area is free until the survivors are gathered)
                unsigned *tm_s = reinterpret_cast<unsigned *>(uni);
                tm_s[tid] = tmax;
                __syncthreads();
                if (wid == 0) {
                    uint32_t mine[MAXW];
#pragma unroll
                    for (int t = 0; t < MAXW; t++) mine[t] = 32 * t + lane < NT ? tm_s[32 * t + lane] : 0u;
                    uint32_t pref = 0u;
                    for (int bit = 31; bit >= 0; bit--) {
                        const uint32_t cv = pref | (1u << bit);
                        int cnt = 0;
#pragma unroll
                        for (int t = 0; t < MAXW; t++) cnt += __popc(__ballot_sync(0xffffffffu, mine[t] >= cv));
                        if (cnt >= k) pref = cv;
                    }
                    if (lane == 0) {
                        sh.xs.theta = pref;
                        sh.xs.ncand = 0;
                    }
                }
                cluster.sync();  // ---- threshold
                uint32_t tv = 0u;
                if (lane < C) tv = remote_xs(lane)->theta;
                const uint32_t theta = warp_allreduce(tv, [](uint32_t x, uint32_t y) { return max(x, y); });
                // survivors -> CTA 0
                int *ncand0 = &remote_xs(0)->ncand;
                unsigned long long *cand0 = cluster.map_shared_rank(cand, 0);
                for (int i0 = 0; i0 < S; i0 += NT) {
                    const int li = i0 + tid;
                    const uint32_t key = li < slen ? key_of(vals[li]) : 0u;
                    const bool take = li < slen && key >= theta;
                    const unsigned m = __ballot_sync(0xffffffffu, take);
                    if (m) {
                        const int leader = __ffs(m) - 1;
                        int base = 0;
                        if (lane == leader) base = atomicAdd(ncand0, __popc(m));
                        base = __shfl_sync(0xffffffffu, base, leader);
                        if (take) {
                            const int o = base + __popc(m & ((1u << lane) - 1u));
                            const uint32_t gid = (uint32_t)(slice0 + li);
                            if (o < cap) cand0[o] = ((unsigned long long)key << 32) | (0xffffffffu - gid);
                        }
                    }
                }
                cluster.sync();  // ---- survivors gathered
                use_threshold = remote_xs(0)->ncand <= cap;
                if (!use_threshold && timing) dbg_add(DBG_TOPK_FALLBACK, 1);
            }
            if (!use_threshold) {
                // 4-pass cluster radix select of the k-th key, then exact gather (ties by id)
                uint32_t prefix = 0, pmask = 0;
                int krem = k;
                for (int pass = 0; pass < 4; pass++) {
                    const int shift = 24 - 8 * pass;
                    unsigned *h = sh.xs.hist[pass & 1];
                    for (int i = tid; i < 256; i += NT) h[i] = 0;
                    __syncthreads();
                    for (int i0 = 0; i0 < S; i0 += NT) {
                        const int li = i0 + tid;
                        int d = -1;
                        if (li < slen) {
                            const uint32_t key = key_of(vals[li]);
                            if ((key & pmask) == prefix) d = (int)((key >> shift) & 255u);
                        }
                        const unsigned peers = __match_any_sync(0xffffffffu, d);
                        if (d >= 0 && lane == __ffs(peers) - 1) atomicAdd(&h[d], (unsigned)__popc(peers));
                    }
                    __syncthreads();
                    cluster.sync();  // ---- radix pass
                    if (wid == 0) {
                        unsigned cntb[8];
#pragma unroll
                        for (int b = 0; b < 8; b++) cntb[b] = 0;
                        for (int rr = 0; rr < C; rr++) {
                            const unsigned *hr = remote_xs(rr)->hist[pass & 1];
#pragma unroll
                            for (int b = 0; b < 8; b++) cntb[b] += hr[lane * 8 + b];
                        }
                        unsigned mysum = 0;
#pragma unroll
                        for (int b = 0; b < 8; b++) mysum += cntb[b];
                        unsigned x = mysum;
#pragma unroll
                        for (int o = 1; o < 32; o <<= 1) {
                            unsigned y = __shfl_down_sync(0xffffffffu, x, o);
                            if (lane + o < 32) x += y;
                        }
                        const unsigned above = x - mysum;
                        int sel = -1;
                        unsigned gt = 0, acc = above;
                        if (above < (unsigned)krem && x >= (unsigned)krem) {
#pragma unroll
                            for (int b = 7; b >= 0; b--) {
                                if (sel < 0) {
                                    if (acc + cntb[b] >= (unsigned)krem) {
                                        sel = lane * 8 + b;
                                        gt = acc;
                                    } else {
                                        acc += cntb[b];
                                    }
                                }
                            }
                        }
                        const unsigned own = __ballot_sync(0xffffffffu, sel >= 0);
                        const int src = own ? __ffs(own) - 1 : 0;
                        sel = __shfl_sync(0xffffffffu, sel, src);
                        gt = __shfl_sync(0xffffffffu, gt, src);
                        if (lane == 0) {
                            sh.bcast_i[0] = sel;
                            sh.bcast_i[1] = (int)gt;
                        }
                    }
                    __syncthreads();
                    const int sel = sh.bcast_i[0];
                    krem -= sh.bcast_i[1];
                    prefix |= (uint32_t)max(sel, 0) << shift;
                    pmask |= 255u << shift;
                }
                const uint32_t kstar = prefix;
                const int ngt = k - krem;
                // counts per (quarter, thread) sub-chunk: sub-chunks in that order are in id order
                int cgt[4], ceq[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    cgt[q] = ceq[q] = 0;
                    for (int j = 0; j < SUBT; j++) {
                        const int li = kb[q] + j;
                        if (li < slen) {
                            const uint32_t key = key_of(vals[li]);
                            cgt[q] += key > kstar;
                            ceq[q] += key == kstar;
                        }
                    }
                }
                int egt[4], eeq[4], tgt, teq;
                block_scan4_i(cgt, sh.red_i, egt, tgt);
                block_scan4_i(ceq, sh.red_i, eeq, teq);
                if (tid == 0) {
                    sh.xs.cnt_gt = tgt;
                    sh.xs.cnt_eq = teq;
                }
                cluster.sync();  // ---- counts
                int ogt = 0, oeq = 0;
                for (int rr = 0; rr < rank; rr++) {
                    Xch *x = remote_xs(rr);
                    ogt += x->cnt_gt;
                    oeq += x->cnt_eq;
                }
                unsigned long long *cand0 = cluster.map_shared_rank(cand, 0);
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    int pg = ogt + egt[q], pe = oeq + eeq[q];
                    for (int j = 0; j < SUBT; j++) {
                        const int li = kb[q] + j;
                        if (li < slen) {
                            const uint32_t key = key_of(vals[li]);
                            const uint32_t gid = (uint32_t)(slice0 + li);
                            const unsigned long long comp = ((unsigned long long)key << 32) | (0xffffffffu - gid);
                            if (key > kstar) {
                                cand0[pg++] = comp;
                            } else if (key == kstar) {
                                if (pe < krem) cand0[ngt + pe] = comp;
                                pe++;
                            }
                        }
                    }
                }
                if (tid == 0 && rank == 0) sh.xs.ncand = k;
                cluster.sync();  // ---- candidates in CTA 0
            }
            if (a.probs) {
                float *pr = a.probs + (int64_t)row * a.probs_stride + slice0;
                for (int i = tid; i < slen; i += NT) pr[i] = 0.0f;
            }
            if (rank == 0) {
                const int n = sh.xs.ncand;
                int P = 1;
                while (P < n) P <<= 1;
                float *tl = reinterpret_cast<float *>(cand + P);
                int *il = reinterpret_cast<int *>(tl + k);
                if (n <= 512) {
                    // the k best by rank: (key, ~id) composites are distinct, so a survivor's rank
                    // is the count of larger ones; ranks < k are kept (t descending, lower id first)
                    for (int i = tid; i < n; i += NT) {
                        const unsigned long long ci = cand[i];
                        int rk = 0;
                        for (int j = 0; j < n; j++) rk += cand[j] > ci;
                        if (rk < k) {
                            tl[rk] = okey_inv((uint32_t)(ci >> 32));
                            il[rk] = (int)(0xffffffffu - (uint32_t)(ci & 0xffffffffu));
                        }
                    }
                } else {
                    for (int i = n + tid; i < P; i += NT) cand[i] = 0ull;
                    __syncthreads();
                    // bitonic sort, descending on (key, ~id)
                    for (int size = 2; size <= P; size <<= 1) {
                        for (int stride = size >> 1; stride > 0; stride >>= 1) {
                            for (int i = tid; i < P; i += NT) {
                                const int j = i ^ stride;
                                if (j > i) {
                                    const bool desc = (i & size) == 0;
                                    const unsigned long long x = cand[i], y = cand[j];
                                    if (desc ? (x < y) : (x > y)) {
                                        cand[i] = y;
                                        cand[j] = x;
                                    }
                                }
                            }
                            __syncthreads();
                        }
                    }
                    for (int i = tid; i < k; i += NT) {
                        const unsigned long long c = cand[i];
                        tl[i] = okey_inv((uint32_t)(c >> 32));
                        il[i] = (int)(0xffffffffu - (uint32_t)(c & 0xffffffffu));
                    }
                }
                __syncthreads();
                if (a.topk_ids)
                    for (int i = tid; i < k; i += NT) a.topk_ids[(int64_t)row * a.topk_stride + i] = il[i] + a.vocab_offset;
                if (wid == 0) {
                    float *pr = a.probs ? a.probs + (int64_t)row * a.probs_stride : nullptr;
                    token = sample_sorted_list(tl, il, k, p, r, pr, (a.flags & DLLM_MODE_MINP_RELATIVE) != 0);
                }
            }
            }
        } else {
            // ---------------- index-order path -------------------------------------------------
            done = false;
            const float inv_temp = __fdiv_rn(1.0f, p.temperature);
            float mv;
            if (inv_temp > 0.0f && inv_temp < INFINITY) {
                mv = __fmul_rn(__fsub_rn(M, M), inv_temp);
            } else {
                float tm = -INFINITY;
                for (int i = tid; i < slen; i += NT) tm = fmaxf(tm, __fmul_rn(__fsub_rn(vals[i], M), inv_temp));
                tm = block_allreduce(tm, sh.red_f, [](float x, float y) { return fmaxf(x, y); }, -INFINITY);
                if (tid == 0) sh.xs.mt = tm;
                cluster.sync();  // ---- odd temperature
                float tv = -INFINITY;
                if (lane < C) tv = remote_xs(lane)->mt;
                mv = warp_allreduce(tv, [](float x, float y) { return fmaxf(x, y); });
            }
            // P2: exponentials (in place) and fp32 sums per sub-chunk, scanned (in double) in
            // sub-chunk order; the prefix sums of e place the top-p cut
            double sube[4];
            p2_scan<NV4>(vals, kb, S, M, inv_temp, mv, sube);
            mark(DBG_P2L);
            double exE[4], inE[4], totE[4];
            block_scan4_d(sube, sh.red_d, exE, inE, totE);
            double QE[5];
            QE[0] = 0.0;
#pragma unroll
            for (int q = 0; q < 4; q++) QE[q + 1] = QE[q] + totE[q];
            if (tid == 0) mbar_arrive_expect_tx(&sh.xbar[1][par], (uint32_t)(C * sizeof(Push2)));
            if (tid < C) {
                const unsigned long long db = (unsigned long long)__double_as_longlong(QE[4]);
                push16(&sh.in2[par][rank], &sh.xbar[1][par], tid, (uint32_t)db, (uint32_t)(db >> 32),
                       __float_as_uint(vals[0]), 0u);
            }
            mark(DBG_P2);
            if (!xwait(1, par)) rowflags |= ROW_ERR_TIMEOUT;  // ---- #2
            mark(DBG_W2);
            // the pushed values, folded in rank order
            double sum = 0.0, offE = 0.0;
            float e_first;
            {
                const double xd = lane < C ? sh.in2[par][lane].dsum : 0.0;
                e_first = sh.in2[par][0].first_e;
                for (int rr = 0; rr < C; rr++) {
                    if (rr == rank) offE = sum;
                    sum = sum + __shfl_sync(0xffffffffu, xd, rr);
                }
            }
            if (isnan(sum)) {
                // a NaN logit (the maximum ignores it) makes the reference's sum, and so every
                // probability, NaN: no cut is reached and its draw returns the list's last
                // entry (src/sampler.c:176-233).  Every CTA of the cluster sees the same sum.
                token = a.vocab_total - 1;
                done = true;
                goto row_done;
            }

            Chain ch;
            ch.inv_sum = __double2float_rn(1.0 / sum);
            // relative min-p: the largest probability is 1 * inv_sum (its exponential is exp(0))
            ch.min_p = (a.flags & DLLM_MODE_MINP_RELATIVE) ? __fmul_rn(p.min_p, ch.inv_sum) : p.min_p;
            ch.minp = !IDX && p.min_p > 0.0f;
            ch.nokept = 0;
            ch.inv_s2 = 1.0f;
            ch.topp = p.top_p < 1.0f;
            ch.inv_s3 = 1.0f;
            ch.cut_idx = INT_MAX;

            if (ch.minp) {
                CSum s2c = csum_zero(), sac = csum_zero();
                int nk = 0;
                for (int i = tid; i < S; i += NT) {
                    const float pp = __fmul_rn(vals[i], ch.inv_sum);
                    csum_add(sac, pp);
                    if (pp >= ch.min_p) {
                        csum_add(s2c, pp);
                        nk++;
                    }
                }
                const double s2 = block_allreduce(csum_val(s2c), sh.red_d, [](double x, double y) { return x + y; }, 0.0);
                const double sall = block_allreduce(csum_val(sac), sh.red_d, [](double x, double y) { return x + y; }, 0.0);
                nk = block_allreduce(nk, sh.red_i, [](int x, int y) { return x + y; }, 0);
                if (tid == 0) {
                    sh.xs.s2 = s2;
                    sh.xs.s2all = sall;
                    sh.xs.nkept = nk;
                }
                cluster.sync();  // ---- min-p
                double S2 = 0.0, SA = 0.0;
                int NK = 0;
                {
                    Xch *x = remote_xs(lane < C ? lane : 0);
                    const double a2 = lane < C ? x->s2 : 0.0, aa = lane < C ? x->s2all : 0.0;
                    const int an = lane < C ? x->nkept : 0;
                    for (int rr = 0; rr < C; rr++) {
                        S2 = S2 + __shfl_sync(0xffffffffu, a2, rr);
                        SA = SA + __shfl_sync(0xffffffffu, aa, rr);
                        NK += __shfl_sync(0xffffffffu, an, rr);
                    }
                }
                ch.nokept = NK == 0;
                ch.inv_s2 = __double2float_rn(1.0 / (ch.nokept ? SA : S2));
            }

            const bool trk = ch.minp && !ch.nokept;
            double P0[4], P1[4], grand = 0.0;
            int gfm = INT_MAX, glm = -1;
            float gfw = 0.0f;
            if (!trk) {
                // every element is on the list and w = fl(e * inv_sum) [* inv_s2]: prefix sums of
                // w from those of e (the per-element roundings add ~1e-10 at most in practice)
                const double sw = ch.minp ? (double)ch.inv_sum * (double)ch.inv_s2 : (double)ch.inv_sum;
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    P0[q] = sw * (offE + (QE[q] + exE[q]));
                    P1[q] = sw * (offE + (QE[q] + inE[q]));
                }
                grand = sw * sum;
                gfm = 0;
                gfw = w_of(ch, e_first);
                glm = V - 1;
            } else {
            // P3 (min-p filters the list): sums of the list probabilities over this thread's
            // four sub-chunks
            double subd[4];
            int fmem = INT_MAX, lmem = -1;
            float fw = 0.0f;
            p3_scan<true, true, NV4>(vals, kb, slen, slice0, ch, subd, fmem, lmem, fw);
            mark(DBG_P3L);
            double excl[4], incl[4], qtot[4];
            block_scan4_d(subd, sh.red_d, excl, incl, qtot);
            mark(DBG_P3S);
            double Q[5];
            Q[0] = 0.0;
#pragma unroll
            for (int q = 0; q < 4; q++) Q[q + 1] = Q[q] + qtot[q];
            const int bfm = block_allreduce(fmem, sh.red_i, [](int x, int y) { return min(x, y); }, INT_MAX);
            const int blm = block_allreduce(lmem, sh.red_i2, [](int x, int y) { return max(x, y); }, INT_MIN);
            if (fmem == bfm && fmem != INT_MAX) sh.xs.first_w = fw;
            if (tid == 0) {
                sh.xs.tot = Q[4];
                sh.xs.first_member = bfm;
                sh.xs.last_member = blm;
            }
            mark(DBG_P3);
            cluster.sync();  // ---- #3
            mark(DBG_W3);
            double off = 0.0;
            {
                Xch *x = remote_xs(lane < C ? lane : 0);
                const double xt = lane < C ? x->tot : 0.0;
                const int xf = lane < C ? x->first_member : INT_MAX;
                const float xw = lane < C ? x->first_w : 0.0f;
                const int xl = lane < C ? x->last_member : -1;
                for (int rr = 0; rr < C; rr++) {
                    if (rr == rank) off = grand;
                    grand = grand + __shfl_sync(0xffffffffu, xt, rr);
                    const int f = __shfl_sync(0xffffffffu, xf, rr);
                    const float fwv = __shfl_sync(0xffffffffu, xw, rr);
                    if (f < gfm) {
                        gfm = f;
                        gfw = fwv;
                    }
                    glm = max(glm, __shfl_sync(0xffffffffu, xl, rr));
                }
            }
#pragma unroll
            for (int q = 0; q < 4; q++) {
                P0[q] = off + (Q[q] + excl[q]);
                P1[q] = off + (Q[q] + incl[q]);
            }
            }

            int last_idx = ch.minp && !ch.nokept ? glm : V - 1;
            if (ch.topp) {
                const float tp = p.top_p;
                int cut = -1;
                double s3 = grand;
                if (!(tp > 0.0f)) {
                    cut = gfm;
                    s3 = (double)gfw;
                } else {
                    // the single sub-chunk where (float)cumsum first reaches top_p; its warp finds
                    // the cut element cooperatively
                    int qx = -1;
                    unsigned cmx = 0u;
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const bool crosses = __double2float_rn(P1[q]) >= tp && !(__double2float_rn(P0[q]) >= tp);
                        const unsigned cm = __ballot_sync(0xffffffffu, crosses);
                        if (cm && qx < 0) {
                            qx = q;
                            cmx = cm;
                        }
                    }
                    {
                        if (qx >= 0) {
                            const int src = __ffs(cmx) - 1;
                            const double base = __shfl_sync(0xffffffffu, pick4(P0, qx), src);
                            const int cb0 = __shfl_sync(0xffffffffu, pick4(kb, qx), src);
                            constexpr int SL = (SUBT + 31) / 32;
                            const int j0 = lane * SL;
                            double part = 0.0;
                            float wv[SL];
                            bool mem[SL];
#pragma unroll
                            for (int k = 0; k < SL; k++) {
                                const int li = cb0 + j0 + k;
                                const bool in = j0 + k < SUBT && li < slen;
                                const float e = in ? vals[li] : 0.0f;
                                mem[k] = in && member_of(ch, e);
                                wv[k] = mem[k] ? w_of(ch, e) : 0.0f;
                                part = part + (double)wv[k];
                            }
                            double x = part;
#pragma unroll
                            for (int o = 1; o < 32; o <<= 1) {
                                double y = __shfl_up_sync(0xffffffffu, x, o);
                                if (lane >= o) x = y + x;
                            }
                            const double ex = __shfl_up_sync(0xffffffffu, x, 1);
                            double cum = lane == 0 ? base : base + ex;
                            int hitk = -1, lastm = -1;
                            double hitc = 0.0, hitb = 0.0;
#pragma unroll
                            for (int k = 0; k < SL; k++) {
                                if (mem[k] && hitk < 0) {
                                    const double before = cum;
                                    cum = cum + (double)wv[k];
                                    lastm = k;
                                    if (__double2float_rn(cum) >= tp) {
                                        hitk = k;
                                        hitc = cum;
                                        hitb = before;
                                    }
                                }
                            }
                            const unsigned hm = __ballot_sync(0xffffffffu, hitk >= 0);
                            int ci;
                            double cs3;
                            int cfl = 0;
                            if (hm) {
                                const int hl = __ffs(hm) - 1;
                                ci = __shfl_sync(0xffffffffu, cb0 + j0 + hitk, hl);
                                cs3 = __shfl_sync(0xffffffffu, hitc, hl);
                                const double cb4 = __shfl_sync(0xffffffffu, hitb, hl);
                                // (float)x >= tp exactly when x >= thr, the midpoint below tp.  The
                                // reference's prefixes can sit up to thr * w from these: its
                                // (float)(1/sum) may be one ulp away, and its exponentials add a
                                // few 1e-8 relative (TOPP_EXP_DIFF) on their own
                                const double thr = 0.5 * ((double)nextafterf(tp, 0.0f) + (double)tp);
                                double w = ulp_rel(ch.inv_sum) + TOPP_EXP_DIFF;
                                if (ch.minp) w += ulp_rel(ch.inv_s2);
                                w *= thr;
                                if (fabs(cs3 - thr) <= w || fabs(cb4 - thr) <= w) cfl = ROW_TOPP_EDGE;
                            } else {
                                // rounding disagreed with the sub-chunk sum: cut at its last member
                                const unsigned lm2 = __ballot_sync(0xffffffffu, lastm >= 0);
                                const int ll = lm2 ? 31 - __clz(lm2) : 0;
                                ci = __shfl_sync(0xffffffffu, cb0 + j0 + lastm, ll);
                                cs3 = base + __shfl_sync(0xffffffffu, x, 31);
                                cfl = ROW_TOPP_EDGE;  // the sub-chunk sums and the elements disagree on the crossing
                            }
                            if (lane == 0) {
                                sh.xs.cut_idx = slice0 + ci;
                                sh.xs.cut_flags = cfl;
                                sh.xs.cut_s3 = cs3;
                            }
                        }
                    }
                    __syncthreads();
                    if (tid == 0) mbar_arrive_expect_tx(&sh.xbar[2][par], (uint32_t)(C * sizeof(Push4)));
                    if (tid < C) {
                        const unsigned long long sb = (unsigned long long)__double_as_longlong(sh.xs.cut_s3);
                        push16(&sh.in4[par][rank], &sh.xbar[2][par], tid, (uint32_t)sh.xs.cut_idx,
                               (uint32_t)sh.xs.cut_flags, (uint32_t)sb,
                               (uint32_t)(sb >> 32));
                    }
                    if (IDX && row + ncl < a.rows) {
                        // the next row's history table, while the cut comes in (its ids and
                        // offsets were loaded during this row's P1)
                        const dllm_sampler_params pn = a.bparams;
                        pre_flags = build_table(a.hist_ids && a.hist_off &&
                                                (pn.repetition > 1.0f || pn.presence != 0.0f || pn.frequency != 0.0f));
                        prebuilt = true;
                    }
                    if (!xwait(2, par)) rowflags |= ROW_ERR_TIMEOUT;  // ---- #4
                    {
                        const int xc = lane < C ? sh.in4[par][lane].cut_idx : -1;
                        const double xs3 = lane < C ? sh.in4[par][lane].cut_s3 : 0.0;
                        const unsigned hm = __ballot_sync(0xffffffffu, xc >= 0);
                        const int xf = lane < C ? sh.in4[par][lane].cut_flags : 0;
                        if (hm) {
                            const int src = __ffs(hm) - 1;
                            cut = __shfl_sync(0xffffffffu, xc, src);
                            s3 = __shfl_sync(0xffffffffu, xs3, src);
                            rowflags |= __shfl_sync(0xffffffffu, xf, src);
                        }
                    }
                }
                if (cut >= 0) {
                    ch.cut_idx = cut;
                    last_idx = cut;
                }
                ch.inv_s3 = __double2float_rn(1.0 / s3);
            }
            if (rank == 0 && tid == 0) {
                hdr->M = M;
                hdr->inv_temp = inv_temp;
                hdr->mv = mv;
                hdr->inv_sum = ch.inv_sum;
                hdr->min_p = ch.min_p;
                hdr->inv_s2 = ch.inv_s2;
                hdr->inv_s3 = ch.inv_s3;
                hdr->r = r;
                hdr->cut_idx = ch.cut_idx;
                hdr->last_idx = last_idx;
                hdr->flags = rowflags;
                hdr->minp = ch.minp;
                hdr->nokept = ch.nokept;
                hdr->topp = ch.topp;
                hdr->done = 0;
            }
            mark(DBG_CUT);

            // P4: sub-chunk records (exact fp32 running-sum functions) and warp records
            {
                const double inv3 = ch.topp ? (double)ch.inv_s3 : 1.0;
                uint32_t gb[4];
                bool pred[4], near[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const float A0 = __double2float_rn(P0[q] * inv3);
                    const float A1 = __double2float_rn(P1[q] * inv3);
                    const uint32_t e0 = fbits(A0) >> 23, e1 = fbits(A1) >> 23;
                    pred[q] = A0 > 0.0f && e0 == e1 && e0 >= 1u && e0 <= 253u;
                    gb[q] = (pred[q] ? e0 : 127u) << 23;
                    // the draw can land here: the running sum stays within DRAW_WINDOW of the
                    // exact prefix (the fp32 drift), so the walk will replay this warp range
                    near[q] = A1 > 0.0f && A1 + DRAW_WINDOW > r && A0 - DRAW_WINDOW <= r;
                }
                float g0[4], g1[4];
                bool anyq[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    g0[q] = bitsf(gb[q]);
                    g1[q] = bitsf(gb[q] | 1u);
                }
                float *pr = a.probs ? a.probs + (int64_t)row * a.probs_stride + slice0 : nullptr;
                // elements of sub-chunk q at offset <= lim[q] lie inside the top-p prefix.  A
                // sub-chunk wholly past the cut gets scale 0; the entries past the cut in the
                // crossing sub-chunk are zeroed here (the walk forms q = 0 for them by index
                // anyway).  Without min-p a sub-chunk has a nonzero draw probability iff some
                // e > 0 in it (sube > 0), up to underflow of e * inv_sum, which leaves an all-zero
                // run that the walk handles like any other; min-p removes whole sub-chunks, so
                // there the loop tracks the largest probability instead.
                const float scale3 = ch.topp ? ch.inv_s3 : 1.0f;
                float s3q[4], qmax[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    qmax[q] = 0.0f;
                    const long long d = (long long)ch.cut_idx - (slice0 + kb[q]);
                    const int lim = !ch.topp ? SUBT : (int)(d < 0 ? -1 : (d > SUBT ? SUBT : d));
                    s3q[q] = lim < 0 ? 0.0f : scale3;
                    anyq[q] = lim >= 0 && sube[q] > 0.0;
                    if (lim >= 0 && lim < SUBT - 1 && kb[q] < S)
                        for (int k = lim + 1; k < SUBT; k++) vals[kb[q] + k] = 0.0f;
                }
                __syncwarp();
                if (ch.minp) {
                    p4_scan<true, NV4>(vals, kb, ch, s3q, g0, g1, qmax);
#pragma unroll
                    for (int q = 0; q < 4; q++) anyq[q] = anyq[q] && qmax[q] > 0.0f;
                } else {
                    p4_scan<false, NV4>(vals, kb, ch, s3q, g0, g1, qmax);
                }
                mark(DBG_P4L);
                if (pr) {
#pragma unroll 1
                    for (int q = 0; q < 4; q++)
#pragma unroll 1
                        for (int j = 0; j < SUBT; j++) {
                            const int li = pick4(kb, q) + j;
                            if (li < slen) pr[li] = q_of(ch, vals[li], slice0 + li);
                        }
                }
                WRec *recs = row_recs(a, row);
                float *stash = row_stash(a, row);
                // warp records for the four quarters.  Per quarter: the prefix of CLEAN
                // sub-chunks in one binade, an optional boundary sub-chunk, and the suffix after
                // it (PBS), else MIXED.  The record types, the slot claims and the copies out of
                // the slice come first; then the next row's bulk copy is issued, and the
                // composition scans (registers and shuffles only) overlap it.
                int ctype[4], ce[4];
                uint32_t c0[4], c1[4];
                unsigned cleanm[4], nonconf[4];
                int e_first[4], jx[4], sfrom[4], e_s[4], type[4], bchunk[4];
                uint32_t a0[4], a1[4], b0[4], b1[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const uint32_t lim = gb[q] + (1u << 23);
                    ctype[q] = !anyq[q] ? REC_IDENT
                                        : ((pred[q] && fbits(g0[q]) < lim && fbits(g1[q]) < lim) ? REC_CLEAN : REC_MIXED);
                    ce[q] = (int)(gb[q] >> 23);
                    c0[q] = fbits(g0[q]) - gb[q];
                    c1[q] = fbits(g1[q]) - (gb[q] | 1u);
                    cleanm[q] = __ballot_sync(0xffffffffu, ctype[q] == REC_CLEAN);
                }
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    e_first[q] = cleanm[q] ? __shfl_sync(0xffffffffu, ce[q], __ffs(cleanm[q]) - 1) : 0;
                    nonconf[q] = __ballot_sync(0xffffffffu, ctype[q] == REC_MIXED ||
                                                                (ctype[q] == REC_CLEAN && ce[q] != e_first[q]));
                    jx[q] = nonconf[q] ? __ffs(nonconf[q]) - 1 : 32;
                    const bool pin = lane < jx[q] && ctype[q] == REC_CLEAN;
                    a0[q] = pin ? c0[q] : 0u;
                    a1[q] = pin ? c1[q] : 0u;
                }
                const bool any_nonconf = (nonconf[0] | nonconf[1] | nonconf[2] | nonconf[3]) != 0u;
                if (!any_nonconf) {
                    // every quarter is one run (or empty): no boundary, no suffix
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        sfrom[q] = 32;
                        bchunk[q] = -1;
                        e_s[q] = 0;
                        type[q] = cleanm[q] ? REC_CLEAN : REC_IDENT;
                        b0[q] = b1[q] = 0u;
                    }
                } else {
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const int tj = __shfl_sync(0xffffffffu, ctype[q], jx[q] & 31);
                        sfrom[q] = !nonconf[q] ? 32 : (tj == REC_MIXED ? jx[q] + 1 : jx[q]);
                        bchunk[q] = nonconf[q] && tj == REC_MIXED ? jx[q] : -1;
                        const unsigned sclean = __ballot_sync(0xffffffffu, lane >= sfrom[q] && ctype[q] == REC_CLEAN);
                        e_s[q] = sclean ? __shfl_sync(0xffffffffu, ce[q], __ffs(sclean) - 1) : 0;
                        const unsigned sbad = __ballot_sync(
                            0xffffffffu,
                            lane >= sfrom[q] && (ctype[q] == REC_MIXED || (ctype[q] == REC_CLEAN && ce[q] != e_s[q])));
                        type[q] = !nonconf[q] ? (cleanm[q] ? REC_CLEAN : REC_IDENT) : (sbad ? REC_MIXED : REC_PBS);
                        const bool sin = lane >= sfrom[q] && ctype[q] == REC_CLEAN;
                        b0[q] = sin ? c0[q] : 0u;
                        b1[q] = sin ? c1[q] : 0u;
                    }
                }
                mark(DBG_P3);  // (index-order path: record classification)
                // stash / wide slots for the four quarters: one claim per warp on CTA 0's counter
                bool need_st[4], need_wd[4];
                int n_st = 0, n_wd = 0;
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    need_st[q] = type[q] == REC_PBS && bchunk[q] >= 0;
                    need_wd[q] = type[q] == REC_MIXED || __any_sync(0xffffffffu, near[q]);
                    n_st += need_st[q];
                    n_wd += need_wd[q];
                }
                int nslot[4] = {-1, -1, -1, -1}, wslot[4] = {-1, -1, -1, -1};
                if (n_st + n_wd) {
                    int base = 0;
                    if (lane == 0) base = atomicAdd(cluster.map_shared_rank(&sh.slots[par], 0), n_st | (n_wd << 16));
                    base = __shfl_sync(0xffffffffu, base, 0);
                    int st_next = base & 0xffff, wd_next = base >> 16;
#pragma unroll 1
                    for (int q = 0; q < 4; q++) {
                        const int bchunkq = pick4(bchunk, q);
                        // boundary sub-chunk exponentials -> a stash slot (when one is free)
                        if (pick4(need_st, q)) {
                            const int ns = st_next < STASH_SLOTS ? st_next : -1;
                            st_next++;
                            if (ns >= 0) {
                                const int sb = (q * NT + 32 * wid + bchunkq) * SUBT;
                                float *qs = stash + ns * STASH_STRIDE;
                                if (lane == 0) qs[0] = __int_as_float(slice0 + sb);
                                for (int k = lane; k < SUBT; k += 32) qs[1 + k] = vals[sb + k];  // e; the walk forms q
                            } else if (timing) {
                                dbg_add(DBG_STASH_MISS, 1);
                            }
                            if (q == 0) nslot[0] = ns;
                            else if (q == 1) nslot[1] = ns;
                            else if (q == 2) nslot[2] = ns;
                            else nslot[3] = ns;
                        }
                        // several binade changes in this warp's range, or the draw may land in it:
                        // keep every exponential so the walk replays them without recomputing
                        if (pick4(need_wd, q)) {
                            const int wsl = wd_next < WIDE_SLOTS ? wd_next : -1;
                            wd_next++;
                            if (wsl >= 0) {
                                const int kq = pick4(kb, q);
                                float *ws = row_wide(a, row) + wsl * wide_stride(SUBT) + lane * SUBT;
#pragma unroll 1
                                for (int k = 0; k < SUBT; k += 4)
                                    *reinterpret_cast<float4 *>(ws + k) = *reinterpret_cast<const float4 *>(vals + kq + k);
                            } else if (timing) {
                                dbg_add(DBG_STASH_MISS, 1);
                            }
                            if (q == 0) wslot[0] = wsl;
                            else if (q == 1) wslot[1] = wsl;
                            else if (q == 2) wslot[2] = wsl;
                            else wslot[3] = wsl;
                        }
                    }
                }
                mark(DBG_W3);  // (slot claims and copies)
                // the slice is no longer read: the next row's bulk copy starts here
                if (use_tma && !dbuf) {
                    fence_proxy_async();
                    __syncthreads();
                    if (tid == 0 && row + ncl < a.rows) issue_row_copy(row + ncl, 0);
                    copy_issued = true;
                }
                mark(DBG_P3L);  // (barrier and bulk-copy issue)
                compose_scan4(a0, a1);
                if (any_nonconf) compose_scan4(b0, b1);
                mark(DBG_P3S);  // (compositions)
                if (lane == 31) {
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        WRec wr;
                        wr.meta = pack_meta(type[q], bchunk[q], sfrom[q], e_first[q], e_s[q]);
                        wr.p0 = a0[q];
                        wr.p1 = a1[q];
                        wr.s0 = b0[q];
                        wr.s1 = b1[q];
                        wr.nslot = (int16_t)nslot[q];
                        wr.wslot = (int16_t)wslot[q];
                        recs[rank * 4 * NW + q * NW + wid] = wr;
                        if (type[q] == REC_PBS && timing) dbg_add(DBG_PBS, 1);
                    }
                }
            }
            mark(DBG_P4);
        }

    row_done:
        if (use_tma && !dbuf && !copy_issued) {
            // every read of this row's slice is done: the next row's bulk copy starts now and
            // overlaps the end of this row and the start of the next
            __syncthreads();
            if (tid == 0 && row + ncl < a.rows) {
                fence_proxy_async();
                issue_row_copy(row + ncl, 0);
            }
        }
        if (done && rank == 0 && tid == 0) {
            if (token < 0) token = 0;
            a.token[row] = token + a.vocab_offset;
            if (a.status) a.status[row] = rowflags;
            hdr->done = 1;
        }
        mark(DBG_TOPK);
        // the status bits this CTA saw; the walk kernel ORs every CTA's into the row's status
        if (tid == 0) hdr->rank_flags[rank] = rowflags;
        fence_proxy_async();    // order this row's generic accesses of the slice before the next bulk copy
        cluster_sync_relaxed();  // ---- end of row: peers may reuse their shared memory
        if (dbuf && tid == 0 && use_tma && row + 2 * ncl < a.rows) issue_row_copy(row + 2 * ncl, buf);
        mark(DBG_WEND);
    }
}

// ----------------------------------------------------------------------------------------
// kernel B: one warp per row draws with the exact fp32 running sum

template <int DT, int SUBT>
__global__ void __launch_bounds__(WALK_WARPS * 32, 4) walk_rows_kernel(const KernelArgs a) {
    __shared__ int hls[WALK_WARPS][HLIST];
    __shared__ __align__(16) float rbuf[WALK_WARPS][32 * SUBT];
    extern __shared__ __align__(16) unsigned char wdyn[];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int row = blockIdx.x * WALK_WARPS + wid;
    if (threadIdx.x == 0) g_dbg = a.dbg;
    __syncthreads();
    if (row >= a.rows) return;
    const RowHdr h = *row_hdr(a, row);
    int cl_flags = 0;  // status bits of the row's other CTAs (a bounded wait that ran out)
    for (int c = 0; c < a.cluster; c++) cl_flags |= h.rank_flags[c];
    if (h.done) {
        if (lane == 0 && a.status && cl_flags) a.status[row] |= cl_flags;
        return;
    }
    const long long t_start = clock64();
    // the row's warp records and used stash slots -> shared memory, all copies in flight at once
    const size_t recb = ((size_t)a.nrec * sizeof(WRec) + 127) & ~(size_t)127;
    unsigned char *wsm = wdyn + (size_t)wid * walk_smem_per_warp(a.nrec);
    const WRec *recs = reinterpret_cast<const WRec *>(wsm);
    const float *stash = reinterpret_cast<const float *>(wsm + recb);
    {
        const unsigned char *grec = reinterpret_cast<const unsigned char *>(row_recs(a, row));
        const int nrec16 = (int)(((size_t)a.nrec * sizeof(WRec) + 15) / 16);
        for (int i = lane; i < nrec16; i += 32) cp_async16(wsm + 16 * i, grec + 16 * i);
        const int ns = STASH_SLOTS;  // all slots: which ones are used shows only in the records
        const unsigned char *gst = reinterpret_cast<const unsigned char *>(row_stash(a, row));
        for (int i = lane; i < ns * STASH_STRIDE / 4; i += 32) cp_async16(wsm + recb + 16 * i, gst + 16 * i);
        cp_async_wait_all();
        __syncwarp();
    }
    if (lane == 0) dbg_add(DBG_B_PRE, (unsigned long long)(clock64() - t_start));
    const dllm_sampler_params p = a.rparams ? a.rparams[row] : a.bparams;
    Chain ch;
    ch.inv_sum = h.inv_sum;
    ch.min_p = h.min_p;
    ch.inv_s2 = h.inv_s2;
    ch.inv_s3 = h.inv_s3;
    ch.cut_idx = h.cut_idx;
    ch.minp = h.minp;
    ch.nokept = h.nokept;
    ch.topp = h.topp;
    const float r = h.r;
    const int C = a.cluster, NW = a.nrec / (4 * C), NT = NW * 32, S = a.S, V = a.vocab;
    const bool use_hist = a.hist_ids && a.hist_off &&
                          (p.repetition > 1.0f || p.presence != 0.0f || p.frequency != 0.0f);
    const float inv_rep = __fdiv_rn(1.0f, p.repetition);
    const bool true_div = (a.flags & DLLM_MODE_PEN_TRUE_DIV) != 0;
    const uint32_t *mrow = a.mask ? a.mask + (int64_t)row * a.mask_stride : nullptr;
    int *hl = hls[wid];
    int nh = 0;
    bool hist_overflow = false;

    // history ids that fall in [lo, hi) (local indices) -> this warp's list
    auto load_region_hist = [&](int lo, int hi) {
        nh = 0;
        hist_overflow = false;
        if (!use_hist) return;
        const int64_t h0 = a.hist_off[row], h1 = a.hist_off[row + 1];
        for (int64_t j0 = h0; j0 < h1; j0 += 32) {
            const int64_t j = j0 + lane;
            int li = -1;
            if (j < h1) {
                const int id = a.hist_ids[j];
                if (id >= 0 && id < a.vocab_total) li = id - a.vocab_offset;
            }
            const bool in = li >= lo && li < hi;
            const unsigned m = __ballot_sync(0xffffffffu, in);
            if (in) {
                const int o = nh + __popc(m & ((1u << lane) - 1u));
                if (o < HLIST) hl[o] = li;
            }
            nh += __popc(m);
        }
        __syncwarp();
        if (nh > HLIST) hist_overflow = true;
    };
    // raw (masked) logit of element li
    auto raw_of = [&](int li) -> float {
        if (li >= V) return -INFINITY;
        float v;
        if (DT == DLLM_DTYPE_F32)
            v = __ldcs((const float *)a.logits + (int64_t)row * a.row_stride + li);
        else
            v = bitsf((uint32_t)__ldcs((const unsigned short *)a.logits + (int64_t)row * a.row_stride + li) << 16);
        if (mrow && !((mrow[li >> 5] >> (li & 31)) & 1u)) v = -INFINITY;
        return v;
    };
    // draw probability of element li from its raw logit v: penalties, temperature, softmax, cuts
    auto qval = [&](float v, int li) -> float {
        if (use_hist && nh > 0) {
            int c = 0;
            if (!hist_overflow) {
                for (int i = 0; i < min(nh, HLIST); i++) c += hl[i] == li;
            } else {
                const int64_t h0 = a.hist_off[row], h1 = a.hist_off[row + 1];
                for (int64_t j = h0; j < h1; j++) {
                    const int id = a.hist_ids[j];
                    c += id >= 0 && id < a.vocab_total && id - a.vocab_offset == li;
                }
            }
            if (c > 0) {
                if (p.presence != 0.0f) v = __fsub_rn(v, p.presence);
                if (p.frequency != 0.0f) v = __fsub_rn(v, __fmul_rn(__int2float_rn(c), p.frequency));
                if (p.repetition > 1.0f)
                    for (int k = 0; k < c; k++) {
                        if (v < 0.0f) v = __fmul_rn(v, p.repetition);
                        else v = true_div ? __fdiv_rn(v, p.repetition) : __fmul_rn(v, inv_rep);
                    }
            }
        }
        const float e = exp_t(__fsub_rn(__fmul_rn(__fsub_rn(v, h.M), h.inv_temp), h.mv));
        return q_of(ch, e, li);
    };
    // replays elements [start, start + n) (n <= 32 * SUBT) on the exact running sum, from the
    // row's inputs staged in shared memory with coalesced loads
    float *rv = rbuf[wid];
    auto replay_region = [&](int start, int n, uint32_t &cbv) -> int {
        const long long t0 = clock64();
        if (lane == 0) dbg_add(DBG_RECOMP, 1);
        load_region_hist(start, start + n);
        // raw logits of the region: 16-byte asynchronous copies where aligned, all in flight
        const int nv = max(0, min(n, V - start));
        int nc = 0;
        if (DT == DLLM_DTYPE_F32 && a.vec_ok) {
            nc = nv & ~3;
            const float *src = (const float *)a.logits + (int64_t)row * a.row_stride + start;
            for (int i = lane; i < nc / 4; i += 32) cp_async16(rv + 4 * i, src + 4 * i);
        }
#pragma unroll 1
        for (int i = nc + lane; i < n; i += 32) rv[i] = raw_of(start + i);
        cp_async_wait_all();
        __syncwarp();
#pragma unroll 1
        for (int i = lane; i < n; i += 32) {
            const int li = start + i;
            float v = rv[i];
            if (i < nc && mrow && !((mrow[li >> 5] >> (li & 31)) & 1u)) v = -INFINITY;
            rv[i] = li < V ? qval(v, li) : 0.0f;
        }
        __syncwarp();
        const int res = replay_elems<SUBT>(n, start, cbv, r, rv);
        __syncwarp();
        if (lane == 0) dbg_add(DBG_B_RECOMP, (unsigned long long)(clock64() - t0));
        return res;
    };

    uint32_t cb = 0u;  // running sum, starts at +0.0f
    int res = -1;
    for (int gw0 = 0; gw0 < a.nrec && res == -1; gw0 += 32) {
        const int n = min(32, a.nrec - gw0);
        WRec wl;
        wl.meta = REC_IDENT;
        wl.p0 = wl.p1 = wl.s0 = wl.s1 = 0u;
        wl.nslot = wl.wslot = -1;
        if (lane < n) wl = recs[gw0 + lane];
        const int ty = (int)(wl.meta & 3u);
        const int ep = (int)((wl.meta >> 16) & 255u);
        auto expandA0 = [&](int j, uint32_t &cbv) -> int {
            if (lane == 0) dbg_add(DBG_EXPAND, 1);
            const int g = gw0 + j;
            const int rr = g / (4 * NW), kk = g % (4 * NW), q = kk / NW, w = kk % NW;
            const int start = rr * S + (q * NT + 32 * w) * SUBT;
            const int rend = rr * S + S;  // sub-chunks past the slice end hold nothing
            const int wslot = __shfl_sync(0xffffffffu, (int)wl.wslot, j);
            bool wide_in = false;
            // replays [st, st + n) of this warp range: from its wide slot when the cluster
            // kernel kept one (copied in once), else recomputed from the row's inputs
            auto replay_clamped = [&](int st, int n, uint32_t &cbv) -> int {
                n = min(n, rend - st);
                if (n <= 0) return -1;
                if (wslot < 0) return replay_region(st, n, cbv);
                if (!wide_in) {
                    const float *wsrc = row_wide(a, row) + wslot * wide_stride(SUBT);
                    for (int i = lane; i < 8 * SUBT; i += 32) cp_async16(rv + 4 * i, wsrc + 4 * i);
                    cp_async_wait_all();
                    __syncwarp();
                    // the slot holds exponentials: draw probabilities as the cluster kernel forms them
                    for (int i = lane; i < 32 * SUBT; i += 32) rv[i] = q_of(ch, rv[i], start + i);
                    __syncwarp();
                    wide_in = true;
                }
                const int res = replay_elems<SUBT>(n, st, cbv, r, rv + (st - start));
                __syncwarp();
                return res;
            };
            const uint32_t meta = __shfl_sync(0xffffffffu, wl.meta, j);
            // at most two replays (a PBS record's boundary sub-chunk, then its suffix) through
            // one call site: stage 0 whole range, 1 boundary, 2 suffix check, 3 suffix
            int st = start, nn = 32 * SUBT, stage = 0;
            uint32_t c = cbv, s0 = 0u, s1 = 0u;
            int esuf = 0, sfrom = 32;
            if ((int)(meta & 3u) == REC_PBS) {
                const int bc = (int)((meta >> 2) & 63u);
                const int epre = (int)((meta >> 16) & 255u);
                sfrom = (int)((meta >> 8) & 63u);
                esuf = (int)(meta >> 24);
                const uint32_t p0 = __shfl_sync(0xffffffffu, wl.p0, j), p1 = __shfl_sync(0xffffffffu, wl.p1, j);
                s0 = __shfl_sync(0xffffffffu, wl.s0, j);
                s1 = __shfl_sync(0xffffffffu, wl.s1, j);
                const int slot = __shfl_sync(0xffffffffu, (int)wl.nslot, j);
                if (apply_run(c, epre, p0, p1) && !(r < bitsf(c))) {
                    stage = 2;
                    if (bc != 63 && slot >= 0) {
                        const float *qs = stash + slot * STASH_STRIDE;
                        const int sbase = __float_as_int(qs[0]);
                        // the slot holds exponentials: probabilities into the region buffer
                        for (int k = lane; k < SUBT; k += 32) rv[k] = q_of(ch, qs[1 + k], sbase + k);
                        __syncwarp();
                        const int found = replay_elems<SUBT>(SUBT, sbase, c, r, rv);
                        __syncwarp();
                        wide_in = false;  // the region buffer no longer holds the wide slot
                        if (found != -1) return found;
                    } else if (bc != 63) {
                        st = start + bc * SUBT;
                        nn = SUBT;
                        stage = 1;
                    }
                } else {
                    c = cbv;
                }
            }
            for (int it = 0; it < 2; it++) {
                if (stage == 2) {
                    uint32_t c2 = c;
                    if (apply_run(c2, esuf, s0, s1) && !(r < bitsf(c2))) {
                        cbv = c2;
                        return -1;
                    }
                    st = start + sfrom * SUBT;
                    nn = (32 - sfrom) * SUBT;
                    stage = 3;
                }
                const int found = replay_clamped(st, nn, c);
                if (found != -1 || stage != 1) {
                    cbv = c;
                    return found;
                }
                stage = 2;
            }
            cbv = c;
            return -2;
        };
        const int tyw = ty == REC_PBS ? REC_MIXED : ty;
        res = walk_records(n, tyw, ep, wl.p0, wl.p1, cb, r, 1 << 12, expandA0);
    }
    if (lane == 0) {
        int flags = h.flags | cl_flags;
        if (res == -2) flags |= ROW_ERR_WALK;
        a.token[row] = (res >= 0 ? res : h.last_idx) + a.vocab_offset;
        if (a.status) a.status[row] = flags;
        dbg_add(DBG_WALK_CYC, (unsigned long long)(clock64() - t_start));
    }
}

}  // namespace
}  // namespace dllm
