// dllm_launch.cu -- launch configuration and launch of the fused sampler kernels.
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>

#include <mutex>
#include <utility>
#include <vector>

#include "dllm_kernel.cuh"

namespace dllm {

static unsigned long long *g_host_dbg = nullptr;  // device counters for KernelArgs::dbg
static int g_sm_count = 0;

static const int kSUBs[] = {4, 12, 20, 28, 36, 44, 52, 60};

// getters per instantiation, defined in dllm_kernel_inst.cu (compiled once per sub-chunk length)
#define DLLM_DECL(L) KernelFn kernel_a_f32_##L(); KernelFn kernel_a_bf16_##L(); \
    KernelFn kernel_b_f32_##L(); KernelFn kernel_b_bf16_##L(); KernelFn kernel_a_idx_f32_##L();
DLLM_DECL(4) DLLM_DECL(12) DLLM_DECL(20) DLLM_DECL(28) DLLM_DECL(36) DLLM_DECL(44) DLLM_DECL(52) DLLM_DECL(60)
#undef DLLM_DECL

// which = 0: the cluster kernel, 1: the walk kernel, 2: the cluster kernel's index-order-only
// variant (fp32)
static KernelFn kernel_for(int dtype, int SUB, int which = 0) {
    const bool bf = dtype == DLLM_DTYPE_BF16;
    if (which == 2 && bf) return nullptr;
    switch (SUB) {
#define DLLM_CASE(L) case L: return which == 1 ? (bf ? kernel_b_bf16_##L() : kernel_b_f32_##L()) \
                                  : which == 2 ? kernel_a_idx_f32_##L() \
                                               : (bf ? kernel_a_bf16_##L() : kernel_a_f32_##L());
        DLLM_CASE(4) DLLM_CASE(12) DLLM_CASE(20) DLLM_CASE(28) DLLM_CASE(36) DLLM_CASE(44) DLLM_CASE(52) DLLM_CASE(60)
#undef DLLM_CASE
        default: return nullptr;
    }
}

static size_t union_bytes(int htab, int cand_entries) {
    const size_t u = (size_t)8 * htab, cb = (size_t)8 * cand_entries;
    return u > cb ? u : cb;
}

int nrec_for(const LaunchCfg &cfg) { return 4 * (cfg.threads / 32) * cfg.cluster; }

// Function attributes, set once per (device, kernel): the largest dynamic shared memory the
// device allows the kernel (a launch still asks only for what it uses) and cluster sizes above 8.
namespace {
std::mutex g_attr_mu;
std::vector<std::pair<int, const void *>> g_attr_done;
}  // namespace

static cudaError_t set_attrs(KernelFn fn, size_t smem, bool cluster = true) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(g_attr_mu);
    for (auto &d : g_attr_done)
        if (d.first == dev && d.second == (const void *)fn) return cudaSuccess;
    int optin = 0;
    e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, (const void *)fn);
    if (e != cudaSuccess) return e;
    // the dynamic part may use what the kernel's static shared memory leaves of the block limit
    const int dyn_max = optin - (int)fa.sharedSizeBytes;
    if (dyn_max < 0 || (size_t)dyn_max < smem) return cudaErrorInvalidValue;
    e = cudaFuncSetAttribute((const void *)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn_max);
    if (e != cudaSuccess) return e;
    if (cluster) {
        e = cudaFuncSetAttribute((const void *)fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
    }
    g_attr_done.push_back({dev, (const void *)fn});
    return cudaSuccess;
}

// Environment switches, read once per process.
static bool no_idx_variant() {
    static const bool v = getenv("DLLM_NO_IDX_VARIANT") != nullptr;
    return v;
}
static int dbg_rank_env() {
    static const int v = getenv("DLLM_DBG_RANK") ? atoi(getenv("DLLM_DBG_RANK")) : 0;
    return v;
}

// Test hook: the bounded wait that the next launches make run out (FAULT_NONE = none).
static int g_fault_site = FAULT_NONE;
static long long g_fault_limit = WAIT_LIMIT;

dllm_status set_fault_injection(int site, long long polls) {
    if (site < FAULT_NONE || site > FAULT_EXCHANGE_WAIT || (site != FAULT_NONE && polls < 1))
        return DLLM_ERR_INVALID_ARG;
    g_fault_site = site;
    g_fault_limit = site == FAULT_NONE ? WAIT_LIMIT : polls;
    return DLLM_OK;
}

static int active_clusters(KernelFn fn, int C, int NT, size_t smem) {
    if (set_attrs(fn, smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cudaLaunchConfig_t lc = {};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = C;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    lc.gridDim = dim3(C * 16);
    lc.blockDim = dim3(NT);
    lc.dynamicSmemBytes = smem;
    lc.attrs = at;
    lc.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, (const void *)fn, &lc) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

static int pow2_at_least(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}

dllm_status choose_config(int vocab, int dtype, int hist_bound, int topk_bound, bool latency, LaunchCfg *cfg) {
    if (vocab <= 0 || !cfg) return DLLM_ERR_INVALID_ARG;
    if (topk_bound > KMAX) return DLLM_ERR_UNSUPPORTED;
    if (g_sm_count == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev);
        if (g_sm_count <= 0) g_sm_count = 148;
    }
    // top-k: survivor sort buffer plus the final list
    const int cand_entries = topk_bound > 0 ? CAND_CAP + 2 * pow2_at_least(topk_bound) : 0;
    // DLLM_FORCE_CFG="C,NT[,SUB[,NBUF]]" pins the cluster size / block size / sub-chunk (tuning)
    int force_c = 0, force_nt = 0, force_l = 0, force_b = 0;
    if (const char *f = getenv("DLLM_FORCE_CFG")) sscanf(f, "%d,%d,%d,%d", &force_c, &force_nt, &force_l, &force_b);
    static const int Cs[] = {1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16};
    static const int NTs[] = {128, 160, 192, 224, 256, 320, 384, 448, 512};
    double best = 1e300;
    LaunchCfg bc = {};
    // Latency mode: 512 threads per CTA and the smallest cluster whose slices give each thread
    // at most about 32 elements (measured on B200 for one-row decode at vocab 128256: 27 us per
    // step at 8 x 512 against 33 us with the throughput configuration, 7 x 256).
    int lat_c = 0;
    if (latency && !force_c) {
        lat_c = (vocab + 512 * 32 - 1) / (512 * 32);
        if (lat_c > 16) lat_c = 16;
        if (lat_c < 1) lat_c = 1;
    }
    for (int C : Cs) {
        for (int NT : NTs) {
            if (force_c && (C != force_c || (force_nt && NT != force_nt))) continue;
            if (lat_c && (C != lat_c || NT != 512)) continue;
            // slice: the smallest multiple of the sub-chunk length covering vocab / C; a thread owns
            // up to four sub-chunks, so the sub-chunk length is the smallest that covers the slice
            const int need = (vocab + C - 1) / C;
            const int per = (need + 4 * NT - 1) / (4 * NT);
            int L = -1;
            for (int lt : kSUBs)
                if (lt >= per && (!force_l || lt == force_l)) {
                    L = lt;
                    break;
                }
            if (L < 0) continue;
            const int S = (need + L - 1) / L * L;
            if ((long long)S * (C - 1) >= vocab && C > 1) continue;  // an idle CTA
            int hb = hist_bound < S ? hist_bound : S;
            int htab = pow2_at_least(2 * (hb > 16 ? hb : 16));
            if (htab > 16384) htab = 16384;
            // one or two slice buffers (with two, the next row's bulk copy overlaps this row)
            for (int nbuf = 2; nbuf >= 1; nbuf--) {
                if (force_b && nbuf != force_b) continue;
                const size_t smem = (size_t)nbuf * (S + L) * 4 + union_bytes(htab, cand_entries);
                if (smem > 220 * 1024) continue;
                KernelFn fn = kernel_for(dtype, L);
                const int nact = active_clusters(fn, C, NT, smem);
                if (nact <= 0) continue;
                // cost: modelled time of a 1024-row batch: rows per co-resident cluster times a
                // per-row latency made of a fixed part (barriers, exchanges, serial phases; grows
                // with the cluster size) and the streaming loops (elements per thread, slowed by
                // the threads sharing each SM).  Fitted to B200 measurements of vocab 256000.
                const double per_sm = (double)nact * C / g_sm_count;
                const double sm_threads = (per_sm < 1.0 ? 1.0 : per_sm) * NT;
                const double load = sm_threads / 512.0 < 1.0 ? 1.0 : sm_threads / 512.0;  // fewer warps: latency-bound
                // two or more CTAs of different clusters per SM overlap one row's serial phases
                // with another's loops
                const double fixed_us = (10.0 + 0.2 * C) * (per_sm >= 1.5 ? 0.75 : 1.0) + (nbuf == 2 ? 0.0 : 2.5);
                const double row_us = fixed_us + 0.1 * (4.0 * L) * load;
                const double cost = ((1024 + nact - 1) / nact) * row_us * (1.0 + 1.0 / L);
                if (getenv("DLLM_LIST_CFGS"))
                    fprintf(stderr, "dllm candidate: C %d NT %d SUB %d S %d nbuf %d smem %zu clusters %d cost %.3f\n", C, NT, L, S,
                            nbuf, smem, nact, cost);
                if (cost < best) {
                    best = cost;
                    bc.cluster = C;
                    bc.threads = NT;
                    bc.SUB = L;
                    bc.S = S;
                    bc.htab = htab;
                    bc.smem = smem;
                    bc.max_clusters = nact;
                    bc.nbuf = nbuf;
                }
            }
        }
    }
    if (best >= 1e299) return lat_c ? choose_config(vocab, dtype, hist_bound, topk_bound, false, cfg)
                                    : DLLM_ERR_UNSUPPORTED;
    if (getenv("DLLM_VERBOSE"))
        fprintf(stderr, "dllm config: vocab %d dtype %d -> cluster %d threads %d SUB %d S %d htab %d smem %zu clusters %d nbuf %d\n",
                vocab, dtype, bc.cluster, bc.threads, bc.SUB, bc.S, bc.htab, bc.smem, bc.max_clusters, bc.nbuf);
    *cfg = bc;
    return DLLM_OK;
}

static cudaEvent_t g_ev_before = nullptr, g_ev_after = nullptr;  // optional cluster-kernel timing

dllm_status set_timing_events(cudaEvent_t before, cudaEvent_t after) {
    g_ev_before = before;
    g_ev_after = after;
    return DLLM_OK;
}

dllm_status set_debug_counters(unsigned long long *dev_counters) {
    g_host_dbg = dev_counters;
    return DLLM_OK;
}
unsigned long long *debug_counters() { return g_host_dbg; }

dllm_status launch_sample(const KernelArgs &a, const LaunchCfg &cfg, cudaStream_t stream) {
    if (a.rows == 0) return DLLM_OK;
    KernelFn fn = kernel_for(a.dtype, cfg.SUB);
    KernelFn fnb = kernel_for(a.dtype, cfg.SUB, 1);
    // every row on the index-order path (broadcast parameters: temperature > 0, top-k off, no
    // min-p): the variant without the other paths' code
    const dllm_sampler_params &bp = a.bparams;
    const bool idx_only = !a.rparams && a.dtype == DLLM_DTYPE_F32 && bp.temperature > 0.0f &&
                          !(bp.top_k > 0 && bp.top_k < a.vocab_total) && !(bp.min_p > 0.0f) && !no_idx_variant();
    if (idx_only) {
        KernelFn fi = kernel_for(a.dtype, cfg.SUB, 2);
        if (fi) fn = fi;
    }
    if (!fn || !fnb) return DLLM_ERR_UNSUPPORTED;
    cudaError_t e = set_attrs(fn, cfg.smem);
    if (e != cudaSuccess) return DLLM_ERR_CUDA;
    const int ncl = a.rows < cfg.max_clusters ? a.rows : cfg.max_clusters;
    cudaLaunchConfig_t lc = {};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = cfg.cluster;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    lc.gridDim = dim3(ncl * cfg.cluster);
    lc.blockDim = dim3(cfg.threads);
    lc.dynamicSmemBytes = cfg.smem;
    lc.stream = stream;
    lc.attrs = at;
    lc.numAttrs = 1;
    KernelArgs args = a;
    args.dbg = g_host_dbg;
    args.dbg_rank = g_host_dbg ? dbg_rank_env() : 0;
    args.fault_site = g_fault_site;
    args.wait_limit = g_fault_limit;
    if (g_ev_before) cudaEventRecord(g_ev_before, stream);
    e = cudaLaunchKernelEx(&lc, fn, args);
    if (e != cudaSuccess) return DLLM_ERR_CUDA;
    if (g_ev_after) cudaEventRecord(g_ev_after, stream);
    // the walk kernel: one warp per row, after the cluster kernel on the same stream
    const int wb = (a.rows + WALK_WARPS - 1) / WALK_WARPS;
    const size_t wsmem = (size_t)WALK_WARPS * walk_smem_per_warp(a.nrec);
    e = set_attrs(fnb, wsmem, false);
    if (e != cudaSuccess) return DLLM_ERR_CUDA;
    fnb<<<wb, WALK_WARPS * 32, wsmem, stream>>>(args);
    e = cudaGetLastError();
    return e == cudaSuccess ? DLLM_OK : DLLM_ERR_CUDA;
}

}  // namespace dllm
