// dllm_capi.cu -- the C ABI of libdiskllm_cuda.so (include/diskllm_cuda.h, include/sampler.h).
//
// dllm_cuda_sample_batch validates a descriptor, picks (and caches) a launch configuration
// for the row length and starts the fused sampler kernel.  The sampler.h drop-ins keep the
// reference's host-pointer contract: they copy the row to the device, run the same kernels
// and copy results back.  None of them computes on the host.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <new>
#include <vector>

#include "dllm_internal.h"
#include "sampler.h"

using namespace dllm;

static thread_local char g_last_error[256] = "";

static void set_error(const char *what, cudaError_t e) {
    snprintf(g_last_error, sizeof g_last_error, "%s: %s", what, cudaGetErrorString(e));
}

extern "C" const char *dllm_cuda_last_error(void) { return g_last_error; }

namespace dllm {
void set_last_error_message(const char *msg) { snprintf(g_last_error, sizeof g_last_error, "%s", msg); }
}  // namespace dllm

extern "C" dllm_status dllm_cuda_set_timing_events(void *before, void *after) {
    return set_timing_events((cudaEvent_t)before, (cudaEvent_t)after);
}
extern "C" dllm_status dllm_cuda_set_debug_counters(unsigned long long *device_counters) {
    return set_debug_counters(device_counters);
}
extern "C" dllm_status dllm_cuda_debug_inject_wait_timeout(int site, long long polls) {
    return set_fault_injection(site, polls);
}

extern "C" const char *dllm_cuda_version(void) { return "diskllm_cuda 0.1.0 sm_100a"; }

// ----------------------------------------------------------------------------------------
// launch configuration cache

namespace {
struct CfgKey {
    int dev, vocab, dtype, hist_bound, topk_cap;
    bool latency;
    bool operator==(const CfgKey &o) const {
        return dev == o.dev && vocab == o.vocab && dtype == o.dtype && hist_bound == o.hist_bound &&
               topk_cap == o.topk_cap && latency == o.latency;
    }
};
std::mutex g_cfg_mu;
std::vector<std::pair<CfgKey, LaunchCfg>> g_cfgs;

int bucket(int x) {
    if (x <= 0) return 0;
    int p = 16;
    while (p < x) p <<= 1;
    return p;
}
}  // namespace

static dllm_status get_config(int rows, int vocab, int dtype, int hist_max, int topk_max, LaunchCfg *out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        set_error("cudaGetDevice", e);
        return DLLM_ERR_CUDA;
    }
    CfgKey key{dev, vocab, dtype, bucket(hist_max), topk_max > 0 ? bucket(topk_max) : 0, rows <= LATENCY_ROWS};
    std::lock_guard<std::mutex> lk(g_cfg_mu);
    for (auto &kv : g_cfgs)
        if (kv.first == key) {
            *out = kv.second;
            return DLLM_OK;
        }
    LaunchCfg c;
    dllm_status st = choose_config(vocab, dtype, key.hist_bound, key.topk_cap, key.latency, &c);
    if (st != DLLM_OK) return st;
    g_cfgs.push_back({key, c});
    *out = c;
    return DLLM_OK;
}

// ----------------------------------------------------------------------------------------
// library-managed workspace: one grow-only buffer per (device, stream)

namespace {
struct WsEntry {
    int dev;
    void *stream;
    void *ptr;
    size_t bytes;
};
std::mutex g_ws_mu;
std::vector<WsEntry> g_ws;
}  // namespace

// Test hook: this many of the next library allocations fail as if cudaMalloc had run out of
// memory (dllm_cuda_debug_fail_allocations).
static std::atomic<int> g_fail_allocs{0};

static cudaError_t lib_malloc(void **p, size_t bytes) {
    int n = g_fail_allocs.load();
    while (n > 0)
        if (g_fail_allocs.compare_exchange_weak(n, n - 1)) return cudaErrorMemoryAllocation;
    return cudaMalloc(p, bytes);
}

extern "C" dllm_status dllm_cuda_debug_fail_allocations(int count) {
    if (count < 0) return DLLM_ERR_INVALID_ARG;
    g_fail_allocs.store(count);
    return DLLM_OK;
}

static void *internal_workspace(void *stream, size_t bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lk(g_ws_mu);
    for (auto &w : g_ws) {
        if (w.dev != dev || w.stream != stream) continue;
        if (w.bytes >= bytes) return w.ptr;
        cudaFree(w.ptr);  // waits for kernels still using the old buffer
        w.ptr = nullptr;
        w.bytes = 0;
        if (lib_malloc(&w.ptr, bytes) != cudaSuccess) {
            w.ptr = nullptr;
            return nullptr;
        }
        w.bytes = bytes;
        return w.ptr;
    }
    void *p = nullptr;
    if (lib_malloc(&p, bytes) != cudaSuccess) return nullptr;
    g_ws.push_back({dev, stream, p, bytes});
    return p;
}

// ----------------------------------------------------------------------------------------
// batched entry point

static dllm_status validate(const dllm_batch_desc *d) {
    if (!d) return DLLM_ERR_INVALID_ARG;
    if (d->rows < 0 || d->vocab <= 0 || !d->logits || !d->uniforms || !d->token) return DLLM_ERR_INVALID_ARG;
    if (d->row_stride < d->vocab) return DLLM_ERR_INVALID_ARG;
    if (d->dtype != DLLM_DTYPE_F32 && d->dtype != DLLM_DTYPE_BF16) return DLLM_ERR_INVALID_ARG;
    if (d->mask && d->mask_stride < (d->vocab + 31) / 32) return DLLM_ERR_INVALID_ARG;
    if ((d->hist_ids == nullptr) != (d->hist_off == nullptr)) return DLLM_ERR_INVALID_ARG;
    if (d->hist_ids && d->hist_max < 0) return DLLM_ERR_INVALID_ARG;
    if (d->probs && d->probs_stride < d->vocab) return DLLM_ERR_INVALID_ARG;
    if (d->pen_logits && d->pen_stride < d->vocab) return DLLM_ERR_INVALID_ARG;
    if (d->topk_ids && d->topk_stride < (d->row_params ? d->topk_max : d->params.top_k))
        return DLLM_ERR_INVALID_ARG;
    if (d->flags & ~(unsigned)(DLLM_MODE_PEN_TRUE_DIV | DLLM_MODE_TOPP_SORTED | DLLM_MODE_MINP_RELATIVE))
        return DLLM_ERR_UNSUPPORTED;
    if ((d->flags & DLLM_MODE_TOPP_SORTED) && d->vocab > (1 << 21)) return DLLM_ERR_UNSUPPORTED;
    if (d->workspace && ((uintptr_t)d->workspace % 256 != 0)) return DLLM_ERR_INVALID_ARG;
    return DLLM_OK;
}

// ----------------------------------------------------------------------------------------
// decode-loop glue: append each row's sampled token to its device-resident history

// One sequence's history is hist_ids[hist_off[0], hist_off[1]) with room for `cap` ids from
// hist_off[0]; the sampled token is appended (when full, the window slides: the oldest id goes),
// so a decode loop can run step after step -- sample, append -- with no host round trip, and can
// be captured once as a CUDA graph.
__global__ void append_history_kernel(const int32_t *token, int32_t *hist_ids, int64_t *hist_off, int64_t cap) {
    if (threadIdx.x != 0) return;
    const int64_t start = hist_off[0], end = hist_off[1];
    if (end - start < cap) {
        hist_ids[end] = token[0];
        hist_off[1] = end + 1;
        return;
    }
    for (int64_t j = start; j + 1 < end; j++) hist_ids[j] = hist_ids[j + 1];
    hist_ids[end - 1] = token[0];
}

extern "C" dllm_status dllm_cuda_append_history(const int32_t *token, int32_t *hist_ids, int64_t *hist_off,
                                                int64_t cap, void *stream) {
    if (!token || !hist_ids || !hist_off || cap <= 0) return DLLM_ERR_INVALID_ARG;
    append_history_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(token, hist_ids, hist_off, cap);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error("history append kernel launch", e);
        return DLLM_ERR_CUDA;
    }
    return DLLM_OK;
}

// ----------------------------------------------------------------------------------------
// LM-head tail: final norm, logits matvec, softcap (no sampling)

extern "C" dllm_status dllm_cuda_lmhead_logits(int rows, int hidden, int vocab, const float *h, const float *norm_w,
                                               float eps, int add_one, const void *w, int w_dtype, float softcap,
                                               float *logits, void *stream) {
    if (rows < 0 || hidden < 8 || hidden % 8 != 0 || vocab < 1) return DLLM_ERR_INVALID_ARG;
    if (rows > 0 && (!h || !w || !logits)) return DLLM_ERR_INVALID_ARG;
    if ((uintptr_t)w % 16 != 0) return DLLM_ERR_INVALID_ARG;
    if (w_dtype != DLLM_DTYPE_F32 && w_dtype != DLLM_DTYPE_BF16 && w_dtype != DLLM_DTYPE_F16)
        return DLLM_ERR_INVALID_ARG;
    if (lmh_max_rows(hidden) < 1) return DLLM_ERR_UNSUPPORTED;
    if (rows == 0) return DLLM_OK;
    float *scratch = (float *)internal_workspace(stream, (size_t)rows * hidden * sizeof(float));
    if (!scratch) {
        set_error("lm-head scratch", cudaErrorMemoryAllocation);
        return DLLM_ERR_OOM;
    }
    const dllm_status st = launch_lmhead(rows, hidden, vocab, h, norm_w, eps, add_one, w, w_dtype, softcap, logits,
                                         scratch, (cudaStream_t)stream);
    if (st == DLLM_ERR_CUDA) set_error("lm-head kernel launch", cudaGetLastError());
    return st;
}

// ----------------------------------------------------------------------------------------
// vocabulary-sharded sampling (no counterpart in the reference, whose sampler sees whole rows)

extern "C" dllm_status dllm_cuda_shard_candidates(const dllm_batch_desc *d, int64_t vocab_offset, int64_t vocab_total,
                                                  int k, float *cand_val, int32_t *cand_id, void *stream) {
    if (!d || d->rows < 0 || d->vocab <= 0 || (d->rows > 0 && !d->logits)) return DLLM_ERR_INVALID_ARG;
    if (d->row_stride < d->vocab) return DLLM_ERR_INVALID_ARG;
    if (d->dtype != DLLM_DTYPE_F32 && d->dtype != DLLM_DTYPE_BF16) return DLLM_ERR_INVALID_ARG;
    if (d->mask && d->mask_stride < (d->vocab + 31) / 32) return DLLM_ERR_INVALID_ARG;
    if ((d->hist_ids == nullptr) != (d->hist_off == nullptr)) return DLLM_ERR_INVALID_ARG;
    if (vocab_offset < 0 || vocab_total <= 0 || vocab_offset + d->vocab > vocab_total) return DLLM_ERR_INVALID_ARG;
    if (!cand_val || !cand_id || k < 1) return DLLM_ERR_INVALID_ARG;
    if (d->flags & ~(unsigned)DLLM_MODE_PEN_TRUE_DIV) return DLLM_ERR_UNSUPPORTED;
    // per-chunk candidates of rows wider than one chunk: the grow-only internal buffer
    const size_t pb = shard_part_bytes(d->rows, d->vocab, k);
    void *part = pb ? internal_workspace(stream, pb) : nullptr;
    if (pb && !part) {
        set_error("shard candidate scratch", cudaErrorMemoryAllocation);
        return DLLM_ERR_OOM;
    }
    const dllm_status st = launch_shard_candidates(d, vocab_offset, vocab_total, k, cand_val, cand_id, part,
                                                   (cudaStream_t)stream);
    if (st == DLLM_ERR_CUDA) set_error("shard candidate kernel launch", cudaGetLastError());
    return st;
}

extern "C" dllm_status dllm_cuda_merge_sample(int rows, int nshards, int k, const float *cand_val,
                                              const int32_t *cand_id, const dllm_sampler_params *params,
                                              const dllm_sampler_params *row_params, const float *uniforms,
                                              int32_t *token, int32_t *status, void *stream) {
    if (rows < 0 || nshards < 1 || k < 1 || !params) return DLLM_ERR_INVALID_ARG;
    if (rows > 0 && (!cand_val || !cand_id || !uniforms || !token)) return DLLM_ERR_INVALID_ARG;
    if (!row_params && params->temperature != 0.0f && (params->top_k < 1 || params->top_k > k))
        return DLLM_ERR_UNSUPPORTED;
    const dllm_status st = launch_merge_sample(rows, nshards, k, cand_val, cand_id, params, row_params, uniforms,
                                               token, status, (cudaStream_t)stream);
    if (st == DLLM_ERR_CUDA) set_error("merge kernel launch", cudaGetLastError());
    return st;
}

// ----------------------------------------------------------------------------------------
// peer exchange of vocabulary-sharded candidates (NVLink stores instead of a collective)

extern "C" dllm_status dllm_cuda_peer_exchange_create(int rows, int k, int world, void **buf, void *ipc_handle) {
    if (!buf || !ipc_handle) return DLLM_ERR_INVALID_ARG;
    const size_t bytes = peer_exchange_bytes(rows, k, world);
    if (!bytes) return DLLM_ERR_INVALID_ARG;
    *buf = nullptr;
    cudaError_t e = lib_malloc(buf, bytes);
    if (e != cudaSuccess) {
        set_error("peer exchange buffer", e);
        *buf = nullptr;
        return DLLM_ERR_OOM;
    }
    e = cudaMemset(*buf, 0, bytes);  // arrival counters start at zero
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t *>(ipc_handle), *buf);
    if (e != cudaSuccess) {
        set_error("peer exchange buffer set-up", e);
        cudaFree(*buf);
        *buf = nullptr;
        return DLLM_ERR_CUDA;
    }
    return DLLM_OK;
}

extern "C" dllm_status dllm_cuda_peer_exchange_open(const void *ipc_handle, void **peer_buf) {
    if (!ipc_handle || !peer_buf) return DLLM_ERR_INVALID_ARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof h);
    const cudaError_t e = cudaIpcOpenMemHandle(peer_buf, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        set_error("cudaIpcOpenMemHandle", e);
        return DLLM_ERR_CUDA;
    }
    return DLLM_OK;
}

extern "C" dllm_status dllm_cuda_peer_exchange_close(void *peer_buf) {
    if (!peer_buf) return DLLM_ERR_INVALID_ARG;
    return cudaIpcCloseMemHandle(peer_buf) == cudaSuccess ? DLLM_OK : DLLM_ERR_CUDA;
}

extern "C" dllm_status dllm_cuda_peer_exchange_free(void *buf) {
    if (!buf) return DLLM_ERR_INVALID_ARG;
    return cudaFree(buf) == cudaSuccess ? DLLM_OK : DLLM_ERR_CUDA;
}

extern "C" dllm_status dllm_cuda_shard_candidates_peer(const dllm_batch_desc *d, int64_t vocab_offset,
                                                       int64_t vocab_total, int k, void *const *peer_bufs, int rank,
                                                       int world, uint64_t epoch, void *stream) {
    if (!d || d->rows < 0 || d->vocab <= 0 || (d->rows > 0 && !d->logits)) return DLLM_ERR_INVALID_ARG;
    if (d->row_stride < d->vocab) return DLLM_ERR_INVALID_ARG;
    if (d->dtype != DLLM_DTYPE_F32 && d->dtype != DLLM_DTYPE_BF16) return DLLM_ERR_INVALID_ARG;
    if (d->mask && d->mask_stride < (d->vocab + 31) / 32) return DLLM_ERR_INVALID_ARG;
    if ((d->hist_ids == nullptr) != (d->hist_off == nullptr)) return DLLM_ERR_INVALID_ARG;
    if (vocab_offset < 0 || vocab_total <= 0 || vocab_offset + d->vocab > vocab_total) return DLLM_ERR_INVALID_ARG;
    if (!peer_bufs || world < 1 || rank < 0 || rank >= world || epoch < 1 || k < 1) return DLLM_ERR_INVALID_ARG;
    if (!peer_exchange_bytes(d->rows > 0 ? d->rows : 1, k, world)) return DLLM_ERR_INVALID_ARG;
    if (d->flags & ~(unsigned)DLLM_MODE_PEN_TRUE_DIV) return DLLM_ERR_UNSUPPORTED;
    PeerArgs px{peer_bufs, rank, world, (unsigned long long)epoch};
    const dllm_status st = launch_shard_candidates(d, vocab_offset, vocab_total, k, nullptr, nullptr, nullptr,
                                                   (cudaStream_t)stream, &px);
    if (st == DLLM_ERR_CUDA) set_error("shard candidate kernel launch (peer exchange)", cudaGetLastError());
    return st;
}

extern "C" dllm_status dllm_cuda_merge_sample_peer(int rows, int world, int k, const void *local_buf, uint64_t epoch,
                                                   const dllm_sampler_params *params,
                                                   const dllm_sampler_params *row_params, const float *uniforms,
                                                   int32_t *token, int32_t *status, void *stream) {
    if (rows < 0 || world < 1 || k < 1 || !params || !local_buf || epoch < 1) return DLLM_ERR_INVALID_ARG;
    if (!peer_exchange_bytes(rows > 0 ? rows : 1, k, world)) return DLLM_ERR_INVALID_ARG;
    if (rows > 0 && (!uniforms || !token)) return DLLM_ERR_INVALID_ARG;
    if (!row_params && params->temperature != 0.0f && (params->top_k < 1 || params->top_k > k))
        return DLLM_ERR_UNSUPPORTED;
    const long long wait_ns = 2000000000ll;  // a rank that has not arrived after 2 s times the rows out
    const dllm_status st = launch_merge_sample_peer(rows, world, k, local_buf, (unsigned long long)epoch, params,
                                                    row_params, uniforms, token, status, wait_ns,
                                                    (cudaStream_t)stream);
    if (st == DLLM_ERR_CUDA) set_error("merge kernel launch (peer exchange)", cudaGetLastError());
    return st;
}

static int topk_bound(const dllm_batch_desc *d) {
    int topk_max = d->row_params ? d->topk_max : d->params.top_k;
    if (topk_max >= d->vocab || topk_max < 0) topk_max = 0;
    if (!d->row_params && d->params.temperature == 0.0f) topk_max = 0;  // greedy ignores top-k
    return topk_max;
}

// Which kernels a descriptor runs: the fused sampler, the sorted-nucleus passes, the large-k pass,
// or a combination.  Per-row parameters under the sorted flag: the fused kernel samples every
// row, then the sorted passes resample the rows with top-k off and temperature > 0.  Top-k above
// the fused kernel's list capacity (KMAX): the large-k pass samples those rows (all of them for
// broadcast parameters; after the fused kernel, the rows whose own top_k exceeds KMAX, for
// per-row parameters).
struct Plan {
    bool fused, sorted, large;
    int fused_topk;  // top-k bound the fused kernel is configured for
};

static Plan plan(const dllm_batch_desc *d) {
    Plan pl;
    pl.sorted = (d->flags & DLLM_MODE_TOPP_SORTED) != 0;
    pl.fused = true;
    if (pl.sorted && !d->row_params) {
        const dllm_sampler_params &p = d->params;
        const bool eligible = p.temperature > 0.0f && !(p.top_k > 0 && p.top_k < d->vocab);
        pl.fused = !eligible;
        pl.sorted = eligible;
    }
    const int tk = topk_bound(d);
    pl.large = tk > KMAX;
    if (pl.large && !d->row_params) pl.fused = false;
    pl.fused_topk = tk > KMAX ? KMAX : tk;
    return pl;
}

static size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

// Workspace layout: [fused kernel rows][sorted-nucleus passes][large-k pass], each 256-aligned.
struct WsLayout {
    size_t fused, sorted_off, large_off, total;
};

static dllm_status ws_layout(const dllm_batch_desc *d, const Plan &pl, LaunchCfg *cfg, WsLayout *out) {
    WsLayout L = {};
    if (pl.fused) {
        const dllm_status st = get_config(d->rows, d->vocab, d->dtype, d->hist_ids ? d->hist_max : 0, pl.fused_topk, cfg);
        if (st != DLLM_OK) return st;
        L.fused = (size_t)d->rows * row_ws_bytes(nrec_for(*cfg), cfg->SUB);
    }
    L.sorted_off = al256(L.fused);
    L.large_off = al256(L.sorted_off + (pl.sorted ? sorted_ws_bytes(d->rows, d->vocab) : 0));
    L.total = L.large_off + (pl.large ? largek_ws_bytes(d->rows, d->vocab) : 0);
    *out = L;
    return DLLM_OK;
}

extern "C" size_t dllm_cuda_workspace_bytes(const dllm_batch_desc *d) {
    if (validate(d) != DLLM_OK || d->rows == 0) return 0;
    const Plan pl = plan(d);
    LaunchCfg cfg;
    WsLayout L;
    if (ws_layout(d, pl, &cfg, &L) != DLLM_OK) return 0;
    return L.total;
}

extern "C" dllm_status dllm_cuda_sample_batch(const dllm_batch_desc *d, void *stream) {
    dllm_status st = validate(d);
    if (st != DLLM_OK) return st;
    if (d->rows == 0) return DLLM_OK;
    const Plan pl = plan(d);
    const bool fused = pl.fused, sorted = pl.sorted;

    LaunchCfg cfg = {};
    WsLayout L;
    st = ws_layout(d, pl, &cfg, &L);
    if (st != DLLM_OK) return st;
    const int nrec = fused ? nrec_for(cfg) : 0;
    const size_t ws_need = L.total;
    void *ws = d->workspace;
    if (ws) {
        if (d->workspace_bytes < ws_need) return DLLM_ERR_INVALID_ARG;
    } else {
        ws = internal_workspace(stream, ws_need);
        if (!ws) {
            set_error("workspace allocation", cudaErrorMemoryAllocation);
            return DLLM_ERR_OOM;
        }
    }

    KernelArgs a = {};
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
    a.vocab_total = d->vocab;
    a.vocab_offset = 0;
    a.S = cfg.S;
    a.SUB = cfg.SUB;
    a.ws = (unsigned char *)ws;
    a.nrec = nrec;
    a.htab = cfg.htab;
    a.nbuf = cfg.nbuf;
    a.uni_bytes = (int)(cfg.smem - (size_t)cfg.nbuf * (cfg.S + cfg.SUB) * 4);
    a.cluster = cfg.cluster;
    a.flags = d->flags;
    a.token = d->token;
    a.probs = d->probs;
    a.probs_stride = d->probs_stride;
    a.pen_out = d->pen_logits;
    a.pen_stride = d->pen_stride;
    a.status = d->status;
    a.topk_ids = d->topk_ids;
    a.topk_stride = d->topk_stride;
    if (fused) {
        st = launch_sample(a, cfg, (cudaStream_t)stream);
        if (st != DLLM_OK) {
            set_error("sample kernel launch", cudaGetLastError());
            return st;
        }
    }
    if (sorted) {
        st = launch_sorted(d, fused, (unsigned char *)ws + L.sorted_off, (cudaStream_t)stream);
        if (st == DLLM_ERR_CUDA) set_error("sorted-nucleus kernel launch", cudaGetLastError());
        if (st != DLLM_OK) return st;
    }
    if (pl.large) {
        st = launch_largek(d, fused, (unsigned char *)ws + L.large_off, (cudaStream_t)stream);
        if (st == DLLM_ERR_CUDA) set_error("large top-k pass launch", cudaGetLastError());
    }
    return st;
}

// ----------------------------------------------------------------------------------------
// history penalty kernel for the host-pointer drop-ins (src/sampler.c:21-52).  Sparse: the host
// gathers the logits of the n history entries, the kernel computes each entry's penalised value
// (every occurrence of an id gets the same value: its logit after the penalty, applied once per
// id for presence and once per occurrence for repetition), and the host writes them back.  Only
// 8 bytes per history entry cross PCIe each way, not the row.

__global__ void penalty_kernel(const float *vals, float *out, const int *seen, int n, int vocab, float value,
                               int mode) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int id = seen[i];
        if (id < 0 || id >= vocab) continue;
        int count = 0;
        for (int j = 0; j < n; j++) count += seen[j] == id;
        float v = vals[i];
        if (mode == 0) {  // repetition, once per occurrence
            const float inv = __fdiv_rn(1.0f, value);
            for (int k = 0; k < count; k++) v = v < 0.0f ? __fmul_rn(v, value) : __fmul_rn(v, inv);
        } else {          // presence, once per id
            v = __fsub_rn(v, value);
        }
        out[i] = v;
    }
}

// ----------------------------------------------------------------------------------------
// drop-in sampler.h

struct DevBuf {
    int dev = -1;
    cudaStream_t stream = nullptr;
    float *row = nullptr;
    int cap = 0;
    int *ids = nullptr;
    int ids_cap = 0;
    float *u = nullptr;
    int32_t *tok = nullptr;
};

struct sampler {
    sampler_config cfg;
    uint64_t rng;
    DevBuf buf;
};

[[noreturn]] static void die(const char *what, cudaError_t e) {
    fprintf(stderr, "libdiskllm_cuda: %s failed: %s\n", what, cudaGetErrorString(e));
    abort();
}
#define DLLM_CHECK(x)                          \
    do {                                       \
        cudaError_t _e = (x);                  \
        if (_e != cudaSuccess) die(#x, _e);    \
    } while (0)

static void buf_reserve(DevBuf &b, int vocab, int nids) {
    if (!b.stream) {
        DLLM_CHECK(cudaGetDevice(&b.dev));
        DLLM_CHECK(cudaStreamCreateWithFlags(&b.stream, cudaStreamNonBlocking));
        DLLM_CHECK(cudaMalloc(&b.u, sizeof(float)));
        DLLM_CHECK(cudaMalloc(&b.tok, sizeof(int32_t)));
    }
    if (vocab > b.cap) {
        if (b.row) DLLM_CHECK(cudaFree(b.row));
        DLLM_CHECK(cudaMalloc(&b.row, sizeof(float) * (size_t)vocab));
        b.cap = vocab;
    }
    if (nids > b.ids_cap) {
        if (b.ids) DLLM_CHECK(cudaFree(b.ids));
        DLLM_CHECK(cudaMalloc(&b.ids, sizeof(int) * (size_t)nids));
        b.ids_cap = nids;
    }
}

static void buf_release(DevBuf &b) {
    if (b.row) cudaFree(b.row);
    if (b.ids) cudaFree(b.ids);
    if (b.u) cudaFree(b.u);
    if (b.tok) cudaFree(b.tok);
    if (b.stream) cudaStreamDestroy(b.stream);
    b = DevBuf();
}

static thread_local DevBuf t_free_buf;  // for greedy_sample / penalties (no sampler object)

static int run_one_row(DevBuf &b, const float *host_logits, int vocab, const dllm_sampler_params &p, float r) {
    buf_reserve(b, vocab, 0);
    DLLM_CHECK(cudaMemcpyAsync(b.row, host_logits, sizeof(float) * (size_t)vocab, cudaMemcpyHostToDevice, b.stream));
    DLLM_CHECK(cudaMemcpyAsync(b.u, &r, sizeof(float), cudaMemcpyHostToDevice, b.stream));
    dllm_batch_desc d = {};
    d.rows = 1;
    d.vocab = vocab;
    d.row_stride = vocab;
    d.dtype = DLLM_DTYPE_F32;
    d.logits = b.row;
    d.uniforms = b.u;
    d.params = p;
    d.token = b.tok;
    dllm_status st = dllm_cuda_sample_batch(&d, b.stream);
    if (st != DLLM_OK) {
        fprintf(stderr, "libdiskllm_cuda: dllm_cuda_sample_batch failed (%d): %s\n", (int)st, g_last_error);
        abort();
    }
    int32_t tok = 0;
    DLLM_CHECK(cudaMemcpyAsync(&tok, b.tok, sizeof(int32_t), cudaMemcpyDeviceToHost, b.stream));
    DLLM_CHECK(cudaStreamSynchronize(b.stream));
    return tok;
}

extern "C" sampler *sampler_create(const sampler_config *cfg) {
    if (!cfg) return nullptr;
    sampler *s = (sampler *)calloc(1, sizeof(sampler));
    if (!s) return nullptr;
    new (&s->buf) DevBuf();
    s->cfg = *cfg;
    s->rng = cfg->seed ? cfg->seed : 0xDEADBEEF12345678ULL;
    return s;
}

extern "C" void sampler_free(sampler *s) {
    if (!s) return;
    buf_release(s->buf);
    free(s);
}

extern "C" uint64_t dllm_sampler_get_rng_state(const sampler *s) { return s ? s->rng : 0; }
extern "C" void dllm_sampler_set_rng_state(sampler *s, uint64_t st) {
    if (s) s->rng = st;
}

// xorshift64 and its uniform, src/sampler.c:69-81
static float next_uniform(uint64_t *state) {
    uint64_t x = *state;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    *state = x;
    return (float)(x >> 11) * (1.0f / (float)(1ULL << 53));
}

extern "C" int sampler_sample(sampler *s, float *logits, int vocab_size) {
    if (!s || !logits || vocab_size <= 0) return 0;
    dllm_sampler_params p = {};
    p.temperature = s->cfg.temperature;
    p.top_k = s->cfg.top_k;
    p.top_p = s->cfg.top_p;
    p.min_p = s->cfg.min_p;
    p.repetition = 1.0f;
    const float r = p.temperature == 0.0f ? 0.0f : next_uniform(&s->rng);
    return run_one_row(s->buf, logits, vocab_size, p, r);
}

extern "C" int greedy_sample(const float *logits, int vocab_size) {
    if (!logits || vocab_size <= 0) return 0;
    dllm_sampler_params p = {};
    p.temperature = 0.0f;
    p.top_p = 1.0f;
    p.repetition = 1.0f;
    return run_one_row(t_free_buf, logits, vocab_size, p, 0.0f);
}

static void apply_penalty(float *logits, int vocab, const int *seen, int n, float value, int mode) {
    DevBuf &b = t_free_buf;
    buf_reserve(b, 2 * n, n);
    std::vector<float> vals((size_t)n, 0.0f);
    for (int i = 0; i < n; i++)
        if (seen[i] >= 0 && seen[i] < vocab) vals[i] = logits[seen[i]];
    DLLM_CHECK(cudaMemcpyAsync(b.row, vals.data(), sizeof(float) * (size_t)n, cudaMemcpyHostToDevice, b.stream));
    DLLM_CHECK(cudaMemcpyAsync(b.ids, seen, sizeof(int) * (size_t)n, cudaMemcpyHostToDevice, b.stream));
    penalty_kernel<<<(n + 255) / 256, 256, 0, b.stream>>>(b.row, b.row + n, b.ids, n, vocab, value, mode);
    DLLM_CHECK(cudaGetLastError());
    DLLM_CHECK(cudaMemcpyAsync(vals.data(), b.row + n, sizeof(float) * (size_t)n, cudaMemcpyDeviceToHost, b.stream));
    DLLM_CHECK(cudaStreamSynchronize(b.stream));
    for (int i = 0; i < n; i++)
        if (seen[i] >= 0 && seen[i] < vocab) logits[seen[i]] = vals[i];
}

extern "C" void sampler_apply_repetition_penalty(float *logits, int vocab_size, const int *seen_tokens,
                                                 int num_seen, float penalty) {
    if (penalty <= 1.0f || !seen_tokens || num_seen <= 0 || !logits || vocab_size <= 0) return;
    apply_penalty(logits, vocab_size, seen_tokens, num_seen, penalty, 0);
}

extern "C" void sampler_apply_presence_penalty(float *logits, int vocab_size, const int *seen_tokens,
                                               int num_seen, float presence_penalty) {
    if (presence_penalty == 0.0f || !seen_tokens || num_seen <= 0 || !logits || vocab_size <= 0) return;
    apply_penalty(logits, vocab_size, seen_tokens, num_seen, presence_penalty, 1);
}
