// dllm_internal.h -- launch arguments shared by the sampler kernels and their host launchers.
// Not part of the public C ABI (that is include/diskllm_cuda.h).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "diskllm_cuda.h"

namespace dllm {

// Per-row status bits written to dllm_batch_desc::status (0 = OK).
enum : int32_t {
    ROW_ERR_HIST_TABLE = 1,   // more distinct in-slice history ids than the table holds
    ROW_ERR_NONFINITE  = 2,   // a NaN among a top-k row's candidates (order undefined in the reference)
    ROW_ERR_TOPK_LARGE = 4,   // top_k above the list capacity (fused kernel: the large-k pass takes the row over)
    ROW_ERR_WALK       = 8,   // internal consistency check of the draw walk failed
    ROW_ERR_TIMEOUT    = 16,  // a bounded wait on a bulk copy expired
    ROW_TOPP_EDGE      = 32,  // information, not an error: see DLLM_ROW_TOPP_EDGE
};

// Largest top-k list the fused kernel handles.
constexpr int KMAX = 1024;

struct KernelArgs {
    const void     *logits;
    int64_t         row_stride;     // elements between rows of logits
    int             dtype;          // DLLM_DTYPE_F32 / DLLM_DTYPE_BF16
    int             vec_ok;         // 16-byte vector loads legal for every row
    const uint32_t *mask;
    int64_t         mask_stride;    // uint32 words between rows of mask
    const int32_t  *hist_ids;
    const int64_t  *hist_off;
    const float    *uniforms;
    dllm_sampler_params bparams;    // broadcast params
    const dllm_sampler_params *rparams; // per-row params (device) or null
    int             rows;
    int             vocab;          // ids in this logits slice
    int             vocab_total;    // full vocabulary (history ids are checked against it)
    int             vocab_offset;   // global id of local index 0
    int             S;              // slice length per CTA (= 4 * NT * SUB)
    int             SUB;            // elements per thread sub-chunk (SUB % 8 == 4)
    int             htab;           // history hash-table entries (power of 2)
    int             uni_bytes;      // bytes of the shared area after the slice buffers
    int             nbuf;           // slice buffers per CTA: 2 = next row's copy overlaps this row
    int             cluster;        // CTAs per row (cluster size)
    unsigned        flags;
    int32_t        *token;
    float          *probs;          // dense [rows][vocab] final probabilities or null
    int64_t         probs_stride;
    float          *pen_out;        // dense [rows][vocab] penalised logits or null
    int64_t         pen_stride;
    int32_t        *status;         // [rows] or null
    int32_t        *topk_ids;       // [rows][topk_stride] or null
    int64_t         topk_stride;
    unsigned long long *dbg;        // diagnostic counters or null
    unsigned char  *ws;             // workspace (row headers, warp records, stash)
    int             nrec;           // warp records per row (4 * warps * cluster)
    int             dbg_rank;       // cluster rank whose phases the diagnostic counters time
    long long       wait_limit;     // polls before a bounded wait on an mbarrier gives up
    int             fault_site;     // test hook: FAULT_* wait made to run out, 0 = none
};

// Bounded waits: polls of an mbarrier before the wait gives up and the row is marked
// ROW_ERR_TIMEOUT (about a second on B200).
constexpr long long WAIT_LIMIT = 1ll << 26;
// Test hook sites (dllm_cuda_debug_inject_wait_timeout): the cluster kernel adds one wait that
// nothing completes, on the cluster's first row, with no copy or store in flight to it.
enum : int {
    FAULT_NONE = 0,
    FAULT_COPY_WAIT = 1,      // CTA 0, after its slice's bulk copy landed
    FAULT_EXCHANGE_WAIT = 2,  // the last CTA, after exchange #1 completed
};

// Launch configuration chosen by the host for one (vocab, dtype, history bound, top-k bound).
struct LaunchCfg {
    int cluster;     // C
    int threads;     // NT
    int SUB;
    int S;
    int htab;
    size_t smem;     // dynamic shared memory bytes
    int max_clusters;// co-resident clusters on the device
    int nbuf;        // slice buffers per CTA (1 or 2)
};

// Workspace layout per row: RowHdr, nrec warp records, STASH_SLOTS stash slots.
constexpr int STASH_SLOTS = 32;
constexpr int STASH_STRIDE = 64;   // floats per stash slot: [0] = first index (as int), then SUB values
constexpr int MAX_SUB = 60;
constexpr int WIDE_SLOTS = 4;              // warp ranges (32 sub-chunks) kept whole for the walk
// floats per wide slot: one warp range, 32 sub-chunks of `sub` elements
__host__ __device__ inline int wide_stride(int sub) { return 32 * sub; }
// RowHdr (128 B) + nrec 24-byte warp records (rounded to 128 B) + the stash + the wide slots
__host__ __device__ inline size_t row_ws_bytes(int nrec, int sub) {
    return 128 + (((size_t)nrec * 24 + 127) & ~(size_t)127) + (size_t)STASH_SLOTS * STASH_STRIDE * 4 +
           (size_t)WIDE_SLOTS * wide_stride(sub) * 4;
}

// shared memory of one walk-kernel warp: its row's warp records and stash, copied in at the start
__host__ __device__ inline size_t walk_smem_per_warp(int nrec) {
    return (((size_t)nrec * 24 + 127) & ~(size_t)127) + (size_t)STASH_SLOTS * STASH_STRIDE * 4;
}

// latency: a batch of a few rows (decode of one or several sequences), where one row's latency
// matters, not the throughput of many co-resident rows
dllm_status choose_config(int vocab, int dtype, int hist_bound, int topk_bound, bool latency, LaunchCfg *cfg);
constexpr int LATENCY_ROWS = 4;  // batches of at most this many rows use the latency configuration
dllm_status set_debug_counters(unsigned long long *dev_counters);
unsigned long long *debug_counters();  // the device array set by set_debug_counters, or null
dllm_status set_timing_events(cudaEvent_t before, cudaEvent_t after);
dllm_status set_fault_injection(int site, long long polls);
size_t shard_part_bytes(int rows, int vlocal, int k);
size_t sorted_ws_bytes(int rows, int vocab);
size_t largek_ws_bytes(int rows, int vocab);
dllm_status launch_largek(const dllm_batch_desc *d, bool after_fused, void *ws, cudaStream_t stream);
dllm_status launch_sorted(const dllm_batch_desc *d, bool after_fused, void *ws, cudaStream_t stream);
int lmh_max_rows(int hidden);
dllm_status launch_lmhead(int rows, int hidden, int vocab, const float *h, const float *norm_w, float eps, int add_one,
                          const void *w, int w_dtype, float softcap, float *logits, float *scratch,
                          cudaStream_t stream);
// Peer exchange of vocabulary-sharded candidates (see dllm_cuda_peer_exchange_create).
struct PeerArgs {
    void *const *peers;         // device array [world] of every rank's exchange buffer, mapped here
    int rank, world;
    unsigned long long epoch;   // step number, from 1
};
size_t peer_exchange_bytes(int rows, int k, int world);
dllm_status launch_shard_candidates(const dllm_batch_desc *d, int64_t voff, int64_t vtotal, int k, float *cand_val,
                                    int32_t *cand_id, void *part, cudaStream_t stream, const PeerArgs *px = nullptr);
dllm_status launch_merge_sample_peer(int rows, int world, int k, const void *local_buf, unsigned long long epoch,
                                     const dllm_sampler_params *params, const dllm_sampler_params *row_params,
                                     const float *uniforms, int32_t *token, int32_t *status, long long wait_ns,
                                     cudaStream_t stream);
dllm_status launch_merge_sample(int rows, int nsh, int k, const float *vals, const int32_t *ids,
                                const dllm_sampler_params *params, const dllm_sampler_params *row_params,
                                const float *uniforms, int32_t *token, int32_t *status, cudaStream_t stream,
                                const unsigned long long *arrive = nullptr, unsigned long long target = 0,
                                long long wait_ns = 0);
dllm_status launch_sample(const KernelArgs &a, const LaunchCfg &cfg, cudaStream_t stream);
int nrec_for(const LaunchCfg &cfg);

}  // namespace dllm
