/*
 * diskllm_cuda.h -- C ABI of libdiskllm_cuda.so, the B200 (sm_100a) sampler for DiskLLM.
 *
 * Two layers:
 *   1. Drop-in replacements for DiskLLM's sampler.h (include/sampler.h:7-34 in DiskLLM),
 *      declared in this repo's include/sampler.h with identical names and signatures.
 *      Linking libdiskllm_cuda.so instead of compiling src/sampler.c keeps
 *      src/core/sampler_api.c and every caller unchanged.
 *   2. A batched, device-resident entry point (dllm_cuda_sample_batch) that runs the whole
 *      per-row chain of src/core/sampler_api.c:48-63 -- grammar mask, presence,
 *      frequency, repetition, sampler_sample -- for many rows in one launch.
 *
 * Every pointer in dllm_batch_desc is a device pointer unless stated otherwise.  The
 * caller owns all buffers.  Streams are passed as void* (a cudaStream_t).
 */
#ifndef DISKLLM_CUDA_H
#define DISKLLM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifndef DLLM_API
#if defined(__GNUC__)
#define DLLM_API __attribute__((visibility("default")))
#else
#define DLLM_API
#endif
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    DLLM_OK = 0,
    DLLM_ERR_INVALID_ARG = 1,
    DLLM_ERR_OOM = 2,
    DLLM_ERR_CUDA = 3,
    DLLM_ERR_NCCL = 4,
    DLLM_ERR_TIMEOUT = 5,
    DLLM_ERR_UNSUPPORTED = 6,
} dllm_status;

enum {
    DLLM_DTYPE_F32 = 0,
    DLLM_DTYPE_BF16 = 1,
    DLLM_DTYPE_F16 = 2,   /* output weights of dllm_cuda_lmhead_logits only */
};

/* mode flags */
#define DLLM_MODE_TOPP_SORTED   0x1u  /* sorted-nucleus mode for rows with top-k off and
                                         temperature > 0: entries ordered by (t desc, id asc),
                                         masses rint(expf(t) * 2^42) summed exactly, min-p the
                                         sorted prefix above the threshold, top-p the shortest
                                         prefix reaching top_p of the kept mass, the draw the
                                         first entry whose prefix mass exceeds r * (nucleus
                                         mass).  Not the reference's behaviour (its top-p keeps
                                         an index-order prefix when top-k is off); vocab <= 2^21 */
#define DLLM_MODE_PEN_TRUE_DIV  0x2u  /* positive logits divided by the repetition penalty
                                         (IEEE) instead of multiplied by 1/penalty, which is
                                         what the reference's -ffast-math build computes */
#define DLLM_MODE_MINP_RELATIVE 0x4u  /* min-p keeps p >= min_p * (largest p) instead of the
                                         reference's absolute p >= min_p */

/* Sampling parameters of one row.  Fields mirror DiskLLM's sampler_config
 * (include/sampler.h:10-16) plus the penalties of diskllm_sampler_params
 * (include/diskllm.h:48-56) and the frequency extension. */
typedef struct {
    float temperature;   /* 0 -> greedy (src/sampler.c:140-142) */
    float top_p;         /* >= 1 -> off */
    float min_p;         /* <= 0 -> off; absolute threshold as in src/sampler.c:188-202 */
    int   top_k;         /* <= 0 or >= vocab -> off */
    float repetition;    /* <= 1 -> off (src/sampler.c:21-33, src/core/sampler_api.c:59) */
    float presence;      /* 0 -> off (src/sampler.c:35-52, src/core/sampler_api.c:55) */
    float frequency;     /* 0 -> off; not in the reference: x -= (float)count * frequency,
                            applied after presence, before repetition */
} dllm_sampler_params;

typedef struct {
    int rows;                 /* batch rows */
    int vocab;                /* columns of logits (= vocabulary) */
    int64_t row_stride;       /* elements between consecutive rows (>= vocab) */
    int dtype;                /* DLLM_DTYPE_F32 or DLLM_DTYPE_BF16 (upcast exactly) */
    const void *logits;       /* [rows][row_stride] */

    const uint32_t *mask;     /* grammar allow-mask or NULL: bit (i & 31) of word (i >> 5)
                                 set = token i allowed; cleared -> -INFINITY, the effect of
                                 diskllm_grammar_apply_mask (src/core/grammar.c:275-308) */
    int64_t mask_stride;      /* words between rows (>= (vocab + 31) / 32) */

    const int32_t *hist_ids;  /* token history, CSR; NULL = none */
    const int64_t *hist_off;  /* [rows + 1] offsets into hist_ids */
    int hist_max;             /* upper bound on any row's history length (host value) */

    const float *uniforms;    /* [rows] draws in [0, 1), one per row */

    dllm_sampler_params params;            /* host value, used for every row ... */
    const dllm_sampler_params *row_params; /* ... unless this device array is given */
    int topk_max;             /* upper bound on top_k over rows when row_params is given.
                                 Any top_k works (as in the reference, src/sampler.c:165-170);
                                 rows with top_k above 1024 take a slower sort-based pass */

    unsigned flags;           /* DLLM_MODE_* */

    int32_t *token;           /* [rows] out: sampled token id */
    float *probs;             /* optional [rows][probs_stride] out: final draw probability
                                 of every token (0 outside the draw list) */
    int64_t probs_stride;
    float *pen_logits;        /* optional [rows][pen_stride] out: logits after mask and
                                 penalties (what the reference leaves in its logits array) */
    int64_t pen_stride;
    int32_t *status;          /* optional [rows] out: 0 or DLLM_ROW_ERR_* bits */
    int32_t *topk_ids;        /* optional [rows][topk_stride] out: the top-k ids, best first
                                 (rows where top-k is active) */
    int64_t topk_stride;

    void *workspace;          /* optional device scratch of >= dllm_cuda_workspace_bytes()
                                 bytes (256-byte aligned); NULL: the library keeps one
                                 buffer per (device, stream) and grows it with cudaMalloc */
    size_t workspace_bytes;
} dllm_batch_desc;

/* per-row status bits */
#define DLLM_ROW_ERR_HIST_TABLE 1   /* more distinct history ids than the table holds */
#define DLLM_ROW_ERR_NONFINITE  2   /* a NaN among a top-k row's candidates: the reference's
                                       -ffast-math build leaves its order undefined.  (Rows with
                                       +inf, all-NaN rows and NaN rows with top-k off get the
                                       reference's id: its list's last entry) */
#define DLLM_ROW_ERR_TOPK_LARGE 4   /* a top_k dllm_cuda_merge_sample cannot serve (above its
                                       gathered k); whole-row calls serve every top_k */
#define DLLM_ROW_ERR_WALK       8   /* internal consistency check of the draw failed */
#define DLLM_ROW_ERR_TIMEOUT   16   /* a bounded wait on a bulk copy expired */
#define DLLM_ROW_TOPP_EDGE     32   /* information, not an error: the index-order top-p prefix
                                       at the cut, or just before it, lies within
                                       top_p * (one ulp of (float)(1/sum) + 6e-8) of the
                                       threshold.  The reference's exponentials (glibc's scalar
                                       and vector expf) differ from this library's by a few ulp,
                                       so its (float)(1/sum) can be one ulp away and, on such a
                                       row only, its cut one entry earlier or later
                                       (src/sampler.c:204-222); its probabilities and id follow
                                       that cut */

/* Samples every row of the batch on `stream` (stream-ordered; returns after the launch).
 * Replaces, per row, the sequence of src/core/sampler_api.c:48-63:
 *   diskllm_grammar_apply_mask -> sampler_apply_presence_penalty ->
 *   sampler_apply_repetition_penalty -> sampler_sample.
 * Row i draws with uniforms[i] where the reference draws rand_f32 (src/sampler.c:225). */
DLLM_API dllm_status dllm_cuda_sample_batch(const dllm_batch_desc *desc, void *stream);

/* Scratch the sampler needs for this descriptor: per-row headers, warp-level draw records and
 * stashed probabilities (the size depends on the vocabulary's launch configuration: about 30 KB
 * per row at vocab 256000), plus the sorted-nucleus passes' and the large-top-k pass's buffers
 * when the descriptor uses them.  0 on invalid descriptors. */
DLLM_API size_t dllm_cuda_workspace_bytes(const dllm_batch_desc *desc);

/* Allocation-free variant of dllm_cuda_sample_batch; it has no counterpart in the reference.
 * For callers that cannot call cudaMalloc -- an embedder whose device memory is all owned by
 * its own allocator, or a decode loop that must not stall on the device-wide synchronisation
 * of cudaMalloc/cudaFree.  Instead of a caller buffer or a library-grown one, it uses a
 * 16 MiB scratch array compiled into the library (held on every GPU that loads the library
 * until the process exits); desc->workspace is ignored.  Batches whose
 * dllm_cuda_workspace_bytes() exceeds 16 MiB (about 550 rows of vocab 256000) are rejected
 * with DLLM_ERR_UNSUPPORTED and a message in dllm_cuda_last_error().  The first call on a
 * device looks up the array's device address and picks the launch configuration, so make it
 * before any stream capture.  The address is kept for the life of the process: after a
 * cudaDeviceReset of a device this entry point must not be called on it again.  Every call shares the one array: calls whose work overlaps on the
 * GPU (other streams, other host threads) race and must be serialised by the caller.  The
 * kernels write every scratch field before reading it, so leftover contents from an earlier
 * call need no clearing. */
DLLM_API dllm_status dllm_cuda_sample_batch_static(const dllm_batch_desc *desc, void *stream);

/* Diagnostics: when given a device array of 32 zeroed unsigned 64-bit counters, the sampler
 * kernels accumulate per-phase cycle counts of each cluster's first CTA and draw-walk
 * statistics into it; NULL switches it off.  No effect on results. */
DLLM_API dllm_status dllm_cuda_set_debug_counters(unsigned long long *device_counters);

/* Test hooks for failure detection (no counterpart in the reference).  Both are off by default
 * and change nothing while off.
 *   dllm_cuda_debug_inject_wait_timeout(site, polls): from the next sampling launch on, the
 *     cluster kernel adds, on each cluster's first row, one bounded wait that nothing completes
 *     (site 1: CTA 0 waits for its slice barrier's next phase after the bulk copy landed; site 2:
 *     the last CTA waits for exchange #1's next phase after the exchange completed), giving up
 *     after `polls` polls instead of about a second.  No copy or store is in flight to the waited
 *     barrier, so the kernel goes on and the row's status gets DLLM_ROW_ERR_TIMEOUT.  Site 0
 *     switches it off.
 *   dllm_cuda_debug_fail_allocations(count): the next `count` device allocations the library
 *     makes for its own buffers fail as if cudaMalloc had run out of memory, so the calls that
 *     needed them return DLLM_ERR_OOM. */
DLLM_API dllm_status dllm_cuda_debug_inject_wait_timeout(int site, long long polls);
DLLM_API dllm_status dllm_cuda_debug_fail_allocations(int count);

/* Vocabulary-sharded sampling (a row's logits split over N GPUs, as a tensor-parallel LM head
 * leaves them).  No counterpart in the reference, whose sampler sees whole rows; together the
 * two calls and one all-gather give the tokens sampler_sample would (src/sampler.c:136-234)
 * for rows with 0 < top_k <= k.
 *
 * Step 1, on each GPU: `desc` describes this GPU's columns [vocab_offset, vocab_offset +
 * desc->vocab) of vocab_total-wide rows (logits, mask words of those columns, history as global
 * ids, params; uniforms and token are not used).  Writes the k best entries of each row after
 * mask and penalties, by (value desc, id asc): cand_val / cand_id [rows][k] (device), values are
 * the penalised logits (fp32), ids global.  k <= 256.
 * Step 2, the caller: all-gather the two arrays over the N GPUs into [N][rows][k].
 * Step 3, on any GPU: one token per row from the gathered candidates (per-row or broadcast
 * params; uniforms, token and the optional status are device arrays [rows]).  A sampling row
 * (temperature > 0) needs 1 <= top_k <= k: broadcast params outside that range are rejected
 * with DLLM_ERR_UNSUPPORTED; a per-row top_k outside it gets the greedy token and status bit
 * DLLM_ROW_ERR_TOPK_LARGE. */
DLLM_API dllm_status dllm_cuda_shard_candidates(const dllm_batch_desc *desc, int64_t vocab_offset,
                                                int64_t vocab_total, int k, float *cand_val,
                                                int32_t *cand_id, void *stream);
DLLM_API dllm_status dllm_cuda_merge_sample(int rows, int nshards, int k, const float *cand_val,
                                            const int32_t *cand_id, const dllm_sampler_params *params,
                                            const dllm_sampler_params *row_params,
                                            const float *uniforms, int32_t *token, int32_t *status,
                                            void *stream);

/* Peer exchange for vocabulary-sharded sampling (no counterpart in the reference): the candidate
 * kernel stores each row's k candidates straight into every rank's exchange buffer over NVLink
 * (plain peer stores, no multicast) and counts the row in that rank's arrival counter, so the
 * exchange overlaps the candidate computation row by row instead of following it as a collective.
 *   dllm_cuda_peer_exchange_create: on each rank, a zeroed device buffer for `rows` x `k`
 *     candidates of `world` ranks (arrival counters, then two slots used by alternate steps) and
 *     its cudaIpcMemHandle (64 bytes, written to ipc_handle) for the other ranks.
 *   dllm_cuda_peer_exchange_open / _close: map / unmap another rank's buffer on this GPU.
 *   dllm_cuda_peer_exchange_free: release this rank's buffer.
 *   dllm_cuda_shard_candidates_peer: step `epoch` (1, 2, ...; the same on every rank) of
 *     dllm_cuda_shard_candidates, writing into every rank's buffer; peer_bufs is a DEVICE array
 *     [world] of the buffers as mapped on this GPU (this rank's own buffer at index rank).
 *     Needs k + the history bound <= 256.
 *   dllm_cuda_merge_sample_peer: dllm_cuda_merge_sample over this rank's buffer for step `epoch`;
 *     each row's block waits until every rank's rows have arrived.  The wait is bounded: a rank
 *     missing after 2 s makes the rows time out (token 0, status DLLM_ROW_ERR_TIMEOUT) and the
 *     kernel returns.
 * Every rank must run every step, in the same order, on one stream per rank: a rank's next step's
 * stores reuse the slot of the step before last, which every rank has finished merging by then. */
DLLM_API dllm_status dllm_cuda_peer_exchange_create(int rows, int k, int world, void **buf, void *ipc_handle);
DLLM_API dllm_status dllm_cuda_peer_exchange_open(const void *ipc_handle, void **peer_buf);
DLLM_API dllm_status dllm_cuda_peer_exchange_close(void *peer_buf);
DLLM_API dllm_status dllm_cuda_peer_exchange_free(void *buf);
DLLM_API dllm_status dllm_cuda_shard_candidates_peer(const dllm_batch_desc *desc, int64_t vocab_offset,
                                                     int64_t vocab_total, int k, void *const *peer_bufs, int rank,
                                                     int world, uint64_t epoch, void *stream);
DLLM_API dllm_status dllm_cuda_merge_sample_peer(int rows, int world, int k, const void *local_buf, uint64_t epoch,
                                                 const dllm_sampler_params *params,
                                                 const dllm_sampler_params *row_params, const float *uniforms,
                                                 int32_t *token, int32_t *status, void *stream);

/* The step before the sampler (src/core/context.c:854-876): the final RMSNorm of `rows` hidden
 * states h [rows][hidden] (fp32; src/rmsnorm.c:4-27, norm_w may be NULL, add_one for Gemma's
 * (w + 1)), the logits matvec against unquantised output weights w [vocab][hidden]
 * (DLLM_DTYPE_F32 / BF16 / F16, 16-byte aligned; src/matvec.c:251-366, a double-precision dot
 * product per row rounded once), and, when softcap > 0, logit = softcap * tanhf(logit / softcap).
 * Writes logits [rows][vocab] (fp32) ready for dllm_cuda_sample_batch.  hidden must be a multiple
 * of 8.  All pointers are device memory. */
DLLM_API dllm_status dllm_cuda_lmhead_logits(int rows, int hidden, int vocab, const float *h, const float *norm_w,
                                             float eps, int add_one, const void *w, int w_dtype, float softcap,
                                             float *logits, void *stream);

/* Decode-loop glue (no counterpart in the reference, whose caller appends to its seen-token
 * array on the host): appends token[0] (device) to one sequence's device history
 * hist_ids[hist_off[0], hist_off[1]), which has room for `cap` ids from hist_off[0]; when full,
 * the oldest id is dropped.  Stream-ordered, so "sample, append" steps can run back to back and
 * be captured in a CUDA graph (sample with a caller-provided workspace, or make one call before
 * the capture, so that nothing is allocated during it). */
DLLM_API dllm_status dllm_cuda_append_history(const int32_t *token, int32_t *hist_ids, int64_t *hist_off,
                                              int64_t cap, void *stream);

/* Diagnostics: when given two CUDA events (cudaEvent_t, created by the caller), every later
 * sampling call records `before` on its stream right before the cluster kernel and `after` right
 * after it, so the caller can time that kernel alone; NULLs switch it off.  No counterpart in
 * the reference. */
DLLM_API dllm_status dllm_cuda_set_timing_events(void *before, void *after);

/* Version and build information ("diskllm_cuda <ver> sm_100a"). */
DLLM_API const char *dllm_cuda_version(void);

/* Last CUDA error string recorded by the library on this thread (or ""). */
DLLM_API const char *dllm_cuda_last_error(void);

/* Draw state of a drop-in sampler (the xorshift64 state of src/sampler.c:63), so that a
 * resumed stream reproduces its ids. */
struct sampler;
DLLM_API uint64_t dllm_sampler_get_rng_state(const struct sampler *s);
DLLM_API void     dllm_sampler_set_rng_state(struct sampler *s, uint64_t state);

#ifdef __cplusplus
}
#endif
#endif /* DISKLLM_CUDA_H */
