/*
 * dllm_oracle.h -- CPU restatement of DiskLLM's sampler chain (TEST INFRASTRUCTURE ONLY).
 *
 * This header and dllm_oracle.c are the parity checker for the CUDA sampler in
 * diskllm_b200/csrc.  Only tests, __graft_entry__.smoke() and bench.py's CPU baseline
 * leg may load it.  The product library (libdiskllm_cuda.so) never links or calls it.
 *
 * It restates, in batched form with caller-supplied uniforms, the per-row sequence that
 * DiskLLM runs for one sampled token:
 *   grammar mask    src/core/grammar.c:275-308      (here: packed uint32 allow-bitmask)
 *   presence        src/sampler.c:35-52             (once per distinct id)
 *   frequency       -- absent from the reference; builder-defined extension (see .c)
 *   repetition      src/sampler.c:21-33             (once per occurrence)
 *   sampler_sample  src/sampler.c:136-234           (temperature, top-k, softmax, min-p,
 *                                                    top-p, fp32 sequential draw)
 *   ordering        src/core/sampler_api.c:48-63    (mask -> presence -> repetition -> sample)
 */
#ifndef DLLM_ORACLE_H
#define DLLM_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* mode flags (same bit values as the product's DLLM_MODE_* flags) */
#define DLLM_ORACLE_TOPP_SORTED   0x1u  /* sorted-nucleus mode when top-k is off (temperature
                                           > 0): the corrected definition in dllm_oracle.c */
#define DLLM_ORACLE_PEN_TRUE_DIV  0x2u  /* positive logits divided by the penalty (strict build)
                                           instead of multiplied by 1/penalty (as-built) */
#define DLLM_ORACLE_MINP_RELATIVE 0x4u  /* min-p threshold min_p * (largest probability)
                                           instead of the reference's absolute min_p */
#define DLLM_ORACLE_CUT_EARLIER   0x200u /* oracle only: index-order top-p cut one entry earlier */
#define DLLM_ORACLE_CUT_LATER     0x400u /* oracle only: index-order top-p cut one entry later */
#define DLLM_ORACLE_PLAIN_MATH    0x100u /* oracle only: scalar expf + sequential sums instead
                                            of the as-built build's libmvec/2-lane numerics */

typedef struct {
    float temperature;   /* 0 -> greedy */
    float top_p;         /* >= 1 -> off */
    float min_p;         /* <= 0 -> off (absolute threshold, as in the reference) */
    int   top_k;         /* <= 0 or >= V -> off */
    float repetition;    /* <= 1 -> off */
    float presence;      /* 0 -> off */
    float frequency;     /* 0 -> off (extension) */
} dllm_oracle_params;

typedef struct {
    int rows;
    int vocab;
    const float    *logits;      /* [rows][vocab] */
    const uint32_t *mask;        /* [rows][(vocab+31)/32] allow-bits, LSB-first; NULL = none */
    const int32_t  *hist_ids;    /* CSR history ids; NULL = none */
    const int64_t  *hist_off;    /* [rows+1] */
    const float    *uniforms;    /* [rows] draws in [0,1) */
    const dllm_oracle_params *params;
    int   params_per_row;        /* 0: params[0] for all rows */
    unsigned flags;

    int32_t *token;              /* [rows] out */
    float   *pen_logits;         /* [rows][vocab] out (mask + penalties applied) or NULL */
    int32_t *kept_n;             /* [rows] out: length of the final draw list, or NULL */
    int32_t *kept_idx;           /* [rows][kept_cap] out: token ids in draw order, or NULL */
    float   *kept_prob;          /* [rows][kept_cap] out: final probabilities, or NULL */
    float   *kept_cdf;           /* [rows][kept_cap] out: fp32 running sum after each id, or NULL */
    int      kept_cap;
    int32_t *topk_idx;           /* [rows][topk_cap] out: ids after top-k/sort stage, or NULL */
    int      topk_cap;
} dllm_oracle_batch;

/* Runs every row; returns 0 or a negative error.  Sets x86 MXCSR FTZ|DAZ for the
 * duration when `ftz` is nonzero (the as-built reference executables are linked with
 * -ffast-math, which loads crtfastmath and sets both bits at start-up). */
int dllm_oracle_sample_batch(const dllm_oracle_batch *b, int ftz, int threads);

/* xorshift64 uniform exactly as src/sampler.c:69-81 computes it. */
float    dllm_oracle_xorshift_uniform(uint64_t *state);
/* Inverse of one xorshift64 step: returns s with xorshift64(s) == x. */
uint64_t dllm_oracle_xorshift_inverse(uint64_t x);

#ifdef __cplusplus
}
#endif
#endif
