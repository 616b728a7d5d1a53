/*
 * ref_harness.c -- drives DiskLLM's own sampler (src/sampler.c, compiled unmodified from
 * the reference tree by oracle/Makefile) over a batch of rows.  TEST INFRASTRUCTURE: used
 * by the parity tests to pin the restated oracle, and by bench.py's reference arm / CPU
 * baseline.  Never linked into the product.
 *
 * Per row it performs what src/core/sampler_api.c:48-63 does for one token:
 *   mask (-INFINITY on cleared allow-bits, the effect of grammar.c:275-308)
 *   -> sampler_apply_presence_penalty   (only when presence != 0, sampler_api.c:55)
 *   -> sampler_apply_repetition_penalty (only when repetition > 1, sampler_api.c:59)
 *   -> sampler_sample
 * The reference draws its uniform from its private xorshift64 state (sampler.c:225).  To
 * feed a chosen uniform r, the harness creates the sampler with the seed whose next
 * xorshift64 output encodes r (xorshift64 is a bijection, so the seed is its inverse).
 */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#if defined(__x86_64__) || defined(__i386__)
#include <xmmintrin.h>
#endif

#include "sampler.h" /* the reference's include/sampler.h */

typedef struct {
    float temperature, top_p, min_p;
    int   top_k;
    float repetition, presence, frequency;
} ref_params; /* same layout as dllm_oracle_params */

typedef struct {
    int rows, vocab;
    const float    *logits;
    const uint32_t *mask;
    const int32_t  *hist_ids;
    const int64_t  *hist_off;
    const float    *uniforms;
    const ref_params *params;
    int params_per_row;
    int32_t *token;
    float   *pen_logits;
} ref_batch;

static uint64_t xs_inverse(uint64_t y)
{
    uint64_t x = y ^ (y << 17) ^ (y << 34) ^ (y << 51);
    uint64_t z = x;
    for (int s = 7; s < 64; s += 7) z ^= x >> s;
    return z ^ (z << 13) ^ (z << 26) ^ (z << 39) ^ (z << 52);
}

/* seed s such that the reference's first rand_f32() after sampler_create(seed=s) == r;
 * returns 0 when r is not an exact output of rand_f32. */
uint64_t ref_seed_for_uniform(float r)
{
    if (!(r >= 0.0f && r < 1.0f)) return 0;
    uint64_t m = (uint64_t)((double)r * 9007199254740992.0); /* r * 2^53 */
    if ((float)m * (1.0f / (float)(1ULL << 53)) != r) return 0;
    uint64_t x = m << 11;
    if (x == 0) x = 1; /* (1 >> 11) == 0 still encodes r == 0 */
    return xs_inverse(x);
}

typedef struct {
    const ref_batch *b;
    int r0, r1, stream, err;
    uint64_t stream_seed;
} job_t;

static void run_row_prefix(const ref_batch *b, int row, const ref_params *p, float *w)
{
    const int V = b->vocab;
    memcpy(w, b->logits + (size_t)row * V, sizeof(float) * (size_t)V);
    if (b->mask) {
        const uint32_t *m = b->mask + (size_t)row * ((V + 31) / 32);
        for (int i = 0; i < V; i++)
            if (!((m[i >> 5] >> (i & 31)) & 1u)) w[i] = -INFINITY;
    }
    if (b->hist_ids && b->hist_off) {
        const int32_t *h = b->hist_ids + b->hist_off[row];
        int n = (int)(b->hist_off[row + 1] - b->hist_off[row]);
        if (p->presence != 0.0f && n > 0)
            sampler_apply_presence_penalty(w, V, h, n, p->presence);
        if (p->repetition > 1.0f && n > 0)
            sampler_apply_repetition_penalty(w, V, h, n, p->repetition);
    }
}

static void *run_rows(void *arg)
{
    job_t *j = arg;
    const ref_batch *b = j->b;
#if defined(__x86_64__) || defined(__i386__)
    /* the reference executables link crtfastmath (-ffast-math at link): FTZ | DAZ */
    unsigned saved = _mm_getcsr();
    _mm_setcsr(saved | 0x8040u);
#endif
    float *w = malloc(sizeof(float) * (size_t)b->vocab);
    sampler *shared = NULL;
    if (!w) { j->err = -2; goto out; }
    if (j->stream) {
        const ref_params *p = b->params;
        sampler_config c = { p->temperature, p->top_k, p->top_p, p->min_p, j->stream_seed };
        shared = sampler_create(&c);
        if (!shared) { j->err = -2; goto out; }
    }
    for (int row = j->r0; row < j->r1; row++) {
        const ref_params *p = b->params + (b->params_per_row ? row : 0);
        run_row_prefix(b, row, p, w);
        if (b->pen_logits)
            memcpy(b->pen_logits + (size_t)row * b->vocab, w, sizeof(float) * (size_t)b->vocab);
        if (j->stream) {
            b->token[row] = sampler_sample(shared, w, b->vocab);
        } else {
            uint64_t seed = ref_seed_for_uniform(b->uniforms[row]);
            if (!seed) { j->err = -3; break; }
            sampler_config c = { p->temperature, p->top_k, p->top_p, p->min_p, seed };
            sampler *s = sampler_create(&c);
            if (!s) { j->err = -2; break; }
            b->token[row] = sampler_sample(s, w, b->vocab);
            sampler_free(s);
        }
    }
out:
    if (shared) sampler_free(shared);
    free(w);
#if defined(__x86_64__) || defined(__i386__)
    _mm_setcsr(saved);
#endif
    return NULL;
}

/*
 * stream == 0: parity mode, row i is drawn with uniforms[i] (a fresh sampler per row).
 * stream != 0: throughput mode, one sampler per thread advancing its own xorshift state
 *              (how the reference runs); uniforms are ignored, params[0] is used.
 * Returns 0 or a negative error; *seconds gets the wall time of the row loop
 * (CLOCK_MONOTONIC, thread start to join).
 */
int ref_sample_batch(const ref_batch *b, int threads, int stream, double *seconds)
{
    if (!b || b->rows < 0 || b->vocab <= 0 || !b->logits || !b->params || !b->token) return -1;
    if (!stream && !b->uniforms) return -1;
    if (threads < 1) threads = 1;
    if (threads > b->rows) threads = b->rows > 0 ? b->rows : 1;
    job_t *jobs = calloc((size_t)threads, sizeof(job_t));
    pthread_t *tid = calloc((size_t)threads, sizeof(pthread_t));
    if (!jobs || !tid) { free(jobs); free(tid); return -2; }
    int per = (b->rows + threads - 1) / threads;
    for (int t = 0; t < threads; t++) {
        jobs[t].b = b;
        jobs[t].r0 = t * per < b->rows ? t * per : b->rows;
        jobs[t].r1 = (t + 1) * per < b->rows ? (t + 1) * per : b->rows;
        jobs[t].stream = stream;
        jobs[t].stream_seed = 0x9E3779B97F4A7C15ULL * (uint64_t)(t + 1);
    }
    struct timespec a, z;
    clock_gettime(CLOCK_MONOTONIC, &a);
    if (threads == 1) {
        run_rows(&jobs[0]);
    } else {
        for (int t = 0; t < threads; t++) pthread_create(&tid[t], NULL, run_rows, &jobs[t]);
        for (int t = 0; t < threads; t++) pthread_join(tid[t], NULL);
    }
    clock_gettime(CLOCK_MONOTONIC, &z);
    if (seconds) *seconds = (double)(z.tv_sec - a.tv_sec) + 1e-9 * (double)(z.tv_nsec - a.tv_nsec);
    int err = 0;
    for (int t = 0; t < threads; t++) if (jobs[t].err) err = jobs[t].err;
    free(jobs); free(tid);
    return err;
}

/* single greedy call, for the greedy_sample drop-in parity test */
int ref_greedy(const float *logits, int vocab)
{
    return greedy_sample(logits, vocab);
}
