/*
 * dllm_oracle.c -- CPU restatement of DiskLLM's sampler chain.
 *
 * TEST INFRASTRUCTURE.  This is the checker the CUDA sampler is compared against; it is
 * never linked into libdiskllm_cuda.so and the product path never calls it.  Its own
 * parity with the reference is pinned by tests/test_oracle_vs_reference.py, which runs
 * the reference's src/sampler.c compiled with the reference's Makefile:10 flags
 * (oracle/_ref/libref_asbuilt.so) on the same rows and uniforms.
 *
 * Build: oracle/Makefile (-O2 -ffp-contract=off: every float operation below is one IEEE
 * binary32 operation, in the order written).
 *
 * Numerics restated from the reference (file:line within DiskLLM):
 *  - repetition: src/sampler.c:21-33.  Negative logits are multiplied by the penalty.
 *    The shipped build (-ffast-math, Makefile:10) turns `x /= p` into `x * (1.0f/p)`; that
 *    is the default here, DLLM_ORACLE_PEN_TRUE_DIV selects the IEEE division of the
 *    strict build.  Applied once per history occurrence, so an id seen c times is scaled
 *    c times with a rounding each time.
 *  - presence: src/sampler.c:35-52, subtracted once per distinct in-range id.
 *  - frequency: not in the reference.  Defined here as x -= (float)count * frequency
 *    (one multiply, one subtract, no fused multiply-add), applied right after presence.
 *  - greedy: src/sampler.c:9-19 (strict >, first maximum wins).
 *  - temperature: src/sampler.c:153-162, t = (x - max) * (1.0f/temp).
 *  - top-k: src/sampler.c:109-134,164-170.  The result is the k best entries by
 *    (t descending, id ascending), sorted that way.  Only when 0 < k < V.
 *  - softmax: src/sampler.c:172-185 (expf, double sum, float multiply by (float)(1/sum)).
 *  - min-p: src/sampler.c:187-202 (absolute threshold, compaction, double renormalise).
 *  - top-p: src/sampler.c:204-222 (prefix in the CURRENT order until (float)cumul >= p;
 *    with top-k off that order is token-id order).
 *  - draw: src/sampler.c:224-233 (float running sum, first r < cumul, else the last).
 *
 * Two modes that are not the reference's (flags; both off by default):
 *  - DLLM_ORACLE_MINP_RELATIVE: min-p keeps p >= min_p * p_max, p_max the largest
 *    probability (fp32 product), instead of the reference's absolute p >= min_p.
 *  - DLLM_ORACLE_TOPP_SORTED (top-k off, temperature > 0): the sorted-nucleus sampler with
 *    exact cumulative sums -- see sample_row_sorted.
 */
#define _GNU_SOURCE
#include "dllm_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#if defined(__x86_64__) || defined(__i386__)
#include <xmmintrin.h>
#endif

typedef struct {
    int32_t idx;
    float   val;
} entry_t;

/*
 * Numerics of the as-built reference.  Makefile:10 builds src/sampler.c with
 * -O3 -ffast-math; gcc 13 then vectorises the softmax and renormalisation loops of
 * sampler.c:177-185,198-201,218-221 four entries at a time.  Two consequences fix the
 * exact bits of every probability, and both are restated here:
 *  - expf: entries [0, 4*floor((k-1)/4)) go through glibc's 4-wide libmvec expf
 *    (_ZGVbN4v_expf, glibc 2.39; differs from scalar expf by up to 3 ulp); the remaining
 *    1..4 entries, and every entry when k <= 4, through scalar expf.
 *  - double sums: over the same vector body the sum runs in two lanes, each block of four
 *    adding (x0 + x2) to lane 0 and (x1 + x3) to lane 1; the lanes are then added and the
 *    tail entries added one at a time.  For k <= 4 the sum is sequential.
 * With DLLM_ORACLE_PLAIN_MATH the oracle instead uses scalar expf and sequential sums
 * (the literal C semantics, as the strict build computes them).
 */
#if defined(__x86_64__)
#include <immintrin.h>
__m128 _ZGVbN4v_expf(__m128);
#define HAVE_LIBMVEC 1
#endif

static inline int vec_body(int k) { return k >= 5 ? 4 * ((k - 1) / 4) : 0; }

static void exp_entries(entry_t *b, int k, float mv, int plain)
{
    int i = 0;
#ifdef HAVE_LIBMVEC
    if (!plain) {
        for (int nb = vec_body(k); i < nb; i += 4) {
            __m128 x = _mm_set_ps(b[i + 3].val - mv, b[i + 2].val - mv,
                                  b[i + 1].val - mv, b[i].val - mv);
            float o[4];
            _mm_storeu_ps(o, _ZGVbN4v_expf(x));
            for (int j = 0; j < 4; j++) b[i + j].val = o[j];
        }
    }
#else
    (void)plain;
#endif
    for (; i < k; i++) b[i].val = expf(b[i].val - mv);
}

static double sum_entries(const entry_t *b, int k, int plain)
{
    double s = 0.0;
    int i = 0;
    if (!plain) {
        int nb = vec_body(k);
        if (nb) {
            double lo = 0.0, hi = 0.0;
            for (; i < nb; i += 4) {
                lo += (double)b[i].val + (double)b[i + 2].val;
                hi += (double)b[i + 1].val + (double)b[i + 3].val;
            }
            s = lo + hi;
        }
    }
    for (; i < k; i++) s += b[i].val;
    return s;
}

typedef struct {
    float    *w;      /* penalised row */
    entry_t  *buf;    /* candidate list */
    int32_t  *cnt;    /* per-id occurrence counts (zero between rows) */
    uint64_t *mass;   /* sorted-nucleus mode: fixed-point mass per sorted entry */
    int       vocab;
} scratch_t;

/* ---- xorshift64, src/sampler.c:69-81 --------------------------------------------- */

float dllm_oracle_xorshift_uniform(uint64_t *state)
{
    uint64_t x = *state;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    *state = x;
    return (float)(x >> 11) * (1.0f / (float)(1ULL << 53));
}

uint64_t dllm_oracle_xorshift_inverse(uint64_t y)
{
    /* undo x ^= x << 17 */
    uint64_t x = y ^ (y << 17) ^ (y << 34) ^ (y << 51);
    /* undo x ^= x >> 7 */
    uint64_t z = x;
    for (int s = 7; s < 64; s += 7) z ^= x >> s;
    /* undo x ^= x << 13 */
    x = z ^ (z << 13) ^ (z << 26) ^ (z << 39) ^ (z << 52);
    return x;
}

/* ---- ordering helpers --------------------------------------------------------------- */

/* a ranks before b: larger value first, ties toward the lower id. */
static inline int ranks_before(const entry_t *a, const entry_t *b)
{
    if (a->val > b->val) return 1;
    if (a->val < b->val) return 0;
    return a->idx < b->idx;
}

static int cmp_rank(const void *pa, const void *pb)
{
    const entry_t *a = pa, *b = pb;
    if (ranks_before(a, b)) return -1;
    if (ranks_before(b, a)) return 1;
    return 0;
}

/* min-heap on rank (root = the worst kept entry) */
static void heap_sift_down(entry_t *h, int n, int i)
{
    for (;;) {
        int l = 2 * i + 1, r = l + 1, w = i;
        if (l < n && ranks_before(&h[w], &h[l])) w = l;
        if (r < n && ranks_before(&h[w], &h[r])) w = r;
        if (w == i) return;
        entry_t t = h[i]; h[i] = h[w]; h[w] = t;
        i = w;
    }
}

/* Moves the k best entries of buf[0..n) (by rank) to buf[0..k), sorted best first. */
static void select_top_k(entry_t *buf, int n, int k)
{
    /* NaN keys compare false both ways; the reference's insertion sort then leaves the
     * first k entries in id order (every comparison fails).  Only reachable when the row
     * maximum is -inf (fully masked row), where every key is NaN. */
    int any_nan = 0;
    for (int i = 0; i < n; i++) if (isnan(buf[i].val)) { any_nan = 1; break; }
    if (any_nan) return;
    for (int i = k / 2 - 1; i >= 0; i--) heap_sift_down(buf, k, i);
    for (int i = k; i < n; i++) {
        if (ranks_before(&buf[i], &buf[0])) {
            buf[0] = buf[i];
            heap_sift_down(buf, k, 0);
        }
    }
    qsort(buf, (size_t)k, sizeof(entry_t), cmp_rank);
}

/* ---- one row -------------------------------------------------------------------------- */

static void penalise_row(const dllm_oracle_batch *b, int row, const dllm_oracle_params *p,
                         scratch_t *s)
{
    const int V = b->vocab;
    float *w = s->w;
    memcpy(w, b->logits + (size_t)row * V, sizeof(float) * (size_t)V);

    if (b->mask) {
        const uint32_t *m = b->mask + (size_t)row * ((V + 31) / 32);
        for (int i = 0; i < V; i++)
            if (!((m[i >> 5] >> (i & 31)) & 1u)) w[i] = -INFINITY;
    }
    if (!b->hist_ids || !b->hist_off) return;
    const int64_t h0 = b->hist_off[row], h1 = b->hist_off[row + 1];
    if (h1 <= h0) return;
    const int32_t *h = b->hist_ids + h0;
    const int64_t n = h1 - h0;

    if (p->presence != 0.0f || p->frequency != 0.0f) {
        for (int64_t i = 0; i < n; i++)
            if (h[i] >= 0 && h[i] < V) s->cnt[h[i]]++;
        for (int64_t i = 0; i < n; i++) {
            int id = h[i];
            if (id < 0 || id >= V || s->cnt[id] == 0) continue;
            if (p->presence != 0.0f) w[id] = w[id] - p->presence;
            if (p->frequency != 0.0f) {
                float f = (float)s->cnt[id] * p->frequency;
                w[id] = w[id] - f;
            }
            s->cnt[id] = 0; /* first occurrence handled; later ones skip */
        }
    }
    if (p->repetition > 1.0f) {
        const float inv = 1.0f / p->repetition;
        const int true_div = (b->flags & DLLM_ORACLE_PEN_TRUE_DIV) != 0;
        for (int64_t i = 0; i < n; i++) {
            int id = h[i];
            if (id < 0 || id >= V) continue;
            if (w[id] < 0.0f) w[id] = w[id] * p->repetition;
            else w[id] = true_div ? w[id] / p->repetition : w[id] * inv;
        }
    }
}

/*
 * Sorted-nucleus mode.  The reference's top-p keeps an index-order prefix when top-k is off
 * (src/sampler.c:165-170 sort only under top-k) and draws with a float running sum that drifts
 * by up to ~1e-5 over 256000 entries.  This mode is the corrected sampler, defined exactly:
 *   1. t_i = (x_i - max) * (1.0f / temp) as the reference; order by (t desc, id asc) (the order
 *      partial_sort_top_k gives, src/sampler.c:109-134);
 *   2. mass E_i = rint(expf(t_i) * 2^42), an integer (exact for expf >= 2^-19), so every sum
 *      below is exact;
 *   3. min-p (optional): inv_sum = (float)(1 / (sum E * 2^-42)); keep the sorted prefix with
 *      (float)(expf(t_i) * inv_sum) >= threshold (absolute min_p, or min_p * inv_sum with
 *      DLLM_ORACLE_MINP_RELATIVE); none kept -> keep all (src/sampler.c:188-196);
 *      S2 = mass of the kept entries;
 *   4. top-p (top_p < 1): T = max(ceil((double)top_p * (double)S2), 1) - 1; the cut is the
 *      first entry whose inclusive prefix mass exceeds T; S3 = that prefix mass (else S3 = S2);
 *   5. draw: T = floor((double)r * (double)S3); the token is the first entry whose inclusive
 *      prefix mass exceeds T.
 * kept_prob / kept_cdf report E_i / S3 and prefix / S3 (rounded to float).
 */
static int32_t sample_row_sorted(const dllm_oracle_batch *b, int row, const dllm_oracle_params *p,
                                 scratch_t *s, float m)
{
    const int V = b->vocab;
    entry_t *buf = s->buf;
    const float inv_temp = 1.0f / p->temperature;
    for (int i = 0; i < V; i++) {
        buf[i].idx = i;
        buf[i].val = (s->w[i] - m) * inv_temp;
    }
    select_top_k(buf, V, V);
    uint64_t *E = s->mass;
    uint64_t sall = 0;
    int npos = 0;
    for (int i = 0; i < V; i++) {
        const float e = expf(buf[i].val);
        E[i] = (uint64_t)rint((double)e * 4398046511104.0);
        sall += E[i];
        if (E[i]) npos = i + 1;
    }
    int nk = npos;  /* entries past npos have no mass and are never kept */
    if (p->min_p > 0.0f) {
        const float inv_sum = (float)(1.0 / ((double)sall * 0x1p-42));
        const float thr = (b->flags & DLLM_ORACLE_MINP_RELATIVE) ? p->min_p * inv_sum : p->min_p;
        int n = 0;
        while (n < npos && expf(buf[n].val) * inv_sum >= thr) n++;
        if (n > 0) nk = n;
    }
    uint64_t s2 = 0;
    for (int i = 0; i < nk; i++) s2 += E[i];
    int kc = nk;
    uint64_t s3 = s2;
    if (p->top_p < 1.0f) {
        double x = ceil((double)p->top_p * (double)s2);
        const uint64_t T = (x < 1.0 ? 1ull : (uint64_t)x) - 1ull;
        uint64_t cum = 0;
        for (int i = 0; i < nk; i++) {
            cum += E[i];
            if (cum > T) { kc = i + 1; break; }
        }
        s3 = 0;
        for (int i = 0; i < kc; i++) s3 += E[i];
    }
    if (b->kept_n) b->kept_n[row] = kc;
    if (b->kept_idx || b->kept_prob || b->kept_cdf) {
        uint64_t cum = 0;
        for (int i = 0; i < kc && i < b->kept_cap; i++) {
            size_t o = (size_t)row * b->kept_cap + i;
            cum += E[i];
            if (b->kept_idx) b->kept_idx[o] = buf[i].idx;
            if (b->kept_prob) b->kept_prob[o] = (float)((double)E[i] / (double)s3);
            if (b->kept_cdf) b->kept_cdf[o] = (float)((double)cum / (double)s3);
        }
    }
    const uint64_t T = (uint64_t)floor((double)b->uniforms[row] * (double)s3);
    uint64_t cum = 0;
    for (int i = 0; i < kc; i++) {
        cum += E[i];
        if (cum > T) return buf[i].idx;
    }
    return buf[kc - 1].idx;
}

static int32_t sample_row(const dllm_oracle_batch *b, int row, const dllm_oracle_params *p,
                          scratch_t *s)
{
    const int V = b->vocab;
    const float *w = s->w;
    entry_t *buf = s->buf;

    if (b->kept_n) b->kept_n[row] = 0;
    if (p->temperature == 0.0f) {
        int best = 0;
        float bv = w[0];
        for (int i = 1; i < V; i++) if (w[i] > bv) { bv = w[i]; best = i; }
        return best;
    }

    const float inv_temp = 1.0f / p->temperature;
    float m = w[0];
    for (int i = 1; i < V; i++) if (w[i] > m) m = w[i];
    for (int i = 0; i < V; i++) {
        buf[i].idx = i;
        buf[i].val = (w[i] - m) * inv_temp;
    }

    int k = V;
    if (p->top_k > 0 && p->top_k < V) {
        k = p->top_k;
        select_top_k(buf, V, k);
    } else if ((b->flags & DLLM_ORACLE_TOPP_SORTED) && m > -INFINITY && m < INFINITY) {
        return sample_row_sorted(b, row, p, s, m);
    }
    if (b->topk_idx) {
        int32_t *o = b->topk_idx + (size_t)row * b->topk_cap;
        for (int i = 0; i < k && i < b->topk_cap; i++) o[i] = buf[i].idx;
    }

    const int plain = (b->flags & DLLM_ORACLE_PLAIN_MATH) != 0;
    float mv = buf[0].val;
    for (int i = 1; i < k; i++) if (buf[i].val > mv) mv = buf[i].val;
    exp_entries(buf, k, mv, plain);
    const double sum = sum_entries(buf, k, plain);
    const float inv_sum = (float)(1.0 / sum);
    for (int i = 0; i < k; i++) buf[i].val = buf[i].val * inv_sum;

    if (p->min_p > 0.0f) {
        float thr = p->min_p;
        if (b->flags & DLLM_ORACLE_MINP_RELATIVE) {
            float pmax = buf[0].val;
            for (int i = 1; i < k; i++) if (buf[i].val > pmax) pmax = buf[i].val;
            thr = p->min_p * pmax;
        }
        int nk = 0;
        for (int i = 0; i < k; i++)
            if (buf[i].val >= thr) buf[nk++] = buf[i];
        if (nk > 0) k = nk;
        const double s2 = sum_entries(buf, k, plain);
        const float inv2 = (float)(1.0 / s2);
        for (int i = 0; i < k; i++) buf[i].val = buf[i].val * inv2;
    }

    if (p->top_p < 1.0f) {
        double cum = 0.0;
        int nk = k;
        for (int i = 0; i < k; i++) {
            cum += buf[i].val;
            if ((float)cum >= p->top_p) { nk = i + 1; break; }
        }
        /* test-only alternatives: the cut one entry earlier / later (a prefix within rounding
           distance of top_p), used to classify GPU draws at knife-edge cuts */
        if ((b->flags & DLLM_ORACLE_CUT_EARLIER) && nk > 1) nk--;
        if ((b->flags & DLLM_ORACLE_CUT_LATER) && nk < k) nk++;
        k = nk;
        const double s3 = sum_entries(buf, k, plain);
        const float inv3 = (float)(1.0 / s3);
        for (int i = 0; i < k; i++) buf[i].val = buf[i].val * inv3;
    }

    if (b->kept_n) b->kept_n[row] = k;
    if (b->kept_idx || b->kept_prob || b->kept_cdf) {
        float c = 0.0f;
        for (int i = 0; i < k && i < b->kept_cap; i++) {
            size_t o = (size_t)row * b->kept_cap + i;
            c = c + buf[i].val;
            if (b->kept_idx) b->kept_idx[o] = buf[i].idx;
            if (b->kept_prob) b->kept_prob[o] = buf[i].val;
            if (b->kept_cdf) b->kept_cdf[o] = c;
        }
    }

    const float r = b->uniforms[row];
    float c = 0.0f;
    for (int i = 0; i < k; i++) {
        c = c + buf[i].val;
        if (r < c) return buf[i].idx;
    }
    return buf[k - 1].idx;
}

/* ---- batch driver -------------------------------------------------------------------- */

typedef struct {
    const dllm_oracle_batch *b;
    int r0, r1, ftz, err;
} job_t;

static void *run_rows(void *arg)
{
    job_t *j = arg;
    const dllm_oracle_batch *b = j->b;
#if defined(__x86_64__) || defined(__i386__)
    unsigned saved = _mm_getcsr();
    if (j->ftz) _mm_setcsr(saved | 0x8040u); /* FTZ (bit 15) | DAZ (bit 6) */
#endif
    scratch_t s;
    s.vocab = b->vocab;
    s.w = malloc(sizeof(float) * (size_t)b->vocab);
    s.buf = malloc(sizeof(entry_t) * (size_t)b->vocab);
    s.cnt = calloc((size_t)b->vocab, sizeof(int32_t));
    s.mass = malloc(sizeof(uint64_t) * (size_t)b->vocab);
    if (!s.w || !s.buf || !s.cnt || !s.mass) {
        j->err = -2;
    } else {
        for (int row = j->r0; row < j->r1; row++) {
            const dllm_oracle_params *p = b->params + (b->params_per_row ? row : 0);
            penalise_row(b, row, p, &s);
            if (b->pen_logits)
                memcpy(b->pen_logits + (size_t)row * b->vocab, s.w,
                       sizeof(float) * (size_t)b->vocab);
            b->token[row] = sample_row(b, row, p, &s);
        }
    }
    free(s.w); free(s.buf); free(s.cnt); free(s.mass);
#if defined(__x86_64__) || defined(__i386__)
    _mm_setcsr(saved);
#endif
    return NULL;
}

int dllm_oracle_sample_batch(const dllm_oracle_batch *b, int ftz, int threads)
{
    if (!b || b->rows < 0 || b->vocab <= 0 || !b->logits || !b->uniforms || !b->params ||
        !b->token)
        return -1;
    if ((b->kept_idx || b->kept_prob || b->kept_cdf) && b->kept_cap <= 0) return -1;
    if (b->topk_idx && b->topk_cap <= 0) return -1;
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
        jobs[t].ftz = ftz;
    }
    if (threads == 1) {
        run_rows(&jobs[0]);
    } else {
        for (int t = 0; t < threads; t++) pthread_create(&tid[t], NULL, run_rows, &jobs[t]);
        for (int t = 0; t < threads; t++) pthread_join(tid[t], NULL);
    }
    int err = 0;
    for (int t = 0; t < threads; t++) if (jobs[t].err) err = jobs[t].err;
    free(jobs); free(tid);
    return err;
}
