/*
 * dropin_driver.c -- link test of the drop-in claim (test infrastructure).
 *
 * Written against DiskLLM's own headers (include/diskllm_internal.h, sampler.h, grammar.h) and
 * linked with DiskLLM's own, unchanged src/core/sampler_api.c.  oracle/Makefile builds it twice:
 *   _ref/dropin_ref   + the reference's src/sampler.c and src/core/grammar.c
 *   _ref/dropin_cuda  + libdiskllm_cuda.so (no sampler.c, no grammar.c)
 * Both print one line per sampled token; tests/test_c_dropin.py compares the two.
 *
 * Every step builds a fresh seeded row (splitmix64 + Box-Muller, the same code in both builds),
 * appends the sampled token to the history like a decode loop, and calls diskllm_sample or
 * diskllm_sample_grammar (src/core/sampler_api.c:48-77): mask, presence, repetition, sample.
 * The tokenizer is outside the sampler path; a fixed synthetic vocabulary stands in for it.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "diskllm_internal.h"

static uint64_t g_rng;
static uint64_t splitmix(void) {
    uint64_t z = (g_rng += 0x9E3779B97F4A7C15ULL);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}
static double unit(void) { return ((double)(splitmix() >> 11) + 0.5) * (1.0 / 9007199254740992.0); }
static float gauss(void) {
    const double u = unit(), v = unit();
    return (float)(sqrt(-2.0 * log(u)) * cos(6.283185307179586 * v));
}

/* synthetic vocabulary: JSON punctuation and words first, then filler pieces */
#define GV 3000
static char g_pieces[GV][12];
static void make_vocab(void) {
    static const char *base[] = {"{", "}", "[", "]", ":", ",", " ", "\"", "\"a\"", "\"key\"", "true", "false",
                                 "null", "0", "1", "2", "3", "42", "-", ".", "e", "\"x", "y\"", "\n", "\"v\":",
                                 "{\"", "\"}", "abc", "10", "]}"};
    const int nb = (int)(sizeof base / sizeof base[0]);
    for (int i = 0; i < GV; i++) {
        if (i < nb) {
            snprintf(g_pieces[i], sizeof g_pieces[i], "%s", base[i]);
        } else {
            const int len = 1 + (int)(splitmix() % 5);
            for (int c = 0; c < len; c++) g_pieces[i][c] = (char)('a' + splitmix() % 26);
            g_pieces[i][len] = 0;
        }
    }
}
const char *tokenizer_decode_raw(const tokenizer *tok, int32_t token_id) {
    (void)tok;
    return token_id >= 0 && token_id < GV ? g_pieces[token_id] : NULL;
}

static int run(const char *tag, int V, diskllm_sampler_params sp, int steps, int boost, float sigma, int grammar) {
    diskllm_sampler *s = diskllm_sampler_init(sp);
    if (!s) return 1;
    float *row = malloc(sizeof(float) * (size_t)V);
    int *seen = malloc(sizeof(int) * (size_t)(steps + 64));
    int n_seen = 0;
    for (int i = 0; i < 32; i++) seen[n_seen++] = (int)(splitmix() % (uint64_t)V);
    diskllm_grammar *g = grammar ? diskllm_grammar_init_json() : NULL;
    diskllm_tokenizer tw = {(tokenizer *)(uintptr_t)1};
    const int eos = grammar ? 6 : -1;
    for (int t = 0; t < steps; t++) {
        for (int i = 0; i < V; i++) row[i] = gauss() * sigma;
        for (int b = 0; b < boost; b++) row[splitmix() % (uint64_t)V] += 8.0f;
        const int tok = g ? diskllm_sample_grammar(s, row, V, seen, n_seen, g, &tw, eos)
                          : diskllm_sample(s, row, V, seen, n_seen);
        seen[n_seen++] = tok;
        printf("%s %d %d\n", tag, t, tok);
    }
    if (g) diskllm_grammar_free(g);
    diskllm_sampler_free(s);
    free(row);
    free(seen);
    return 0;
}

int main(void) {
    g_rng = 20240601u;
    make_vocab();
    diskllm_sampler_params a = diskllm_sampler_params_default();
    a.temp = 0.8f, a.top_k = 40, a.top_p = 0.95f, a.min_p = 0.05f, a.repeat_penalty = 1.1f;
    a.presence_penalty = 0.2f, a.seed = 1234;
    int rc = run("topk", 32000, a, 40, 20, 2.5f, 0);
    diskllm_sampler_params b = a;
    b.top_k = 0, b.top_p = 0.9f, b.min_p = 0.0f, b.repeat_penalty = 1.05f, b.presence_penalty = 0.0f, b.seed = 99;
    rc |= run("index_order", 5000, b, 20, 0, 0.5f, 0);
    diskllm_sampler_params c = a;
    c.temp = 1.0f, c.top_k = 0, c.top_p = 0.95f, c.min_p = 0.0f, c.seed = 7;
    rc |= run("grammar", GV, c, 24, 0, 2.0f, 1);
    diskllm_sampler_params d = a;
    d.top_k = 2500, d.top_p = 0.9f, d.min_p = 0.0f, d.seed = 5;
    rc |= run("topk_large", 8000, d, 6, 0, 1.5f, 0);
    diskllm_sampler_params e = a;
    e.temp = 0.0f, e.seed = 3;
    rc |= run("greedy", 20000, e, 8, 5, 2.0f, 0);
    return rc;
}
