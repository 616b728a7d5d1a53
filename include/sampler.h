/*
 * sampler.h -- DiskLLM's sampler interface, served by libdiskllm_cuda.so.
 *
 * Names, types and signatures are those of DiskLLM's include/sampler.h:1-36 so that
 * src/core/sampler_api.c and main/diskllm.c compile and link unchanged against this
 * library instead of src/sampler.c.  Each entry point replaces the function at the cited
 * line of DiskLLM's src/sampler.c and keeps its argument meaning and error behaviour.
 * The work runs on the GPU; host arrays are copied to the device and back.
 */
#ifndef SAMPLER_H
#define SAMPLER_H

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

typedef struct sampler sampler;

/* include/sampler.h:10-16 */
typedef struct {
    float temperature;   /* 0.0 = greedy */
    int   top_k;         /* 0 = disabled */
    float top_p;         /* 1.0 = disabled */
    float min_p;         /* 0.0 = disabled */
    uint64_t seed;       /* xorshift64 seed; 0 -> 0xDEADBEEF12345678 */
} sampler_config;

/* replaces src/sampler.c:83-89; NULL on allocation failure */
DLLM_API sampler *sampler_create(const sampler_config *cfg);

/* replaces src/sampler.c:91-95; NULL is a no-op */
DLLM_API void sampler_free(sampler *s);

/* replaces src/sampler.c:21-33: in place on host logits; ids outside [0, vocab_size) are
 * skipped; no-op when penalty <= 1, seen_tokens is NULL or num_seen <= 0 */
DLLM_API void sampler_apply_repetition_penalty(float *logits, int vocab_size, const int *seen_tokens,
                                               int num_seen, float penalty);

/* replaces src/sampler.c:35-52: once per distinct in-range id; no-op when
 * presence_penalty == 0, seen_tokens is NULL or num_seen <= 0 */
DLLM_API void sampler_apply_presence_penalty(float *logits, int vocab_size, const int *seen_tokens,
                                             int num_seen, float presence_penalty);

/* replaces src/sampler.c:136-234: does not modify logits; advances the xorshift state by
 * one draw unless temperature == 0 */
DLLM_API int sampler_sample(sampler *s, float *logits, int vocab_size);

/* replaces src/sampler.c:9-19: first maximum wins */
DLLM_API int greedy_sample(const float *logits, int vocab_size);

#ifdef __cplusplus
}
#endif
#endif /* SAMPLER_H */
