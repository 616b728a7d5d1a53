/*
 * grammar.h -- DiskLLM's grammar-constraint interface, served by libdiskllm_cuda.so, plus the
 * packed allow-bitmask builder that feeds the CUDA sampler.
 *
 * The diskllm_grammar_* names, types and signatures are those of DiskLLM's include/grammar.h
 * (lines 12-41) so that src/core/sampler_api.c links against this library instead of
 * src/core/grammar.c; each keeps the argument meaning, results and error behaviour of the
 * function it replaces (cited per declaration).  The prefix checks are the reference's JSON
 * and receipt validators, restated as incremental state machines: the committed text is
 * scanned once per decode step and each vocabulary piece only continues from that state.
 */
#ifndef DISKLLM_GRAMMAR_H
#define DISKLLM_GRAMMAR_H

#include <stdbool.h>
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

typedef struct diskllm_grammar diskllm_grammar;

/* src/core/grammar.c:16-28 (receipt mode if the text names "bbox_2d", JSON mode if it names
 * "object" or "value"), :30-45 (from a file), :47-51 (JSON) */
DLLM_API diskllm_grammar *diskllm_grammar_init_from_file(const char *filepath);
DLLM_API diskllm_grammar *diskllm_grammar_init_from_str(const char *grammar_str);
DLLM_API diskllm_grammar *diskllm_grammar_init_json(void);
/* src/core/grammar.c:53-55, :57-62 */
DLLM_API void diskllm_grammar_free(diskllm_grammar *g);
DLLM_API void diskllm_grammar_reset(diskllm_grammar *g);
/* src/core/grammar.c:215-233: would the committed text followed by `piece` still be a valid
 * prefix (false when the total reaches 8191 bytes) */
DLLM_API bool diskllm_grammar_accept_str(const diskllm_grammar *g, const char *piece);
/* src/core/grammar.c:235-243: commit `piece` (dropped when the text would reach 8191 bytes) */
DLLM_API void diskllm_grammar_advance(diskllm_grammar *g, const char *piece);
/* src/core/grammar.c:245-259: balanced braces and brackets, outside a string, > 1 byte */
DLLM_API bool diskllm_grammar_is_finished(const diskllm_grammar *g);
/* src/core/grammar.c:261-308: logits of disallowed tokens (empty or missing pieces, pieces that
 * break the prefix, EOS before the text is finished) become -INFINITY; returns the allowed count.
 * With a NULL grammar, logits or callback, or vocab_size <= 0: no change, returns vocab_size. */
DLLM_API int diskllm_grammar_apply_mask(diskllm_grammar *g, float *logits, int vocab_size, void *tok_ctx,
                                        const char *(*get_token_str)(void *ctx, int token_id),
                                        int eos_token_id);

/* Packed allow-bitmask for dllm_batch_desc::mask (no counterpart in the reference, which writes
 * -INFINITY into the logits): bit (i & 31) of word i >> 5 is set iff diskllm_grammar_apply_mask
 * would leave token i alone; bits past vocab_size are cleared.  `out_words` holds
 * (vocab_size + 31) / 32 words.  Returns the allowed count (vocab_size, all bits set, for the
 * argument cases where apply_mask changes nothing). */
DLLM_API int dllm_grammar_build_bitmask(const diskllm_grammar *g, int vocab_size, void *tok_ctx,
                                        const char *(*get_token_str)(void *ctx, int token_id),
                                        int eos_token_id, uint32_t *out_words);

/* The vocabulary's pieces read once through the callback and kept, so that each decode step's
 * bitmask costs one pass over the pieces and no callback.  No counterpart in the reference. */
typedef struct dllm_grammar_vocab dllm_grammar_vocab;
DLLM_API dllm_grammar_vocab *dllm_grammar_vocab_create(int vocab_size, void *tok_ctx,
                                                       const char *(*get_token_str)(void *ctx, int token_id),
                                                       int eos_token_id);
DLLM_API void dllm_grammar_vocab_free(dllm_grammar_vocab *v);
DLLM_API int dllm_grammar_build_bitmask_cached(const diskllm_grammar *g, const dllm_grammar_vocab *v,
                                               uint32_t *out_words);

#ifdef __cplusplus
}
#endif

#endif /* DISKLLM_GRAMMAR_H */
