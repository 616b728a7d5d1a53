// dllm_grammar.cu -- host code: DiskLLM's grammar constraint (include/grammar.h) and the packed
// allow-bitmask builder for the CUDA sampler.
//
// The reference (src/core/grammar.c) decides each vocabulary token by copying the committed text
// and the token's piece into a scratch buffer and re-running a prefix validator over all of it
// (:215-233), for every token of every decode step.  Both validators it uses -- a JSON
// brace/bracket balance check (:191-213) and a fixed receipt schema,
// {"bbox_2d": [int, int, int, int], "text_content": "string"} (:67-189) -- only ever fail on a
// character, never on reaching the end of the text.  So each is a per-character state machine:
// the committed text is run through it once per step, and every piece continues from that
// state over its own characters only.  The machines below restate the validators' decisions
// character by character, including their quirks (whitespace may stand in for the ':' of
// "bbox_2d":, a digit right after a number's trailing blanks starts the next number, a quote
// preceded by a backslash does not toggle a string).
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <new>
#include <string>
#include <vector>

#include "grammar.h"

namespace {

constexpr int GRAMMAR_CAP = 8192;  // text capacity; the reference rejects at cap - 1 bytes

inline bool is_space(unsigned char c) { return c == ' ' || (c >= '\t' && c <= '\r'); }
inline bool is_digit(unsigned char c) { return c >= '0' && c <= '9'; }

// ---- JSON prefix: the first non-blank is '{' or '['; outside strings, closing braces and
// brackets never outnumber opening ones (src/core/grammar.c:191-213) ----
struct JsonState {
    bool started = false, in_str = false, has_prev = false;
    int braces = 0, brackets = 0;
    unsigned char prev = 0;
};

inline bool json_step(JsonState &s, unsigned char c) {
    if (!s.started) {
        if (!is_space(c)) {
            if (c != '{' && c != '[') return false;
            s.started = true;
        }
    }
    if (s.started) {
        if (c == '"' && !(s.has_prev && s.prev == '\\')) {
            s.in_str = !s.in_str;
        } else if (!s.in_str) {
            if (c == '{') {
                s.braces++;
            } else if (c == '}') {
                if (--s.braces < 0) return false;
            } else if (c == '[') {
                s.brackets++;
            } else if (c == ']') {
                if (--s.brackets < 0) return false;
            }
        }
    }
    s.prev = c;
    s.has_prev = true;
    return true;
}

// ---- receipt prefix (src/core/grammar.c:67-189) ----
const char KEY1[] = "\"bbox_2d\":";
const char KEY2[] = "\"text_content\":";
constexpr int KEY1_LEN = sizeof(KEY1) - 1, KEY2_LEN = sizeof(KEY2) - 1;

enum : unsigned char {
    R_LEAD,      // blanks, then '{'
    R_KEY1_WS,   // blanks before "bbox_2d":
    R_KEY1,      // matching "bbox_2d": (a blank may stand in for its ':')
    R_LB_WS,     // blanks, then '['
    R_NUM_WS,    // blanks before number `num`
    R_NUM_DIG,   // digits of number `num`
    R_SEP_WS,    // blanks after number `num`, then ',' (or ']' after the fourth)
    R_AFTER_WS,  // blanks, then ','
    R_KEY2_WS,   // blanks before "text_content":
    R_KEY2,      // matching "text_content": exactly
    R_Q_WS,      // blanks, then the opening quote
    R_STR,       // string body until a quote not preceded by a backslash
    R_END_WS,    // blanks, then '}'
    R_TAIL_WS,   // only blanks may follow
};

struct ReceiptState {
    unsigned char st = R_LEAD, k = 0, num = 0;
    bool had = false;
    unsigned char prev = 0;
};

inline bool receipt_step(ReceiptState &s, unsigned char c) {
    for (;;) {
        switch (s.st) {
            case R_LEAD:
                if (is_space(c)) goto take;
                if (c == '{') {
                    s.st = R_KEY1_WS;
                    goto take;
                }
                return false;
            case R_KEY1_WS:
                if (is_space(c)) goto take;
                s.st = R_KEY1;
                s.k = 0;
                continue;
            case R_KEY1:
                if (c == (unsigned char)KEY1[s.k] || (KEY1[s.k] == ':' && is_space(c))) {
                    if (++s.k == KEY1_LEN) s.st = R_LB_WS;
                    goto take;
                }
                return false;
            case R_LB_WS:
                if (is_space(c)) goto take;
                if (c == '[') {
                    s.st = R_NUM_WS;
                    s.num = 0;
                    goto take;
                }
                return false;
            case R_NUM_WS:
                if (is_space(c)) goto take;
                s.st = R_NUM_DIG;
                s.had = false;
                continue;
            case R_NUM_DIG:
                if (is_digit(c)) {
                    s.had = true;
                    goto take;
                }
                if (!s.had && c != ']' && c != ',') return false;
                s.st = R_SEP_WS;
                continue;
            case R_SEP_WS:
                if (is_space(c)) goto take;
                if (s.num < 3) {
                    if (c == ',') {
                        s.num++;
                        s.st = R_NUM_WS;
                        goto take;
                    }
                    if (is_digit(c)) {  // read as the start of the next number
                        s.num++;
                        s.st = R_NUM_DIG;
                        s.had = false;
                        continue;
                    }
                    return false;
                }
                if (c == ']') {
                    s.st = R_AFTER_WS;
                    goto take;
                }
                return false;
            case R_AFTER_WS:
                if (is_space(c)) goto take;
                if (c == ',') {
                    s.st = R_KEY2_WS;
                    goto take;
                }
                return false;
            case R_KEY2_WS:
                if (is_space(c)) goto take;
                s.st = R_KEY2;
                s.k = 0;
                continue;
            case R_KEY2:
                if (c == (unsigned char)KEY2[s.k]) {
                    if (++s.k == KEY2_LEN) s.st = R_Q_WS;
                    goto take;
                }
                return false;
            case R_Q_WS:
                if (is_space(c)) goto take;
                if (c == '"') {
                    s.st = R_STR;
                    goto take;
                }
                return false;
            case R_STR:
                if (c == '"' && s.prev != '\\') s.st = R_END_WS;
                goto take;
            case R_END_WS:
                if (is_space(c)) goto take;
                if (c == '}') {
                    s.st = R_TAIL_WS;
                    goto take;
                }
                return false;
            case R_TAIL_WS:
                if (is_space(c)) goto take;
                return false;
            default:
                return false;
        }
    }
take:
    s.prev = c;
    return true;
}

}  // namespace

struct diskllm_grammar {
    char raw_grammar[GRAMMAR_CAP];
    char buffer[GRAMMAR_CAP];
    int buf_len;
    bool is_json;
    bool is_receipt;
};

struct dllm_grammar_vocab {
    int vocab_size;
    int eos;
    std::vector<int> off, len;  // len -1: no piece
    std::string text;
};

namespace {

// The committed text's state, and whether it is already invalid (then no piece can fix it).
struct Prefix {
    JsonState js;
    ReceiptState rs;
    bool dead = false;
};

Prefix scan_committed(const diskllm_grammar *g) {
    Prefix p;
    for (int i = 0; i < g->buf_len && !p.dead; i++) {
        const unsigned char c = (unsigned char)g->buffer[i];
        if (g->is_receipt) p.dead = !receipt_step(p.rs, c);
        else if (g->is_json) p.dead = !json_step(p.js, c);
    }
    return p;
}

// src/core/grammar.c:215-233 for one piece, continuing from the committed text's state
bool accept_from(const diskllm_grammar *g, const Prefix &p, const char *piece, int plen) {
    if (g->buf_len + plen >= GRAMMAR_CAP - 1) return false;
    if (!g->is_receipt && !g->is_json) return true;
    if (p.dead) return false;
    if (g->is_receipt) {
        ReceiptState s = p.rs;
        for (int i = 0; i < plen; i++)
            if (!receipt_step(s, (unsigned char)piece[i])) return false;
        return true;
    }
    JsonState s = p.js;
    for (int i = 0; i < plen; i++)
        if (!json_step(s, (unsigned char)piece[i])) return false;
    return true;
}

}  // namespace

extern "C" {

DLLM_API diskllm_grammar *diskllm_grammar_init_from_str(const char *grammar_str) {
    if (!grammar_str) return nullptr;
    diskllm_grammar *g = (diskllm_grammar *)calloc(1, sizeof(diskllm_grammar));
    if (!g) return nullptr;
    strncpy(g->raw_grammar, grammar_str, sizeof(g->raw_grammar) - 1);
    g->is_receipt = strstr(grammar_str, "bbox_2d") != nullptr;
    g->is_json = strstr(grammar_str, "object") != nullptr || strstr(grammar_str, "value") != nullptr;
    return g;
}

DLLM_API diskllm_grammar *diskllm_grammar_init_from_file(const char *filepath) {
    if (!filepath) return nullptr;
    FILE *f = fopen(filepath, "rb");
    if (!f) return nullptr;
    std::string text;
    char chunk[4096];
    size_t n;
    while ((n = fread(chunk, 1, sizeof(chunk), f)) > 0) text.append(chunk, n);
    fclose(f);
    return diskllm_grammar_init_from_str(text.c_str());
}

DLLM_API diskllm_grammar *diskllm_grammar_init_json(void) {
    diskllm_grammar *g = diskllm_grammar_init_from_str("root ::= object | array\n");
    if (g) g->is_json = true;
    return g;
}

DLLM_API void diskllm_grammar_free(diskllm_grammar *g) { free(g); }

DLLM_API void diskllm_grammar_reset(diskllm_grammar *g) {
    if (!g) return;
    g->buf_len = 0;
    g->buffer[0] = '\0';
}

DLLM_API bool diskllm_grammar_accept_str(const diskllm_grammar *g, const char *piece) {
    if (!g || !piece) return true;
    return accept_from(g, scan_committed(g), piece, (int)strlen(piece));
}

DLLM_API void diskllm_grammar_advance(diskllm_grammar *g, const char *piece) {
    if (!g || !piece) return;
    const int plen = (int)strlen(piece);
    if (g->buf_len + plen < GRAMMAR_CAP - 1) {
        memcpy(g->buffer + g->buf_len, piece, plen);
        g->buf_len += plen;
        g->buffer[g->buf_len] = '\0';
    }
}

DLLM_API bool diskllm_grammar_is_finished(const diskllm_grammar *g) {
    if (!g || g->buf_len == 0) return false;
    int braces = 0, brackets = 0;
    bool in_str = false;
    for (int i = 0; i < g->buf_len; i++) {
        const char c = g->buffer[i];
        if (c == '"' && (i == 0 || g->buffer[i - 1] != '\\')) in_str = !in_str;
        if (in_str) continue;
        braces += (c == '{') - (c == '}');
        brackets += (c == '[') - (c == ']');
    }
    return braces == 0 && brackets == 0 && !in_str && g->buf_len > 1;
}

DLLM_API int dllm_grammar_build_bitmask(const diskllm_grammar *g, int vocab_size, void *tok_ctx,
                                        const char *(*get_token_str)(void *ctx, int token_id), int eos_token_id,
                                        uint32_t *out_words) {
    if (!out_words || vocab_size <= 0) return vocab_size;
    const int words = (vocab_size + 31) / 32;
    if (!g || !get_token_str) {
        for (int w = 0; w < words; w++) out_words[w] = 0xffffffffu;
        if (vocab_size & 31) out_words[words - 1] = (1u << (vocab_size & 31)) - 1u;
        return vocab_size;
    }
    const bool finished = diskllm_grammar_is_finished(g);
    const Prefix p = scan_committed(g);
    int valid = 0;
    for (int w = 0; w < words; w++) {
        uint32_t bits = 0u;
        const int base = 32 * w;
        for (int b = 0; b < 32 && base + b < vocab_size; b++) {
            const int i = base + b;
            bool ok;
            if (i == eos_token_id) {
                ok = finished;
            } else {
                const char *t = get_token_str(tok_ctx, i);
                ok = t && t[0] != '\0' && accept_from(g, p, t, (int)strlen(t));
            }
            bits |= (uint32_t)ok << b;
            valid += ok;
        }
        out_words[w] = bits;
    }
    return valid;
}

DLLM_API int diskllm_grammar_apply_mask(diskllm_grammar *g, float *logits, int vocab_size, void *tok_ctx,
                                        const char *(*get_token_str)(void *ctx, int token_id), int eos_token_id) {
    if (!g || !logits || vocab_size <= 0 || !get_token_str) return vocab_size;
    std::vector<uint32_t> words((vocab_size + 31) / 32);
    const int valid = dllm_grammar_build_bitmask(g, vocab_size, tok_ctx, get_token_str, eos_token_id, words.data());
    for (int i = 0; i < vocab_size; i++)
        if (!((words[i >> 5] >> (i & 31)) & 1u)) logits[i] = -INFINITY;
    return valid;
}

DLLM_API dllm_grammar_vocab *dllm_grammar_vocab_create(int vocab_size, void *tok_ctx,
                                                       const char *(*get_token_str)(void *ctx, int token_id),
                                                       int eos_token_id) {
    if (vocab_size <= 0 || !get_token_str) return nullptr;
    dllm_grammar_vocab *v = new (std::nothrow) dllm_grammar_vocab;
    if (!v) return nullptr;
    v->vocab_size = vocab_size;
    v->eos = eos_token_id;
    v->off.resize(vocab_size);
    v->len.resize(vocab_size);
    for (int i = 0; i < vocab_size; i++) {
        const char *t = i == eos_token_id ? nullptr : get_token_str(tok_ctx, i);
        v->off[i] = (int)v->text.size();
        v->len[i] = t ? (int)strlen(t) : -1;
        if (t) v->text.append(t, v->len[i]);
    }
    return v;
}

DLLM_API void dllm_grammar_vocab_free(dllm_grammar_vocab *v) { delete v; }

DLLM_API int dllm_grammar_build_bitmask_cached(const diskllm_grammar *g, const dllm_grammar_vocab *v,
                                               uint32_t *out_words) {
    if (!v || !out_words) return 0;
    const int V = v->vocab_size, words = (V + 31) / 32;
    if (!g) {
        for (int w = 0; w < words; w++) out_words[w] = 0xffffffffu;
        if (V & 31) out_words[words - 1] = (1u << (V & 31)) - 1u;
        return V;
    }
    const bool finished = diskllm_grammar_is_finished(g);
    const Prefix p = scan_committed(g);
    const char *text = v->text.data();
    int valid = 0;
    for (int w = 0; w < words; w++) {
        uint32_t bits = 0u;
        const int base = 32 * w;
        for (int b = 0; b < 32 && base + b < V; b++) {
            const int i = base + b;
            bool ok;
            if (i == v->eos) ok = finished;
            else ok = v->len[i] > 0 && accept_from(g, p, text + v->off[i], v->len[i]);
            bits |= (uint32_t)ok << b;
            valid += ok;
        }
        out_words[w] = bits;
    }
    return valid;
}

}  // extern "C"
