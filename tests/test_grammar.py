"""The grammar constraint (include/grammar.h) and its bitmask builder, against DiskLLM's own
src/core/grammar.c compiled from the reference sources (oracle/_ref/libref_asbuilt.so):
accept_str / is_finished on randomised JSON and receipt texts split at random points, and
dllm_grammar_build_bitmask against diskllm_grammar_apply_mask's -INFINITY pattern on random
vocabularies.  The reference's own tools/test_grammar_unit.c assertions run on this library too.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest

import oracle as O
from diskllm_b200 import capi

RECEIPT_GBNF = ('root ::= "{" ws "\\"bbox_2d\\":" ws "[" ws int "]" ws "}"\n'
                'int ::= [0-9]+\nws ::= [ \\t\\n\\r]*\n')
JSON_GBNF = "root ::= object | array\n"


def _ref_lib():
    lib = C.CDLL(O.REF_ASBUILT_SO)
    lib.diskllm_grammar_init_from_str.restype = C.c_void_p
    lib.diskllm_grammar_init_from_str.argtypes = [C.c_char_p]
    lib.diskllm_grammar_free.argtypes = [C.c_void_p]
    lib.diskllm_grammar_reset.argtypes = [C.c_void_p]
    lib.diskllm_grammar_accept_str.restype = C.c_bool
    lib.diskllm_grammar_accept_str.argtypes = [C.c_void_p, C.c_char_p]
    lib.diskllm_grammar_advance.argtypes = [C.c_void_p, C.c_char_p]
    lib.diskllm_grammar_is_finished.restype = C.c_bool
    lib.diskllm_grammar_is_finished.argtypes = [C.c_void_p]
    lib.diskllm_grammar_apply_mask.restype = C.c_int
    lib.diskllm_grammar_apply_mask.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, capi.TOKEN_STR_CB,
                                               C.c_int]
    return lib


def test_reference_unit_test_assertions_hold():
    """tools/test_grammar_unit.c:8-26 on this library"""
    g = capi.Grammar(RECEIPT_GBNF)
    assert g.accept(b"{")
    g.advance(b"{")
    assert g.accept(b'"bbox_2d":')
    assert not g.accept(b"invalid")
    g.advance(b'"bbox_2d": [123] }')
    assert g.finished()


def _receipt_texts(rng, n):
    base = '{"bbox_2d": [12, 340, 5, 6789], "text_content": "a \\"b\\" c"}'
    specials = list(' \t\n{}[],:"\\0123456789abx_')
    out = []
    for _ in range(n):
        s = list(base)
        for _ in range(rng.integers(0, 4)):  # mutations
            op = rng.integers(0, 3)
            pos = int(rng.integers(0, len(s) + 1))
            ch = specials[int(rng.integers(0, len(specials)))]
            if op == 0 and s:
                s[min(pos, len(s) - 1)] = ch
            elif op == 1:
                s.insert(pos, ch)
            elif s:
                del s[min(pos, len(s) - 1)]
        t = "".join(s)
        out.append(t[: int(rng.integers(0, len(t) + 1))])
    return out


def _json_texts(rng, n):
    alphabet = list(' {}[]"\\:,a1\n')
    out = []
    for _ in range(n):
        L = int(rng.integers(0, 24))
        t = "".join(alphabet[int(i)] for i in rng.integers(0, len(alphabet), L))
        if rng.random() < 0.6:
            t = ("  " if rng.random() < 0.3 else "") + rng.choice(["{", "["]) + t
        out.append(t)
    return out


@pytest.mark.parametrize("kind", ["receipt", "json", "plain"])
def test_accept_and_finished_match_reference(have_reference, kind):
    ref = _ref_lib()
    rng = np.random.default_rng({"receipt": 1, "json": 2, "plain": 3}[kind])
    text = {"receipt": RECEIPT_GBNF, "json": JSON_GBNF, "plain": "root ::= [a-z]+"}[kind]
    texts = _receipt_texts(rng, 3000) if kind == "receipt" else _json_texts(rng, 3000)
    ours = capi.Grammar(text)
    rg = ref.diskllm_grammar_init_from_str(text.encode())
    try:
        for t in texts:
            b = t.encode()
            cut = int(rng.integers(0, len(b) + 1))
            ours.reset()
            ref.diskllm_grammar_reset(rg)
            ours.advance(b[:cut])
            ref.diskllm_grammar_advance(rg, b[:cut])
            assert ours.accept(b[cut:]) == bool(ref.diskllm_grammar_accept_str(rg, b[cut:])), (kind, t, cut)
            assert ours.finished() == bool(ref.diskllm_grammar_is_finished(rg)), (kind, t, cut)
    finally:
        ref.diskllm_grammar_free(rg)


@pytest.mark.parametrize("kind", ["receipt", "json"])
def test_bitmask_matches_reference_apply_mask(have_reference, kind):
    ref = _ref_lib()
    rng = np.random.default_rng(10 + (kind == "json"))
    text = RECEIPT_GBNF if kind == "receipt" else JSON_GBNF
    alphabet = list(' \t{}[],:"\\0123456789abtx_e')
    V = 5000
    pieces = []
    for i in range(V):
        r = rng.random()
        if r < 0.02:
            pieces.append(None)
        elif r < 0.04:
            pieces.append(b"")
        else:
            L = int(rng.integers(1, 6))
            pieces.append("".join(alphabet[int(j)] for j in rng.integers(0, len(alphabet), L)).encode())
    eos = 17
    prefixes = _receipt_texts(rng, 40) if kind == "receipt" else _json_texts(rng, 40)
    ours = capi.Grammar(text)
    vocab = capi.GrammarVocab(pieces, eos)
    rg = ref.diskllm_grammar_init_from_str(text.encode())
    cb, keep = capi._pieces_callback(pieces)
    try:
        for pre in prefixes + ["", '{"bbox_2d": [1,2,3,4], "text_content": "x"}', "{}", "[[]]"]:
            ours.reset()
            ref.diskllm_grammar_reset(rg)
            ours.advance(pre.encode())
            ref.diskllm_grammar_advance(rg, pre.encode())
            logits = np.zeros(V, dtype=np.float32)
            n_ref = ref.diskllm_grammar_apply_mask(rg, logits.ctypes.data, V, None, cb, eos)
            allowed_ref = np.isfinite(logits)
            words, n = ours.bitmask(pieces, eos)
            bits = ((words[np.arange(V) >> 5] >> (np.arange(V) & 31).astype(np.uint32)) & 1).astype(bool)
            np.testing.assert_array_equal(bits, allowed_ref, err_msg=repr(pre))
            assert n == n_ref
            words2, n2 = vocab.bitmask(ours)
            np.testing.assert_array_equal(words2, words)
            assert n2 == n
            lg2 = np.zeros(V, dtype=np.float32)
            assert ours.apply_mask(lg2, pieces, eos) == n_ref
            np.testing.assert_array_equal(np.isfinite(lg2), allowed_ref)
    finally:
        ref.diskllm_grammar_free(rg)


def test_bitmask_bits_past_vocab_are_clear_and_null_grammar_allows_all():
    pieces = [b"{", b"}", b"a"] * 11  # 33 tokens: two words
    g = capi.Grammar(JSON_GBNF)
    words, n = g.bitmask(pieces, eos=-1)
    assert words.shape == (2,) and int(words[1]) >> 1 == 0
    lib = capi._grammar_lib()
    out = np.zeros(2, dtype=np.uint32)
    cb, keep = capi._pieces_callback(pieces)
    assert lib.dllm_grammar_build_bitmask(None, 33, None, cb, -1, out.ctypes.data) == 33
    assert int(out[0]) == 0xffffffff and int(out[1]) == 1


def test_length_cap_rejects_like_the_reference():
    g = capi.Grammar(JSON_GBNF)
    g.advance(b"[" + b"a" * 8185)  # 8186 bytes committed
    assert g.accept(b"abcd")       # 8190 < 8191
    assert not g.accept(b"abcde")  # 8191
    g.advance(b"abcdef")           # dropped (would reach 8192)
    assert g.accept(b"abcd")
