"""Tokenizer and chat-template parity with the reference FISH engine, on the
CPU. The reference, compiled here from its own sources (oracle/_ref), loads
the same synthetic GGUF with fish_load (its CPU engine) and tokenizes,
detokenizes and formats chat prompts through its own C API
(model/fish/include/fish/c_api.h:108-121); this library does the same from
the GGUF's metadata through the host-only fbx_*_gguf entry points, which
build the tokenizer fish_load builds. Two vocabularies: SentencePiece-style
(<unk> <s> </s>, 256 byte tokens, then "▁t<i>" pieces: byte fallback, the
space prefix, BOS, special-token text and the pieces that do match), and
byte-level BPE (256 byte characters, 400 merges learned from a built-in text,
control tokens) under the llama3 and qwen2 pre-splits, where seeded random
strings over a mix of letters, digits, contractions, punctuation, whitespace
kinds, non-Latin scripts, emoji, special-token text and malformed UTF-8
exercise every pre-split rule and the merge order. The chat cases cover
every format the reference detects, from files carrying a template with
that format's marker."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from imurun_b200 import native

P, I, CP = ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p
TEXTS = ["Hello world", "  leading spaces", "tabs\tand\nnewlines", "héllo 世界 \U0001f642", "",
         "<s>hi</s>", "t300 t1000 t31999", "a", " ", "x" * 300]
CHATS = [[("system", "Be brief."), ("user", "Hi there"), ("assistant", "Hello!"), ("user", "t300?")],
         [("user", "éè and <s> tags")],
         # tool results, two system turns, an empty turn, a role no format
         # names, and a conversation that ends on the assistant
         [("system", "Tools: lookup"), ("user", "find t17"), ("assistant", "calling lookup"),
          ("tool", "{\"t17\": 4}"), ("user", "and?")],
         [("system", "one"), ("system", "two"), ("user", ""), ("function", "raw"), ("assistant", "ok")],
         [("system", "only a system turn")]]


@pytest.fixture(scope="module")
def ref_lib():
    from oracle.binding import REF_SO
    if not REF_SO.exists():
        pytest.skip("reference build (oracle/_ref) not present")
    L = ctypes.CDLL(str(REF_SO))
    L.fish_create.restype = P
    L.fish_destroy.argtypes = [P]
    L.fish_load.argtypes = [P, CP, I]
    L.fish_load.restype = I
    L.fish_tokenize.argtypes = [P, CP, I, P, I]
    L.fish_tokenize.restype = I
    L.fish_detokenize.argtypes = [P, P, I, ctypes.c_char_p, I]
    L.fish_detokenize.restype = I
    L.fish_chat_prompt.argtypes = [P, P, P, I, ctypes.c_char_p, I]
    L.fish_chat_prompt.restype = I
    L.fish_count_chat_tokens.argtypes = [P, P, P, I]
    L.fish_count_chat_tokens.restype = I
    L.fish_chat_format.argtypes = [P]
    L.fish_chat_format.restype = ctypes.c_char_p
    return L


@pytest.fixture(scope="module")
def ours():
    L = native.load_library()
    L.fbx_tokenize_gguf.argtypes = [CP, CP, I, P, I]
    L.fbx_tokenize_gguf.restype = I
    L.fbx_detokenize_gguf.argtypes = [CP, P, I, ctypes.c_char_p, I]
    L.fbx_detokenize_gguf.restype = I
    L.fbx_chat_prompt_gguf.argtypes = [CP, P, P, I, ctypes.c_char_p, I]
    L.fbx_chat_prompt_gguf.restype = I
    L.fbx_chat_info_gguf.argtypes = [CP, P, P, I, ctypes.c_char_p, I]
    L.fbx_chat_info_gguf.restype = I
    return L


GGUFS = {
    "tiny": lambda synth: synth.preset("tiny"),
    "qwen7b": lambda synth: synth.preset("qwen7b", layers=1),
    "bpe-llama3": lambda synth: synth.preset("tiny", layers=1, bpe_pre="llama-bpe"),
    "bpe-qwen2": lambda synth: synth.preset("tiny", layers=1, bpe_pre="qwen2"),
    # the GPT-2 family (digit runs of any length) and a pre-tokenizer name
    # the reference does not list (its default split)
    "bpe-gpt2": lambda synth: synth.preset("tiny", layers=1, bpe_pre="gpt-2"),
    "bpe-unlisted": lambda synth: synth.preset("tiny", layers=1, bpe_pre="not-a-listed-pre"),
    # a file that asks for no BOS (tokenizer.ggml.add_bos_token false, as
    # Qwen's do): chat prompts and counts start without one
    "bpe-qwen2-nobos": lambda synth: synth.preset("tiny", layers=1, bpe_pre="qwen2", no_bos=1),
}


@pytest.fixture(scope="module", params=list(GGUFS))
def gguf(request, synth_dir):
    from imurun_b200 import synth
    return synth.cached(GGUFS[request.param](synth), synth_dir)


# pieces the fuzz strings are drawn from
PARTS = ["the", "The", "THE", "quick", "hello", "world", "running", " ", "  ", "   ", "\t", "\n", "\n\n", "\r\n",
         " \n ", "'s", "'T", "'re", "'VE", "'m", "'ll", "'d", "'x", "'", "0", "7", "42", "2024", "123456789", "3.14",
         "1,000", ".", "...", "!", "?!", "--", "(", ")", "{", "}", "**", "_", "-", "café", "naïve", "straße", "Привет",
         "日本語", "テスト", "٣٤٥", "१२३", "²³", "½", "\u00a0", "\u3000", "\u1680", "\u2003", "\u0085", "🙂", "👍🏽",
         "<|im_start|>", "<|eot_id|>", "<|begin_of_text|>", "<s>", "</s>", "<|end_header_id|>", "é", "ß", "×", "÷"]


def _fuzz_texts(seed, n):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        parts = [PARTS[int(i)] for i in rng.integers(0, len(PARTS), int(rng.integers(1, 14)))]
        t = "".join(parts).encode("utf-8")
        if rng.random() < 0.2:          # malformed UTF-8: a stray lead or continuation byte
            k = int(rng.integers(0, len(t) + 1))
            t = t[:k] + bytes([int(rng.choice([0xC3, 0xE6, 0xF0, 0x80, 0xBF, 0xFF]))]) + t[k:]
        out.append(t)
    return out


@pytest.mark.parametrize("seed", range(2))
def test_tokenize_fuzz_matches_reference(ref_lib, ours, ref_ctx, gguf, seed):
    for t in _fuzz_texts(1000 + seed, 30):
        for bos in (0, 1):
            want = _tok(ref_lib.fish_tokenize, ref_ctx, text=t, bos=bos)
            got = _tok(ours.fbx_tokenize_gguf, str(gguf).encode(), text=t, bos=bos)
            assert np.array_equal(got, want), (t, list(got), list(want))
        ids = np.ascontiguousarray(want, np.int32)
        assert _str(ours.fbx_detokenize_gguf, str(gguf).encode(), ids.ctypes.data, ids.size) == \
            _str(ref_lib.fish_detokenize, ref_ctx, ids.ctypes.data, ids.size)


@pytest.fixture(scope="module")
def ref_ctx(ref_lib, gguf):
    ctx = ref_lib.fish_create()
    assert ref_lib.fish_load(ctx, str(gguf).encode(), 512) == 0
    yield ctx
    ref_lib.fish_destroy(ctx)


def _tok(fn, *head, text: bytes, bos: int):
    n = fn(*head, text, bos, None, 0)
    assert n >= 0
    out = np.zeros(max(n, 1), np.int32)
    assert fn(*head, text, bos, out.ctypes.data, out.size) == n
    return out[:n]


def _str(fn, *args):
    n = fn(*args, None, 0)
    assert n >= 0
    buf = ctypes.create_string_buffer(n + 1)
    assert fn(*args, buf, n + 1) == n
    return buf.raw[:n]


def _chat_args(msgs):
    roles = (ctypes.c_char_p * len(msgs))(*[r.encode() for r, _ in msgs])
    contents = (ctypes.c_char_p * len(msgs))(*[c.encode() for _, c in msgs])
    return ctypes.cast(roles, P), ctypes.cast(contents, P), len(msgs)


@pytest.mark.parametrize("text", TEXTS)
@pytest.mark.parametrize("bos", [0, 1])
def test_tokenize_matches_reference(ref_lib, ours, ref_ctx, gguf, text, bos):
    t = text.encode()
    want = _tok(ref_lib.fish_tokenize, ref_ctx, text=t, bos=bos)
    got = _tok(ours.fbx_tokenize_gguf, str(gguf).encode(), text=t, bos=bos)
    assert np.array_equal(got, want), (list(got), list(want))
    # detokenising the ids gives the reference's text, byte for byte
    ids = np.ascontiguousarray(want, np.int32)
    assert _str(ours.fbx_detokenize_gguf, str(gguf).encode(), ids.ctypes.data, ids.size) == \
        _str(ref_lib.fish_detokenize, ref_ctx, ids.ctypes.data, ids.size)


@pytest.mark.parametrize("k", range(len(CHATS)))
def test_chat_prompt_matches_reference(ref_lib, ours, ref_ctx, gguf, k):
    args = _chat_args(CHATS[k])
    assert _str(ours.fbx_chat_prompt_gguf, str(gguf).encode(), *args) == _str(ref_lib.fish_chat_prompt, ref_ctx, *args)


@pytest.mark.parametrize("k", range(len(CHATS)))
def test_chat_count_and_format_match_reference(ref_lib, ours, ref_ctx, gguf, k):
    args = _chat_args(CHATS[k])
    fmt = ctypes.create_string_buffer(64)
    n = ours.fbx_chat_info_gguf(str(gguf).encode(), *args, fmt, 64)
    assert n == ref_lib.fish_count_chat_tokens(ref_ctx, *args) > 0
    assert fmt.value == ref_lib.fish_chat_format(ref_ctx)


# Minimal templates carrying the marker each chat format is detected by
# (model/fish/src/tokenizer.cpp:274-288); "" writes no template.
TEMPLATES = {
    "plain": "",
    "llama3": "{{ '<|start_header_id|>' + role + '<|end_header_id|>' + content }}",
    "chatml": "{{ '<|im_start|>' + role + content }}",
    "gemma": "{{ '<start_of_turn>' + role + content }}",
    "phi3": "{{ '<|user|>' + content + '<|end|>' }}",
    "deepseek": "{{ '<\uff5cUser\uff5c>' + content }}",
    "mistral": "{{ '[INST] ' + content + ' [/INST]' }}",
}


@pytest.mark.parametrize("name", list(TEMPLATES))
def test_chat_formats_match_reference(ref_lib, ours, synth_dir, name):
    from imurun_b200 import synth
    path = synth.cached(synth.preset("tiny", layers=1, chat_template=TEMPLATES[name]), synth_dir)
    ctx = ref_lib.fish_create()
    try:
        assert ref_lib.fish_load(ctx, str(path).encode(), 256) == 0
        assert ref_lib.fish_chat_format(ctx) == name.encode()
        fmt = ctypes.create_string_buffer(64)
        for msgs in CHATS:
            args = _chat_args(msgs)
            assert _str(ours.fbx_chat_prompt_gguf, str(path).encode(), *args) == _str(ref_lib.fish_chat_prompt, ctx, *args)
            assert ours.fbx_chat_info_gguf(str(path).encode(), *args, fmt, 64) == \
                ref_lib.fish_count_chat_tokens(ctx, *args)
            assert fmt.value == name.encode()
    finally:
        ref_lib.fish_destroy(ctx)


def test_unreadable_file(ours):
    assert ours.fbx_tokenize_gguf(b"/nonexistent.gguf", b"hi", 1, None, 0) == -1


def test_detokenize_edge_ids_match_reference(ref_lib, ours, ref_ctx, gguf):
    """Ids the vocabulary does not hold (negative, past the end), control
    tokens, byte tokens that do not form UTF-8, and an empty list: the same
    bytes (or the same refusal) as the reference's fish_detokenize."""
    vocab = 32000
    cases = [[], [1], [2], [0], [-1], [vocab], [vocab + 5], [3, 4, 5], [3 + 0xC3], [3 + 0xE6, 3 + 0x97],
             [1, 300, 2, 301], [259, -7, 260]]
    for ids in cases:
        a = np.ascontiguousarray(ids if ids else [0], np.int32)
        n = len(ids)
        want = ref_lib.fish_detokenize(ref_ctx, a.ctypes.data, n, None, 0)
        got = ours.fbx_detokenize_gguf(str(gguf).encode(), a.ctypes.data, n, None, 0)
        assert (got < 0) == (want < 0), (ids, got, want)
        if want >= 0:
            assert _str(ours.fbx_detokenize_gguf, str(gguf).encode(), a.ctypes.data, n) == \
                _str(ref_lib.fish_detokenize, ref_ctx, a.ctypes.data, n), ids
