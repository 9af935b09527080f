"""Tokenizer and chat-template parity with the reference FISH engine, on the
CPU. The reference, compiled here from its own sources (oracle/_ref), loads
the same synthetic GGUF with fish_load (its CPU engine) and tokenizes,
detokenizes and formats chat prompts through its own C API
(model/fish/include/fish/c_api.h:108-121); this library does the same from
the GGUF's metadata through the host-only fbx_*_gguf entry points, which
build the tokenizer fish_load builds. The synthetic vocabulary is
SentencePiece-style (<unk> <s> </s>, 256 byte tokens, then "▁t<i>" pieces),
so the cases exercise byte fallback, the space prefix, BOS, special-token
text and the pieces that do match. The chat cases cover every format the
reference detects, from files carrying a template with that format's
marker."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from imurun_b200 import native

P, I, CP = ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p
TEXTS = ["Hello world", "  leading spaces", "tabs\tand\nnewlines", "héllo 世界 \U0001f642", "",
         "<s>hi</s>", "t300 t1000 t31999", "a", " ", "x" * 300]
CHATS = [[("system", "Be brief."), ("user", "Hi there"), ("assistant", "Hello!"), ("user", "t300?")],
         [("user", "éè and <s> tags")]]


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


@pytest.fixture(scope="module", params=["tiny", "qwen7b"])
def gguf(request, synth_dir):
    from imurun_b200 import synth
    cfg = synth.preset("tiny") if request.param == "tiny" else synth.preset("qwen7b", layers=1)
    return synth.cached(cfg, synth_dir)


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
