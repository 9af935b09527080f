"""UTF-8 streaming parity with the reference FISH engine, on the CPU. The
reference, compiled here from its own sources (oracle/_ref), generates
greedily with fish_generate on a synthetic GGUF and reports every token
callback: the text chunk and its token id. Its emitter holds back a UTF-8
lead byte until the sequence is complete, so a chunk can carry several
tokens' bytes, and what is left at the end is flushed with id -1
(model/fish/src/c_api.cpp:81-101, 774-779). The ids it generated are
recomputed with the reference's own model (greedy: the first index of the
largest logit, stopping at end of sequence, max_tokens or the context), and
this library's emitter (fbx_stream_gguf: the generation loop's emit_utf8 and
flush over the GGUF tokenizer's token texts) must give the same callbacks,
byte for byte and id for id. The synthetic vocabulary has all 256 byte
tokens, so random-init models emit lead bytes and merged chunks occur."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from imurun_b200 import native

P, I, CP, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_float
CB = ctypes.CFUNCTYPE(None, ctypes.c_char_p, ctypes.c_int, ctypes.c_void_p)
N_CTX, MAX_TOKENS, EOS = 512, 300, 2
# (prompt words, seed): two streams of whole characters, and three in which
# lead bytes are held back and merged (1, 1 and 12 merged tokens)
CASES = [(12, 0), (12, 1), (12, 5), (3, 7), (30, 5)]


@pytest.fixture(scope="module")
def ref():
    from oracle.binding import REF_SO, Reference
    if not REF_SO.exists():
        pytest.skip("reference build (oracle/_ref) not present")
    r = Reference()
    L = r.L
    L.fish_create.restype = P
    L.fish_destroy.argtypes = [P]
    L.fish_load.argtypes = [P, CP, I]
    L.fish_load.restype = I
    L.fish_tokenize.argtypes = [P, CP, I, P, I]
    L.fish_tokenize.restype = I
    L.fish_generate.argtypes = [P, CP, I, I, F, I, F, F, CB, P]
    L.fish_generate.restype = I
    L.fish_get_stats.argtypes = [P, P]
    r.set_threads(4)
    return r


@pytest.fixture(scope="module")
def ours():
    L = native.load_library()
    L.fbx_stream_gguf.argtypes = [CP, P, I, ctypes.c_char_p, I]
    L.fbx_stream_gguf.restype = I
    return L


@pytest.fixture(scope="module")
def tiny(synth_dir):
    from imurun_b200 import synth
    return synth.cached(synth.preset("tiny", layers=1), synth_dir)


def _parse(rec: bytes):
    out, i = [], 0
    while i < len(rec):
        nl = rec.index(b"\n", i)
        tid, n = (int(v) for v in rec[i:nl].split(b" "))
        out.append((tid, rec[nl + 1:nl + 1 + n]))
        i = nl + 1 + n
    return out


def _ours(L, path, ids):
    ids = np.ascontiguousarray(ids, np.int32)
    n = L.fbx_stream_gguf(str(path).encode(), ids.ctypes.data, ids.size, None, 0)
    assert n >= 0
    buf = ctypes.create_string_buffer(n + 1)
    assert L.fbx_stream_gguf(str(path).encode(), ids.ctypes.data, ids.size, buf, n + 1) == n
    return _parse(buf.raw[:n])


def test_stream_matches_reference(ref, ours, tiny):
    from imurun_b200.native import FishStats
    L = ref.L
    model = ref.load(tiny, N_CTX)
    merged = 0
    try:
        for n_words, seed in CASES:
            rng = np.random.default_rng(seed)
            text = " ".join(f"t{int(v)}" for v in rng.integers(300, 31000, n_words)).encode()
            ctx = L.fish_create()
            try:
                assert L.fish_load(ctx, str(tiny).encode(), N_CTX) == 0
                chunks = []

                @CB
                def cb(piece, tid, user):
                    chunks.append((tid, piece))

                assert L.fish_generate(ctx, text, 1, MAX_TOKENS, 0.0, 0, 1.0, 1.0, cb, None) >= 0
                st = FishStats()
                L.fish_get_stats(ctx, ctypes.byref(st))
                n = L.fish_tokenize(ctx, text, 1, None, 0)
                ids = np.zeros(n, np.int32)
                assert L.fish_tokenize(ctx, text, 1, ids.ctypes.data, n) == n
            finally:
                L.fish_destroy(ctx)
            # the same greedy decode on the reference's own model
            model.reset()
            logits, pos, gen = model.prefill(ids), n, []
            while len(gen) < MAX_TOKENS and pos < N_CTX:
                nxt = int(np.argmax(logits))
                if nxt == EOS:
                    break
                gen.append(nxt)
                logits = model.forward(np.array([nxt], np.int32), pos)
                pos += 1
            assert len(gen) == st.generated_tokens, (seed, len(gen), st.generated_tokens)
            got = _ours(ours, tiny, gen)
            assert got == chunks, (seed, next(i for i, (a, b) in enumerate(zip(got, chunks)) if a != b)
                                   if any(a != b for a, b in zip(got, chunks)) else (len(got), len(chunks)))
            merged += len(gen) - len(chunks)
    finally:
        model.close()
    assert merged > 0   # some chunks carried several tokens' bytes


def test_stream_edges(ours, tiny):
    # a lone lead byte is flushed at the end with id -1; an empty stream sends nothing
    lead = 3 + 0xE3     # byte tokens follow <unk> <s> </s>
    assert _ours(ours, tiny, [lead]) == [(-1, bytes([0xE3]))]
    assert _ours(ours, tiny, []) == []
    # a complete three-byte character split over three byte tokens arrives once, with the last id
    euro = [3 + b for b in "€".encode()]
    assert _ours(ours, tiny, euro) == [(euro[-1], "€".encode())]
    assert ours.fbx_stream_gguf(b"/nonexistent.gguf", None, 0, None, 0) == -1
