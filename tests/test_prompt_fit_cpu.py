"""Prompt fit and prefix-cache parity with the reference FISH engine, on the
CPU. The reference, compiled here from its own sources (oracle/_ref), runs
fish_generate on a synthetic GGUF with its CPU engine over a scripted series
of turns: prompts below the budget, over-long prompts (head + tail cut),
chat-like growth that keeps the previous cut, repeats of the same prompt,
and short unrelated prompts. After every turn its fish_stats say what it
decided (prompt_tokens kept, truncated, cached_tokens served by the KV
prefix cache, model/fish/src/c_api.cpp:516-567 and 784-786). This library
makes the same decisions in fb::fit_prompt / fb::cached_prefix, which its
generation loop calls and the host-only fbx_prompt_plan exposes; the test
feeds it the same token ids (the reference's tokenizer) and, after each turn,
the cache contents the reference leaves: the kept prompt and every generated
token (reported through the token callback)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from imurun_b200 import native

P, I, CP, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_float
CB = ctypes.CFUNCTYPE(None, ctypes.c_char_p, ctypes.c_int, ctypes.c_void_p)


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
    L.fish_generate.argtypes = [P, CP, I, I, F, I, F, F, CB, P]
    L.fish_generate.restype = I
    L.fish_get_stats.argtypes = [P, P]
    L.fish_reset.argtypes = [P]
    L.fish_set_threads.argtypes = [P, I]
    return L


@pytest.fixture(scope="module")
def ours():
    L = native.load_library()
    L.fbx_prompt_state_create.restype = P
    L.fbx_prompt_state_destroy.argtypes = [P]
    L.fbx_prompt_plan.argtypes = [P, P, I, I, I, P, I, P, P]
    L.fbx_prompt_plan.restype = I
    L.fbx_prompt_commit.argtypes = [P, P, I]
    L.fbx_prompt_commit.restype = I
    return L


@pytest.fixture(scope="module")
def tiny(synth_dir):
    from imurun_b200 import synth
    return synth.cached(synth.preset("tiny", layers=1), synth_dir)


def _words(rng, n):
    return " ".join(f"t{int(v)}" for v in rng.integers(300, 31000, n))


class _Turns:
    """One reference context and one planner state, advanced together."""

    def __init__(self, ref, ours, path, n_ctx):
        self.ref, self.ours, self.n_ctx = ref, ours, n_ctx
        self.ctx = ref.fish_create()
        assert ref.fish_load(self.ctx, str(path).encode(), n_ctx) == 0
        self.state = ours.fbx_prompt_state_create()
        self.seen = []
        self.merged = 0

    def close(self):
        self.ref.fish_destroy(self.ctx)
        self.ours.fbx_prompt_state_destroy(self.state)

    def tokenize(self, text):
        n = self.ref.fish_tokenize(self.ctx, text.encode(), 1, None, 0)
        ids = np.zeros(n, np.int32)
        assert self.ref.fish_tokenize(self.ctx, text.encode(), 1, ids.ctypes.data, n) == n
        return ids

    def turn(self, text, max_tokens):
        """Runs one reference turn, checks the planner against its stats, and
        returns the text generated (to build the next chat-like prompt)."""
        ids = self.tokenize(text)
        gen, pieces = [], []

        @CB
        def cb(piece, tid, user):
            gen.append(tid)
            pieces.append(piece)

        from imurun_b200.native import FishStats
        assert self.ref.fish_generate(self.ctx, text.encode(), 1, max_tokens, 0.0, 0, 1.0, 1.0, cb, None) >= 0
        st = FishStats()
        self.ref.fish_get_stats(self.ctx, ctypes.byref(st))
        kept = np.zeros(ids.size, np.int32)
        cached, trunc = I(), I()
        nk = self.ours.fbx_prompt_plan(self.state, ids.ctypes.data, ids.size, self.n_ctx, max_tokens,
                                       kept.ctypes.data, kept.size, ctypes.byref(cached), ctypes.byref(trunc))
        got = (nk, cached.value, trunc.value)
        want = (st.prompt_tokens, st.cached_tokens, st.truncated)
        assert got == want, (len(self.seen), ids.size, got, want)
        self.seen.append(want)
        # every generated token was fed back and is in the reference's cache;
        # when the callback reported each by id the planner gets the same
        # cache, otherwise (a UTF-8 lead byte held back and merged into a later
        # chunk, or never sent) both caches start empty (the cut is kept)
        if st.generated_tokens == len(gen) and min(gen, default=0) >= 0:
            cache = np.ascontiguousarray(np.concatenate([kept[:nk], np.asarray(gen, np.int32)]), np.int32)
            assert self.ours.fbx_prompt_commit(self.state, cache.ctypes.data, cache.size) == 0
        else:
            self.merged += 1
            self.reset()
        return b"".join(pieces).decode("utf-8", "replace")

    def reset(self):
        self.ref.fish_reset(self.ctx)
        empty = np.zeros(1, np.int32)
        assert self.ours.fbx_prompt_commit(self.state, empty.ctypes.data, 0) == 0


def _budget(n_ctx, max_tokens):
    mt = n_ctx if max_tokens <= 0 else max_tokens
    return max(32, n_ctx - max(64, min(mt, n_ctx // 4)))


# reserve = max(64, min(max_tokens, n_ctx / 4)): 64 from the floor, 100 from
# max_tokens, 96 from n_ctx / 4 (max_tokens <= 0 reads as n_ctx)
@pytest.mark.parametrize("n_ctx,max_tokens", [(256, 3), (512, 100), (384, 0), (384, 200)])
def test_prompt_fit_and_prefix_match_reference(ref_lib, ours, tiny, n_ctx, max_tokens):
    rng = np.random.default_rng(n_ctx * 7 + max_tokens)
    ref_lib.fish_set_threads(None, 4)
    t = _Turns(ref_lib, ours, tiny, n_ctx)
    reused = 0
    try:
        system = _words(rng, 40)
        # below the budget, then the same prompt again (cache serves n - 1)
        t.turn(system, max_tokens)
        t.turn(system, max_tokens)
        # chat-like growth under the budget: previous prompt + answer + new words
        text = system
        for k in range(2):
            out = t.turn(text, 3)
            text = text + out + " " + _words(rng, 25 + 5 * k)
        # over-long: a new cut, then growth that keeps the same cut until it no
        # longer fits and a new cut is made; turns alternate between this case's
        # max_tokens and 3 (a short answer, and a budget that changes between turns)
        text = system + " " + _words(rng, n_ctx)
        for k in range(10):
            mt = max_tokens if k % 2 else 3
            out = t.turn(text, mt)
            _, c, tr = t.seen[-1]
            reused += bool(tr and c > _budget(n_ctx, mt) // 4)   # served past the head: the cut was kept
            text = text + out + " " + _words(rng, 2)    # about 16 tokens
        # a short unrelated prompt (no cache below 8 tokens, the cut is dropped),
        # the long prompt again (a fresh cut), a reset, and the long prompt once more
        t.turn("t301 t302 t303", max_tokens)
        t.turn(text, max_tokens)
        t.reset()
        t.turn(text, max_tokens)
    finally:
        t.close()
    truncs = [s[2] for s in t.seen]
    cached = [s[1] for s in t.seen]
    assert any(truncs) and not all(truncs)          # both branches of the fit ran
    assert max(cached) >= 8 and 0 in cached[1:]     # the cache served turns, and declined some
    assert reused > 0, t.seen                       # a cut was applied again to a longer prompt


def test_prompt_plan_arguments(ours):
    s = ours.fbx_prompt_state_create()
    try:
        ids = np.arange(3, 403, dtype=np.int32)
        kept = np.zeros(8, np.int32)
        c, tr = I(), I()
        # the kept prompt does not fit a buffer of 8
        assert ours.fbx_prompt_plan(s, ids.ctypes.data, ids.size, 4096, 16, kept.ctypes.data, kept.size,
                                    ctypes.byref(c), ctypes.byref(tr)) == -1
        assert ours.fbx_prompt_plan(s, None, 0, 4096, 16, kept.ctypes.data, kept.size,
                                    ctypes.byref(c), ctypes.byref(tr)) == -1
        # n_ctx 256: reserve 64, budget 192, head 48, tail 96
        big = np.zeros(ids.size, np.int32)
        n = ours.fbx_prompt_plan(s, ids.ctypes.data, ids.size, 256, 16, big.ctypes.data, big.size,
                                 ctypes.byref(c), ctypes.byref(tr))
        assert (n, tr.value, c.value) == (144, 1, 0)
        assert np.array_equal(big[:48], ids[:48]) and np.array_equal(big[48:n], ids[-96:])
    finally:
        ours.fbx_prompt_state_destroy(s)
