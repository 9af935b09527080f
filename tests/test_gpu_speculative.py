"""Speculative decoding through the FISH C ABI (fish_set_draft; reference
model/fish/src/c_api.cpp:410-456 and the draft loop at 630-773).

The rejection rule keeps the target's sampling distribution, so with a
greedy sampler (one-hot p and q) speculative generation emits the ids of
plain greedy generation whatever the draft proposes. Here that holds bit for
bit: the verify forward is the batched decode step over consecutive
positions of one sequence, whose logits per row are the bits a single-token
decode gives (batch invariance of the GEMV and decode-attention kernels), so
the tests compare ids exactly. The rule itself is checked on fixed
distributions on the CPU (tests/test_sampler_cpu.py).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

PROMPT = b"t17 t99 t4000 the quick brown fox t12 t12 t12 jumps over t300 t301"


@pytest.fixture(scope="module")
def gpu():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return True


@pytest.fixture(scope="module")
def lib():
    from imurun_b200 import native
    lib = native.load_library()
    lib.fbx_last_generated.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    lib.fbx_last_generated.restype = ctypes.c_int
    return lib


def _ctx(lib, path, n_ctx=2048, draft=None, k=4):
    ctx = lib.fish_create()
    assert lib.fish_load(ctx, str(path).encode(), n_ctx) == 0, lib.fish_last_error(ctx)
    if draft is not None:
        assert lib.fish_set_draft(ctx, str(draft).encode(), k) == 0, lib.fish_last_error(ctx)
    return ctx


def _generate(lib, ctx, n_gen, temp=0.0, top_k=40, top_p=0.9, pen=1.1, prompt=PROMPT):
    from imurun_b200 import native
    n = lib.fish_generate(ctx, prompt, 1, n_gen, temp, top_k, top_p, pen, native.FISH_TOKEN_CB(), None)
    assert n >= 0, lib.fish_last_error(ctx)
    out = np.zeros(max(n, 1), np.int32)
    assert lib.fbx_last_generated(ctx, out.ctypes.data, out.size) == n
    return out[:n].tolist()


def _stats(lib, ctx):
    from imurun_b200 import native
    st = native.FishStats()
    lib.fish_get_stats(ctx, ctypes.byref(st))
    return st


def _prompt_ids(lib, ctx):
    ids = np.zeros(512, np.int32)
    n = lib.fish_tokenize(ctx, PROMPT, 1, ids.ctypes.data, 512)
    assert 0 < n < 512
    return ids[:n].tolist()


@pytest.mark.parametrize("pen", [1.0, 1.3])
def test_self_draft_greedy_equals_plain_greedy(gpu, lib, tiny_gguf, pen):
    """The target as its own draft: every proposal is the target's own
    greedy choice, so nearly all are accepted, and the ids equal plain
    greedy decoding. A second call with the same prompt reuses both caches
    (the target's prefix cache, the draft's common prefix) and repeats it."""
    n_gen = 48
    plain = _ctx(lib, tiny_gguf)
    want = _generate(lib, plain, n_gen, pen=pen)
    spec = _ctx(lib, tiny_gguf, draft=tiny_gguf, k=4)
    got = _generate(lib, spec, n_gen, pen=pen)
    st = _stats(lib, spec)
    assert st.draft_active == 1 and st.draft_proposed > 0
    assert st.draft_accepted >= 0.9 * st.draft_proposed, (st.draft_accepted, st.draft_proposed)
    assert st.generated_tokens == len(got)
    assert got == want
    again = _generate(lib, spec, n_gen, pen=pen)
    assert _stats(lib, spec).cached_tokens == len(_prompt_ids(lib, plain)) - 1
    assert again == want
    lib.fish_destroy(spec)
    lib.fish_destroy(plain)


def test_unrelated_draft_greedy_equals_plain_greedy(gpu, lib, tiny_gguf, synth_dir):
    """A draft with other weights (same vocabulary) proposes mostly wrong
    tokens: the rejections, replacements and cache rewinds must still give
    plain greedy's ids."""
    from imurun_b200 import synth
    other = synth.cached(synth.preset("tiny", layers=2, seed=77), synth_dir)
    n_gen = 40
    plain = _ctx(lib, tiny_gguf)
    want = _generate(lib, plain, n_gen, pen=1.1)
    spec = _ctx(lib, tiny_gguf, draft=other, k=6)
    got = _generate(lib, spec, n_gen, pen=1.1)
    st = _stats(lib, spec)
    assert st.draft_proposed > 0 and st.draft_accepted < st.draft_proposed
    assert got == want
    lib.fish_destroy(spec)
    lib.fish_destroy(plain)


def test_top1_sampling_with_draft_equals_greedy(gpu, lib, tiny_gguf):
    """temperature > 0 with top_k = 1 takes the sampled branch (all logits of
    the verify forward on the host, distributions, the rejection rule) with
    one-hot distributions: the ids of greedy decoding."""
    n_gen = 32
    plain = _ctx(lib, tiny_gguf)
    want = _generate(lib, plain, n_gen, temp=0.0, pen=1.1)
    spec = _ctx(lib, tiny_gguf, draft=tiny_gguf, k=5)
    got = _generate(lib, spec, n_gen, temp=0.8, top_k=1, pen=1.1)
    st = _stats(lib, spec)
    assert st.draft_proposed > 0 and st.draft_accepted >= 0.9 * st.draft_proposed
    assert got == want
    lib.fish_destroy(spec)
    lib.fish_destroy(plain)


def test_sampled_self_draft_accepts_nearly_everything(gpu, lib, tiny_gguf):
    """Full sampling (temperature, top-k, top-p, penalty) with the target as
    its own draft: q equals p up to rounding, so min(1, p/q) keeps nearly
    every proposal, and the output is max_tokens valid ids."""
    spec = _ctx(lib, tiny_gguf, draft=tiny_gguf, k=5)
    got = _generate(lib, spec, 64, temp=0.8, top_k=40, top_p=0.9, pen=1.1)
    st = _stats(lib, spec)
    assert 0 < len(got) <= 64 and all(0 <= t < 32000 for t in got)
    assert st.draft_proposed > 0 and st.draft_accepted >= 0.8 * st.draft_proposed
    lib.fish_destroy(spec)


def test_context_end_with_a_draft(gpu, lib, tiny_gguf):
    """Near the end of the context the loop falls back to plain decode steps
    (a round needs k + 2 free positions) and stops at n_ctx like plain
    generation."""
    plain = _ctx(lib, tiny_gguf, n_ctx=256)
    want = _generate(lib, plain, 400, pen=1.1)
    n_prompt = len(_prompt_ids(lib, plain))
    spec = _ctx(lib, tiny_gguf, n_ctx=256, draft=tiny_gguf, k=8)
    got = _generate(lib, spec, 400, pen=1.1)
    assert n_prompt + len(want) == 256       # stopped by the context, not by an end token
    assert got == want
    lib.fish_destroy(spec)
    lib.fish_destroy(plain)


def test_draft_checks_and_resets(gpu, lib, tiny_gguf, synth_dir):
    """A draft with another vocabulary is refused with -3 (reference
    c_api.cpp:421-434); a missing file with -2; fish_load drops the draft;
    fish_clear_draft and fish_reset keep the context usable."""
    from imurun_b200 import synth
    small_vocab = synth.cached(synth.preset("tiny", layers=1, vocab=1000), synth_dir)
    ctx = _ctx(lib, tiny_gguf)
    assert lib.fish_set_draft(ctx, str(small_vocab).encode(), 4) == -3
    assert b"vocabulary" in lib.fish_last_error(ctx)
    assert _stats(lib, ctx).draft_active == 0
    assert lib.fish_set_draft(ctx, b"/nonexistent/draft.gguf", 4) == -2
    assert lib.fish_set_draft(ctx, str(tiny_gguf).encode(), 0) == 0   # k <= 0: the default 5
    assert _stats(lib, ctx).draft_active == 1
    a = _generate(lib, ctx, 8)
    lib.fish_reset(ctx)
    b = _generate(lib, ctx, 8)
    assert a == b
    lib.fish_clear_draft(ctx)
    assert _stats(lib, ctx).draft_active == 0
    assert lib.fish_set_draft(ctx, str(tiny_gguf).encode(), 99) == 0   # capped at 16
    assert lib.fish_load(ctx, str(tiny_gguf).encode(), 2048) == 0
    assert _stats(lib, ctx).draft_active == 0
    assert _generate(lib, ctx, 8) == a
    lib.fish_destroy(ctx)
