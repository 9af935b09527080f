"""End-to-end parity of the engine (through the FISH C ABI) against the CPU
oracle and, where its build is present, the reference FISH engine.

Teacher-forced like the reference's GPU acceptance test (test/test_gpu.cpp:
577-591): both engines see the same ids at every step. Criteria, written in
each test:
  * the reference's engine-vs-engine bar: max |dlogit| <= 2% of max |logit|
    and the same argmax wherever the oracle's top-1/top-2 margin exceeds the
    logit tolerance;
  * the north-star tolerance |dlogit| <= 1e-2 + 1e-3 |logit| for at least 90%
    of the logits of every step. The bar is per logit, not all-of-them: int8
    activation rounding flips, set off by 1-ulp float-order differences, move
    a step's logits by up to ~0.02 on these random-init models. The reference
    and the C restatement (two CPU engines) show the same floor: 96-99% of
    logits inside the bar, max ~0.02 (tests/test_oracle_pin.py pins it);
  * integer-exact parts (page tables, greedy ids vs the engine's own
    teacher-forced argmax) must be identical.
"""
from __future__ import annotations

import os
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return True


def _margin(logits):
    s = np.sort(logits)
    return float(s[-1] - s[-2])


def compare_steps(gpu_steps, ref_steps, label, rel_max=0.02):
    """Returns the smallest per-step fraction of logits inside the north-star bar.
    rel_max: max |dlogit| allowed as a fraction of max |logit| (0.02 is the
    reference's own bar; models whose CPU-engine floor exceeds it get the
    floor's value, pinned in tests/test_oracle_pin.py)."""
    worst = 1.0
    for i, (a, b) in enumerate(zip(gpu_steps, ref_steps)):
        d = np.abs(a - b)
        assert d.max() <= rel_max * np.abs(b).max(), f"{label} step {i}: max diff {d.max():.4f} of {np.abs(b).max():.3f}"
        if _margin(b) > 2 * (1e-2 + 1e-3 * np.abs(b).max()):
            assert int(np.argmax(a)) == int(np.argmax(b)), f"{label} step {i}: argmax differs"
        worst = min(worst, float(np.mean(d <= 1e-2 + 1e-3 * np.abs(b))))
    print(f"{label}: worst per-step fraction inside 1e-2 abs + 1e-3 rel = {worst:.4f}")
    return worst


def run_teacher_forced(model, ids, n_prompt, n_dec):
    steps = [model.prefill(ids[:n_prompt], 0)]
    for s in range(n_prompt, n_prompt + n_dec):
        lg, _ = model.decode(ids[s:s + 1], s)
        steps.append(lg[0])
    return steps


def oracle_teacher_forced(om, ids, n_prompt, n_dec):
    steps = [om.forward(ids[:n_prompt], 0)]
    for s in range(n_prompt, n_prompt + n_dec):
        steps.append(om.forward(ids[s:s + 1], s))
    return steps


@pytest.mark.parametrize("kv_f32", [1, 0])
def test_tiny_teacher_forced_vs_oracle(gpu, oracle, tiny_gguf, kv_f32, monkeypatch):
    from imurun_b200.native import Model
    monkeypatch.setenv("FISH_KV_F32", str(kv_f32))
    ids = np.random.default_rng(123).integers(3, 32000, 160).astype(np.int32)
    with Model(tiny_gguf, 2048) as m:
        g = run_teacher_forced(m, ids, 128, 24)
    om = oracle.load(tiny_gguf, 2048, kv_f16=not kv_f32)
    o = oracle_teacher_forced(om, ids, 128, 24)
    frac = compare_steps(g, o, f"tiny kv_f32={kv_f32}")
    assert frac >= 0.9, frac


def test_tiny_vs_reference(gpu, reference, tiny_gguf, monkeypatch):
    from imurun_b200.native import Model
    monkeypatch.setenv("FISH_KV_F32", "1")
    ids = np.random.default_rng(7).integers(3, 32000, 136).astype(np.int32)
    with Model(tiny_gguf, 2048) as m:
        g = run_teacher_forced(m, ids, 128, 8)
    rm = reference.load(tiny_gguf, 2048)
    r = [rm.prefill(ids[:128])] + [rm.forward(ids[s:s + 1], s) for s in range(128, 136)]
    assert compare_steps(g, r, "tiny vs reference") >= 0.9


def test_tiny_config1_full_greedy_vs_reference(gpu, reference, oracle, tiny_gguf, monkeypatch):
    """Configuration 1 in full against the live reference engine (built from
    its own sources): a 128-id prompt, then 128 greedy decode tokens. The
    reference picks its own greedy chain; this engine is teacher-forced along
    that chain (the acceptance pattern of test/test_gpu.cpp:577-631) and must
    (a) keep every step's logits within the reference's engine-vs-engine bar
    (max |d| <= 2% of max |logit|) and, per step, the fraction of logits
    inside 1e-2 + 1e-3 |x| no lower than the CPU-vs-CPU floor (the oracle
    restatement against the reference on the same chain) minus 5 points,
    (b) pick the reference's token at every step whose top-1/top-2 margin
    clears twice the logit tolerance. Its own on-device greedy loop from the
    same prompt must reproduce the reference's chain up to the first step
    whose margin does not clear that bar (random-init models have near-ties);
    the number of identical leading tokens and the first divergence are
    printed."""
    from imurun_b200.native import Model
    monkeypatch.setenv("FISH_KV_F32", "1")
    P, N = 128, 128
    prompt = np.random.default_rng(2024).integers(3, 32000, P).astype(np.int32)
    rm = reference.load(tiny_gguf, 2048)
    ref_steps = [rm.prefill(prompt)]
    chain = []
    for s in range(N):
        tok = int(np.argmax(ref_steps[-1]))
        chain.append(tok)
        if s < N - 1:
            ref_steps.append(rm.forward(np.array([tok], np.int32), P + s))
    ids = np.concatenate([prompt, np.array(chain[:-1], np.int32)])
    with Model(tiny_gguf, 2048) as m:
        g = run_teacher_forced(m, ids, P, N - 1)
        m.set_kv_len(0)
        first = int(np.argmax(m.prefill(prompt, 0)))
        own = [first] + list(m.greedy(first, N - 1))
    frac = compare_steps(g, ref_steps, "config 1 teacher-forced on the reference's greedy chain")
    # the CPU-vs-CPU floor on the same chain: the oracle restatement against
    # the reference (both on the CPU, f32 KV); the GPU must not be worse
    # than that floor by more than 5 points
    om = oracle.load(tiny_gguf, 2048)
    o = oracle_teacher_forced(om, ids, P, N - 1)
    floor = compare_steps(o, ref_steps, "config 1 oracle vs reference (CPU floor)", rel_max=0.05)
    print(f"config 1: worst step {frac:.4f} of logits inside 1e-2 + 1e-3|x| (CPU floor {floor:.4f})")
    assert frac >= min(0.9, floor - 0.05), (frac, floor)
    tol = lambda lg: 2 * (1e-2 + 1e-3 * float(np.abs(lg).max()))
    cleared = [_margin(lg) > tol(lg) for lg in ref_steps]
    for s in range(N):
        if cleared[s]:
            assert int(np.argmax(g[s])) == chain[s], f"step {s}: {int(np.argmax(g[s]))} vs {chain[s]}"
    same = 0
    while same < N and own[same] == chain[same]:
        same += 1
    first_low = next((s for s in range(N) if not cleared[s]), N)
    # the oracle's own greedy chain (CPU restatement) against the reference's,
    # for scale: how far two CPU engines agree on this random-init model
    om.set_kv_len(0)
    ochain = [int(np.argmax(om.forward(prompt, 0)))]
    for s in range(N - 1):
        ochain.append(int(np.argmax(om.forward(np.array([ochain[-1]], np.int32), P + s))))
    osame = 0
    while osame < N and ochain[osame] == chain[osame]:
        osame += 1
    print(f"config 1: {same} of {N} greedy tokens identical to the reference's chain (oracle restatement: {osame}); "
          f"first step whose margin does not clear the bar: {first_low}; {sum(cleared)} of {N} steps clear it")
    assert same >= min(first_low, N), (same, first_low)
    if first_low >= 64:
        assert same >= 64


def test_greedy_device_loop_matches_teacher_forced(gpu, tiny_gguf):
    from imurun_b200.native import Model
    ids = np.random.default_rng(3).integers(3, 32000, 64).astype(np.int32)
    with Model(tiny_gguf, 2048) as m:
        lg = m.prefill(ids, 0)
        first = int(np.argmax(lg))
        out = m.greedy(first, 32)
        assert m.kv_len() == 64 + 32
        # replay the same chain step by step with the id-level call
        m.set_kv_len(64)
        chain = [first] + list(out[:-1])
        _, am = m.decode(np.array(chain, np.int32), 64, logits=False)
        # batched teacher-forced argmax equals the device greedy chain
        assert np.array_equal(am, out)


def test_prefill_below_2048_keys_in_a_longer_context(gpu, tiny_gguf):
    """A context longer than 2048 positions with a prompt between a quarter of
    it and 2048 tokens: prefill attention then splits the keys 32 a CTA, more
    splits than the longest context needs, and its scratch must hold them.
    The result equals the same prefill in a 2048-position context (same
    splits, same bits)."""
    from imurun_b200.native import Model
    ids = np.random.default_rng(11).integers(3, 32000, 1500).astype(np.int32)
    with Model(tiny_gguf, 4096) as m:
        long_ctx = m.prefill(ids, 0)
    with Model(tiny_gguf, 2048) as m:
        short_ctx = m.prefill(ids, 0)
    assert np.array_equal(long_ctx, short_ctx)


def test_greedy_on_a_fresh_process_and_context(gpu, tiny_gguf):
    """The first kernel launches of a process may be inside the greedy loop's
    graph capture (no prefill before it): nothing may allocate there. Run in
    a child process, so no earlier test has made the first launches."""
    import subprocess
    import sys
    code = (
        "import sys, numpy as np\n"
        f"sys.path.insert(0, {str(ROOT)!r})\n"
        "from imurun_b200.native import Model\n"
        f"with Model({str(tiny_gguf)!r}, 256) as m:\n"
        "    out = m.greedy(5, 8)\n"
        "    m.set_kv_len(0)\n"
        "    _, am = m.decode(np.array([5] + list(out[:-1]), np.int32), 0, logits=False)\n"
        "    assert np.array_equal(am, out), (list(am), list(out))\n"
        "print('ok')\n")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


def test_llama8b_shape_two_layers_vs_oracle(gpu, oracle, synth_dir, monkeypatch):
    """Q4_K_M mixture (Q4_K + Q6_K) at the Llama-3-8B widths, 2 layers.

    On this model two CPU engines (reference vs restatement) already keep only
    29-49% of logits inside 1e-2 + 1e-3|l| and reach 2.2% of max |logit|:
    the small random-init residual stream amplifies int8 rounding flips
    through the final RMSNorm. The GPU is held to that floor: >= 25% inside
    the bar, max <= 3% of max |logit|, median |dlogit| <= 0.03, argmax with
    the margin guard (floor pinned by test_oracle_pin.py)."""
    from imurun_b200 import synth
    from imurun_b200.native import Model
    path = synth.cached(synth.preset("llama8b", layers=2), synth_dir)
    monkeypatch.setenv("FISH_KV_F32", "1")
    ids = np.random.default_rng(8).integers(3, 128256, 20).astype(np.int32)
    with Model(path, 1024) as m:
        g = run_teacher_forced(m, ids, 16, 4)
    om = oracle.load(path, 1024)
    o = oracle_teacher_forced(om, ids, 16, 4)
    assert compare_steps(g, o, "llama8b-2L", rel_max=0.03) >= 0.25
    for a, b in zip(g, o):
        assert np.median(np.abs(a - b)) <= 0.03


def test_qwen_shape_bias_neox_vs_oracle(gpu, oracle, synth_dir, monkeypatch):
    """qwen2 architecture: q/k/v biases, NeoX RoPE, 28/4 heads (G = 7)."""
    from imurun_b200 import synth
    from imurun_b200.native import Model
    path = synth.cached(synth.preset("qwen7b", layers=1, vocab=32000), synth_dir)
    monkeypatch.setenv("FISH_KV_F32", "1")
    ids = np.random.default_rng(9).integers(3, 32000, 12).astype(np.int32)
    with Model(path, 1024) as m:
        g = run_teacher_forced(m, ids, 9, 3)
    om = oracle.load(path, 1024)
    o = oracle_teacher_forced(om, ids, 9, 3)
    assert compare_steps(g, o, "qwen-1L") >= 0.9


def test_qwen3_qk_norm_vs_oracle(gpu, oracle, synth_dir, monkeypatch):
    """qwen3 architecture: per-head q/k RMSNorm (non-unit weights) before
    NeoX RoPE, no qkv bias, 2 layers (model.cpp:1714-1722 of the reference).

    On this model the two CPU engines (reference vs restatement, same ids and
    steps) keep 71-75% of logits inside 1e-2 + 1e-3|l| with max |dlogit|
    1.4-1.6% of max |logit| (test_oracle_pin.py::
    test_live_reference_qwen3_qk_norm pins it); the GPU is held to that
    floor: >= 60% inside, max <= 3%, argmax with the margin guard."""
    from imurun_b200 import synth
    from imurun_b200.native import Model
    path = synth.cached(synth.preset("qwen3", layers=2), synth_dir)
    monkeypatch.setenv("FISH_KV_F32", "1")
    ids = np.random.default_rng(11).integers(3, 32000, 14).astype(np.int32)
    with Model(path, 1024) as m:
        g = run_teacher_forced(m, ids, 10, 4)
    om = oracle.load(path, 1024)
    o = oracle_teacher_forced(om, ids, 10, 4)
    assert compare_steps(g, o, "qwen3-2L", rel_max=0.03) >= 0.6


def test_mixtral_shape_moe_vs_oracle(gpu, oracle, synth_dir, monkeypatch):
    """8 experts, top-2 softmax router, renormalised weights, 1 layer."""
    from imurun_b200 import synth
    from imurun_b200.native import Model
    path = synth.cached(synth.preset("mixtral", layers=1, n_embd=1024, n_ff=2816, n_head=8, n_head_kv=2), synth_dir)
    monkeypatch.setenv("FISH_KV_F32", "1")
    ids = np.random.default_rng(10).integers(3, 32000, 12).astype(np.int32)
    with Model(path, 1024) as m:
        g = run_teacher_forced(m, ids, 8, 4)
    om = oracle.load(path, 1024)
    o = oracle_teacher_forced(om, ids, 8, 4)
    assert compare_steps(g, o, "moe-1L") >= 0.9


def test_prefix_cache_hit_through_generate(gpu, tiny_gguf):
    """Second turn reuses the cached prefix (reference test/test_fish.py:231-249)."""
    import ctypes
    from imurun_b200 import native
    lib = native.load_library()
    ctx = lib.fish_create()
    assert lib.fish_load(ctx, str(tiny_gguf).encode(), 2048) == 0
    buf = ctypes.create_string_buffer(4096)
    prompt = b"the quick brown fox jumps over the lazy dog " * 4
    n1 = lib.fish_generate_to(ctx, prompt, 1, 12, 0.0, 1, 1.0, 1.0, buf, 4096)
    assert n1 >= 0
    first = buf.value
    st = native.FishStats()
    lib.fish_get_stats(ctx, ctypes.byref(st))
    assert st.cached_tokens == 0 and st.prompt_tokens > 8
    n2 = lib.fish_generate_to(ctx, prompt + b"and more", 1, 12, 0.0, 1, 1.0, 1.0, buf, 4096)
    assert n2 >= 0
    lib.fish_get_stats(ctx, ctypes.byref(st))
    assert st.cached_tokens > 8
    # identical prompt: prefix = n - 1, same greedy continuation as the first turn
    n3 = lib.fish_generate_to(ctx, prompt, 1, 12, 0.0, 1, 1.0, 1.0, buf, 4096)
    lib.fish_get_stats(ctx, ctypes.byref(st))
    assert st.cached_tokens == st.prompt_tokens - 1
    assert buf.value == first and n3 == n1
    lib.fish_destroy(ctx)


@pytest.mark.parametrize("penalty", [1.0, 1.3])
def test_greedy_generate_device_argmax_matches_host_sampler(gpu, tiny_gguf, penalty):
    """fish_generate at temperature 0 takes the sampler's greedy branch on the
    device (penalty + first-index argmax, only the id copied back). The same
    loop replayed step by step with the logits copied to the host and the
    host sampler (fbx_sample, pinned to the reference's Sampler::sample)
    must give the same token callbacks (ids and UTF-8 chunks)."""
    import ctypes
    from imurun_b200 import native
    lib = native.load_library()
    lib.fbx_sample.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_float,
                               ctypes.c_float, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_ulonglong,
                               ctypes.c_int, ctypes.c_void_p]
    lib.fbx_sample.restype = ctypes.c_int
    ctx = lib.fish_create()
    assert lib.fish_load(ctx, str(tiny_gguf).encode(), 2048) == 0
    vocab = 32000
    prompt = b"t17 t99 t4000 the quick brown fox t12 t12 t12 jumps"
    n_gen = 24
    chunks = []

    def on_token(text, tid, user):
        t = ctypes.string_at(text) if text else b""
        chunks.append(b"%d %d\n" % (tid, len(t)) + t)

    cb = native.FISH_TOKEN_CB(on_token)
    assert lib.fish_generate(ctx, prompt, 1, n_gen, 0.0, 40, 0.9, penalty, cb, None) >= 0
    got = b"".join(chunks)
    # replay: same prompt ids, logits to the host, host sampler
    lib.fish_reset(ctx)
    ids = np.zeros(512, np.int32)
    n = lib.fish_tokenize(ctx, prompt, 1, ids.ctypes.data, 512)
    assert 0 < n < 512
    ids = ids[:n].copy()
    lg = np.zeros((n, vocab), np.float32)
    am = np.zeros(n, np.int32)
    assert lib.fish_decode_ids(ctx, ids.ctypes.data, n, 0, lg.ctypes.data, am.ctypes.data) == 0
    recent = list(ids[-128:])
    logits = lg[-1].copy()
    out = []
    pos = n
    one = np.zeros(1, np.int32)
    for _ in range(n_gen):
        r = np.array(recent, np.int32)
        nxt = np.zeros(1, np.int32)
        assert lib.fbx_sample(logits.ctypes.data, vocab, 0.0, 40, 0.9, penalty, 64, r.ctypes.data, r.size, 1, 1,
                              nxt.ctypes.data) == 0
        tok = int(nxt[0])
        if tok == 2:   # end of generation
            break
        out.append(tok)
        recent.append(tok)
        recent = recent[-128:]
        one[0] = tok
        lg1 = np.zeros((1, vocab), np.float32)
        assert lib.fish_decode_ids(ctx, one.ctypes.data, 1, pos, lg1.ctypes.data, am.ctypes.data) == 0
        logits = lg1[0].copy()
        pos += 1
    # the callbacks the loop's emitter makes for these ids
    o = np.array(out, np.int32)
    buf = ctypes.create_string_buffer(1 << 16)
    lib.fbx_stream_gguf.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_int]
    lib.fbx_stream_gguf.restype = ctypes.c_int
    need = lib.fbx_stream_gguf(str(tiny_gguf).encode(), o.ctypes.data, o.size, buf, 1 << 16)
    assert 0 <= need < (1 << 16)
    assert got == buf.raw[:need], (got[:120], buf.raw[:120])
    lib.fish_destroy(ctx)


def test_chat_turns_stats_and_cancel(gpu, tiny_gguf):
    """The call sequence IMURUN's client makes for chat (model/fish_native.py:
    load, model info, chat prompt and token count, fish_generate_chat with a
    token callback on a worker thread, stats, cancel): two chat turns share
    their prefix through the prefix cache (cached_tokens > 8 on turn 2, as the
    reference's test_fish.py:231-249 checks), the stats carry the turn's
    counts and rates, and fish_cancel from another thread mid-generation ends
    the loop early with the tokens generated so far."""
    import ctypes
    import threading
    from imurun_b200 import native
    lib = native.load_library()
    ctx = lib.fish_create()
    assert lib.fish_load(ctx, str(tiny_gguf).encode(), 2048) == 0
    info = native.FishModelInfo()
    assert lib.fish_model_info_of(ctx, ctypes.byref(info)) == 0 and info.vocab == 32000

    def chat_args(msgs):
        roles = (ctypes.c_char_p * len(msgs))(*[r.encode() for r, _ in msgs])
        contents = (ctypes.c_char_p * len(msgs))(*[c.encode() for _, c in msgs])
        return ctypes.cast(roles, ctypes.c_void_p), ctypes.cast(contents, ctypes.c_void_p), len(msgs)

    msgs = [("system", "be brief t300 t301 t302 t303"), ("user", "hello there t17 t99 t4000 t12 t12")]
    n_chat = lib.fish_count_chat_tokens(ctx, *chat_args(msgs))
    assert n_chat > 8
    chunks = []
    cb = native.FISH_TOKEN_CB(lambda text, tid, user: chunks.append((ctypes.string_at(text), tid)))
    n1 = lib.fish_generate_chat(ctx, *chat_args(msgs), 16, 0.0, 40, 0.9, 1.1, cb, None)
    assert n1 > 0 and len(chunks) > 0
    st = native.FishStats()
    lib.fish_get_stats(ctx, ctypes.byref(st))
    assert st.prompt_tokens == n_chat and st.generated_tokens == n1 and st.cached_tokens == 0
    assert st.tokens_per_second > 0 and st.prefill_tokens_per_second > 0
    # turn 2: the history grows; its prefix comes from the cache
    reply = b"".join(c for c, _ in chunks).decode("utf-8", "replace")
    msgs2 = msgs + [("assistant", reply), ("user", "and more t5 t6 t7")]
    n2 = lib.fish_generate_chat(ctx, *chat_args(msgs2), 16, 0.7, 40, 0.9, 1.1, cb, None)
    assert n2 > 0
    lib.fish_get_stats(ctx, ctypes.byref(st))
    assert st.cached_tokens > 8
    # cancel from another thread while the generating thread is in the loop
    seen = []
    started = threading.Event()

    def on_tok(text, tid, user):
        seen.append(tid)
        if len(seen) == 5:
            started.set()

    cb2 = native.FISH_TOKEN_CB(on_tok)
    res = {}
    th = threading.Thread(target=lambda: res.setdefault(
        "n", lib.fish_generate_chat(ctx, *chat_args(msgs2), 1500, 0.7, 40, 0.9, 1.0, cb2, None)))
    th.start()
    assert started.wait(60)
    lib.fish_cancel(ctx)
    th.join(60)
    assert not th.is_alive()
    assert 5 <= res["n"] < 1500, res
    lib.fish_get_stats(ctx, ctypes.byref(st))
    assert st.generated_tokens == res["n"]
    lib.fish_destroy(ctx)


class PageModel:
    """CPU model of the engine's page allocator: LIFO free list, refcounts,
    shared full pages on fork, copy-on-write of a shared partial page."""

    def __init__(self, n_pages, P):
        self.free = list(range(n_pages - 1, -1, -1))
        self.ref = [0] * n_pages
        self.P = P
        self.seqs = {0: ([], 0)}

    def _take(self):
        p = self.free.pop()
        self.ref[p] = 1
        return p

    def ensure(self, s, new_len):
        pages, ln = self.seqs[s]
        pages = list(pages)
        if ln % self.P and pages:
            pi = ln // self.P
            if self.ref[pages[pi]] > 1:
                self.ref[pages[pi]] -= 1
                pages[pi] = self._take()
        while len(pages) < (new_len + self.P - 1) // self.P:
            pages.append(self._take())
        self.seqs[s] = (pages, new_len)

    def fork(self, s_new, parent, prefix):
        pages, _ = self.seqs[parent]
        n = (prefix + self.P - 1) // self.P
        for p in pages[:n]:
            self.ref[p] += 1
        self.seqs[s_new] = (list(pages[:n]), prefix)


def test_sessions_share_prefix_pages_and_match_fresh_prefill(gpu, tiny_gguf, monkeypatch):
    from imurun_b200.native import Model
    monkeypatch.setenv("FISH_KV_POSITIONS", "4096")
    rng = np.random.default_rng(11)
    prefix = rng.integers(3, 32000, 40).astype(np.int32)
    suffixes = [rng.integers(3, 32000, 5 + i).astype(np.int32) for i in range(3)]
    with Model(tiny_gguf, 1024) as m:
        P = m.lib.fish_kv_page_size(m.ctx)
        n_pages = (4096 + P - 1) // P
        model = PageModel(n_pages, P)
        base = m.session_open()
        model.seqs[base] = ([], 0)
        m.session_prefill(base, prefix)
        model.ensure(base, 40)
        forks, got = [], []
        for sfx in suffixes:
            s = m.session_fork(base, 40)
            model.fork(s, base, 40)
            assert np.array_equal(m.session_pages(s), model.seqs[s][0])
            got.append(m.session_prefill(s, sfx))
            model.ensure(s, 40 + sfx.size)
            assert np.array_equal(m.session_pages(s), model.seqs[s][0]), "page table differs from the allocator model"
            forks.append(s)
        # full prefix pages are shared, not copied
        for s in forks:
            assert list(m.session_pages(s)[:40 // P]) == list(m.session_pages(base)[:40 // P])
        assert np.array_equal(m.session_pages(base), model.seqs[base][0])
        # a fork continues exactly like a fresh session that prefilled prefix + suffix
        for sfx, lg in zip(suffixes, got):
            fresh = m.session_open()
            want = m.session_prefill(fresh, np.concatenate([prefix, sfx]))
            assert np.array_equal(lg, want)
            m.session_close(fresh)


def test_decode_batch_equals_single_decodes(gpu, tiny_gguf):
    from imurun_b200.native import Model
    rng = np.random.default_rng(12)
    prompts = [rng.integers(3, 32000, 20 + 3 * i).astype(np.int32) for i in range(5)]
    nxt = rng.integers(3, 32000, 5).astype(np.int32)
    with Model(tiny_gguf, 1024) as m:
        ss = [m.session_open() for _ in prompts]
        for s, p in zip(ss, prompts):
            m.session_prefill(s, p)
        am, lg = m.decode_batch(ss, nxt, logits=True)
        for i, (s, p) in enumerate(zip(ss, prompts)):
            t = m.session_open()
            m.session_prefill(t, p)
            am1, lg1 = m.decode_batch([t], nxt[i:i + 1], logits=True)
            assert np.array_equal(lg1[0], lg[i])
            assert am1[0] == am[i]
            m.session_close(t)


@pytest.mark.parametrize("P,n", [(700, 5), (2100, 17), (4200, 3)])
def test_shared_prefix_batch_equals_single_decodes(gpu, tiny_gguf, P, n):
    """Sessions forked from one P-token prompt (its pages shared), each with
    its own suffix, decoded as one batch: attention reads the shared 64-key
    blocks once for all sessions (the shared-prefix kernel, whose warps hand
    their state to the decode kernel) and every session's logits equal, bit
    for bit, those of the same session decoded alone (one cluster per kv
    head). P = 700: ranks with one prefix block; 2100: two; 4200: four (the
    resident maximum) plus a capped remainder; n = 17: three token groups."""
    import json
    from imurun_b200.native import Model
    rng = np.random.default_rng(P + n)
    prompt = rng.integers(3, 32000, P).astype(np.int32)
    suffixes = [rng.integers(3, 32000, 3 + 7 * i % 40).astype(np.int32) for i in range(n)]
    nxt = rng.integers(3, 32000, (2, n)).astype(np.int32)
    with Model(tiny_gguf, 4608) as m:
        m.prefill(prompt, 0)
        ss = [m.session_fork(0, P) for _ in range(n)]
        for s, u in zip(ss, suffixes):
            m.session_prefill(s, u)
        got = []
        for step in range(2):
            am, lg = m.decode_batch(ss, nxt[step], logits=True)
            got.append(lg)
            eng = json.loads(m.lib.fish_engine_json(m.ctx).decode())
            want_blocks = min(P // 64, 64)
            assert eng["last_batch_prefix_blocks"] == want_blocks, eng["last_batch_prefix_blocks"]
        for s in ss:
            m.session_close(s)
        for i, u in enumerate(suffixes):
            t = m.session_fork(0, P)
            m.session_prefill(t, u)
            for step in range(2):
                am1, lg1 = m.decode_batch([t], nxt[step, i:i + 1], logits=True)
                assert np.array_equal(lg1[0], got[step][i]), (i, step, float(np.abs(lg1[0] - got[step][i]).max()))
            m.session_close(t)


@pytest.mark.parametrize("n", [2, 5, 16])
def test_moe_grouped_batch_equals_single_decodes(gpu, synth_dir, n):
    """Batched MoE decode groups the tokens per expert (inside the step
    graph: one launch per (expert, 4-row chunk), expert ids read on the
    device); each session's logits must equal its own single-token decode
    (one GEMV per token and expert) bit for bit. The prompts' prefill runs
    the eager grouped path (exact per-expert row counts)."""
    from imurun_b200 import synth
    from imurun_b200.native import Model
    path = synth.cached(synth.preset("mixtral", layers=2, n_embd=1024, n_ff=2816, n_head=8, n_head_kv=2), synth_dir)
    rng = np.random.default_rng(40 + n)
    prompts = [rng.integers(3, 32000, 9 + 2 * i).astype(np.int32) for i in range(n)]
    nxt = rng.integers(3, 32000, n).astype(np.int32)
    with Model(path, 1024) as m:
        ss = [m.session_open() for _ in prompts]
        for s, p in zip(ss, prompts):
            m.session_prefill(s, p)
        am, lg = m.decode_batch(ss, nxt, logits=True)
        for i, (s, p) in enumerate(zip(ss, prompts)):
            t = m.session_open()
            m.session_prefill(t, p)
            am1, lg1 = m.decode_batch([t], nxt[i:i + 1], logits=True)
            assert np.array_equal(lg1[0], lg[i]), i
            assert am1[0] == am[i]
            m.session_close(t)


@pytest.mark.parametrize("kv_f32", [0, 1])
def test_persistent_step_matches_graph_path(gpu, synth_dir, monkeypatch, kv_f32):
    """The persistent decode kernel (k_step) against the graph path on one
    8B-shaped model (2 layers). Both run the same GEMV jobs (identical rows,
    one RMSNorm summation order); attention is split and merged differently
    (key chunks merged by the o projection's prologue), and on this model a
    1-ulp difference in the attention output re-quantises to a different
    int8 activation now and then, which the random-init residual stream
    amplifies (two CPU engines differ by up to 2.2% of max |logit| here, see
    test_llama8b_shape_two_layers_vs_oracle). Bar: max |dlogit| <= 3% of max
    |logit|, median <= 0.03, argmax equal where the margin clears the bar.
    Exact: greedy ids of one launch running 8 steps equal those of 8
    single-token launches of the same kernel (device-side token feedback and
    K/V appends). The 300-id prompt puts positions past one 64-key chunk, so
    the partial merge runs."""
    import json
    from imurun_b200 import synth
    from imurun_b200.native import Model
    path = synth.cached(synth.preset("llama8b", layers=2), synth_dir)
    if kv_f32:
        monkeypatch.setenv("FISH_KV_F32", "1")
    ids = np.random.default_rng(31).integers(3, 128256, 306).astype(np.int32)
    res = {}
    for persist in (1, 0):
        if persist:
            monkeypatch.setenv("FISH_PERSIST", "1")
        else:
            monkeypatch.delenv("FISH_PERSIST", raising=False)
        with Model(path, 1024) as m:
            m.prefill(ids[:300], 0)
            steps = [m.decode(ids[s:s + 1], s)[0][0].copy() for s in range(300, 306)]
            info = json.loads(m.lib.fish_engine_json(m.ctx).decode())
            extra = None
            if persist:
                m.set_kv_len(303)
                greedy = m.greedy(int(ids[303]), 8)          # one launch, 8 steps
                m.set_kv_len(303)
                tok, one_by_one = int(ids[303]), []
                for s in range(8):                           # 8 launches, 1 step each
                    _, am = m.decode(np.array([tok], np.int32), 303 + s)
                    tok = int(am[0])
                    one_by_one.append(tok)
                extra = (greedy, np.array(one_by_one, np.int32))
        res[persist] = (steps, info, extra)
    assert res[1][1]["step_kernel"] == 1, res[1][1].get("step_unavailable")
    assert res[0][1]["step_kernel"] == 0
    for i, (a, b) in enumerate(zip(res[1][0], res[0][0])):
        d = np.abs(a - b)
        assert d.max() <= 0.03 * np.abs(b).max(), (i, float(d.max()), float(np.abs(b).max()))
        assert np.median(d) <= 0.03, (i, float(np.median(d)))
        if _margin(b) > 2 * (1e-2 + 1e-3 * np.abs(b).max()):
            assert int(np.argmax(a)) == int(np.argmax(b)), i
    greedy, one_by_one = res[1][2]
    assert np.array_equal(greedy, one_by_one)
