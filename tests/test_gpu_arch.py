"""Architecture variants on the same kernels, against the reference engine
itself (oracle/_ref, compiled from the reference's sources), which runs both:

* gemma2 (reference src/model.cpp:488-496, 1614-1627, 1735-1739, 1760-1806):
  norm weights stored as w - 1, the embedding scaled by sqrt(n_embd), GELU in
  the FFN, post-attention and post-FFN norms before the residual adds, an
  attention-score soft cap, a sliding window on the even layers and a final
  logit soft cap. The synthetic file's caps (0.5 on scores, 2.0 on logits) and
  64-position window are small enough to change every output;
* phi3 (src/model.cpp:253, 310-316, 522-530): fused q|k|v and gate|up
  tensors, longrope factors (the long set: the 1024-position context exceeds
  the file's 512-position original context) and the rotation scale; also at
  Phi-3-mini's head dimension 96 ("phi3-d96"), and with a fused q|k|v bias
  and an output-projection bias ("phi3-bias", src/model.cpp:343-348);
* qwen2moe (src/model.cpp:303-308, 1582-1599): routed experts plus a shared
  expert every token takes, scaled by the sigmoid of its own one-row gate.

Teacher-forced like tests/test_gpu_model.py: a 192-id prompt (past the
window), then 8 single-token steps, with the f32 cache on the SIMT kernels and
the fp16 cache on the tensor-core ones. These 4-layer Q4_K_M random-init
models amplify any rounding difference: the same engine with an fp16 instead
of an f32 cache differs from itself by up to 3.5% of max |logit| (gemma2) and
3.3% (phi3), with 54% / 43% of logits inside 1e-2 + 1e-3|x|. Measured against
the reference: f32 cache 2.7% / 2.3% and 63% / 58%; fp16 cache 3.3% / 3.1%
and 53% / 42%; the argmax equal at every step. Bars, set at that floor: max
|dlogit| <= 3% (f32) or 4% (fp16) of max |logit|, the argmax equal wherever
the reference's margin clears the tolerance (compare_steps), and at least 50%
(f32) or 35% (fp16) of each step's logits inside the north-star bar. A missing
post norm, soft cap, window, GELU, embedding scale or longrope factor set
moves logits by far more.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from test_gpu_model import compare_steps, run_teacher_forced

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return True


@pytest.mark.parametrize("kv_f32", [0, 1])
@pytest.mark.parametrize("preset", ["gemma2", "phi3", "phi3-d96", "phi3-bias", "qwen2moe"])
def test_arch_variant_vs_reference(gpu, reference, synth_dir, monkeypatch, preset, kv_f32):
    from imurun_b200 import synth
    from imurun_b200.native import Model
    if kv_f32:
        monkeypatch.setenv("FISH_KV_F32", "1")
    path = synth.cached(synth.preset(preset), synth_dir)
    ids = np.random.default_rng(23).integers(3, 32000, 200).astype(np.int32)
    with Model(path, 1024) as m:
        g = run_teacher_forced(m, ids, 192, 8)
    rm = reference.load(path, 1024)
    r = [rm.prefill(ids[:192])] + [rm.forward(ids[s:s + 1], s) for s in range(192, 200)]
    rel_max, frac = (0.03, 0.5) if kv_f32 else (0.04, 0.35)
    assert compare_steps(g, r, f"{preset} kv_f32={kv_f32}", rel_max=rel_max) >= frac


@pytest.mark.parametrize("preset", ["gemma2", "phi3-d96", "qwen2moe"])
def test_batch_equals_single_decodes(gpu, synth_dir, preset):
    """Batched decode (rank CTAs + merge) equals single-token decode (one
    cluster per kv head) bit for bit: gemma2 with the soft cap and the window
    on, at contexts on both sides of the 64-position window; phi3 with head
    dimension 96; qwen2moe with its routed experts grouped per expert and the
    shared expert over the whole batch."""
    from imurun_b200 import synth
    from imurun_b200.native import Model
    path = synth.cached(synth.preset(preset), synth_dir)
    rng = np.random.default_rng(5)
    prompts = [rng.integers(3, 32000, n).astype(np.int32) for n in (20, 63, 64, 65, 150, 300)]
    nxt = rng.integers(3, 32000, len(prompts)).astype(np.int32)
    with Model(path, 1024) as m:
        ss = [m.session_open() for _ in prompts]
        for s, p in zip(ss, prompts):
            m.session_prefill(s, p)
        am, lg = m.decode_batch(ss, nxt, logits=True)
        for i, p in enumerate(prompts):
            t = m.session_open()
            m.session_prefill(t, p)
            am1, lg1 = m.decode_batch([t], nxt[i:i + 1], logits=True)
            assert np.array_equal(lg1[0], lg[i]), i
            assert am1[0] == am[i]
            m.session_close(t)


def test_gemma2_self_draft_equals_plain_greedy(gpu, synth_dir):
    """Speculative verification under the window and soft caps: the target
    as its own draft gives plain greedy's ids exactly (the verify step's rows
    are single-token decodes' bits)."""
    from imurun_b200 import native, synth
    path = synth.cached(synth.preset("gemma2"), synth_dir)
    lib = native.load_library()
    lib.fbx_last_generated.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    lib.fbx_last_generated.restype = ctypes.c_int
    prompt = b"t17 t99 t4000 the quick brown fox t12 t12 t12 jumps over t300 t301 " * 3

    def run(draft):
        ctx = lib.fish_create()
        assert lib.fish_load(ctx, str(path).encode(), 1024) == 0, lib.fish_last_error(ctx)
        if draft:
            assert lib.fish_set_draft(ctx, str(path).encode(), 4) == 0, lib.fish_last_error(ctx)
        n = lib.fish_generate(ctx, prompt, 1, 48, 0.0, 40, 0.9, 1.1, native.FISH_TOKEN_CB(), None)
        assert n > 0, lib.fish_last_error(ctx)
        out = np.zeros(n, np.int32)
        assert lib.fbx_last_generated(ctx, out.ctypes.data, n) == n
        st = native.FishStats()
        lib.fish_get_stats(ctx, ctypes.byref(st))
        lib.fish_destroy(ctx)
        return out.tolist(), st

    want, _ = run(False)
    got, st = run(True)
    assert st.draft_proposed > 0 and st.draft_accepted >= 0.9 * st.draft_proposed
    assert got == want
