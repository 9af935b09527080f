"""Pin the C restatement (oracle/fish_oracle.c) before it is trusted.

Against the golden vectors made by the reference engine (tests/golden/), and,
where the reference build is present, against the live reference on fresh
seeded inputs. Mirrors the reference's own kernel test:
test/test_kernels.cpp:154-235 (byte-identical activation quantisation, int8
dots equal to the scalar path within 1e-5 of sum |w x|) and the Q4_K layout
known-answer test test/test_m1.cpp:35-71.
"""
from __future__ import annotations

import numpy as np
import pytest

TYPES = {"Q4_0": 2, "Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14}


def test_activation_quantisers_byte_identical(golden, oracle):
    for kind in range(4):
        for n in (256, 4096):
            x = golden[f"acts_x{kind}_{n}"]
            assert np.array_equal(oracle.quantize_acts(x), golden[f"acts_q32_{kind}_{n}"]), (kind, n)
            assert np.array_equal(oracle.quantize_acts_k(x), golden[f"acts_qk_{kind}_{n}"]), (kind, n)


def test_int8_dots_match_reference(golden, oracle):
    for name, t in TYPES.items():
        for i in range(12):
            row, acts = golden[f"row_{name}_{i}"], golden[f"rowx_{name}_{i}"]
            n = 256 if i < 6 else 4096
            want = float(golden[f"rowdot_{name}_{i}"][0])
            y = oracle.vec_dot(t, row, acts, n)
            # mass = sum |w * xq| (test/test_kernels.cpp:197-205)
            mass = 1e-9 + abs(want) + 1.0
            if n == 256:
                w = golden[f"rowdeq_{name}_{i}"]
                mass = 1e-9 + float(np.abs(w).sum()) * 2.0
            assert abs(y - want) <= 1e-5 * mass + 1e-6 * abs(want), (name, i, y, want)


def test_dequant_matches_reference(golden, oracle):
    for name, t in TYPES.items():
        for i in range(6):
            row = golden[f"row_{name}_{i}"]
            assert np.array_equal(oracle.dequant(t, row, 256), golden[f"rowdeq_{name}_{i}"]), (name, i)


def test_q4k_known_answer(golden, oracle):
    y = oracle.dequant(12, golden["q4k_kat"], 256)
    want = np.array([(l & 15) for j in range(0, 256, 64) for l in list(range(32)) * 2], np.float32)
    assert np.array_equal(y, want)
    assert np.array_equal(y, golden["q4k_kat_deq"])


def test_tiny_model_logits_match_reference_golden(golden, oracle, tiny_gguf):
    m = oracle.load(tiny_gguf, 2048)
    ids = golden["tiny_ids"]
    steps = [m.forward(ids[:16], 0)] + [m.forward(ids[s:s + 1], s) for s in range(16, 18)]
    for got, want in zip(steps, golden["tiny_logits"]):
        diff = np.abs(got - want)
        # reference's own engine-vs-engine criterion (test/test_gpu.cpp:577-591)
        assert diff.max() <= 0.02 * np.abs(want).max()
        assert int(np.argmax(got)) == int(np.argmax(want))


def test_block_sums_equal_float_definition(oracle, reference):
    """Integer block sums: y reconstructed from (sumi, mins) equals the reference dot."""
    rng = np.random.default_rng(3)
    for t in (8, 12, 14):
        n = 4096
        w = rng.standard_normal(n).astype(np.float32) * 0.05
        row = reference.quantize_row(t, w)
        x = rng.standard_normal(n).astype(np.float32)
        acts = reference.quantize_acts_k(x) if t in (12, 14) else reference.quantize_acts(x)
        s, m = oracle.block_sums(t, row, acts, n)
        ref_y = reference.vec_dot(t, row, acts, n)
        bb = {8: 34, 12: 144, 14: 210}[t]
        nb = s.size
        y = 0.0
        for b in range(nb):
            blk = row[b * bb:(b + 1) * bb]
            if t == 8:
                dx = np.frombuffer(acts[b * 40:b * 40 + 4].tobytes(), np.float32)[0]
                dw = np.frombuffer(blk[0:2].tobytes(), np.float16)[0].astype(np.float32)
                y += float(np.float32(dw * dx)) * s[b]
            else:
                dx = np.frombuffer(acts[b * 276:b * 276 + 4].tobytes(), np.float32)[0]
                if t == 14:
                    dw = np.frombuffer(blk[208:210].tobytes(), np.float16)[0].astype(np.float32)
                    y += float(np.float32(dw * dx)) * s[b]
                else:
                    dw = np.frombuffer(blk[0:2].tobytes(), np.float16)[0].astype(np.float32)
                    dm = np.frombuffer(blk[2:4].tobytes(), np.float16)[0].astype(np.float32)
                    y += float(np.float32(dw * dx)) * s[b] - float(np.float32(dm * dx)) * m[b]
        assert abs(y - ref_y) <= 1e-5 * (abs(ref_y) + 1.0), (t, y, ref_y)


def test_live_reference_quantisers(oracle, reference):
    rng = np.random.default_rng(99)
    for n in (256, 4096, 14336):
        for scale in (1e-3, 1.0, 300.0):
            x = (rng.standard_normal(n) * scale).astype(np.float32)
            x[::97] = np.round(x[::97])  # some integral values
            assert np.array_equal(oracle.quantize_acts(x), reference.quantize_acts(x))
            if n % 256 == 0:
                assert np.array_equal(oracle.quantize_acts_k(x), reference.quantize_acts_k(x))
                assert np.array_equal(reference.quantize_acts_k(x), reference.quantize_acts_k(x, scalar=True))


def test_live_reference_model(oracle, reference, tiny_gguf):
    rm = reference.load(tiny_gguf, 2048)
    om = oracle.load(tiny_gguf, 2048)
    ids = np.random.default_rng(21).integers(3, 32000, 40).astype(np.int32)
    a, b = rm.forward(ids[:32], 0), om.forward(ids[:32], 0)
    assert np.abs(a - b).max() <= 0.02 * np.abs(a).max()
    for s in range(32, 40):
        a, b = rm.forward(ids[s:s + 1], s), om.forward(ids[s:s + 1], s)
        assert np.abs(a - b).max() <= 0.02 * np.abs(a).max()


def test_engine_noise_floor_between_cpu_engines(oracle, reference, tiny_gguf):
    """Two CPU implementations of the same algorithm (reference AVX2 vs the C
    restatement) on 128-token prompts: int8 activation rounding flips keep
    max |dlogit| near 0.02 while >= 95% of logits stay inside the north-star
    bar 1e-2 abs + 1e-3 rel. This floor calibrates the GPU parity criteria."""
    ids = np.random.default_rng(123).integers(3, 32000, 140).astype(np.int32)
    rm, om = reference.load(tiny_gguf, 2048), oracle.load(tiny_gguf, 2048)
    a = [rm.forward(ids[:128], 0)] + [rm.forward(ids[s:s + 1], s) for s in range(128, 140)]
    b = [om.forward(ids[:128], 0)] + [om.forward(ids[s:s + 1], s) for s in range(128, 140)]
    for x, y in zip(a, b):
        d = np.abs(x - y)
        assert d.max() <= 0.02 * np.abs(x).max()
        assert np.mean(d <= 1e-2 + 1e-3 * np.abs(x)) >= 0.95


def test_engine_noise_floor_llama8b_two_layers(oracle, reference, synth_dir):
    """Same measurement at the Llama-3-8B widths (2 layers, Q4_K_M mixture):
    the floor is much wider (the residual stream of a random-init model is
    small, so the final RMSNorm amplifies flips): per step 25-60% of logits
    inside the bar, max |dlogit| <= 3% of max |logit|, median <= 0.03."""
    from imurun_b200 import synth
    path = synth.cached(synth.preset("llama8b", layers=2), synth_dir)
    ids = np.random.default_rng(8).integers(3, 128256, 20).astype(np.int32)
    rm, om = reference.load(path, 1024), oracle.load(path, 1024)
    a = [rm.forward(ids[:16], 0)] + [rm.forward(ids[s:s + 1], s) for s in range(16, 20)]
    b = [om.forward(ids[:16], 0)] + [om.forward(ids[s:s + 1], s) for s in range(16, 20)]
    fr = []
    for x, y in zip(a, b):
        d = np.abs(x - y)
        assert d.max() <= 0.03 * np.abs(x).max()
        assert np.median(d) <= 0.03
        fr.append(np.mean(d <= 1e-2 + 1e-3 * np.abs(x)))
    assert 0.25 <= min(fr) and max(fr) <= 0.6


def test_live_reference_qwen3_qk_norm(oracle, reference, synth_dir):
    """The qwen3 layers (per-head q/k RMSNorm with non-unit weights, NeoX
    RoPE, no qkv bias): the restatement against the reference built here on
    the GPU test's ids and steps (prefill 10, 4 decode steps). Measured: 71-75%
    of logits inside 1e-2 + 1e-3|l| per step, max |dlogit| 1.4-1.6% of max
    |logit| (int8 rounding flips); held at >= 65% and <= 2.5%."""
    from imurun_b200 import synth
    path = synth.cached(synth.preset("qwen3", layers=2), synth_dir)
    ids = np.random.default_rng(11).integers(3, 32000, 14).astype(np.int32)
    rm, om = reference.load(path, 1024), oracle.load(path, 1024)
    qn = om.tensor_f32("blk.1.attn_q_norm.weight")
    assert qn is not None and qn.shape == (64,) and np.abs(qn - 1).max() > 0.1
    a = [rm.forward(ids[:10], 0)] + [rm.forward(ids[s:s + 1], s) for s in range(10, 14)]
    b = [om.forward(ids[:10], 0)] + [om.forward(ids[s:s + 1], s) for s in range(10, 14)]
    for x, y in zip(a, b):
        d = np.abs(x - y)
        assert d.max() <= 0.025 * np.abs(x).max()
        assert np.mean(d <= 1e-2 + 1e-3 * np.abs(x)) >= 0.65


@pytest.mark.parametrize("n_tok", [1, 5])
def test_live_reference_attention(oracle, reference, n_tok):
    rng = np.random.default_rng(n_tok)
    H, HKV, D, n_ctx, pos0 = 8, 2, 128, 64, 30
    q = rng.standard_normal((n_tok, H * D)).astype(np.float32)
    k = rng.standard_normal((n_ctx, HKV * D)).astype(np.float32)
    v = rng.standard_normal((n_ctx, HKV * D)).astype(np.float32)
    a = reference.attention(q, k, v, n_ctx, H, HKV, D, pos0, n_tok, 1 / np.sqrt(D))
    b = oracle.attention(q, k, v, H, HKV, D, pos0, n_tok, 1 / np.sqrt(D))
    assert np.abs(a - b).max() < 1e-5


@pytest.mark.parametrize("preset", ["gemma2", "phi3", "phi3-d96", "phi3-bias", "qwen2moe"])
def test_live_reference_arch_variants(oracle, reference, synth_dir, preset):
    """The restatement's gemma2 (norms stored as w - 1, embedding scale, GELU,
    post norms, score and logit soft caps, a 64-position window on even
    layers), phi3 (fused q|k|v and gate|up, longrope, head dimension 96, fused
    q|k|v and output biases) and qwen2moe (unnormalised top-k, gated shared
    expert) against the reference built here: a 70-id prompt (past the window)
    then 4 decode steps on 2-layer files. Measured on 4-layer files with a
    92-id prompt: max |dlogit| 1.5-2.6% of max |logit|, 58-80% of logits
    inside 1e-2 + 1e-3|l| per step; held at <= 3% and >= 50%, the argmax equal
    wherever the reference's top-2 margin clears twice the bar."""
    from imurun_b200 import synth
    path = synth.cached(synth.preset(preset, layers=2), synth_dir)
    ids = np.random.default_rng(29).integers(3, 32000, 74).astype(np.int32)
    rm, om = reference.load(path, 1024), oracle.load(path, 1024)
    a = [rm.forward(ids[:70], 0)] + [rm.forward(ids[s:s + 1], s) for s in range(70, 74)]
    b = [om.forward(ids[:70], 0)] + [om.forward(ids[s:s + 1], s) for s in range(70, 74)]
    for x, y in zip(a, b):
        d = np.abs(x - y)
        assert d.max() <= 0.03 * np.abs(x).max()
        assert np.mean(d <= 1e-2 + 1e-3 * np.abs(x)) >= 0.5
        top = np.sort(x)
        if top[-1] - top[-2] > 2 * (1e-2 + 1e-3 * np.abs(x).max()):
            assert int(np.argmax(x)) == int(np.argmax(y))


@pytest.mark.parametrize("preset", ["tiny", "gemma2", "phi3", "qwen2moe"])
def test_quality_metric_against_reference(oracle, reference, synth_dir, preset):
    """The reference's own GPU quality gate (test/test_gpu.cpp:597-631: top-1
    agreement >= 95% and KL(P_ref || P_other) per step), applied to the
    restatement: teacher-forced, a 32-id prompt then 64 decode steps.
    Measured: top-1 agreement 100% (tiny, gemma2), 95.4% (phi3), 96.9%
    (qwen2moe: near-ties of the random-init logits), KL mean 0.8-3.3e-5, max
    <= 7e-5; held at >= 95% and mean KL <= 1e-4, max <= 1e-3."""
    from imurun_b200 import synth
    cfg = synth.preset("tiny") if preset == "tiny" else synth.preset(preset, layers=2)
    path = synth.cached(cfg, synth_dir)
    ids = np.random.default_rng(31).integers(3, 32000, 96).astype(np.int32)
    rm, om = reference.load(path, 1024), oracle.load(path, 1024)
    a = [rm.forward(ids[:32], 0)] + [rm.forward(ids[s:s + 1], s) for s in range(32, 96)]
    b = [om.forward(ids[:32], 0)] + [om.forward(ids[s:s + 1], s) for s in range(32, 96)]

    def logp(x):
        x = x.astype(np.float64)
        x = x - x.max()
        return x - np.log(np.exp(x).sum())

    kl = [float(np.sum(np.exp(logp(x)) * (logp(x) - logp(y)))) for x, y in zip(a, b)]
    top1 = float(np.mean([np.argmax(x) == np.argmax(y) for x, y in zip(a, b)]))
    print(f"{preset}: top-1 {top1:.3f}, KL mean {np.mean(kl):.2e} max {max(kl):.2e}")
    assert top1 >= 0.95
    assert np.mean(kl) <= 1e-4 and max(kl) <= 1e-3


@pytest.mark.parametrize("n_tok,softcap,window", [(1, 0.5, 16), (5, 0.0, 8), (5, 2.0, 0), (7, 0.3, 40)])
def test_live_reference_attention_softcap_window(oracle, reference, n_tok, softcap, window):
    """Gemma-2's attention deltas in the restatement (ops.cpp attention_batch:
    cap * tanh(score / cap), keys pos - window + 1 .. pos) against the
    reference's own attention on the same rows."""
    rng = np.random.default_rng(n_tok + window)
    H, HKV, D, n_ctx, pos0 = 8, 4, 128, 64, 37
    q = rng.standard_normal((n_tok, H * D)).astype(np.float32)
    k = rng.standard_normal((n_ctx, HKV * D)).astype(np.float32)
    v = rng.standard_normal((n_ctx, HKV * D)).astype(np.float32)
    a = reference.attention(q, k, v, n_ctx, H, HKV, D, pos0, n_tok, 1 / np.sqrt(D), softcap, window)
    b = oracle.attention(q, k, v, H, HKV, D, pos0, n_tok, 1 / np.sqrt(D), softcap, window)
    assert np.abs(a - b).max() < 1e-5
    plain = oracle.attention(q, k, v, H, HKV, D, pos0, n_tok, 1 / np.sqrt(D))
    assert np.abs(b - plain).max() > 1e-3   # the cap / window change the output


def test_live_reference_activations(oracle, reference):
    """SiLU and gemma2's tanh-form GELU (ops.cpp:25-38): the restatement's
    values equal the reference's bit for bit over a wide input range."""
    import ctypes
    x = np.concatenate([np.linspace(-20, 20, 40001), np.random.default_rng(3).standard_normal(4096) * 4]).astype(np.float32)
    reference.L.ref_act.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
    oracle.L.or_gelu_inplace.argtypes = [ctypes.c_void_p, ctypes.c_int]
    oracle.L.or_silu_inplace.argtypes = [ctypes.c_void_p, ctypes.c_int]
    for gelu in (0, 1):
        a, b = x.copy(), x.copy()
        reference.L.ref_act(a.ctypes.data, a.size, gelu)
        (oracle.L.or_gelu_inplace if gelu else oracle.L.or_silu_inplace)(b.ctypes.data, b.size)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), gelu
