"""Sampler parity with the reference on the CPU: the same logits, parameters,
recent-token window and seed through this library's fbx_sample and the
reference's own Sampler::sample (oracle/_ref, ref_sample), draw after draw
with one generator each. Both seed a std::mt19937_64 with the seed, so equal
ids mean the penalty, temperature, top-k, top-p and draw steps agree."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from imurun_b200 import native

P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
ARGS = [P, I, F, I, F, F, I, P, I, ctypes.c_uint64, I, P]
PARAMS = [  # temperature, top_k, top_p, repeat_penalty, repeat_last_n
    (0.7, 40, 0.9, 1.1, 64), (1.0, 0, 1.0, 1.0, 64), (0.2, 5, 0.95, 1.3, 8), (1.5, 100, 0.5, 1.0, 64),
    (0.0, 40, 0.9, 1.1, 64), (0.8, 1, 0.9, 1.1, 64), (1.0, 40, 0.0, 1.2, 0),
    # edges: a tiny temperature, top-k past the vocabulary, a penalty below 1,
    # a window longer than the recent ids, a non-positive penalty (ignored)
    (0.01, 0, 1.0, 1.0, 64), (1.0, 50000, 1.0, 1.0, 64), (0.7, 40, 0.9, 0.5, 64), (0.7, 40, 0.9, 1.1, 500),
    (0.9, 20, 0.8, 0.0, 64)]


@pytest.fixture(scope="module")
def libs():
    from oracle.binding import REF_SO
    if not REF_SO.exists():
        pytest.skip("reference build (oracle/_ref) not present")
    ref = ctypes.CDLL(str(REF_SO))
    ref.ref_sample.argtypes = ARGS
    ref.ref_sample.restype = None
    ours = native.load_library()
    ours.fbx_sample.argtypes = ARGS
    ours.fbx_sample.restype = I
    return ref, ours


@pytest.mark.parametrize("vocab", [1000, 32000])
@pytest.mark.parametrize("k", range(len(PARAMS)))
def test_sampler_matches_reference(libs, vocab, k):
    ref, ours = libs
    temp, top_k, top_p, pen, last_n = PARAMS[k]
    rng = np.random.default_rng(100 * k + vocab)
    logits = (rng.standard_normal(vocab) * 3.0).astype(np.float32)
    recent = rng.integers(0, vocab, 90).astype(np.int32)
    logits[recent[-5:]] += 4.0          # some recent ids among the likely ones: the penalty matters
    n = 64
    want = np.zeros(n, np.int32)
    got = np.zeros(n, np.int32)
    ref.ref_sample(logits.ctypes.data, vocab, temp, top_k, top_p, pen, last_n, recent.ctypes.data, recent.size,
                   4242 + k, n, want.ctypes.data)
    assert ours.fbx_sample(logits.ctypes.data, vocab, temp, top_k, top_p, pen, last_n, recent.ctypes.data,
                           recent.size, 4242 + k, n, got.ctypes.data) == 0
    assert np.array_equal(got, want), (list(got[:16]), list(want[:16]))
    if temp >= 0.5 and top_k != 1 and top_p >= 0.5 and pen >= 1.0:
        assert len(set(want.tolist())) > 1    # the draws do vary: the generator is exercised


def test_bad_arguments(libs):
    _, ours = libs
    assert ours.fbx_sample(None, 10, 1.0, 0, 1.0, 1.0, 64, None, 0, 1, 1, None) == -1


@pytest.fixture(scope="module")
def dist_libs(libs):
    ref, ours = libs
    dargs = [P, I, F, I, F, F, I, P, I, P]
    ref.ref_distribution.argtypes = dargs
    ref.ref_distribution.restype = None
    ours.fbx_sample_distribution.argtypes = dargs
    ours.fbx_sample_distribution.restype = I
    wargs = [P, I, ctypes.c_uint64, I, P]
    ref.ref_draw.argtypes = wargs
    ref.ref_draw.restype = None
    ours.fbx_sample_draw.argtypes = wargs
    ours.fbx_sample_draw.restype = I
    return ref, ours


@pytest.mark.parametrize("vocab", [1000, 32000])
@pytest.mark.parametrize("k", range(len(PARAMS)))
def test_distribution_matches_reference(dist_libs, vocab, k):
    """Speculative decoding's acceptance test compares the target's and the
    draft's sampling distributions (reference sampler.cpp:42-89): the same
    probabilities, bit for bit, over the whole vocabulary."""
    ref, ours = dist_libs
    temp, top_k, top_p, pen, last_n = PARAMS[k]
    rng = np.random.default_rng(7 * k + vocab)
    logits = (rng.standard_normal(vocab) * 3.0).astype(np.float32)
    recent = rng.integers(0, vocab, 90).astype(np.int32)
    logits[recent[-5:]] += 4.0
    want = np.full(vocab, -1.0, np.float32)
    got = np.full(vocab, -2.0, np.float32)
    ref.ref_distribution(logits.ctypes.data, vocab, temp, top_k, top_p, pen, last_n, recent.ctypes.data,
                         recent.size, want.ctypes.data)
    assert ours.fbx_sample_distribution(logits.ctypes.data, vocab, temp, top_k, top_p, pen, last_n,
                                        recent.ctypes.data, recent.size, got.ctypes.data) == 0
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert abs(float(got.sum(dtype=np.float64)) - 1.0) < 1e-5
    if temp <= 0 or top_k == 1:
        assert np.count_nonzero(got) == 1


@pytest.mark.parametrize("case", ["dense", "sparse", "one", "none"])
def test_draw_matches_reference(dist_libs, case):
    """Sampler::draw (reference sampler.cpp:91-105): an index in proportion to
    the positive weights, -1 when none is positive, from the seeded stream."""
    ref, ours = dist_libs
    rng = np.random.default_rng(11)
    n = 5000
    w = rng.random(n).astype(np.float32)
    if case == "sparse":
        w[rng.random(n) < 0.95] = 0.0
        w[:10] = -1.0                      # negative weights count as zero
    elif case == "one":
        w[:] = 0.0
        w[1234] = 0.5
    elif case == "none":
        w[:] = 0.0
    want = np.zeros(200, np.int32)
    got = np.zeros(200, np.int32)
    ref.ref_draw(w.ctypes.data, n, 99, want.size, want.ctypes.data)
    assert ours.fbx_sample_draw(w.ctypes.data, n, 99, got.size, got.ctypes.data) == 0
    assert np.array_equal(got, want)
    if case == "none":
        assert (got == -1).all()
    elif case == "one":
        assert (got == 1234).all()
    else:
        assert (w[got] > 0).all()


@pytest.mark.parametrize("case", ["close", "far", "disjoint", "greedy"])
def test_speculative_rejection_rule_keeps_the_target_distribution(case):
    """Speculative decoding commits a draft token d ~ q with probability
    min(1, p(d)/q(d)) and otherwise a draw from max(0, p - q): the committed
    token is distributed as the target's p whatever the draft's q (reference
    c_api.cpp:719-741). 200k trials through the library's own step; every
    token's frequency within 5 standard errors of p."""
    lib = native.load_library()
    lib.fbx_speculative_draws.argtypes = [P, P, I, ctypes.c_uint64, I, P]
    lib.fbx_speculative_draws.restype = I
    rng = np.random.default_rng(5)
    n = 24
    p = rng.random(n) ** 3
    q = p * rng.uniform(0.7, 1.3, n) if case == "close" else rng.random(n) ** 3
    if case == "disjoint":          # no overlap: every draft is rejected
        p[n // 2:] = 0.0
        q[:n // 2] = 0.0
    if case == "greedy":            # one-hot target and draft disagreeing
        p = np.zeros(n)
        p[3] = 1.0
        q = np.zeros(n)
        q[5] = 1.0
    p = (p / p.sum()).astype(np.float32)
    q = (q / q.sum()).astype(np.float32)
    trials = 200_000
    out = np.zeros(trials, np.int32)
    assert lib.fbx_speculative_draws(p.ctypes.data, q.ctypes.data, n, 1234, trials, out.ctypes.data) == 0
    assert (out >= 0).all() and (out < n).all()
    freq = np.bincount(out, minlength=n) / trials
    se = np.sqrt(p * (1 - p) / trials) + 1e-7
    assert (np.abs(freq - p) <= 5 * se).all(), np.max(np.abs(freq - p) / se)
    assert (freq[p == 0] == 0).all()
    assert lib.fbx_speculative_draws(None, q.ctypes.data, n, 1, 1, out.ctypes.data) == -1
