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
    (0.0, 40, 0.9, 1.1, 64), (0.8, 1, 0.9, 1.1, 64), (1.0, 40, 0.0, 1.2, 0)]


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
    if temp > 0 and top_k != 1 and top_p >= 0.5:
        assert len(set(want.tolist())) > 1    # the draws do vary: the generator is exercised


def test_bad_arguments(libs):
    _, ours = libs
    assert ours.fbx_sample(None, 10, 1.0, 0, 1.0, 1.0, 64, None, 0, 1, 1, None) == -1
