"""Kernel-level parity of the CUDA path against the CPU oracle, through the
C ABI (include/fish/fish_kernels.h). Integer and byte results must be
bit-exact; float results are compared with the tolerance written in each test.

Patterns follow the reference's kernel test (test/test_kernels.cpp:87-235):
rows of every integer-kernel type from random bytes with sane fp16 scales,
the four activation families, byte-identical activation quantisation and
dots within 1e-5 of sum |w x|.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

BSIZE = {8: 34, 12: 144, 14: 210, 0: 4, 1: 2}
BLK = {8: 32, 12: 256, 14: 256, 0: 1, 1: 1}
D_OFF = {8: (0, -1), 12: (0, 2), 14: (208, -1)}


@pytest.fixture(scope="module")
def lib():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from imurun_b200 import native
    return native.load_library()


def _p(a):
    return None if a is None else a.ctypes.data


def rand_rows(t: int, n_in: int, n_out: int, rng) -> np.ndarray:
    """Random bytes with sane fp16 scales (test/test_kernels.cpp:98-106)."""
    if t == 0:
        return rng.standard_normal((n_out, n_in)).astype(np.float32).view(np.uint8).reshape(n_out, -1)
    if t == 1:
        return rng.standard_normal((n_out, n_in)).astype(np.float16).view(np.uint8).reshape(n_out, -1)
    nb = n_in // BLK[t]
    rows = rng.integers(0, 256, (n_out, nb, BSIZE[t]), dtype=np.uint8)
    d_off, m_off = D_OFF[t]
    d = (0.001 + rng.uniform(size=(n_out, nb)) * 0.05).astype(np.float16).view(np.uint8).reshape(n_out, nb, 2)
    rows[:, :, d_off:d_off + 2] = d
    if m_off >= 0:
        m = (0.001 + rng.uniform(size=(n_out, nb)) * 0.05).astype(np.float16).view(np.uint8).reshape(n_out, nb, 2)
        rows[:, :, m_off:m_off + 2] = m
    return rows.reshape(n_out, -1)


def acts_family(n, kind, rng):
    if kind == 0:
        return rng.uniform(-2, 2, n).astype(np.float32)
    if kind == 1:
        return (rng.uniform(-1, 1, n) * np.where(rng.uniform(0, 1, n) < 0.01, 50.0, 1.0)).astype(np.float32)
    if kind == 2:
        i = np.arange(n)
        return np.where((i // 64) % 3 == 0, 0.0, rng.uniform(-0.01, 0.01, n)).astype(np.float32)
    i = np.arange(n)
    r = rng.integers(-126, 127, n).astype(np.float32) + 0.5 * rng.integers(0, 2, n)
    return np.where(i % 32 == 0, 127.0, r).astype(np.float32)


def test_quantizer_byte_identical_golden(lib, golden):
    for kind in range(4):
        for n in (256, 4096):
            x = golden[f"acts_x{kind}_{n}"]
            q32 = np.zeros(n // 32 * 40, np.uint8)
            qk = np.zeros(n // 256 * 276, np.uint8)
            assert lib.fbx_quantize_acts(_p(x), 1, n, _p(q32), _p(qk)) == 0
            assert np.array_equal(q32, golden[f"acts_q32_{kind}_{n}"]), (kind, n)
            assert np.array_equal(qk, golden[f"acts_qk_{kind}_{n}"]), (kind, n)


@pytest.mark.parametrize("K", [512, 1408, 4096, 14336, 28672])
def test_quantizer_byte_identical_oracle(lib, oracle, K):
    rng = np.random.default_rng(K)
    rows = 5
    x = np.stack([acts_family(K, k % 4, rng) * (10.0 ** (k - 2)) for k in range(rows)]).astype(np.float32)
    q32 = np.zeros(rows * K // 32 * 40, np.uint8)
    qk = np.zeros(rows * (K // 256) * 276, np.uint8) if K % 256 == 0 else None
    assert lib.fbx_quantize_acts(_p(x), rows, K, _p(q32), _p(qk)) == 0
    want32 = np.concatenate([oracle.quantize_acts(r) for r in x])
    assert np.array_equal(q32, want32)
    if qk is not None:
        wantk = np.concatenate([oracle.quantize_acts_k(r) for r in x])
        assert np.array_equal(qk, wantk)


@pytest.mark.parametrize("t,n_in", [(8, 512), (8, 1408), (12, 4096), (12, 14336), (14, 4096), (14, 3584), (12, 3584)])
def test_block_sums_bit_exact(lib, oracle, t, n_in):
    rng = np.random.default_rng(t * 1000 + n_in)
    n_out = 67
    w = rand_rows(t, n_in, n_out, rng)
    x = acts_family(n_in, 0, rng)
    acts = oracle.quantize_acts_k(x) if t in (12, 14) else oracle.quantize_acts(x)
    nb = n_in // BLK[t]
    s = np.zeros((n_out, nb), np.int32)
    m = np.zeros((n_out, nb), np.int32)
    assert lib.fbx_block_sums(t, _p(w), n_in, n_out, _p(acts), _p(s), _p(m)) == 0
    for r in range(n_out):
        ws, wm = oracle.block_sums(t, w[r], acts, n_in)
        assert np.array_equal(s[r], ws), (t, r)
        if t == 12:
            assert np.array_equal(m[r], wm), (t, r)


def test_block_sums_golden_rows(lib, golden, oracle):
    for name, t in (("Q8_0", 8), ("Q4_K", 12), ("Q6_K", 14)):
        for i in range(12):
            row, acts = golden[f"row_{name}_{i}"], golden[f"rowx_{name}_{i}"]
            n = 256 if i < 6 else 4096
            nb = n // BLK[t]
            s = np.zeros(nb, np.int32)
            m = np.zeros(nb, np.int32)
            assert lib.fbx_block_sums(t, _p(row), n, 1, _p(acts), _p(s), _p(m)) == 0
            ws, wm = oracle.block_sums(t, row, acts, n)
            assert np.array_equal(s, ws) and (t != 12 or np.array_equal(m, wm)), (name, i)


@pytest.mark.parametrize("t", [8, 12, 14, 0, 1])
@pytest.mark.parametrize("T", [1, 3, 8, 16, 29, 37, 130])
def test_matmul_vs_oracle(lib, oracle, t, T):
    """T < 16: GEMV kernels; T >= 16: the int8 tensor-core kernel for the
    quantised types, in its 16-, 32- and 64-token tiles (partial 64-row tiles
    at 300 rows, partial token tiles at T = 29, 37, 130)."""
    rng = np.random.default_rng(100 * t + T)
    n_in = 512 if t in (0, 1, 8) else 4096
    n_out = 300
    w = rand_rows(t, n_in, n_out, rng)
    x = rng.standard_normal((T, n_in)).astype(np.float32)
    y = np.zeros((T, n_out), np.float32)
    assert lib.fbx_matmul(t, _p(w), n_in, n_out, _p(x), T, _p(y)) == 0
    want = oracle.matmul(t, w, x, n_in, n_out)
    # mass-relative criterion of the reference kernel test: |dy| <= 1e-5 * sum|w||x|
    wd = np.stack([oracle.dequant(t, w[r], n_in) for r in range(n_out)])
    mass = np.abs(x) @ np.abs(wd).T + 1e-9
    assert np.all(np.abs(y - want) <= 1e-5 * mass), float(np.max(np.abs(y - want) / mass))


@pytest.mark.parametrize("t", [8, 12, 14])
@pytest.mark.parametrize("T", [16, 29])
def test_matmul_tall_small_batch(lib, oracle, t, T):
    """A matrix with more 64-row tiles than SMs (9500 rows): the tensor-core
    kernel's 64-row tiles with 16- and 32-token widths (smaller matrices take
    32-row tiles), against the oracle."""
    rng = np.random.default_rng(31 * t + T)
    n_in, n_out = 256, 9500
    w = rand_rows(t, n_in, n_out, rng)
    x = rng.standard_normal((T, n_in)).astype(np.float32)
    y = np.zeros((T, n_out), np.float32)
    assert lib.fbx_matmul(t, _p(w), n_in, n_out, _p(x), T, _p(y)) == 0
    want = oracle.matmul(t, w, x, n_in, n_out)
    wd = np.stack([oracle.dequant(t, w[r], n_in) for r in range(n_out)])
    mass = np.abs(x) @ np.abs(wd).T + 1e-9
    assert np.all(np.abs(y - want) <= 1e-5 * mass), float(np.max(np.abs(y - want) / mass))


@pytest.mark.parametrize("t", [8, 12, 14])
@pytest.mark.parametrize("n_in", [4096, 3584, 2816, 18944])
@pytest.mark.parametrize("T", [16, 29, 37, 70])
def test_matmul_rows_batch_invariant(lib, t, n_in, T):
    """A token's outputs are the same bits whatever the number of tokens in
    the call: the tensor-core kernels (T = 16: a 16-token tile; 29: a
    32-token tile; 37, 70: the tcgen05 kernel's 64-token tiles for Q4_K) add
    each block's float term in the GEMV kernels' order (pairwise over a
    group's blocks, groups in order, +0 for a short last group: 3584 = 1 full
    + 1 partial group), so they match the streamed GEMV (T = 1) exactly. With
    200 rows the tcgen05 kernel splits K over CTAs in half-group units
    (2816: an odd unit count, the last group's second half missing; 18944:
    19 units) and the reduce adds the halves and the groups in the same
    order. This is what makes a prefix-cache hit reproduce a fresh prefill
    bit for bit."""
    rng = np.random.default_rng(7 * t + n_in)
    n_out = 200
    w = rand_rows(t, n_in, n_out, rng)
    x = rng.standard_normal((T, n_in)).astype(np.float32)
    y = np.zeros((T, n_out), np.float32)
    assert lib.fbx_matmul(t, _p(w), n_in, n_out, _p(x), T, _p(y)) == 0
    for i in (0, 5, T // 2, T - 1):
        y1 = np.zeros((1, n_out), np.float32)
        xi = np.ascontiguousarray(x[i:i + 1])
        assert lib.fbx_matmul(t, _p(w), n_in, n_out, _p(xi), 1, _p(y1)) == 0
        assert np.array_equal(y[i], y1[0]), (i, float(np.abs(y[i] - y1[0]).max()))


def test_rmsnorm_vs_oracle(lib, oracle):
    rng = np.random.default_rng(5)
    for K in (512, 4096, 8192):
        x = (rng.standard_normal((3, K)) * 0.05).astype(np.float32)
        w = rng.uniform(0.5, 1.5, K).astype(np.float32)
        out = np.zeros_like(x)
        assert lib.fbx_rmsnorm(_p(x), _p(w), 3, K, 1e-5, _p(out)) == 0
        want = np.stack([oracle.rmsnorm(r, w, 1e-5) for r in x])
        # double-precision sum of squares in both; results agree to 1 ulp
        assert np.max(np.abs(out - want)) <= 2e-7 * np.max(np.abs(want))


@pytest.mark.parametrize("neox", [0, 1])
def test_rope_bit_exact(lib, oracle, neox):
    rng = np.random.default_rng(9 + neox)
    T, H, HKV, D, pos0 = 5, 8, 2, 128, 37
    q = rng.standard_normal((T, H * D)).astype(np.float32)
    k = rng.standard_normal((T, HKV * D)).astype(np.float32)
    qg, kg = q.copy(), k.copy()
    assert lib.fbx_rope(_p(qg), _p(kg), T, H, HKV, D, D, neox, 500000.0, pos0) == 0
    # oracle: table built like rope_build, rotation like rope_apply
    import ctypes as C

    class RP(C.Structure):
        _fields_ = [("head_dim", C.c_int), ("rot_dim", C.c_int), ("neox", C.c_int), ("freq_base", C.c_float),
                    ("freq_scale", C.c_float), ("mscale", C.c_float), ("yarn_factor", C.c_float),
                    ("yarn_attn_factor", C.c_float), ("yarn_beta_fast", C.c_float), ("yarn_beta_slow", C.c_float),
                    ("yarn_orig_ctx", C.c_int), ("freq_factors", C.c_void_p)]
    n_ctx = pos0 + T
    cs = np.zeros(n_ctx * D // 2, np.float32)
    sn = np.zeros_like(cs)
    rp = RP(D, D, neox, 500000.0, 1.0, 1.0, 0.0, 1.0, 32.0, 1.0, 0, None)
    oracle.L.or_rope_build.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
    oracle.L.or_rope_build(_p(cs), _p(sn), n_ctx, C.addressof(rp))
    for t in range(T):
        pos = pos0 + t
        qo, ko = q[t].copy(), k[t].copy()
        oracle.L.or_rope_apply(_p(qo), _p(ko), H, HKV, D, D, neox, cs[pos * D // 2:].ctypes.data,
                               sn[pos * D // 2:].ctypes.data)
        assert np.array_equal(qg[t], qo)
        assert np.array_equal(kg[t], ko)


@pytest.mark.parametrize("f16", [0, 1])
@pytest.mark.parametrize("T,pos0,H,HKV,D", [(1, 0, 8, 4, 64), (1, 300, 32, 8, 128), (7, 120, 28, 4, 128),
                                            (33, 0, 8, 8, 64), (1, 1000, 64, 8, 128), (9, 70, 12, 4, 96),
                                            (1, 2500, 32, 32, 96)])
def test_attention_vs_oracle(lib, oracle, f16, T, pos0, H, HKV, D):
    rng = np.random.default_rng(T + pos0 + H)
    n_keys = pos0 + T
    q = rng.standard_normal((T, H * D)).astype(np.float32)
    k = rng.standard_normal((n_keys, HKV * D)).astype(np.float32)
    v = rng.standard_normal((n_keys, HKV * D)).astype(np.float32)
    out = np.zeros((T, H * D), np.float32)
    assert lib.fbx_attention(_p(q), _p(k), _p(v), n_keys, H, HKV, D, pos0, T, f16, _p(out)) == 0
    if f16:
        k, v = oracle.fp16_round(k), oracle.fp16_round(v)
    want = oracle.attention(q, k, v, H, HKV, D, pos0, T, 1.0 / np.sqrt(D))
    # online-softmax vs two-pass softmax in float: 2e-5 of the output scale
    assert np.max(np.abs(out - want)) <= 2e-5 * max(1.0, np.max(np.abs(want)))


@pytest.mark.parametrize("T,pos0,H,HKV,D", [(5, 0, 8, 4, 64), (16, 40, 32, 8, 128), (37, 120, 28, 4, 128),
                                            (70, 1000, 64, 8, 128), (256, 256, 32, 8, 128), (33, 7, 8, 8, 64),
                                            (19, 63, 16, 2, 128), (21, 100, 32, 32, 96), (40, 0, 12, 4, 96)])
def test_attention_prefill_tc_vs_oracle(lib, oracle, T, pos0, H, HKV, D):
    """The tensor-core prefill kernel (16 tokens x kv head per CTA, 64-key
    tiles, q and p as f16 hi + lo parts) against the oracle's attention on the
    same fp16 cache, with the attention tests' bar (2e-5 of the output scale):
    partial query tiles, key tiles cut by the causal mask, G = 1 .. 8."""
    rng = np.random.default_rng(T + pos0 + H + 5)
    n_keys = pos0 + T
    q = rng.standard_normal((T, H * D)).astype(np.float32)
    k = rng.standard_normal((n_keys, HKV * D)).astype(np.float32)
    v = rng.standard_normal((n_keys, HKV * D)).astype(np.float32)
    out = np.zeros((T, H * D), np.float32)
    assert lib.fbx_attention_prefill(_p(q), _p(k), _p(v), n_keys, H, HKV, D, pos0, T, _p(out)) == 0
    k16, v16 = oracle.fp16_round(k), oracle.fp16_round(v)
    want = oracle.attention(q, k16, v16, H, HKV, D, pos0, T, 1.0 / np.sqrt(D))
    assert np.max(np.abs(out - want)) <= 2e-5 * max(1.0, np.max(np.abs(want)))
    # a token's row does not depend on the other tokens of the call (what a
    # prefix-cache hit relies on): the last rows alone, same cache, same bits
    a = T // 2
    tail = np.zeros((T - a, H * D), np.float32)
    qt = np.ascontiguousarray(q[a:])
    assert lib.fbx_attention_prefill(_p(qt), _p(k), _p(v), n_keys, H, HKV, D, pos0 + a, T - a, _p(tail)) == 0
    assert np.array_equal(tail, out[a:])


@pytest.mark.parametrize("f16", [0, 1])
@pytest.mark.parametrize("pos,H,HKV,D,rot,neox", [(0, 8, 4, 64, 64, 0), (37, 32, 8, 128, 128, 0),
                                                  (200, 28, 4, 128, 128, 1), (1000, 64, 8, 128, 128, 0),
                                                  (3000, 8, 8, 64, 32, 1), (70, 16, 2, 128, 64, 0),
                                                  (300, 32, 32, 96, 96, 1), (65, 12, 4, 96, 96, 0),
                                                  (1000, 8, 8, 96, 64, 1)])
def test_fused_decode_attention(lib, oracle, f16, pos, H, HKV, D, rot, neox):
    """RoPE + KV append + attention in one kernel vs the unfused pieces:
    RoPE on the GPU (bit-exact with the oracle, test_rope_bit_exact) then the
    oracle's attention; the appended row is bit-exact."""
    rng = np.random.default_rng(pos + H + D + f16)
    base = 500000.0
    q = rng.standard_normal(H * D).astype(np.float32)
    kc = rng.standard_normal((max(pos, 1), HKV * D)).astype(np.float32)
    vc = rng.standard_normal((max(pos, 1), HKV * D)).astype(np.float32)
    kn = rng.standard_normal(HKV * D).astype(np.float32)
    vn = rng.standard_normal(HKV * D).astype(np.float32)
    out = np.zeros(H * D, np.float32)
    ks = np.zeros(HKV * D, np.float32)
    vs = np.zeros(HKV * D, np.float32)
    assert lib.fbx_attention_decode(_p(q), _p(kc), _p(vc), _p(kn), _p(vn), pos, H, HKV, D, rot, neox, base, f16,
                                    _p(out), _p(ks), _p(vs)) == 0
    qr, kr = q.copy(), kn.copy()
    assert lib.fbx_rope(_p(qr), _p(kr), 1, H, HKV, D, rot, neox, base, pos) == 0
    rnd = oracle.fp16_round if f16 else (lambda a: a)
    assert np.array_equal(ks, rnd(kr)) and np.array_equal(vs, rnd(vn))
    keys = rnd(np.concatenate([kc[:pos], kr[None, :]]))
    vals = rnd(np.concatenate([vc[:pos], vn[None, :]]))
    want = oracle.attention(qr[None, :], keys, vals, H, HKV, D, pos, 1, 1.0 / np.sqrt(D))[0]
    # online softmax over blocks and a cluster merge vs the two-pass softmax
    assert np.max(np.abs(out - want)) <= 2e-5 * max(1.0, np.max(np.abs(want)))


def test_argmax_first_index(lib):
    x = np.zeros((3, 100000), np.float32)
    x[0, 5] = 1.0
    x[1, 7] = 2.0
    x[1, 99999] = 2.0
    x[2, :] = -1.0
    out = np.zeros(3, np.int32)
    assert lib.fbx_argmax(_p(x), 3, 100000, _p(out)) == 0
    assert list(out) == [5, 7, 0]


@pytest.mark.parametrize("vocab,pen,last_n", [(32000, 1.1, 64), (128256, 1.3, 64), (152064, 0.8, 32),
                                               (1000, 1.1, 200), (50000, 1.0, 64)])
def test_argmax_penalized_matches_host_sampler(lib, vocab, pen, last_n):
    """The generation loop's greedy branch on the device (penalty per
    occurrence in the window, then the first index of the maximum) equals
    the host sampler's (fbx_sample at temperature 0, pinned to the
    reference's Sampler::sample on the CPU), recent ids repeated and the
    penalised ids among the likely ones."""
    lib.fbx_sample.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_float,
                               ctypes.c_float, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_ulonglong,
                               ctypes.c_int, ctypes.c_void_p]
    lib.fbx_sample.restype = ctypes.c_int
    rng = np.random.default_rng(vocab + int(pen * 10))
    for trial in range(20):
        logits = (rng.standard_normal(vocab) * 2.0).astype(np.float32)
        recent = rng.integers(0, vocab, 128).astype(np.int32)
        recent[-10:-5] = recent[-5:]                      # repeats: penalised twice
        logits[recent[-6:]] = np.abs(logits[recent[-6:]]) + 6.0 + 0.01 * trial
        logits[recent[-1]] = -logits[recent[-1]]          # a negative penalised logit
        if trial % 5 == 0:
            logits[7] = logits.max()                       # ties resolve to the first index
        want = np.zeros(1, np.int32)
        assert lib.fbx_sample(_p(logits), vocab, 0.0, 40, 0.9, pen, last_n, _p(recent), recent.size, 1, 1,
                              _p(want)) == 0
        window = recent[max(0, recent.size - last_n):].copy()
        got = np.zeros(1, np.int32)
        assert lib.fbx_argmax_penalized(_p(logits), vocab, _p(window), window.size, pen, _p(got)) == 0
        assert int(got[0]) == int(want[0]), (trial, int(got[0]), int(want[0]))


@pytest.mark.parametrize("t", [8, 12, 14])
def test_embed_dequant_bit_exact(lib, oracle, t):
    rng = np.random.default_rng(t)
    E, n_rows = 512, 50
    w = rand_rows(t, E, n_rows, rng)
    ids = np.array([0, 49, 7, 7, 23], np.int32)
    out = np.zeros((ids.size, E), np.float32)
    assert lib.fbx_embed(t, _p(w), E, n_rows, _p(ids), ids.size, _p(out)) == 0
    for i, r in enumerate(ids):
        assert np.array_equal(out[i], oracle.dequant(t, w[r], E))
