"""fbx_attention_static — the attention entry point that allocates nothing —
against fbx_attention (which allocates its own device buffers) and against
the CPU oracle's attention on the same inputs, through the C ABI, on two
calls in a row.

The file name sorts last so it also runs after every other test in one
process; it must pass alone in a fresh process too. Device buffers for the
inputs are the test's own (torch); the entry point itself takes them as plain
pointers and allocates nothing.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from imurun_b200 import native
    return native.load_library(), torch


@pytest.fixture(scope="module")
def oracle():
    from oracle.binding import Oracle
    return Oracle()


def _p(a):
    return a.ctypes.data


def _host_reference(lib, q, k, v, n_keys, H, HKV, D, pos0, T, f16):
    out = np.zeros((T, H * D), np.float32)
    rc = lib.fbx_attention(_p(q), _p(k), _p(v), n_keys, H, HKV, D, pos0, T, f16, _p(out))
    assert rc == 0
    return out


# (T, pos0, H, HKV, D): decode at a short and a long context (1 and 4 warps
# per split), a small prefill chunk, MHA with D = 64, and a 16-token chunk
# just past 2048 keys (the documented partials limit admits it).
SHAPES = [(1, 300, 32, 8, 128), (1, 3000, 32, 8, 128), (7, 120, 28, 4, 128), (5, 0, 8, 8, 64),
          (16, 2984, 32, 8, 128)]


@pytest.mark.parametrize("f16", [0, 1])
@pytest.mark.parametrize("T,pos0,H,HKV,D", SHAPES)
def test_static_matches_allocating_entry(env, oracle, f16, T, pos0, H, HKV, D):
    lib, torch = env
    dev = torch.device("cuda:0")
    n_keys = pos0 + T
    stream = torch.cuda.current_stream(dev)
    for call in range(2):   # two calls in a row share the static scratch
        rng = np.random.default_rng(1000 * call + T + pos0 + H + f16)
        q = rng.standard_normal((T, H * D)).astype(np.float32)
        k = rng.standard_normal((n_keys, HKV * D)).astype(np.float32)
        v = rng.standard_normal((n_keys, HKV * D)).astype(np.float32)
        want = _host_reference(lib, q, k, v, n_keys, H, HKV, D, pos0, T, f16)
        kv_dtype = torch.float16 if f16 else torch.float32
        dq = torch.from_numpy(q).to(dev)
        dk = torch.from_numpy(k).to(dev, kv_dtype)
        dv = torch.from_numpy(v).to(dev, kv_dtype)
        dout = torch.full((T, H * D), float("nan"), dtype=torch.float32, device=dev)
        torch.cuda.synchronize(dev)
        rc = lib.fbx_attention_static(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), f16, n_keys, H, HKV, D, pos0, T,
                                      dout.data_ptr(), stream.cuda_stream)
        assert rc == 0
        torch.cuda.synchronize(dev)
        got = dout.cpu().numpy()
        # same kernels and split layout as fbx_attention; the attention tests'
        # tolerance (2e-5 of the output scale) is the bar
        assert np.all(np.isfinite(got))
        assert np.max(np.abs(got - want)) <= 2e-5 * max(1.0, float(np.max(np.abs(want))))
        # and against the CPU oracle (cache values rounded to fp16 when the
        # cache is fp16), with the attention tests' bar
        if f16:
            k, v = oracle.fp16_round(k), oracle.fp16_round(v)
        ref = oracle.attention(q, k, v, H, HKV, D, pos0, T, 1.0 / np.sqrt(D))
        assert np.max(np.abs(got - ref)) <= 2e-5 * max(1.0, float(np.max(np.abs(ref))))


def test_static_rejects_oversize(env):
    lib, torch = env
    dev = torch.device("cuda:0")
    buf = torch.zeros(16, dtype=torch.float32, device=dev)
    p = buf.data_ptr()
    # more keys than the static page table holds
    assert lib.fbx_attention_static(p, p, p, 0, 9000, 8, 8, 64, 8999, 1, p, None) == -1
    # more tokens than the static position table holds
    assert lib.fbx_attention_static(p, p, p, 0, 300, 8, 8, 64, 0, 300, p, None) == -1
    # partials beyond 2^21 floats: 256 tokens x 64 heads x 64 splits x 130
    assert lib.fbx_attention_static(p, p, p, 0, 8192, 64, 8, 128, 7936, 256, p, None) == -1
    # misaligned pointer
    assert lib.fbx_attention_static(p + 4, p, p, 0, 1, 8, 8, 64, 0, 1, p, None) == -1


def test_static_allocates_nothing(env):
    """After the first call (which resolves the static scratch's address),
    calls of every shape leave the device's free memory and torch's
    reservation unchanged: the entry point allocates nothing."""
    lib, torch = env
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream(dev)
    bufs = []
    for T, pos0, H, HKV, D in SHAPES:
        n_keys = pos0 + T
        g = torch.Generator(device=dev).manual_seed(T + pos0)
        q = torch.randn((T, H * D), device=dev, generator=g)
        k = torch.randn((n_keys, HKV * D), device=dev, generator=g).half()
        v = torch.randn((n_keys, HKV * D), device=dev, generator=g).half()
        out = torch.empty((T, H * D), device=dev)
        bufs.append((q, k, v, out, T, pos0, H, HKV, D))

    def call(b):
        q, k, v, out, T, pos0, H, HKV, D = b
        return lib.fbx_attention_static(q.data_ptr(), k.data_ptr(), v.data_ptr(), 1, pos0 + T, H, HKV, D, pos0, T,
                                        out.data_ptr(), stream.cuda_stream)

    assert call(bufs[0]) == 0
    torch.cuda.synchronize(dev)
    free0, _ = torch.cuda.mem_get_info(dev)
    reserved0 = torch.cuda.memory_reserved(dev)
    for _ in range(10):
        for b in bufs:
            assert call(b) == 0
    torch.cuda.synchronize(dev)
    free1, _ = torch.cuda.mem_get_info(dev)
    assert free1 == free0, (free0, free1)
    assert torch.cuda.memory_reserved(dev) == reserved0
    assert all(bool(torch.isfinite(b[3]).all()) for b in bufs)
