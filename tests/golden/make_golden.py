"""Generate tests/golden/golden.npz from the REFERENCE FISH build.

Run in a checkout where oracle/_ref/libfish_ref.so has been built from the
reference sources (`make -C oracle ref`):

    python tests/golden/make_golden.py

Contents (all produced by the reference engine's own code paths):
  acts_x{kind}_{n}      f32 inputs, the four activation families of the
                        reference's kernel test (test/test_kernels.cpp:135-152)
  acts_q32_{kind}_{n}   Q8Act bytes  (quantize_acts, quant.cpp:400-415)
  acts_qk_{kind}_{n}    Q8ActK bytes (quantize_acts_k, quant.cpp:417-434)
  row_{T}_{i}           weight rows: mode 0 = reference quantize_row of random
                        floats, mode 1 = random bytes with sane fp16 scales
                        (test/test_kernels.cpp:87-107)
  rowx_{T}_{i}          the activation bytes used with that row
  rowdot_{T}_{i}        the reference int8 dot (vec_dot_q8 / vec_dot_q8k)
  rowdeq_{T}_{i}        the reference dequantised row (dequant_row), 256-wide rows
  q4k_kat               test/test_m1.cpp:35-71 hand-built Q4_K block
  tiny_ids / tiny_logits  teacher-forced logits of the tiny synthetic model
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle.binding import Reference  # noqa: E402
from imurun_b200 import synth  # noqa: E402

TYPES = {"Q4_0": 2, "Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14}
D_OFF = {2: (0, -1), 8: (0, -1), 12: (0, 2), 13: (0, 2), 14: (208, -1)}
BSIZE = {2: 18, 8: 34, 12: 144, 13: 176, 14: 210}
BLK = {2: 32, 8: 32, 12: 256, 13: 256, 14: 256}


def make_acts(n: int, kind: int, rng: np.random.Generator) -> np.ndarray:
    """The four activation families of test/test_kernels.cpp:135-152."""
    if kind == 0:
        return rng.uniform(-2, 2, n).astype(np.float32)
    if kind == 1:
        x = rng.uniform(-1, 1, n)
        x *= np.where(rng.uniform(0, 1, n) < 0.01, 50.0, 1.0)
        return x.astype(np.float32)
    if kind == 2:
        i = np.arange(n)
        return np.where((i // 64) % 3 == 0, 0.0, rng.uniform(-0.01, 0.01, n)).astype(np.float32)
    i = np.arange(n)
    r = rng.integers(-126, 127, n).astype(np.float32) + 0.5 * rng.integers(0, 2, n)
    return np.where(i % 32 == 0, 127.0, r).astype(np.float32)


def fp16_bytes(v: float) -> bytes:
    return np.array([v], np.float16).tobytes()


def make_row(ref: Reference, t: int, n: int, mode: int, rng: np.random.Generator) -> np.ndarray:
    if mode == 0:
        w = rng.uniform(-1, 1, n) * np.where(rng.uniform(0, 1, n) < 0.02, 8.0, 1.0)
        return ref.quantize_row(t, w.astype(np.float32))
    row = rng.integers(0, 256, n // BLK[t] * BSIZE[t], dtype=np.uint8)
    d_off, m_off = D_OFF[t]
    for off in range(0, row.size, BSIZE[t]):
        row[off + d_off: off + d_off + 2] = np.frombuffer(fp16_bytes(0.001 + rng.uniform() * 0.05), np.uint8)
        if m_off >= 0:
            row[off + m_off: off + m_off + 2] = np.frombuffer(fp16_bytes(0.001 + rng.uniform() * 0.05), np.uint8)
    return row


def main() -> None:
    ref = Reference()
    out: dict[str, np.ndarray] = {}
    rng = np.random.default_rng(7)
    for kind in range(4):
        for n in (256, 4096):
            x = make_acts(n, kind, rng)
            out[f"acts_x{kind}_{n}"] = x
            out[f"acts_q32_{kind}_{n}"] = ref.quantize_acts(x)
            out[f"acts_qk_{kind}_{n}"] = ref.quantize_acts_k(x)
    for name, t in TYPES.items():
        rng = np.random.default_rng(1000 + t)
        i = 0
        for n in (256, 4096):
            for r in range(6):
                row = make_row(ref, t, n, r & 1, rng)
                x = make_acts(n, r % 3, rng)
                acts = ref.quantize_acts_k(x) if BLK[t] == 256 else ref.quantize_acts(x)
                out[f"row_{name}_{i}"] = row
                out[f"rowx_{name}_{i}"] = acts
                out[f"rowdot_{name}_{i}"] = np.array([ref.vec_dot(t, row, acts, n)], np.float32)
                if n == 256:
                    deq = np.zeros(n, np.float32)
                    ref.L.ref_dequant_row(t, row.ctypes.data, deq.ctypes.data, n)
                    out[f"rowdeq_{name}_{i}"] = deq
                i += 1
    # test/test_m1.cpp:35-71: d = 1, all scales 1, mins 0, nibble = l & 15.
    kat = np.zeros(144, np.uint8)
    kat[0:2] = np.frombuffer(fp16_bytes(1.0), np.uint8)
    for j in (0, 1, 2, 3, 8, 9, 10, 11):
        kat[4 + j] = 1
    for i in range(128):
        nib = i & 15
        kat[16 + i] = nib | (nib << 4)
    out["q4k_kat"] = kat
    deq = np.zeros(256, np.float32)
    ref.L.ref_dequant_row(12, kat.ctypes.data, deq.ctypes.data, 256)
    out["q4k_kat_deq"] = deq

    path = synth.cached(synth.preset("tiny"))
    m = ref.load(path, 2048)
    ids = np.random.default_rng(11).integers(3, 32000, 18).astype(np.int32)
    out["tiny_ids"] = ids
    logits = [m.forward(ids[:16], 0)]
    for s in range(16, 18):
        logits.append(m.forward(ids[s:s + 1], s))
    out["tiny_logits"] = np.stack(logits).astype(np.float32)
    np.savez_compressed(Path(__file__).with_name("golden.npz"), **out)
    print("wrote", len(out), "arrays")


if __name__ == "__main__":
    main()
