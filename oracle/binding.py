"""ctypes bindings for the CPU checkers (test infrastructure only).

  Oracle     liboracle.so: the C restatement in fish_oracle.c
  Reference  _ref/libfish_ref.so: the reference FISH engine built from its own
             sources (oracle/Makefile), reached through ref_probe.cpp

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this module, and only as the checker / the timed CPU baseline.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libfish_ref.so"

P = ctypes.c_void_p
I = ctypes.c_int
U64 = ctypes.c_uint64
F = ctypes.c_float

Q8ACT_BYTES = 40      # include/fish/quant.h:58-63
Q8ACTK_BYTES = 276    # include/fish/quant.h:65-70

BLOCK = {0: (1, 4), 1: (1, 2), 2: (32, 18), 8: (32, 34), 12: (256, 144), 13: (256, 176), 14: (256, 210)}


def ref_root():
    """The reference checkout (test infrastructure): REF_ROOT from the
    environment, else the default the oracle Makefile names; None if absent."""
    import os
    root = os.environ.get("REF_ROOT")
    if not root:
        mk = Path(__file__).resolve().parent / "Makefile"
        for ln in mk.read_text().splitlines():
            if ln.startswith("REF_ROOT") and "?=" in ln:
                root = ln.split("?=", 1)[1].strip()
                break
    return Path(root) if root and Path(root).exists() else None


def row_bytes(t: int, n: int) -> int:
    be, bb = BLOCK[t]
    return n // be * bb


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


class Oracle:
    def __init__(self, path: Path = ORACLE_SO):
        if not Path(path).exists():
            raise FileNotFoundError(f"{path} missing: run `make -C oracle oracle`")
        L = ctypes.CDLL(str(path))
        self.L = L
        L.or_quantize_acts.argtypes = [P, U64, P]
        L.or_quantize_acts_k.argtypes = [P, U64, P]
        L.or_block_sums.argtypes = [I, P, P, U64, P, P]
        L.or_block_sums.restype = I
        L.or_vec_dot_q8.argtypes = [I, P, P, U64, P]
        L.or_vec_dot_q8.restype = I
        L.or_vec_dot_q8k.argtypes = [I, P, P, U64, P]
        L.or_vec_dot_q8k.restype = I
        L.or_matmul.argtypes = [I, P, P, I, I, I, P]
        L.or_dequant_row.argtypes = [I, P, P, U64]
        L.or_dequant_row.restype = I
        L.or_rmsnorm.argtypes = [P, P, P, I, F]
        L.or_attention.argtypes = [P, P, P, I, I, I, I, I, P, F, F, I]
        L.or_rope_apply.argtypes = [P, P, I, I, I, I, I, P, P]
        L.or_fp32_to_fp16.argtypes = [F]
        L.or_fp32_to_fp16.restype = ctypes.c_uint16
        L.or_model_load.argtypes = [ctypes.c_char_p, I, I, ctypes.c_char_p, I]
        L.or_model_load.restype = P
        L.or_model_free.argtypes = [P]
        L.or_model_forward.argtypes = [P, P, I, I, P, P]
        L.or_model_forward.restype = I
        L.or_model_set_kv_len.argtypes = [P, I]
        L.or_model_kv_len.argtypes = [P]
        L.or_model_kv_len.restype = I
        L.or_model_last_hidden.argtypes = [P, P, I]
        L.or_model_last_hidden.restype = I
        L.or_model_layer.argtypes = [P, I, P, I, I, P]
        L.or_model_layer.restype = I
        L.or_model_layer_acts.argtypes = [P, I, P, I, I, P, P]
        L.or_model_layer_acts.restype = I
        L.or_model_tensor.argtypes = [P, ctypes.c_char_p, P, P, P, P]
        L.or_model_tensor.restype = P

    # ---- activation quantisers
    def quantize_acts(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(x.size // 32 * Q8ACT_BYTES, np.uint8)
        self.L.or_quantize_acts(_ptr(x), x.size, _ptr(out))
        return out

    def quantize_acts_k(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(x.size // 256 * Q8ACTK_BYTES, np.uint8)
        self.L.or_quantize_acts_k(_ptr(x), x.size, _ptr(out))
        return out

    def block_sums(self, t: int, row: np.ndarray, acts: np.ndarray, n: int):
        nb = n // (256 if t in (12, 13, 14) else 32)
        s = np.zeros(nb, np.int32)
        m = np.zeros(nb, np.int32)
        ok = self.L.or_block_sums(t, _ptr(row), _ptr(acts), n, _ptr(s), _ptr(m))
        if not ok:
            raise ValueError(f"no integer kernel for type {t}")
        return s, m

    def vec_dot(self, t: int, row, acts, n: int) -> float:
        """Integer-path row dot (quant_x86.cpp kernels restated)."""
        f = ctypes.c_float()
        fn = self.L.or_vec_dot_q8k if t in (12, 13, 14) else self.L.or_vec_dot_q8
        if not fn(t, _ptr(row), _ptr(acts), n, ctypes.addressof(f)):
            raise ValueError(f"no integer kernel for type {t}")
        return f.value

    def matmul(self, t: int, w: np.ndarray, x: np.ndarray, n_in: int, n_out: int) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).reshape(-1, n_in)
        y = np.zeros((x.shape[0], n_out), np.float32)
        self.L.or_matmul(t, _ptr(w), _ptr(x), x.shape[0], n_in, n_out, _ptr(y))
        return y

    def dequant(self, t: int, src: np.ndarray, n: int) -> np.ndarray:
        y = np.zeros(n, np.float32)
        if not self.L.or_dequant_row(t, _ptr(src), _ptr(y), n):
            raise ValueError("dequant failed")
        return y

    def rmsnorm(self, x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        self.L.or_rmsnorm(_ptr(out), _ptr(x), _ptr(np.ascontiguousarray(w, np.float32)), x.size, eps)
        return out

    def attention(self, q, kc, vc, H, HKV, D, pos0, n_tok, scale, softcap=0.0, window=0):
        out = np.zeros((n_tok, H * D), np.float32)
        self.L.or_attention(_ptr(q), _ptr(kc), _ptr(vc), H, HKV, D, pos0, n_tok, _ptr(out), scale, softcap, window)
        return out

    def fp16_round(self, x: np.ndarray) -> np.ndarray:
        return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)

    # ---- whole model
    def load(self, path, n_ctx: int, kv_f16: bool = False) -> "OracleModel":
        err = ctypes.create_string_buffer(256)
        h = self.L.or_model_load(str(path).encode(), n_ctx, 1 if kv_f16 else 0, err, 256)
        if not h:
            raise RuntimeError(err.value.decode())
        return OracleModel(self, h)


class OracleModel:
    def __init__(self, o: Oracle, h):
        self.o, self.h = o, h
        info = (ctypes.c_int * 24)()
        # or_model_info layout: 16 ints (n_layers..tied_output) + 2 floats + 2 ints
        o.L.or_model_info_of.argtypes = [P, P]
        o.L.or_model_info_of(h, ctypes.addressof(info))
        self.n_layers, self.n_embd, self.n_ff, self.n_head, self.n_head_kv, self.head_dim, \
            self.n_ctx, self.vocab = list(info)[:8]

    def forward(self, ids, pos0: int, all_logits: bool = False) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        last = np.zeros(self.vocab, np.float32)
        allv = np.zeros((ids.size, self.vocab), np.float32) if all_logits else None
        if not self.o.L.or_model_forward(self.h, _ptr(ids), ids.size, pos0, _ptr(last), _ptr(allv)):
            raise RuntimeError("oracle forward failed")
        return allv if all_logits else last

    def set_kv_len(self, n: int):
        self.o.L.or_model_set_kv_len(self.h, n)

    def layer(self, layer: int, x: np.ndarray, pos0: int) -> np.ndarray:
        """One layer alone on hidden rows x [n_tok][n_embd] at positions pos0..
        (or_model_layer): returns the layer's output rows."""
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        if not self.o.L.or_model_layer(self.h, layer, _ptr(x), x.shape[0], pos0, _ptr(out)):
            raise RuntimeError("oracle layer failed")
        return out

    def layer_acts(self, layer: int, x: np.ndarray, pos0: int, qk, q32) -> np.ndarray:
        """One layer on hidden rows x with the given int8 activations at its
        four quantisation points (qk / q32: per stage, Q8ActK / Q8Act record
        bytes or None), or_model_layer_acts."""
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        keep = [None if a is None else np.ascontiguousarray(a) for a in list(qk) + list(q32)]
        arr = (P * 8)(*[None if a is None else a.ctypes.data for a in keep])
        if not self.o.L.or_model_layer_acts(self.h, layer, _ptr(x), x.shape[0], pos0, ctypes.addressof(arr), _ptr(out)):
            raise RuntimeError("oracle layer failed")
        return out

    def tensor(self, name: str):
        """(type, (ne0, ne1, ne2), address of the GGUF data) of a tensor, or None."""
        t = ctypes.c_int(0)
        ne = [ctypes.c_int64(0) for _ in range(3)]
        a = self.o.L.or_model_tensor(self.h, name.encode(), ctypes.byref(t), ctypes.byref(ne[0]),
                                     ctypes.byref(ne[1]), ctypes.byref(ne[2]))
        if not a:
            return None
        return t.value, (ne[0].value, ne[1].value, ne[2].value), a

    def tensor_rows(self, name: str, rows, expert: int = 0) -> np.ndarray:
        """GGUF bytes of the given rows of a 2-D (or one expert of a 3-D) tensor."""
        t, (n0, n1, _), a = self.tensor(name)
        rb = row_bytes(t, n0)
        base = a + expert * rb * n1
        return np.stack([np.frombuffer(ctypes.string_at(int(base) + int(r) * int(rb), int(rb)), np.uint8) for r in rows])

    def tensor_f32(self, name: str) -> np.ndarray:
        t, (n0, n1, n2), a = self.tensor(name)
        assert t == 0, "f32 tensors only"
        n = n0 * n1 * n2
        return np.frombuffer(ctypes.string_at(a, 4 * n), np.float32).copy()

    def close(self):
        if self.h:
            self.o.L.or_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Reference:
    """The reference FISH engine (its own sources) through ref_probe.cpp."""

    def __init__(self, path: Path = REF_SO):
        if not Path(path).exists():
            raise FileNotFoundError(f"{path} missing: run `make -C oracle ref` where the reference is present")
        L = ctypes.CDLL(str(path))
        self.L = L
        for n in ("ref_quantize_acts", "ref_quantize_acts_k", "ref_quantize_acts_scalar", "ref_quantize_acts_k_scalar"):
            getattr(L, n).argtypes = [P, U64, P]
        L.ref_vec_dot_q8.argtypes = [I, P, P, U64, P]
        L.ref_vec_dot_q8k.argtypes = [I, P, P, U64, P]
        L.ref_dequant_row.argtypes = [I, P, P, U64]
        L.ref_quantize_row.argtypes = [I, P, P, U64]
        L.ref_quantize_row.restype = I
        L.ref_rmsnorm.argtypes = [P, P, P, I, F]
        L.ref_attention.argtypes = [P, P, P, I, I, I, I, I, I, P, F]
        L.ref_attention_capped.argtypes = [P, P, P, I, I, I, I, I, I, P, F, F, I]
        L.ref_rope_table.argtypes = [I, I, I, I, F, P, P]
        L.ref_kernel_name.restype = ctypes.c_char_p
        L.ref_set_threads.argtypes = [I]
        L.ref_threads.restype = I
        L.ref_model_load.argtypes = [ctypes.c_char_p, I, ctypes.c_char_p, I]
        L.ref_model_load.restype = P
        L.ref_model_free.argtypes = [P]
        L.ref_model_forward.argtypes = [P, P, I, I, P, P]
        L.ref_model_forward.restype = I
        L.ref_model_vocab.argtypes = [P]
        L.ref_model_vocab.restype = I
        L.ref_model_set_kv_len.argtypes = [P, I]
        L.ref_model_reset.argtypes = [P]
        L.ref_model_max_batch.argtypes = [P]
        L.ref_model_max_batch.restype = I

    def kernel_name(self) -> str:
        return self.L.ref_kernel_name().decode()

    def quantize_acts(self, x, scalar=False):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(x.size // 32 * Q8ACT_BYTES, np.uint8)
        (self.L.ref_quantize_acts_scalar if scalar else self.L.ref_quantize_acts)(_ptr(x), x.size, _ptr(out))
        return out

    def quantize_acts_k(self, x, scalar=False):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(x.size // 256 * Q8ACTK_BYTES, np.uint8)
        (self.L.ref_quantize_acts_k_scalar if scalar else self.L.ref_quantize_acts_k)(_ptr(x), x.size, _ptr(out))
        return out

    def quantize_row(self, t: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(row_bytes(t, x.size), np.uint8)
        if not self.L.ref_quantize_row(t, _ptr(x), _ptr(out), x.size):
            raise ValueError("quantize_row failed")
        return out

    def vec_dot(self, t: int, row, acts, n: int) -> float:
        f = ctypes.c_float()
        fn = self.L.ref_vec_dot_q8k if t in (12, 13, 14) else self.L.ref_vec_dot_q8
        fn(t, _ptr(row), _ptr(acts), n, ctypes.addressof(f))
        return f.value

    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        self.L.ref_rmsnorm(_ptr(out), _ptr(x), _ptr(np.ascontiguousarray(w, np.float32)), x.size, eps)
        return out

    def attention(self, q, kc, vc, n_ctx, H, HKV, D, pos0, n_tok, scale, softcap=0.0, window=0):
        out = np.zeros((n_tok, H * D), np.float32)
        if softcap or window:
            self.L.ref_attention_capped(_ptr(q), _ptr(kc), _ptr(vc), n_ctx, H, HKV, D, pos0, n_tok, _ptr(out), scale,
                                        softcap, window)
        else:
            self.L.ref_attention(_ptr(q), _ptr(kc), _ptr(vc), n_ctx, H, HKV, D, pos0, n_tok, _ptr(out), scale)
        return out

    def rope_table(self, n_ctx, D, rot, neox, base):
        half = rot // 2
        c = np.zeros(n_ctx * half, np.float32)
        s = np.zeros_like(c)
        self.L.ref_rope_table(n_ctx, D, rot, int(neox), base, _ptr(c), _ptr(s))
        return c.reshape(n_ctx, half), s.reshape(n_ctx, half)

    def set_threads(self, n: int):
        self.L.ref_set_threads(n)

    def threads(self) -> int:
        return self.L.ref_threads()

    def load(self, path, n_ctx: int) -> "ReferenceModel":
        err = ctypes.create_string_buffer(256)
        h = self.L.ref_model_load(str(path).encode(), n_ctx, err, 256)
        if not h:
            raise RuntimeError(err.value.decode())
        return ReferenceModel(self, h)


class ReferenceModel:
    def __init__(self, r: Reference, h):
        self.r, self.h = r, h
        self.vocab = r.L.ref_model_vocab(h)
        self.max_batch = r.L.ref_model_max_batch(h)

    def forward(self, ids, pos0: int, all_logits: bool = False) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        last = np.zeros(self.vocab, np.float32)
        allv = np.zeros((ids.size, self.vocab), np.float32) if all_logits else None
        if not self.r.L.ref_model_forward(self.h, _ptr(ids), ids.size, pos0, _ptr(last), _ptr(allv)):
            raise RuntimeError("reference forward failed")
        return allv if all_logits else last

    def prefill(self, ids, pos0: int = 0) -> np.ndarray:
        """Chunks of at most max_batch tokens, like generate_ids_locked (c_api.cpp:586-595)."""
        ids = np.ascontiguousarray(ids, np.int32)
        pos = 0
        out = None
        while pos < ids.size:
            n = min(self.max_batch, ids.size - pos)
            out = self.forward(ids[pos:pos + n], pos0 + pos)
            pos += n
        return out

    def set_kv_len(self, n: int):
        self.r.L.ref_model_set_kv_len(self.h, n)

    def reset(self):
        self.r.L.ref_model_reset(self.h)

    def close(self):
        if self.h:
            self.r.L.ref_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
