"""ctypes bindings for libfish.so (the FISH C ABI, include/fish/c_api.h, and
the kernel-level entry points, include/fish/fish_kernels.h).

The ABI-4 struct mirrors match model/fish_native.py's (FishStats 1104 B,
FishModelInfo 168 B, FishAdapterInfo 208 B), so this module also serves as
the check that IMURUN's own binding will load the library unchanged.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from . import libpath

P = ctypes.c_void_p
I = ctypes.c_int
F = ctypes.c_float
CP = ctypes.c_char_p

FISH_TOKEN_CB = ctypes.CFUNCTYPE(None, ctypes.c_char_p, ctypes.c_int, ctypes.c_void_p)


class FishStats(ctypes.Structure):
    _fields_ = [
        ("load_seconds", ctypes.c_double), ("prefill_seconds", ctypes.c_double),
        ("decode_seconds", ctypes.c_double), ("tokens_per_second", ctypes.c_double),
        ("prompt_tokens", I), ("generated_tokens", I), ("context_used", I), ("context_size", I),
        ("weights_bytes", ctypes.c_ulonglong), ("kv_bytes", ctypes.c_ulonglong), ("peak_rss_mb", ctypes.c_double),
        ("truncated", I), ("cached_tokens", I), ("n_threads", I), ("streaming", I),
        ("prefill_tokens_per_second", ctypes.c_double),
        ("gpu_layers", I), ("ram_layers", I), ("disk_layers", I), ("gpu_bytes", ctypes.c_ulonglong),
        ("gpu_name", ctypes.c_char * 64),
        ("draft_proposed", I), ("draft_accepted", I), ("draft_active", I),
        ("gpu_mix", ctypes.c_char * 160), ("placement", ctypes.c_char * 320), ("load_profile", ctypes.c_char * 400),
        ("vram_total", ctypes.c_ulonglong), ("vram_free", ctypes.c_ulonglong), ("vram_headroom", ctypes.c_ulonglong),
    ]


class FishModelInfo(ctypes.Structure):
    _fields_ = [
        ("arch", ctypes.c_char * 32), ("n_layers", I), ("n_embd", I), ("n_ff", I), ("n_head", I),
        ("n_head_kv", I), ("head_dim", I), ("n_ctx", I), ("vocab", I), ("tied_output", I),
        ("quant", ctypes.c_char * 64), ("n_experts", I), ("n_experts_per_tok", I), ("n_ctx_train", I),
        ("chat_format", ctypes.c_char * 16), ("tokenizer", ctypes.c_char * 8),
    ]


class FishAdapterInfo(ctypes.Structure):
    _fields_ = [
        ("active", I), ("pending", I), ("name", ctypes.c_char * 128), ("rank", I), ("rank_min", I),
        ("alpha", F), ("scale", F), ("effective_scale", F), ("tensors", I),
        ("merged_bytes", ctypes.c_ulonglong), ("merge_seconds", ctypes.c_double), ("retention", ctypes.c_double),
        ("residual", ctypes.c_double), ("blocks", ctypes.c_ulonglong), ("blocks_refit", ctypes.c_ulonglong),
    ]


ABI4_FUNCTIONS = [
    "fish_version", "fish_abi_version", "fish_supported_archs", "fish_create", "fish_destroy", "fish_load",
    "fish_loaded", "fish_last_error", "fish_model_info_of", "fish_tokenize", "fish_detokenize", "fish_chat_prompt",
    "fish_chat_format", "fish_count_chat_tokens", "fish_generate", "fish_generate_chat", "fish_generate_to",
    "fish_cancel", "fish_reset", "fish_get_stats", "fish_kernel_name", "fish_specs_json", "fish_set_threads",
    "fish_set_draft", "fish_clear_draft", "fish_set_adapter", "fish_clear_adapter", "fish_adapter_info_of",
]
ABI5_FUNCTIONS = [
    "fish_prefill_ids", "fish_decode_ids", "fish_decode_greedy", "fish_kv_len", "fish_set_kv_len",
    "fish_session_open", "fish_session_fork", "fish_session_close", "fish_session_len", "fish_session_prefill",
    "fish_decode_batch", "fish_session_pages", "fish_kv_page_size", "fish_engine_json", "fish_profile_decode_json",
    "fish_trace_decode", "fish_tp_unique_id", "fish_tp_init",
]
KERNEL_FUNCTIONS = [
    "fbx_quantize_acts", "fbx_rmsnorm", "fbx_matmul", "fbx_block_sums", "fbx_attention", "fbx_rope",
    "fbx_argmax", "fbx_argmax_penalized", "fbx_layer_probe", "fbx_tp_plan", "fbx_moe_localize_host", "fbx_embed", "fbx_time_matmul", "fbx_attention_static", "fbx_attention_decode",
    "fbx_profiler", "fbx_attention_prefill",
]


class LayerProbeOut(ctypes.Structure):
    """fbx_layer_probe_out (include/fish/fish_kernels.h)."""
    _fields_ = [
        ("f", P * 4), ("qk", P * 4), ("q32", P * 4), ("gate3", P), ("up3", P),
        ("rows", I * 4), ("K", I * 4), ("has_k", I * 4), ("has_32", I * 4), ("silu_in_prologue", I),
    ]


def _p(a):
    return None if a is None else a.ctypes.data


def load_library(path: str | Path | None = None) -> ctypes.CDLL:
    lib = ctypes.CDLL(str(path or libpath("libfish.so")))
    sig = {
        "fish_version": ([], CP), "fish_abi_version": ([], I), "fish_supported_archs": ([], CP),
        "fish_create": ([], P), "fish_destroy": ([P], None), "fish_load": ([P, CP, I], I),
        "fish_loaded": ([P], I), "fish_last_error": ([P], CP),
        "fish_model_info_of": ([P, ctypes.POINTER(FishModelInfo)], I),
        "fish_tokenize": ([P, CP, I, P, I], I), "fish_detokenize": ([P, P, I, ctypes.c_char_p, I], I),
        "fish_chat_prompt": ([P, P, P, I, ctypes.c_char_p, I], I), "fish_chat_format": ([P], CP),
        "fish_count_chat_tokens": ([P, P, P, I], I),
        "fish_generate": ([P, CP, I, I, F, I, F, F, FISH_TOKEN_CB, P], I),
        "fish_generate_chat": ([P, P, P, I, I, F, I, F, F, FISH_TOKEN_CB, P], I),
        "fish_generate_to": ([P, CP, I, I, F, I, F, F, ctypes.c_char_p, I], I),
        "fish_cancel": ([P], None), "fish_reset": ([P], None),
        "fish_get_stats": ([P, ctypes.POINTER(FishStats)], None), "fish_kernel_name": ([], CP),
        "fish_specs_json": ([P], CP), "fish_set_threads": ([P, I], I), "fish_set_draft": ([P, CP, I], I),
        "fish_clear_draft": ([P], None), "fish_set_adapter": ([P, CP, F], I), "fish_clear_adapter": ([P], I),
        "fish_adapter_info_of": ([P, ctypes.POINTER(FishAdapterInfo)], I),
        "fish_prefill_ids": ([P, P, I, I, P], I), "fish_decode_ids": ([P, P, I, I, P, P], I),
        "fish_decode_greedy": ([P, ctypes.c_int32, I, P], I), "fish_kv_len": ([P], I),
        "fish_set_kv_len": ([P, I], I), "fish_session_open": ([P], I), "fish_session_fork": ([P, I, I], I),
        "fish_session_close": ([P, I], I), "fish_session_len": ([P, I], I),
        "fish_session_prefill": ([P, I, P, I, P], I), "fish_decode_batch": ([P, P, P, I, P, P], I),
        "fish_session_pages": ([P, I, P, I], I), "fish_kv_page_size": ([P], I),
        "fish_engine_json": ([P], CP), "fish_profile_decode_json": ([P, ctypes.c_int32, I], CP),
        "fish_trace_decode": ([P, ctypes.c_int32, I, P, I], I),
        "fish_tp_unique_id": ([P, I], I), "fish_tp_init": ([P, I, I, P, I], I),
        "fbx_quantize_acts": ([P, I, I, P, P], I), "fbx_rmsnorm": ([P, P, I, I, F, P], I),
        "fbx_matmul": ([I, P, I, I, P, I, P], I), "fbx_block_sums": ([I, P, I, I, P, P, P], I),
        "fbx_attention": ([P, P, P, I, I, I, I, I, I, I, P], I),
        "fbx_rope": ([P, P, I, I, I, I, I, I, F, I], I), "fbx_argmax": ([P, I, I, P], I),
        "fbx_argmax_penalized": ([P, I, P, I, F, P], I),
        "fbx_layer_probe": ([P, I, I, P, I, P, P], I),
        "fbx_tp_plan": ([I, I, I, I, I, I, I, I, P], I), "fbx_moe_localize_host": ([P, I, I, I, P], I),
        "fbx_embed": ([I, P, I, I, P, I, P], I),
        "fbx_time_matmul": ([I, I, I, I, I, P, P], I),
        "fbx_profiler": ([I], I),
        "fbx_attention_prefill": ([P, P, P, I, I, I, I, I, I, P], I),
        "fbx_attention_static": ([P, P, P, I, I, I, I, I, I, I, P, P], I),
        "fbx_attention_decode": ([P, P, P, P, P, I, I, I, I, I, I, F, I, P, P, P], I),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


class FishError(RuntimeError):
    pass


def tp_unique_id(lib: ctypes.CDLL | None = None) -> bytes:
    """A new tensor-parallel group id (on one rank; share it with the others)."""
    lib = lib or load_library()
    buf = ctypes.create_string_buffer(128)
    n = lib.fish_tp_unique_id(buf, 128)
    if n <= 0 or n > 128:
        raise FishError("fish_tp_unique_id failed")
    return buf.raw[:n]


class Model:
    """One fish_ctx with a loaded model; thin id-level convenience wrapper."""

    def __init__(self, path, n_ctx: int = 4096, lib: ctypes.CDLL | None = None, tp: tuple | None = None):
        """tp = (rank, world, group id bytes from tp_unique_id()): tensor
        parallelism, one process per GPU; every rank makes the same calls."""
        self.lib = lib or load_library()
        self.ctx = self.lib.fish_create()
        if tp is not None and tp[1] > 1:
            rank, world, gid = tp
            buf = ctypes.create_string_buffer(bytes(gid), len(gid))
            if self.lib.fish_tp_init(self.ctx, int(rank), int(world), buf, len(gid)) != 0:
                err = self.lib.fish_last_error(self.ctx).decode()
                self.lib.fish_destroy(self.ctx)
                self.ctx = None
                raise FishError(f"fish_tp_init: {err}")
        rc = self.lib.fish_load(self.ctx, str(path).encode(), int(n_ctx))
        if rc != 0:
            err = self.lib.fish_last_error(self.ctx).decode()
            self.lib.fish_destroy(self.ctx)
            self.ctx = None
            raise FishError(f"fish_load rc={rc}: {err}")
        info = FishModelInfo()
        self.lib.fish_model_info_of(self.ctx, ctypes.byref(info))
        self.info = info
        self.vocab = info.vocab
        self.n_ctx = info.n_ctx

    def _check(self, rc, what):
        if rc < 0:
            raise FishError(f"{what} rc={rc}: {self.lib.fish_last_error(self.ctx).decode()}")
        return rc

    def prefill(self, ids, pos0: int = 0) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.zeros(self.vocab, np.float32)
        self._check(self.lib.fish_prefill_ids(self.ctx, _p(ids), ids.size, pos0, _p(out)), "fish_prefill_ids")
        return out

    def decode(self, ids, pos0: int, logits: bool = True):
        ids = np.ascontiguousarray(ids, np.int32)
        lg = np.zeros((ids.size, self.vocab), np.float32) if logits else None
        am = np.zeros(ids.size, np.int32)
        self._check(self.lib.fish_decode_ids(self.ctx, _p(ids), ids.size, pos0, _p(lg), _p(am)), "fish_decode_ids")
        return lg, am

    def greedy(self, first: int, n: int) -> np.ndarray:
        out = np.zeros(n, np.int32)
        got = self._check(self.lib.fish_decode_greedy(self.ctx, int(first), n, _p(out)), "fish_decode_greedy")
        return out[:got]

    def kv_len(self) -> int:
        return self.lib.fish_kv_len(self.ctx)

    def set_kv_len(self, n: int):
        self._check(self.lib.fish_set_kv_len(self.ctx, n), "fish_set_kv_len")

    def session_open(self) -> int:
        return self._check(self.lib.fish_session_open(self.ctx), "fish_session_open")

    def session_fork(self, parent: int, prefix: int) -> int:
        return self._check(self.lib.fish_session_fork(self.ctx, parent, prefix), "fish_session_fork")

    def session_close(self, s: int):
        self._check(self.lib.fish_session_close(self.ctx, s), "fish_session_close")

    def session_len(self, s: int) -> int:
        return self.lib.fish_session_len(self.ctx, s)

    def session_prefill(self, s: int, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.zeros(self.vocab, np.float32)
        self._check(self.lib.fish_session_prefill(self.ctx, s, _p(ids), ids.size, _p(out)), "fish_session_prefill")
        return out

    def decode_batch(self, sessions, ids, logits: bool = False):
        s = np.ascontiguousarray(sessions, np.int32)
        ids = np.ascontiguousarray(ids, np.int32)
        am = np.zeros(ids.size, np.int32)
        lg = np.zeros((ids.size, self.vocab), np.float32) if logits else None
        self._check(self.lib.fish_decode_batch(self.ctx, _p(s), _p(ids), ids.size, _p(am), _p(lg)), "fish_decode_batch")
        return am, lg

    def session_pages(self, s: int) -> np.ndarray:
        n = self.lib.fish_session_pages(self.ctx, s, None, 0)
        out = np.zeros(max(n, 1), np.int32)
        self.lib.fish_session_pages(self.ctx, s, _p(out), out.size)
        return out[:n]

    def layer_probe(self, layer: int, x, pos0: int) -> dict:
        """fbx_layer_probe: one layer on hidden rows x [T][n_embd] at positions
        pos0.., with every int8 activation the kernels built (stage s in 0..3:
        attention-norm input, attention output, FFN-norm input, SwiGLU
        product) as Q8ActK / Q8Act record bytes and the float rows they came
        from."""
        info = self.info
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[0]
        E, Q = info.n_embd, info.n_head * info.head_dim
        kx = max(1, info.n_experts_per_tok) if info.n_experts > 0 else 1
        F = info.n_ff
        widths = [E, Q, E, F]
        rows = [T, T, T, T * kx]
        f = [np.zeros((rows[i], widths[i]), np.float32) for i in range(4)]
        qk = [np.zeros((rows[i], max(1, widths[i] // 256) * 276), np.uint8) for i in range(4)]
        q32 = [np.zeros((rows[i], max(1, widths[i] // 32) * 40), np.uint8) for i in range(4)]
        gate3 = np.zeros((rows[3], F), np.float32)
        up3 = np.zeros((rows[3], F), np.float32)
        out = LayerProbeOut()
        for i in range(4):
            out.f[i] = f[i].ctypes.data
            out.qk[i] = qk[i].ctypes.data
            out.q32[i] = q32[i].ctypes.data
        out.gate3 = gate3.ctypes.data
        out.up3 = up3.ctypes.data
        y = np.zeros_like(x)
        self._check(self.lib.fbx_layer_probe(self.ctx, layer, pos0, _p(x), T, _p(y), ctypes.byref(out)),
                    "fbx_layer_probe")
        st = []
        for i in range(4):
            r = out.rows[i]
            st.append({"rows": r, "K": out.K[i], "f": f[i][:r], "has_k": bool(out.has_k[i]),
                       "has_32": bool(out.has_32[i]), "qk": qk[i][:r], "q32": q32[i][:r]})
        return {"x_out": y, "stages": st, "silu_in_prologue": bool(out.silu_in_prologue),
                "gate3": gate3[:out.rows[3]], "up3": up3[:out.rows[3]]}

    def stats(self) -> FishStats:
        st = FishStats()
        self.lib.fish_get_stats(self.ctx, ctypes.byref(st))
        return st

    def close(self):
        if self.ctx:
            self.lib.fish_destroy(self.ctx)
            self.ctx = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
