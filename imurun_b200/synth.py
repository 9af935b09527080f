"""Seeded synthetic GGUF models matching the benchmark configurations.

The writer itself is native (csrc/synth/gguf_synth.cpp, built into
lib/libfishsynth.so); this module holds the shape presets and a ctypes call.

Presets (shapes from the benchmark configurations):
  tiny      llama, 4 layers, d_model 512, 8/4 heads (head_dim 64), FFN 1408,
            vocab 32000, eps 1e-5, theta 1e4, every matrix Q8_0
  llama8b   Llama-3-8B shape: 32 layers, 4096, 32/8 heads, FFN 14336,
            vocab 128256, theta 5e5, Q4_K_M mixture
  qwen7b    Qwen2.5-7B shape: 28 layers, 3584, 28/4 heads, qkv bias,
            FFN 18944, vocab 152064, theta 1e6, Q4_K_M mixture
  mixtral   Mixtral-8x7B shape: 32 layers, 4096, 32/8 heads, 8 experts top-2,
            expert FFN 14336, vocab 32000, theta 1e6, Q4_K_M mixture
  llama70b  Llama-3-70B shape: 80 layers, 8192, 64/8 heads, FFN 28672,
            vocab 128256, theta 5e5, Q4_K_M mixture
  qwen3     Qwen3-style layers (not a benchmark config): 4 layers, 1024,
            16/8 heads, per-head q/k RMSNorm, no qkv bias, FFN 3072,
            vocab 32000, theta 1e6, Q4_K_M mixture

`layers=` truncates a preset (same widths, fewer blocks) for parity runs.
"""
from __future__ import annotations

import ctypes
import hashlib
import os
from dataclasses import dataclass, replace
from pathlib import Path

from . import libpath


@dataclass(frozen=True)
class SynthConfig:
    arch: str = "llama"
    n_layers: int = 4
    n_embd: int = 512
    n_ff: int = 1408
    n_head: int = 8
    n_head_kv: int = 4
    vocab: int = 32000
    n_ctx_train: int = 8192
    eps: float = 1e-5
    freq_base: float = 10000.0
    n_experts: int = 0
    n_experts_per_tok: int = 0
    qkv_bias: int = 0
    wtype: int = 8          # 8 = all Q8_0, 12 = Q4_K_M mixture
    seed: int = 1234
    wstd: float = 0.02
    router_std: float = 0.015625   # 1/64: router logits on a unit-RMS 4096-wide input ~ N(0, 1)
    chat_template: str = ""   # written as tokenizer.chat_template when not empty
    bpe_pre: str = ""         # non-empty: byte-level BPE vocabulary with this tokenizer.ggml.pre name
    qk_norm: int = 0          # 1: per-head q/k RMSNorm weights (qwen3)
    attn_softcap: float = 0.0   # gemma2: score soft cap (0: 50)
    final_softcap: float = 0.0  # gemma2: logit soft cap (0: 30)
    sliding_window: int = 0     # gemma2: window of the even layers (0: 4096)
    rope_orig_ctx: int = 0      # phi3 longrope: original context (0: n_ctx_train)
    rope_attn_factor: float = 0.0   # phi3 longrope: rotation scale (0: 1)
    n_ff_shexp: int = 0         # MoE shared expert rows with a sigmoid gate (qwen2moe; 0: none)
    o_bias: int = 0             # 1: attn_output.bias
    no_bos: int = 0             # 1: tokenizer.ggml.add_bos_token false


PRESETS = {
    "tiny": SynthConfig(),
    "llama8b": SynthConfig(n_layers=32, n_embd=4096, n_ff=14336, n_head=32, n_head_kv=8,
                           vocab=128256, freq_base=500000.0, wtype=12),
    "qwen7b": SynthConfig(arch="qwen2", n_layers=28, n_embd=3584, n_ff=18944, n_head=28,
                          n_head_kv=4, vocab=152064, freq_base=1000000.0, eps=1e-6,
                          qkv_bias=1, wtype=12, n_ctx_train=32768),
    # Qwen3-shaped (not a benchmark config): per-head q/k RMSNorm, no qkv bias
    "qwen3": SynthConfig(arch="qwen3", n_layers=4, n_embd=1024, n_ff=3072, n_head=16, n_head_kv=8,
                         vocab=32000, freq_base=1000000.0, eps=1e-6, qk_norm=1, wtype=12),
    # Gemma2-shaped (not a benchmark config): soft caps small enough to bite
    # on random weights, a 64-position window on the even layers
    "gemma2": SynthConfig(arch="gemma2", n_layers=4, n_embd=1024, n_ff=2816, n_head=8, n_head_kv=4,
                          vocab=32000, freq_base=10000.0, eps=1e-6, wtype=12, attn_softcap=0.5,
                          final_softcap=2.0, sliding_window=64),
    # Phi3-shaped (not a benchmark config): fused q|k|v and gate|up, longrope
    # factors (the long set past a 512-position original context)
    "phi3": SynthConfig(arch="phi3", n_layers=4, n_embd=1024, n_ff=2816, n_head=8, n_head_kv=8,
                        vocab=32000, freq_base=10000.0, wtype=12, rope_orig_ctx=512, rope_attn_factor=1.19),
    # Phi-3-mini's head dimension (96) on the phi3 layout
    "phi3-d96": SynthConfig(arch="phi3", n_layers=4, n_embd=768, n_ff=2048, n_head=8, n_head_kv=8,
                            vocab=32000, freq_base=10000.0, wtype=12, rope_orig_ctx=512, rope_attn_factor=1.19),
    # Qwen2-MoE-shaped (not a benchmark config): 8 experts, top-4, and a
    # gated shared expert; qkv biases, NeoX rotation, unnormalised top-k weights
    "qwen2moe": SynthConfig(arch="qwen2moe", n_layers=2, n_embd=1024, n_ff=768, n_head=8, n_head_kv=8,
                            vocab=32000, freq_base=1000000.0, eps=1e-6, qkv_bias=1, n_experts=8,
                            n_experts_per_tok=4, n_ff_shexp=2048, wtype=12, n_ctx_train=32768),
    # phi3 layout with a fused q|k|v bias and an output-projection bias
    "phi3-bias": SynthConfig(arch="phi3", n_layers=2, n_embd=1024, n_ff=2816, n_head=8, n_head_kv=8,
                             vocab=32000, freq_base=10000.0, wtype=12, qkv_bias=1, o_bias=1,
                             rope_orig_ctx=512, rope_attn_factor=1.19),
    "mixtral": SynthConfig(n_layers=32, n_embd=4096, n_ff=14336, n_head=32, n_head_kv=8,
                           vocab=32000, freq_base=1000000.0, n_experts=8, n_experts_per_tok=2,
                           wtype=12, n_ctx_train=32768),
    "llama70b": SynthConfig(n_layers=80, n_embd=8192, n_ff=28672, n_head=64, n_head_kv=8,
                            vocab=128256, freq_base=500000.0, wtype=12),
}


class _CConfig(ctypes.Structure):
    _fields_ = [
        ("arch", ctypes.c_char_p),
        ("n_layers", ctypes.c_int), ("n_embd", ctypes.c_int), ("n_ff", ctypes.c_int),
        ("n_head", ctypes.c_int), ("n_head_kv", ctypes.c_int), ("vocab", ctypes.c_int),
        ("n_ctx_train", ctypes.c_int),
        ("eps", ctypes.c_float), ("freq_base", ctypes.c_float),
        ("n_experts", ctypes.c_int), ("n_experts_per_tok", ctypes.c_int),
        ("qkv_bias", ctypes.c_int), ("wtype", ctypes.c_int),
        ("seed", ctypes.c_ulonglong), ("wstd", ctypes.c_float), ("router_std", ctypes.c_float),
        ("chat_template", ctypes.c_char_p),
        ("bpe_pre", ctypes.c_char_p),
        ("qk_norm", ctypes.c_int),
        ("attn_softcap", ctypes.c_float), ("final_softcap", ctypes.c_float),
        ("sliding_window", ctypes.c_int),
        ("rope_orig_ctx", ctypes.c_int), ("rope_attn_factor", ctypes.c_float),
        ("n_ff_shexp", ctypes.c_int), ("o_bias", ctypes.c_int), ("no_bos", ctypes.c_int),
    ]


def preset(name: str, layers: int | None = None, **overrides) -> SynthConfig:
    cfg = PRESETS[name]
    if layers is not None:
        cfg = replace(cfg, n_layers=layers)
    if overrides:
        cfg = replace(cfg, **overrides)
    return cfg


def write(path: str | os.PathLike, cfg: SynthConfig, threads: int = 0) -> Path:
    """Write the synthetic GGUF; returns the path. Raises on failure."""
    lib = ctypes.CDLL(str(libpath("libfishsynth.so")))
    fn = lib.fish_synth_write
    fn.argtypes = [ctypes.c_char_p, ctypes.POINTER(_CConfig), ctypes.c_int, ctypes.c_char_p, ctypes.c_int]
    fn.restype = ctypes.c_int
    c = _CConfig(cfg.arch.encode(), cfg.n_layers, cfg.n_embd, cfg.n_ff, cfg.n_head, cfg.n_head_kv,
                 cfg.vocab, cfg.n_ctx_train, cfg.eps, cfg.freq_base, cfg.n_experts,
                 cfg.n_experts_per_tok, cfg.qkv_bias, cfg.wtype, cfg.seed, cfg.wstd, cfg.router_std,
                 cfg.chat_template.encode(), cfg.bpe_pre.encode(), cfg.qk_norm, cfg.attn_softcap,
                 cfg.final_softcap, cfg.sliding_window, cfg.rope_orig_ctx, cfg.rope_attn_factor, cfg.n_ff_shexp,
                 cfg.o_bias, cfg.no_bos)
    err = ctypes.create_string_buffer(256)
    rc = fn(str(path).encode(), ctypes.byref(c), int(threads), err, 256)
    if rc != 0:
        raise RuntimeError(f"fish_synth_write failed: {err.value.decode()}")
    return Path(path)


def size_estimate(cfg: SynthConfig) -> int:
    """The file's bytes to within a few percent (the Q4_K_M mixture rule:
    Q4_K at 0.5625 bytes per weight, Q6_K at 0.8203 for the output matrix and
    half the attn_v / ffn_down matrices; Q8_0 at 1.0625), plus slack, for a
    free-space check."""
    E, F, H = cfg.n_embd, cfg.n_ff, cfg.n_head
    D = E // H
    HKV = cfg.n_head_kv or H
    q8 = cfg.wtype == 8
    r4, r6 = (1.0625, 1.0625) if q8 else (0.5625, 0.8203)
    rv = r4 if q8 else (r4 + r6) / 2
    ne = max(1, cfg.n_experts)
    per_layer = (E * (H * D + HKV * D) * r4 + E * HKV * D * rv + H * D * E * r4
                 + ne * (2 * E * F * r4 + F * E * rv) + 4 * E * max(0, cfg.n_experts) + 8 * E
                 + 2 * E * cfg.n_ff_shexp * r4 + cfg.n_ff_shexp * E * rv)
    total = cfg.vocab * E * r4 + cfg.vocab * E * (r4 if q8 else r6) + cfg.n_layers * per_layer
    return int(total * 1.03) + (64 << 20)


def cached(cfg: SynthConfig, directory: str | os.PathLike | None = None, threads: int = 0) -> Path:
    """Write the model once per (config) into a cache directory and reuse it.
    Refuses to start when the directory's file system has less free space
    than the file needs, and removes a partial file when the write fails."""
    import shutil
    d = Path(directory or os.environ.get("FISH_SYNTH_DIR", "/tmp/fish_synth"))
    d.mkdir(parents=True, exist_ok=True)
    key = int(hashlib.sha1(repr(cfg).encode()).hexdigest()[:12], 16)
    path = d / f"{cfg.arch}_L{cfg.n_layers}_E{cfg.n_embd}_w{cfg.wtype}_s{cfg.seed}_{key:012x}.gguf"
    if not path.exists():
        tmp = path.with_suffix(".tmp")
        tmp.unlink(missing_ok=True)
        need, free = size_estimate(cfg), shutil.disk_usage(d).free
        if free < need:
            raise RuntimeError(f"not enough disk space in {d} for the synthetic model: "
                               f"{need / 1e9:.1f} GB needed, {free / 1e9:.1f} GB free")
        try:
            write(tmp, cfg, threads)
        except BaseException:
            tmp.unlink(missing_ok=True)
            raise
        tmp.rename(path)
    return path
