"""Device timing of single hot-path kernels through the C ABI.

    python -m imurun_b200.timing matmul --type 12 --n-in 4096 --n-out 14336 [--tokens 1] [--iters 20]
    python -m imurun_b200.timing attention --pos 575 [--heads 32 --kv-heads 8 --dim 128 --calls 3]
    python -m imurun_b200.timing prefill --tokens 512 [--layers 32]
    python -m imurun_b200.timing greedy --layers 32 --steps 3 --prompt 512
    python -m imurun_b200.timing batch --preset qwen7b --prompt 2048 --sessions 64 --suffix 128 [--layers 0]
    python -m imurun_b200.timing spec --preset llama8b --draft-layers 2 --k 5 --tokens 128 [--penalty 1.0]

Runs fbx_time_matmul: 3 warm-up launches, then `iters` launches timed with
CUDA events, each launch reading a different copy of the weights (>= 512 MB
of copies, so every launch streams from HBM). Prints one JSON line with the
mean launch time, the algorithmic bytes of a launch and their ratio. Also
the command used for profiler captures of one GEMV launch (`-s 3 -c 1`).
`prefill` prefills `tokens` random ids into the seeded Llama-3-8B-shaped
Q4_K_M GGUF (synthesised and cached under $FISH_SYNTH_DIR, default
/tmp/fish_synth; `--layers` truncates it) after a 64-token warm-up, and prints
the wall time and tok/s. `attention` runs the fused decode-attention kernel (fp16 cache, one
token at position pos) `calls` times through fbx_attention_decode — the small
case for profiler captures of that kernel.
"""
from __future__ import annotations

import argparse
import json

import numpy as np

from . import native


def time_matmul(lib, type_id: int, n_in: int, n_out: int, tokens: int = 1, iters: int = 20) -> dict:
    ms = np.zeros(1, np.float32)
    nbytes = np.zeros(1, np.float64)
    rc = lib.fbx_time_matmul(type_id, n_in, n_out, tokens, iters, ms.ctypes.data, nbytes.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"fbx_time_matmul failed: {rc}")
    us = float(ms[0]) * 1e3
    return {"type": type_id, "n_in": n_in, "n_out": n_out, "tokens": tokens, "iters": iters,
            "us_per_launch": round(us, 3), "bytes_per_launch": float(nbytes[0]),
            "gb_s": round(float(nbytes[0]) / (us * 1e-6) / 1e9, 1),
            "tops": round(2.0 * n_in * n_out * tokens / (us * 1e-6) / 1e12, 2)}


def attention(lib, pos: int, heads: int, kv_heads: int, dim: int, calls: int) -> dict:
    rng = np.random.default_rng(pos)
    q = rng.standard_normal(heads * dim).astype(np.float32)
    kc = rng.standard_normal((max(pos, 1), kv_heads * dim)).astype(np.float32)
    vc = rng.standard_normal((max(pos, 1), kv_heads * dim)).astype(np.float32)
    kn = rng.standard_normal(kv_heads * dim).astype(np.float32)
    vn = rng.standard_normal(kv_heads * dim).astype(np.float32)
    out = np.zeros(heads * dim, np.float32)
    for _ in range(calls):
        rc = lib.fbx_attention_decode(q.ctypes.data, kc.ctypes.data, vc.ctypes.data, kn.ctypes.data, vn.ctypes.data, pos,
                                      heads, kv_heads, dim, dim, 0, 500000.0, 1, out.ctypes.data, None, None)
        if rc != 0:
            raise RuntimeError(f"fbx_attention_decode failed: {rc}")
    return {"pos": pos, "heads": heads, "kv_heads": kv_heads, "dim": dim, "calls": calls,
            "out_absmax": float(np.abs(out).max())}


def prefill(tokens: int, layers: int) -> dict:
    import os
    import time
    from . import synth
    from .native import Model
    cfg = synth.preset("llama8b") if layers == 32 else synth.preset("llama8b", layers=layers)
    path = synth.cached(cfg, os.environ.get("FISH_SYNTH_DIR", "/tmp/fish_synth"))
    ids = np.random.default_rng(1).integers(3, 128256, tokens).astype(np.int32)
    with Model(path, max(1024, tokens + 64)) as m:
        m.prefill(ids[:64], 0)
        t0 = time.perf_counter()
        m.prefill(ids, 0)
        dt = time.perf_counter() - t0
    return {"tokens": tokens, "layers": layers, "seconds": round(dt, 5), "tok_s": round(tokens / dt, 1)}


def greedy(layers: int, steps: int, prompt: int = 0) -> dict:
    """Greedy decode on a Llama-3-8B-shaped model of `layers` layers, after a
    prefill of `prompt` random ids (none by default: the first streamed-GEMV
    launches are then layer 0's qkv, o, gate/up and down, a small case for
    ncu captures; with a prompt, the decode steps see a realistic context)."""
    import os
    import time
    from . import synth
    from .native import Model
    cfg = synth.preset("llama8b") if layers == 32 else synth.preset("llama8b", layers=layers)
    path = synth.cached(cfg, os.environ.get("FISH_SYNTH_DIR", "/tmp/fish_synth"))
    ids = np.random.default_rng(1).integers(3, 128256, max(prompt, 1)).astype(np.int32)
    with Model(path, max(1024, (prompt + steps + 64 + 255) // 256 * 256)) as m:
        first = int(np.argmax(m.prefill(ids, 0))) if prompt > 0 else 5
        t0 = time.perf_counter()
        out = m.greedy(first, steps)
        dt = time.perf_counter() - t0
    return {"layers": layers, "steps": steps, "ids": [int(v) for v in out], "seconds": round(dt, 5)}


def batch(preset: str, prompt: int, sessions: int, suffix: int, layers: int, steps: int = 5) -> dict:
    """One batched greedy decode step of `sessions` sessions forked from one
    `prompt`-token random prompt (its KV pages shared), each with its own
    `suffix` random ids, on the synthetic GGUF of `preset` (`layers` > 0
    truncates it). Three warm-up steps, `steps` steps each timed with CUDA
    events on the engine stream (`last_batch_device_ms`), then one more step
    inside a profiler capture range (fbx_profiler), so that
    `ncu --profile-from-start off` records exactly one step."""
    import os
    from . import synth
    from .native import Model
    cfg = synth.preset(preset, layers=layers) if layers else synth.preset(preset)
    path = synth.cached(cfg, os.environ.get("FISH_SYNTH_DIR", "/tmp/fish_synth"))
    rng = np.random.default_rng(1)
    with Model(path, (prompt + suffix + steps + 64 + 255) // 256 * 256) as m:
        m.prefill(rng.integers(3, m.vocab, prompt).astype(np.int32), 0)
        sids = [m.session_fork(0, prompt) for _ in range(sessions)]
        tok = np.zeros(sessions, np.int32)
        for i, sid in enumerate(sids):
            if suffix:
                tok[i] = int(np.argmax(m.session_prefill(sid, rng.integers(3, m.vocab, suffix).astype(np.int32))))
        for _ in range(3):
            tok = m.decode_batch(sids, tok)[0]
        ms = []
        for _ in range(steps):
            tok = m.decode_batch(sids, tok)[0]
            ms.append(float(json.loads(m.lib.fish_engine_json(m.ctx).decode())["last_batch_device_ms"]))
        m.lib.fbx_profiler(1)
        tok = m.decode_batch(sids, tok)[0]
        m.lib.fbx_profiler(0)
    return {"preset": preset, "prompt": prompt, "sessions": sessions, "suffix": suffix, "layers": layers or cfg.n_layers,
            "step_ms": [round(v, 4) for v in ms], "tok_s": round(sessions / (sum(ms) / len(ms) / 1e3), 1)}


def spec(preset: str, draft_layers: int, k: int, tokens: int, penalty: float) -> dict:
    """Greedy generation of `tokens` ids through fish_generate on the synthetic
    GGUF of `preset`, plain and with a draft model: the same preset truncated
    to `draft_layers` layers. The synthetic weights are seeded by tensor name,
    so the draft is the target's own first layers, embedding and output head
    (a layer-skip draft). Reports tok/s of both (the stats' decode rate, host
    loop included), the draft's acceptance and the first index where the two
    id sequences differ (-1: identical)."""
    import ctypes
    import os
    from . import synth
    d = os.environ.get("FISH_SYNTH_DIR", "/tmp/fish_synth")
    tgt = synth.cached(synth.preset(preset), d)
    drf = synth.cached(synth.preset(preset, layers=draft_layers), d)
    lib = native.load_library()
    lib.fbx_last_generated.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    lib.fbx_last_generated.restype = ctypes.c_int
    prompt = b"the quick brown fox jumps over the lazy dog, and then it runs far away into the woods " * 4
    out = {"preset": preset, "draft_layers": draft_layers, "k": k, "tokens": tokens, "penalty": penalty}
    runs = {}
    for name, draft in (("plain", None), ("draft", drf)):
        ctx = lib.fish_create()
        assert lib.fish_load(ctx, str(tgt).encode(), 4096) == 0, lib.fish_last_error(ctx)
        if draft is not None:
            assert lib.fish_set_draft(ctx, str(draft).encode(), k) == 0, lib.fish_last_error(ctx)
        no_cb = native.FISH_TOKEN_CB()
        lib.fish_generate(ctx, prompt, 1, 16, 0.0, 40, 0.9, penalty, no_cb, None)   # warm-up
        n = lib.fish_generate(ctx, prompt, 1, tokens, 0.0, 40, 0.9, penalty, no_cb, None)
        st = native.FishStats()
        lib.fish_get_stats(ctx, ctypes.byref(st))
        ids = np.zeros(max(n, 1), np.int32)
        lib.fbx_last_generated(ctx, ids.ctypes.data, ids.size)
        runs[name] = ids[:n].tolist()
        out[name] = {"generated": n, "tok_s": round(st.tokens_per_second, 1),
                     "proposed": st.draft_proposed, "accepted": st.draft_accepted}
        lib.fish_destroy(ctx)
    a, b = runs["plain"], runs["draft"]
    out["first_difference"] = next((i for i in range(min(len(a), len(b))) if a[i] != b[i]),
                                   -1 if len(a) == len(b) else min(len(a), len(b)))
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    mm = sub.add_parser("matmul")
    mm.add_argument("--type", type=int, required=True, help="ggml type id: 8 Q8_0, 12 Q4_K, 14 Q6_K, 0 F32, 1 F16")
    mm.add_argument("--n-in", type=int, required=True)
    mm.add_argument("--n-out", type=int, required=True)
    mm.add_argument("--tokens", type=int, default=1)
    mm.add_argument("--iters", type=int, default=20)
    at = sub.add_parser("attention")
    at.add_argument("--pos", type=int, required=True)
    at.add_argument("--heads", type=int, default=32)
    at.add_argument("--kv-heads", type=int, default=8)
    at.add_argument("--dim", type=int, default=128)
    at.add_argument("--calls", type=int, default=3)
    pf = sub.add_parser("prefill")
    pf.add_argument("--tokens", type=int, default=512)
    pf.add_argument("--layers", type=int, default=32)
    gr = sub.add_parser("greedy")
    gr.add_argument("--layers", type=int, default=2)
    gr.add_argument("--steps", type=int, default=3)
    gr.add_argument("--prompt", type=int, default=0)
    bt = sub.add_parser("batch")
    bt.add_argument("--preset", default="qwen7b")
    bt.add_argument("--prompt", type=int, default=2048)
    bt.add_argument("--sessions", type=int, default=64)
    bt.add_argument("--suffix", type=int, default=128)
    bt.add_argument("--layers", type=int, default=0)
    bt.add_argument("--steps", type=int, default=5)
    sp = sub.add_parser("spec")
    sp.add_argument("--preset", default="llama8b")
    sp.add_argument("--draft-layers", type=int, default=2)
    sp.add_argument("--k", type=int, default=5)
    sp.add_argument("--tokens", type=int, default=128)
    sp.add_argument("--penalty", type=float, default=1.0)
    a = ap.parse_args()
    if a.cmd == "spec":
        print(json.dumps(spec(a.preset, a.draft_layers, a.k, a.tokens, a.penalty)), flush=True)
        return
    if a.cmd == "batch":
        print(json.dumps(batch(a.preset, a.prompt, a.sessions, a.suffix, a.layers, a.steps)), flush=True)
        return
    if a.cmd == "prefill":
        print(json.dumps(prefill(a.tokens, a.layers)), flush=True)
        return
    if a.cmd == "greedy":
        print(json.dumps(greedy(a.layers, a.steps, a.prompt)), flush=True)
        return
    lib = native.load_library()
    if a.cmd == "matmul":
        print(json.dumps(time_matmul(lib, a.type, a.n_in, a.n_out, a.tokens, a.iters)), flush=True)
    else:
        print(json.dumps(attention(lib, a.pos, a.heads, a.kv_heads, a.dim, a.calls)), flush=True)


if __name__ == "__main__":
    main()
