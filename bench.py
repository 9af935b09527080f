"""Decode throughput of the B200 FISH engine on the Llama-3-8B-shaped Q4_K_M
workload (batch 1, prompt 512 random ids, greedy decode), one JSON line.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one decode token. `value` is device-timed (CUDA events on the
engine's stream around K graph-replayed greedy steps, weights resident);
`e2e` is the same metric through the C ABI call a user makes per token
(fish_decode_ids with host buffers: the token id goes up and the argmax comes
back every step). Under torchrun each rank runs an independent replica on its
own GPU (the 8B model fits one GPU: replicas only) and the max time over
ranks is used. `--impl reference` times the reference FISH CPU engine
(oracle/_ref, its own sources) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
LOCAL_RANK = int(os.environ.get("LOCAL_RANK", "0"))
RANK = int(os.environ.get("RANK", "0"))
WORLD = int(os.environ.get("WORLD_SIZE", "1"))
if WORLD > 1:
    # one GPU per rank: the LOCAL_RANK-th of the visible devices (all of
    # them when the variable is unset), set before any CUDA call
    _vis = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    os.environ["CUDA_VISIBLE_DEVICES"] = _vis[LOCAL_RANK % len(_vis)] if _vis else str(LOCAL_RANK)
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

BASELINE = json.loads((ROOT / "BASELINE.json").read_text())
PEAKS_PATH = ROOT / "MEASURED_PEAKS.json"
PROMPT = 512
N_CTX = 1024


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def dist_init():
    if WORLD <= 1:
        return None
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("gloo", timeout=timedelta(seconds=600))
    return dist


def max_over_ranks(dist, v: float) -> float:
    if dist is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(dist):
    if dist is not None:
        dist.barrier()


def share_group_id(dist, make):
    """Rank 0 makes the NCCL group id (make()); every rank receives it over
    the gloo group. None without a process group."""
    if dist is None:
        return None
    obj = [make() if RANK == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    return obj[0]


def model_path(dist):
    from imurun_b200 import synth
    cfg = synth.preset("llama8b")
    d = os.environ.get("FISH_SYNTH_DIR", "/tmp/fish_synth")
    if RANK == 0:
        t0 = time.time()
        p = synth.cached(cfg, d)
        log(f"[bench] model {p} ({p.stat().st_size / 1e9:.2f} GB, {time.time() - t0:.1f} s)")
    barrier(dist)
    return synth.cached(cfg, d)


def peaks():
    if PEAKS_PATH.exists():
        p = json.loads(PEAKS_PATH.read_text())
        return float(p["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def gemv_share_from_profiles():
    """The streamed GEMV's share of one decode step's launch time, from the
    committed ncu launch list of the same build."""
    import re
    f = ROOT / "profiles" / "decode_step_llama8b_launches.md"
    if not f.exists():
        return None
    m = re.search(r"dominant kernel \((\d+) launches, ([\d.]+) %", f.read_text())
    return float(m.group(2)) / 100.0 if m else None


def int8_peak():
    """Dense int8 tensor peak for the prefill roofline: twice the measured
    bf16 GEMM burst (B200's dense int8 rate is twice its bf16 rate)."""
    if PEAKS_PATH.exists():
        p = json.loads(PEAKS_PATH.read_text())
        return round(2.0 * float(p["bf16_tflops"]), 1), "2x measured bf16 burst (MEASURED_PEAKS.json)"
    return 4500.0, "nominal dense int8"


def traffic_ratio_from_profiles():
    """DRAM bytes per algorithmic byte of the GEMV, from the committed ncu
    summary (one captured launch of the same kernel on an 8B-shaped matrix)."""
    f = ROOT / "profiles" / "gemv_stream_q4k_4096x14336.md"
    if not f.exists():
        return None
    for ln in f.read_text().splitlines():
        if "dram_bytes_per_algorithmic_byte:" in ln:
            try:
                return float(ln.split("dram_bytes_per_algorithmic_byte:", 1)[1].split()[0])
            except (ValueError, IndexError):
                return None
    return None


class Clocks:
    """nvidia-smi samples during the timed region."""

    def __init__(self):
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={os.environ.get('CUDA_VISIBLE_DEVICES', '0').split(',')[0]}",
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for ln in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) >= 8:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[4 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_info() -> dict:
    """Host CPU model, physical cores (distinct (package, core) pairs) and
    logical CPUs, from /proc/cpuinfo."""
    model, cores, cur = None, set(), {}
    try:
        lines = Path("/proc/cpuinfo").read_text().splitlines() + [""]
    except OSError:
        lines = []
    for ln in lines:
        if ":" not in ln:
            if "core id" in cur:
                cores.add((cur.get("physical id", "0"), cur["core id"]))
            cur = {}
            continue
        k, v = (x.strip() for x in ln.split(":", 1))
        if k == "model name" and model is None:
            model = v
        if k in ("physical id", "core id"):
            cur[k] = v
    return {"cpu_model": model, "physical_cores": len(cores) or None, "logical_cpus": os.cpu_count()}


def synth_in_child(preset: str) -> Path:
    """Write (or find) a preset's synthetic GGUF in a separate process, so the
    process that times the reference maps only the reference's library."""
    code = ("import sys; sys.path.insert(0, %r); from imurun_b200 import synth; "
            "print(synth.cached(synth.preset(%r), %r))" % (str(ROOT), preset,
                                                           os.environ.get("FISH_SYNTH_DIR", "/tmp/fish_synth")))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, check=True)
    return Path(r.stdout.strip().splitlines()[-1])


def cpu_reference_decode(path, n_prompt: int, n_decode: int):
    """Reference FISH CPU engine (oracle/_ref) with all host threads:
    prefill n_prompt ids, then time n_decode greedy decode steps."""
    from oracle.binding import REF_SO, Oracle, Reference
    cores = os.cpu_count() or 1
    ids = np.random.default_rng(1).integers(3, 128256, n_prompt).astype(np.int32)
    if REF_SO.exists():
        ref = Reference()
        ref.set_threads(cores)
        m = ref.load(path, N_CTX)
        lg = m.prefill(ids)
        tok = int(np.argmax(lg))
        t0 = time.perf_counter()
        for s in range(n_decode):
            lg = m.forward(np.array([tok], np.int32), n_prompt + s)
            tok = int(np.argmax(lg))
        dt = time.perf_counter() - t0
        m.close()
        return n_decode / dt, "reference", ref.threads(), dt, ref.kernel_name()
    o = Oracle()
    m = o.load(path, N_CTX)
    lg = m.forward(ids, 0)
    tok = int(np.argmax(lg))
    t0 = time.perf_counter()
    for s in range(n_decode):
        lg = m.forward(np.array([tok], np.int32), n_prompt + s)
        tok = int(np.argmax(lg))
    dt = time.perf_counter() - t0
    return n_decode / dt, "port", 1, dt, "scalar C restatement"


def run_reference(args):
    if RANK != 0:
        return 0
    path = synth_in_child("llama8b")
    n_prompt = 32
    k = min(args.steps, 32)
    w = min(args.warmup, 4)
    value, kind, cores, dt, kname = cpu_reference_decode(path, n_prompt, k + w)
    sample = (f"Llama-3-8B-shaped Q4_K_M, prompt {n_prompt} random ids, {k + w} greedy decode steps "
              f"(steps capped at 32 + 4 for the CPU), batch 1")
    line = {
        "impl": "reference", "metric": BASELINE["metric"], "value": round(value, 4), "unit": "tok/s",
        "n_gpus": args.gpus, "steps": k, "warmup": w, "ms_per_step": round(1000.0 / value, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": "llama8b-shaped Q4_K_M decode, batch 1 (reference FISH CPU engine)",
                   "global_batch": 1, "seq_len": n_prompt + k + w, "parallelism": "cpu"},
        "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "cores": cores, "kind": kind, "sample": sample,
                         "kernel_name": kname, **cpu_info()},
        "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    from imurun_b200.native import Model
    dist = dist_init()
    path = model_path(dist)
    K, W = args.steps, args.warmup
    n_ctx = max(N_CTX, (PROMPT + W + K + 64 + 255) // 256 * 256)
    if n_ctx > 8192:
        raise SystemExit("steps + warmup too large for the 8192-token context")
    m = Model(path, n_ctx)
    rng = np.random.default_rng(1234 + RANK)
    ids = rng.integers(3, m.vocab, PROMPT).astype(np.int32)

    # prefill (wall clock, host ids in, last logits out)
    m.prefill(ids[:64], 0)                   # warm the prefill kernels
    t0 = time.perf_counter()
    lg = m.prefill(ids, 0)
    prefill_s = time.perf_counter() - t0
    first = int(np.argmax(lg))

    # warm-up: W greedy steps (captures the graph)
    out = m.greedy(first, W)
    nxt = int(out[-1])
    pos_start = m.kv_len()

    # timed region: K graph-replayed greedy steps, device-timed
    barrier(dist)
    clocks = Clocks()
    clocks.start()
    out = m.greedy(nxt, K)
    eng = json.loads(m.lib.fish_engine_json(m.ctx).decode())
    dev_ms = float(eng["last_decode_device_ms"])
    clk = clocks.stop()
    barrier(dist)
    dev_ms_max = max_over_ranks(dist, dev_ms)
    value = WORLD * K / (dev_ms_max / 1000.0)

    # e2e: the per-token C-ABI call with host buffers, same positions
    m.set_kv_len(pos_start)
    tok = np.array([nxt], np.int32)
    am = np.zeros(1, np.int32)
    barrier(dist)
    t0 = time.perf_counter()
    for s in range(K):
        rc = m.lib.fish_decode_ids(m.ctx, tok.ctypes.data, 1, pos_start + s, None, am.ctypes.data)
        if rc != 0:
            raise RuntimeError(m.lib.fish_last_error(m.ctx).decode())
        tok[0] = am[0]
    e2e_s = time.perf_counter() - t0
    e2e_s = max_over_ranks(dist, e2e_s)
    e2e_value = WORLD * K / e2e_s

    # e2e through the generation loop a user's chat turn runs (fish_generate_to,
    # greedy: penalty and argmax on the device, only the id crosses back);
    # decode tok/s from fish_stats, the reference's own semantics
    from imurun_b200.native import FishStats
    import ctypes
    text = " ".join(f"t{int(i)}" for i in ids[:64]).encode()
    gbuf = ctypes.create_string_buffer(1 << 16)
    m.lib.fish_reset(m.ctx)
    barrier(dist)
    ng = m.lib.fish_generate_to(m.ctx, text, 1, K, 0.0, 1, 1.0, 1.0, gbuf, 1 << 16)
    st = FishStats()
    m.lib.fish_get_stats(m.ctx, ctypes.byref(st))
    gen_tps = -max_over_ranks(dist, -float(st.tokens_per_second)) * WORLD   # slowest rank x ranks
    if ng <= 0:
        gen_tps = None

    # per-launch events of the eager path (context for the class split), from
    # the same 512-id prompt
    m.set_kv_len(0)
    m.prefill(ids, 0)
    prof = json.loads(m.lib.fish_profile_decode_json(m.ctx, nxt, 16).decode())
    cls = {c["name"]: c for c in prof["classes"]}
    g = cls["gemv"]
    peak, peak_kind = peaks()
    total_ms = sum(c["ms"] for c in prof["classes"])
    # the timed decode step against HBM: algorithmic bytes = weights in their
    # GGUF encoding (embedding: one row) + the K/V rows every step reads
    info = m.info
    kv_row = 2 * info.n_layers * info.n_head_kv * info.head_dim * 2
    avg_pos = pos_start + K / 2
    step_bytes = g["bytes"] / prof["steps"] + kv_row * avg_pos
    step_ms = dev_ms / K
    step_gbs = step_bytes / (step_ms / 1e3) / 1e9
    ratio = traffic_ratio_from_profiles()
    share = gemv_share_from_profiles()
    persistent = bool(eng.get("step_kernel"))
    if persistent:
        # one cooperative launch of k_step ran all K steps; its algorithmic
        # bytes are the weights (GGUF encoding) and the K/V rows every step
        # reads, over the launch's event-timed duration
        step_alg = eng["step_weight_bytes"] + kv_row * avg_pos
        achieved = step_alg * K / (float(eng["last_step_ms"]) / 1e3) / 1e9
        traffic = None
        kernel = "k_step (persistent decode step: all GEMV phases, attention, argmax)"
        timed_launches = 1
    else:
        achieved = step_gbs
        traffic = round(ratio * step_bytes) if ratio else None
        kernel = ("decode step: one CUDA graph per token (streamed GEMV x129, decode attention x32, embedding, "
                  "argmax), the K replays timed with CUDA events on the engine stream")
        timed_launches = eng["greedy_graph_kernels"] * K
    gemv = None
    if share and not persistent:
        gemv_ms = share * step_ms
        gemv_bytes = g["bytes"] / prof["steps"]
        gemv = {"kernel": "k_gemv_stream<1, TM, PM> (Q4_K/Q6_K decode GEMV)", "share_of_step": share,
                "ms_per_step_est": round(gemv_ms, 4),
                "achieved_gbs_est": round(gemv_bytes / (gemv_ms / 1e3) / 1e9, 1),
                "frac_est": round(gemv_bytes / (gemv_ms / 1e3) / 1e9 / peak, 4),
                "note": "share of the step's launch time from the committed ncu launch list "
                        "(profiles/decode_step_llama8b_launches.md) times the timed step"}
    # prefill against the int8 tensor roofline: 2 x int8 MACs of the layers
    # for every prompt token + the output projection of the last one
    E, F, V, L = info.n_embd, info.n_ff, info.vocab, info.n_layers
    Qd, KVd = info.n_head * info.head_dim, info.n_head_kv * info.head_dim
    macs = PROMPT * L * (E * (Qd + 2 * KVd) + Qd * E + 3 * E * F) + V * E
    i8_peak, i8_kind = int8_peak()
    prefill_tops = 2.0 * macs / prefill_s / 1e12
    m.close()

    # the sharded configuration on the same N GPUs (strong scaling over one
    # model), reported beside the replicas' value
    sharded = None
    if WORLD > 1 and args.sharded != "none":
        sharded = sharded_measure(dist, args.sharded, 8, 3)

    cpu = None
    if RANK == 0 and WORLD == 1 and not args.no_cpu:
        v, kind, cores, dt, kname = cpu_reference_decode(path, 16, 8)
        cpu = {"value": round(v, 4), "unit": "tok/s", "cores": cores, "kind": kind,
               "sample": f"same GGUF, prompt 16 random ids, 8 greedy decode steps, {dt:.1f} s of CPU decode",
               "kernel_name": kname, **cpu_info()}
    if RANK == 0:
        line = {
            "metric": BASELINE["metric"], "value": round(value, 3), "unit": "tok/s", "n_gpus": WORLD,
            "steps": K, "warmup": W, "ms_per_step": round(dev_ms_max / K, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {
                "workload": "llama8b-shaped Q4_K_M (32 L, d 4096, 32/8 heads, FFN 14336, vocab 128256), batch 1, "
                            f"prompt {PROMPT} random ids, {K} greedy decode steps per replica",
                "global_batch": WORLD, "seq_len": PROMPT + W + K, "parallelism": f"replicas x{WORLD}",
                "l2": "inputs larger than L2 (4.6 GB of weights streamed per step)",
                "prefill_tok_s": round(PROMPT / prefill_s, 1),
                "prefill_roofline": {"bound": "tensor", "achieved": round(prefill_tops, 2), "peak": i8_peak,
                                     "unit": "TOP/s (int8)", "frac": round(prefill_tops / i8_peak, 4),
                                     "peak_kind": i8_kind,
                                     "work": f"{2.0 * macs / 1e12:.3f} T int8 ops for {PROMPT} tokens"},
                "decode_step_gbs": round(step_gbs, 1),
                "decode_step_hbm_frac": round(step_gbs / peak, 4),
                "profile_ms_per_step": {k: round(v["ms"] / prof["steps"], 4) for k, v in cls.items()},
                "profile_note": "per-launch events of the eager multi-kernel path (streamed GEMV etc.), for comparison",
                "decode_kernel": "k_step (one cooperative launch per greedy call)" if persistent else "graph of per-op kernels",
                "profile_total_ms_per_step": round(total_ms / prof["steps"], 4),
                "sharded": sharded,
            },
            "e2e": {"value": round(e2e_value, 3), "unit": "tok/s", "h2d_bytes_per_step": 12, "d2h_bytes_per_step": 4,
                    "generate_tok_s": round(gen_tps, 3) if gen_tps else None,
                    "generate_note": "fish_generate_to, greedy, 64-token text prompt, fish_stats decode tok/s"},
            "gpu_launches": int(timed_launches * WORLD),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": kernel, "peak_kind": peak_kind,
                         "algorithmic_bytes_per_step": round(step_bytes), "gemv": gemv},
            "cpu_baseline": cpu,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0


# Sharded workloads (one model over the ranks): preset, decode batch, prompt.
SHARDED = {
    "llama70b-tp": ("llama70b", 32, 4096, "Llama-3-70B-shaped Q4_K_M (80 L, d 8192, 64/8 heads, FFN 28672, "
                    "vocab 128256), tensor-parallel over heads / FFN rows / vocab rows"),
    "mixtral-ep": ("mixtral", 16, 1024, "Mixtral-8x7B-shaped Q4_K_M (32 L, d 4096, 32/8 heads, 8 experts top-2, "
                   "expert FFN 14336, vocab 32000), experts split over the ranks, attention by heads"),
}


def sharded_measure(dist, workload: str, K: int, W: int, batch: int = 0, prompt: int = 0, layers: int = 0) -> dict:
    """One model sharded over WORLD GPUs (tensor or expert parallelism; one
    process per GPU, NCCL group id from rank 0 over the gloo group): B
    sessions fork one shared random prompt (its KV pages referenced, not
    copied), then batched greedy decode steps. Every rank makes the same
    calls; each step's device time is the batch graph's CUDA-event time on the
    engine stream, max over ranks. Returns the measurement (every rank)."""
    from imurun_b200 import native, synth
    from imurun_b200.native import Model
    preset, B, P, desc = SHARDED[workload]
    B = batch or B
    P = prompt or P
    cfg = synth.preset(preset, layers=layers) if layers else synth.preset(preset)
    if layers:
        desc += f"; TRUNCATED to {layers} layers (plumbing check, not the config)"
    d = os.environ.get("FISH_SYNTH_DIR", "/tmp/fish_synth")
    why = None
    if RANK == 0:
        t0 = time.time()
        try:
            p = synth.cached(cfg, d)
            log(f"[bench] model {p} ({p.stat().st_size / 1e9:.2f} GB, {time.time() - t0:.1f} s)")
        except (RuntimeError, OSError) as e:   # e.g. no room for the synthetic file: every rank skips
            why = f"synthetic {preset} GGUF not written: {e}"
            log(f"[bench] {why}")
    if dist is not None:
        box = [why]
        dist.broadcast_object_list(box, src=0)
        why = box[0]
    if why:
        return {"workload": workload, "desc": desc, "unavailable": why}
    path = synth.cached(cfg, d)
    lib = native.load_library()
    gid = share_group_id(dist, lambda: native.tp_unique_id(lib))
    n_ctx = (P + W + K + 2 + 255) // 256 * 256
    t0 = time.time()
    m = Model(path, n_ctx, lib=lib, tp=(RANK, WORLD, gid) if WORLD > 1 else None)
    load_s = time.time() - t0
    ids = np.random.default_rng(4321).integers(3, m.vocab, P).astype(np.int32)   # same on every rank
    barrier(dist)
    t0 = time.perf_counter()
    lg = m.prefill(ids, 0)
    prefill_s = max_over_ranks(dist, time.perf_counter() - t0)
    sids = [0] + [m.session_fork(0, P) for _ in range(B - 1)]
    tok = np.full(B, int(np.argmax(lg)), np.int32)
    for _ in range(W):
        tok = m.decode_batch(sids, tok)[0]
    barrier(dist)
    clocks = Clocks()
    clocks.start()
    dev_ms = 0.0
    t0 = time.perf_counter()
    for _ in range(K):
        tok = m.decode_batch(sids, tok)[0]
        dev_ms += float(json.loads(m.lib.fish_engine_json(m.ctx).decode())["last_batch_device_ms"])
    wall_s = time.perf_counter() - t0
    clk = clocks.stop()
    barrier(dist)
    dev_ms_max = max_over_ranks(dist, dev_ms)
    wall_s = max_over_ranks(dist, wall_s)
    eng = json.loads(m.lib.fish_engine_json(m.ctx).decode())
    wbytes = float(eng["weights_device_bytes"])
    m.close()
    peak, _ = peaks()
    step_s = dev_ms_max / K / 1e3
    return {"workload": workload, "desc": desc, "batch": B, "prompt": P, "steps": K, "warmup": W,
            "value": round(B / step_s, 3), "ms_per_step": round(step_s * 1e3, 4),
            "e2e_tok_s": round(B * K / wall_s, 3), "prefill_tok_s": round(P / prefill_s, 1), "load_s": round(load_s, 1),
            "weights_bytes_per_gpu": wbytes, "weights_gbs_per_gpu": round(wbytes / step_s / 1e9, 1),
            "hbm_frac_per_gpu": round(wbytes / step_s / 1e9 / peak, 4),
            "parallelism": f"{'tp' if workload.endswith('tp') else 'ep'}{WORLD}", "clocks": clk}


def run_sharded(args):
    """`--workload llama70b-tp / mixtral-ep`: the sharded measurement as the
    bench line (value = B tokens per step / step time, strong scaling)."""
    dist = dist_init()
    r = sharded_measure(dist, args.workload, args.steps, args.warmup, args.batch, args.prompt, args.layers)
    if "unavailable" in r:   # this workload was asked for by name: fail loudly
        if dist is not None:
            dist.destroy_process_group()
        log(f"[bench] {args.workload}: {r['unavailable']}")
        return 1
    _, peak_kind = peaks()
    if RANK == 0:
        line = {
            "metric": BASELINE["metric"], "value": r["value"], "unit": "tok/s", "n_gpus": WORLD,
            "steps": r["steps"], "warmup": r["warmup"], "ms_per_step": r["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {
                "workload": f"{r['desc']}; batch {r['batch']} sessions forked from one {r['prompt']}-token random "
                            f"prompt, {r['steps']} batched greedy decode steps",
                "global_batch": r["batch"], "seq_len": r["prompt"] + r["warmup"] + r["steps"],
                "parallelism": r["parallelism"], "prefill_tok_s": r["prefill_tok_s"], "load_s": r["load_s"],
                "weights_bytes_per_gpu": r["weights_bytes_per_gpu"],
                "weights_gbs_per_gpu": r["weights_gbs_per_gpu"], "hbm_frac_per_gpu": r["hbm_frac_per_gpu"],
                "l2": "inputs larger than L2 (the rank's weights are streamed every step)",
            },
            "e2e": {"value": r["e2e_tok_s"], "unit": "tok/s", "h2d_bytes_per_step": 12 * r["batch"],
                    "d2h_bytes_per_step": 4 * r["batch"]},
            "peak_kind": peak_kind,
            "clocks": r["clocks"],
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0


def run_prefix(args):
    """Configuration 3: the KV prefix cache on a Qwen2.5-7B-shaped model. One
    2048-token seeded random prefix is prefilled once; S sessions fork it (its
    KV pages referenced, not copied), each prefills its own 128 random suffix
    ids, then all S decode greedily together, one batched step per token.
    value = S tokens per step / device step time (CUDA events around the
    batch graph on the engine stream); steps are capped at the configuration's
    128 decode tokens. Single GPU (the model fits one): replicas at N > 1."""
    from imurun_b200 import synth
    from imurun_b200.native import Model
    dist = dist_init()
    S = args.batch or 64
    P, U = args.prompt or 2048, 128
    K, W = min(args.steps, 128 - min(args.warmup, 8)), min(args.warmup, 8)
    cfg = synth.preset("qwen7b", layers=args.layers) if args.layers else synth.preset("qwen7b")
    d = os.environ.get("FISH_SYNTH_DIR", "/tmp/fish_synth")
    if RANK == 0:
        t0 = time.time()
        p = synth.cached(cfg, d)
        log(f"[bench] model {p} ({p.stat().st_size / 1e9:.2f} GB, {time.time() - t0:.1f} s)")
    barrier(dist)
    path = synth.cached(cfg, d)
    n_ctx = (P + U + W + K + 2 + 255) // 256 * 256
    m = Model(path, n_ctx)
    rng = np.random.default_rng(2048 + RANK)
    prefix = rng.integers(3, m.vocab, P).astype(np.int32)
    t0 = time.perf_counter()
    m.prefill(prefix, 0)
    prefix_s = time.perf_counter() - t0
    sids = [m.session_fork(0, P) for _ in range(S)]
    shared = len(set(m.session_pages(0)[:P // m.lib.fish_kv_page_size(m.ctx)]) &
                 set(m.session_pages(sids[-1])[:P // m.lib.fish_kv_page_size(m.ctx)]))
    tok = np.zeros(S, np.int32)
    t0 = time.perf_counter()
    for i, sid in enumerate(sids):
        tok[i] = int(np.argmax(m.session_prefill(sid, rng.integers(3, m.vocab, U).astype(np.int32))))
    suffix_s = time.perf_counter() - t0
    for _ in range(W):
        tok = m.decode_batch(sids, tok)[0]
    barrier(dist)
    clocks = Clocks()
    clocks.start()
    dev_ms = 0.0
    t0 = time.perf_counter()
    prefix_blocks = 0
    for _ in range(K):
        tok = m.decode_batch(sids, tok)[0]
        eng_step = json.loads(m.lib.fish_engine_json(m.ctx).decode())
        dev_ms += float(eng_step["last_batch_device_ms"])
        prefix_blocks = int(eng_step.get("last_batch_prefix_blocks", 0))
    wall_s = time.perf_counter() - t0
    clk = clocks.stop()
    barrier(dist)
    dev_ms_max = max_over_ranks(dist, dev_ms)
    wall_s = max_over_ranks(dist, wall_s)
    eng = json.loads(m.lib.fish_engine_json(m.ctx).decode())
    wbytes = float(eng["weights_device_bytes"])
    info = m.info
    m.close()
    peak, peak_kind = peaks()
    step_s = dev_ms_max / K / 1e3
    kv_pos = 2 * info.n_layers * info.n_head_kv * info.head_dim * 2          # fp16 K and V, every layer
    own_pos = U + W + K / 2                                                   # each session's own positions (mean)
    unique = wbytes + kv_pos * (P + S * own_pos)
    per_session = wbytes + kv_pos * S * (P + own_pos)
    if RANK == 0:
        line = {
            "metric": BASELINE["metric"], "value": round(WORLD * S / step_s, 3), "unit": "tok/s", "n_gpus": WORLD,
            "steps": K, "warmup": W, "ms_per_step": round(step_s * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {
                "workload": f"qwen2.5-7b-shaped Q4_K_M (28 L, d 3584, 28/4 heads, qkv bias, FFN 18944, vocab "
                            f"152064), {S} sessions forked from one {P}-token random prefix (pages shared), each "
                            f"with its own {U}-token random suffix, {K} batched greedy decode steps, fp16 KV",
                "global_batch": S * WORLD, "seq_len": P + U + W + K, "parallelism": f"replicas x{WORLD}",
                "prefix_prefill_tok_s": round(P / prefix_s, 1), "suffix_prefill_tok_s": round(S * U / suffix_s, 1),
                "prefix_pages_shared": shared,
                "unique_bytes_per_step": round(unique), "unique_gbs": round(unique / step_s / 1e9, 1),
                "unique_hbm_frac": round(unique / step_s / 1e9 / peak, 4),
                "per_session_read_bytes_per_step": round(per_session),
                "per_session_read_gbs": round(per_session / step_s / 1e9, 1),
                "attention": "shared-prefix (cascade) attention: the sessions' common 64-key blocks are read once "
                             "per step for the whole batch, each session's own keys by its rank CTAs, the partials "
                             "merged per session (same bits as decoding each session alone)",
                "prefix_blocks_shared": prefix_blocks,
                "peak_kind": peak_kind,
                "l2": "inputs larger than L2 (4.4 GB of weights streamed per step)",
            },
            "e2e": {"value": round(WORLD * S * K / wall_s, 3), "unit": "tok/s", "h2d_bytes_per_step": 12 * S,
                    "d2h_bytes_per_step": 4 * S},
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=192)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--workload", default="llama8b", choices=["llama8b", "qwen-prefix"] + sorted(SHARDED),
                    help="llama8b: the headline config (replicas at N > 1); the others shard one model over N GPUs")
    ap.add_argument("--batch", type=int, default=0, help="sharded workloads: decode batch (default: the config's)")
    ap.add_argument("--prompt", type=int, default=0, help="sharded workloads: prompt tokens (default: the config's)")
    ap.add_argument("--sharded", default=os.environ.get("FISH_BENCH_SHARDED", "llama70b-tp"),
                    choices=["none"] + sorted(SHARDED),
                    help="at N > 1, the sharded workload also measured and reported in config.sharded")
    ap.add_argument("--layers", type=int, default=0,
                    help="sharded workloads: truncate the model (a plumbing check; the line says so)")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "qwen-prefix":
        return run_prefix(args)
    if args.workload != "llama8b":
        return run_sharded(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
