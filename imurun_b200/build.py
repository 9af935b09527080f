"""Build the native libraries in-tree.

  lib/libfish.so       the product: C++ host + sm_100a CUDA kernels, FISH C ABI
  lib/libfishsynth.so  synthetic GGUF writer (test and benchmark inputs)

Usage: python -m imurun_b200.build [--clean]
Objects go to imurun_b200/_build/ (not tracked). Every CUDA translation unit
is compiled for sm_100a only (-gencode arch=compute_100a,code=sm_100a).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "lib"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc" if Path("/usr/local/cuda/bin/nvcc").exists() else "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
          f"-I{ROOT / 'include'}", f"-I{CSRC}"]
# FISH_TRACE_CTA_BUILD=1 compiles the every-CTA trace events (kernels/trace.cuh)
# into the kernels; off by default, since they cost time on every launch.
if os.environ.get("FISH_TRACE_CTA_BUILD", "0") not in ("", "0"):
    COMMON.append("-DFB_TRACE_CTA=1")
# extra preprocessor definitions for experiment builds, e.g. "-DFOO=1 -DBAR=2"
COMMON += [d for d in os.environ.get("FISH_NVCC_DEFINES", "").split() if d.startswith("-D")]

SOURCES = [
    "kernels/quant_act.cu", "kernels/gemv.cu", "kernels/attention.cu", "kernels/misc.cu", "kernels/step.cu", "kernels/gemm.cu", "kernels/gemm_tc.cu",
    "gguf.cpp", "tokenizer.cpp", "sampler.cpp", "engine.cpp", "c_api.cpp", "kernel_api.cpp",
    "attention_static.cu",
]


def _obj(src: str) -> Path:
    return BUILD / (src.replace("/", "_").rsplit(".", 1)[0] + ".o")


def _headers_mtime() -> float:
    hs = list(CSRC.rglob("*.h")) + list(CSRC.rglob("*.cuh")) + list((ROOT / "include").rglob("*.h"))
    t = max((h.stat().st_mtime for h in hs), default=0.0)
    # a change of compiler flags makes every object stale
    stamp = BUILD / "flags.txt"
    flags = " ".join(ARCH + COMMON)
    if not stamp.exists() or stamp.read_text() != flags:
        stamp.write_text(flags)
    return max(t, stamp.stat().st_mtime)


def _compile(src: str, hdr_mtime: float) -> str:
    s = CSRC / src
    o = _obj(src)
    if o.exists() and o.stat().st_mtime > max(s.stat().st_mtime, hdr_mtime):
        return f"up to date {src}"
    cmd = [NVCC, *ARCH, *COMMON, "-x", "cu", "-c", str(s), "-o", str(o)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
    return f"compiled {src}"


def build_fish(jobs: int = 8, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.mkdir(exist_ok=True)
    hm = _headers_mtime()
    with cf.ThreadPoolExecutor(jobs) as ex:
        for msg in ex.map(lambda s: _compile(s, hm), SOURCES):
            if verbose:
                print(msg)
    out = LIB / "libfish.so"
    objs = [str(_obj(s)) for s in SOURCES]
    newest = max(Path(o).stat().st_mtime for o in objs)
    if not out.exists() or out.stat().st_mtime < newest:
        cmd = [NVCC, *ARCH, "-shared", "-o", str(out), *objs, "-lpthread", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    return out


def build_synth() -> Path:
    LIB.mkdir(exist_ok=True)
    src = CSRC / "synth" / "gguf_synth.cpp"
    out = LIB / "libfishsynth.so"
    if not out.exists() or out.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-o", str(out), str(src), "-lpthread"],
                       check=True)
    return out


def build_all(verbose: bool = False) -> None:
    build_synth()
    build_fish(verbose=verbose)


if __name__ == "__main__":
    if "--clean" in sys.argv:
        shutil.rmtree(BUILD, ignore_errors=True)
    build_all(verbose=True)
    print("built", LIB / "libfish.so")
