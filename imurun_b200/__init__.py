"""imurun_b200 — a B200-native engine behind FISH's C ABI.

The product is the native library ``lib/libfish.so``: a C++ host plus
hand-written sm_100a CUDA kernels that exports FISH's ``fish_*`` C ABI
(ABI 4, plus the additive ABI-5 id-level and session calls), so IMURUN's
``model/fish_native.py`` loads it unchanged through ``FISH_LIBRARY``.

This Python package only locates and builds the native libraries and offers a
ctypes mirror of the ABI for tests and benchmarks (``native.py``); no tensor
work happens in Python.
"""
from __future__ import annotations

from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_DIR = PKG_DIR / "lib"


def libpath(name: str = "libfish.so") -> Path:
    """Path of a built native library; raises if it has not been built."""
    p = LIB_DIR / name
    if not p.exists():
        raise FileNotFoundError(
            f"{p} is missing: build the native libraries first "
            "(python -c 'import __graft_entry__ as g; g.build()' or python -m imurun_b200.build)")
    return p
