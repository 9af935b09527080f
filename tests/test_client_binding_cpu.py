"""The reference's own Python client binds this library unchanged.

IMURUN's server reaches FISH through model/fish_native.py (FishNativeClient),
which finds the engine through FISH_LIBRARY and binds every export by name
with ctypes (fish_native.py:123-141, 271-345). Here that client module is
imported from the reference checkout (read where it lies; nothing of it is
copied into this repository) and pointed at this library: its binding step
must succeed for every function it binds, its struct mirrors must have this
library's sizes, the ABI it reads must be one it accepts, and a load on a
machine without a CUDA device must fail cleanly through fish_last_error (the
client's own error path), not with a binding or ctypes error. Skipped where
the reference checkout is absent (the GPU boxes); the GPU side of the same
call sequence is tests/test_gpu_model.py::test_chat_turns_stats_and_cancel."""
from __future__ import annotations

import ctypes
import importlib.util
import sys

import pytest

from imurun_b200 import libpath, native


@pytest.fixture(scope="module")
def client_mod():
    from oracle.binding import ref_root
    root = ref_root()
    src = root / "model" / "fish_native.py" if root else None
    if not src or not src.exists():
        pytest.skip("reference checkout not present")
    spec = importlib.util.spec_from_file_location("fish_native_ref", src)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["fish_native_ref"] = mod
    spec.loader.exec_module(mod)
    return mod


def test_struct_mirrors_match(client_mod):
    for theirs, ours, size in ((client_mod.FishStats, native.FishStats, 1104),
                               (client_mod.FishModelInfo, native.FishModelInfo, 168),
                               (client_mod.FishAdapterInfo, native.FishAdapterInfo, 208)):
        assert ctypes.sizeof(theirs) == ctypes.sizeof(ours) == size
        assert [f[0] for f in theirs._fields_] == [f[0] for f in ours._fields_]


def test_client_binds_and_fails_cleanly_without_a_device(client_mod, monkeypatch, tmp_path):
    import torch
    if torch.cuda.is_available():
        pytest.skip("this case checks the no-device error path")
    lib_path = libpath("libfish.so")
    monkeypatch.setenv("FISH_LIBRARY", str(lib_path))
    assert client_mod.default_library_path() == lib_path

    class Cfg:
        model_path = str(tmp_path / "model.gguf")
        context_size = 256
    (tmp_path / "model.gguf").write_bytes(b"GGUF")
    client = client_mod.FishNativeClient(Cfg())
    assert client.configured and client.library_path == lib_path
    assert client.load() is False
    err = client.error or ""
    # the engine's own message came back through fish_last_error: the binding
    # step (every symbol, argtypes and restypes) passed
    assert err and not err.startswith("FISH initialisation failed"), err
    lib = ctypes.CDLL(str(lib_path))
    client._bind(lib)
    assert lib.fish_abi_version() >= 4
    assert lib.fish_version().startswith(b"fish")
    assert b"llama" in lib.fish_supported_archs()
