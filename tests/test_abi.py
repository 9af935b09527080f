"""The C-ABI library builds, loads and exports what include/fish/*.h declares,
with the reference's struct layouts (CPU only: no compute calls).

Struct sizes are pinned by the reference: fish_stats 1104, fish_model_info
168, fish_adapter_info 208 (reference tests/test_fish_adapter_binding.py:177
and model/fish_native.py:43-120).
"""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def lib():
    from imurun_b200 import native
    return native.load_library()


def declared_symbols():
    names = set()
    for h in (ROOT / "include" / "fish").glob("*.h"):
        txt = h.read_text()
        for m in re.finditer(r"^FISH_API\s+[^;(]*?\b(\w+)\s*\(", txt, re.M):
            names.add(m.group(1))
    return names


def test_exports_every_declared_symbol():
    from imurun_b200 import libpath
    out = subprocess.run(["nm", "-D", "--defined-only", str(libpath())], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    declared = declared_symbols()
    assert len(declared) >= 28 + 15 + 8
    missing = declared - exported
    assert not missing, missing


def test_reference_abi4_set_is_complete():
    from imurun_b200 import native
    assert len(native.ABI4_FUNCTIONS) == 28
    assert set(native.ABI4_FUNCTIONS) <= declared_symbols()


def test_struct_sizes_match_reference():
    from imurun_b200.native import FishAdapterInfo, FishModelInfo, FishStats
    assert ctypes.sizeof(FishStats) == 1104
    assert ctypes.sizeof(FishModelInfo) == 168
    assert ctypes.sizeof(FishAdapterInfo) == 208


def test_c_header_struct_sizes():
    """Compile the public header and check the C struct sizes directly."""
    src = (
        '#include <fish/c_api.h>\n#include <stdio.h>\n'
        'int main(void){printf("%zu %zu %zu", sizeof(fish_stats), sizeof(fish_model_info), sizeof(fish_adapter_info));return 0;}\n'
    )
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        c = Path(d) / "s.c"
        c.write_text(src)
        exe = Path(d) / "s"
        subprocess.run(["gcc", f"-I{ROOT / 'include'}", str(c), "-o", str(exe)], check=True)
        out = subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()
    assert out == ["1104", "168", "208"]


def test_version_and_context_lifecycle(lib):
    assert lib.fish_abi_version() == 5
    assert lib.fish_version().startswith(b"fish-b200")
    assert b"llama" in lib.fish_supported_archs()
    ctx = lib.fish_create()
    assert ctx
    assert lib.fish_loaded(ctx) == 0
    assert lib.fish_chat_format(ctx) == b"none"
    assert lib.fish_tokenize(ctx, b"hi", 1, None, 0) == -1
    assert lib.fish_kv_len(ctx) == -1
    assert lib.fish_prefill_ids(ctx, None, 0, 0, None) == -1
    # adapter requested before a model: remembered, reported as pending
    from imurun_b200.native import FishAdapterInfo, FishStats
    assert lib.fish_set_adapter(ctx, b"/tmp/x/lora.gguf", 1.0) == 0
    info = FishAdapterInfo()
    assert lib.fish_adapter_info_of(ctx, ctypes.byref(info)) == 0
    assert info.pending == 1 and info.name == b"lora.gguf"
    assert lib.fish_clear_adapter(ctx) == 0
    # a draft model needs a loaded target (reference c_api.cpp:410-413)
    assert lib.fish_set_draft(ctx, b"/tmp/x/draft.gguf", 4) == -1
    assert b"target" in lib.fish_last_error(ctx)
    assert lib.fish_set_draft(None, b"x", 4) == -1
    lib.fish_clear_draft(ctx)
    lib.fish_clear_draft(None)
    st = FishStats()
    lib.fish_get_stats(ctx, ctypes.byref(st))
    assert st.draft_active == 0
    lib.fish_destroy(ctx)


def test_null_context_is_safe(lib):
    assert lib.fish_load(None, b"x", 0) == -1
    assert lib.fish_last_error(None) == b"null context"
    lib.fish_destroy(None)
    lib.fish_cancel(None)
    lib.fish_reset(None)


def test_load_without_gpu_fails_loudly(lib, tiny_gguf):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    ctx = lib.fish_create()
    rc = lib.fish_load(ctx, str(tiny_gguf).encode(), 2048)
    assert rc == -2
    assert b"no CUDA device" in lib.fish_last_error(ctx)
    lib.fish_destroy(ctx)
