"""GGUF container parity with the reference FISH engine, on the CPU. Both
readers open the same synthetic GGUF: the reference's GgufFile
(model/fish/include/fish/gguf.h:77-116, compiled here from its own sources
into oracle/_ref with the ref_gguf_digest probe) and this library's reader
(fbx_gguf_digest). Each returns one line per tensor (name, type, dimensions,
absolute file offset of the data, byte count) and one line per requested
metadata key (kind and value, arrays as counts plus an FNV-1a digest of the
contents); the two texts must be equal. The keys are the ones the model
loaders read (hyperparameters, tokenizer tables, MoE counts) and one that no
file has."""
from __future__ import annotations

import ctypes

import pytest

from imurun_b200 import native

P, I, CP = ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p
SUFFIXES = ["block_count", "context_length", "embedding_length", "feed_forward_length",
            "attention.head_count", "attention.head_count_kv", "attention.layer_norm_rms_epsilon",
            "rope.freq_base", "rope.dimension_count", "expert_count", "expert_used_count", "vocab_size",
            "attn_logit_softcapping", "final_logit_softcapping", "attention.sliding_window",
            "rope.scaling.type", "rope.scaling.original_context_length", "rope.scaling.attn_factor",
            "expert_feed_forward_length", "expert_shared_feed_forward_length"]
GENERAL = ["general.architecture", "general.name", "general.alignment", "tokenizer.ggml.model",
           "tokenizer.ggml.tokens", "tokenizer.ggml.scores", "tokenizer.ggml.token_type",
           "tokenizer.ggml.bos_token_id", "tokenizer.ggml.eos_token_id", "tokenizer.ggml.add_bos_token",
           "tokenizer.chat_template", "no.such.key"]


@pytest.fixture(scope="module")
def ref_lib():
    from oracle.binding import REF_SO
    if not REF_SO.exists():
        pytest.skip("reference build (oracle/_ref) not present")
    L = ctypes.CDLL(str(REF_SO))
    L.ref_gguf_digest.argtypes = [CP, P, I, ctypes.c_char_p, I]
    L.ref_gguf_digest.restype = I
    return L


@pytest.fixture(scope="module")
def ours():
    L = native.load_library()
    L.fbx_gguf_digest.argtypes = [CP, P, I, ctypes.c_char_p, I]
    L.fbx_gguf_digest.restype = I
    return L


def _digest(fn, path, keys):
    arr = (ctypes.c_char_p * max(len(keys), 1))(*[k.encode() for k in keys])
    n = fn(str(path).encode(), ctypes.cast(arr, P), len(keys), None, 0)
    assert n >= 0
    buf = ctypes.create_string_buffer(n + 1)
    assert fn(str(path).encode(), ctypes.cast(arr, P), len(keys), buf, n + 1) == n
    return buf.raw[:n].decode()


@pytest.mark.parametrize("name", ["tiny", "qwen7b", "mixtral", "gemma2", "phi3", "qwen2moe"])
def test_gguf_digest_matches_reference(ref_lib, ours, synth_dir, name):
    from imurun_b200 import synth
    cfg = {"tiny": lambda: synth.preset("tiny"),
           "qwen7b": lambda: synth.preset("qwen7b", layers=1),
           "mixtral": lambda: synth.preset("mixtral", layers=1, n_embd=512, n_ff=1024, n_head=8,
                                                 n_head_kv=2),
           "gemma2": lambda: synth.preset("gemma2", layers=1),
           "phi3": lambda: synth.preset("phi3", layers=1),
           "qwen2moe": lambda: synth.preset("qwen2moe", layers=1)}[name]()
    path = synth.cached(cfg, synth_dir)
    arch_line = _digest(ours.fbx_gguf_digest, path, ["general.architecture"]).splitlines()[-1]
    arch = arch_line.split(" ", 3)[3]
    keys = GENERAL + [f"{arch}.{s}" for s in SUFFIXES]
    got = _digest(ours.fbx_gguf_digest, path, keys)
    want = _digest(ref_lib.ref_gguf_digest, path, keys)
    assert got.count("\nT ") + got.startswith("T ") > 0
    assert got.splitlines() == want.splitlines()


def test_unreadable_file(ours):
    assert ours.fbx_gguf_digest(b"/nonexistent.gguf", None, 0, None, 0) == -1


def test_synth_refuses_without_disk_space_and_leaves_no_partial_file(tmp_path, monkeypatch):
    """The synthetic-model cache checks free space against the file's size
    before writing (a 70B file is 42.5 GB) and leaves no partial file behind
    when it refuses or when a write fails."""
    import shutil
    from collections import namedtuple
    from imurun_b200 import synth
    cfg = synth.preset("llama70b")
    est = synth.size_estimate(cfg)
    assert 42e9 < est < 46e9   # the real file is 42.5 GB
    Usage = namedtuple("Usage", "total used free")
    monkeypatch.setattr(shutil, "disk_usage", lambda p: Usage(10 ** 12, 10 ** 12 - 10 ** 9, 10 ** 9))
    with pytest.raises(RuntimeError, match="not enough disk space"):
        synth.cached(cfg, tmp_path)
    assert list(tmp_path.iterdir()) == []

    def failing_write(path, c, threads=0):
        open(path, "wb").write(b"partial")
        raise RuntimeError("fish_synth_write failed: write failed")
    monkeypatch.setattr(shutil, "disk_usage", lambda p: Usage(10 ** 12, 0, 10 ** 12))
    monkeypatch.setattr(synth, "write", failing_write)
    with pytest.raises(RuntimeError, match="write failed"):
        synth.cached(synth.preset("tiny"), tmp_path)
    assert list(tmp_path.iterdir()) == []


@pytest.mark.parametrize("damage", ["magic", "version", "truncated_header", "truncated_data", "huge_count",
                                    "bad_type", "empty"])
def test_damaged_files_rejected_like_reference(ref_lib, ours, synth_dir, tmp_path, damage):
    """A damaged GGUF is refused by this library's reader exactly when the
    reference's GgufFile refuses it (src/gguf.cpp), and when both accept it
    they read the same directory: wrong magic or version, a header or data
    cut short, an absurd tensor count, an unknown tensor type, an empty
    file."""
    import struct
    from imurun_b200 import synth
    src = synth.cached(synth.preset("tiny", layers=1), synth_dir)
    b = bytearray(src.read_bytes())
    if damage == "magic":
        b[0:4] = b"GGUX"
    elif damage == "version":
        b[4:8] = struct.pack("<I", 99)
    elif damage == "truncated_header":
        b = b[:200]
    elif damage == "truncated_data":
        b = b[:len(b) - 4096]
    elif damage == "huge_count":
        b[8:16] = struct.pack("<Q", 1 << 40)
    elif damage == "bad_type":
        # the first tensor's type field: after its name, n_dims and dims
        hdr_end = b.find(b"token_embd.weight")
        assert hdr_end > 0
        p = hdr_end + len(b"token_embd.weight")
        n_dims = struct.unpack_from("<I", b, p)[0]
        p += 4 + 8 * n_dims
        b[p:p + 4] = struct.pack("<I", 250)
    elif damage == "empty":
        b = bytearray()
    path = tmp_path / f"{damage}.gguf"
    path.write_bytes(bytes(b))
    keys = ["general.architecture"]
    arr = (ctypes.c_char_p * 1)(*[k.encode() for k in keys])
    want = ref_lib.ref_gguf_digest(str(path).encode(), ctypes.cast(arr, P), 1, None, 0)
    got = ours.fbx_gguf_digest(str(path).encode(), ctypes.cast(arr, P), 1, None, 0)
    assert (got < 0) == (want < 0), (damage, got, want)
    if want >= 0:
        assert _digest(ours.fbx_gguf_digest, path, keys).splitlines() == \
            _digest(ref_lib.ref_gguf_digest, path, keys).splitlines()
