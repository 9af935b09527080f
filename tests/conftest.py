"""Shared fixtures.

Markers: `gpu` tests need a B200 (they run through the product's C ABI);
everything else runs on the CPU.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "golden.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device")


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="session")
def oracle():
    from oracle.binding import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.binding import REF_SO, Reference
    if not REF_SO.exists():
        pytest.skip("reference build (oracle/_ref) not present")
    return Reference()


@pytest.fixture(scope="session")
def synth_dir(tmp_path_factory):
    d = os.environ.get("FISH_SYNTH_DIR")
    return Path(d) if d else tmp_path_factory.mktemp("synth")


@pytest.fixture(scope="session")
def tiny_gguf(synth_dir):
    from imurun_b200 import synth
    return synth.cached(synth.preset("tiny"), synth_dir)
