"""Shared fixtures: golden vectors produced by the reference's own kernel code."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden"
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(GOLDEN))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    config.addinivalue_line("markers", "slow: long-running (full-size) case")


@pytest.fixture(scope="session")
def golden_lhs_t():
    """(manifest, arrays) of the reference's strassen_matmul_lhs_transposed outputs."""
    manifest = json.loads((GOLDEN / "golden_cases.json").read_text())["lhs_transposed_cases"]
    arrays = np.load(GOLDEN / "golden_outputs.npz")
    return manifest, {k.split("/", 1)[1]: arrays[k] for k in arrays.files if k.startswith("lhs_t/")}


@pytest.fixture(scope="session")
def golden():
    """(manifest, arrays): reference outputs keyed by case name."""
    manifest = json.loads((GOLDEN / "golden_cases.json").read_text())["cases"]
    arrays = np.load(GOLDEN / "golden_outputs.npz")
    return manifest, {k: arrays[k] for k in arrays.files if "/" not in k}


def golden_output(p, arr):
    from oracle import strassen_ref as ref
    if p["output"] == "bf16_bits":
        return ref.from_bf16_bits(arr)
    return np.asarray(arr, np.float32)
