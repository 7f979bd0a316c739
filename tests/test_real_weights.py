"""The real-weight fixture (Qwen3-0.6B layer-0 slices, tests/golden/real_weights.*) on CPU.

The slices come from the reference's SHA-256-pinned tensors
(Strassen_MM_Focus/data/qwen3-0.6b-real-v001/tensors/*.json); here they are
checked against their own recorded digests, against the reference's files when
the reference checkout is present, and the oracle is checked on them against
the reference test suite's error bound (0 < rel-L2 < 0.02 vs fp64,
Strassen_MM_Focus/tests/test_kernels_v001.py:82-96).  The CUDA kernel's parity
on the same weights is in test_gpu_real_weights.py.
"""

from __future__ import annotations

import json
import os
from pathlib import Path

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import strassen_ref as ref


def load_real_weights():
    """{name: float32 array of the bf16 slice} and the fixture's records."""
    records = json.loads((GOLDEN / "real_weights.json").read_text())
    arrays = np.load(GOLDEN / "real_weights.npz")
    return {k: ref.from_bf16_bits(arrays[k]) for k in records}, records


def test_slices_match_their_recorded_digests():
    from make_real_weights import slice_sha256
    arrays = np.load(GOLDEN / "real_weights.npz")
    records = json.loads((GOLDEN / "real_weights.json").read_text())
    for name, rec in records.items():
        assert list(arrays[name].shape) == rec["slice_shape"]
        assert slice_sha256(arrays[name]) == rec["slice_sha256"], name


REFERENCE = Path(os.environ.get("STRASSEN_REFERENCE", "/root/reference"))


@pytest.mark.skipif(not (REFERENCE / "Strassen_MM_Focus").is_dir(), reason="reference checkout absent")
def test_slices_equal_the_reference_tensors():
    from make_real_weights import DATA, SLICES
    arrays = np.load(GOLDEN / "real_weights.npz")
    for name, (stem, rows, cols) in SLICES.items():
        meta = json.loads((REFERENCE / DATA / f"{stem}.json").read_text())
        w = np.frombuffer((REFERENCE / DATA / f"{stem}.bf16").read_bytes(), dtype="<u2").reshape(meta["shape"])
        np.testing.assert_array_equal(arrays[name], w.T[rows[0]:rows[1], cols[0]:cols[1]])


@pytest.mark.parametrize("name", ["down_t", "q_t"])
def test_oracle_error_bound_on_real_weights(name):
    w, _ = load_real_weights()
    x = ref.normal_bf16((256, w[name].shape[0]), 61)
    got = ref.strassen_matmul_ref(x, w[name], bm=256, bn=256, bk=256, output_dtype="float32")
    exact = ref.classical_f64(x, w[name])
    rel = np.linalg.norm(got - exact) / np.linalg.norm(exact)
    assert 0 < rel < 0.02, rel
