"""bench.py's synthetic inputs and its use of the oracle (no GPU).

The GPU arm builds its inputs itself; the oracle is the checker and the CPU
baseline only, so `cpu_baseline` is the one function of bench.py that may
import it.  The inputs must still be the oracle's recipe bit for bit, since
the CPU leg times the same sample.
"""

import ast
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO))

import bench  # noqa: E402
from oracle import strassen_ref as ref  # noqa: E402


@pytest.mark.parametrize("shape,seed,chunk", [((64, 96), 1, 1024), ((3000, 40), bench.SEED_A, 7),
                                              ((1, 1), 5, 1), ((257, 33), bench.SEED_B, 256)])
def test_inputs_are_the_oracle_recipe_bit_for_bit(shape, seed, chunk):
    got = bench.normal_bf16_bits(shape, seed, rows_per_chunk=chunk)
    want = ref.bf16_bits(ref.normal_bf16(shape, seed))
    assert got.dtype == np.uint16 and got.shape == want.shape
    assert np.array_equal(got, want)


def test_only_the_cpu_baseline_imports_the_oracle():
    tree = ast.parse((REPO / "bench.py").read_text())
    importers = set()
    for fn in ast.walk(tree):
        if not isinstance(fn, ast.FunctionDef):
            continue
        for node in ast.walk(fn):
            if isinstance(node, ast.ImportFrom) and (node.module or "").split(".")[0] == "oracle":
                importers.add(fn.name)
            if isinstance(node, ast.Import) and any(a.name.split(".")[0] == "oracle" for a in node.names):
                importers.add(fn.name)
    top_level = [n for n in tree.body if isinstance(n, (ast.Import, ast.ImportFrom))
                 and "oracle" in ast.dump(n)]
    assert not top_level
    assert importers == {"cpu_baseline"}
