"""Parity at every shape of the benchmark sweep, at the tile the
tuning table records for it (needs a B200).

The reference gates every timed shape on correctness before it reports a time
(experiments/qwen3/benchmark_cubic_control.py:387-451): the Strassen output
against an fp32 classical product, rmse <= 4x the native bf16 GEMM's rmse and
max-norm relative error <= 0.01 (:322-384).  Here each shape gets that gate on
the whole output, plus an oracle comparison on sampled rows:

* tile-local Strassen pairs output row I*bm + r' only with row I*bm + bm/2 + r'
  (the A quadrant split, strassen_pallas.py:188-204), so the rows r' < 64 of both
  halves of a block are reproduced exactly by the oracle run on just those 128 A
  rows with bm = 128 and the same bn, bk;
* those rows are checked at the strict bar in fp32 output (max|diff| <=
  2e-2 rms, error vs fp64 <= 2x the oracle's) and at the bf16 rounding-step bar
  in bf16 output, for the first and the last block row.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import strassen_ref as ref
from test_gpu_parity import assert_parity, dev_bf16, host

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

TABLE = Path(__file__).resolve().parent.parent / "strassen_tpu_b200" / "b200_tuning.json"
SAMPLE_ROWS = 64

# (m, k, n): squares 2048/4096/16384 (8192^3 has its own test) and the Qwen3-8B
# projection shapes at M = 4096 tokens (K x N = 4096x4096 is the 4096^3 square).
SWEEP = [
    (2048, 2048, 2048),
    (4096, 4096, 4096),
    (16384, 16384, 16384),
    (4096, 4096, 1024),
    (4096, 4096, 12288),
    (4096, 12288, 4096),
]


def table_tile(m, k, n):
    shapes = json.loads(TABLE.read_text())["shapes"]
    entry = shapes.get(f"{m}x{k}x{n}")
    if entry is not None:
        return tuple(entry["tile"])
    return (1024, 1024, 512)


def sampled_rows(m, bm):
    """Output rows r' < SAMPLE_ROWS of both halves of the first and last block."""
    h = bm // 2
    rows = []
    for blk in (0, m // bm - 1):
        base = blk * bm
        rows.append(np.arange(base, base + SAMPLE_ROWS))
        rows.append(np.arange(base + h, base + h + SAMPLE_ROWS))
    return np.concatenate(rows)


@pytest.mark.slow
@pytest.mark.parametrize("m, k, n", SWEEP, ids=[f"{m}x{k}x{n}" for m, k, n in SWEEP])
def test_sweep_shape(m, k, n):
    import strassen_tpu_b200 as sb
    from strassen_tpu_b200 import _native
    bm, bn, bk = table_tile(m, k, n)
    assert m % bm == 0 and n % bn == 0 and k % bk == 0
    a = ref.normal_bf16((m, k), 20260902)
    b = ref.normal_bf16((k, n), 20260903)
    ad, bd = dev_bf16(a), dev_bf16(b)
    got = sb.strassen_matmul(ad, bd, bm=bm, bn=bn, bk=bk)
    got32 = sb.strassen_matmul(ad, bd, bm=bm, bn=bn, bk=bk, output_dtype=torch.float32)
    torch.cuda.synchronize()
    assert _native.device_status() == 0

    rows = sampled_rows(m, bm)
    a_rows = a[rows]
    # Two blocks of 2 x SAMPLE_ROWS rows each, at bm = 2 * SAMPLE_ROWS.
    want32 = ref.strassen_matmul_ref(a_rows, b, bm=2 * SAMPLE_ROWS, bn=bn, bk=bk, output_dtype="float32")
    exact = ref.classical_f64(a_rows, b)
    idx = torch.from_numpy(rows).cuda()
    assert_parity(host(got32.index_select(0, idx)), want32, exact)
    assert_parity(host(got.index_select(0, idx)), ref.bf16_round(want32), exact, rounding_step=True)

    # Whole output: the reference's gate against an fp32 classical product.
    fp32 = torch.matmul(ad.float(), bd.float())
    native = torch.matmul(ad, bd).float()
    err = got.float() - fp32
    rmse = err.pow(2).mean().sqrt().item()
    nat_rmse = (native - fp32).pow(2).mean().sqrt().item()
    maxnorm = (err.abs().max() / fp32.abs().max()).item()
    assert rmse <= 4.0 * nat_rmse, (rmse, nat_rmse)
    assert maxnorm <= 0.01, maxnorm


@pytest.mark.slow
@pytest.mark.parametrize("path", ["one_cta", "planes"])
def test_whole_output_against_the_oracle_2048(path):
    """The parity rule on a whole 2048^3 output (not sampled rows): max|diff|
    <= 2e-2 rms and rmse vs fp64 <= 2x the oracle's, in fp32 and in bf16, for
    the one-CTA kernel and the planes path."""
    import strassen_tpu_b200 as sb
    m = k = n = 2048
    tile = dict(bm=1024, bn=1024, bk=512)
    a = ref.normal_bf16((m, k), 20260904)
    b = ref.normal_bf16((k, n), 20260905)
    ad, bd = dev_bf16(a), dev_bf16(b)
    if path == "planes":
        got32 = sb.planes_matmul(ad, bd, output_dtype=torch.float32, **tile)
        got = sb.planes_matmul(ad, bd, **tile)
    else:
        got32 = sb.strassen_matmul(ad, bd, output_dtype=torch.float32, **tile)
        got = sb.strassen_matmul(ad, bd, **tile)
    torch.cuda.synchronize()
    want32 = ref.strassen_matmul_ref(a, b, output_dtype="float32", **tile)
    exact = ref.classical_f64(a, b)
    assert_parity(host(got32), want32, exact)
    assert_parity(host(got), ref.bf16_round(want32), exact, rounding_step=True)
