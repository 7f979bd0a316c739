"""The measured Strassen-vs-native dispatcher and the tile tuner's host logic.

Reference: strassen_pallas.py:1428-1461 (tuned_matmul),
benchmark_common.py:94-120 (rotated arm order),
benchmark_qwen3_site_tile_tune.py (per-site tile screen).
"""

from __future__ import annotations

import json

import pytest
import torch

from strassen_tpu_b200 import tuning
from strassen_tpu_b200.tuning import ShapeEntry, TuningTable


def _table(crossover=None, **shapes):
    t = TuningTable(square_crossover=crossover)
    for key, (winner, tile) in shapes.items():
        m, k, n = (int(x) for x in key.lstrip("s").split("x"))
        t.shapes[ShapeEntry.key(m, k, n)] = ShapeEntry(m, k, n, winner, tile)
    return t


def test_shipped_table_loads_and_is_measured():
    t = TuningTable.load(tuning.DEFAULT_TABLE)
    assert "B200" in t.device
    assert len(t.shapes) >= 10
    for e in t.shapes.values():
        assert e.strassen_ms and e.native_ms and e.ci95
        # the winner follows the recorded paired CI
        assert (e.winner == "strassen") == (e.ci95[0] > 1.0)
    assert t.square_crossover == tuning.square_crossover(t.shapes.values())


def test_table_round_trips(tmp_path):
    t = _table(8192, s8192x4096x8192=("strassen", (1024, 1024, 512)),
               s4096x4096x1024=("native", (512, 512, 512)))
    path = tmp_path / "t.json"
    t.save(path)
    u = TuningTable.load(path)
    assert u.square_crossover == 8192 and u.shapes == t.shapes


@pytest.mark.parametrize("bad, msg", [
    ({"schema": 99}, "schema"),
    ({"schema": 1, "square_crossover": -4}, "square_crossover"),
    ({"schema": 1, "shapes": {"1x2x3": {"m": 1, "k": 2, "n": 4, "winner": "native", "tile": [1, 1, 1]}}},
     "does not match"),
    ({"schema": 1, "shapes": {"1x2x3": {"m": 1, "k": 2, "n": 3, "winner": "xla", "tile": [1, 1, 1]}}},
     "winner"),
])
def test_table_validation(bad, msg):
    with pytest.raises(ValueError, match=msg):
        TuningTable.from_json(bad)


def test_plan_follows_measured_wins():
    t = _table(None, s8192x4096x8192=("strassen", (1024, 1024, 512)),
               s4096x4096x4096=("native", (1024, 1024, 512)))
    d = tuning.plan(8192, 4096, 8192, table=t)
    assert d.arm == "strassen" and d.tile == (1024, 1024, 512)
    assert tuning.plan(4096, 4096, 4096, table=t).arm == "native"
    assert tuning.plan(2048, 2048, 2048, table=t).arm == "native"          # unmeasured
    assert tuning.plan(8192, 4096, 8192, k2=2048, table=t).arm == "native"  # inner mismatch
    assert tuning.plan(8192, 4096, 8192, bf16=False, table=t).arm == "native"
    assert tuning.plan(8192, 4096, 8192, on_device=False, table=t).arm == "native"


def test_plan_square_crossover_uses_default_tile():
    t = _table(8192)
    d = tuning.plan(16384, 16384, 16384, table=t)
    assert d.arm == "strassen" and d.tile == (tuning.TUNED_BM, tuning.TUNED_BN, tuning.TUNED_BK)
    assert tuning.plan(4096, 4096, 4096, table=t).arm == "native"
    assert tuning.plan(8192, 8192, 4096, table=t).arm == "native"          # not square
    # a crossover square that the default tile does not divide stays native
    assert tuning.plan(8192 + 512, 8192 + 512, 8192 + 512, table=t).arm == "native"


def test_tuned_matmul_non_matrix_and_cpu_go_native():
    t = _table(256)
    a = torch.randn(2, 3, 4)
    b = torch.randn(4, 5)
    torch.testing.assert_close(tuning.tuned_matmul(a, b, table=t), torch.matmul(a, b))
    # CPU bf16 operands at a qualifying size: no device, so the native arm
    x = torch.randn(1024, 1024).bfloat16()
    got = tuning.tuned_matmul(x, x, table=t)
    assert torch.equal(got, torch.matmul(x, x))


def test_tuned_matmul_interpret_reaches_strassen_and_refuses():
    # The reference routes interpret=True through the Strassen kernel; the B200
    # build has no CPU path and says so.
    t = _table(1024)
    x = torch.randn(1024, 1024).bfloat16()
    with pytest.raises(NotImplementedError, match="interpret"):
        tuning.tuned_matmul(x, x, interpret=True, table=t)


def test_env_selects_table(tmp_path, monkeypatch):
    path = tmp_path / "t.json"
    _table(4096).save(path)
    monkeypatch.setenv(tuning.ENV_TABLE, str(path))
    assert tuning.active_table().square_crossover == 4096
    monkeypatch.delenv(tuning.ENV_TABLE)
    assert tuning.active_table().square_crossover == TuningTable.load(tuning.DEFAULT_TABLE).square_crossover


def test_candidate_tiles_respect_kernel_rules():
    tiles = tuning.candidate_tiles(8192, 4096, 8192)
    assert (1024, 1024, 512) in tiles and (2048, 1024, 2048) in tiles
    assert tuning.candidate_tiles(16384, 4096, 1024) == [
        (bm, bn, bk) for bm in (512, 1024, 2048) for bn in (512, 1024) for bk in (512, 2048)]
    assert tuning.candidate_tiles(1000, 4096, 4096) == []
    # bm/2 must be a multiple of 128 or a power of two below it
    assert tuning.candidate_tiles(4096, 512, 512, bms=(96, 384, 64), bns=(512,), bks=(512,)) == [
        (64, 512, 512)]


def test_rotated_order_balances_positions():
    names = ["native", "a", "b"]
    firsts = [tuning.rotated_order(names, r)[0] for r in range(6)]
    assert sorted(firsts) == sorted(names * 2)
    assert tuning.rotated_order(names, 0) == names
    assert tuning.rotated_order(names, 1) == list(reversed(names[1:] + names[:1]))


def test_paired_speedup_and_crossover():
    s, ci = tuning.paired_speedup([2.0, 2.2, 2.1], [1.0, 1.1, 1.05])
    assert s == pytest.approx(2.0) and ci[0] <= 2.0 <= ci[1]
    e = lambda m, w: ShapeEntry(m, m, m, w, (1024, 1024, 512))
    assert tuning.square_crossover([e(2048, "native"), e(4096, "strassen"), e(8192, "strassen")]) == 4096
    assert tuning.square_crossover([e(4096, "strassen"), e(8192, "native")]) is None
    assert tuning.square_crossover([]) is None


@pytest.mark.gpu
def test_tuned_matmul_matches_the_chosen_arm():
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(5)
    a = torch.randn(2048, 1024, device=dev, generator=g).bfloat16()
    b = torch.randn(1024, 2048, device=dev, generator=g).bfloat16()
    from strassen_tpu_b200 import native_matmul, strassen_matmul
    win = _table(None, s2048x1024x2048=("strassen", (1024, 1024, 512)))
    torch.testing.assert_close(tuning.tuned_matmul(a, b, table=win),
                               strassen_matmul(a, b, bm=1024, bn=1024, bk=512), rtol=0, atol=0)
    lose = _table(None, s2048x1024x2048=("native", (1024, 1024, 512)))
    assert torch.equal(tuning.tuned_matmul(a, b, table=lose), native_matmul(a, b))


@pytest.mark.gpu
def test_tuner_measures_a_shape():
    lines = []
    e = tuning.tune_shape(1024, 1024, 1024, tiles=[(512, 512, 512), (1024, 1024, 1024)],
                          screen_runs=2, warmups=3, runs=4, log=lines.append)
    assert e.tile in ((512, 512, 512), (1024, 1024, 1024))
    assert e.strassen_ms > 0 and e.native_ms > 0 and e.winner in ("strassen", "native")
    assert lines and "1024x1024x1024" in lines[0]
    json.dumps(TuningTable(shapes={"x": e}).to_json())
