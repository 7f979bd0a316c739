"""Tensor-parallel Qwen3 decoder: sharding math and failure handling on CPU ranks.

world_size-2 gloo process groups on 127.0.0.1 run the decoder with the native
(classical) arm, so the column/row splits, the per-rank layouts and the
residual-once all-reduce are checked without a GPU.  The failure test makes a
rank die before its collective and checks that the survivor gets an error
within the process-group timeout instead of hanging.
"""

from __future__ import annotations

import os
import socket
import time
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from strassen_tpu_b200 import qwen3

CFG = qwen3.QWEN3_TINY
BATCH, SEQ = 2, 32


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tokens():
    g = torch.Generator().manual_seed(5)
    return torch.randint(0, CFG.vocab, (BATCH, SEQ), generator=g)


def _tp_worker(rank, world, port, out_path, chunks=1):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        tp = qwen3.TensorParallel()
        model = qwen3.Qwen3Prefill(CFG, tp, "cpu", backend="native")
        logits = model.forward(_tokens(), chunks=chunks)
        if rank == 0:
            torch.save(logits, out_path)
    finally:
        dist.destroy_process_group()


def test_tp2_matches_tp1_on_cpu_ranks(tmp_path):
    out = tmp_path / "tp2.pt"
    mp.spawn(_tp_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    tp2 = torch.load(out).float()
    single = qwen3.Qwen3Prefill(CFG, qwen3.TensorParallel(), "cpu", backend="native")
    tp1 = single.forward(_tokens()).float()
    rel = (tp2 - tp1).norm() / tp1.norm()
    assert rel < 3e-2, rel.item()


def test_shards_partition_the_full_weights():
    class FakeTP:
        def __init__(self, rank, world):
            self.rank, self.world = rank, world

        def all_reduce(self, x):
            return x

    full = qwen3.build_layer(CFG, 0, FakeTP(0, 1), "cpu", backend="native")
    parts = [qwen3.build_layer(CFG, 0, FakeTP(r, 2), "cpu", backend="native") for r in range(2)]
    for name in ("q", "k", "v"):
        joined = torch.cat([p.sites[name].weight for p in parts], dim=1)
        assert torch.equal(joined, full.sites[name].weight), name
    for name in ("o", "down"):
        joined = torch.cat([p.sites[name].weight for p in parts], dim=0)
        assert torch.equal(joined, full.sites[name].weight), name
    # gate/up: each rank holds [gate_r | up_r]; together they are the full gate and up.
    ir = CFG.intermediate
    gate = torch.cat([p.sites["up"].weight[:, : ir // 2] for p in parts], dim=1)
    up = torch.cat([p.sites["up"].weight[:, ir // 2:] for p in parts], dim=1)
    assert torch.equal(gate, full.sites["up"].weight[:, :ir])
    assert torch.equal(up, full.sites["up"].weight[:, ir:])


def test_tp_size_must_divide_heads():
    class FakeTP:
        rank, world = 0, 3

    with pytest.raises(ValueError, match="does not divide"):
        qwen3.build_layer(CFG, 0, FakeTP(), "cpu", backend="native")


def _dying_worker(rank, world, port, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # dies between steps, with nothing in flight
    t0 = time.monotonic()
    x = torch.ones(8)
    try:
        dist.all_reduce(x)
        outcome = "completed"
    except Exception as exc:  # the survivor must learn of the failure, not hang
        outcome = f"error:{type(exc).__name__}"
    with open(result_path, "w") as f:
        f.write(f"{outcome} {time.monotonic() - t0:.1f}")
    os._exit(0)


def test_dead_rank_surfaces_as_an_error_not_a_hang(tmp_path):
    result = tmp_path / "r0.txt"
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, str(result))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    outcome, seconds = result.read_text().split()
    assert outcome.startswith("error:"), outcome
    assert float(seconds) < 30


def test_chunked_pipeline_is_exact_on_one_rank():
    # Chunks are whole sequences: every op is per token or per sequence, so the
    # pipelined order changes nothing.
    model = qwen3.Qwen3Prefill(CFG, qwen3.TensorParallel(), "cpu", backend="native")
    tok = torch.randint(0, CFG.vocab, (4, SEQ), generator=torch.Generator().manual_seed(9))
    want = model.forward(tok)
    for chunks in (2, 4):
        assert torch.equal(model.forward(tok, chunks=chunks), want)
    assert torch.equal(model.forward(tok, chunks=3), want)  # 4 % 3: falls back to unchunked


def test_tp2_chunked_matches_unchunked_on_cpu_ranks(tmp_path):
    outs = []
    for chunks in (1, 2):
        out = tmp_path / f"tp2_c{chunks}.pt"
        mp.spawn(_tp_worker, args=(2, _free_port(), str(out), chunks), nprocs=2, join=True)
        outs.append(torch.load(out).float())
    # The all-reduces sum the same partials; only their message sizes differ.
    rel = (outs[1] - outs[0]).norm() / outs[0].norm()
    assert rel < 1e-2, rel.item()


def test_one_head_kv_shards_take_narrow_tiles():
    """At TP=8 with 8 kv heads every rank holds one 128-wide k and v head: those
    sites run on 128-wide Strassen tiles (narrow_bn) instead of the native arm,
    with the weight in its natural order (one head per tile is already the rope
    layout)."""
    class FakeTP:
        rank, world = 3, 8

    cfg = qwen3.Qwen3Config(hidden=1024, layers=1, heads=16, kv_heads=8, head_dim=128,
                            intermediate=4096, vocab=1000)
    layer = qwen3.build_layer(cfg, 0, FakeTP(), "cpu", backend="strassen")
    native = qwen3.build_layer(cfg, 0, FakeTP(), "cpu", backend="native")
    for name in ("k", "v"):
        site = layer.sites[name]
        assert (site.strassen, site.bn, site.narrow) == (True, 128, True), name
        assert torch.equal(site.weight, native.sites[name].weight), name
    q = layer.sites["q"]
    assert (q.strassen, q.bn, q.narrow) == (True, 256, False)
    # Two heads per rank fit the reference's bn = 2*head_dim rule: no narrow tiles.
    layer2 = qwen3.build_layer(cfg, 0, type("TP4", (), {"rank": 1, "world": 4})(), "cpu", backend="strassen")
    assert (layer2.sites["k"].bn, layer2.sites["k"].narrow) == (256, False)


def test_native_sites_take_the_native_arm():
    class FakeTP:
        rank, world = 0, 2

    layer = qwen3.build_layer(CFG, 0, FakeTP(), "cpu", backend="strassen", native_sites=frozenset({"v", "up"}))
    native = qwen3.build_layer(CFG, 0, FakeTP(), "cpu", backend="native")
    for name in ("v", "up"):
        assert not layer.sites[name].strassen
        assert torch.equal(layer.sites[name].weight, native.sites[name].weight), name
    assert layer.sites["q"].strassen and layer.sites["down"].strassen
