"""The peer-memory row reduction without a GPU: the kernel's element partition
(restated here) covers every element once per phase and pairs each phase-2 read
with the phase-1 write of the same CTA index, and the C ABI and the Python
wrapper reject bad arguments on the host."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from strassen_tpu_b200 import _native, qwen3

THREADS = 512  # kP2PThreads in csrc/p2p_reduce.cuh


def slice_begin(vecs, r, world):
    return vecs * r // world


def assignment(vecs, world, blocks):
    """(phase-1 writer CTA per vector, phase-2 reader CTA per (rank, vector)), as
    p2p_reduce_kernel indexes: CTA b, thread t handles lo + b*T + t + k*G*T."""
    stride = blocks * THREADS
    writer = np.full(vecs, -1)
    count1 = np.zeros(vecs, dtype=int)
    for r in range(world):
        lo, hi = slice_begin(vecs, r, world), slice_begin(vecs, r + 1, world)
        for b in range(blocks):
            for t in range(THREADS):
                v = np.arange(lo + b * THREADS + t, hi, stride)
                writer[v] = b
                count1[v] += 1
    readers = np.full((world, vecs), -1)
    count2 = np.zeros((world, vecs), dtype=int)
    for q in range(world):
        for j in range(world):
            r = (q + j) % world
            lo, hi = slice_begin(vecs, r, world), slice_begin(vecs, r + 1, world)
            for b in range(blocks):
                for t in range(THREADS):
                    v = np.arange(lo + b * THREADS + t, hi, stride)
                    readers[q, v] = b
                    count2[q, v] += 1
    return writer, count1, readers, count2


@pytest.mark.parametrize("vecs,world,blocks", [(1, 1, 1), (37, 2, 3), (4096, 8, 2), (100003, 3, 5),
                                                (8 * 512 * 4 + 5, 8, 4)])
def test_partition_covers_once_and_pairs_reads_with_writes(vecs, world, blocks):
    writer, count1, readers, count2 = assignment(vecs, world, blocks)
    assert (count1 == 1).all()          # phase 1: every vector reduced exactly once
    assert (count2 == 1).all()          # phase 2: every rank copies every vector once
    assert (readers == writer[None, :]).all()  # CTA b reads only what CTA b wrote


def test_slices_tile_the_range():
    for vecs in (0, 1, 7, 8, 1000, 2**33 + 3):
        for world in range(1, 9):
            edges = [slice_begin(vecs, r, world) for r in range(world + 1)]
            assert edges[0] == 0 and edges[-1] == vecs
            assert all(a <= b for a, b in zip(edges, edges[1:]))


def test_flag_bytes():
    lib = _native.load()
    assert lib.sb_p2p_flag_bytes() == (2 * 256 * 8 + 32) * 4


def _group(world=2, rank=0, base=0x10000):
    g = _native.SbP2PGroup()
    g.rank, g.world = rank, world
    for q in range(min(world, 8)):
        g.partial[q] = base + 0x1000 * (3 * q)
        g.reduced[q] = base + 0x1000 * (3 * q + 1)
        g.flags[q] = base + 0x1000 * (3 * q + 2)
    return g


def _call(g, offset=0, elems=64, residual=None, dtype=_native.SB_BF16, out=0x900000, blocks=4):
    lib = _native.load()
    return lib.sb_p2p_reduce(None, ctypes.byref(g) if g is not None else None, offset, elems,
                             residual, dtype, out, blocks)


@pytest.mark.parametrize("mutate,status", [
    (lambda g: setattr(g, "world", 0), _native.SB_ERR_P2P),
    (lambda g: setattr(g, "world", 9), _native.SB_ERR_P2P),
    (lambda g: setattr(g, "rank", 2), _native.SB_ERR_P2P),
    (lambda g: setattr(g, "rank", -1), _native.SB_ERR_P2P),
    (lambda g: g.partial.__setitem__(1, None), _native.SB_ERR_P2P),
    (lambda g: g.flags.__setitem__(0, 0x10008), 9),  # SB_ERR_ALIGNMENT
])
def test_bad_groups_are_rejected_on_the_host(mutate, status):
    g = _group()
    mutate(g)
    assert _call(g) == status


def test_bad_arguments_are_rejected_on_the_host():
    g = _group()
    assert _call(None) == _native.SB_ERR_P2P
    assert _call(g, elems=60) == _native.SB_ERR_P2P
    assert _call(g, elems=0) == _native.SB_ERR_P2P
    assert _call(g, offset=4) == _native.SB_ERR_P2P
    assert _call(g, out=0x900008) == 9
    assert _call(g, out=None) == 9
    assert _call(g, residual=0x800004) == 9
    assert _call(g, dtype=7) == 3  # SB_ERR_DTYPE
    assert _call(g, blocks=0) == _native.SB_ERR_P2P
    assert _call(g, blocks=257) == _native.SB_ERR_P2P
    msg = _native.load().sb_last_error_message().decode()
    assert "blocks" in msg


def test_buffer_calls_reject_null_arguments():
    lib = _native.load()
    assert lib.sb_p2p_buffer_alloc(0, None, None) == _native.SB_ERR_P2P
    assert lib.sb_p2p_buffer_open(None, None) == _native.SB_ERR_P2P
    assert lib.sb_p2p_buffer_close(None) == _native.SB_ERR_P2P
    assert lib.sb_p2p_buffer_free(None) == _native.SB_ERR_P2P


def test_peer_reduce_rejects_bad_shapes_before_touching_a_device():
    from strassen_tpu_b200.p2p import PeerReduce
    with pytest.raises(ValueError, match="multiple of 8"):
        PeerReduce(16, 12, "cpu")
    with pytest.raises(ValueError, match="blocks"):
        PeerReduce(16, 16, "cpu", blocks=0)


def test_tensor_parallel_collective_choice():
    with pytest.raises(ValueError, match="collective"):
        qwen3.TensorParallel(collective="mpi")
    tp = qwen3.TensorParallel(collective="p2p")
    assert not tp.peer_reduce  # one rank: nothing to reduce
    tp.ensure_buffers(16, 64, "cpu")
    assert tp.peer is None and tp.partial_out(0, 16) is None
    x = torch.ones(4, 8)
    assert tp.all_reduce(x) is x
    out, handle = tp.all_reduce_async(x)
    assert out is x and handle is None


def test_p2p_without_buffers_is_a_clear_error():
    tp = qwen3.TensorParallel(collective="p2p")
    tp.world = 2  # as a two-rank group would report, before ensure_buffers
    with pytest.raises(RuntimeError, match="ensure_buffers"):
        tp.partial_out(0, 16)


def test_single_rank_forward_is_the_same_for_either_collective():
    cfg = qwen3.QWEN3_TINY
    tokens = torch.randint(0, cfg.vocab, (2, 16), generator=torch.Generator().manual_seed(3))
    a = qwen3.Qwen3Prefill(cfg, qwen3.TensorParallel(), "cpu", backend="native", layers=2)
    b = qwen3.Qwen3Prefill(cfg, qwen3.TensorParallel(collective="p2p"), "cpu", backend="native", layers=2)
    assert torch.equal(a.forward(tokens), b.forward(tokens))


def _mismatch_worker(rank, world, port, out_dir):
    import os
    from datetime import timedelta
    import torch.distributed as dist
    from strassen_tpu_b200.p2p import PeerReduce
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    try:
        try:
            PeerReduce(64, 64, "cpu", blocks=16 * (rank + 1))  # ranks disagree on the grid
            msg = "no error"
        except ValueError as exc:
            msg = str(exc)
        with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
            f.write(msg)
    finally:
        dist.destroy_process_group()


def test_peer_reduce_ranks_must_agree_on_grid(tmp_path):
    """Every rank learns of a (rows, cols, blocks) mismatch and raises before any
    buffer is allocated (world size 2, gloo, CPU)."""
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_mismatch_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        assert "differ across ranks" in (tmp_path / f"rank{r}.txt").read_text()
