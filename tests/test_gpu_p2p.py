"""sb_p2p_reduce on B200s: exact against a torch fp32 sum on one GPU (also under
CUDA-graph replay), the bounded barrier giving up on a peer that never comes
(no fault, the context stays usable), and on two GPUs the two-rank reduce and
the TP=2 decoder with the peer-memory collective against NCCL."""

from __future__ import annotations

import ctypes
import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parent.parent


def _need_gpu(n=1):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} CUDA device(s)")


def expected(parts, residual):
    """Ranks summed in order in fp32, then the residual, one bf16 rounding."""
    acc = torch.zeros(parts[0].shape, dtype=torch.float32, device=parts[0].device)
    for p in parts:
        acc += p.float()
    if residual is not None:
        acc += residual.float()
    return acc.to(torch.bfloat16)


def _rand(shape, seed, device, dtype=torch.bfloat16):
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(shape, generator=g, device=device).to(dtype)


def test_single_rank_reduce_is_exact():
    _need_gpu()
    from strassen_tpu_b200.p2p import PeerReduce
    dev = torch.device("cuda", 0)
    pr = PeerReduce(1024, 384, dev, blocks=64)
    try:
        for step, (lo, hi) in enumerate([(0, 1024), (256, 768), (1000, 1001)]):
            part = pr.partial_rows(lo, hi)
            part.copy_(_rand(part.shape, 10 + step, dev))
            res = _rand(part.shape, 20 + step, dev)
            out = pr.reduce(part, res)
            assert torch.equal(out, expected([part], res)), (lo, hi)
        part = pr.partial_rows(0, 512)
        part.copy_(_rand(part.shape, 31, dev))
        res32 = _rand(part.shape, 32, dev, torch.float32)
        assert torch.equal(pr.reduce(part, res32), expected([part], res32))
        given = torch.empty_like(part)
        got, handle = pr.reduce(part, None, out=given, async_op=True)
        handle.wait()
        assert got is given and torch.equal(got, part)
        from strassen_tpu_b200 import _native
        assert _native.device_status() == 0
    finally:
        pr.close()


def test_single_rank_reduce_replays_from_a_cuda_graph():
    _need_gpu()
    from strassen_tpu_b200.p2p import PeerReduce
    dev = torch.device("cuda", 0)
    pr = PeerReduce(512, 256, dev, blocks=32)
    try:
        part = pr.partial_rows(0, 512)
        res = torch.empty_like(part)
        part.copy_(_rand(part.shape, 1, dev))
        res.copy_(_rand(part.shape, 2, dev))
        pr.reduce(part, res)  # warm-up outside the capture
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = pr.reduce(part, res)
        for i in range(3):  # the call counter advances in device memory
            part.copy_(_rand(part.shape, 40 + i, dev))
            res.copy_(_rand(part.shape, 50 + i, dev))
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, expected([part], res)), i
        del graph
        from strassen_tpu_b200 import _native
        assert _native.device_status() == 0
    finally:
        pr.close()


def test_barrier_gives_up_on_a_missing_peer():
    """Rank 0 of a two-rank group whose rank 1 never launches: the barrier wait
    runs out (2 s), the error word reads SB_P2P_ERROR_CODE, and the same
    context then computes correctly."""
    _need_gpu()
    from strassen_tpu_b200 import _native
    import strassen_tpu_b200 as sb
    lib = _native.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    assert _native.device_status() == 0
    ptrs = []
    try:
        def alloc(n):
            p, h = ctypes.c_void_p(), _native.SbIpcHandle()
            _native.check(lib.sb_p2p_buffer_alloc(n, ctypes.byref(p), ctypes.byref(h)))
            ptrs.append(p.value)
            return p.value
        g = _native.SbP2PGroup()
        g.rank, g.world = 0, 2
        for q in range(2):  # "rank 1" is local memory nobody signals from
            g.partial[q], g.reduced[q] = alloc(4096 * 2), alloc(4096 * 2)
            g.flags[q] = alloc(lib.sb_p2p_flag_bytes())
        out = torch.empty(4096, dtype=torch.bfloat16, device=dev)
        stream = torch.cuda.current_stream(dev)
        _native.check(lib.sb_p2p_reduce(stream.cuda_stream, ctypes.byref(g), 0, 4096, None,
                                        _native.SB_BF16, out.data_ptr(), 2))
        assert _native.device_status() == _native.P2P_ERROR_CODE
        assert _native.device_status() == 0  # reset by the previous read
        a = _rand((512, 512), 5, dev)
        b = _rand((512, 512), 6, dev)
        got = sb.strassen_matmul(a, b, bm=256, bn=256, bk=256).float()
        want = a.float() @ b.float()
        assert ((got - want).norm() / want.norm()).item() < 1e-2
        assert _native.device_status() == 0
    finally:
        torch.cuda.synchronize()
        for p in ptrs:
            lib.sb_p2p_buffer_free(p)


# ---------------------------------------------------------------- two GPUs
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_rank_worker(rank, world, port, result_dir):
    sys.path.insert(0, str(REPO))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    lines = []
    try:
        from strassen_tpu_b200.p2p import PeerReduce
        from strassen_tpu_b200 import _native, qwen3
        rows, cols = 2048, 1024
        pr = PeerReduce(rows, cols, dev, blocks=96)
        ok = True
        for step, (lo, hi, r32) in enumerate([(0, 2048, False), (512, 1536, True), (0, 3, False)]):
            part = pr.partial_rows(lo, hi)
            part.copy_(_rand(part.shape, 100 * step + rank, dev))
            res = _rand(part.shape, 100 * step + 77, dev, torch.float32 if r32 else torch.bfloat16)
            out = pr.reduce(part, res)
            parts = [_rand(part.shape, 100 * step + q, dev) for q in range(world)]
            ok &= torch.equal(out, expected(parts, res))
        # asynchronous, then a captured graph replayed with new partials
        part = pr.partial_rows(0, rows)
        part.copy_(_rand(part.shape, 500 + rank, dev))
        out, handle = pr.reduce(part, None, async_op=True)
        handle.wait()
        ok &= torch.equal(out, expected([_rand(part.shape, 500 + q, dev) for q in range(world)], None))
        res = _rand(part.shape, 600, dev)
        torch.cuda.synchronize()
        dist.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            gout = pr.reduce(part, res)
        for i in range(3):
            part.copy_(_rand(part.shape, 700 + 10 * i + rank, dev))
            graph.replay()
            torch.cuda.synchronize()
            ok &= torch.equal(gout, expected([_rand(part.shape, 700 + 10 * i + q, dev)
                                              for q in range(world)], res))
        del graph
        lines.append(f"reduce {'ok' if ok else 'MISMATCH'}")
        lines.append(f"status {_native.device_status()}")
        pr.close()
        # TP=2 decoder: p2p collective against NCCL, same weights and tokens.
        cfg = qwen3.QWEN3_TINY
        tokens = torch.randint(0, cfg.vocab, (4, 256), generator=torch.Generator().manual_seed(9)).to(dev)
        logits = {}
        for coll in ("nccl", "p2p"):
            tp = qwen3.TensorParallel(collective=coll)
            model = qwen3.Qwen3Prefill(cfg, tp, dev, backend="strassen",
                                       tiles=qwen3.StrassenTiles(bm=256, bk=256, qk_bn=512, up_bn=512,
                                                                 bn=512))
            logits[coll] = [model.forward(tokens, chunks=c).float() for c in (1, 2)]
            tp.close()
        n, p = logits["nccl"], logits["p2p"]
        rel = max(((p[c] - n[c]).norm() / n[c].norm()).item() for c in range(2))
        lines.append(f"decoder_rel {rel:.3e}")
        lines.append(f"p2p_chunks_equal {torch.equal(p[0], p[1])}")
        lines.append(f"status {_native.device_status()}")
    except Exception as exc:  # reported to the parent, which fails the test
        lines.append(f"error {type(exc).__name__}: {exc}")
    finally:
        (Path(result_dir) / f"rank{rank}.txt").write_text("\n".join(lines) + "\n")
        torch.cuda.synchronize()
        dist.destroy_process_group()


def test_two_rank_reduce_and_decoder():
    _need_gpu(2)
    import multiprocessing as mp
    import tempfile
    ctx = mp.get_context("spawn")
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=_two_rank_worker, args=(r, 2, port, d)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=600)
        for p in procs:
            if p.is_alive():
                p.kill()
        reports = [(Path(d) / f"rank{r}.txt").read_text() for r in range(2)]
    for r, text in enumerate(reports):
        assert "error" not in text, (r, text)
        assert "reduce ok" in text, (r, text)
        statuses = [line.split()[1] for line in text.splitlines() if line.startswith("status ")]
        assert statuses == ["0", "0"], (r, text)
        rel = float(text.split("decoder_rel ")[1].split()[0])
        assert rel < 2e-2, (r, text)
        assert "p2p_chunks_equal True" in text, (r, text)
