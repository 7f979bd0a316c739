"""Tensor-parallel row reduction over NVLink peer memory (``sb_p2p_reduce``).

The tensor-parallel decoder's row-parallel projections (o and down) leave one
partial product per rank; the block output is their sum plus the residual.
:class:`PeerReduce` owns the symmetric buffers that computation needs and runs
it as one kernel over peer memory instead of an NCCL all-reduce:

* every rank allocates a ``partial`` buffer ``[rows, cols]`` bf16, a ``reduced``
  buffer of the same size and a flag buffer (``sb_p2p_buffer_alloc``), the
  IPC handles go round with ``all_gather_object``, and every rank maps the
  others' buffers (``sb_p2p_buffer_open``);
* the row-parallel GEMM writes its partial straight into
  :meth:`PeerReduce.partial_rows` (no copy);
* :meth:`PeerReduce.reduce` launches ``sb_p2p_reduce`` on a side stream: each
  rank sums its slice of the rows over every rank's partial (fp32, ranks in
  order) plus the residual, then gathers the other slices.  The result is the
  same bf16 tensor on every rank.

Calls must come in the same order on every rank (the decoder's program order
guarantees it); each rank's calls run on one stream, which keeps the buffers'
reuse safe (see ``csrc/p2p_reduce.cuh``).  The reduce may be captured in a
CUDA graph.  One process per GPU, all GPUs of one node (NVLink peers).
"""

from __future__ import annotations

import ctypes

import torch

from . import _native


class _DeviceArray:
    """A raw device allocation exposed through ``__cuda_array_interface__``."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class _Pending:
    """Handle of an asynchronous reduce: ``wait()`` orders the current stream after it."""

    def __init__(self, event: torch.cuda.Event):
        self.event = event

    def wait(self) -> None:
        torch.cuda.current_stream().wait_event(self.event)


class PeerReduce:
    """Symmetric buffers and the ``sb_p2p_reduce`` call for one process group.

    ``rows`` x ``cols`` bounds every reduction (the decoder passes its token
    count and hidden size).  ``group``: a ``torch.distributed`` group (None =
    the default group, or a single rank when torch.distributed is not
    initialised).  ``blocks`` CTAs per call (1..256), the same on every rank.
    """

    def __init__(self, rows: int, cols: int, device, group=None, blocks: int = 128):
        import torch.distributed as dist

        if cols % 8:
            raise ValueError(f"cols must be a multiple of 8, got {cols}")
        if not 1 <= blocks <= _native.P2P_MAX_BLOCKS:
            raise ValueError(f"blocks must be 1..{_native.P2P_MAX_BLOCKS}, got {blocks}")
        self.dist = dist if dist.is_available() and dist.is_initialized() else None
        self.group = group
        self.rank = self.dist.get_rank(group) if self.dist else 0
        self.world = self.dist.get_world_size(group) if self.dist else 1
        if self.world > _native.P2P_MAX_RANKS:
            raise ValueError(f"at most {_native.P2P_MAX_RANKS} ranks, got {self.world}")
        self.device = torch.device(device)
        self.rows, self.cols, self.blocks = rows, cols, blocks
        if self.world > 1:
            # CTA b of one rank meets CTA b of every other rank at the flag
            # barriers, so the ranks must launch the same grid over the same
            # bounds; a mismatch would surface only as 2 s barrier timeouts.
            config = (rows, cols, blocks)
            configs = [None] * self.world
            self.dist.all_gather_object(configs, config, group=group)
            if any(tuple(c) != config for c in configs):
                raise ValueError(f"PeerReduce (rows, cols, blocks) differ across ranks: {configs}")
        self.lib = _native.load()
        self._own: list[int] = []
        self._opened: list[int] = []
        nbytes = rows * cols * 2
        with torch.cuda.device(self.device):
            own = [self._alloc(nbytes), self._alloc(nbytes), self._alloc(self.lib.sb_p2p_flag_bytes())]
            handles = [bytes(h.bytes) for _, h in own]
            if self.world > 1:
                gathered = [None] * self.world
                self.dist.all_gather_object(gathered, handles, group=group)
            else:
                gathered = [handles]
            g = _native.SbP2PGroup()
            g.rank, g.world = self.rank, self.world
            for q in range(self.world):
                ptrs = [p for p, _ in own] if q == self.rank else [self._open(h) for h in gathered[q]]
                g.partial[q], g.reduced[q], g.flags[q] = ptrs
            self.group_struct = g
            self._partial = torch.as_tensor(_DeviceArray(own[0][0], (rows, cols), "<i2"),
                                            device=self.device).view(torch.bfloat16)
            self.stream = torch.cuda.Stream(self.device)

    def _alloc(self, nbytes: int):
        ptr = ctypes.c_void_p()
        handle = _native.SbIpcHandle()
        _native.check(self.lib.sb_p2p_buffer_alloc(nbytes, ctypes.byref(ptr), ctypes.byref(handle)))
        self._own.append(ptr.value)
        return ptr.value, handle

    def _open(self, raw: bytes) -> int:
        handle = _native.SbIpcHandle()
        ctypes.memmove(handle.bytes, raw, len(raw))
        ptr = ctypes.c_void_p()
        _native.check(self.lib.sb_p2p_buffer_open(ctypes.byref(handle), ctypes.byref(ptr)))
        self._opened.append(ptr.value)
        return ptr.value

    def partial_rows(self, lo: int, hi: int) -> torch.Tensor:
        """Rows lo:hi of this rank's partial buffer (the GEMM's ``out``).  The view
        aliases library-owned memory and is invalid after :meth:`close`."""
        if not 0 <= lo < hi <= self.rows:
            raise ValueError(f"rows {lo}:{hi} outside the buffer's {self.rows}")
        return self._partial[lo:hi]

    def reduce(self, part: torch.Tensor, residual: torch.Tensor | None = None,
               out: torch.Tensor | None = None, async_op: bool = False):
        """Sum ``part`` (a :meth:`partial_rows` view) over the ranks, plus ``residual``.

        Returns the bf16 result (a new tensor unless ``out`` is given); with
        ``async_op`` returns ``(result, handle)`` and the caller waits the handle
        before using the result.
        """
        if self._partial is None:
            raise RuntimeError("PeerReduce is closed")
        base = self._partial.data_ptr()
        off_bytes = part.data_ptr() - base
        if (part.dtype != torch.bfloat16 or not part.is_contiguous() or part.dim() != 2
                or part.shape[1] != self.cols or off_bytes < 0
                or off_bytes + part.numel() * 2 > self.rows * self.cols * 2):
            raise ValueError("part must be a partial_rows() view of this PeerReduce")
        if residual is not None:
            if tuple(residual.shape) != tuple(part.shape) or not residual.is_contiguous() \
                    or residual.dtype not in (torch.bfloat16, torch.float32) or residual.device != self.device:
                raise ValueError(f"residual must be a contiguous {tuple(part.shape)} bf16/f32 tensor on {self.device}")
        cur = torch.cuda.current_stream(self.device)
        if out is None:
            out = torch.empty_like(part)
        elif (tuple(out.shape) != tuple(part.shape) or out.dtype != torch.bfloat16
              or not out.is_contiguous() or out.device != self.device):
            raise ValueError(f"out must be a contiguous {tuple(part.shape)} bf16 tensor on {self.device}")
        self.stream.wait_stream(cur)
        res_ptr = residual.data_ptr() if residual is not None else None
        res_dt = _native.SB_F32 if residual is not None and residual.dtype == torch.float32 else _native.SB_BF16
        with torch.cuda.device(self.device):
            status = self.lib.sb_p2p_reduce(self.stream.cuda_stream, ctypes.byref(self.group_struct),
                                            off_bytes // 2, part.numel(), res_ptr, res_dt,
                                            out.data_ptr(), self.blocks)
        _native.check(status)
        if residual is not None:
            residual.record_stream(self.stream)
        out.record_stream(self.stream)
        if async_op:
            done = torch.cuda.Event()
            done.record(self.stream)
            return out, _Pending(done)
        cur.wait_stream(self.stream)
        return out

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (all ranks call it)."""
        if self._partial is None:
            return
        self.group_struct = None
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for ptr in self._opened:
                _native.check(self.lib.sb_p2p_buffer_close(ptr))
            if self.world > 1:
                self.dist.barrier(group=self.group)  # nobody maps our buffers any more
            for ptr in self._own:
                _native.check(self.lib.sb_p2p_buffer_free(ptr))
        self._opened, self._own, self._partial = [], [], None


def benchmark(sizes_mib=(32, 128), cols: int = 4096, steps: int = 20, warmup: int = 5) -> list[dict]:
    """Times one ``PeerReduce.reduce`` (with a bf16 residual) against NCCL's
    in-place all-reduce of the same [rows, cols] bf16 partial (without one), per
    size, on the default process group: CUDA events around ``steps`` calls after
    ``warmup`` calls, max over ranks.  Run under torchrun, one rank per GPU:

      python -m torch.distributed.run --nproc-per-node 2 -m strassen_tpu_b200.p2p
    """
    import torch.distributed as dist

    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    results = []
    for mib in sizes_mib:
        rows = mib * (1 << 20) // (cols * 2)
        pr = PeerReduce(rows, cols, dev)
        part = pr.partial_rows(0, rows)
        part.copy_(torch.randn(rows, cols, device=dev).to(torch.bfloat16))
        residual = torch.randn(rows, cols, device=dev).to(torch.bfloat16)
        x = torch.randn(rows, cols, device=dev).to(torch.bfloat16)
        out = torch.empty_like(part)

        def timed(fn):
            for _ in range(warmup):
                fn()
            torch.cuda.synchronize(dev)
            dist.barrier()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(steps):
                fn()
            e.record()
            torch.cuda.synchronize(dev)
            t = torch.tensor([s.elapsed_time(e) / steps], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item()) * 1e3  # microseconds

        p2p_us = timed(lambda: pr.reduce(part, residual, out=out))
        nccl_us = timed(lambda: dist.all_reduce(x))
        status = _native.device_status()
        pr.close()
        results.append({"ranks": world, "mib": mib, "rows": rows, "cols": cols, "p2p_us": p2p_us,
                        "nccl_us": nccl_us, "p2p_bus_gbs": 2 * (world - 1) / world * mib * (1 << 20) / p2p_us / 1e3,
                        "nccl_bus_gbs": 2 * (world - 1) / world * mib * (1 << 20) / nccl_us / 1e3,
                        "device_status": status, "rank": rank})
    return results


if __name__ == "__main__":
    import json
    import os
    from datetime import timedelta

    import torch.distributed as _dist

    _local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(_local)
    _dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", _local))
    try:
        for _r in benchmark():
            if _r["rank"] == 0:
                print(json.dumps(_r), flush=True)
    finally:
        _dist.barrier()
        _dist.destroy_process_group()
