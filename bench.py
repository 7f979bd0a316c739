#!/usr/bin/env python3
"""Benchmark of the sm_100a tile-local Strassen GEMM (the north-star hot path).

Workload: BASELINE.json metric "Strassen GEMM effective TFLOP/s (2MNK/t) vs
cuBLAS" at its quoted point M = N = K = 8192 (config 3), bf16 inputs ~N(0,1)
from numpy default_rng(20260902) / (20260903), fp32 accumulation, bf16 output,
the reference's default tile (bm, bn, bk) = (1024, 1024, 512).  A "step" is one
GEMM: by default the planes path a plain ``strassen_matmul`` takes at this size
(operand passes, seven product GEMMs on CTA pairs, recombination; ``--kernel``
picks another kernel).  Inputs are 256 MiB (> 126 MiB L2), so no L2 flush is
needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

N > 1 runs under torchrun, one rank per GPU; every rank computes its own
independent GEMM of the same shape (weak scaling, no collective on the data
path); times are CUDA-event times, max over ranks.  The same run also measures
the tensor-parallel decoder the north star scales (Qwen3-8B
prefill, batch 8 x 2048, TP = N over NCCL) and reports it in a ``decoder``
object with TP=1 measured on rank 0's GPU, so the 1..8-GPU runs carry the
decoder's scaling curve.  ``--impl reference`` times the CPU restatement of the
reference's algorithm (``oracle/``) on the host cores -- the reference itself
is JAX/Pallas-on-TPU and cannot run here.

  python bench.py --profile --steps 3 --warmup 2   # only the timed GEMM launches
                                                  # (the command the ncu captures run)
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

M = N = K = 8192
TILE = (1024, 1024, 512)
SEED_A, SEED_B = 20260902, 20260903
METRIC = "strassen_gemm_effective_tflops"
UNIT = "TFLOP/s"
L2_BYTES = 126 * 1024 * 1024


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-cpu-baseline", action="store_true",
                   help="skip the CPU oracle timing (used for ncu captures)")
    p.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end loop")
    p.add_argument("--kernel", default="planes", choices=["planes", "single", "pair", "pair-planes", "quad"],
                   help="GEMM workload: the seven full-width product GEMMs on CTA pairs (the default path "
                        "of a plain strassen_matmul at this size: operand passes, GEMM, recombination, all "
                        "timed), the one-CTA Strassen kernel, the two-CTA cluster kernel, the two-CTA kernel "
                        "on B operand planes formed inside each step, or the four-CTA paired-tensor-core "
                        "kernel (its operand passes inside each step)")
    p.add_argument("--quad-raster", type=int, default=0,
                   help="--kernel quad: product-row tiles per column sweep (0 = the kernel's default)")
    p.add_argument("--profile", action="store_true",
                   help="time only the GEMM launches (no comparisons, e2e, CPU baseline or decoder); "
                        "the command the committed ncu captures run")
    p.add_argument("--no-decoder", action="store_true", help="skip the decoder measurement of the GEMM run")
    p.add_argument("--epilogue", default="none", choices=["none", "norm_residual_add"],
                   help="GEMM workload with a fused epilogue, tile (1024, N, 512) since the norm spans "
                        "the row: on the planes path (default) one pass over the products normalises; "
                        "with --kernel single the GEMM writes fp32 rows and the row pass normalises "
                        "(the command the row pass's ncu capture runs)")
    p.add_argument("--workload", default="gemm", choices=["gemm", "qwen3-8b", "qwen3-32b"],
                   help="gemm: the 8192^3 Strassen GEMM (default, the driver's line); "
                        "qwen3-*: tensor-parallel decoder prefill tokens/s (BASELINE configs 4/5)")
    p.add_argument("--backend", default="strassen", choices=["strassen", "native"],
                   help="decoder GEMM sites: sm_100a Strassen kernels or the cuBLAS classical arm")
    p.add_argument("--layers", type=int, default=None, help="decoder layers (default: the model's)")
    p.add_argument("--eager", action="store_true",
                   help="decoder: launch op by op instead of replaying a CUDA graph of the forward")
    p.add_argument("--chunks", type=int, default=None,
                   help="decoder: token chunks pipelined so all-reduces overlap compute "
                        "(default: 2 with more than one rank, else 1)")
    p.add_argument("--site-times", type=int, default=0, metavar="TP",
                   help="decoder: time every op of one layer of rank 0's shard at tensor-parallel size TP "
                        "for both backends on one GPU (per-rank shapes of a TP run, no collectives)")
    p.add_argument("--site-policy", default="measured", choices=["measured", "all", "fixed"],
                   help="decoder, strassen backend: each GEMM site on the faster of its Strassen and "
                        "native arms at the shard's shapes (measured before the timed region), every "
                        "site a Strassen tile fits on Strassen, or the sites --native-sites names on the "
                        "native arm (no timing run; used by the committed launch-list capture)")
    p.add_argument("--native-sites", default="",
                   help="with --site-policy fixed: comma-separated GEMM sites (q,k,v,o,up,down) on the native arm")
    p.add_argument("--collective", default="nccl", choices=["nccl", "p2p"],
                   help="decoder: row-parallel sums by NCCL all-reduce (residual fused on rank 0) "
                        "or by sb_p2p_reduce over NVLink peer memory")
    return p.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def normal_bf16_bits(shape, seed: int, rows_per_chunk: int = 1024) -> np.ndarray:
    """Seeded N(0,1) inputs as bf16 bit patterns: numpy ``default_rng(seed)``
    float32 normals rounded to the nearest bf16, ties to even (BASELINE's
    synthetic-input recipe).  Rounded in row chunks to bound host memory."""
    x = np.random.default_rng(seed).standard_normal(shape).astype(np.float32)
    bits = np.empty(shape, dtype=np.uint16)
    for r in range(0, shape[0], rows_per_chunk):
        u = x[r:r + rows_per_chunk].view(np.uint32).astype(np.uint64)
        bits[r:r + rows_per_chunk] = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return bits


def host_inputs():
    """The workload's A and B as uint16 bf16 bit patterns (seeds SEED_A, SEED_B)."""
    return normal_bf16_bits((M, K), SEED_A), normal_bf16_bits((K, N), SEED_B)


# ------------------------------------------------------------- clock sampler
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
        "display_clock_setting": 0x100,
    }

    def __init__(self, index: int, period_s: float = 0.01):
        self.index, self.period = index, period_s
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as exc:  # pragma: no cover - depends on the box
            self.error = repr(exc)

    def _run(self):
        nv = self.nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                for name, bit in self.REASONS.items():
                    if mask & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": len(self.samples)}
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------------------- CPU baseline
def cpu_baseline(a_bits, b_bits, rows: int, cols: int | None = None, repeats: int = 1):
    """Oracle (CPU restatement of the reference) on a bounded sample."""
    from oracle import strassen_ref as ref
    a = ref.from_bf16_bits(a_bits[:rows])
    b = ref.from_bf16_bits(b_bits if cols is None else b_bits[:, :cols])
    n = b.shape[1]
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        ref.strassen_matmul_ref(a, b, bm=TILE[0], bn=min(TILE[1], n), bk=TILE[2])
        times.append(time.perf_counter() - t0)
    t = min(times)
    flops = 2.0 * rows * n * K
    return flops / t / 1e12, t, rows, n


# The CPU sample both CPU legs time: the first Strassen block row (bm = 1024
# rows of A against all of B) of the 8192^3 GEMM -- a block row depends only on
# its own A rows, so this is a self-contained slice of the workload.
CPU_SAMPLE_ROWS = TILE[0]


def cpu_sample_text(threads: int) -> str:
    return (f"first block row ({CPU_SAMPLE_ROWS} x {N} output, K={K}) of the {M}x{N}x{K} GEMM per step, "
            f"tile {TILE}, numpy/BLAS restatement of the reference, {threads} threads")


def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        info = [x for x in threadpool_info() if x.get("user_api") == "blas"]
        if info:
            return int(info[0]["num_threads"])
    except Exception:
        pass
    return os.cpu_count() or 1


# ------------------------------------------------------------- reference arm
def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    a_bits, b_bits = host_inputs()
    rows = CPU_SAMPLE_ROWS
    for _ in range(args.warmup):
        cpu_baseline(a_bits, b_bits, rows)
    vals, ts = [], []
    for _ in range(args.steps):
        v, t, _, _ = cpu_baseline(a_bits, b_bits, rows)
        vals.append(v)
        ts.append(t)
    total_t = sum(ts)
    value = args.steps * 2.0 * rows * N * K / total_t / 1e12
    threads = cpu_threads()
    sample = cpu_sample_text(threads)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total_t / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"strassen_gemm_{M}x{N}x{K}_bf16", "tile": list(TILE),
                   "sample": sample},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ our arm
def run_ours(args):
    import torch
    import torch.distributed as dist

    import strassen_tpu_b200 as sb
    from strassen_tpu_b200 import _native

    rank, world, local = dist_env()
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
        nccl_init_log(rank, world, torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)

    a_bits, b_bits = host_inputs()
    a_host = torch.from_numpy(a_bits.view(np.int16)).view(torch.bfloat16).pin_memory()
    b_host = torch.from_numpy(b_bits.view(np.int16)).view(torch.bfloat16).pin_memory()
    a = a_host.to(device)
    b = b_host.to(device)
    c = torch.empty(M, N, dtype=torch.bfloat16, device=device)
    stream = torch.cuda.current_stream(device)
    flops = 2.0 * M * N * K

    launches_per_step = 1
    tile = TILE
    gemm_events = []  # (start, end) CUDA events around the dominant kernel, when it is one of several
    if args.epilogue != "none" and args.kernel not in ("single", "planes"):
        raise SystemExit("--epilogue runs with --kernel planes (the default) or --kernel single")
    if args.epilogue == "norm_residual_add":
        tile = (TILE[0], N, TILE[2])  # the norm spans the whole row: bn = N
        g = torch.Generator(device=device).manual_seed(SEED_B + 1)
        residual = torch.randn(M, N, device=device, generator=g).to(torch.bfloat16)
        norm_scale = (1.0 + 0.02 * torch.randn(N, device=device, generator=g)).to(torch.bfloat16)
        if args.kernel == "single":
            # The fp32 rows only: the one-CTA kernel's GEMM, then its row pass.
            workspace = torch.empty(M * N * 4, dtype=torch.uint8, device=device)
            launches_per_step = 2
        else:
            # The planes workspace: operand passes, product GEMMs, one pass over
            # the products that recombines, normalises and adds the residual.
            workspace = torch.empty(sb.workspace_bytes(M, N, K, epilogue="norm_residual_add"),
                                    dtype=torch.uint8, device=device)
            launches_per_step = 4

        def step():
            sb.strassen_matmul(a, b, bm=tile[0], bn=tile[1], bk=tile[2], epilogue="norm_residual_add",
                               residual=residual, norm_scale=norm_scale, workspace=workspace, out=c)
    elif args.kernel == "planes":
        ws_planes = torch.empty(sb.workspace_bytes(M, N, K), dtype=torch.uint8, device=device)
        launches_per_step = 7  # B planes, 2 x (A planes, product GEMM, recombination)
        kw_planes = dict(bm=TILE[0], bn=TILE[1], bk=TILE[2], out=c, workspace=ws_planes)

        def step():
            # The whole product in one call (two row halves overlapped on two
            # streams); the call records events around each half's GEMM launch.
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            sb.planes_matmul(a, b, timing_events=ev, **kw_planes)
            gemm_events.append(ev)
    elif args.kernel == "pair-planes":
        planes = torch.empty(7, K // 2, N // 2, dtype=torch.bfloat16, device=device)
        launches_per_step = 2

        def step():
            # B's operand planes are formed inside the timed step (B is an input).
            ops = sb.strassen_b_operands(b, bn=TILE[1], bk=TILE[2], out=planes)
            sb.pair_matmul(a, None, b_operands=ops, bm=TILE[0], bn=TILE[1], bk=TILE[2], out=c)
    elif args.kernel == "quad":
        workspace = torch.empty(_native.load().sb_quad_workspace_bytes(M, N, K), dtype=torch.uint8, device=device)
        launches_per_step = 3  # A operand pass, B operand planes, the four-CTA GEMM

        def step():
            sb.quad_matmul(a, b, bm=TILE[0], bn=TILE[1], bk=TILE[2], out=c, workspace=workspace,
                           raster=args.quad_raster)
    elif args.kernel == "pair":
        def step():
            sb.pair_matmul(a, b, bm=TILE[0], bn=TILE[1], bk=TILE[2], out=c)
    else:
        one_ws = torch.empty(0, dtype=torch.uint8, device=device)  # keeps the product on the one-CTA kernel

        def step():
            sb.strassen_matmul(a, b, bm=TILE[0], bn=TILE[1], bk=TILE[2], out=c, workspace=one_ws)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(fn, steps, warmup):
        for _ in range(warmup):
            fn()
        barrier()
        torch.cuda.synchronize(device)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(steps):
            fn()
        end.record(stream)
        torch.cuda.synchronize(device)
        barrier()
        return max_over_ranks(start.elapsed_time(end))

    # --- the device-resident timed region (value), with clocks sampled during it
    with ClockSampler(device.index) as clocks:
        elapsed_ms = timed(step, args.steps, args.warmup)
    ms = elapsed_ms / args.steps
    # The dominant kernel inside the timed region: on the planes path its two
    # launches per step (each half of the products' rows, on two streams that
    # overlap) timed as one span, from the first half's start to the later end.
    timed_events = gemm_events[-args.steps:]
    kernel_ms = (max_over_ranks(sum(max(ev[0].elapsed_time(ev[1]), ev[0].elapsed_time(ev[3]))
                                    for ev in timed_events) / len(timed_events))
                 if timed_events else ms)
    value = world * flops * args.steps / (elapsed_ms * 1e-3) / 1e12
    dev_err = _native.device_status(reset=True)
    if dev_err:
        raise RuntimeError(f"bounded in-kernel wait timed out (code {dev_err})")

    # --- roofline of the dominant kernel: raw tensor FLOPs (7/8 of 2MNK) per launch
    peaks = {}
    peaks_path = REPO / "MEASURED_PEAKS.json"
    if peaks_path.exists():
        peaks = json.loads(peaks_path.read_text())
    peak = peaks.get("bf16_tflops")
    peak_src = "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    if peak is None:
        peak, peak_src = 1590.0, "fallback 1.59 PFLOP/s"
    raw_flops = flops * 7.0 / 8.0
    achieved = raw_flops / (kernel_ms * 1e-3) / 1e12
    traffic = None
    # Committed DRAM captures exist for the planes GEMM and the one-CTA kernel
    # at the default shape; the other kernels report no traffic figure.
    traffic_file = {"planes": "strassen_planes_8192_traffic.json",
                    "single": "strassen_gemm_8192_traffic.json"}.get(args.kernel)
    traffic_path = REPO / "profiles" / traffic_file if traffic_file else None
    if traffic_path is not None and traffic_path.exists() and args.epilogue == "none":
        traffic = json.loads(traffic_path.read_text()).get("dram_bytes_per_launch")

    # --- comparison arms on identical tensors (informational)
    cublas_ms = control_ms = one_cta_ms = None
    if not args.profile:
        n_cmp = max(10, args.steps // 2)
        cublas_ms = timed(lambda: torch.matmul(a, b, out=c), n_cmp, 3) / n_cmp
        control_ms = timed(lambda: sb.classical_matmul(a, b, bm=TILE[0], bn=TILE[1], bk=TILE[2], out=c),
                           n_cmp, 3) / n_cmp
        no_ws = torch.empty(0, dtype=torch.uint8, device=device)  # keeps the product on the one-CTA kernel
        one_cta_ms = timed(lambda: sb.strassen_matmul(a, b, bm=TILE[0], bn=TILE[1], bk=TILE[2], out=c,
                                                      workspace=no_ws), n_cmp, 3) / n_cmp

    # --- end to end through the reference-facing operator with host buffers:
    # every step copies A and B from pinned host memory, calls strassen_matmul
    # (the drop-in for strassen_pallas.strassen_matmul) and copies C back.
    e2e = e2e_streamed = None
    if not args.no_e2e and not args.profile:
        c_host = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
        a_in = torch.empty_like(a)
        b_in = torch.empty_like(b)

        def e2e_step():
            a_in.copy_(a_host, non_blocking=True)
            b_in.copy_(b_host, non_blocking=True)
            sb.strassen_matmul(a_in, b_in, bm=TILE[0], bn=TILE[1], bk=TILE[2], out=c)
            c_host.copy_(c, non_blocking=True)

        e2e_steps = max(5, args.steps // 5)
        e2e_ms = timed(e2e_step, e2e_steps, 2) / e2e_steps
        e2e = {"value": world * flops / (e2e_ms * 1e-3) / 1e12, "unit": UNIT,
               "h2d_bytes_per_step": 2 * M * K * 2, "d2h_bytes_per_step": M * N * 2,
               "ms_per_step": e2e_ms, "api": "strassen_matmul (sb_strassen_gemm), copies in stream order"}

        def streamed_step():
            # The same copies overlapped with the GEMMs: B, then A in block-row
            # chunks on a copy stream, each chunk's GEMM and copy-back overlapping.
            sb.strassen_matmul_streamed(a_host, b_host, bm=TILE[0], bn=TILE[1], bk=TILE[2], device=device,
                                        out=c_host)

        st_ms = timed(streamed_step, e2e_steps, 2) / e2e_steps
        e2e_streamed = {"value": world * flops / (st_ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": st_ms,
                        "api": "strassen_matmul_streamed (copies overlapped with block-row GEMMs)"}

    # --- CPU baseline (rank 0 at N=1 only): the reference arm's sample
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not args.profile:
        v, t, r, n = cpu_baseline(a_bits, b_bits, CPU_SAMPLE_ROWS, repeats=2)
        threads = cpu_threads()
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": cpu_sample_text(threads) + f", {t:.1f} s"}

    # --- the tensor-parallel decoder at TP = world
    decoder = None
    if not args.no_decoder and not args.profile:
        decoder = decoder_scaling(rank, world, local, device)

    if world > 1:
        barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    clock = clocks.summary()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"strassen_gemm_{M}x{N}x{K}_bf16", "tile": list(tile),
                   "epilogue": args.epilogue,
                   "kernel": {"planes": "seven product GEMMs on CTA pairs (sb_strassen_gemm_planes: operand "
                                        "passes, GEMM, recombination), all timed",
                              "single": "one-CTA (sb_strassen_gemm)",
                              "pair": "two-CTA cluster (sb_strassen_gemm_pair)",
                              "pair-planes": "B operand planes + two-CTA cluster (sb_strassen_b_operands, "
                                             "sb_strassen_gemm_pair_planes), both timed",
                              "quad": "four-CTA paired-tensor-core kernel (sb_strassen_gemm_quad: A operand "
                                      "pass, B operand planes, GEMM), all timed"}[args.kernel],
                   "l2": "inputs 256 MiB > 126 MiB L2, no flush",
                   "inputs": f"N(0,1) bf16, default_rng({SEED_A}) / ({SEED_B})",
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": UNIT,
                     "frac": achieved / peak, "traffic": traffic,
                     "basis": "raw tensor FLOPs 7/8*2MNK per launch / CUDA-event launch time",
                     "kernel": ("strassen_planes_gemm_kernel (the seven product GEMMs; two launches per "
                                "step, one per half of the product rows on two overlapping streams, timed "
                                "with CUDA events as one span)" if gemm_events else
                                "the step's Strassen GEMM launch"),
                     "kernel_ms": kernel_ms,
                     "peak_source": peak_src, "effective_tflops": flops / (ms * 1e-3) / 1e12},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "e2e_streamed": e2e_streamed,
        "clocks": clock,
        "gpu_launches": args.steps * launches_per_step,
        "comparison": None if cublas_ms is None else {
            "cublas_tflops": flops / (cublas_ms * 1e-3) / 1e12,
            "strassen_vs_cublas": (flops / (ms * 1e-3)) / (flops / (cublas_ms * 1e-3)),
            "classical_control_tflops": flops / (control_ms * 1e-3) / 1e12,
            "one_cta_tflops": None if one_cta_ms is None else flops / (one_cta_ms * 1e-3) / 1e12,
        },
        "decoder": decoder,
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------ decoder helpers
def nccl_init_log(rank: int, world: int, device) -> None:
    """One line per rank on stderr once the NCCL process group is up (rank,
    world size, NCCL version, device), so a run's rank count can be read from
    its log; stdout keeps the single JSON line."""
    import torch
    v = torch.cuda.nccl.version()
    ver = ".".join(str(x) for x in v) if isinstance(v, tuple) else str(v)
    print(f"nccl communicator: rank {rank} of {world}, NCCL {ver}, {torch.cuda.get_device_name(device)} "
          f"cuda:{device.index}", file=sys.stderr, flush=True)


def measure_prefill(workload, tp, device, steps, warmup, chunks, backend="strassen", eager=False, layers=None,
                    group=None, site_policy="measured", fixed_native=frozenset()):
    """Qwen3 prefill on `tp`'s ranks: ms per forward (CUDA events, max over the
    group's ranks), tokens/s, FLOP rate, an end-to-end figure with the token
    ids copied in and the logits copied out, and the launch count per step.

    site_policy "measured": each GEMM site takes the faster of its Strassen and
    native arms at this shard's shapes (qwen3.measured_native_sites, timed before
    the model is built, outside the timed region); "all": every site a Strassen
    tile fits runs on Strassen."""
    import torch
    import torch.distributed as dist

    from strassen_tpu_b200 import qwen3

    cfg, (batch, seq) = ({"qwen3-8b": (qwen3.QWEN3_8B, (8, 2048)),
                          "qwen3-32b": (qwen3.QWEN3_32B, (16, 4096))}[workload])
    native_sites = frozenset()
    if backend == "strassen" and site_policy == "measured":
        native_sites = qwen3.measured_native_sites(cfg, tp, batch * seq // max(1, chunks), device, seq=seq)
    elif backend == "strassen" and site_policy == "fixed":
        unknown = set(fixed_native) - set(qwen3.GEMM_SITES)
        if unknown:
            raise ValueError(f"--native-sites names unknown sites {sorted(unknown)}; sites: {qwen3.GEMM_SITES}")
        native_sites = frozenset(fixed_native)
    model = qwen3.Qwen3Prefill(cfg, tp, device, backend=backend, layers=layers, native_sites=native_sites)
    g = torch.Generator().manual_seed(20260911)
    tokens_host = torch.randint(0, cfg.vocab, (batch, seq), generator=g).pin_memory()
    tokens = tokens_host.to(device)
    rope = model.rope(batch, seq)
    stream = torch.cuda.current_stream(device)
    multi = tp.world > 1

    def barrier():
        if multi:
            dist.barrier(group=group, device_ids=[device.index])

    def max_over_ranks(x):
        if not multi:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        return float(t.item())

    def timed(fn, n, w):
        for _ in range(w):
            fn()
        barrier()
        torch.cuda.synchronize(device)
        s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(n):
            fn()
        e0.record(stream)
        torch.cuda.synchronize(device)
        barrier()
        return max_over_ranks(s0.elapsed_time(e0))

    if eager:
        forward = lambda t: model.forward(t, rope, chunks=chunks)  # noqa: E731
        captured = None
    else:
        # One CUDA graph of the whole prefill (kernels, torch ops, NCCL calls).
        captured = qwen3.CapturedPrefill(model, tokens, rope, chunks=chunks)
        forward = captured
    ms = timed(lambda: forward(tokens), steps, warmup) / steps
    logits_host = torch.empty(batch, cfg.vocab, dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        t = tokens_host.to(device, non_blocking=True)
        logits_host.copy_(forward(t), non_blocking=True)

    e2e_n = max(2, steps // 2)
    e2e_ms = timed(e2e_step, e2e_n, 1) / e2e_n
    n_layers = len(model.blocks)
    flops = qwen3.prefill_flops(cfg, batch, seq, n_layers)
    strassen_sites = sorted(k for k, v in model.blocks[0].sites.items() if v.strassen)
    per_chunk = chunks if batch % chunks == 0 else 1
    launches = 0
    if backend == "strassen":
        # two RMSNorm row passes + one GEMM per Strassen site, per block and token chunk
        launches = n_layers * (2 + len(strassen_sites)) * per_chunk
    if tp.peer_reduce:
        launches += n_layers * 2 * per_chunk  # sb_p2p_reduce
    if captured is not None:
        torch.cuda.synchronize(device)
        captured.release()  # a graph holding NCCL calls goes before the process group
    del model, captured, forward
    torch.cuda.empty_cache()
    tok = batch * seq
    return {"ms": ms, "tokens_per_s": tok / (ms * 1e-3), "tflops": flops / (ms * 1e-3) / 1e12,
            "e2e_tokens_per_s": tok / (e2e_ms * 1e-3), "launches": launches, "batch": batch, "seq": seq,
            "layers": n_layers, "strassen_sites": strassen_sites, "vocab": cfg.vocab,
            "site_policy": site_policy if backend == "strassen" else None}


def decoder_scaling(rank, world, local, device, workload="qwen3-8b", steps=3, warmup=1):
    """The decoder the north star scales, inside the GEMM run: Qwen3-8B prefill
    (8 x 2048 tokens, 36 layers, Strassen sites, NCCL) at TP = world, and at
    TP = 1 on rank 0's GPU for the strong-scaling efficiency."""
    import torch.distributed as dist

    from strassen_tpu_b200 import qwen3

    chunks_n = 2 if world > 1 else 1
    solo = dist.new_group([0]) if world > 1 else None  # every rank takes part in creating it
    tp1 = None
    if rank == 0:
        tp = qwen3.TensorParallel(group=solo) if world > 1 else qwen3.TensorParallel()
        tp1 = measure_prefill(workload, tp, device, steps, warmup, chunks=1, group=solo)
    if world > 1:
        dist.barrier(device_ids=[local])
        tpn = measure_prefill(workload, qwen3.TensorParallel(), device, steps, warmup, chunks=chunks_n)
    else:
        tpn = tp1
    if rank != 0:
        return None
    return {
        "metric": f"{workload.replace('-', '_')}_prefill_tokens_per_s", "unit": "tokens/s",
        "tokens_per_s": tpn["tokens_per_s"], "tp": world, "ms_per_step": tpn["ms"],
        "tp1_tokens_per_s": tp1["tokens_per_s"],
        "efficiency": tpn["tokens_per_s"] / (world * tp1["tokens_per_s"]),
        "achieved_tflops": tpn["tflops"], "e2e_tokens_per_s": tpn["e2e_tokens_per_s"],
        "config": {"model": workload, "global_batch": tpn["batch"], "seq_len": tpn["seq"],
                   "layers": tpn["layers"], "parallelism": f"tp{world}", "collective": "nccl",
                   "token_chunks": chunks_n, "cuda_graph": True, "strassen_sites": tpn["strassen_sites"],
                   "site_policy": tpn["site_policy"], "tp1_strassen_sites": tp1["strassen_sites"],
                   "lm_head": "last position per sequence", "steps": steps, "warmup": warmup,
                   "tp1": "rank 0's GPU alone, same box, same run"},
        "gpu_launches_per_step": tpn["launches"],
    }


# --------------------------------------------------------------- decoder arm
def run_decoder(args):
    """Qwen3 prefill at TP = world size: tokens/s (strong scaling), max over ranks."""
    import torch
    import torch.distributed as dist

    from strassen_tpu_b200 import qwen3

    rank, world, local = dist_env()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
        nccl_init_log(rank, world, device)
    tp = qwen3.TensorParallel(collective=args.collective)
    chunks = args.chunks if args.chunks is not None else (2 if world > 1 else 1)
    with ClockSampler(device.index) as clocks:
        r = measure_prefill(args.workload, tp, device, args.steps, args.warmup, chunks, backend=args.backend,
                            eager=args.eager, layers=args.layers, site_policy=args.site_policy,
                            fixed_native=frozenset(s for s in args.native_sites.split(",") if s))
    tp.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank != 0:
        return 0
    tok = r["batch"] * r["seq"]
    line = {
        "metric": f"{args.workload.replace('-', '_')}_prefill_tokens_per_s", "value": r["tokens_per_s"],
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": r["ms"], "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (uniform token ids, random N(0,0.02) weights)",
        "config": {"workload": args.workload, "model": args.workload, "global_batch": r["batch"],
                   "seq_len": r["seq"], "layers": r["layers"], "parallelism": f"tp{world}",
                   "backend": args.backend, "strassen_sites": r["strassen_sites"],
                   "site_policy": r["site_policy"],
                   "token_chunks": chunks, "cuda_graph": not args.eager,
                   "collective": args.collective if world > 1 else None,
                   "lm_head": "last position per sequence"},
        "achieved_tflops": r["tflops"],
        "e2e": {"value": r["e2e_tokens_per_s"], "unit": "tokens/s",
                "h2d_bytes_per_step": tok * 8, "d2h_bytes_per_step": r["batch"] * r["vocab"] * 2},
        "clocks": clocks.summary(),
        "gpu_launches": r["launches"] * args.steps,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_site_times(args):
    """One line: per-op device ms of one decoder layer at TP = --site-times, both backends."""
    import torch

    from strassen_tpu_b200 import qwen3

    cfg, (batch, seq) = ({"qwen3-8b": (qwen3.QWEN3_8B, (8, 2048)),
                          "qwen3-32b": (qwen3.QWEN3_32B, (16, 4096))}[args.workload])
    tp = args.site_times
    chunks = args.chunks if args.chunks is not None else (2 if tp > 1 else 1)
    tokens = batch * seq // chunks
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    times = qwen3.site_times(cfg, tp, tokens, device, steps=args.steps, warmup=args.warmup, seq=seq)
    total = {arm: sum(t[arm] for t in times.values()) for arm in ("strassen", "native")}
    print(json.dumps({"metric": f"{args.workload.replace('-', '_')}_layer_op_ms", "unit": "ms",
                      "tp": tp, "token_rows": tokens, "token_chunks": chunks, "ops": times,
                      "layer_ms": total, "steps": args.steps, "warmup": args.warmup,
                      "note": "rank 0's shard on one GPU; collectives not included"}), flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload != "gemm" and args.site_times:
        return run_site_times(args)
    if args.workload != "gemm":
        return run_decoder(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
