"""Measured Strassen-vs-cuBLAS dispatch (``tuned_matmul``) and its B200 tile tuner.

The reference dispatches a BF16 GEMM to Strassen only for shapes where it won a
same-run timing against the native GEMM (strassen_pallas.py:1428-1461: squares
from ``TUNED_SQUARE_CROSSOVER`` up, plus an exact-shape allow list, each with the
profile's tile) and screens tiles per GEMM site with interleaved, order-rotated
timings (experiments/qwen3/benchmark_qwen3_site_tile_tune.py:76-110,
benchmark_qwen3_scaling_tile_tune.py:86-133, benchmark_common.py:94-120).

On B200 the same decision is data: a tuning table (JSON) written by
:func:`tune` from CUDA-event timings on the device, read by
:func:`tuned_matmul`.  The table shipped in the package
(``b200_tuning.json``) was measured on a B200; ``STRASSEN_B200_TUNING=<path>``
points the dispatcher at another one (the counterpart of the reference's
``STRASSEN_VMEM_PROFILE`` switch).  A shape dispatches to Strassen only when its
entry says Strassen won, or when it is a square at or above the table's
measured crossover; everything else runs the native GEMM.

Command line (on a GPU)::

    python -m strassen_tpu_b200.tuning --suite default --out table.json
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable, Iterable, Sequence

import torch

from .strassen import TUNED_BK, TUNED_BM, TUNED_BN, native_matmul, strassen_matmul

TABLE_SCHEMA = 1
DEFAULT_TABLE = Path(__file__).with_name("b200_tuning.json")
ENV_TABLE = "STRASSEN_B200_TUNING"

# Screen grid.  On B200 the tile is semantic (it fixes which quadrants are
# summed) while the kernel's own CTA tile is fixed, so the screen mostly sees
# partial-tile waste and cache behaviour; it is kept small on purpose.
BM_CANDIDATES = (512, 1024, 2048)
BN_CANDIDATES = (512, 1024)
BK_CANDIDATES = (512, 2048)
FORMULAS = ("classical",)

SEED = 20260902  # the reference's pure-GEMM seed (benchmark_qwen3_v6e_pure_gemm.py:53)


# --------------------------------------------------------------------------- table

@dataclass(frozen=True)
class ShapeEntry:
    """One measured GEMM shape: which arm won and with which Strassen tile."""

    m: int
    k: int
    n: int
    winner: str                      # "strassen" or "native"
    tile: tuple[int, int, int]       # best Strassen tile (bm, bn, bk)
    formula: str = "classical"
    strassen_ms: float | None = None
    native_ms: float | None = None
    speedup: float | None = None     # native time / Strassen time (paired mean)
    ci95: tuple[float, float] | None = None

    @staticmethod
    def key(m: int, k: int, n: int) -> str:
        return f"{m}x{k}x{n}"


@dataclass
class TuningTable:
    shapes: dict[str, ShapeEntry] = field(default_factory=dict)
    square_crossover: int | None = None   # smallest square size from which Strassen wins
    device: str = ""
    protocol: dict = field(default_factory=dict)

    def lookup(self, m: int, k: int, n: int) -> ShapeEntry | None:
        return self.shapes.get(ShapeEntry.key(m, k, n))

    # ----------------------------------------------------------- (de)serialise
    def to_json(self) -> dict:
        out = {"schema": TABLE_SCHEMA, "device": self.device, "protocol": self.protocol,
               "square_crossover": self.square_crossover, "shapes": {}}
        for key, e in sorted(self.shapes.items()):
            out["shapes"][key] = {
                "m": e.m, "k": e.k, "n": e.n, "winner": e.winner, "tile": list(e.tile),
                "formula": e.formula, "strassen_ms": e.strassen_ms, "native_ms": e.native_ms,
                "speedup": e.speedup, "ci95": list(e.ci95) if e.ci95 else None,
            }
        return out

    @classmethod
    def from_json(cls, data: dict) -> "TuningTable":
        if data.get("schema") != TABLE_SCHEMA:
            raise ValueError(f"tuning table schema {data.get('schema')!r} != {TABLE_SCHEMA}")
        crossover = data.get("square_crossover")
        if crossover is not None and (not isinstance(crossover, int) or crossover <= 0):
            raise ValueError(f"square_crossover must be a positive integer or null, got {crossover!r}")
        shapes = {}
        for key, s in data.get("shapes", {}).items():
            entry = ShapeEntry(
                m=int(s["m"]), k=int(s["k"]), n=int(s["n"]), winner=s["winner"],
                tile=tuple(int(t) for t in s["tile"]), formula=s.get("formula", "classical"),
                strassen_ms=s.get("strassen_ms"), native_ms=s.get("native_ms"),
                speedup=s.get("speedup"),
                ci95=tuple(s["ci95"]) if s.get("ci95") else None)
            if key != ShapeEntry.key(entry.m, entry.k, entry.n):
                raise ValueError(f"tuning table key {key!r} does not match its shape")
            if entry.winner not in ("strassen", "native"):
                raise ValueError(f"winner for {key} must be 'strassen' or 'native'")
            if len(entry.tile) != 3:
                raise ValueError(f"tile for {key} must be (bm, bn, bk)")
            shapes[key] = entry
        return cls(shapes=shapes, square_crossover=crossover, device=data.get("device", ""),
                   protocol=data.get("protocol", {}))

    @classmethod
    def load(cls, path: str | os.PathLike) -> "TuningTable":
        return cls.from_json(json.loads(Path(path).read_text()))

    def save(self, path: str | os.PathLike) -> None:
        Path(path).write_text(json.dumps(self.to_json(), indent=1, sort_keys=True) + "\n")


_cached: tuple[str, float, TuningTable] | None = None


def active_table() -> TuningTable:
    """The table ``tuned_matmul`` reads: ``$STRASSEN_B200_TUNING`` or the shipped one."""
    global _cached
    path = os.environ.get(ENV_TABLE) or str(DEFAULT_TABLE)
    mtime = os.stat(path).st_mtime
    if _cached is None or _cached[0] != path or _cached[1] != mtime:
        _cached = (path, mtime, TuningTable.load(path))
    return _cached[2]


# --------------------------------------------------------------------------- dispatch

@dataclass(frozen=True)
class Dispatch:
    arm: str                                  # "strassen" or "native"
    tile: tuple[int, int, int] | None = None
    formula: str = "classical"
    reason: str = ""


def plan(m: int, k: int, n: int, *, k2: int | None = None, bf16: bool = True,
         on_device: bool = True, table: TuningTable | None = None) -> Dispatch:
    """The dispatch decision for an (m, k) @ (k2, n) GEMM, without running it.

    Mirrors the conditions of strassen_pallas.py:1434-1452: matching inner
    dimensions, BF16 operands, a measured win (exact shape, or a square at or
    above the crossover), a tile that divides the shape, and a device to run on.
    """
    table = active_table() if table is None else table
    k2 = k if k2 is None else k2
    entry = table.lookup(m, k, n)
    if entry is not None and entry.winner == "strassen":
        tile, formula, why = entry.tile, entry.formula, "measured shape"
    elif (m == k == n and table.square_crossover is not None and m >= table.square_crossover):
        tile, formula, why = (TUNED_BM, TUNED_BN, TUNED_BK), "classical", "square crossover"
    else:
        return Dispatch("native", reason="no measured Strassen win for this shape")
    if k != k2:
        return Dispatch("native", reason="inner dimensions disagree")
    if not bf16:
        return Dispatch("native", reason="Strassen runs BF16 operands")
    bm, bn, bk = tile
    if m % bm or n % bn or k % bk:
        return Dispatch("native", reason=f"tile {tile} does not divide the shape")
    if not on_device:
        return Dispatch("native", reason="operands are not on a CUDA device")
    return Dispatch("strassen", tile=tile, formula=formula, reason=why)


def tuned_matmul(a: torch.Tensor, b: torch.Tensor, *, interpret: bool = False,
                 table: TuningTable | None = None) -> torch.Tensor:
    """Dispatch measured BF16 shapes to Strassen, everything else to the native GEMM.

    Same contract as strassen_pallas.tuned_matmul (strassen_pallas.py:1428-1461):
    non-matrix operands and every shape without a measured win go to
    ``native_matmul``.  ``interpret=True`` routes a qualifying shape to
    ``strassen_matmul(interpret=True)`` as the reference does, which on B200
    raises ``NotImplementedError`` (there is no CPU path).
    """
    if a.dim() != 2 or b.dim() != 2:
        return native_matmul(a, b)
    m, k = a.shape
    k2, n = b.shape
    d = plan(m, k, n, k2=k2, bf16=a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16,
             on_device=interpret or (a.is_cuda and b.is_cuda), table=table)
    if d.arm == "native":
        return native_matmul(a, b)
    bm, bn, bk = d.tile
    return strassen_matmul(a, b, bm=bm, bn=bn, bk=bk, formula_variant=d.formula,
                           interpret=interpret)


# --------------------------------------------------------------------------- tuner

def candidate_tiles(m: int, k: int, n: int, bms: Sequence[int] = BM_CANDIDATES,
                    bns: Sequence[int] = BN_CANDIDATES,
                    bks: Sequence[int] = BK_CANDIDATES) -> list[tuple[int, int, int]]:
    """Screen candidates that divide the shape and that the kernel accepts.

    Kernel rules: bm a multiple of 16 with bm/2 a multiple of 128 (or a power of
    two below it), bn and bk multiples of 256 (the reference's alignment rules,
    strassen_pallas.py:162-180).  The reference's VMEM estimate has no B200
    counterpart: the kernel's shared-memory and TMEM footprint does not depend on
    the API tile.
    """
    out = []
    for bm in bms:
        half = bm // 2
        if bm % 16 or not (half % 128 == 0 or (half & (half - 1) == 0 and half < 128)):
            continue
        for bn in bns:
            if bn % 256:
                continue
            for bk in bks:
                if bk % 256:
                    continue
                if m % bm == 0 and n % bn == 0 and k % bk == 0:
                    out.append((bm, bn, bk))
    return out


def rotated_order(names: Sequence[str], run: int) -> list[str]:
    """Arm order for timing run ``run``: rotate by the run index, reverse odd runs.

    The order-bias control of benchmark_common.py:94-120.
    """
    names = list(names)
    offset = run % len(names)
    order = names[offset:] + names[:offset]
    return order[::-1] if run % 2 else order


def summarize(samples_ms: Sequence[float]) -> dict:
    mean = statistics.fmean(samples_ms)
    sd = statistics.stdev(samples_ms) if len(samples_ms) > 1 else 0.0
    half = 1.96 * sd / math.sqrt(len(samples_ms))
    return {"mean_ms": mean, "median_ms": statistics.median(samples_ms), "min_ms": min(samples_ms),
            "ci95_ms": [mean - half, mean + half], "runs": len(samples_ms)}


def paired_speedup(native_ms: Sequence[float], strassen_ms: Sequence[float]) -> tuple[float, tuple]:
    """Mean and 95% CI of the per-run ratio native/Strassen (> 1: Strassen faster)."""
    ratios = [x / y for x, y in zip(native_ms, strassen_ms)]
    s = summarize(ratios)
    return s["mean_ms"], tuple(s["ci95_ms"])


def interleaved_timings(arms: dict[str, Callable[[], object]], *, warmups: int,
                        runs: int) -> dict[str, list[float]]:
    """CUDA-event time of each arm per run, arms interleaved in rotated order."""
    names = list(arms)
    for w in range(warmups):
        for name in rotated_order(names, w):
            arms[name]()
    torch.cuda.synchronize()
    samples = {name: [] for name in names}
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for r in range(runs):
        for name in rotated_order(names, r):
            start.record()
            arms[name]()
            stop.record()
            stop.synchronize()
            samples[name].append(start.elapsed_time(stop))
    return samples


def _inputs(m: int, k: int, n: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator(device=device)
    g.manual_seed(SEED)
    a = torch.randn(m, k, device=device, generator=g).to(torch.bfloat16)
    b = torch.randn(k, n, device=device, generator=g).to(torch.bfloat16)
    return a, b


def tune_shape(m: int, k: int, n: int, *, tiles: Iterable[tuple[int, int, int]] | None = None,
               formulas: Sequence[str] = FORMULAS, screen_warmups: int = 2, screen_runs: int = 5,
               warmups: int = 5, runs: int = 30, device="cuda", log=print) -> ShapeEntry | None:
    """Screen Strassen tiles for one shape, then requalify the best against cuBLAS.

    Screen: every candidate (tile x formula) and the native GEMM, interleaved,
    ``screen_runs`` each (benchmark_qwen3_site_tile_tune.py: one arm per
    candidate, same budget).  Requalify: the screen winner against the native
    GEMM at the full protocol (``warmups`` >= 5, ``runs`` = 30,
    benchmark_qwen3_v6e_pure_gemm.py:56-57); Strassen wins only if the lower end
    of the paired 95% CI of native/Strassen is above 1.
    """
    tiles = list(candidate_tiles(m, k, n) if tiles is None else tiles)
    if not tiles:
        log(f"{m}x{k}x{n}: no candidate tile divides the shape; skipped")
        return None
    a, b = _inputs(m, k, n, device)
    arms = {"native": lambda: native_matmul(a, b)}
    for tile in tiles:
        for f in formulas:
            bm, bn, bk = tile
            arms[f"{f}:{bm},{bn},{bk}"] = (
                lambda bm=bm, bn=bn, bk=bk, f=f: strassen_matmul(a, b, bm=bm, bn=bn, bk=bk,
                                                                 formula_variant=f))
    screen = interleaved_timings(arms, warmups=screen_warmups, runs=screen_runs)
    best = min((n_ for n_ in arms if n_ != "native"), key=lambda n_: statistics.median(screen[n_]))
    formula, tile_s = best.split(":")
    tile = tuple(int(t) for t in tile_s.split(","))
    final = interleaved_timings({"native": arms["native"], best: arms[best]},
                                warmups=warmups, runs=runs)
    speedup, ci = paired_speedup(final["native"], final[best])
    s_ms, n_ms = summarize(final[best])["median_ms"], summarize(final["native"])["median_ms"]
    entry = ShapeEntry(m=m, k=k, n=n, winner="strassen" if ci[0] > 1.0 else "native", tile=tile,
                       formula=formula, strassen_ms=round(s_ms, 4), native_ms=round(n_ms, 4),
                       speedup=round(speedup, 4), ci95=(round(ci[0], 4), round(ci[1], 4)))
    log(f"{m}x{k}x{n}: best Strassen {best} {s_ms:.3f} ms, native {n_ms:.3f} ms, "
        f"native/strassen {speedup:.3f} CI [{ci[0]:.3f}, {ci[1]:.3f}] -> {entry.winner}")
    del a, b
    torch.cuda.empty_cache()
    return entry


def square_crossover(entries: Iterable[ShapeEntry]) -> int | None:
    """Smallest measured square size from which Strassen wins at every larger square."""
    squares = sorted((e for e in entries if e.m == e.k == e.n), key=lambda e: e.m)
    crossover = None
    for e in reversed(squares):
        if e.winner != "strassen":
            break
        crossover = e.m
    return crossover


# Shapes (m, k, n) of the default suite: the reference's square sweep and the
# Qwen3-8B projection shapes at M=4096 tokens (the benchmark sweep), its tuned
# projection shapes (strassen_pallas.py:54-62) and the Qwen3-8B prefill sites at
# 16384 tokens, TP=1 (q, k/v, o, gate/up, down).
SUITES = {
    "default": [
        (2048, 2048, 2048), (4096, 4096, 4096), (8192, 8192, 8192), (16384, 16384, 16384),
        (4096, 4096, 4096), (4096, 4096, 1024), (4096, 4096, 12288), (4096, 12288, 4096),
        (8192, 4096, 8192), (8192, 4096, 12288), (8192, 4096, 28672), (8192, 14336, 4096),
        (16384, 4096, 4096), (16384, 4096, 1024), (16384, 4096, 24576), (16384, 12288, 4096),
    ],
    "quick": [(2048, 2048, 2048), (8192, 8192, 8192)],
}


def tune(shapes: Iterable[tuple[int, int, int]], *, runs: int = 30, warmups: int = 5,
         log=print, **kw) -> TuningTable:
    if not torch.cuda.is_available():
        raise RuntimeError("tuning measures on a CUDA device; none is visible")
    entries = [e for e in (tune_shape(m, k, n, runs=runs, warmups=warmups, log=log, **kw)
                           for m, k, n in shapes) if e is not None]
    props = torch.cuda.get_device_properties(0)
    return TuningTable(
        shapes={ShapeEntry.key(e.m, e.k, e.n): e for e in entries},
        square_crossover=square_crossover(entries),
        device=f"{props.name} (sm_{props.major}{props.minor}, {props.multi_processor_count} SMs)",
        protocol={"timer": "CUDA events per call, arms interleaved in rotated/reversed order",
                  "screen": "2 warm-ups + 5 runs per candidate", "requalify":
                  f"{warmups} warm-ups + {runs} runs, winner iff paired 95% CI of native/strassen > 1",
                  "inputs": f"N(0,1) bf16, torch.Generator seed {SEED}", "l2": "not flushed"})


def main(argv: Sequence[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--suite", choices=sorted(SUITES), default="default")
    ap.add_argument("--shape", action="append", default=[], help="extra MxKxN shape")
    ap.add_argument("--runs", type=int, default=30)
    ap.add_argument("--warmups", type=int, default=5)
    ap.add_argument("--out", required=True)
    args = ap.parse_args(argv)
    shapes = list(dict.fromkeys(list(SUITES[args.suite]) +
                                [tuple(int(x) for x in s.split("x")) for s in args.shape]))
    table = tune(shapes, runs=args.runs, warmups=args.warmups)
    table.save(args.out)
    print(f"wrote {args.out}: {len(table.shapes)} shapes, square crossover {table.square_crossover}")


if __name__ == "__main__":
    main()
