"""Build recipe for the in-tree CUDA library ``libstrassen_b200.so``.

The library is plain C ABI (``include/strassen_b200.h``) compiled by ``nvcc``
for sm_100a only, with the CUDA runtime linked statically so the shared object
loads through ``ctypes`` on any host (the driver is resolved lazily at the first
CUDA call).  No torch headers are involved.

Run ``python -m strassen_tpu_b200.build`` (or ``__graft_entry__.build()``).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_ROOT = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = REPO_ROOT / "include"
LIB_NAME = "libstrassen_b200.so"
LIB_PATH = PACKAGE_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
]


def nvcc_path() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise FileNotFoundError("nvcc not found; set NVCC or put /usr/local/cuda/bin on PATH")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile every ``csrc/*.cu`` into ``libstrassen_b200.so`` (in-tree)."""
    deps = sources() + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    if not force and not _stale(LIB_PATH, deps):
        return LIB_PATH
    build_dir = REPO_ROOT / "_build"
    build_dir.mkdir(exist_ok=True)
    nvcc = nvcc_path()
    objects = []
    for src in sources():
        obj = build_dir / (src.stem + ".o")
        cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, *(extra_flags or []),
               f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objects.append(str(obj))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    link = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-Xcompiler", "-fPIC",
            *objects, "-o", str(tmp)]
    if verbose:
        print(" ".join(link), flush=True)
    subprocess.run(link, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra_flags=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None)
