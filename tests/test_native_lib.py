"""The C-ABI library: builds, loads without a GPU, exports every declared symbol,
and rejects bad arguments on the host with reference-mapped status codes."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from strassen_tpu_b200 import _native, build

HEADER = Path(__file__).resolve().parent.parent / "include" / "strassen_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"SB_API\s+[\w\s\*]+?\b(sb_\w+)\s*\(", text)))


def test_library_builds_and_loads():
    path = build.build()
    assert path.exists()
    lib = _native.load()
    assert b"sm_100a" in lib.sb_version()


def test_every_declared_symbol_is_exported_and_bound():
    symbols = declared_symbols()
    assert len(symbols) >= 9
    lib = ctypes.CDLL(str(_native.library_path()))
    for name in symbols:
        assert hasattr(lib, name), name
        assert name in _native.SIGNATURES, f"{name} has no ctypes signature"


def test_query_tile_and_workspace():
    bm, bn, bk = _native.query_tile()
    assert (bm, bn) == (128, 64) and bk in (16, 32, 64)
    lib = _native.load()
    assert lib.sb_workspace_bytes(256, 512, 512, 0) == 0
    assert lib.sb_workspace_bytes(256, 512, 512, 6) == 256 * 512 * 4


def _gemm(lib, m=256, n=256, k=256, bm=256, bn=256, bk=256, out_dtype=0, ep=None, ptr=4096):
    p = ctypes.c_void_p(ptr)
    return lib.sb_strassen_gemm(None, p, p, p, m, n, k, k, n, n, bm, bn, bk, out_dtype,
                                ctypes.byref(ep) if ep is not None else None, None, 0)


@pytest.mark.parametrize("kw, status, text", [
    (dict(m=300), 4, "M=300 is not divisible by 256"),
    (dict(bn=128, n=256), 5, "bn=128 must be a multiple of 256"),
    (dict(out_dtype=7), 7, "output_dtype"),
    (dict(bm=48, m=48 * 4), 8, "bm/2"),
    (dict(ptr=4100), 9, "16-byte aligned"),
])
def test_host_validation_codes(kw, status, text):
    lib = _native.load()
    assert _gemm(lib, **kw) == status
    assert text in lib.sb_last_error_message().decode()


def test_epilogue_validation_codes():
    lib = _native.load()
    ep = _native.SbEpilogue()
    ep.kind = 3  # residual_add without a residual
    assert _gemm(lib, ep=ep) == 6
    ep.kind = 1  # swiglu with fp32 output
    assert _gemm(lib, ep=ep, out_dtype=1) == 7
    ep.kind = 6  # norm_residual_add, bn != n
    ep.residual = 4096
    ep.ld_residual = 512
    ep.norm_scale = 4096
    assert _gemm(lib, n=512, ep=ep) == 6
    assert "must equal n=512" in lib.sb_last_error_message().decode()
    ep.kind = 99
    assert _gemm(lib, ep=ep) == 6


def test_status_strings():
    lib = _native.load()
    for code in range(14):
        assert lib.sb_status_string(code)
    with pytest.raises(_native.StrassenError):
        assert _gemm(lib, m=300) == 4
        _native.check(4)


def test_planes_path_choice_follows_the_cost_model():
    """sb_workspace_bytes asks for the planes workspace only where the planes path
    is expected to beat the one-CTA kernel: large squares and wide K, not the
    small-K row-parallel shards of a tensor-parallel decoder."""
    from strassen_tpu_b200 import _native
    lib = _native.load()
    wants = lambda m, n, k, e=0: lib.sb_workspace_bytes(m, n, k, e) > 0
    assert wants(8192, 8192, 8192) and wants(16384, 16384, 16384)
    assert wants(16384, 24576, 4096, 1)            # Qwen3-8B gate/up + SwiGLU at TP=1
    assert not wants(8192, 4096, 512, 3)           # o projection shard at TP=8 (K = 512)
    assert not wants(2048, 2048, 2048)             # too few tiles
    # norm_residual_add: the planes workspace where the planes path takes it
    # (N <= 8192, one pass over the products), else the one-CTA kernel's fp32 rows.
    assert lib.sb_workspace_bytes(8192, 8192, 8192, 6) == lib.sb_planes_workspace_bytes(8192, 8192, 8192)
    assert lib.sb_workspace_bytes(8192, 16384, 8192, 6) == 8192 * 16384 * 4
    assert lib.sb_workspace_bytes(1024, 1024, 1024, 6) == 1024 * 1024 * 4


def _planes(lib, m=512, n=512, k=256, ws=4096, ws_bytes=None, raster=0, stages=7, ptr=4096):
    p = ctypes.c_void_p(ptr)
    need = lib.sb_planes_workspace_bytes(m, n, k)
    return lib.sb_strassen_gemm_planes(None, p, p, p, m, n, k, k, n, n, 256, 256, 256, 0,
                                       ctypes.c_void_p(ws) if ws else None,
                                       need if ws_bytes is None else ws_bytes, raster, stages, None)


@pytest.mark.parametrize("kw, status, text", [
    (dict(m=256), 5, "M and N divisible by 512"),
    (dict(k=64), 4, "K=64 is not divisible by 256"),
    (dict(ws=0), 10, "sb_planes_workspace_bytes"),
    (dict(ws_bytes=16), 10, "needs a workspace of"),
    (dict(ws=4100), 9, "workspace must be 16-byte aligned"),
    (dict(raster=-1), 8, "raster must be >= 0"),
    (dict(stages=0), 8, "stages must be a nonzero mask"),
    (dict(stages=8), 8, "stages must be a nonzero mask"),
])
def test_planes_entry_validation_codes(kw, status, text):
    """sb_strassen_gemm_planes refuses bad arguments on the host, before any
    device call, with the status and message a caller can act on."""
    lib = _native.load()
    assert _planes(lib, **kw) == status
    assert text in lib.sb_last_error_message().decode()


def test_planes_workspace_bytes_formula():
    """Operand planes (bf16) plus the seven fp32 products, per the header."""
    lib = _native.load()
    for m, n, k in ((512, 512, 128), (8192, 8192, 8192), (16384, 24576, 4096)):
        planes = 7 * (m // 2 * k // 2 + k // 2 * n // 2) * 2
        products = 7 * (m // 2) * (n // 2) * 4
        assert lib.sb_planes_workspace_bytes(m, n, k) == planes + products
