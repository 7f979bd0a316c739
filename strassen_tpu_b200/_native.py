"""ctypes binding of the C ABI in ``include/strassen_b200.h``.

The shared object is built in-tree (``strassen_tpu_b200/libstrassen_b200.so``)
by :mod:`strassen_tpu_b200.build`.  Loading it needs no GPU; calling the GEMM
entry points does.  There is no CPU fallback: if the library is missing, every
operator raises :class:`NativeLibraryError`.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from .build import LIB_PATH

# Every function the header declares, with its ctypes signature.
_c_int = ctypes.c_int32
_c_i64 = ctypes.c_int64
_c_ptr = ctypes.c_void_p
_c_size = ctypes.c_size_t


class SbEpilogue(ctypes.Structure):
    """Mirror of ``struct sb_epilogue``."""

    _fields_ = [
        ("kind", ctypes.c_int32),
        ("residual", ctypes.c_void_p),
        ("ld_residual", ctypes.c_int64),
        ("residual_dtype", ctypes.c_int32),
        ("aux_dtype", ctypes.c_int32),
        ("bias", ctypes.c_void_p),
        ("rope_cos", ctypes.c_void_p),
        ("rope_sin", ctypes.c_void_p),
        ("ld_rope", ctypes.c_int64),
        ("rope_scale", ctypes.c_void_p),
        ("rope_head_dim", ctypes.c_int32),
        ("rope_eps", ctypes.c_float),
        ("norm_scale", ctypes.c_void_p),
        ("norm_eps", ctypes.c_float),
    ]


class SbOptions(ctypes.Structure):
    """Mirror of ``struct sb_options``."""

    _fields_ = [
        ("formula_variant", ctypes.c_int32),
        ("block_permutation", ctypes.c_int32),
        ("panel_schedule", ctypes.c_void_p),
        ("narrow_bn", ctypes.c_int32),
    ]


P2P_MAX_RANKS = 8
P2P_MAX_BLOCKS = 256
P2P_ERROR_CODE = 10


class SbIpcHandle(ctypes.Structure):
    """Mirror of ``struct sb_ipc_handle`` (a cudaIpcMemHandle_t)."""

    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


class SbP2PGroup(ctypes.Structure):
    """Mirror of ``struct sb_p2p_group``."""

    _fields_ = [
        ("rank", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("partial", ctypes.c_void_p * P2P_MAX_RANKS),
        ("reduced", ctypes.c_void_p * P2P_MAX_RANKS),
        ("flags", ctypes.c_void_p * P2P_MAX_RANKS),
    ]


SIGNATURES = {
    "sb_strassen_gemm": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64,
                                  _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_int,
                                  ctypes.POINTER(SbEpilogue), _c_ptr, _c_size]),
    "sb_strassen_gemm_ex": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64,
                                     _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_int,
                                     ctypes.POINTER(SbEpilogue), ctypes.POINTER(SbOptions),
                                     _c_ptr, _c_size]),
    "sb_workspace_bytes": (_c_size, [_c_i64, _c_i64, _c_i64, _c_int]),
    "sb_strassen_gemm_norm_residual_noalloc": (
        _c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                 _c_int, _c_int, _c_int, ctypes.POINTER(SbEpilogue)]),
    "sb_classical_gemm": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64,
                                   _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_int]),
    "sb_strassen_gemm_pair": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64,
                                       _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_int]),
    "sb_b_operands_bytes": (_c_size, [_c_i64, _c_i64]),
    "sb_strassen_b_operands": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_int, _c_int]),
    "sb_strassen_gemm_pair_planes": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64,
                                              _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_int]),
    "sb_quad_workspace_bytes": (_c_size, [_c_i64, _c_i64, _c_i64]),
    "sb_planes_workspace_bytes": (_c_size, [_c_i64, _c_i64, _c_i64]),
    "sb_strassen_gemm_planes": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64,
                                         _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_int,
                                         _c_ptr, _c_size, _c_int, _c_int, _c_ptr]),
    "sb_strassen_gemm_quad": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64,
                                       _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_int,
                                       _c_ptr, _c_size, _c_int]),
    "sb_strassen_gemm_lhs_transposed": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64,
                                                 _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_int,
                                                 _c_int, _c_int]),
    "sb_rms_norm": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_int,
                             ctypes.c_float]),
    "sb_query_tile": (None, [ctypes.POINTER(_c_int)] * 3),
    "sb_status_string": (ctypes.c_char_p, [_c_int]),
    "sb_last_error_message": (ctypes.c_char_p, []),
    "sb_device_status": (_c_int, [ctypes.POINTER(_c_int), _c_int]),
    "sb_wait_selftest": (_c_int, [ctypes.c_void_p]),
    "sb_p2p_buffer_alloc": (_c_int, [_c_size, ctypes.POINTER(_c_ptr), ctypes.POINTER(SbIpcHandle)]),
    "sb_p2p_buffer_open": (_c_int, [ctypes.POINTER(SbIpcHandle), ctypes.POINTER(_c_ptr)]),
    "sb_p2p_buffer_close": (_c_int, [_c_ptr]),
    "sb_p2p_buffer_free": (_c_int, [_c_ptr]),
    "sb_p2p_flag_bytes": (_c_size, []),
    "sb_p2p_reduce": (_c_int, [_c_ptr, ctypes.POINTER(SbP2PGroup), _c_i64, _c_i64, _c_ptr, _c_int,
                               _c_ptr, _c_int]),
    "sb_version": (ctypes.c_char_p, []),
}

# sb_status values (include/strassen_b200.h)
SB_OK = 0
SB_ERR_UNSUPPORTED = 8
SB_ERR_DEVICE_TIMEOUT = 13
SB_ERR_P2P = 14
SB_BF16, SB_F32 = 0, 1
FORMULAS = {"classical": 0, "dual": 1, "powers": 2}
EPILOGUE_KINDS = {
    None: 0,
    "swiglu": 1,
    "geglu": 2,
    "residual_add": 3,
    "bias_add": 4,
    "qk_norm_rope": 5,
    "norm_residual_add": 6,
}


class NativeLibraryError(RuntimeError):
    """The CUDA library is missing or failed to load."""


class StrassenError(ValueError):
    """A non-zero sb_status returned by the library."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


_lock = threading.Lock()
_lib = None


def library_path() -> Path:
    return LIB_PATH


def load(path: Path | None = None) -> ctypes.CDLL:
    """Load (once) and return the library, with every signature bound."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise NativeLibraryError(
                f"{p} is missing; build it with `python -m strassen_tpu_b200.build` "
                "(there is no CPU fallback)")
        try:
            lib = ctypes.CDLL(str(p))
        except OSError as exc:  # pragma: no cover - depends on the host
            raise NativeLibraryError(f"cannot load {p}: {exc}") from exc
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if path is None:
            _lib = lib
        return lib


def check(status: int) -> None:
    """Raise :class:`StrassenError` (or NotImplementedError) for a failing status."""
    if status == SB_OK:
        return
    lib = load()
    message = lib.sb_last_error_message().decode() or lib.sb_status_string(status).decode()
    if status == SB_ERR_UNSUPPORTED:
        raise NotImplementedError(message)
    raise StrassenError(status, message)


def device_status(reset: bool = True) -> int:
    """Synchronise and return the device error word of the bounded waits."""
    lib = load()
    word = _c_int(0)
    status = lib.sb_device_status(ctypes.byref(word), 1 if reset else 0)
    if status not in (SB_OK, SB_ERR_DEVICE_TIMEOUT):
        check(status)
    return int(word.value)


def query_tile() -> tuple[int, int, int]:
    lib = load()
    bm, bn, bk = _c_int(), _c_int(), _c_int()
    lib.sb_query_tile(ctypes.byref(bm), ctypes.byref(bn), ctypes.byref(bk))
    return bm.value, bn.value, bk.value
