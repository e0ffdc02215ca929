"""ctypes binding of ``liblithe_b200.so`` (declarations: ``include/lithe_b200.h``).

The library is loaded from ``lithe_b200/_lib/`` (built in-tree by ``python -m
lithe_b200.build``).  There is no fallback: if the library is missing or does not export
an entry point, every call raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "liblithe_b200.so"

OK = 0
ERR_ARG = -1
ERR_UNSUPPORTED = -2
ERR_CUDA = -3

DEVERR_SLOT = 1
DEVERR_INDEX = 2
DEVERR_TIMEOUT = 4

IDX_PACKED9 = 0
IDX_I16 = 1
IDX_I32 = 2

DTYPE_BF16 = 0
DTYPE_F32 = 1
DTYPE_F16 = 2

MAX_LEVELS = 4
NOALLOC_WS_BYTES = 4 << 20       # LITHE_NOALLOC_WS_BYTES
ABI_VERSION = 1

# Every symbol include/lithe_b200.h declares, with (restype, argtypes).
_c = ctypes
_SIGNATURES = {
    "lithe_abi_version": (_c.c_int32, []),
    "lithe_last_error": (_c.c_char_p, []),
}


class IndexView(ctypes.Structure):
    """``lithe_index_view``: where one side of one module sits in a resident index bank."""

    _fields_ = [
        ("base", ctypes.c_void_p),
        ("format", ctypes.c_int32),
        ("num_levels", ctypes.c_int32),
        ("slot_stride", ctypes.c_int64),
        ("offset", ctypes.c_int64),
        ("level_stride", ctypes.c_int64),
    ]


class PackSegment(ctypes.Structure):
    """lithe_pack_segment: one (module, side) of a raw .lithe payload."""
    _fields_ = [("raw_offset", ctypes.c_int64), ("first_block", ctypes.c_int64), ("n_blocks", ctypes.c_int64)]


_SIGNATURES.update({
    "lithe_sgmv_index": (_c.c_int32, [
        _c.c_void_p, _c.c_void_p, _c.c_int32, _c.POINTER(IndexView), _c.POINTER(IndexView), _c.c_int64,
        _c.c_void_p, _c.c_void_p, _c.c_int32, _c.c_int32, _c.c_int32, _c.c_int32, _c.c_int32,
        _c.POINTER(_c.c_float), _c.c_float, _c.c_void_p, _c.c_void_p]),
    "lithe_sgmv_index_typed": (_c.c_int32, [
        _c.c_void_p, _c.c_void_p, _c.c_int32, _c.POINTER(IndexView), _c.POINTER(IndexView), _c.c_int64,
        _c.c_void_p, _c.c_void_p, _c.c_int32, _c.c_int32, _c.c_int32, _c.c_int32, _c.c_int32,
        _c.POINTER(_c.c_float), _c.c_float, _c.c_int32, _c.c_int32, _c.c_void_p, _c.c_void_p]),
    "lithe_sgmv_workspace_bytes": (_c.c_int64, [_c.c_int32, _c.c_int32, _c.c_int32]),
    "lithe_sgmv_index_ws": (_c.c_int32, [
        _c.c_void_p, _c.c_void_p, _c.c_int32, _c.POINTER(IndexView), _c.POINTER(IndexView), _c.c_int64,
        _c.c_void_p, _c.c_void_p, _c.c_int32, _c.c_int32, _c.c_int32, _c.c_int32, _c.c_int32,
        _c.POINTER(_c.c_float), _c.c_float, _c.c_void_p, _c.c_void_p, _c.c_int64, _c.c_void_p]),
    "lithe_sgmv_index_noalloc": (_c.c_int32, [
        _c.c_void_p, _c.c_void_p, _c.c_int32, _c.POINTER(IndexView), _c.POINTER(IndexView), _c.c_int64,
        _c.c_void_p, _c.c_void_p, _c.c_int32, _c.c_int32, _c.c_int32, _c.c_int32, _c.c_int32,
        _c.POINTER(_c.c_float), _c.c_float, _c.c_void_p, _c.c_void_p]),
    "lithe_lora_prep": (_c.c_int32, [
        _c.c_void_p, _c.POINTER(IndexView), _c.POINTER(IndexView), _c.c_int64, _c.c_void_p, _c.c_void_p, _c.c_int32,
        _c.c_int32, _c.c_int32, _c.c_int32, _c.c_int32, _c.POINTER(_c.c_float), _c.c_float, _c.c_void_p,
        _c.c_void_p, _c.c_void_p, _c.c_void_p]),
    "lithe_lora_prep_ws": (_c.c_int32, [
        _c.c_void_p, _c.POINTER(IndexView), _c.POINTER(IndexView), _c.c_int64, _c.c_void_p, _c.c_void_p, _c.c_int32,
        _c.c_int32, _c.c_int32, _c.c_int32, _c.c_int32, _c.POINTER(_c.c_float), _c.c_float, _c.c_void_p,
        _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_int64, _c.c_void_p]),
    "lithe_lora_prep_workspace_bytes": (_c.c_int64, [_c.c_int32, _c.c_int32, _c.c_int32]),
    "lithe_lora_prep_multi_workspace_bytes": (_c.c_int64, [_c.c_int32, _c.c_int32, _c.c_int32]),
    "lithe_lora_prep_multi": (_c.c_int32, [
        _c.c_void_p, _c.c_int32, _c.POINTER(IndexView), _c.POINTER(IndexView), _c.POINTER(_c.c_int32), _c.c_int64,
        _c.c_void_p, _c.c_void_p, _c.c_int32, _c.c_int32, _c.c_int32, _c.c_int32, _c.POINTER(_c.c_float),
        _c.POINTER(_c.c_float), _c.POINTER(_c.c_void_p), _c.POINTER(_c.c_void_p), _c.c_void_p, _c.c_void_p,
        _c.c_int64, _c.c_void_p]),
    "lithe_lora_gemm": (_c.c_int32, [
        _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_int32, _c.c_int32, _c.c_int32, _c.c_void_p,
        _c.c_void_p, _c.c_int32, _c.c_int32, _c.c_void_p, _c.c_void_p]),
    "lithe_pack_raw": (_c.c_int32, [
        _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_int32, _c.c_int32, _c.c_void_p, _c.c_int64, _c.c_void_p,
        _c.c_void_p]),
    "lithe_pack_raw_batch": (_c.c_int32, [
        _c.c_void_p, _c.c_int64, _c.c_int32, _c.c_int64, _c.c_void_p, _c.c_int32, _c.c_int32, _c.c_void_p,
        _c.c_int64, _c.c_int64, _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_void_p]),
    "lithe_selftest_wait_timeout": (_c.c_int32, [_c.c_void_p, _c.c_void_p, _c.c_void_p]),
    "lithe_decode_packed": (_c.c_int32, [
        _c.c_void_p, _c.c_int64, _c.c_int32, _c.c_void_p, _c.POINTER(_c.c_float), _c.c_void_p,
        _c.c_int32, _c.c_void_p]),
    "lithe_decode_packed_batch": (_c.c_int32, [
        _c.c_void_p, _c.c_int64, _c.c_int64, _c.c_void_p, _c.c_int32, _c.c_int64, _c.c_int32,
        _c.c_void_p, _c.POINTER(_c.c_float), _c.c_void_p, _c.c_int32, _c.c_void_p, _c.c_void_p]),
})

_lock = threading.Lock()
_lib = None


class LitheError(RuntimeError):
    """A CUDA failure reported by liblithe_b200."""


def exported_symbols():
    return tuple(_SIGNATURES)


def lib() -> ctypes.CDLL:
    """The loaded library (loaded once).  Raises if it is not built or is incomplete."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(f"{LIB_PATH} is not built; run `python -m lithe_b200.build` "
                                   "(lithe_b200 has no CPU or PyTorch fallback)")
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (restype, argtypes) in _SIGNATURES.items():
                fn = getattr(handle, name)     # AttributeError if the symbol is missing
                fn.restype = restype
                fn.argtypes = argtypes
            if handle.lithe_abi_version() != ABI_VERSION:
                raise RuntimeError(f"{LIB_PATH} has ABI {handle.lithe_abi_version()}, expected {ABI_VERSION}")
            _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    """Map a non-zero return code to the exception the reference raises for that case."""
    if rc == OK:
        return
    msg = lib().lithe_last_error().decode(errors="replace")
    if rc == ERR_ARG:
        raise ValueError(f"{what}: {msg}")
    if rc == ERR_UNSUPPORTED:
        raise NotImplementedError(f"{what}: {msg}")
    raise LitheError(f"{what}: {msg}")


def float_array(values) -> ctypes.Array:
    vals = [float(v) for v in values]
    return (ctypes.c_float * len(vals))(*vals)
