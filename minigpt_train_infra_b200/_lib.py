"""ctypes binding of the C ABI declared in ``include/b200_optim.h``.

The shared library is built in-tree (``_build.py``) and loaded from ``lib/``.  There is no
fallback: if the library is missing or fails to load, every entry point raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import numpy as np

from . import _build

ABI_VERSION = 1
MAX_GROUPS = 16
VEC = 8

BF16 = 0
F32 = 1

STATS_FINALIZE = 1
STATS_CLEAR = 2

FLAG_VECTOR = 1

NOALLOC_MAX_CHUNKS = 32768
NOALLOC_MAX_SLOTS = 4096
ERR_TOO_LARGE = -6

# Host mirrors of the C structs (same field order, sizes and alignment as b200_optim.h).
TENSOR_DTYPE = np.dtype([
    ("grad", "<u8"), ("param", "<u8"), ("master", "<u8"), ("exp_avg", "<u8"),
    ("exp_avg_sq", "<u8"), ("numel", "<i8"), ("group", "<i4"), ("slot", "<i4"),
    ("chunk_begin", "<i4"), ("chunk_count", "<i4"), ("flags", "<i4"), ("reserved", "<i4"),
])
CHUNK_DTYPE = np.dtype([("tensor", "<i4"), ("reserved", "<i4"), ("begin", "<i8"), ("end", "<i8")])
GROUP_DTYPE = np.dtype([("lr", "<f8"), ("beta1", "<f8"), ("beta2", "<f8"), ("eps", "<f8"),
                        ("weight_decay", "<f8")])
assert TENSOR_DTYPE.itemsize == 72 and CHUNK_DTYPE.itemsize == 24 and GROUP_DTYPE.itemsize == 40


class B2OError(RuntimeError):
    """A C-ABI entry point returned a non-zero b2o_status."""

    def __init__(self, fn: str, status: int, text: str):
        super().__init__(f"{fn} failed with status {status} ({text})")
        self.status = status


_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F32 = ctypes.c_float
_F64 = ctypes.c_double

# name -> (restype, argtypes); exactly the symbols of include/b200_optim.h.
SIGNATURES = {
    "b2o_abi_version": (ctypes.c_int, []),
    "b2o_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "b2o_plan_chunks": (ctypes.c_int, [_P, _I32, _I32, _I32, _I64, _I32, _P, _I64, _P]),
    "b2o_workspace_bytes": (ctypes.c_size_t, [_I64, _I32]),
    "b2o_workspace_init": (ctypes.c_int, [_P, ctypes.c_size_t, _P]),
    "b2o_grad_stats": (ctypes.c_int, [_P, _I32, _P, _I64, _I32, _I32, _P, _P, _P, _I32, _P, _P,
                                      _P]),
    "b2o_grad_stats_noalloc": (ctypes.c_int, [_P, _I32, _P, _I64, _I32, _I32, _P, _P, _P, _P]),
    "b2o_finalize_norm": (ctypes.c_int, [_P, _I32, _I32, _P, _P, _P]),
    "b2o_adamw_step": (ctypes.c_int, [_P, _I32, _P, _I64, _P, _I32, _I32, _I32, _P, _P, _P, _P,
                                      _F32, _P, _P, _P]),
    "b2o_scaler_update": (ctypes.c_int, [_P, _P, _P, _F64, _F64, _I32, _P]),
    "b2o_adamw_step_dev": (ctypes.c_int, [_P, _I32, _P, _I64, _P, _I32, _I32, _I32, _P, _P, _P,
                                          _P, _F32, _P, _P]),
    "b2o_peer_alloc": (ctypes.c_int, [ctypes.c_size_t, _P]),
    "b2o_peer_free": (ctypes.c_int, [_P]),
    "b2o_peer_export": (ctypes.c_int, [_P, _P]),
    "b2o_peer_import": (ctypes.c_int, [_P, _P]),
    "b2o_peer_close": (ctypes.c_int, [_P]),
    "b2o_reduce_scatter_stats": (ctypes.c_int, [_P, _I32, _P, _F32, _P, _I32, _P, _I64, _I32, _P,
                                                _P, _P, _P]),
    "b2o_adamw_step_bcast": (ctypes.c_int, [_P, _I32, _P, _I64, _P, _I32, _I32, _P, _P, _P, _P,
                                            _F32, _P, _I32, _I32, _P, _P, _P]),
}

IPC_HANDLE_BYTES = 64
MAX_PEERS = 8


def ptr_array(ptrs) -> ctypes.Array:
    """A host array of device pointers for the entry points that take one per rank."""
    return (ctypes.c_void_p * len(ptrs))(*ptrs)

_lock = threading.Lock()
_handle: ctypes.CDLL | None = None


def library_path() -> Path:
    return _build.lib_path()


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load (building first when stale and nvcc is available) the shared library."""
    global _handle
    with _lock:
        if _handle is not None:
            return _handle
        path = library_path()
        if build_if_missing and (not path.exists() or _build.needs_build()):
            try:
                _build.build()
            except RuntimeError:
                if not path.exists():
                    raise
        if not path.exists():
            raise RuntimeError(f"CUDA library not built: {path} (run python -m "
                               "minigpt_train_infra_b200._build)")
        lib = ctypes.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.b2o_abi_version() != ABI_VERSION:
            raise RuntimeError(f"{path} has ABI {lib.b2o_abi_version()}, expected {ABI_VERSION}")
        _handle = lib
        return lib


def check(fn: str, status: int) -> None:
    if status != 0:
        text = load().b2o_status_string(status).decode()
        raise B2OError(fn, status, text)


_FUNCS: dict = {}


def call(fn: str, *args) -> int:
    """Call an entry point returning b2o_status and raise on failure."""
    f = _FUNCS.get(fn)
    if f is None:
        f = _FUNCS[fn] = getattr(load(), fn)
    status = f(*args)
    if status:
        check(fn, status)
    return status


def ptr(a: np.ndarray | None) -> int | None:
    return None if a is None else a.ctypes.data
