"""ctypes binding of libsparseconv_b200.so (the C ABI in include/sparse_conv_b200.h).

The library is loaded from this package directory.  There is no fallback:
if the shared library is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import re
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsparseconv_b200.so")
HEADER_PATH = os.path.join(os.path.dirname(HERE), "include", "sparse_conv_b200.h")

# status codes (sc_status)
SC_OK, SC_EINVAL, SC_EDUP_COORD, SC_ERANGE, SC_ECUDA, SC_ENCCL, SC_ETIMEOUT, SC_ENOMEM, SC_EUNSUPPORTED = range(9)
STATUS_NAMES = {
    SC_OK: "SC_OK", SC_EINVAL: "SC_EINVAL", SC_EDUP_COORD: "SC_EDUP_COORD", SC_ERANGE: "SC_ERANGE",
    SC_ECUDA: "SC_ECUDA", SC_ENCCL: "SC_ENCCL", SC_ETIMEOUT: "SC_ETIMEOUT", SC_ENOMEM: "SC_ENOMEM",
    SC_EUNSUPPORTED: "SC_EUNSUPPORTED",
}
# dtypes
SC_F32, SC_BF16, SC_F16 = 0, 1, 2
# map modes / kinds / flags
SC_MAP_HASH, SC_MAP_SORT = 0, 1
SC_KMAP_SUBM, SC_KMAP_DOWN2, SC_KMAP_UP2 = 0, 1, 2
SC_BUILD_NO_TILE_SORT, SC_BUILD_DEFER_CHECK, SC_BUILD_HALO = 1, 2, 4
SC_EPI_SILU, SC_EPI_RESIDUAL, SC_EPI_LAYERNORM = 1, 2, 4
SC_NOALLOC_MAX_VOXELS = 131072


class SparseConvError(RuntimeError):
    """Raised when a C-ABI call returns a status other than SC_OK."""

    def __init__(self, status, message):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class DuplicateCoordError(SparseConvError):
    pass


class CoordRangeError(SparseConvError):
    pass


class ScConfig(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int32), ("map_mode", ctypes.c_int32),
                ("debug_bounds", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class ScKmapInfo(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("kernel_volume", ctypes.c_int32), ("n_in", ctypes.c_int64),
                ("n_out", ctypes.c_int64), ("num_pairs", ctypes.c_int64), ("num_tiles", ctypes.c_int64),
                ("tile_pairs", ctypes.c_int64),
                ("halo_max", ctypes.c_int64)]


_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_U32 = ctypes.c_uint32
_F = ctypes.c_float
_PP = ctypes.POINTER(ctypes.c_void_p)

_SIGNATURES = {
    "sc_version": (ctypes.c_char_p, []),
    "sc_config_default": (None, [ctypes.POINTER(ScConfig)]),
    "sc_create": (_I32, [_PP, ctypes.POINTER(ScConfig)]),
    "sc_destroy": (_I32, [_P]),
    "sc_set_stream": (_I32, [_P, _P]),
    "sc_set_conv_ctas": (_I32, [_P, _I32]),
    "sc_synchronize": (_I32, [_P]),
    "sc_last_error": (ctypes.c_char_p, [_P]),
    "sc_launch_count": (ctypes.c_uint64, [_P]),
    "sc_kmap_build": (_I32, [_P, _P, _I64, _I32, _I32, _U32, _PP]),
    "sc_kmap_build_ex": (_I32, [_P, _P, _I64, _I64, _I32, _I32, _U32, _PP]),
    "sc_kmap_build_range": (_I32, [_P, _P, _I64, _I64, _I64, _I32, _I32, _U32, _PP]),
    "sc_kmap_build_dilated": (_I32, [_P, _P, _I64, _I64, _I64, _I32, _I32, _I32, _U32, _PP]),
    "sc_kmap_build_down2": (_I32, [_P, _P, _I64, _U32, _PP]),
    "sc_kmap_build_up2": (_I32, [_P, _P, _U32, _PP]),
    "sc_kmap_build_noalloc": (_I32, [_P, _P, _I64, _I32, _P]),
    "sc_kmap_out_coords": (_I32, [_P, _P, _P]),
    "sc_kmap_export": (_I32, [_P, _P, _P]),
    "sc_kmap_concat": (_I32, [_P, _P, _P, _U32, _PP]),
    "sc_kmap_get_info": (_I32, [_P, _P, ctypes.POINTER(ScKmapInfo)]),
    "sc_kmap_check": (_I32, [_P, _P]),
    "sc_kmap_free": (_I32, [_P, _P]),
    "sc_conv3d": (_I32, [_P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _U32, _F]),
    "sc_conv3d_subm": (_I32, [_P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _U32, _F]),
    "sc_conv3d_down2": (_I32, [_P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _U32]),
    "sc_conv3d_up2": (_I32, [_P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _U32]),
    "sc_conv3d_depthwise": (_I32, [_P, _P, _P, _P, _P, _P, _I32, _I32]),
    "sc_subdivide2": (_I32, [_P, _P, _I64, _P, _P, _I32, _P, _P, _P, _I64, _P]),
    "sc_attention_varlen": (_I32, [_P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _F, _I32]),
    "sc_layernorm_silu": (_I32, [_P, _P, _I64, _I32, _I32, _I32, _F]),
    "sc_peer_alloc": (_I32, [_P, ctypes.c_size_t, _PP, _P]),
    "sc_peer_free": (_I32, [_P, _P]),
    "sc_peer_open": (_I32, [_P, _P, _PP]),
    "sc_peer_close": (_I32, [_P, _P]),
    "sc_halo_push": (_I32, [_P, _P, _I32, _P, _P, _P, _I64, _P, _P, _I32, _I32, _U32]),
    "sc_halo_wait": (_I32, [_P, _P, _I32, _I32, _U32]),
    "sc_conv3d_halo": (_I32, [_P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _U32, _F, _P, _I32, _I32, _U32]),
}

SC_IPC_HANDLE_BYTES = 64

_lib = None
_lock = threading.Lock()


def header_symbols(path=HEADER_PATH):
    """Names of every function the public header declares (``SC_API ... sc_x(``)."""
    text = open(path).read()
    return sorted(set(re.findall(r"^SC_API[^;(]*?\b(sc_[a-z0-9_]+)\s*\(", text, flags=re.M)))


def lib():
    """The loaded library (raises OSError when it is missing: no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise OSError(f"{LIB_PATH} is missing; build it with build.py (nvcc, sm_100a)")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(status, handle=None, what=""):
    if status == SC_OK:
        return
    msg = ""
    if handle:
        raw = lib().sc_last_error(handle)
        msg = raw.decode() if raw else ""
    msg = f"{what}: {msg}" if what else msg
    if status == SC_EDUP_COORD:
        raise DuplicateCoordError(status, msg)
    if status == SC_ERANGE:
        raise CoordRangeError(status, msg)
    raise SparseConvError(status, msg)
