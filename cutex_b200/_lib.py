"""ctypes binding of libcutex_mxfp8.so (the C ABI declared in include/cutex_mxfp8.h).

The library is loaded from ``cutex_b200/_lib`` (built in-tree by
``cutex_b200.build``). There is no fallback: if the library is missing or
fails to load, every GEMM/quantiser call raises. With ``CUTEX_B200_CHECKED=1``
in the environment the checked build (``libcutex_mxfp8_checked.so``, device-side
index checks in every kernel) is loaded instead.
"""

from __future__ import annotations

import ctypes
import os
import threading

from .build import CHECKED_LIB_PATH, LIB_PATH

CHECKED_ENV = "CUTEX_B200_CHECKED"

CUTEX_OK = 0
CUTEX_ERR_INVALID_ARGUMENT = 1
CUTEX_ERR_SHAPE = 2
CUTEX_ERR_ALIGN = 3
CUTEX_ERR_UNSUPPORTED_DEVICE = 4
CUTEX_ERR_CUDA = 5
CUTEX_ERR_TIMEOUT = 6
CUTEX_ERR_WORKSPACE = 7
CUTEX_ERR_DEVICE_CHECK = 8

KERNEL_AUTO = 0
KERNEL_1CTA = 1
KERNEL_2CTA = 2
KERNEL_SKINNY = 3


class GemmConfigC(ctypes.Structure):
    _fields_ = [
        ("kernel", ctypes.c_int32),
        ("tile_n", ctypes.c_int32),
        ("stages", ctypes.c_int32),
        ("raster_group", ctypes.c_int32),
        ("raster_along_n", ctypes.c_int32),
        ("split_k", ctypes.c_int32),
        ("max_ctas", ctypes.c_int32),
        ("epi_buffers", ctypes.c_int32),
        ("sf_buffers", ctypes.c_int32),
        ("scheduler", ctypes.c_int32),
        ("reserved", ctypes.c_int32 * 6),
    ]


class GemmInfoC(ctypes.Structure):
    _fields_ = [
        ("kernel", ctypes.c_int32),
        ("tile_m", ctypes.c_int32),
        ("tile_n", ctypes.c_int32),
        ("tile_k", ctypes.c_int32),
        ("stages", ctypes.c_int32),
        ("cluster_size", ctypes.c_int32),
        ("grid_ctas", ctypes.c_int32),
        ("smem_bytes", ctypes.c_int32),
        ("num_tiles", ctypes.c_int32),
        ("split_k", ctypes.c_int32),
        ("epi_buffers", ctypes.c_int32),
        ("raster_group", ctypes.c_int32),
        ("sf_buffers", ctypes.c_int32),
        ("scheduler", ctypes.c_int32),
        ("workspace_bytes", ctypes.c_int64),
    ]


class EpilogueC(ctypes.Structure):
    """``cutex_epilogue``: D = alpha * acc + beta * C + bias, BF16 or E4M3 (+ scales) out."""

    _fields_ = [
        ("alpha", ctypes.c_float),
        ("beta", ctypes.c_float),
        ("c", ctypes.c_void_p),
        ("ldc", ctypes.c_int64),
        ("bias", ctypes.c_void_p),
        ("out_dtype", ctypes.c_int32),
        ("reserved0", ctypes.c_int32),
        ("d_scales", ctypes.c_void_p),
        ("reserved", ctypes.c_int64 * 4),
    ]


class CutexError(RuntimeError):
    """A non-zero cutex_status returned by the native library."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class CutexArgumentError(CutexError, ValueError):
    """Shape, alignment or configuration rejected by the library (a ValueError, as in the reference)."""


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32

# Exported symbol -> (restype, argtypes). Kept in the same order as include/cutex_mxfp8.h.
SIGNATURES = {
    "cutex_mxfp8_gemm": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.POINTER(GemmConfigC), _vp, _i64, _vp],
    ),
    "cutex_mxfp8_gemm_ex": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.POINTER(GemmConfigC), ctypes.POINTER(EpilogueC),
         _vp, _i64, _vp],
    ),
    "cutex_ipc_export": (ctypes.c_int, [_vp, _vp, ctypes.POINTER(_i64)]),
    "cutex_ipc_import": (ctypes.c_int, [_vp, _i64, ctypes.POINTER(_vp), ctypes.POINTER(_vp)]),
    "cutex_ipc_close": (ctypes.c_int, [_vp]),
    "cutex_mxfp8_selftest_wait_timeout": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp]),
    "cutex_mxfp8_allgather_maps": (ctypes.c_int, [ctypes.POINTER(_vp), _i32, _i64, _i64, _i64, _vp, _i64, _vp]),
    "cutex_mxfp8_gemm_allgather": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i32, ctypes.POINTER(GemmConfigC), _vp],
    ),
    "cutex_mxfp8_query": (
        ctypes.c_int,
        [ctypes.POINTER(GemmConfigC), _i64, _i64, _i64, ctypes.POINTER(GemmInfoC)],
    ),
    "cutex_mxfp8_gemm_trace": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.POINTER(GemmConfigC), _vp, _i32, _vp],
    ),
    "cutex_dense_gemm_v13": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _i32, _vp]),
    "cutex_mxfp8_gemm_skinny_static": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "cutex_mxfp8_gemm_host": (
        ctypes.c_int,
        [_vp] * 10 + [_i64, _i64, _i64, ctypes.POINTER(GemmConfigC), _i32, _vp, _i64, _vp],
    ),
    "cutex_mxfp8_quantize": (ctypes.c_int, [_vp, _i32, _i64, _i64, _i64, _vp, _vp, _vp]),
    "cutex_mxfp8_quantize_columnwise": (ctypes.c_int, [_vp, _i32, _i64, _i64, _i64, _vp, _vp, _vp]),
    "cutex_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "cutex_last_device_status": (ctypes.c_int, [_vp]),
    "cutex_build_checked": (ctypes.c_int, []),
    "cutex_device_check_record": (ctypes.c_int, [_vp, ctypes.POINTER(_i32), ctypes.POINTER(_i64)]),
    "cutex_selftest_device_check": (ctypes.c_int, [_vp]),
    "cutex_device_sm_count": (ctypes.c_int, [ctypes.POINTER(_i32)]),
    "cutex_version": (ctypes.c_char_p, []),
}


def load() -> ctypes.CDLL:
    """Load (once) and return the native library; raise if it is not built."""

    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            checked = os.environ.get(CHECKED_ENV) == "1"
            path = CHECKED_LIB_PATH if checked else LIB_PATH
            if not path.exists():
                raise RuntimeError(
                    f"cutex_b200 native library not found at {path}; build it with "
                    f"`python -m cutex_b200.build{' --checked' if checked else ''}` (there is no CPU fallback)"
                )
            lib = ctypes.CDLL(str(path))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
    return _lib


def status_string(status: int) -> str:
    return load().cutex_status_string(int(status)).decode()


def check(status: int, what: str) -> None:
    if status == CUTEX_OK:
        return
    msg = f"{what}: {status_string(status)}"
    if status in (CUTEX_ERR_INVALID_ARGUMENT, CUTEX_ERR_SHAPE, CUTEX_ERR_ALIGN, CUTEX_ERR_WORKSPACE):
        raise CutexArgumentError(status, msg)
    raise CutexError(status, msg)


def make_config(**fields) -> GemmConfigC:
    cfg = GemmConfigC()
    for name, value in fields.items():
        if name not in {f[0] for f in GemmConfigC._fields_} or name == "reserved":
            raise ValueError(f"unknown GEMM config field {name!r}")
        setattr(cfg, name, int(value))
    return cfg


def version() -> str:
    return load().cutex_version().decode()


def check_record(stream=None) -> tuple[int, int]:
    """(site code, offending value) of the failed device-side check that set the status word, then cleared.

    (0, 0) when none failed; always (0, 0) in a build without checks."""

    site, value = ctypes.c_int32(), ctypes.c_int64()
    check(load().cutex_device_check_record(stream, ctypes.byref(site), ctypes.byref(value)),
          "cutex_device_check_record")
    return site.value, value.value
