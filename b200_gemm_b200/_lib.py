"""ctypes binding of the C-ABI declared in include/b200gemm.h.

The shared library is built in-tree (b200_gemm_b200/lib/libb200gemm.so) by
b200_gemm_b200/build.py.  There is no fallback: if the library is missing or
does not load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libb200gemm.so"

OK = 0
ERR_INVALID_ARG = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_DEVICE_TIMEOUT = 4
ERR_NO_DEVICE = 5
ERR_TOO_LARGE = 6

ORDER_HILBERT = 0
ORDER_BANDS = 1

ACT_NONE, ACT_RELU, ACT_GELU, ACT_GELU_TANH, ACT_SILU = 0, 1, 2, 3, 4
OUT_BF16, OUT_F32, OUT_E4M3 = 0, 1, 2
PDL_OFF, PDL_ON, PDL_WEIGHTS_EARLY = 0, 1, 2

_c_int, _c_uint, _c_ull, _vp = ctypes.c_int, ctypes.c_uint, ctypes.c_ulonglong, ctypes.c_void_p


class Epilogue(ctypes.Structure):
    """struct b200gemm_epilogue (include/b200gemm.h)."""
    _fields_ = [
        ("alpha", ctypes.c_float),
        ("beta", ctypes.c_float),
        ("bias", _vp),
        ("residual", _vp),
        ("ldr", _c_int),
        ("activation", _c_int),
        ("out_type", _c_int),
        ("out_scale", ctypes.c_float),
    ]


# name -> (restype, argtypes); one line per declaration in include/b200gemm.h
SIGNATURES = {
    "b200gemm_create": (_c_int, [ctypes.POINTER(_vp), _c_int]),
    "b200gemm_destroy": (None, [_vp]),
    "b200gemm_bf16_nt": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _vp, _vp, _c_int, _vp]),
    "b200gemm_bf16_nt_host": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _vp, _vp, _c_int, _vp]),
    "b200gemm_bf16_nt_epilogue": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _vp, _vp, _c_int,
                                           ctypes.POINTER(Epilogue), _vp]),
    "b200gemm_bf16_nt_allgather": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _vp, _vp, _c_int,
                                            ctypes.POINTER(_vp), _c_int, _vp]),
    "b200gemm_bf16_nt_allgather_multicast": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _vp, _vp, _c_int,
                                                      _vp, _vp]),
    "b200gemm_ipc_get_handle": (_c_int, [_vp, _vp, ctypes.POINTER(_c_ull)]),
    "b200gemm_ipc_open": (_c_int, [_vp, ctypes.POINTER(_vp)]),
    "b200gemm_ipc_close": (_c_int, [_vp]),
    "b200gemm_last_device_status": (_c_int, [_vp, ctypes.POINTER(_c_uint)]),
    "b200gemm_set_timeout_ns": (_c_int, [_vp, _c_ull]),
    "b200gemm_selftest_watchdog": (_c_int, [_vp, _c_ull, _vp]),
    "b200gemm_run_kernel": (_c_int, [_c_int, _c_int, _c_int, _vp, _vp, _vp, ctypes.POINTER(_c_int)]),
    "b200gemm_device_info": (_c_int, [_vp, ctypes.POINTER(_c_int), ctypes.POINTER(_c_int)]),
    "b200gemm_plan": (_c_int, [_vp, _c_int, _c_int, _c_int, ctypes.POINTER(_c_int)]),
    "b200gemm_set_tail_split": (_c_int, [_vp, _c_int]),
    "b200gemm_set_tile_width": (_c_int, [_vp, _c_int]),
    "b200gemm_tile_width_for": (_c_int, [_vp, _c_int, _c_int, _c_int]),
    "b200gemm_set_small_m": (_c_int, [_vp, _c_int]),
    "b200gemm_set_pdl": (_c_int, [_vp, _c_int]),
    "b200gemm_set_tail_half": (_c_int, [_vp, _c_int]),
    "b200gemm_small_m_split": (_c_int, [_vp, _c_int, _c_int, _c_int]),
    "b200gemm_set_schedule": (_c_int, [_vp, _c_int, _c_int]),
    "b200gemm_schedule_host": (_c_int, [_c_uint, _c_uint, _c_int, _c_int, ctypes.POINTER(_c_uint)]),
    "b200gemm_bf16_nt_noalloc": (_c_int, [_c_int, _c_int, _c_int, _vp, _vp, _vp, _c_int, _vp]),
    "b200gemm_strerror": (ctypes.c_char_p, [_c_int]),
    "b200gemm_version": (_c_int, []),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class B200GemmError(RuntimeError):
    """A b200gemm entry point returned a non-zero status."""

    def __init__(self, code: int, where: str):
        self.code = code
        super().__init__(f"{where}: {strerror(code)} (status {code})")


def load() -> ctypes.CDLL:
    """Load the library (once).  Raises if it is missing: there is no fallback."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing; build it with `python -m b200_gemm_b200.build`")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
        return _lib


def strerror(code: int) -> str:
    return load().b200gemm_strerror(int(code)).decode()


def check(code: int, where: str) -> None:
    if code != OK:
        raise B200GemmError(code, where)
