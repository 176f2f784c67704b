"""The C-ABI library loads without a GPU and exports every entry point that
include/b200gemm.h declares; host-only logic (status strings, argument
checks that precede any CUDA call, the tile schedule) works on the CPU."""
import ctypes
import re
from pathlib import Path

import pytest

from b200_gemm_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def _declared_symbols():
    names = set()
    for hdr in (ROOT / "include").glob("*.h"):
        text = hdr.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(b200gemm_\w+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared_symbols()
    assert declared, "no declarations found"
    assert declared == set(_lib.SIGNATURES), declared ^ set(_lib.SIGNATURES)
    for name in declared:
        assert hasattr(lib, name), name


def test_strerror_and_version():
    for code in range(7):
        assert _lib.strerror(code)
    assert "unknown" in _lib.strerror(99)
    assert _lib.load().b200gemm_version() >= 10000


def test_null_handle_is_rejected_without_cuda():
    lib = _lib.load()
    assert lib.b200gemm_bf16_nt(None, 1, 1, 8, None, None, None, 8, None) == _lib.ERR_INVALID_ARG
    assert lib.b200gemm_set_timeout_ns(None, 1) == _lib.ERR_INVALID_ARG
    assert lib.b200gemm_last_device_status(None, None) == _lib.ERR_INVALID_ARG
    assert lib.b200gemm_selftest_watchdog(None, 1, None) == _lib.ERR_INVALID_ARG
    assert lib.b200gemm_create(None, 0) == _lib.ERR_INVALID_ARG
    epi = _lib.Epilogue(alpha=1.0)
    assert lib.b200gemm_bf16_nt_epilogue(None, 1, 1, 8, None, None, None, 8, ctypes.byref(epi),
                                         None) == _lib.ERR_INVALID_ARG
    assert ctypes.sizeof(_lib.Epilogue) == 40  # the header's struct layout on LP64
    lib.b200gemm_destroy(None)


def test_create_without_gpu_reports_no_device():
    try:
        import torch

        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    h = ctypes.c_void_p()
    assert _lib.load().b200gemm_create(ctypes.byref(h), 0) == _lib.ERR_NO_DEVICE
    assert not h.value


def test_python_constants_match_header():
    """Every #define the Python side mirrors has the header's value."""
    text = (ROOT / "include" / "b200gemm.h").read_text()
    defines = {m.group(1): int(m.group(2)) for m in re.finditer(r"#define\s+B200GEMM_(\w+)\s+(\d+)", text)}
    mirror = {
        "OK": _lib.OK, "ERR_INVALID_ARG": _lib.ERR_INVALID_ARG, "ERR_UNSUPPORTED": _lib.ERR_UNSUPPORTED,
        "ERR_CUDA": _lib.ERR_CUDA, "ERR_DEVICE_TIMEOUT": _lib.ERR_DEVICE_TIMEOUT,
        "ERR_NO_DEVICE": _lib.ERR_NO_DEVICE, "ERR_TOO_LARGE": _lib.ERR_TOO_LARGE,
        "ORDER_HILBERT": _lib.ORDER_HILBERT, "ORDER_BANDS": _lib.ORDER_BANDS,
        "ACT_NONE": _lib.ACT_NONE, "ACT_RELU": _lib.ACT_RELU, "ACT_GELU": _lib.ACT_GELU,
        "ACT_GELU_TANH": _lib.ACT_GELU_TANH, "ACT_SILU": _lib.ACT_SILU,
        "OUT_BF16": _lib.OUT_BF16, "OUT_F32": _lib.OUT_F32, "OUT_E4M3": _lib.OUT_E4M3,
        "PDL_OFF": _lib.PDL_OFF, "PDL_ON": _lib.PDL_ON, "PDL_WEIGHTS_EARLY": _lib.PDL_WEIGHTS_EARLY,
    }
    for name, value in mirror.items():
        assert defines.get(name) == value, name
    # struct b200gemm_epilogue field order as the ctypes mirror declares it
    body = re.search(r"typedef struct b200gemm_epilogue \{(.*?)\} b200gemm_epilogue;", text, re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    fields = re.findall(r"(\w+);", body)
    assert fields == [f for f, _ in _lib.Epilogue._fields_]


def test_allgather_argument_checks_without_cuda():
    """The fused all-gather entry points reject bad arguments before any CUDA
    call: no multicast address, a misaligned one, N % 8 != 0, and K == 0
    (with K == 0 the other ranks' blocks would never be written)."""
    lib = _lib.load()
    mc_ok, mc_bad = 0x100000, 0x100008
    assert lib.b200gemm_bf16_nt_allgather_multicast(None, 64, 64, 64, None, None, None, 64, None,
                                                    None) == _lib.ERR_INVALID_ARG
    assert lib.b200gemm_bf16_nt_allgather_multicast(None, 64, 64, 64, None, None, None, 64, mc_bad,
                                                    None) == _lib.ERR_UNSUPPORTED
    assert lib.b200gemm_bf16_nt_allgather_multicast(None, 64, 60, 64, None, None, None, 64, mc_ok,
                                                    None) == _lib.ERR_UNSUPPORTED
    assert lib.b200gemm_bf16_nt_allgather_multicast(None, 64, 64, 0, None, None, None, 64, mc_ok,
                                                    None) == _lib.ERR_UNSUPPORTED
    assert lib.b200gemm_bf16_nt_allgather_multicast(None, 64, 64, 64, None, None, None, 64, mc_ok,
                                                    None) == _lib.ERR_INVALID_ARG  # null handle
    assert lib.b200gemm_bf16_nt_allgather(None, 64, 64, 0, None, None, None, 64, None, 0,
                                          None) == _lib.ERR_UNSUPPORTED
    assert lib.b200gemm_bf16_nt_allgather(None, 64, 64, 64, None, None, None, 64, None, 8,
                                          None) == _lib.ERR_INVALID_ARG  # more than 7 peers
