"""ctypes wrapper of oracle/gemm_oracle.c.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, as the checker or the timed CPU baseline.  The
product path (b200_gemm_b200) never imports it.

Arithmetic restated: C[i][j] = bf16_rne(sum_k A[i][k] * B[j][k]) with A
[M,K] and B [N,K] row-major bf16 (reference b200_kernels/matmul_1.cuh:
329-381; rounding :293-295; input conversion include/utils.cuh:24-29).
Parity is pinned by known-answer tests (exact integer products), by golden
outputs of the reference kernel itself (tests/golden/, made by
tests/golden/make_golden.py from oracle/_ref) and by cuBLASLt on the GPU.
"""
from __future__ import annotations

import ctypes
import subprocess
import threading
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
REF_LIB_PATH = HERE / "_ref" / "libref_gemm.so"

TOL_REL = 2.0 ** -7  # |err| <= 2^-7 * (|ref| + 1)

_lock = threading.Lock()
_lib = None

_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")


def build() -> Path:
    """Compile liboracle.so with the committed Makefile (gcc)."""
    src = HERE / "gemm_oracle.c"
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)
    return LIB_PATH


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(str(LIB_PATH))
            c_int, c_size = ctypes.c_int, ctypes.c_size_t
            L.oracle_f32_to_bf16.argtypes = [_f32p, _u16p, c_size]
            L.oracle_bf16_to_f32.argtypes = [_u16p, _f32p, c_size]
            L.oracle_f64_to_bf16.argtypes = [_f64p, _u16p, c_size]
            L.oracle_gemm_bf16_nt_f64.argtypes = [c_int, c_int, c_int, _u16p, c_int, _u16p, c_int,
                                                  _f64p, c_int, c_int, c_int, c_int]
            L.oracle_gemm_bf16_nt_f64.restype = c_int
            L.oracle_gemm_bf16_nt_f64_sampled.argtypes = [c_int, _u16p, c_int, _u16p, c_int, _i32p,
                                                          _i32p, c_size, _f64p]
            L.oracle_gemm_bf16_nt_f32.argtypes = [c_int, c_int, c_int, _u16p, _u16p, _u16p, c_int,
                                                  c_int, c_int, c_int]
            L.oracle_gemm_bf16_nt_f32.restype = c_int
            L.oracle_num_cpus.restype = c_int
            vp, c_double = ctypes.c_void_p, ctypes.c_double
            L.oracle_epilogue_f64.argtypes = [_f64p, c_int, c_int, c_int, c_double, vp, c_int, vp,
                                              c_int, c_double]
            L.oracle_epilogue_sampled.argtypes = [_f64p, _i32p, _i32p, c_size, c_double, vp, c_int,
                                                  vp, c_int, c_double]
            _u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
            L.oracle_f64_to_e4m3.argtypes = [_f64p, _u8p, c_size]
            L.oracle_e4m3_to_f64.argtypes = [_u8p, _f64p, c_size]
            _lib = L
        return _lib


def f32_to_bf16(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().oracle_f32_to_bf16(x.reshape(-1), out.reshape(-1), x.size)
    return out


def bf16_to_f32(h) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().oracle_bf16_to_f32(h.reshape(-1), out.reshape(-1), h.size)
    return out


def f64_to_bf16(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float64)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().oracle_f64_to_bf16(x.reshape(-1), out.reshape(-1), x.size)
    return out


def gemm_f64(A, B, row_begin: int = 0, row_end: int | None = None, threads: int = 0) -> np.ndarray:
    """fp64 sums of A[rows] . B^T for bf16 bit arrays A [M,K], B [N,K]."""
    A = np.ascontiguousarray(A, dtype=np.uint16)
    B = np.ascontiguousarray(B, dtype=np.uint16)
    M, K = A.shape
    N = B.shape[0]
    assert B.shape[1] == K
    row_end = M if row_end is None else row_end
    C = np.zeros((M, N), dtype=np.float64)
    rc = lib().oracle_gemm_bf16_nt_f64(M, N, K, A, max(K, 1), B, max(K, 1), C, max(N, 1),
                                       row_begin, row_end, threads)
    if rc != 0:
        raise ValueError("oracle_gemm_bf16_nt_f64: bad arguments")
    return C[row_begin:row_end]


def gemm_bf16(A, B, threads: int = 0) -> np.ndarray:
    """Reference output bits: bf16_rne(fp32(fp64 sum))."""
    return f64_to_bf16(gemm_f64(A, B, threads=threads))


def gemm_sampled(A, B, rows, cols) -> np.ndarray:
    A = np.ascontiguousarray(A, dtype=np.uint16)
    B = np.ascontiguousarray(B, dtype=np.uint16)
    rows = np.ascontiguousarray(rows, dtype=np.int32)
    cols = np.ascontiguousarray(cols, dtype=np.int32)
    out = np.empty(rows.shape[0], dtype=np.float64)
    K = A.shape[1]
    lib().oracle_gemm_bf16_nt_f64_sampled(K, A, K, B, K, rows, cols, rows.shape[0], out)
    return out


def gemm_f32_cpu(A, B, row_begin: int = 0, row_end: int | None = None, threads: int = 0):
    """Multithreaded fp32 CPU GEMM (the CPU baseline).  Returns (C_bits rows, threads)."""
    A = np.ascontiguousarray(A, dtype=np.uint16)
    B = np.ascontiguousarray(B, dtype=np.uint16)
    M, K = A.shape
    N = B.shape[0]
    row_end = M if row_end is None else row_end
    C = np.zeros((M, N), dtype=np.uint16)
    used = lib().oracle_gemm_bf16_nt_f32(M, N, K, A, B, C, max(N, 1), row_begin, row_end, threads)
    if used < 0:
        raise ValueError("oracle_gemm_bf16_nt_f32: bad arguments or out of memory")
    return C[row_begin:row_end], used


ACTIVATIONS = {"none": 0, "relu": 1, "gelu": 2, "gelu_tanh": 3, "silu": 4}


def _opt_bits(x):
    """(keep-alive array, pointer) for an optional bf16 bit array."""
    if x is None:
        return None, None
    arr = np.ascontiguousarray(x, dtype=np.uint16)
    return arr, arr.ctypes.data


def epilogue_f64(S, alpha=1.0, bias=None, act="none", residual=None, beta=1.0) -> np.ndarray:
    """D = act(alpha S + bias[j]) + beta R[i][j] on fp64 sums S [M, N] (a copy;
    bias: bf16 bits [N], residual: bf16 bits [M, N] or None)."""
    D = np.array(S, dtype=np.float64, order="C", copy=True)
    M, N = D.shape
    b, bp = _opt_bits(bias)
    r, rp = _opt_bits(residual)
    if b is not None:
        assert b.shape == (N,)
    if r is not None:
        assert r.shape == (M, N)
    lib().oracle_epilogue_f64(D, M, N, max(N, 1), float(alpha), bp, ACTIVATIONS[act], rp, max(N, 1),
                              float(beta))
    return D


def epilogue_sampled(vals, rows, cols, alpha=1.0, bias=None, act="none", residual=None,
                     beta=1.0) -> np.ndarray:
    """The same on sampled sums vals[s] of elements (rows[s], cols[s])."""
    out = np.array(vals, dtype=np.float64, copy=True)
    rows = np.ascontiguousarray(rows, dtype=np.int32)
    cols = np.ascontiguousarray(cols, dtype=np.int32)
    b, bp = _opt_bits(bias)
    r, rp = _opt_bits(residual)
    ldr = r.shape[1] if r is not None else 1
    lib().oracle_epilogue_sampled(out, rows, cols, out.shape[0], float(alpha), bp, ACTIVATIONS[act],
                                  rp, ldr, float(beta))
    return out


def f64_to_e4m3(x) -> np.ndarray:
    """fp64 -> OCP FP8 E4M3 bytes (RNE, saturating to +-448)."""
    x = np.ascontiguousarray(x, dtype=np.float64)
    out = np.empty(x.shape, dtype=np.uint8)
    lib().oracle_f64_to_e4m3(x.reshape(-1), out.reshape(-1), x.size)
    return out


def e4m3_to_f64(b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint8)
    out = np.empty(b.shape, dtype=np.float64)
    lib().oracle_e4m3_to_f64(b.reshape(-1), out.reshape(-1), b.size)
    return out


def e4m3_ulp(x) -> np.ndarray:
    """Spacing of e4m3 values around |x| (2^-9 in the subnormal range)."""
    a = np.abs(np.asarray(x, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -6)))
    return np.ldexp(1.0, (np.minimum(e, 8) - 3).astype(np.int64))


def num_cpus() -> int:
    return int(lib().oracle_num_cpus())


def within_tolerance(got_f32, ref_f64) -> np.ndarray:
    """Elementwise |got - ref| <= 2^-7 (|ref| + 1)."""
    got = np.asarray(got_f32, dtype=np.float64)
    ref = np.asarray(ref_f64, dtype=np.float64)
    return np.abs(got - ref) <= TOL_REL * (np.abs(ref) + 1.0)


def max_scaled_error(got_f32, ref_f64) -> float:
    got = np.asarray(got_f32, dtype=np.float64)
    ref = np.asarray(ref_f64, dtype=np.float64)
    if got.size == 0:
        return 0.0
    return float(np.max(np.abs(got - ref) / (np.abs(ref) + 1.0)))
