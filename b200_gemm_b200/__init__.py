"""b200_gemm_b200: bf16 GEMM (C = A . B^T, fp32 accumulate) for B200 / sm_100a.

Python face of the C-ABI in include/b200gemm.h.  The reference project's
interface is the C++ launcher runKernel1(M, N, K, A, B, C, DB)
(b200_kernels/matmul_1.cuh:386) behind run_kernel(kernel_num, ...)
(matmul_b200.cu:28-38); `run_kernel` below keeps that shape for Python
callers, and `Gemm` exposes the handle-based API with streams and status.

torch is used only for device memory and streams; all GEMM work happens in
the hand-written sm_100a kernel of libb200gemm.so.  There is no CPU or
library fallback: without the built library every call raises.
"""
from __future__ import annotations

import ctypes
import threading

from . import _lib
from ._lib import B200GemmError, strerror

__all__ = ["Gemm", "gemm", "run_kernel", "schedule", "B200GemmError", "strerror", "version"]


def version() -> int:
    return _lib.load().b200gemm_version()


_ACTIVATIONS = {"none": _lib.ACT_NONE, "relu": _lib.ACT_RELU, "gelu": _lib.ACT_GELU,
                "gelu_tanh": _lib.ACT_GELU_TANH, "silu": _lib.ACT_SILU}


def _ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


def _stream_ptr(stream) -> int:
    if stream is None:
        import torch

        return int(torch.cuda.current_stream().cuda_stream)
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)


class Gemm:
    """A b200gemm handle bound to one CUDA device."""

    def __init__(self, device: int = 0):
        self._lib = _lib.load()
        self.device = int(device)
        h = ctypes.c_void_p()
        _lib.check(self._lib.b200gemm_create(ctypes.byref(h), self.device), "b200gemm_create")
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            self._lib.b200gemm_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):  # pragma: no cover - interpreter shutdown order varies
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ------------------------------------------------------------------ raw
    def bf16_nt_ptr(self, M: int, N: int, K: int, a_ptr: int, b_ptr: int, c_ptr: int, ldc: int,
                    stream_ptr: int = 0) -> int:
        """Raw pointer call; returns the status code (no exception)."""
        return self._lib.b200gemm_bf16_nt(self._h, M, N, K, a_ptr, b_ptr, c_ptr, ldc, stream_ptr)

    # --------------------------------------------------------------- tensors
    def bf16_nt(self, A, B, out=None, stream=None):
        """out[M, N] = A[M, K] @ B[N, K]^T for bf16 CUDA tensors.

        `out` may be a column slice of a wider row-major matrix (stride(1) == 1);
        its row stride is passed as ldc.
        """
        import torch

        if A.dtype != torch.bfloat16 or B.dtype != torch.bfloat16:
            raise TypeError("A and B must be torch.bfloat16")
        if A.dim() != 2 or B.dim() != 2 or A.shape[1] != B.shape[1]:
            raise ValueError(f"shape mismatch: A {tuple(A.shape)}, B {tuple(B.shape)}")
        if A.stride(1) != 1 or B.stride(1) != 1 or A.stride(0) != A.shape[1] or B.stride(0) != B.shape[1]:
            raise ValueError("A and B must be contiguous row-major (K-major)")
        M, K = A.shape
        N = B.shape[0]
        if out is None:
            # C rows must start on 16-byte boundaries: pad the pitch to a
            # multiple of 8 elements and hand back the [M, N] view.
            pitch = 8 * ((N + 7) // 8)
            out = torch.empty(M, pitch, device=A.device, dtype=torch.bfloat16)[:, :N]
        if out.dtype != torch.bfloat16 or tuple(out.shape) != (M, N) or out.stride(1) != 1:
            raise ValueError("out must be a bf16 [M, N] row-major view")
        ldc = out.stride(0) if M > 1 else 8 * ((N + 7) // 8)
        rc = self.bf16_nt_ptr(M, N, K, _ptr(A), _ptr(B), _ptr(out), ldc, _stream_ptr(stream))
        _lib.check(rc, "b200gemm_bf16_nt")
        return out

    def bf16_nt_epilogue(self, A, B, bias=None, activation: str = "none", residual=None,
                         alpha: float = 1.0, beta: float = 1.0, out=None, out_dtype=None,
                         out_scale: float = 1.0, stream=None):
        """out = act(alpha * A @ B^T + bias) + beta * residual, fused into the
        GEMM's epilogue (fp32 math, one pass over C).

        bias: bf16 [N] CUDA tensor or None; residual: bf16 [M, N] row-major
        view (row stride = ldr) or None; activation: none, relu, gelu,
        gelu_tanh, silu; out_dtype: torch.bfloat16 (default), torch.float32,
        or torch.float8_e4m3fn (stores e4m3(out_scale * D), saturating).
        """
        import torch

        if A.dtype != torch.bfloat16 or B.dtype != torch.bfloat16:
            raise TypeError("A and B must be torch.bfloat16")
        if A.dim() != 2 or B.dim() != 2 or A.shape[1] != B.shape[1]:
            raise ValueError(f"shape mismatch: A {tuple(A.shape)}, B {tuple(B.shape)}")
        if A.stride(1) != 1 or B.stride(1) != 1 or A.stride(0) != A.shape[1] or B.stride(0) != B.shape[1]:
            raise ValueError("A and B must be contiguous row-major (K-major)")
        if activation not in _ACTIVATIONS:
            raise ValueError(f"activation must be one of {sorted(_ACTIVATIONS)}")
        M, K = A.shape
        N = B.shape[0]
        if out_dtype is None:
            out_dtype = out.dtype if out is not None else torch.bfloat16
        kinds = {torch.bfloat16: (_lib.OUT_BF16, 8), torch.float32: (_lib.OUT_F32, 4),
                 torch.float8_e4m3fn: (_lib.OUT_E4M3, 16)}
        if out_dtype not in kinds:
            raise TypeError("out_dtype must be torch.bfloat16, torch.float32 or torch.float8_e4m3fn")
        out_type, group = kinds[out_dtype]  # group: elements per 16 bytes
        if out is None:
            pitch = group * ((N + group - 1) // group)
            out = torch.empty(M, pitch, device=A.device, dtype=out_dtype)[:, :N]
        if out.dtype != out_dtype or tuple(out.shape) != (M, N) or out.stride(1) != 1:
            raise ValueError("out must be an [M, N] row-major view of out_dtype")
        ldc = out.stride(0) if M > 1 else group * ((N + group - 1) // group)
        epi = _lib.Epilogue(alpha=float(alpha), beta=float(beta), activation=_ACTIVATIONS[activation],
                            out_type=out_type, out_scale=float(out_scale))
        if bias is not None:
            if bias.dtype != torch.bfloat16 or tuple(bias.shape) != (N,) or bias.stride(0) != 1:
                raise ValueError("bias must be a contiguous bf16 [N] tensor")
            epi.bias = _ptr(bias)
        if residual is not None:
            if residual.dtype != torch.bfloat16 or tuple(residual.shape) != (M, N) or residual.stride(1) != 1:
                raise ValueError("residual must be a bf16 [M, N] row-major view")
            epi.residual = _ptr(residual)
            epi.ldr = residual.stride(0) if M > 1 else 8 * ((N + 7) // 8)
        rc = self._lib.b200gemm_bf16_nt_epilogue(self._h, M, N, K, _ptr(A), _ptr(B), _ptr(out), ldc,
                                                 ctypes.byref(epi), _stream_ptr(stream))
        _lib.check(rc, "b200gemm_bf16_nt_epilogue")
        return out

    def bf16_nt_host(self, A, B, out=None, stream=None):
        """out[M, N] = A @ B^T with A, B, out in (preferably pinned) host memory.

        Copies and GEMMs are pipelined on the device; completion is ordered on
        `stream` (default: the current CUDA stream), so synchronise it before
        reading `out`."""
        import torch

        if A.dtype != torch.bfloat16 or B.dtype != torch.bfloat16 or A.is_cuda or B.is_cuda:
            raise TypeError("A and B must be host torch.bfloat16 tensors")
        if A.dim() != 2 or B.dim() != 2 or A.shape[1] != B.shape[1]:
            raise ValueError(f"shape mismatch: A {tuple(A.shape)}, B {tuple(B.shape)}")
        A, B = A.contiguous(), B.contiguous()
        M, K = A.shape
        N = B.shape[0]
        if out is None:
            out = torch.empty(M, N, dtype=torch.bfloat16, pin_memory=True)
        if out.is_cuda or out.dtype != torch.bfloat16 or tuple(out.shape) != (M, N) or out.stride(1) != 1:
            raise ValueError("out must be a host bf16 [M, N] row-major view")
        ldc = out.stride(0) if M > 1 else N
        rc = self._lib.b200gemm_bf16_nt_host(self._h, M, N, K, _ptr(A), _ptr(B), _ptr(out), ldc,
                                             _stream_ptr(stream))
        _lib.check(rc, "b200gemm_bf16_nt_host")
        return out

    def plan(self, M: int, N: int, K: int) -> dict:
        """How a call with this shape would run on this handle now.  For the
        tiled kernel, tail_split tells how the tiles of a partial last wave are
        cut: 1 not at all, S >= 2 into S K slices, -2 into two 256-column halves."""
        out = (ctypes.c_int * 6)()
        _lib.check(self._lib.b200gemm_plan(self._h, M, N, K, out), "b200gemm_plan")
        kind = {1: "tiled", 2: "small_m", 3: "small_m_1cta"}.get(out[0], "?")
        return {"kernel": kind, "tile_width": out[1], "tiles": out[2], "clusters": out[3],
                "tail_split": out[4], "small_m_split": out[5]}

    def set_tail_half(self, enable: bool) -> None:
        """Run a short last wave of 256 x 512 (448) tiles as half-width tiles (default on)."""
        _lib.check(self._lib.b200gemm_set_tail_half(self._h, 1 if enable else 0), "b200gemm_set_tail_half")

    def set_tail_split(self, enable: bool) -> None:
        """Split the last partial wave of tiles along K (default off)."""
        _lib.check(self._lib.b200gemm_set_tail_split(self._h, 1 if enable else 0),
                   "b200gemm_set_tail_split")

    def set_tile_width(self, width: int) -> None:
        """0 = choose per call (default), or 512, 448, 256, 224, 192, 128
        output columns per 256-row tile."""
        _lib.check(self._lib.b200gemm_set_tile_width(self._h, int(width)), "b200gemm_set_tile_width")

    def tile_width_for(self, M: int, N: int, K: int) -> int:
        return int(self._lib.b200gemm_tile_width_for(self._h, M, N, K))

    def set_small_m(self, mode: int) -> None:
        """-1/1: use the small-M kernel for eligible shapes (default); 0: never."""
        _lib.check(self._lib.b200gemm_set_small_m(self._h, int(mode)), "b200gemm_set_small_m")

    def set_pdl(self, mode: int) -> None:
        """Launch overlap with the previous kernel on the stream:
        _lib.PDL_OFF (default), PDL_ON (setup overlaps; every global access
        waits for the previous kernel) or PDL_WEIGHTS_EARLY (the small-M
        kernels also start streaming B before that wait, so the previous
        kernel must not write B; the tiled kernel treats it as PDL_ON)."""
        _lib.check(self._lib.b200gemm_set_pdl(self._h, int(mode)), "b200gemm_set_pdl")

    def small_m_split(self, M: int, N: int, K: int) -> int:
        """K split of the small-M kernel for this shape, or 0 if the tiled kernel runs."""
        return int(self._lib.b200gemm_small_m_split(self._h, M, N, K))

    def set_schedule(self, order: int, band: int = 8) -> None:
        """Tile start order: _lib.ORDER_HILBERT or _lib.ORDER_BANDS (band = tile-rows)."""
        _lib.check(self._lib.b200gemm_set_schedule(self._h, int(order), int(band)),
                   "b200gemm_set_schedule")

    def device_info(self) -> dict:
        sm, cl = ctypes.c_int(), ctypes.c_int()
        _lib.check(self._lib.b200gemm_device_info(self._h, ctypes.byref(sm), ctypes.byref(cl)),
                   "b200gemm_device_info")
        return {"sm_count": sm.value, "max_clusters": cl.value}

    def last_device_status(self):
        detail = (ctypes.c_uint * 4)()
        rc = self._lib.b200gemm_last_device_status(self._h, detail)
        return rc, list(detail)

    def set_timeout_ns(self, ns: int) -> None:
        _lib.check(self._lib.b200gemm_set_timeout_ns(self._h, int(ns)), "b200gemm_set_timeout_ns")

    def selftest_watchdog(self, timeout_ns: int, stream=None) -> None:
        rc = self._lib.b200gemm_selftest_watchdog(self._h, int(timeout_ns), _stream_ptr(stream))
        _lib.check(rc, "b200gemm_selftest_watchdog")


_handles: dict[int, Gemm] = {}
_handles_lock = threading.Lock()


def _handle_for(device: int) -> Gemm:
    with _handles_lock:
        h = _handles.get(device)
        if h is None:
            h = _handles[device] = Gemm(device)
        return h


def gemm(A, B, out=None, stream=None):
    """out = A @ B^T (bf16, fp32 accumulate) on A's device."""
    return _handle_for(A.device.index if A.device.index is not None else 0).bf16_nt(A, B, out, stream)


def run_kernel(kernel_num: int, M: int, N: int, K: int, A, B, C) -> None:
    """Mirror of the reference bench's dispatcher (matmul_b200.cu:28-38).

    kernel 0: cuBLASLt through torch (the reference's cuBLAS comparator,
              matmul_b200.cu:13-26, with the operand order fixed for
              non-square shapes);
    kernel 2: this library's sm_100a kernel (the C++ shim `runKernel2`).
    A [M,K], B [N,K], C [M,N]: bf16 CUDA tensors.
    """
    import torch

    if kernel_num == 0:
        torch.matmul(A.view(M, K), B.view(N, K).t(), out=C.view(M, N))
    elif kernel_num == 2:
        rc = _lib.load().b200gemm_run_kernel(M, N, K, _ptr(A), _ptr(B), _ptr(C), None)
        _lib.check(rc, "b200gemm_run_kernel")
    else:
        raise ValueError(f"kernel {kernel_num}: 0 = cuBLASLt, 2 = b200gemm")


def schedule(tiles_m: int, tiles_n: int, order: int = _lib.ORDER_HILBERT, band: int = 8):
    """Host copy of the kernel's tile order (list of (tile_m, tile_n))."""
    n = tiles_m * tiles_n
    buf = (ctypes.c_uint * n)()
    _lib.check(_lib.load().b200gemm_schedule_host(tiles_m, tiles_n, order, band, buf),
               "b200gemm_schedule_host")
    return [(v >> 16, v & 0xFFFF) for v in buf]
