"""GPU test of b200gemm_bf16_nt_noalloc, the entry point for callers that may
not allocate device memory while running a GEMM (allocator internals,
servers with a fixed memory plan, code without a handle).  Its scratch is a
static array inside the library, shared by every call, so the test makes two
calls in a row with different shapes: the second must not see anything the
first left behind.  Each result is compared with the handle-based entry
point b200gemm_bf16_nt on the same operands, within the tolerance the
other tests use (|err| <= 2^-7 (|ref| + 1)).  This file is collected last so
a failure here cannot hide the results of the other tests."""
import numpy as np
import pytest

from b200_gemm_b200 import Gemm, _lib, data

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _dev(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).cuda().view(torch.bfloat16)


def _bits(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def test_noalloc_matches_handle_entry_point_twice(oracle_mod):
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no GPU is visible")
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    with Gemm(0) as handle:
        for M, N, K in [(1024, 1536, 512), (300, 520, 72)]:
            A_bits, B_bits = data.host_operands(M, N, K, "normal", seed=M + N + K)
            A, B = _dev(A_bits), _dev(B_bits)
            ldc = 8 * ((N + 7) // 8)
            C_ref = torch.empty(M, ldc, dtype=torch.bfloat16, device="cuda")
            C = torch.full((M, ldc), float("nan"), dtype=torch.bfloat16, device="cuda")
            assert handle.bf16_nt_ptr(M, N, K, A.data_ptr(), B.data_ptr(), C_ref.data_ptr(), ldc,
                                      stream) == _lib.OK
            rc = lib.b200gemm_bf16_nt_noalloc(M, N, K, A.data_ptr(), B.data_ptr(), C.data_ptr(), ldc,
                                              stream)
            assert rc == _lib.OK, _lib.strerror(rc)
            torch.cuda.synchronize()
            got = oracle_mod.bf16_to_f32(_bits(C)[:, :N])
            ref = oracle_mod.bf16_to_f32(_bits(C_ref)[:, :N]).astype(np.float64)
            assert not np.isnan(got).any()
            assert oracle_mod.within_tolerance(got, ref).all(), oracle_mod.max_scaled_error(got, ref)


def test_noalloc_rejects_problems_beyond_its_table():
    lib = _lib.load()
    buf = torch.zeros(64, dtype=torch.bfloat16, device="cuda")
    p = buf.data_ptr()
    # 200 x 200 tile rows/columns of 256 exceed the 16384-entry static table;
    # the call must refuse before touching the (too small) buffers.
    M = N = 256 * 200
    rc = lib.b200gemm_bf16_nt_noalloc(M, N, 64, p, p, p, N, None)
    assert rc == _lib.ERR_TOO_LARGE
    assert lib.b200gemm_bf16_nt_noalloc(64, 64, 60, p, p, p, 64, None) == _lib.ERR_UNSUPPORTED
    torch.cuda.synchronize()
