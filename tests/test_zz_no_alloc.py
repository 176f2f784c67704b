"""GPU test of b200gemm_bf16_nt_noalloc, the entry point for callers that may
not allocate device memory while running a GEMM (allocator internals,
servers with a fixed memory plan, code without a handle).  Its scratch is a
static array inside the library, shared by every call, so the tests make
calls in a row with different shapes: a later call must not see anything an
earlier one left behind.  Each result is compared with the fp64 CPU oracle
(every element for small shapes, sampled elements plus a full row and column
for large ones) and with the handle-based entry point b200gemm_bf16_nt on the
same operands, within the tolerance the other tests use
(|err| <= 2^-7 (|ref| + 1)).  The device's free memory must not change
across a call.  This file is collected last so a failure here cannot hide
the results of the other tests."""
import numpy as np
import pytest

from b200_gemm_b200 import Gemm, _lib, data

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _dev(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).cuda().view(torch.bfloat16)


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _noalloc(lib, M, N, K, A, B, C, ldc, stream):
    rc = lib.b200gemm_bf16_nt_noalloc(M, N, K, A.data_ptr(), B.data_ptr(), C.data_ptr(), ldc, stream)
    assert rc == _lib.OK, _lib.strerror(rc)


def test_noalloc_matches_oracle_and_handle_entry_point_twice(oracle_mod):
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
            _noalloc(lib, M, N, K, A, B, C, ldc, stream)
            torch.cuda.synchronize()
            got = oracle_mod.bf16_to_f32(_bits(C)[:, :N])
            assert not np.isnan(got).any()
            exact = oracle_mod.gemm_f64(A_bits, B_bits)
            assert oracle_mod.within_tolerance(got, exact).all(), oracle_mod.max_scaled_error(got, exact)
            ref = oracle_mod.bf16_to_f32(_bits(C_ref)[:, :N]).astype(np.float64)
            assert oracle_mod.within_tolerance(got, ref).all(), oracle_mod.max_scaled_error(got, ref)


def test_noalloc_many_waves_long_k_and_no_allocation(oracle_mod):
    """4096^3 (256 tiles: several waves of the persistent grid through the
    static schedule table) and 512 x 4096 x 16384 (two tile rows, K = 16384),
    one after the other, each against sampled fp64 oracle elements and the
    handle entry point; after a warm-up call of each shape the device's free
    memory is the same before and after a call."""
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    cases = [(4096, 4096, 4096), (512, 4096, 16384)]
    bufs = []
    for M, N, K in cases:
        A, B = data.device_operands(M, N, K, "normal", seed=M + 3 * K)
        C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        bufs.append((A, B, C))
    # Warm-up: both shapes once, so any lazy loading has happened.
    for (M, N, K), (A, B, C) in zip(cases, bufs):
        _noalloc(lib, M, N, K, A, B, C, N, stream)
    torch.cuda.synchronize()
    with Gemm(0) as handle:
        for (M, N, K), (A, B, C) in zip(cases, bufs):
            C.fill_(float("nan"))
            torch.cuda.synchronize()
            free0 = torch.cuda.mem_get_info()[0]
            _noalloc(lib, M, N, K, A, B, C, N, stream)
            torch.cuda.synchronize()
            assert torch.cuda.mem_get_info()[0] == free0, "the call changed the device's free memory"
            C_ref = handle.bf16_nt(A, B)
            torch.cuda.synchronize()
            assert not torch.isnan(C).any()
            g, r = C.float(), C_ref.float()
            assert bool(((g - r).abs() <= 2.0 ** -7 * (r.abs() + 1.0)).all())
            A_bits, B_bits = _bits(A), _bits(B)
            rng = np.random.Generator(np.random.PCG64(M + N))
            rows = np.concatenate([rng.integers(0, M, 2048), np.full(N, M - 1), np.arange(M)])
            cols = np.concatenate([rng.integers(0, N, 2048), np.arange(N), np.full(M, N // 2)])
            exact = oracle_mod.gemm_sampled(A_bits, B_bits, rows, cols)
            got = oracle_mod.bf16_to_f32(_bits(C)[rows, cols])
            assert oracle_mod.within_tolerance(got, exact).all(), oracle_mod.max_scaled_error(got, exact)


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
