"""Parity of the sm_100a kernel (called through the C-ABI) with the CPU
oracle, cuBLASLt and exact known answers.  Tolerance for floating-point
cases: |err| <= 2^-7 (|ref| + 1) per element (oracle.within_tolerance);
integer known-answer cases are bit-exact."""
import ctypes

import numpy as np
import pytest

from b200_gemm_b200 import _lib, data

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

NAN_BF16 = 0x7FC0


def _dev(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).cuda().view(torch.bfloat16)


def _host_bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _run(h, A_bits, B_bits, ldc=None, poison=True):
    M, K = A_bits.shape
    N = B_bits.shape[0]
    full = ldc is not None  # caller wants the whole [M, ldc] buffer back
    ldc = 8 * ((N + 7) // 8) if ldc is None else ldc  # row pitch must be a multiple of 16 bytes
    A, B = _dev(A_bits), _dev(B_bits)
    guard = 64  # poisoned rows after the last row of C: must stay untouched
    C = torch.full((M + guard, ldc), 0, dtype=torch.int16, device="cuda")
    if poison:
        C.fill_(NAN_BF16)
    C = C.view(torch.bfloat16)
    rc = h.bf16_nt_ptr(M, N, K, A.data_ptr(), B.data_ptr(), C.data_ptr(), ldc)
    assert rc == _lib.OK, _lib.strerror(rc)
    torch.cuda.synchronize()
    st, detail = h.last_device_status()
    assert st == _lib.OK, detail
    allc = _host_bits(C)
    fill = NAN_BF16 if poison else 0
    assert np.all(allc[M:] == fill), "write past row M"
    out = allc[:M]
    assert np.all(out[:, N:] == fill), "write outside the N columns"
    return out if full else out[:, :N]


SHAPES = [
    (256, 256, 64),     # one tile, one K block
    (512, 512, 512),    # configs[0]
    (256, 512, 128),
    (300, 200, 72),     # ragged everything, K not a multiple of 64
    (1, 1, 8),
    (1, 300, 8),
    (257, 257, 136),
    (129, 1000, 520),
    (1000, 40, 1032),
    (300, 77, 64),      # N % 8 != 0 inside the first tile
    (40, 1003, 200),    # N % 8 != 0 in the last tile column
    (2560, 2560, 128),  # 100 tiles: more tiles than clusters
    (256, 256, 4096),   # long K: the smem ring wraps many times
]


WIDTHS = [256, 512, 448, 224, 192, 128]


@pytest.fixture(params=WIDTHS, ids=[f"w{w}" for w in WIDTHS])
def width_handle(request, gpu_handle):
    """The session handle forced to one tile width for the test."""
    gpu_handle.set_tile_width(request.param)
    yield gpu_handle
    gpu_handle.set_tile_width(0)


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_parity_vs_oracle(width_handle, oracle_mod, M, N, K):
    A, B = data.host_operands(M, N, K, "normal", seed=M + 7 * N + 13 * K)
    got = _run(width_handle, A, B)
    ref = oracle_mod.gemm_f64(A, B)
    got_f = oracle_mod.bf16_to_f32(got)
    assert not np.isnan(got_f).any(), "unwritten output elements (NaN poison survived)"
    ok = oracle_mod.within_tolerance(got_f, ref)
    assert ok.all(), (np.argwhere(~ok)[:5], oracle_mod.max_scaled_error(got_f, ref))
    # informative: most elements round to the same bf16 as the fp64 oracle
    same = np.mean(got == oracle_mod.f64_to_bf16(ref))
    assert same > 0.9, same


@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (300, 520, 72), (1024, 768, 64)])
def test_known_answer_exact(width_handle, oracle_mod, M, N, K):
    rng = np.random.Generator(np.random.PCG64(M * N + K))
    a = rng.integers(-2, 3, size=(M, K)).astype(np.float32)
    b = rng.integers(-2, 3, size=(N, K)).astype(np.float32)
    exact = (a.astype(np.int64) @ b.astype(np.int64).T).astype(np.float32)
    got = _run(width_handle, oracle_mod.f32_to_bf16(a), oracle_mod.f32_to_bf16(b))
    assert np.array_equal(got, oracle_mod.f32_to_bf16(exact))


def test_identity_and_permutation(gpu_handle, oracle_mod):
    rng = np.random.Generator(np.random.PCG64(5))
    n = 512
    A = oracle_mod.f32_to_bf16(rng.standard_normal((384, n), dtype=np.float32))
    eye = oracle_mod.f32_to_bf16(np.eye(n, dtype=np.float32))
    assert np.array_equal(_run(gpu_handle, A, eye), A)
    perm = rng.permutation(n)
    P = oracle_mod.f32_to_bf16(np.eye(n, dtype=np.float32)[perm])
    assert np.array_equal(_run(gpu_handle, A, P), A[:, perm])


def test_ldc_column_slice(width_handle, oracle_mod):
    """C written into a column window of a wider matrix; the rest untouched."""
    M, N, K, ldc = 300, 264, 128, 1024
    A, B = data.host_operands(M, N, K, "uniform", seed=9)
    got = _run(width_handle, A, B, ldc=ldc)
    assert np.all(got[:, N:] == NAN_BF16)
    ref = oracle_mod.gemm_f64(A, B)
    assert oracle_mod.within_tolerance(oracle_mod.bf16_to_f32(got[:, :N]), ref).all()


def test_k_zero_writes_zeros(gpu_handle):
    A = np.zeros((0,), dtype=np.uint16).reshape(40, 0)
    B = np.zeros((0,), dtype=np.uint16).reshape(24, 0)
    C = torch.full((40, 24), NAN_BF16, dtype=torch.int16, device="cuda").view(torch.bfloat16)
    rc = gpu_handle.bf16_nt_ptr(40, 24, 0, 0, 0, C.data_ptr(), 24)
    assert rc == _lib.OK
    torch.cuda.synchronize()
    assert np.all(_host_bits(C) == 0)


def test_tile_width_selection(gpu_handle):
    h = gpu_handle
    assert h.tile_width_for(8192, 8192, 8192) == 512
    assert h.tile_width_for(256, 256, 64) in WIDTHS
    # N-sharded MLP projection: 1792 = 4 x 448 columns of shared-A tiles,
    # their 34-tile last wave cut into 224-column halves
    assert h.tile_width_for(16384, 1792, 4096) == 448
    assert h.plan(16384, 1792, 4096)["tail_split"] == -2
    # 16384^3 sharded over 8 GPUs: 256 x 512 tiles with their 34-tile last
    # wave cut into 256-column halves, at long and at short K
    assert h.tile_width_for(16384, 2048, 16384) == 512
    assert h.plan(16384, 2048, 16384)["tail_split"] == -2
    assert h.tile_width_for(16384, 2048, 4096) == 512  # half-width last wave, measured 2% over 256
    assert h.tile_width_for(4096, 8192, 8192) == 512  # 256 tiles, a 34-tile last wave in halves
    for w in WIDTHS:
        h.set_tile_width(w)
        assert h.tile_width_for(256, 256, 64) == w
        assert h.plan(512, 1792, 256)["tile_width"] == w
    h.set_tile_width(0)
    for bad in (384, 64, 96, -1):
        with pytest.raises(Exception):
            h.set_tile_width(bad)


def test_device_info(gpu_handle):
    info = gpu_handle.device_info()
    assert info["sm_count"] >= 100
    assert 1 <= info["max_clusters"] <= info["sm_count"] // 2


def test_argument_errors(gpu_handle):
    A = torch.zeros(64, 64, dtype=torch.bfloat16, device="cuda")
    C = torch.zeros(64, 64, dtype=torch.bfloat16, device="cuda")
    p = A.data_ptr()
    h = gpu_handle
    assert h.bf16_nt_ptr(64, 64, 60, p, p, C.data_ptr(), 64) == _lib.ERR_UNSUPPORTED   # K % 8
    assert h.bf16_nt_ptr(64, 64, 64, p + 2, p, C.data_ptr(), 64) == _lib.ERR_UNSUPPORTED  # align
    assert h.bf16_nt_ptr(64, 64, 64, p, p, C.data_ptr(), 60) == _lib.ERR_UNSUPPORTED   # ldc < N
    assert h.bf16_nt_ptr(64, 64, 64, p, p, C.data_ptr(), 68) == _lib.ERR_UNSUPPORTED   # ldc % 8
    assert h.bf16_nt_ptr(-1, 64, 64, p, p, C.data_ptr(), 64) == _lib.ERR_INVALID_ARG
    assert h.bf16_nt_ptr(64, 64, 64, 0, p, C.data_ptr(), 64) == _lib.ERR_INVALID_ARG
    assert h.bf16_nt_ptr(0, 64, 64, 0, 0, 0, 64) == _lib.OK  # empty problem is a no-op
    assert h.bf16_nt_ptr(64, 20000000, 64, p, p, C.data_ptr(), 20000000) == _lib.ERR_TOO_LARGE
    torch.cuda.synchronize()
    assert h.last_device_status()[0] == _lib.OK


def test_stream_and_determinism(gpu_handle, oracle_mod):
    M, N, K = 1024, 1536, 768
    A_bits, B_bits = data.host_operands(M, N, K, "normal", seed=21)
    A, B = _dev(A_bits), _dev(B_bits)
    s = torch.cuda.Stream()
    outs = []
    for _ in range(2):
        C = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        with torch.cuda.stream(s):
            gpu_handle.bf16_nt(A, B, out=C, stream=s)
        s.synchronize()
        outs.append(_host_bits(C))
    assert np.array_equal(outs[0], outs[1])
    ref = oracle_mod.gemm_f64(A_bits, B_bits)
    assert oracle_mod.within_tolerance(oracle_mod.bf16_to_f32(outs[0]), ref).all()


def test_watchdog_times_out_and_context_survives(gpu_handle, oracle_mod):
    h = gpu_handle
    assert h.last_device_status()[0] == _lib.OK
    h.selftest_watchdog(20_000_000)  # 20 ms budget on a wait nothing satisfies
    rc, detail = h.last_device_status()
    assert rc == _lib.ERR_DEVICE_TIMEOUT
    assert detail[0] == _lib.ERR_DEVICE_TIMEOUT and detail[1] == 9
    assert h.last_device_status()[0] == _lib.OK  # reading clears it
    # the context is still usable
    A, B = data.host_operands(256, 256, 128, "normal", seed=1)
    got = _run(h, A, B)
    assert oracle_mod.within_tolerance(oracle_mod.bf16_to_f32(got), oracle_mod.gemm_f64(A, B)).all()


def test_run_kernel_dropin(oracle_mod):
    """The reference-shaped entry point (runKernel1 signature, ldc = N)."""
    from b200_gemm_b200 import run_kernel

    M = N = K = 512
    A_bits, B_bits = data.host_operands(M, N, K, "normal", seed=0)
    A, B = _dev(A_bits), _dev(B_bits)
    C = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    run_kernel(2, M, N, K, A, B, C)
    C0 = torch.empty_like(C)
    run_kernel(0, M, N, K, A, B, C0)
    torch.cuda.synchronize()
    ref = oracle_mod.gemm_f64(A_bits, B_bits)
    assert oracle_mod.within_tolerance(oracle_mod.bf16_to_f32(_host_bits(C)), ref).all()
    assert oracle_mod.within_tolerance(oracle_mod.bf16_to_f32(_host_bits(C0)), ref).all()


def _tol_vs(got, ref):
    g = got.float()
    r = ref.float()
    return (g - r).abs() <= (2.0 ** -7) * (r.abs() + 1.0)


def test_8192_vs_cublaslt_and_sampled_oracle(gpu_handle, oracle_mod):
    """8192^3, U[-1,1].  Every element vs cuBLASLt; 4096 random
    elements plus one full tile row and column vs the fp64 oracle."""
    M = N = K = 8192
    A, B = data.device_operands(M, N, K, "uniform", seed=1)
    C = gpu_handle.bf16_nt(A, B)
    torch.backends.cuda.preferred_blas_library("cublaslt")
    R = torch.matmul(A, B.t())
    torch.cuda.synchronize()
    assert not torch.isnan(C).any()
    assert bool(_tol_vs(C, R).all())
    A_bits, B_bits = _host_bits(A), _host_bits(B)
    rng = np.random.Generator(np.random.PCG64(2))
    rows = np.concatenate([rng.integers(0, M, 4096), np.full(N, 4321), np.arange(M)])
    cols = np.concatenate([rng.integers(0, N, 4096), np.arange(N), np.full(M, 1234)])
    ref = oracle_mod.gemm_sampled(A_bits, B_bits, rows, cols)
    got = oracle_mod.bf16_to_f32(_host_bits(C)[rows, cols])
    assert oracle_mod.within_tolerance(got, ref).all()


@pytest.mark.parametrize("width", WIDTHS[1:])
def test_8192_widths_agree(gpu_handle, width):
    """Every tile width gives the 256-wide result bit for bit (same per-element
    K order)."""
    M = N = K = 8192
    A, B = data.device_operands(M, N, K, "normal", seed=4)
    gpu_handle.set_tile_width(256)
    C1 = gpu_handle.bf16_nt(A, B)
    gpu_handle.set_tile_width(width)
    C2 = gpu_handle.bf16_nt(A, B)
    gpu_handle.set_tile_width(0)
    torch.cuda.synchronize()
    assert torch.equal(C1.view(torch.int16), C2.view(torch.int16))


def test_full_size_properties(gpu_handle):
    """Size-independent properties at 8192 x 8192 x 8192 (N(0,1)):
    permuting rows of A permutes rows of C bit-exactly, and scaling A by 2
    scales C by 2 bit-exactly."""
    M = N = K = 8192
    A, B = data.device_operands(M, N, K, "normal", seed=3)
    C = gpu_handle.bf16_nt(A, B)
    perm = torch.randperm(M, device="cuda", generator=torch.Generator("cuda").manual_seed(0))
    Cp = gpu_handle.bf16_nt(A[perm].contiguous(), B)
    C2 = gpu_handle.bf16_nt((A.float() * 2).to(torch.bfloat16), B)
    torch.cuda.synchronize()
    assert torch.equal(Cp.view(torch.int16), C[perm].view(torch.int16))
    assert torch.equal(C2.view(torch.int16), (C.float() * 2).to(torch.bfloat16).view(torch.int16))
