"""Fused epilogue (b200gemm_bf16_nt_epilogue): C = act(alpha A.B^T + bias) +
beta R, rounded to bf16 or stored as fp32, checked through the C-ABI against
the fp64 oracle (oracle.epilogue_f64 on oracle.gemm_f64):
  * bf16 output: |err| <= 2^-7 (|ref| + 1) per element (oracle.within_tolerance);
  * fp32 output: |err| <= 2^-14 (|ref| + |alpha| sqrt(K) + 1) -- fp32
    accumulation of K products of unit-scale values, plus the activation;
and bit for bit against the plain GEMM where the two must agree (no
epilogue terms; fp32 output rounded to bf16)."""
import ctypes

import numpy as np
import pytest

from b200_gemm_b200 import _lib, data

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

NAN_BF16 = 0x7FC0
ACTS = ["none", "relu", "gelu", "gelu_tanh", "silu"]


def _dev(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).cuda().view(torch.bfloat16)


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _rand_bits(shape, seed, scale=1.0):
    rng = np.random.Generator(np.random.PCG64(seed))
    return data.f32_to_bf16_bits((rng.standard_normal(shape) * scale).astype(np.float32))


def _f32_close(got, ref, alpha, K):
    got = np.asarray(got, dtype=np.float64)
    return np.abs(got - ref) <= 2.0 ** -14 * (np.abs(ref) + abs(alpha) * np.sqrt(K) + 1.0)


def _case(h, oracle_mod, M, N, K, act, use_bias, use_res, alpha, beta, out_dtype, seed):
    A_bits, B_bits = data.host_operands(M, N, K, "normal", seed=seed)
    bias_bits = _rand_bits((N,), seed + 1) if use_bias else None
    res_bits = _rand_bits((M, N), seed + 2) if use_res else None
    A, B = _dev(A_bits), _dev(B_bits)
    bias = _dev(bias_bits) if use_bias else None
    res = None
    if use_res:  # a column window of a wider buffer: ldr != N
        ldr = 8 * ((N + 7) // 8) + 16
        full = torch.zeros(M, ldr, dtype=torch.bfloat16, device="cuda")
        full[:, :N] = _dev(res_bits)
        res = full[:, :N]
    # poisoned guard rows and columns around C must stay untouched
    group = 8 if out_dtype == torch.bfloat16 else 4
    ldc = group * ((N + group - 1) // group) + group
    Cbuf = torch.full((M + 32, ldc), float("nan"), dtype=out_dtype, device="cuda")
    out = Cbuf[:M, :N]
    h.bf16_nt_epilogue(A, B, bias=bias, activation=act, residual=res, alpha=alpha, beta=beta,
                       out=out)
    torch.cuda.synchronize()
    assert h.last_device_status()[0] == 0
    allc = Cbuf.cpu()
    assert torch.isnan(allc[M:]).all() and torch.isnan(allc[:M, N:]).all(), "write outside C"
    ref = oracle_mod.epilogue_f64(oracle_mod.gemm_f64(A_bits, B_bits), alpha=alpha, bias=bias_bits,
                                  act=act, residual=res_bits, beta=beta)
    got = allc[:M, :N].float().numpy()
    if out_dtype == torch.bfloat16:
        ok = oracle_mod.within_tolerance(got, ref)
    else:
        ok = _f32_close(got, ref, alpha, K)
    assert ok.all(), (act, use_bias, use_res, float(np.abs(got - ref).max()))
    return A, B, out


@pytest.mark.parametrize("act", ACTS)
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
def test_epilogue_parity(gpu_handle, oracle_mod, act, out_dtype):
    # ragged in M, N and K-blocks; every term on
    _case(gpu_handle, oracle_mod, 300, 203, 136, act, True, True, 0.5, 0.75, out_dtype, seed=11)


@pytest.mark.parametrize("use_bias,use_res", [(True, False), (False, True), (False, False)])
@pytest.mark.parametrize("width", [256, 512, 224, 128])
def test_epilogue_terms_and_widths(gpu_handle, oracle_mod, use_bias, use_res, width):
    h = gpu_handle
    h.set_tile_width(width)
    try:
        for out_dtype in (torch.bfloat16, torch.float32):
            _case(h, oracle_mod, 520, 600, 256, "gelu", use_bias, use_res, 1.0, -1.0, out_dtype,
                  seed=width + use_bias * 2 + use_res)
    finally:
        h.set_tile_width(0)


# (M, N, K, small-M kernel the plan picks)
SMALL_M = [(1, 1024, 512, "small_m"), (64, 4096, 1024, "small_m_1cta"), (128, 8192, 512, "small_m"),
           (77, 1040, 384, "small_m"), (100, 3968, 704, "small_m_1cta"), (256, 4096, 512, "small_m"),
           (200, 1040, 384, "small_m"), (640, 1024, 512, "small_m"), (2048, 1024, 2048, "small_m")]


@pytest.mark.parametrize("M,N,K,kernel", SMALL_M)
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
def test_epilogue_small_m(gpu_handle, oracle_mod, M, N, K, kernel, out_dtype):
    """Small M keeps the small-M kernels (pair or single-CTA) with the epilogue."""
    assert gpu_handle.plan(M, N, K)["kernel"] == kernel
    for act, use_bias, use_res in (("silu", True, True), ("gelu", True, False), ("none", False, True)):
        _case(gpu_handle, oracle_mod, M, N, K, act, use_bias, use_res, 0.5, -1.0, out_dtype, seed=M + N)


@pytest.mark.parametrize("M,N,K,kernel", SMALL_M)
def test_epilogue_small_m_e4m3(gpu_handle, oracle_mod, M, N, K, kernel):
    if N % 16:
        pytest.skip("e4m3 small-M output needs N % 16 == 0 (the tiled kernel covers the rest)")
    _e4m3_case(gpu_handle, oracle_mod, M, N, K, "gelu_tanh", True, True, 8.0, seed=M + 2 * N)


@pytest.mark.parametrize("M,N,K,kernel", SMALL_M)
def test_small_m_identity_epilogue_bit_exact(gpu_handle, M, N, K, kernel):
    """No terms: the same small-M kernel writes what the plain call writes;
    fp32 output rounded to bf16 is the plain call's output too."""
    h = gpu_handle
    A, B = data.device_operands(M, N, K, "normal", seed=3)
    C0 = h.bf16_nt(A, B)
    C1 = h.bf16_nt_epilogue(A, B)
    C2 = h.bf16_nt_epilogue(A, B, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(C0.view(torch.int16), C1.view(torch.int16))
    assert torch.equal(C0.view(torch.int16), C2.to(torch.bfloat16).view(torch.int16))


def test_large_activation_range(gpu_handle, oracle_mod):
    """Pre-activations far into the tails (|x| up to ~100): SiLU's exp overflow, GELU's erf limit."""
    for act in ("gelu", "gelu_tanh", "silu", "relu"):
        _case(gpu_handle, oracle_mod, 256, 256, 136, act, True, False, 8.0, 1.0, torch.bfloat16, seed=5)


def _e4m3_case(h, oracle_mod, M, N, K, act, use_bias, use_res, scale, seed, width=0):
    A_bits, B_bits = data.host_operands(M, N, K, "normal", seed=seed)
    bias_bits = _rand_bits((N,), seed + 1) if use_bias else None
    res_bits = _rand_bits((M, N), seed + 2) if use_res else None
    A, B = _dev(A_bits), _dev(B_bits)
    bias = _dev(bias_bits) if use_bias else None
    res = None
    if use_res:  # rows 16-byte aligned: pad the pitch to a multiple of 8
        full = torch.zeros(M, 8 * ((N + 7) // 8), dtype=torch.bfloat16, device="cuda")
        full[:, :N] = _dev(res_bits)
        res = full[:, :N]
    ldc = 16 * ((N + 15) // 16) + 16
    Cbuf = torch.full((M + 32, ldc), 0x7F, dtype=torch.uint8, device="cuda")  # 0x7F = NaN
    out = Cbuf.view(torch.float8_e4m3fn)[:M, :N]
    h.set_tile_width(width)
    try:
        h.bf16_nt_epilogue(A, B, bias=bias, activation=act, residual=res, alpha=1.0, beta=1.0,
                           out=out, out_scale=scale)
    finally:
        h.set_tile_width(0)
    torch.cuda.synchronize()
    assert h.last_device_status()[0] == 0
    allc = Cbuf.cpu().numpy()
    assert np.all(allc[M:] == 0x7F) and np.all(allc[:M, N:] == 0x7F), "write outside C"
    ref = scale * oracle_mod.epilogue_f64(oracle_mod.gemm_f64(A_bits, B_bits), bias=bias_bits, act=act,
                                          residual=res_bits, beta=1.0)
    got = oracle_mod.e4m3_to_f64(allc[:M, :N])
    sat = np.abs(ref) >= 448.0
    assert np.all(got[sat] == np.sign(ref[sat]) * 448.0)
    # within one e4m3 step of the exact value (RNE of a value within fp32
    # accumulation error of it)
    ok = np.abs(got - ref) <= oracle_mod.e4m3_ulp(ref)
    assert ok[~sat].all(), float(np.abs(got - ref)[~sat].max())
    return A, B


@pytest.mark.parametrize("act,use_bias,use_res", [("none", False, False), ("gelu_tanh", True, False),
                                                  ("silu", True, True), ("relu", False, True)])
@pytest.mark.parametrize("width", [512, 224])
def test_epilogue_e4m3(gpu_handle, oracle_mod, act, use_bias, use_res, width):
    # ragged N (not a multiple of 16 or 32); scale spreads values over the
    # e4m3 range, some past 448 (saturation)
    _e4m3_case(gpu_handle, oracle_mod, 300, 203, 136, act, use_bias, use_res, 16.0, seed=31, width=width)


def test_epilogue_e4m3_bit_exact_vs_fp32(gpu_handle, oracle_mod):
    """e4m3 output = the oracle's RNE-saturating encoding of (out_scale x the
    fp32 output) bit for bit (ReLU: no transcendental): pins the device
    conversion to the oracle's codec."""
    h = gpu_handle
    M, N, K = 512, 768, 256
    A, B = data.device_operands(M, N, K, "normal", seed=17)
    scale = 3.0
    C32 = h.bf16_nt_epilogue(A, B, activation="relu", out_dtype=torch.float32)
    C8 = h.bf16_nt_epilogue(A, B, activation="relu", out_dtype=torch.float8_e4m3fn, out_scale=scale)
    torch.cuda.synchronize()
    x = (C32.cpu().numpy().astype(np.float32) * np.float32(scale)).astype(np.float64)
    want = oracle_mod.f64_to_e4m3(x)
    got = C8.contiguous().view(torch.uint8).cpu().numpy()
    assert np.array_equal(got, want)


@pytest.mark.parametrize("width", [512, 256, 224])
def test_identity_epilogue_bit_exact(gpu_handle, width):
    """No terms: the fused instance writes exactly what the plain GEMM writes;
    fp32 output rounded to bf16 (RNE) is the plain GEMM's output too."""
    h = gpu_handle
    M, N, K = 1024, 1536, 1024
    A, B = data.device_operands(M, N, K, "normal", seed=7)
    h.set_tile_width(width)
    try:
        C0 = h.bf16_nt(A, B)
        C1 = h.bf16_nt_epilogue(A, B)
        C2 = h.bf16_nt_epilogue(A, B, out_dtype=torch.float32)
        C3 = h.bf16_nt_epilogue(A, B, alpha=1.0, beta=0.0, residual=C0)  # beta = 0: R adds 0
    finally:
        h.set_tile_width(0)
    torch.cuda.synchronize()
    assert torch.equal(C0.view(torch.int16), C1.view(torch.int16))
    assert torch.equal(C0.view(torch.int16), C2.to(torch.bfloat16).view(torch.int16))
    assert torch.equal(C0.view(torch.int16), C3.view(torch.int16))


def test_epilogue_4096_vs_torch_and_sampled_oracle(gpu_handle, oracle_mod):
    """Full size: every element against an fp32 torch composite, sampled
    elements plus a full row and column against the fp64 oracle."""
    h = gpu_handle
    M = N = K = 4096
    A, B = data.device_operands(M, N, K, "normal", seed=21)
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    bias = torch.randn(N, generator=g, device="cuda").to(torch.bfloat16)
    res = torch.randn(M, N, generator=g, device="cuda").to(torch.bfloat16)
    alpha, beta = 0.125, 0.5
    C = h.bf16_nt_epilogue(A, B, bias=bias, activation="gelu", residual=res, alpha=alpha, beta=beta)
    C1 = h.bf16_nt_epilogue(A, B, bias=bias, activation="gelu", residual=res, alpha=alpha, beta=beta)
    torch.cuda.synchronize()
    assert torch.equal(C.view(torch.int16), C1.view(torch.int16))  # deterministic
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        S = A.float() @ B.float().t()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    R = torch.nn.functional.gelu(alpha * S + bias.float()) + beta * res.float()
    diff = (C.float() - R).abs()
    assert bool((diff <= 2.0 ** -7 * (R.abs() + 1.0)).all()), float(diff.max())
    rng = np.random.Generator(np.random.PCG64(9))
    rows = np.concatenate([rng.integers(0, M, 4096), np.full(N, M - 1), np.arange(M)])
    cols = np.concatenate([rng.integers(0, N, 4096), np.arange(N), np.full(M, N - 1)])
    A_bits, B_bits = _bits(A), _bits(B)
    s = oracle_mod.gemm_sampled(A_bits, B_bits, rows, cols)
    ref = oracle_mod.epilogue_sampled(s, rows, cols, alpha=alpha, bias=_bits(bias), act="gelu",
                                      residual=_bits(res), beta=beta)
    got = oracle_mod.bf16_to_f32(_bits(C)[rows, cols])
    assert oracle_mod.within_tolerance(got, ref).all()


def test_epilogue_argument_errors(gpu_handle):
    h = gpu_handle
    L = _lib.load()
    M, N, K = 256, 256, 64
    A, B = data.device_operands(M, N, K, "normal", seed=1)
    C = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    Cf = torch.empty(M, N + 4, dtype=torch.float32, device="cuda")
    bias = torch.zeros(N + 8, dtype=torch.bfloat16, device="cuda")
    res = torch.zeros(M, N, dtype=torch.bfloat16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream

    def call(epi, c=C, ldc=N, k=K):
        return L.b200gemm_bf16_nt_epilogue(h._h, M, N, k, A.data_ptr(), B.data_ptr(), c.data_ptr(),
                                           ldc, ctypes.byref(epi), s)

    assert call(_lib.Epilogue(alpha=1.0, activation=9)) == _lib.ERR_INVALID_ARG
    assert call(_lib.Epilogue(alpha=1.0, out_type=7)) == _lib.ERR_INVALID_ARG
    assert call(_lib.Epilogue(alpha=1.0, bias=bias.data_ptr() + 2)) == _lib.ERR_UNSUPPORTED
    assert call(_lib.Epilogue(alpha=1.0, residual=res.data_ptr(), ldr=N - 8)) == _lib.ERR_UNSUPPORTED
    assert call(_lib.Epilogue(alpha=1.0, residual=res.data_ptr(), ldr=N + 4)) == _lib.ERR_UNSUPPORTED
    assert call(_lib.Epilogue(alpha=1.0), k=0) == _lib.ERR_UNSUPPORTED
    assert call(_lib.Epilogue(alpha=1.0, out_type=_lib.OUT_F32), c=Cf, ldc=N + 2) == _lib.ERR_UNSUPPORTED
    assert call(_lib.Epilogue(alpha=1.0, out_type=_lib.OUT_F32), c=Cf, ldc=N + 4) == _lib.OK
    C8 = torch.empty(M, N + 16, dtype=torch.uint8, device="cuda")
    assert call(_lib.Epilogue(alpha=1.0, out_type=_lib.OUT_E4M3), c=C8, ldc=N + 8) == _lib.ERR_UNSUPPORTED
    assert call(_lib.Epilogue(alpha=1.0, out_type=_lib.OUT_E4M3, out_scale=2.0), c=C8, ldc=N + 16) == _lib.OK
    # NULL epilogue = the plain GEMM
    assert L.b200gemm_bf16_nt_epilogue(h._h, M, N, K, A.data_ptr(), B.data_ptr(), C.data_ptr(), N,
                                       None, s) == _lib.OK
    torch.cuda.synchronize()
    assert h.last_device_status()[0] == 0
    with pytest.raises(ValueError):
        h.bf16_nt_epilogue(A, B, activation="tanh")
