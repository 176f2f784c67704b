"""Randomised shapes through the C-ABI: M, N in [1, 1100], K a multiple of
8 in [8, 1040], every tile width (and the automatic choice, which takes the
small-M kernel for M <= 128), output pitch padded by 0-24 columns.  Each
case is compared element by element with the fp64 oracle
(|err| <= 2^-7 (|ref| + 1)), and the columns past N and the rows past M of
the output buffer must be untouched.  Shapes are drawn by hypothesis from a
fixed seed, so the run is reproducible."""
import numpy as np
import pytest

from b200_gemm_b200 import _lib, data

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
hyp = pytest.importorskip("hypothesis")
st = pytest.importorskip("hypothesis.strategies")

NAN_BF16 = 0x7FC0


@hyp.settings(max_examples=60, deadline=None, derandomize=True,
              suppress_health_check=list(hyp.HealthCheck))
@hyp.given(M=st.integers(1, 1100), N=st.integers(1, 1100), k8=st.integers(1, 130),
           width=st.sampled_from([0, 512, 256, 224, 192, 128]), pad=st.integers(0, 3),
           dist=st.sampled_from(["normal", "uniform", "mlp"]))
def test_random_shapes_vs_oracle(gpu_handle, oracle_mod, M, N, k8, width, pad, dist):
    h = gpu_handle
    K = 8 * k8
    A_bits, B_bits = data.host_operands(M, N, K, dist, seed=M * 7919 + N * 31 + K)
    ldc = 8 * ((N + 7) // 8) + 8 * pad
    A = torch.from_numpy(A_bits.view(np.int16)).cuda()
    B = torch.from_numpy(B_bits.view(np.int16)).cuda()
    C = torch.full((M + 16, ldc), NAN_BF16, dtype=torch.int16, device="cuda")
    h.set_tile_width(width)
    try:
        rc = h.bf16_nt_ptr(M, N, K, A.data_ptr(), B.data_ptr(), C.data_ptr(), ldc)
    finally:
        h.set_tile_width(0)
    assert rc == _lib.OK, _lib.strerror(rc)
    torch.cuda.synchronize()
    assert h.last_device_status()[0] == _lib.OK
    out = C.cpu().numpy().view(np.uint16)
    assert np.all(out[M:] == NAN_BF16), "write past row M"
    assert np.all(out[:M, N:] == NAN_BF16), "write past column N"
    ref = oracle_mod.gemm_f64(A_bits, B_bits)
    got = oracle_mod.bf16_to_f32(out[:M, :N])
    ok = oracle_mod.within_tolerance(got, ref)
    assert ok.all(), (M, N, K, width, int((~ok).sum()))


def test_grid_past_16_bit_tile_coordinates_is_rejected(gpu_handle):
    """Tile coordinates are 16-bit: a grid past 65535 tile rows (M > 65535 *
    256) or 65535 columns of the narrowest tile (N > 65535 * 128) is
    B200GEMM_ERR_TOO_LARGE, checked before any memory is touched, so no
    buffers of that size are needed."""
    h = gpu_handle
    p = torch.empty(16, dtype=torch.int16, device="cuda").data_ptr()
    assert h.bf16_nt_ptr(65535 * 256 + 1, 8, 8, p, p, p, 8) == _lib.ERR_TOO_LARGE
    assert h.bf16_nt_ptr(8, 65535 * 128 + 1, 8, p, p, p, 65535 * 128 + 8) == _lib.ERR_TOO_LARGE


@hyp.settings(max_examples=30, deadline=None, derandomize=True,
              suppress_health_check=list(hyp.HealthCheck))
@hyp.given(M=st.integers(1, 256), n8=st.integers(16, 1536), k8=st.integers(16, 512),
           fused=st.booleans())
def test_random_small_m_shapes_vs_oracle(gpu_handle, oracle_mod, M, n8, k8, fused):
    """Decode-shaped problems (M <= 256, N a multiple of 8 up to 12288, K up
    to 4096) through whichever small-M kernel the plan picks (pair or
    single-CTA, K split 1/2/4), plain or with a fused bias + SiLU epilogue."""
    h = gpu_handle
    N, K = 8 * n8, 8 * k8
    plan = h.plan(M, N, K)
    assert plan["kernel"] in ("small_m", "small_m_1cta"), plan
    A_bits, B_bits = data.host_operands(M, N, K, "normal", seed=M * 131 + N + K)
    rng = np.random.Generator(np.random.PCG64(N + K))
    bias_bits = data.f32_to_bf16_bits(rng.standard_normal(N).astype(np.float32))
    A = torch.from_numpy(A_bits.view(np.int16)).cuda().view(torch.bfloat16)
    B = torch.from_numpy(B_bits.view(np.int16)).cuda().view(torch.bfloat16)
    bias = torch.from_numpy(bias_bits.view(np.int16)).cuda().view(torch.bfloat16)
    Cbuf = torch.full((M + 8, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    out = Cbuf[:M]
    if fused:
        h.bf16_nt_epilogue(A, B, bias=bias, activation="silu", out=out)
    else:
        h.bf16_nt(A, B, out=out)
    torch.cuda.synchronize()
    assert h.last_device_status()[0] == _lib.OK
    allc = Cbuf.view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.all(allc[M:] == NAN_BF16), "write past row M"
    ref = oracle_mod.gemm_f64(A_bits, B_bits)
    if fused:
        ref = oracle_mod.epilogue_f64(ref, bias=bias_bits, act="silu")
    got = oracle_mod.bf16_to_f32(allc[:M])
    ok = oracle_mod.within_tolerance(got, ref)
    assert ok.all(), (M, N, K, plan, int((~ok).sum()))
