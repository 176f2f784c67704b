"""CPU checks of the oracle itself: bf16 rounding, known-answer GEMMs with
exact integer arithmetic, fp32 CPU baseline vs fp64 reference, sampling."""
import numpy as np
import pytest

from b200_gemm_b200 import data


def test_bf16_round_to_nearest_even(oracle_mod):
    o = oracle_mod
    # 1 + 2^-8 is exactly halfway between bf16 1.0 and 1.0078125 -> even (1.0)
    # 1 + 3*2^-8 is halfway between 1.0078125 and 1.015625 -> even (1.015625)
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, 1.0 + 2 ** -8 + 2 ** -20, -2.5,
                  np.inf, -np.inf, 0.0, -0.0, 3.4e38, 1e-40], dtype=np.float32)
    bits = o.f32_to_bf16(x)
    back = o.bf16_to_f32(bits)
    assert back[0] == 1.0
    assert back[1] == 1.0
    assert back[2] == 1.015625
    assert back[3] == 1.0078125
    assert back[4] == -2.5
    assert np.isposinf(back[5]) and np.isneginf(back[6])
    assert bits[7] == 0x0000 and bits[8] == 0x8000
    assert np.isposinf(back[9])  # 3.4e38 is past the bf16 rounding midpoint above its max (3.3895e38)
    nan_bits = o.f32_to_bf16(np.array([np.nan], dtype=np.float32))
    assert np.isnan(o.bf16_to_f32(nan_bits))[0]
    # numpy restatement used by the data generator agrees on random values
    r = np.random.Generator(np.random.PCG64(1)).standard_normal(100000, dtype=np.float32) * 100
    assert np.array_equal(o.f32_to_bf16(r), data.f32_to_bf16_bits(r))


def _exact_int_case(M, N, K, lo, hi, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    a = rng.integers(lo, hi + 1, size=(M, K)).astype(np.int64)
    b = rng.integers(lo, hi + 1, size=(N, K)).astype(np.int64)
    exact = a @ b.T
    return a, b, exact


@pytest.mark.parametrize("M,N,K", [(1, 1, 8), (7, 5, 64), (64, 48, 40), (130, 260, 72)])
def test_known_answer_small_integers(oracle_mod, M, N, K):
    """Entries in [-2, 2] with K <= 72: every partial sum is an integer of
    magnitude <= 288 < 2^24 and the result is a bf16-exact integer only when
    |C| <= 256, so compare in float64 and demand exact equality."""
    o = oracle_mod
    a, b, exact = _exact_int_case(M, N, K, -2, 2, seed=M * 1000 + N)
    A = o.f32_to_bf16(a.astype(np.float32))
    B = o.f32_to_bf16(b.astype(np.float32))
    ref = o.gemm_f64(A, B)
    assert np.array_equal(ref, exact.astype(np.float64))
    bits = o.gemm_bf16(A, B)
    expect = o.f32_to_bf16(exact.astype(np.float32))
    assert np.array_equal(bits, expect)


def test_known_answer_identity_and_permutation(oracle_mod):
    o = oracle_mod
    rng = np.random.Generator(np.random.PCG64(7))
    n = 96
    A = o.f32_to_bf16(rng.standard_normal((80, n), dtype=np.float32))
    eye = o.f32_to_bf16(np.eye(n, dtype=np.float32))
    assert np.array_equal(o.gemm_bf16(A, eye), A)  # A . I^T = A
    perm = rng.permutation(n)
    P = o.f32_to_bf16(np.eye(n, dtype=np.float32)[perm])
    assert np.array_equal(o.gemm_bf16(A, P), A[:, perm])


def test_f32_cpu_baseline_within_tolerance(oracle_mod):
    o = oracle_mod
    A, B = data.host_operands(67, 93, 520, "normal", seed=3)
    ref = o.gemm_f64(A, B)
    got, used = o.gemm_f32_cpu(A, B, threads=3)
    assert used >= 1
    assert o.within_tolerance(o.bf16_to_f32(got), ref).all()
    # row band only
    part, _ = o.gemm_f32_cpu(A, B, row_begin=10, row_end=33, threads=2)
    assert np.array_equal(part, got[10:33])


def test_sampled_matches_full(oracle_mod):
    o = oracle_mod
    A, B = data.host_operands(50, 40, 136, "uniform", seed=5)
    full = o.gemm_f64(A, B)
    rows = np.array([0, 49, 13, 7], dtype=np.int32)
    cols = np.array([39, 0, 22, 7], dtype=np.int32)
    assert np.array_equal(o.gemm_sampled(A, B, rows, cols), full[rows, cols])


def test_tolerance_rule(oracle_mod):
    o = oracle_mod
    ref = np.array([0.0, 100.0, -100.0])
    ok = o.within_tolerance(np.array([2 ** -7, 100.0 + 101 * 2 ** -7, -100.5]), ref)
    assert ok.all()
    bad = o.within_tolerance(np.array([0.01, 100.0 + 2.0, -99.0]), ref)
    assert not bad.any()
    # the planted mistake is caught: flip one oracle output by a few ulps
    A, B = data.host_operands(16, 16, 64, "normal", seed=11)
    ref = o.gemm_f64(A, B)
    wrong = ref.copy()
    wrong[3, 4] += 0.5 + abs(ref[3, 4]) * 0.05
    assert not o.within_tolerance(wrong, ref).all()


@pytest.mark.parametrize("dist", data.DISTS)
def test_generators_are_seeded(dist):
    a1, b1 = data.host_operands(8, 9, 16, dist, seed=42)
    a2, b2 = data.host_operands(8, 9, 16, dist, seed=42)
    a3, _ = data.host_operands(8, 9, 16, dist, seed=43)
    assert np.array_equal(a1, a2) and np.array_equal(b1, b2)
    assert not np.array_equal(a1, a3)
    bf = data.bf16_bits_to_f32(b1)
    if dist == "mlp":
        assert np.abs(bf).max() < 0.2
    if dist == "uniform":
        assert np.abs(bf).max() <= 1.0


@pytest.mark.parametrize("act", ["none", "relu", "gelu", "gelu_tanh", "silu"])
def test_epilogue_restatement(oracle_mod, act):
    """The C restatement of the fused epilogue against an independent numpy /
    scipy evaluation of the same formulas, full and sampled."""
    from scipy.special import erf

    o = oracle_mod
    rng = np.random.Generator(np.random.PCG64(4))
    M, N = 37, 53
    S = rng.standard_normal((M, N)) * 6.0
    bias = data.f32_to_bf16_bits(rng.standard_normal(N).astype(np.float32))
    res = data.f32_to_bf16_bits(rng.standard_normal((M, N)).astype(np.float32))
    alpha, beta = 0.75, -1.5
    x = alpha * S + data.bf16_bits_to_f32(bias).astype(np.float64)[None, :]
    f = {
        "none": lambda v: v,
        "relu": lambda v: np.maximum(v, 0.0),
        "gelu": lambda v: 0.5 * v * (1.0 + erf(v / np.sqrt(2.0))),
        "gelu_tanh": lambda v: 0.5 * v * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (v + 0.044715 * v ** 3))),
        "silu": lambda v: v / (1.0 + np.exp(-v)),
    }[act]
    want = f(x) + beta * data.bf16_bits_to_f32(res).astype(np.float64)
    got = o.epilogue_f64(S, alpha=alpha, bias=bias, act=act, residual=res, beta=beta)
    assert np.allclose(got, want, rtol=1e-12, atol=1e-12)
    rows = rng.integers(0, M, 200).astype(np.int32)
    cols = rng.integers(0, N, 200).astype(np.int32)
    got_s = o.epilogue_sampled(S[rows, cols], rows, cols, alpha=alpha, bias=bias, act=act,
                               residual=res, beta=beta)
    assert np.allclose(got_s, want[rows, cols], rtol=1e-12, atol=1e-12)
    # no bias, no residual: only the scale and the activation
    assert np.allclose(o.epilogue_f64(S, alpha=alpha, act=act), f(alpha * S), rtol=1e-12, atol=1e-12)


def test_e4m3_codec(oracle_mod):
    """The oracle's fp8 e4m3 encoder (RNE, saturating) against torch's
    float8_e4m3fn conversion on in-range values, exact round trips, and the
    saturation / NaN / subnormal edges."""
    torch = pytest.importorskip("torch")
    o = oracle_mod
    rng = np.random.Generator(np.random.PCG64(8))
    x = (rng.standard_normal(100000) * np.exp2(rng.uniform(-12, 10, 100000))).astype(np.float32)
    x = x[np.abs(x) < 448].astype(np.float64)
    want = torch.from_numpy(x.astype(np.float32)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(o.f64_to_e4m3(x), want)
    every = np.arange(256, dtype=np.uint8)
    vals = o.e4m3_to_f64(every)
    finite = ~np.isnan(vals)
    assert np.sum(~finite) == 2  # 0x7F and 0xFF
    assert np.array_equal(o.f64_to_e4m3(vals[finite])[vals[finite] != 0],
                          every[finite][vals[finite] != 0])
    edge = np.array([448.0, 463.9, 464.0, 1e30, -1e30, 2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -11, np.nan])
    assert list(o.f64_to_e4m3(edge)) == [0x7E, 0x7E, 0x7E, 0x7E, 0xFE, 0x01, 0x00, 0x01, 0x7F]
    assert np.allclose(o.e4m3_ulp([1.0, 1.9, 448.0, 1e-3]), [0.125, 0.125, 32.0, 2.0 ** -9])
