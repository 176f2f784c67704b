"""Parity at the full sizes of the benchmark configurations, through the
C-ABI, for the kernel instance each shape actually gets:

  * MLP projection 16384 x 14336 x 4096 (A ~ N(0,1) activations, B ~
    N(0,0.02) weights): the width the cost model picks (256 x 512 tiles) and
    forced 256-wide tiles;
  * its 8-way N shard 16384 x 1792 x 4096 (448- and 224-wide tiles);
  * 16384^3 on one GPU (256 x 512 tiles, 28 waves);
  * its 8-way N shard 16384 x 2048 x 16384 (256 x 512 tiles whose short last
    wave runs as 256-column halves on the re-cut 4-stage ring, K = 16384).

Each result is compared with cuBLASLt on every element and with the fp64 CPU
oracle on 4096 random elements plus one full row and one full column; the
tolerance is |err| <= 2^-7 (|ref| + 1) per element.  The two widths of the
MLP shape must agree bit for bit (every element sums its K products in the
same order)."""
import numpy as np
import pytest

from b200_gemm_b200 import data

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

TOL = 2.0 ** -7


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _check_vs_cublaslt(C, A, B):
    """Every element of C against cuBLASLt, 2048 rows at a time."""
    torch.backends.cuda.preferred_blas_library("cublaslt")
    R = torch.matmul(A, B.t())
    torch.cuda.synchronize()
    assert not torch.isnan(C).any()
    worst = 0.0
    for r0 in range(0, C.shape[0], 2048):
        g, r = C[r0:r0 + 2048].float(), R[r0:r0 + 2048].float()
        scaled = ((g - r).abs() / (r.abs() + 1.0)).max().item()
        worst = max(worst, scaled)
    del R
    assert worst <= TOL, f"max scaled error vs cuBLASLt {worst:.3g}"


def _check_vs_oracle(C, A, B, oracle_mod, seed):
    M, N = C.shape
    A_bits, B_bits = _bits(A), _bits(B)
    rng = np.random.Generator(np.random.PCG64(seed))
    row, col = int(rng.integers(0, M)), int(rng.integers(0, N))
    rows = np.concatenate([rng.integers(0, M, 4096), np.full(N, row), np.arange(M)])
    cols = np.concatenate([rng.integers(0, N, 4096), np.arange(N), np.full(M, col)])
    exact = oracle_mod.gemm_sampled(A_bits, B_bits, rows, cols)
    got = oracle_mod.bf16_to_f32(_bits(C)[rows, cols])
    ok = oracle_mod.within_tolerance(got, exact)
    assert ok.all(), (int((~ok).sum()), oracle_mod.max_scaled_error(got, exact))


def _run(h, M, N, K, dist, seed, width=0):
    A, B = data.device_operands(M, N, K, dist, seed=seed)
    h.set_tile_width(width)
    try:
        plan = h.plan(M, N, K)
        C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        h.bf16_nt(A, B, out=C)
        torch.cuda.synchronize()
    finally:
        h.set_tile_width(0)
    rc, detail = h.last_device_status()
    assert rc == 0, detail
    return A, B, C, plan


def test_mlp_16384x14336x4096_auto_and_256(gpu_handle, oracle_mod):
    M, N, K = 16384, 14336, 4096
    A, B, C, plan = _run(gpu_handle, M, N, K, "mlp", seed=31)
    assert plan["kernel"] == "tiled" and plan["tile_width"] == 512, plan
    _check_vs_cublaslt(C, A, B)
    _check_vs_oracle(C, A, B, oracle_mod, seed=1)
    A2, B2, C256, plan256 = _run(gpu_handle, M, N, K, "mlp", seed=31, width=256)
    assert plan256["tile_width"] == 256, plan256
    assert torch.equal(A, A2) and torch.equal(B, B2)
    assert torch.equal(C.view(torch.int16), C256.view(torch.int16)), "256- and 512-wide tiles differ"
    _check_vs_oracle(C256, A, B, oracle_mod, seed=2)


def test_mlp_shard_16384x1792x4096_widths_448_and_224(gpu_handle, oracle_mod):
    """The 8-way shard of the MLP projection: the chosen width (a tile width
    that divides 1792: 448 with a half-width last wave, or 224), and both
    forced, bit-identical to each other."""
    M, N, K = 16384, 1792, 4096
    A, B, C, plan = _run(gpu_handle, M, N, K, "mlp", seed=32)
    assert plan["tile_width"] in (448, 224), plan
    _check_vs_cublaslt(C, A, B)
    _check_vs_oracle(C, A, B, oracle_mod, seed=3)
    for width in (448, 224):
        _, _, Cw, planw = _run(gpu_handle, M, N, K, "mlp", seed=32, width=width)
        assert planw["tile_width"] == width, planw
        assert torch.equal(C.view(torch.int16), Cw.view(torch.int16)), f"width {width} differs"


def test_square_16384_one_gpu(gpu_handle, oracle_mod):
    M = N = K = 16384
    A, B, C, plan = _run(gpu_handle, M, N, K, "normal", seed=33)
    assert plan["kernel"] == "tiled" and plan["tiles"] == 64 * (N // plan["tile_width"]), plan
    _check_vs_cublaslt(C, A, B)
    _check_vs_oracle(C, A, B, oracle_mod, seed=4)


def test_square_16384_shard_half_tail_k16384(gpu_handle, oracle_mod):
    M, N, K = 16384, 2048, 16384
    A, B, C, plan = _run(gpu_handle, M, N, K, "normal", seed=34)
    # 256 tiles of 256 x 512 on 74 clusters: a last wave of 34 tiles, run as
    # 68 half-width units.
    assert plan["tile_width"] == 512 and plan["tail_split"] == -2, plan
    _check_vs_cublaslt(C, A, B)
    _check_vs_oracle(C, A, B, oracle_mod, seed=5)
