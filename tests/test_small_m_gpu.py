"""Parity of the small-M (decode-shaped) kernels: rows of B on the MMA's M
side, K split over 1, 2, 3 or 4 CTA pairs (pair kernel) or 1, 2 or 4 CTAs
(single-CTA kernel) of a cluster, partial sums reduced through distributed
shared memory; above 256 rows of A the pair kernel runs over blocks of 128 or
256 rows of A.  Compared with the fp64 oracle (|err| <= 2^-7 (|ref| + 1))
and, bit for bit where the K split is 1, with the tiled kernel."""
import numpy as np
import pytest

from b200_gemm_b200 import _lib, data

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _dev(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).cuda().view(torch.bfloat16)


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


# (M, N, K, kernel, split) on a 148-SM B200.  Pair kernel: 256 rows of B per
# CTA pair, clusters of 2S CTAs (33 clusters of 4 and 15 of 8 fit at once;
# clusters of 6, split 3, only for 129..256 rows of A; above 256 rows of A
# a cluster covers 128 or 256 of them, split 2 or 4);
# single-CTA kernel: 128 rows of B per CTA, clusters of S, taken where it
# puts at least 1.5x the CTAs to work (narrow N).
CASES = [
    (128, 4096, 1024, "small_m_1cta", 4),
    (1, 4096, 4096, "small_m_1cta", 4),
    (77, 3976, 1000, "small_m_1cta", 4),  # ragged M, N (3976 = 31 x 128 + 8) and K
    (64, 9216, 512, "small_m_1cta", 2),
    (128, 8192, 512, "small_m", 2),
    (64, 16384, 256, "small_m", 1),
    (1, 512, 1024, "small_m", 4),
    (77, 2048, 1000, "small_m", 4),     # ragged M and K
    (128, 2048, 576, "small_m", 4),     # 9 K blocks over 4 pairs: the last pair has none
    (100, 1032, 384, "small_m", 2),     # N not a multiple of 256: the last cluster is ragged
    (128, 8192, 8128, "small_m", 2),    # 127 K blocks: the last stage's second block lies past K
    (64, 16384, 320, "small_m", 1),     # 5 K blocks in stages of 2
    # 129..256 rows of A: the pair kernel with MMA N = 256, one K block per stage
    (256, 4096, 1024, "small_m", 3),    # 16 clusters of 8 do not fit: split 3 (slices 96 + 96 + 64)
    (160, 4096, 1032, "small_m", 3),    # split 3, ragged K; the third pair's rows all lie past M
    (192, 2048, 1000, "small_m", 4),    # ragged K
    (129, 16384, 256, "small_m", 1),
    (200, 1032, 384, "small_m", 3),     # ragged M and N; 6 K blocks over 3 pairs
    (256, 8192, 520, "small_m", 2),     # 9 K blocks, the last one partial
    # More than 256 rows of A: one cluster per 256 rows of B x 128 (or 256)
    # rows of A, where a CTA then moves at most 0.8x the tiled kernel's bytes.
    (512, 512, 512, "small_m", 2),      # 8 K blocks: too few for split 4
    (384, 512, 2048, "small_m", 4),     # 6 clusters of 8
    (1024, 1024, 1024, "small_m", 2),   # 32 clusters of 4
    (1000, 1024, 1000, "small_m", 2),   # ragged M and K: the last M block is 104 rows
    (768, 1032, 384, "small_m", 2),     # ragged N; 6 K blocks over 2 pairs
    (2048, 1024, 4096, "small_m", 2),   # 256-row blocks of A: 32 clusters of 4
    (2000, 1000, 4000, "small_m", 2),   # 256-row blocks, ragged M, N and K
    (300, 1024, 136, "tiled", 0),       # 3 K blocks: too few to split
    (4096, 512, 512, "tiled", 0),       # the tiled kernel moves fewer bytes per CTA
]


@pytest.mark.parametrize("M,N,K,kernel,split", CASES)
def test_small_m_parity(gpu_handle, oracle_mod, M, N, K, kernel, split):
    h = gpu_handle
    plan = h.plan(M, N, K)
    assert (plan["kernel"], plan["small_m_split"]) == (kernel, split), plan
    assert h.small_m_split(M, N, K) == split
    A_bits, B_bits = data.host_operands(M, N, K, "normal", seed=M * 7 + N + K)
    A, B = _dev(A_bits), _dev(B_bits)
    C = torch.full((M + 16, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    rc = h.bf16_nt_ptr(M, N, K, A.data_ptr(), B.data_ptr(), C.data_ptr(), N,
                       torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.OK, _lib.strerror(rc)
    torch.cuda.synchronize()
    st, detail = h.last_device_status()
    assert st == _lib.OK, detail
    allc = _bits(C)
    assert np.all(allc[M:] == 0x7FC0), "write past row M"
    got = oracle_mod.bf16_to_f32(allc[:M])
    ref = oracle_mod.gemm_f64(A_bits, B_bits)
    ok = oracle_mod.within_tolerance(got, ref)
    assert ok.all(), (np.argwhere(~ok)[:5], oracle_mod.max_scaled_error(got, ref))


@pytest.mark.parametrize("M", [96, 200])
def test_small_m_unsplit_matches_tiled_bitwise(gpu_handle, M):
    """With no K split the small-M kernel sums each element in the same K
    order as the tiled kernel, so the two agree bit for bit."""
    h = gpu_handle
    N, K = 16384, 512
    assert h.small_m_split(M, N, K) == 1
    A, B = data.device_operands(M, N, K, "normal", seed=5)
    C1 = h.bf16_nt(A, B)
    h.set_small_m(0)
    try:
        assert h.small_m_split(M, N, K) == 0
        C2 = h.bf16_nt(A, B)
    finally:
        h.set_small_m(-1)
    torch.cuda.synchronize()
    assert torch.equal(C1.view(torch.int16), C2.view(torch.int16))


def test_decode_config_vs_cublaslt(gpu_handle, oracle_mod):
    """The decode benchmark configuration 128 x 8192 x 8192: every element vs cuBLASLt,
    one full row vs the fp64 oracle."""
    M, N, K = 128, 8192, 8192
    A, B = data.device_operands(M, N, K, "normal", seed=7)
    C = gpu_handle.bf16_nt(A, B)
    torch.backends.cuda.preferred_blas_library("cublaslt")
    R = torch.matmul(A, B.t())
    torch.cuda.synchronize()
    g, r = C.float(), R.float()
    assert bool(((g - r).abs() <= 2.0 ** -7 * (r.abs() + 1.0)).all())
    A_bits, B_bits = _bits(A), _bits(B)
    rows = np.full(N, 77, dtype=np.int32)
    cols = np.arange(N, dtype=np.int32)
    ref = oracle_mod.gemm_sampled(A_bits, B_bits, rows, cols)
    assert oracle_mod.within_tolerance(oracle_mod.bf16_to_f32(_bits(C)[77]), ref).all()
