"""Half-width last wave of 256 x 512 tiles: when the last wave holds at most
half as many tiles as there are clusters, each of its tiles runs as two
256-column halves over the whole of K.  Every element is summed in the same K
order as in a whole tile, so the result must equal the run without halves
bit for bit, and match the fp64 oracle on sampled elements."""
import numpy as np
import pytest

from b200_gemm_b200 import data

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


# (width, M, N, K).  256 x 512: 256 tiles (a last wave of 34 on 74
# clusters); 16 tiles (one partial wave, all halves); ragged 36 tiles whose
# last column is cut at N.  256 x 448 (halves of 224 columns): 256 tiles of
# the 8-way MLP shard width N = 1792; 20 tiles (all halves); ragged M and N,
# 36 tiles.
CASES = [(512, 16384, 2048, 1024), (512, 512, 4096, 512), (512, 3000, 1496, 264),
         (448, 16384, 1792, 1024), (448, 512, 4480, 512), (448, 3000, 1304, 264)]


@pytest.mark.parametrize("width,M,N,K", CASES)
def test_half_tail_bit_exact_and_oracle(gpu_handle, oracle_mod, width, M, N, K):
    h = gpu_handle
    h.set_tile_width(width)
    try:
        h.set_tail_half(False)
        plan0 = h.plan(M, N, K)
        h.set_tail_half(True)
        plan1 = h.plan(M, N, K)
        assert plan1["tile_width"] == width and plan1["tiles"] == plan0["tiles"]
        assert (plan0["tail_split"], plan1["tail_split"]) == (1, -2), (plan0, plan1)
        assert plan1["clusters"] >= plan0["clusters"], (plan0, plan1)
        A, B = data.device_operands(M, N, K, "normal", seed=M + N + K)
        C1 = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        h.bf16_nt(A, B, out=C1)
        h.set_tail_half(False)
        C0 = h.bf16_nt(A, B)
    finally:
        h.set_tail_half(True)
        h.set_tile_width(0)
    torch.cuda.synchronize()
    assert h.last_device_status()[0] == 0
    assert torch.equal(C1.view(torch.int16), C0.view(torch.int16))
    A_bits, B_bits = _bits(A), _bits(B)
    rng = np.random.Generator(np.random.PCG64(11))
    rows = np.concatenate([rng.integers(0, M, 2048), np.full(N, M - 1), np.arange(M)])
    cols = np.concatenate([rng.integers(0, N, 2048), np.arange(N), np.full(M, N - 1)])
    ref = oracle_mod.gemm_sampled(A_bits, B_bits, rows, cols)
    got = oracle_mod.bf16_to_f32(_bits(C1)[rows, cols])
    assert oracle_mod.within_tolerance(got, ref).all()
