"""K split of the last, partial wave of tiles: the tail tiles' K slices run on
otherwise idle clusters, write fp32 partials, and the last slice of each
half-tile adds them up and stores C.  Checked against cuBLASLt on every
element and the fp64 oracle on sampled elements (|err| <= 2^-7 (|ref| + 1)),
twice in a row (the tickets reset themselves), and against the unsplit
kernel."""
import numpy as np
import pytest

from b200_gemm_b200 import data

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _close(got, ref):
    g, r = got.float(), ref.float()
    return bool(((g - r).abs() <= 2.0 ** -7 * (r.abs() + 1.0)).all())


# (M, N, K, tile width): last waves of 26, 4 and 8 tiles on 74 clusters
# (the 512-wide instance carries no K-split tail)
CASES = [(2560, 2560, 512, 256), (16384, 1792, 1024, 256), (16384, 1792, 2048, 128)]


@pytest.mark.parametrize("M,N,K,width", CASES)
def test_tail_split_parity(gpu_handle, oracle_mod, M, N, K, width):
    h = gpu_handle
    h.set_tile_width(width)
    h.set_tail_split(True)
    plan = h.plan(M, N, K)
    assert plan["kernel"] == "tiled" and plan["tile_width"] == width
    assert plan["tiles"] % plan["clusters"] != 0 and plan["tail_split"] >= 2, plan
    try:
        A, B = data.device_operands(M, N, K, "normal", seed=M + N + K)
        C1 = h.bf16_nt(A, B)
        C2 = h.bf16_nt(A, B)  # second launch: tickets were reset by the first
        h.set_tail_split(False)
        C0 = h.bf16_nt(A, B)
        h.set_tail_split(True)
    finally:
        h.set_tile_width(0)
        h.set_tail_split(False)
    torch.backends.cuda.preferred_blas_library("cublaslt")
    R = torch.matmul(A, B.t())
    torch.cuda.synchronize()
    assert h.last_device_status()[0] == 0
    assert torch.equal(C1.view(torch.int16), C2.view(torch.int16))
    assert _close(C1, R) and _close(C0, R)
    assert _close(C1, C0)
    # the tail tiles are the last in the schedule; check a full row and column too
    A_bits, B_bits = _bits(A), _bits(B)
    rng = np.random.Generator(np.random.PCG64(3))
    rows = np.concatenate([rng.integers(0, M, 2048), np.full(N, M - 1), np.arange(M)])
    cols = np.concatenate([rng.integers(0, N, 2048), np.arange(N), np.full(M, N - 1)])
    ref = oracle_mod.gemm_sampled(A_bits, B_bits, rows, cols)
    got = oracle_mod.bf16_to_f32(_bits(C1)[rows, cols])
    assert oracle_mod.within_tolerance(got, ref).all()


def test_no_tail_split_at_width_512(gpu_handle):
    """The 256 x 512 instance carries no K-split tail: its short last wave is
    cut into 256-column halves instead (b200gemm_set_tail_half), or not at all."""
    h = gpu_handle
    h.set_tile_width(512)
    h.set_tail_split(True)
    try:
        plan_halves = h.plan(16384, 2048, 2048)
        h.set_tail_half(False)
        plan_none = h.plan(16384, 2048, 2048)
    finally:
        h.set_tile_width(0)
        h.set_tail_split(False)
        h.set_tail_half(True)
    assert plan_halves["tile_width"] == 512 and plan_halves["tail_split"] == -2
    assert plan_none["tile_width"] == 512 and plan_none["tail_split"] == 1
