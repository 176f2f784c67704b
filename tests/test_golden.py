"""Golden fixtures: outputs of the reference project's own kernel
(runKernel1, b200_kernels/matmul_1.cuh, built from its sources and run on a
B200 by tests/golden/make_golden.py).  On the CPU they pin the oracle; on
the GPU they check this library against the reference bit patterns.
Tolerance: |err| <= 2^-7 (|ref| + 1) per element."""
from pathlib import Path

import numpy as np
import pytest

from b200_gemm_b200 import data

GOLDEN = Path(__file__).resolve().parent / "golden"
FIXTURES = sorted(GOLDEN.glob("ref_*.npz"))


def _load(path):
    z = np.load(path)
    M, N, K = int(z["M"]), int(z["N"]), int(z["K"])
    dist, seed = str(z["dist"]), int(z["seed"])
    A, B = data.host_operands(M, N, K, dist, seed)
    return A, B, z["C"]


def test_fixtures_present():
    assert len(FIXTURES) >= 3, "golden fixtures missing; run tests/golden/make_golden.py on a B200"


@pytest.mark.parametrize("path", FIXTURES, ids=[p.stem for p in FIXTURES])
def test_oracle_matches_reference_kernel(oracle_mod, path):
    A, B, C_ref = _load(path)
    ref = oracle_mod.gemm_f64(A, B)
    got = oracle_mod.bf16_to_f32(C_ref)
    assert oracle_mod.within_tolerance(got, ref).all(), oracle_mod.max_scaled_error(got, ref)
    # the reference rounds the same fp32 sums to bf16: nearly every element agrees exactly
    assert np.mean(C_ref == oracle_mod.f64_to_bf16(ref)) > 0.95


@pytest.mark.gpu
@pytest.mark.parametrize("width", [256, 512])
@pytest.mark.parametrize("path", FIXTURES, ids=[p.stem for p in FIXTURES])
def test_kernel_matches_reference_kernel(gpu_handle, oracle_mod, path, width):
    import torch

    A, B, C_ref = _load(path)
    dev = lambda b: torch.from_numpy(b.view(np.int16)).cuda().view(torch.bfloat16)
    gpu_handle.set_tile_width(width)
    try:
        C = gpu_handle.bf16_nt(dev(A), dev(B))
    finally:
        gpu_handle.set_tile_width(0)
    torch.cuda.synchronize()
    got = C.view(torch.int16).cpu().numpy().view(np.uint16)
    ref = oracle_mod.bf16_to_f32(C_ref).astype(np.float64)
    assert oracle_mod.within_tolerance(oracle_mod.bf16_to_f32(got), ref).all()
    # same MMA shape and K order as the reference: the bits agree almost everywhere
    assert np.mean(got == C_ref) > 0.99, np.mean(got == C_ref)
