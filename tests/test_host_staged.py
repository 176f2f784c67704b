"""b200gemm_bf16_nt_host: operands and result in host memory, copies pipelined
with the GEMMs by row chunks.  Each output element is computed exactly as
by the device-pointer entry point (same kernel, same K order), so the result
must be bit-identical to it."""
import numpy as np
import pytest

from b200_gemm_b200 import data

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _host(bits, pinned):
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)
    return t.pin_memory() if pinned else t


@pytest.mark.parametrize("M,N,K,pinned", [(2000, 1000, 520, True), (300, 77, 64, True),
                                          (4096, 2048, 1024, True), (700, 300, 136, False)])
def test_host_path_matches_device_path(gpu_handle, M, N, K, pinned):
    A_bits, B_bits = data.host_operands(M, N, K, "normal", seed=M ^ N ^ K)
    hA, hB = _host(A_bits, pinned), _host(B_bits, pinned)
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16).pin_memory()
    gpu_handle.bf16_nt_host(hA, hB, out=out)
    torch.cuda.current_stream().synchronize()
    ref = gpu_handle.bf16_nt(hA.cuda(), hB.cuda())
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref.contiguous().cpu().view(torch.int16))


def test_host_path_twice_and_host_pitch(gpu_handle):
    """Two calls back to back reuse the staging buffers; C written with a
    host pitch wider than N leaves the padding untouched."""
    M, N, K, ldc = 1100, 600, 256, 640
    outs = []
    for seed in (1, 2):
        A_bits, B_bits = data.host_operands(M, N, K, "uniform", seed=seed)
        wide = torch.full((M, ldc), 7.0, dtype=torch.bfloat16).pin_memory()
        gpu_handle.bf16_nt_host(_host(A_bits, True), _host(B_bits, True), out=wide[:, :N])
        outs.append((wide, A_bits, B_bits))
    torch.cuda.current_stream().synchronize()
    for wide, A_bits, B_bits in outs:
        assert torch.all(wide[:, N:] == 7.0)
        ref = gpu_handle.bf16_nt(_host(A_bits, False).cuda(), _host(B_bits, False).cuda())
        torch.cuda.synchronize()
        assert torch.equal(wide[:, :N].contiguous().view(torch.int16), ref.cpu().view(torch.int16))


def test_host_path_interleaved_streams(gpu_handle):
    """Calls alternating between two streams overlap through the two staging
    sets; shapes change mid-sequence (the larger one grows a set while the
    other may still be in flight), and every result matches the device path."""
    shapes = [(1024, 768, 512), (1024, 768, 512), (2304, 1280, 768), (1024, 768, 512), (512, 256, 128),
              (2304, 1280, 768)]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    jobs = []
    for i, (M, N, K) in enumerate(shapes):
        A_bits, B_bits = data.host_operands(M, N, K, "normal", seed=100 + i)
        hA, hB = _host(A_bits, True), _host(B_bits, True)
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16).pin_memory()
        gpu_handle.bf16_nt_host(hA, hB, out=out, stream=streams[i % 2])
        jobs.append((hA, hB, out))
    for s in streams:
        s.synchronize()
    for hA, hB, out in jobs:
        ref = gpu_handle.bf16_nt(hA.cuda(), hB.cuda())
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), ref.cpu().view(torch.int16))


def test_host_path_ragged_vs_oracle(gpu_handle, oracle_mod):
    """A ragged shape (M, N, K not multiples of the tile sizes) through the
    host-buffer path, checked directly against the fp64 CPU oracle on every
    element, |err| <= 2^-7 (|ref| + 1)."""
    M, N, K = 1300, 904, 328
    A_bits, B_bits = data.host_operands(M, N, K, "normal", seed=77)
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16).pin_memory()
    gpu_handle.bf16_nt_host(_host(A_bits, True), _host(B_bits, True), out=out)
    torch.cuda.current_stream().synchronize()
    got = oracle_mod.bf16_to_f32(out.view(torch.int16).numpy().view(np.uint16))
    ref = oracle_mod.gemm_f64(A_bits, B_bits)
    assert not np.isnan(got).any()
    assert oracle_mod.within_tolerance(got, ref).all(), oracle_mod.max_scaled_error(got, ref)
