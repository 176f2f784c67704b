"""CUDA graph capture of the library's calls: after one ordinary call per
shape (which builds the tile schedule and waits for it once), the same call
is captured into a graph on a side stream and replayed; every replay writes
exactly what the direct call wrote.  Covers the tiled kernel (two widths),
both small-M kernels and the fused epilogue."""
import pytest

from b200_gemm_b200 import data

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

# (M, N, K, plan kernel)
SHAPES = [(2048, 3072, 1024, "tiled"), (4096, 4096, 512, "tiled"), (128, 8192, 1024, "small_m"),
          (128, 4096, 1024, "small_m_1cta")]


@pytest.mark.parametrize("M,N,K,kernel", SHAPES)
@pytest.mark.parametrize("fused", [False, True], ids=["plain", "bias_gelu"])
def test_capture_and_replay_bit_exact(gpu_handle, M, N, K, kernel, fused):
    h = gpu_handle
    assert h.plan(M, N, K)["kernel"] == kernel
    A, B = data.device_operands(M, N, K, "normal", seed=M + N + K)
    bias = torch.randn(N, device="cuda").to(torch.bfloat16)

    def call(out):
        if fused:
            return h.bf16_nt_epilogue(A, B, bias=bias, activation="gelu_tanh", out=out)
        return h.bf16_nt(A, B, out=out)

    ref = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    call(ref)  # first call: schedule built and tensor maps cached outside the capture
    torch.cuda.synchronize()
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            call(out)
    torch.cuda.synchronize()
    for _ in range(3):
        out.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    assert h.last_device_status()[0] == 0
    del graph
