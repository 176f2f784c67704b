"""Programmatic dependent launch (b200gemm_set_pdl): small-M and tiled kernels.

A chain of decode-shaped GEMMs where every call reads the previous call's
output: X[i+1] = gelu_tanh(X[i] . W[i]^T + bias) + X[i] (the residual is the
previous output too).  With launch overlap on, each kernel may start while the
previous one runs, so any read of X before griddepcontrol.wait would see stale
data; every intermediate must equal the chain run without overlap, bit for
bit, eagerly and replayed from a CUDA graph."""
import pytest

from b200_gemm_b200 import _lib

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

MODES = [_lib.PDL_ON, _lib.PDL_WEIGHTS_EARLY]
# (M, K = N, plan kernel): the pair kernel, the single-CTA kernel, the tiled
# kernel, the pair kernel covering 256 rows of A, the pair kernel over two
# 256-row blocks of A
CHAINS = [(128, 8192, "small_m"), (96, 4096, "small_m_1cta"), (1024, 4096, "tiled"), (256, 4096, "small_m"),
          (512, 4096, "small_m")]
STEPS = 6


def _chain(h, X0, Ws, bias, outs, fused=True):
    x = X0
    for W, out in zip(Ws, outs):
        if fused:
            h.bf16_nt_epilogue(x, W, bias=bias, activation="gelu_tanh", residual=x, out=out)
        else:
            h.bf16_nt(x, W, out=out)
        x = out
    return outs


@pytest.fixture
def chain_operands():
    def make(M, K):
        g = torch.Generator(device="cuda").manual_seed(M + K)
        X0 = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
        Ws = [(torch.randn(K, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16) for _ in range(STEPS)]
        bias = (0.1 * torch.randn(K, device="cuda", generator=g)).to(torch.bfloat16)
        return X0, Ws, bias
    return make


@pytest.mark.parametrize("M,K,kernel", CHAINS)
@pytest.mark.parametrize("mode", MODES, ids=["on", "weights_early"])
@pytest.mark.parametrize("fused", [True, False], ids=["bias_gelu_residual", "plain"])
def test_dependent_chain_matches_serial(gpu_handle, chain_operands, M, K, kernel, mode, fused):
    h = gpu_handle
    assert h.plan(M, K, K)["kernel"] == kernel
    X0, Ws, bias = chain_operands(M, K)
    ref = [torch.empty(M, K, dtype=torch.bfloat16, device="cuda") for _ in range(STEPS)]
    _chain(h, X0, Ws, bias, ref, fused)
    torch.cuda.synchronize()
    h.set_pdl(mode)
    try:
        for _ in range(3):
            outs = [torch.full((M, K), float("nan"), dtype=torch.bfloat16, device="cuda") for _ in range(STEPS)]
            _chain(h, X0, Ws, bias, outs, fused)
            torch.cuda.synchronize()
            for r, o in zip(ref, outs):
                assert torch.equal(r.view(torch.int16), o.view(torch.int16))
    finally:
        h.set_pdl(_lib.PDL_OFF)
    assert h.last_device_status()[0] == 0


@pytest.mark.parametrize("mode", MODES, ids=["on", "weights_early"])
@pytest.mark.parametrize("chain", [0, 2], ids=["small_m", "tiled"])
def test_dependent_chain_in_cuda_graph(gpu_handle, chain_operands, mode, chain):
    h = gpu_handle
    M, K, _ = CHAINS[chain]
    X0, Ws, bias = chain_operands(M, K)
    ref = [torch.empty(M, K, dtype=torch.bfloat16, device="cuda") for _ in range(STEPS)]
    _chain(h, X0, Ws, bias, ref)
    torch.cuda.synchronize()
    outs = [torch.empty(M, K, dtype=torch.bfloat16, device="cuda") for _ in range(STEPS)]
    h.set_pdl(mode)
    try:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph, stream=side):
                _chain(h, X0, Ws, bias, outs)
        torch.cuda.synchronize()
        for _ in range(3):
            for o in outs:
                o.fill_(float("nan"))
            graph.replay()
            torch.cuda.synchronize()
            for r, o in zip(ref, outs):
                assert torch.equal(r.view(torch.int16), o.view(torch.int16))
        del graph
    finally:
        h.set_pdl(_lib.PDL_OFF)
    assert h.last_device_status()[0] == 0


def test_set_pdl_rejects_unknown_mode(gpu_handle):
    with pytest.raises(Exception):
        gpu_handle.set_pdl(3)
    with pytest.raises(Exception):
        gpu_handle.set_pdl(-1)
