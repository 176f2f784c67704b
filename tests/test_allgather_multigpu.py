"""Fused GEMM + all-gather across GPUs (b200gemm_bf16_nt_allgather): every
rank computes its column block of C and its epilogue writes the block into
every rank's full-width C over NVLink.  After a barrier each rank's C must
equal, bit for bit, the single-GPU result of the whole GEMM with the tiled
kernel (the kernel the all-gather entry points run: same per-element K
order).  Needs two or more GPUs; one process per GPU."""
import os
import socket

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _tiled_reference(gemm, A, B):
    """The whole GEMM on one GPU with the tiled kernel (small-M kernel off)."""
    gemm.set_small_m(0)
    try:
        full = gemm.bf16_nt(A, B)
        torch.cuda.synchronize()
    finally:
        gemm.set_small_m(-1)
    return full


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, M, N, K, width, q):
    import datetime

    import torch.distributed as dist

    from b200_gemm_b200 import Gemm, data, shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))
    try:
        gemm = Gemm(rank)
        if width:
            gemm.set_tile_width(width)
        A, B = data.device_operands(M, N, K, "normal", seed=11, device=f"cuda:{rank}")
        fused = shard.FusedAllGather(gemm, M, N)
        n0, n1 = fused.n0, fused.n1
        B_local = B[n0:n1].contiguous()
        fused.C.fill_(float("nan"))
        torch.cuda.synchronize()
        dist.barrier()
        rc = fused.run(A, B_local, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        dist.barrier()
        full = _tiled_reference(gemm, A, B)
        same = bool(torch.equal(fused.view().contiguous().view(torch.int16), full.contiguous().view(torch.int16)))
        if same and rank == 0 and M * N * K <= 600 * 1536 * 264:
            # the gathered C of a ragged shape, directly against the fp64 oracle
            import numpy as np

            from oracle import oracle

            bits = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
            got = oracle.bf16_to_f32(bits(fused.view()))
            same = bool(oracle.within_tolerance(got, oracle.gemm_f64(bits(A), bits(B))).all())
        status = gemm.last_device_status()[0]
        dist.barrier()
        fused.close()
        gemm.close()
        q.put((rank, rc, same, status))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, -1, repr(e), -1))
    finally:
        dist.destroy_process_group()


# width 512 on these shapes puts every rank's few 256 x 512 tiles in one short
# wave, which runs as 256-column halves whose epilogue also writes the peers.
@pytest.mark.parametrize("M,N,K,width", [(1024, 2048, 512, 0), (600, 1536, 264, 0), (1024, 2048, 512, 512)])
def test_fused_allgather_matches_single_gpu(M, N, K, width):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least two GPUs")
    world = min(n, 8)
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, N, K, width, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r = q.get(timeout=300)
        results[r[0]] = r[1:]
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    for rank, (rc, same, status) in results.items():
        assert rc == 0, (rank, rc, same)
        assert same is True, (rank, same)
        assert status == 0, (rank, status)


def _mc_worker(rank, world, port, M, N, K, q):
    """The multicast form: every rank's C is one symmetric-memory buffer bound
    to an NVLink multicast object; torn down collectively in every outcome."""
    import datetime

    import torch.distributed as dist

    from b200_gemm_b200 import Gemm, data, shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))
    gemm = Gemm(rank)
    fused = None
    try:
        A, B = data.device_operands(M, N, K, "normal", seed=13, device=f"cuda:{rank}")
        full = _tiled_reference(gemm, A, B)
        try:
            fused = shard.MulticastAllGather(gemm, M, N)
        except RuntimeError as e:
            q.put((rank, "unsupported", str(e), 0))
            return
        B_local = B[fused.n0:fused.n1].contiguous()
        fused.C.fill_(float("nan"))
        torch.cuda.synchronize()
        dist.barrier()
        rcs = []
        for _ in range(2):  # twice: the second call rewrites every block
            rcs.append(fused.run(A, B_local, torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        dist.barrier()
        same = bool(torch.equal(fused.view().contiguous().view(torch.int16), full.contiguous().view(torch.int16)))
        status = gemm.last_device_status()[0]
        q.put((rank, max(rcs), same, status))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, -1, repr(e), -1))
    finally:
        if fused is not None:
            fused.close()
        gemm.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("M,N,K", [(1024, 2048, 512), (600, 1536, 264)])
def test_multicast_allgather_matches_single_gpu(M, N, K):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least two GPUs")
    world = min(n, 8)
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_mc_worker, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r = q.get(timeout=300)
        results[r[0]] = r[1:]
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    if all(v[0] == "unsupported" for v in results.values()):
        pytest.skip(f"no NVLink multicast on this node: {next(iter(results.values()))[1]}")
    for rank, (rc, same, status) in results.items():
        assert rc == 0, (rank, rc, same)
        assert same is True, (rank, same)
        assert status == 0, (rank, status)
