"""N-sharding host logic on CPU process groups (gloo, world size 2 and 3):
shard ranges, the all-gather + repack of C column shards, max-over-ranks
timing, and a rank that fails between steps.  Each rank's GEMM is a plain
torch fp32 matmul here: these tests cover the distribution logic, not the
kernel."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from b200_gemm_b200 import shard


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("N,world", [(8192, 1), (8192, 2), (16384, 8), (14336, 8), (1000, 3), (300, 4), (0, 2)])
def test_column_shards_partition_n(N, world):
    shards = shard.all_shards(N, world)
    assert shards[0][0] == 0 and shards[-1][1] == N
    for (a0, a1), (b0, b1) in zip(shards, shards[1:]):
        assert a1 == b0
    widths = [b - a for a, b in shards]
    assert all(w >= 0 for w in widths)
    for a, _ in shards:
        assert a % shard.TILE_N == 0 or a == N
    full = [w for (a, b), w in zip(shards, widths) if b != N]
    if full:
        assert max(full) - min(full) <= shard.TILE_N


def test_bad_shard_requests():
    with pytest.raises(ValueError):
        shard.column_shard(100, 0, 0)
    with pytest.raises(ValueError):
        shard.column_shard(100, 2, 2)


def _worker(rank, world, port, M, N, K, fail_rank, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        g = torch.Generator().manual_seed(0)
        A = torch.randn(M, K, generator=g)
        B = torch.randn(N, K, generator=g)
        n0, n1 = shard.column_shard(N, world, rank)
        C_local = A @ B[n0:n1].t()  # this rank's columns only: no communication
        full = shard.allgather_columns(C_local.contiguous(), N)
        ok = torch.allclose(full, A @ B.t(), atol=1e-4, rtol=1e-4)
        t = shard.max_over_ranks(float(rank + 1))
        step2 = None
        if fail_rank is not None:
            # a failure between steps: the failing rank raises before the next
            # collective; the others must see an error, not hang
            if rank == fail_rank:
                raise RuntimeError("injected rank failure")
            try:
                shard.max_over_ranks(1.0)
                step2 = "no-error"
            except Exception:
                step2 = "error"
        q.put((rank, ok, t, step2))
    except RuntimeError as e:
        q.put((rank, "raised", str(e), None))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, M, N, K, fail_rank=None, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, N, K, fail_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r = q.get(timeout=timeout)
        out[r[0]] = r[1:]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("world,M,N,K", [(2, 64, 600, 32), (3, 40, 1000, 16)])
def test_sharded_gemm_allgather_matches_full(world, M, N, K):
    out = _run(world, M, N, K)
    assert set(out) == set(range(world))
    for r, (ok, t, _) in out.items():
        assert ok is True, r
        assert t == float(world)  # max over ranks of (rank + 1)


def test_rank_failure_between_steps_is_reported_not_hung():
    out = _run(2, 32, 512, 16, fail_rank=1, timeout=120)
    assert out[1][0] == "raised"
    assert out[0][2] == "error"


def _host_gemm_worker(rank, world, port, M, N, K, q):
    """One rank of ShardedHostGemm on a CPU process group: it holds only its
    rows of A and its B rows; two calls in a row (both buffer sets)."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        n0, n1 = shard.column_shard(N, world, rank, align=8)
        r0, r1, rows = shard.row_slice(M, world, rank)
        seen_rows = []

        def gemm_fn(A_full, B, C, stream):
            seen_rows.append(A_full.shape[0])
            C.copy_((A_full[:M].float() @ B.float().t()).to(torch.bfloat16))
            return 0

        hg = shard.ShardedHostGemm(M, n1 - n0, K, gemm_fn, "cpu")
        oks = []
        for step in range(2):
            g = torch.Generator().manual_seed(10 + step)
            A = torch.randn(M, K, generator=g).to(torch.bfloat16)
            B = torch.randn(N, K, generator=g).to(torch.bfloat16)
            wide = torch.full((M, n1 - n0 + 8), 7.0, dtype=torch.bfloat16)
            hg.run(A[r0:r1].clone(), B[n0:n1].contiguous(), wide[:, : n1 - n0])
            ref = (A.float() @ B[n0:n1].float().t()).to(torch.bfloat16)
            oks.append(bool(torch.equal(wide[:, : n1 - n0], ref)) and bool(torch.all(wide[:, n1 - n0:] == 7.0)))
        up, down = hg.bytes_per_call()
        q.put((rank, oks, (r0, r1, rows), seen_rows, up, down))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), None, None, None, None))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,M,N,K", [(2, 37, 48, 16), (3, 64, 96, 8), (1, 20, 16, 8)])
def test_sharded_host_gemm_uploads_own_rows_and_gathers_a(world, M, N, K):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_host_gemm_worker, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r = q.get(timeout=120)
        out[r[0]] = r[1:]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    rows = (M + world - 1) // world
    covered = []
    for rank, (oks, sl, seen, up, down) in out.items():
        assert oks == [True, True], (rank, oks)
        r0, r1, rr = sl
        assert rr == rows and r0 == min(M, rank * rows) and r1 == min(M, (rank + 1) * rows)
        covered.extend(range(r0, r1))
        assert seen == [world * rows] * 2
        n0, n1 = shard.column_shard(N, world, rank, align=8)
        assert up == 2 * ((r1 - r0) * K + (n1 - n0) * K) and down == 2 * M * (n1 - n0)
    assert sorted(covered) == list(range(M))  # every row of A is uploaded by exactly one rank
