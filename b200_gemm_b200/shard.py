"""N-sharding of the GEMM across the GPUs of one node (one process per GPU).

C = A . B^T splits along N into independent column blocks: rank r holds all
of A, rows [n0, n1) of B and computes C[:, n0:n1].  No data crosses GPUs on
the compute path.  Gathering C afterwards is optional and separate:
`allgather_columns` runs one NCCL all-gather of the shards (shard-major
[world][M][n_r]) and repacks it into a row-major M x N matrix.

The reference has no multi-GPU code; this module is the host logic for the
N-sharded configurations of the benchmark (16384^3 over 1/2/4/8 GPUs, the
MLP shape over 8 GPUs).
"""
from __future__ import annotations

TILE_N = 256  # shard boundaries fall on kernel tile boundaries


def column_shard(N: int, world: int, rank: int, align: int = TILE_N) -> tuple[int, int]:
    """[n0, n1) columns of C (rows of B) owned by `rank`.  Boundaries are
    multiples of `align` (except the global end), sizes differ by at most one
    `align` unit."""
    if world < 1 or not (0 <= rank < world) or N < 0 or align < 1:
        raise ValueError(f"bad shard request N={N} world={world} rank={rank} align={align}")
    units = (N + align - 1) // align
    u0 = units * rank // world
    u1 = units * (rank + 1) // world
    return min(N, u0 * align), min(N, u1 * align)


def all_shards(N: int, world: int, align: int = TILE_N):
    return [column_shard(N, world, r, align) for r in range(world)]


def allgather_columns(c_local, N: int, group=None):
    """All-gather the C column shards of every rank into a row-major M x N
    tensor (torch).  Shards may differ in width; they are padded to the
    widest for the collective and trimmed in the repack."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    M, n_local = c_local.shape
    shards = all_shards(N, world)
    width = max(n1 - n0 for n0, n1 in shards)
    send = c_local
    if n_local != width:
        send = torch.zeros(M, width, dtype=c_local.dtype, device=c_local.device)
        send[:, :n_local] = c_local
    out = torch.empty(world * M * width, dtype=c_local.dtype, device=c_local.device)
    dist.all_gather_into_tensor(out, send.contiguous().view(-1), group=group)
    blocks = out.view(world, M, width)
    full = torch.empty(M, N, dtype=c_local.dtype, device=c_local.device)
    for r, (n0, n1) in enumerate(shards):
        full[:, n0:n1] = blocks[r, :, : n1 - n0]
    return full


def max_over_ranks(value: float, device=None, group=None) -> float:
    """Maximum of a per-rank float (e.g. elapsed ms) over the group."""
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
