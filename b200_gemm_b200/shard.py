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


class FusedAllGather:
    """Full-width C on every rank, filled by one fused GEMM + all-gather.

    Each rank allocates its own M x N C (row pitch rounded up to 8 elements),
    shares it with the other ranks through CUDA IPC (handles exchanged with
    one all_gather_object on the process group) and then calls
    b200gemm_bf16_nt_allgather, whose epilogue writes every finished chunk of
    this rank's column block into its own C and into every peer's C over
    NVLink.  After `run` the caller's stream holds the completed writes; a
    barrier among the ranks makes all blocks visible everywhere.
    """

    def __init__(self, gemm, M: int, N: int, group=None):
        import ctypes

        import torch
        import torch.distributed as dist

        from . import _lib

        self._lib = _lib.load()
        self.gemm = gemm
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world - 1 > 7:
            raise ValueError("the fused all-gather writes to at most 7 peers")
        self.M, self.N = M, N
        self.pitch = 8 * ((N + 7) // 8)
        self.n0, self.n1 = column_shard(N, self.world, self.rank)
        if (self.n1 - self.n0) % 8 != 0:
            raise ValueError("every column shard must be a multiple of 8 columns")
        dev = torch.device("cuda", gemm.device)
        self.C = torch.empty(M, self.pitch, dtype=torch.bfloat16, device=dev)
        handle = (ctypes.c_char * 64)()
        offset = ctypes.c_ulonglong()
        _lib.check(self._lib.b200gemm_ipc_get_handle(self.C.data_ptr(), handle, ctypes.byref(offset)),
                   "b200gemm_ipc_get_handle")
        mine = (bytes(handle), int(offset.value))
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mine, group=group)
        self._opened = []
        self.peer_bases = []
        for r, (hbytes, off) in enumerate(everyone):
            if r == self.rank:
                continue
            base = ctypes.c_void_p()
            buf = (ctypes.c_char * 64).from_buffer_copy(hbytes)
            _lib.check(self._lib.b200gemm_ipc_open(buf, ctypes.byref(base)), "b200gemm_ipc_open")
            self._opened.append(base.value)
            self.peer_bases.append(base.value + off)

    def run(self, A, B_local, stream_ptr: int) -> int:
        """C[:, n0:n1] = A @ B_local^T on every rank's C; returns the status."""
        import ctypes

        off = self.n0 * 2
        peers = (ctypes.c_void_p * max(1, len(self.peer_bases)))(*[b + off for b in self.peer_bases])
        K = A.shape[1]
        return self._lib.b200gemm_bf16_nt_allgather(
            self.gemm._h, self.M, self.n1 - self.n0, K, A.data_ptr(), B_local.data_ptr(),
            self.C.data_ptr() + off, self.pitch, peers, len(self.peer_bases), stream_ptr)

    def view(self):
        return self.C[:, : self.N]

    def close(self) -> None:
        for base in self._opened:
            self._lib.b200gemm_ipc_close(base)
        self._opened = []
