"""N-sharding of the GEMM across the GPUs of one node (one process per GPU).

C = A . B^T splits along N into independent column blocks: rank r holds all
of A, rows [n0, n1) of B and computes C[:, n0:n1].  No data crosses GPUs on
the compute path.  Gathering C afterwards is optional:
  * `allgather_columns`: one NCCL all-gather of the shards (shard-major
    [world][M][n_r]), repacked into a row-major M x N matrix;
  * `FusedAllGather`: the GEMM's epilogue writes each finished chunk into
    every peer's full-width C over NVLink (CUDA IPC mappings);
  * `MulticastAllGather`: the same through one NVLink multicast mapping of
    every rank's C (NVSwitch replicates each store).
With operands in host memory, `ShardedHostGemm` has each rank upload only
its share of A's rows (plus its B rows) and gathers the rest of A over
NVLink, so the host link carries A once per node.

The reference has no multi-GPU code; this module is the host logic for the
N-sharded configurations of the benchmark (16384^3 over 1/2/4/8 GPUs, the
MLP shape over 8 GPUs).
"""
from __future__ import annotations

import contextlib
import os

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


class MulticastAllGather:
    """Full-width C on every rank, filled by one fused GEMM + all-gather that
    writes through an NVLink multicast (NVLS) mapping.

    C is allocated from torch's symmetric memory and rendezvoused over the
    process group (plumbing only: torch creates the multicast object, binds
    every rank's C to it and exchanges the handles).  `run` calls
    b200gemm_bf16_nt_allgather_multicast, whose epilogue writes each finished
    chunk of this rank's column block once, with multimem.st, to the
    multicast address; NVSwitch replicates it into every rank's C.  After
    `run` the caller's stream holds the completed writes; a barrier among
    the ranks makes all blocks visible everywhere.

    Raises RuntimeError when the node offers no multicast mapping.  `close`
    is collective (a barrier, then the buffer is released on every rank):
    no rank may drop its buffer while others can still write to it.
    """

    def __init__(self, gemm, M: int, N: int, group=None):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        from . import _lib

        self._lib = _lib.load()
        self.gemm = gemm
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.M, self.N = M, N
        self.pitch = 8 * ((N + 7) // 8)
        self.n0, self.n1 = column_shard(N, self.world, self.rank)
        if (self.n1 - self.n0) % 8 != 0:
            raise ValueError("every column shard must be a multiple of 8 columns")
        dev = torch.device("cuda", gemm.device)
        self.C = symm_mem.empty(M, self.pitch, dtype=torch.bfloat16, device=dev)
        self._hdl = symm_mem.rendezvous(self.C, self.group)
        mc = int(self._hdl.multicast_ptr or 0)
        if mc == 0:
            self.close()
            raise RuntimeError("no NVLink multicast mapping on this node (symmetric memory reports none)")
        # The multicast range mirrors the rank's buffer; C sits at the same
        # offset in both.
        self.mc_base = mc + (self.C.data_ptr() - int(self._hdl.buffer_ptrs[self.rank]))

    def run(self, A, B_local, stream_ptr: int) -> int:
        """C[:, n0:n1] = A @ B_local^T on every rank's C; returns the status."""
        off = self.n0 * 2
        K = A.shape[1]
        return self._lib.b200gemm_bf16_nt_allgather_multicast(
            self.gemm._h, self.M, self.n1 - self.n0, K, A.data_ptr(), B_local.data_ptr(),
            self.C.data_ptr() + off, self.pitch, self.mc_base + off, stream_ptr)

    def view(self):
        return self.C[:, : self.N]

    def close(self) -> None:
        import torch
        import torch.distributed as dist

        if getattr(self, "C", None) is None:
            return
        torch.cuda.synchronize(self.C.device)
        dist.barrier(group=self.group)
        self._hdl = None
        self.C = None
        torch.cuda.synchronize()


def row_slice(M: int, world: int, rank: int) -> tuple[int, int, int]:
    """(r0, r1, rows): the rows [r0, r1) of A that `rank` uploads from host
    memory when every rank needs all of A, and the per-rank slot height
    rows = ceil(M / world) of the all-gather (the last slots may be short
    or empty; the gathered buffer has world * rows rows, of which the first
    M are A)."""
    if world < 1 or not (0 <= rank < world) or M < 0:
        raise ValueError(f"bad row slice request M={M} world={world} rank={rank}")
    rows = (M + world - 1) // world
    return min(M, rank * rows), min(M, (rank + 1) * rows), rows


def gpu_local_cpus(device: int):
    """The host CPUs NVML reports as close to `device` (its NUMA node),
    restricted to the CPUs this process may run on; None when unknown."""
    try:
        import pynvml
        import torch

        props = torch.cuda.get_device_properties(device)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        words = pynvml.nvmlDeviceGetCpuAffinity(h, ((os.cpu_count() or 64) + 63) // 64)
        cpus = {64 * i + b for i, w in enumerate(words) for b in range(64) if (int(w) >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        return cpus or None
    except Exception:
        return None


def bind_to_gpu_numa_node(device: int) -> list[int] | None:
    """Run this process on the CPUs next to `device`, so that pinned host
    buffers allocated afterwards sit in that NUMA node's memory and host <->
    device copies do not cross the inter-socket link.  Returns the CPU list,
    or None (nothing changed) when NVML cannot tell."""
    cpus = gpu_local_cpus(device)
    if cpus is None:
        return None
    os.sched_setaffinity(0, cpus)
    return sorted(cpus)


class ShardedHostGemm:
    """One rank of an N-sharded GEMM with host-resident operands:
    C_local = A . B_local^T, where every rank needs all of A (M x K) but holds
    only its rows [r0, r1) of it in host memory (`row_slice`).

    Each `run` copies this rank's rows of A and its B rows from host memory,
    gathers the other ranks' rows of A over NVLink with one all-gather of
    the process group (in place, in rank order), runs the GEMM on the device
    and copies C_local back to host memory.  The host link therefore carries
    A once per node instead of once per GPU.

    Two sets of device buffers alternate between consecutive calls: a call
    issued on another stream uploads while the previous call's GEMM and
    copy-out still run; a set is reused only after the call two back has
    finished with it.  `gemm_fn(A_full, B, C, stream)` runs the GEMM on
    device tensors (A_full has world * rows rows, of which the first M are A)
    and returns a status code (0 = OK).  With device "cpu" (tests on CPU
    process groups) there are no streams or events."""

    def __init__(self, M: int, N_local: int, K: int, gemm_fn, device, group=None):
        import torch
        import torch.distributed as dist

        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.group = group
        self.M, self.N_local, self.K = M, N_local, K
        self.r0, self.r1, self.rows = row_slice(M, self.world, self.rank)
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self._gemm = gemm_fn
        self._sets = []
        for _ in range(2):
            self._sets.append({
                "A": torch.empty(self.world * self.rows, K, dtype=torch.bfloat16, device=self.device),
                "B": torch.empty(N_local, K, dtype=torch.bfloat16, device=self.device),
                "C": torch.empty(M, N_local, dtype=torch.bfloat16, device=self.device),
                "done": torch.cuda.Event() if self.cuda else None,
                "used": False,
            })
        self._next = 0

    def bytes_per_call(self) -> tuple[int, int]:
        """(host -> device, device -> host) bytes one call moves on this rank."""
        return 2 * ((self.r1 - self.r0) * self.K + self.N_local * self.K), 2 * self.M * self.N_local

    def run(self, hA_rows, hB_local, hC_local, stream=None) -> None:
        """hA_rows: host bf16 [r1 - r0, K] (this rank's rows of A); hB_local:
        host bf16 [N_local, K]; hC_local: host bf16 [M, N_local] view (row
        stride may exceed N_local).  Pinned host memory lets the copies run
        asynchronously; completion is ordered on `stream` (default: the
        current stream)."""
        import torch
        import torch.distributed as dist

        if tuple(hA_rows.shape) != (self.r1 - self.r0, self.K):
            raise ValueError(f"hA_rows must be rows [{self.r0}, {self.r1}) of A: got {tuple(hA_rows.shape)}")
        if tuple(hB_local.shape) != (self.N_local, self.K) or tuple(hC_local.shape) != (self.M, self.N_local):
            raise ValueError("hB_local / hC_local shape mismatch")
        s = self._sets[self._next]
        self._next ^= 1
        if self.cuda:
            stream = stream if stream is not None else torch.cuda.current_stream(self.device)
            ctx = torch.cuda.stream(stream)
        else:
            ctx = contextlib.nullcontext()
        with ctx:
            if self.cuda and s["used"]:
                stream.wait_event(s["done"])  # the call two back is done with this set
            slot = s["A"][self.rank * self.rows:(self.rank + 1) * self.rows]
            slot[: self.r1 - self.r0].copy_(hA_rows, non_blocking=True)
            s["B"].copy_(hB_local, non_blocking=True)
            if self.world > 1:
                dist.all_gather_into_tensor(s["A"].view(-1), slot.reshape(-1), group=self.group)
            rc = self._gemm(s["A"], s["B"], s["C"], stream)
            if rc != 0:
                raise RuntimeError(f"sharded host GEMM: status {rc}")
            hC_local.copy_(s["C"], non_blocking=True)
            if self.cuda:
                s["done"].record(stream)
        s["used"] = True


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
