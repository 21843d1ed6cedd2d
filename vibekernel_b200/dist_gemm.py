"""Row-block sharding of C = A * B across the ranks of a torch.distributed group.

One process per GPU.  Rank r owns rows [off[r], off[r+1]) of A and C (``row_blocks``) and a full
copy of B; there is no exchange on the data path.  The only collective is the optional
all-gather of the C row blocks, in place in a full [m, n] buffer on every rank: C is row-major,
so each rank's block is one contiguous span.  Two ways:
  * ``allgather_rows``: NCCL (over NVLink on B200; gloo in the CPU tests) after the GEMM;
  * ``PeerRowGather``: overlapped with the GEMM.  Every rank maps the peers' C buffers into its
    process once (CUDA IPC).  Mode "pipelined": it computes its rows in chunks and, as each chunk
    finishes, pushes it into every peer's C with the copy engines (no SMs taken from the GEMM)
    while the next chunk is computed.  Mode "fused": one GEMM whose epilogue stores every finished
    box of C into the peers' C as well (vk_gemm_peers, plain stores over NVLink).  Either way a
    one-element all-reduce at the end completes on every rank only after every rank's stores have;
  * ``McRowGather``: NVLink SHARP.  C_full is one multicast buffer over all ranks (each rank's view
    is its own memory); the GEMM epilogue stores every finished box once to the multicast view of
    its rows (vk_gemm_mc) and the NVSwitch writes it into every rank's C_full.
The reference has no multi-GPU path (README.md:161); this is the layer BASELINE.json asks for.
"""
from __future__ import annotations

from . import row_blocks  # noqa: F401  (re-exported: the split used here and by vk_gemm_sharded)


def allgather_rows(C_full, off, rank: int, group=None) -> None:
    """In-place all-gather of row blocks C_full[off[r]:off[r+1]] from every rank r."""
    import torch.distributed as dist
    world = len(off) - 1
    sizes = {off[r + 1] - off[r] for r in range(world)}
    if len(sizes) == 1:
        dist.all_gather_into_tensor(C_full, C_full[off[rank]:off[rank + 1]], group=group)
    else:
        for root in range(world):
            if off[root + 1] > off[root]:
                dist.broadcast(C_full[off[root]:off[root + 1]], src=root, group=group)


def chunk_rows(rows: int, chunks: int, align: int = 256):
    """Splits a block of ``rows`` rows into at most ``chunks`` pieces [(r0, r1), ...] whose
    boundaries are multiples of ``align`` rows (one pair tile), the last piece taking the rest."""
    if rows <= 0:
        return []
    step = -(-rows // max(chunks, 1))
    step = -(-step // align) * align
    return [(r0, min(r0 + step, rows)) for r0 in range(0, rows, step)]


def push_plan(off, rank: int, chunks: int, row_bytes: int):
    """The copies rank ``rank`` issues after each chunk: [(chunk_rows, [(peer, byte_offset, nbytes), ...])].
    The byte offset is the same in the local and in every peer's full C buffer."""
    world = len(off) - 1
    plan = []
    for r0, r1 in chunk_rows(off[rank + 1] - off[rank], chunks):
        start = (off[rank] + r0) * row_bytes
        plan.append(((r0, r1), [(p, start, (r1 - r0) * row_bytes) for p in range(world) if p != rank]))
    return plan


class PeerRowGather:
    """Copy-engine all-gather of C row blocks overlapped with the GEMM (one process per GPU).

    Collective: every rank constructs it with the same ``off`` (exchanges IPC handles of the full C
    buffers), calls ``run`` the same number of times and ``close`` once.  ``C_full`` must be a
    contiguous [m, n] device tensor that stays allocated until ``close``.
    """

    def __init__(self, C_full, off, rank: int, group=None):
        import torch
        import torch.distributed as dist
        from . import ipc_export, ipc_import
        if not C_full.is_contiguous():
            raise ValueError("C_full must be contiguous")
        self.C_full, self.off, self.rank, self.group = C_full, list(off), rank, group
        world = len(off) - 1
        handles = [None] * world
        dist.all_gather_object(handles, ipc_export(C_full), group=group)
        self.peers = {p: ipc_import(handles[p]) for p in range(world) if p != rank}
        dev = C_full.device
        self.streams = {p: torch.cuda.Stream(device=dev) for p in self.peers}  # one copy queue per peer
        self.flag = torch.zeros(1, dtype=torch.float32, device=dev)

    def run(self, A_local, B, gemm, chunks: int = 2, mode: str = "pipelined"):
        """Mode "pipelined": ``gemm(A_rows, B, C_rows)`` on each chunk of this rank's rows, each
        finished chunk pushed to every peer while the next one is computed.  Mode "fused": one
        ``gemm(A_local, B, C_rows, peers=[...])`` whose epilogue stores into the peers' C itself.
        Returns when (stream order) every rank's C_full is complete."""
        import torch
        import torch.distributed as dist
        from . import copy_async
        C = self.C_full
        row_bytes = C.stride(0) * C.element_size()
        base = C.data_ptr()
        compute = torch.cuda.current_stream(C.device)
        if mode == "fused":
            lo, hi = self.off[self.rank], self.off[self.rank + 1]
            if hi > lo:
                gemm(A_local, B, C[lo:hi], peers=[self.peers[p] + lo * row_bytes for p in sorted(self.peers)])
            dist.all_reduce(self.flag, group=self.group)
            return C
        if mode != "pipelined":
            raise ValueError(f"unknown mode {mode!r}")
        for (r0, r1), copies in push_plan(self.off, self.rank, chunks, row_bytes):
            lo = self.off[self.rank]
            gemm(A_local[r0:r1], B, C[lo + r0:lo + r1])
            ev = torch.cuda.Event()
            ev.record(compute)
            for p, start, nbytes in copies:
                self.streams[p].wait_event(ev)
                copy_async(self.peers[p] + start, base + start, nbytes, self.streams[p])
        for st in self.streams.values():
            done = torch.cuda.Event()
            done.record(st)
            compute.wait_event(done)
        dist.all_reduce(self.flag, group=self.group)
        return C

    def close(self) -> None:
        import torch
        from . import ipc_release
        torch.cuda.synchronize(self.C_full.device)
        for ptr in self.peers.values():
            ipc_release(ptr)
        self.peers = {}


class McSetupRefused(RuntimeError):
    """The multicast object could not be created or imported; raised on every rank together."""


class McRowGather:
    """All-gather of C row blocks fused into the GEMM through an NVLS multicast buffer (one process
    per GPU, NVSwitch systems: ``vibekernel_b200.mc_supported``).

    Collective: every rank constructs it with the same (m, n, off), calls ``run`` the same number of
    times and ``close`` exactly once (also on error paths), because a rank must not leave while its
    memory is bound to the multicast object and the others may still store into it.  ``C_full`` is
    this rank's view, a [m, n] tensor in its own memory.
    """

    def __init__(self, m: int, n: int, off, rank: int, dtype=None, group=None):
        import ctypes

        import torch
        import torch.distributed as dist

        from . import _view, lib
        dtype = dtype or torch.float16
        self.off, self.rank, self.group = list(off), rank, group
        world = len(off) - 1
        dev = torch.cuda.current_device()
        esize = torch.tensor([], dtype=dtype).element_size()
        team = ctypes.c_void_p()
        share = (ctypes.c_int64 * 3)()
        status = ""
        if rank == 0:
            rc = lib.vk_mc_create(dev, world, m * n * esize, ctypes.byref(team), share)
            status = "" if rc == 0 else f"rank 0: {_err_text(rc)}"
        obj = [(status, list(share))]
        dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group else 0, group=group)
        status, shared = obj[0]
        if not status and rank != 0:
            rc = lib.vk_mc_import(dev, world, (ctypes.c_int64 * 3)(*shared), ctypes.byref(team))
            status = "" if rc == 0 else f"rank {rank}: {_err_text(rc)}"
        # every member must have the object before any member binds memory (binding waits for all)
        statuses = [None] * world
        dist.all_gather_object(statuses, status, group=group)
        failed = [s for s in statuses if s]
        if failed:
            if team.value:
                lib.vk_mc_detach(team)
            raise McSetupRefused("multicast buffer setup failed: " + "; ".join(failed))
        local, mc, size = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_size_t()
        rc = lib.vk_mc_attach(team, ctypes.byref(local), ctypes.byref(mc), ctypes.byref(size))
        if rc != 0:
            msg = _err_text(rc)
            lib.vk_mc_detach(team)  # releases this member's share; nothing of it stays bound
            raise RuntimeError(f"multicast buffer attach failed on rank {rank}: {msg}")
        dist.barrier(group=group)  # every member bound before anyone stores through the multicast view
        self._team = team
        self.mc = int(mc.value)
        self.row_bytes = n * esize
        self.C_full = _view(local.value, (m, n), dtype, torch.device("cuda", dev))
        self.flag = torch.zeros(1, dtype=torch.float32, device=self.C_full.device)

    def run(self, A_local, B, gemm):
        """``gemm(A_local, B, C_rows, mc=...)`` for this rank's rows; returns (stream order) once every
        rank's C_full is complete."""
        import torch.distributed as dist
        lo, hi = self.off[self.rank], self.off[self.rank + 1]
        if hi > lo:
            gemm(A_local, B, self.C_full[lo:hi], mc=self.mc + lo * self.row_bytes)
        dist.all_reduce(self.flag, group=self.group)
        return self.C_full

    def close(self) -> None:
        import torch
        import torch.distributed as dist

        from . import check, lib
        if self._team is None:
            return
        torch.cuda.synchronize(self.C_full.device)
        dist.barrier(group=self.group)  # nobody stores into or reads the buffer any more
        self.C_full = None
        team, self._team = self._team, None
        check(lib.vk_mc_detach(team))
        dist.barrier(group=self.group)  # nobody leaves while another member is still bound


def _err_text(rc: int) -> str:
    from . import last_error
    return f"vkgemm error {rc}: {last_error()}"


def sharded_matmul(A_local, B, C_full, off, rank: int, gemm, allgather: bool = True, group=None):
    """Compute this rank's rows with ``gemm(A_local, B, out)`` then (optionally) all-gather C.

    ``gemm`` is ``vibekernel_b200.gemm`` on a GPU; the CPU tests pass the oracle instead.
    """
    block = C_full[off[rank]:off[rank + 1]]
    if block.shape[0] > 0:
        gemm(A_local, B, block)
    if allgather:
        allgather_rows(C_full, off, rank, group)
    return C_full
