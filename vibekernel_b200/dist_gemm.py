"""Row-block sharding of C = A * B across the ranks of a torch.distributed group.

One process per GPU.  Rank r owns rows [off[r], off[r+1]) of A and C (``row_blocks``) and a full
copy of B; there is no exchange on the data path.  The only collective is the optional
all-gather of the C row blocks (NCCL over NVLink on B200; gloo in the CPU tests), in place in a
full [m, n] buffer on every rank: C is row-major, so each rank's block is one contiguous span.
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
