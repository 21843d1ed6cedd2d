"""CPU: the row-block sharding logic on 2 gloo ranks (the oracle stands in for the GPU kernel)."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import v0
from vibekernel_b200 import dist_gemm, row_blocks


def test_row_blocks_cover_and_balance():
    for m in (0, 1, 7, 4096, 16384, 4001):
        for p in (1, 2, 3, 4, 8):
            off = row_blocks(m, p)
            assert off[0] == 0 and off[-1] == m
            sizes = [off[i + 1] - off[i] for i in range(p)]
            assert max(sizes) - min(sizes) <= 1


def _oracle_gemm(A, B, out):
    out.copy_(torch.from_numpy(v0.v0_f16(A.numpy(), B.numpy())[0]))


def _worker(rank, world, port, m, n, k, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        A, B = v0.make_inputs(m, n, k, 3)
        off = row_blocks(m, world)
        C = torch.zeros((m, n), dtype=torch.float16)
        dist_gemm.sharded_matmul(torch.from_numpy(A[off[rank]:off[rank + 1]]), torch.from_numpy(B), C, off,
                                 rank, _oracle_gemm)
        ref = v0.v0_f16(A, B)[0]
        q.put((rank, bool(np.array_equal(C.numpy().view(np.uint16), ref.view(np.uint16)))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("rows,chunks", [(2048, 2), (2001, 2), (100, 4), (0, 2), (1000, 3), (4096, 1), (256, 8)])
def test_chunk_rows_cover_aligned(rows, chunks):
    from vibekernel_b200 import dist_gemm
    parts = dist_gemm.chunk_rows(rows, chunks)
    assert len(parts) <= max(chunks, 1)
    covered = [r for a, b in parts for r in range(a, b)]
    assert covered == list(range(rows))
    assert all(a % 256 == 0 for a, _ in parts)


@pytest.mark.parametrize("m,world", [(4096, 2), (2001, 2), (16384, 8), (1000, 3)])
def test_push_plan_writes_each_rank_rows_to_every_peer(m, world):
    """Union over ranks of the planned peer copies = every row of C on every rank except the rows the
    rank computes itself, each exactly once."""
    from vibekernel_b200 import dist_gemm, row_blocks
    off = row_blocks(m, world)
    row_bytes = 3
    received = {p: [] for p in range(world)}
    for r in range(world):
        for (r0, r1), copies in dist_gemm.push_plan(off, r, 2, row_bytes):
            assert [p for p, _, _ in copies] == [p for p in range(world) if p != r]
            for p, start, nbytes in copies:
                assert start == (off[r] + r0) * row_bytes and nbytes == (r1 - r0) * row_bytes
                received[p].extend(range(start // row_bytes, (start + nbytes) // row_bytes))
    for p in range(world):
        assert sorted(received[p]) == [i for i in range(m) if not off[p] <= i < off[p + 1]]


@pytest.mark.parametrize("m", [64, 67])  # even split (all-gather) and uneven split (broadcasts)
def test_two_rank_gloo_sharded_matmul(m):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + m
    procs = [ctx.Process(target=_worker, args=(r, 2, port, m, 48, 40, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}


def _failing_worker(rank, world, port, q):
    """Rank 1 dies before the all-gather; rank 0 must see an error, not hang."""
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    A, B = v0.make_inputs(64, 48, 40, 3)
    off = row_blocks(64, world)
    C = torch.zeros((64, 48), dtype=torch.float16)
    if rank == 1:
        os._exit(3)  # a rank that disappears between steps, without a clean shutdown
    try:
        dist_gemm.sharded_matmul(torch.from_numpy(A[off[rank]:off[rank + 1]]), torch.from_numpy(B), C, off, rank,
                                 _oracle_gemm)
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001 - the error type depends on how gloo notices the loss
        q.put((rank, "error: " + type(e).__name__))


def test_rank_loss_is_detected_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, 29577, q)) for r in range(2)]
    for p in procs:
        p.start()
    rank0, msg = q.get(timeout=60)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert procs[1].exitcode == 3
    assert rank0 == 0 and msg.startswith("error"), msg
