"""CPU: the collective set-up and teardown of dist_gemm.McRowGather (the NVLS all-gather of C, one process
per GPU) on gloo ranks, with a fake multicast driver standing in for libvkgemm's vk_mc_* calls.

What must hold, whatever the GPU: a refused multicast object (creation on the owner, or import on any
other rank) is reported to every rank at the same point as McSetupRefused, so that all ranks can fall back
together; the owner releases what it created; a failed attach releases that member's share before
raising; and a normal run detaches every member exactly once, after a barrier."""
import ctypes
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


class FakeMc:
    """vk_mc_create / vk_mc_import / vk_mc_attach / vk_mc_detach with scripted failures."""

    def __init__(self, rank, fail):
        self.rank, self.fail, self.detached = rank, fail, 0

    def vk_mc_create(self, dev, members, nbytes, team_ref, share):
        if self.fail == "create":
            return -3
        team_ref._obj.value = 0x100
        share[0], share[1], share[2] = 4242, 7, nbytes
        return 0

    def vk_mc_import(self, dev, members, share, team_ref):
        if self.fail == "import" and self.rank == 1:
            return -3
        assert share[0] == 4242 and share[1] == 7
        team_ref._obj.value = 0x200 + self.rank
        return 0

    def vk_mc_attach(self, team, local_ref, mc_ref, size_ref):
        if self.fail == "attach":
            return -3
        local_ref._obj.value, mc_ref._obj.value, size_ref._obj.value = 0x1000, 0x2000, 1 << 20
        return 0

    def vk_mc_detach(self, team):
        self.detached += 1
        return 0


def _worker(rank, world, port, fail, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import vibekernel_b200 as vk
    from vibekernel_b200 import dist_gemm
    fake = FakeMc(rank, fail)
    vk.lib = fake
    vk.last_error = lambda: "scripted failure"
    vk._view = lambda ptr, shape, dtype, device: torch.zeros(shape, dtype=torch.float32)
    torch.cuda.current_device = lambda: 0
    torch.cuda.synchronize = lambda *a, **k: None
    outcome = "ok"
    try:
        m, n = 8, 4
        off = vk.row_blocks(m, world)
        try:
            g = dist_gemm.McRowGather(m, n, off, rank, dtype=torch.float32)
        except dist_gemm.McSetupRefused:
            outcome = "refused"
        except RuntimeError:
            outcome = "attach_failed"
        else:
            calls = []
            for _ in range(2):
                g.run(None, None, lambda a, b, out, mc=None: calls.append((out.shape[0], mc)))
            g.close()
            g.close()  # a second close is a no-op
            lo = off[rank]
            assert calls == [(off[rank + 1] - lo, 0x2000 + lo * n * 4)] * 2
        q.put((rank, outcome, fake.detached))
    finally:
        dist.destroy_process_group()


def _run(world, port, fail):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.start_processes(_worker, args=(world, port, fail, q), nprocs=world, join=True, start_method="spawn")
    return sorted(q.get(timeout=60) for _ in range(world))


def test_normal_setup_runs_and_detaches_every_member_once():
    assert _run(2, 29811, None) == [(0, "ok", 1), (1, "ok", 1)]


def test_refused_creation_reaches_every_rank():
    # the owner never created anything, so nothing is released
    assert _run(2, 29812, "create") == [(0, "refused", 0), (1, "refused", 0)]


def test_refused_import_reaches_every_rank_and_the_owner_releases_its_object():
    assert _run(2, 29813, "import") == [(0, "refused", 1), (1, "refused", 0)]


def test_failed_attach_releases_the_member_before_raising():
    # one member (an attach failure on several ranks would leave the others in the driver's bind)
    assert _run(1, 29814, "attach") == [(0, "attach_failed", 1)]
