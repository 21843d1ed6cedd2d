"""torchrun worker for tests/test_sharded_gpu.py: one process per GPU, NCCL all-gather of C, the
copy-engine gather overlapped with the GEMM (dist_gemm.PeerRowGather), the fused peer stores and the
NVLS multicast gather (dist_gemm.McRowGather, where the GPUs support it).

  --big: BASELINE configs[4a] (16384^3, seed 4) with the NCCL and NVLS gathers, every rank's full C
         checked at the golden rows of the reference v0."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import vibekernel_b200 as vk  # noqa: E402
from oracle import v0  # noqa: E402
from vibekernel_b200 import dist_gemm  # noqa: E402


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
    flags = [None] * world
    dist.all_gather_object(flags, vk.mc_supported(local))
    nvls = all(flags)
    if "--big" in sys.argv:
        ok = big(rank, world, dev, nvls)
        finish(ok, rank, dev)
        return
    ok = True
    for m in (2048, 2001):
        A, B = v0.make_inputs(m, 1536, 768, 4)
        off = vk.row_blocks(m, world)
        C = torch.full((m, 1536), float("nan"), dtype=torch.float16, device=dev)
        dist_gemm.sharded_matmul(torch.from_numpy(A[off[rank]:off[rank + 1]]).to(dev), torch.from_numpy(B).to(dev),
                                 C, off, rank, lambda a, b, out: vk.gemm(a, b, out))
        torch.cuda.synchronize(dev)
        g16, _ = v0.v0_f16(A, B)
        c = C.cpu().numpy()
        ok = ok and not np.isnan(c.astype(np.float32)).any() and v0.max_elem_rel(c, g16) <= 2e-3
        # copy-engine gather overlapped with the GEMM (chunks may take another tail split: tolerance)
        C2 = torch.full((m, 1536), float("nan"), dtype=torch.float16, device=dev)
        pg = dist_gemm.PeerRowGather(C2, off, rank)
        for _ in range(2):  # twice: the second run overwrites a complete buffer
            pg.run(torch.from_numpy(A[off[rank]:off[rank + 1]]).to(dev), torch.from_numpy(B).to(dev),
                   lambda a, b, out: vk.gemm(a, b, out), chunks=2)
        torch.cuda.synchronize(dev)
        pg.close()
        c2 = C2.cpu().numpy()
        ok = ok and not np.isnan(c2.astype(np.float32)).any() and v0.max_elem_rel(c2, g16) <= 2e-3
        # fused: the GEMM epilogue stores into the peers' C itself (same kernel plan as the NCCL run)
        C3 = torch.full((m, 1536), float("nan"), dtype=torch.float16, device=dev)
        pg = dist_gemm.PeerRowGather(C3, off, rank)
        for _ in range(2):
            pg.run(torch.from_numpy(A[off[rank]:off[rank + 1]]).to(dev), torch.from_numpy(B).to(dev),
                   lambda a, b, out, peers=None: vk.gemm(a, b, out, peers=peers), mode="fused")
        torch.cuda.synchronize(dev)
        pg.close()
        c3 = C3.cpu().numpy()
        ok = ok and np.array_equal(c3.view(np.uint16), c.view(np.uint16))
        if nvls:
            # NVLS: every box stored once to the multicast view; same kernel plan, so bitwise equal
            mg = dist_gemm.McRowGather(m, 1536, off, rank)
            try:
                mg.C_full.fill_(float("nan"))
                torch.cuda.synchronize(dev)
                dist.barrier()  # every rank's buffer is filled before anyone stores into it
                for _ in range(2):
                    mg.run(torch.from_numpy(A[off[rank]:off[rank + 1]]).to(dev), torch.from_numpy(B).to(dev),
                           lambda a, b, out, mc=None: vk.gemm(a, b, out, mc=mc))
                torch.cuda.synchronize(dev)
                c4 = mg.C_full.cpu().numpy()
            finally:
                mg.close()
            ok = ok and np.array_equal(c4.view(np.uint16), c.view(np.uint16))
    finish(ok, rank, dev)


def big(rank, world, dev, nvls):
    """configs[4a]: 16384^3 split over the ranks, C all-gathered, golden rows checked on every rank."""
    from vibekernel_b200 import testdata
    z = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "cfg4a_16384_seed4.npz"))
    rows, gold = z["rows"], z["C"]
    m = n = k = 16384
    off = vk.row_blocks(m, world)
    hA, hB = testdata.make_inputs(m, n, k, 4, a_rows=(off[rank], off[rank + 1]))
    A, B = torch.from_numpy(hA).to(dev), torch.from_numpy(hB).to(dev)
    idx = torch.from_numpy(rows).to(dev)

    def good(C):
        got = C[idx].cpu().numpy()
        # K = 16384: relative Frobenius of the fp16 output (see tests/test_nvls_gpu.py::_check_rows)
        return (not np.isnan(got.astype(np.float32)).any() and v0.rel_frobenius(got, gold) <= 1e-3
                and v0.max_elem_rel(got, gold) <= 1e-2)

    C = torch.full((m, n), float("nan"), dtype=torch.float16, device=dev)
    dist_gemm.sharded_matmul(A, B, C, off, rank, lambda a, b, out: vk.gemm(a, b, out))
    torch.cuda.synchronize(dev)
    ok = good(C)
    del C
    if nvls:
        mg = dist_gemm.McRowGather(m, n, off, rank)
        try:
            mg.C_full.fill_(float("nan"))
            torch.cuda.synchronize(dev)
            dist.barrier()
            mg.run(A, B, lambda a, b, out, mc=None: vk.gemm(a, b, out, mc=mc))
            torch.cuda.synchronize(dev)
            ok = ok and good(mg.C_full)
        finally:
            mg.close()
    if rank == 0:
        print(f"big: nvls={'on' if nvls else 'off (no multicast)'}", flush=True)
    return ok


def finish(ok, rank, dev):
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    if rank == 0:
        print("rank0 ok" if flag.item() == 1 else "rank0 FAIL", flush=True)
    sys.exit(0 if flag.item() == 1 else 1)


if __name__ == "__main__":
    main()
