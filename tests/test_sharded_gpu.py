"""GPU: the row-block sharding layer against the oracle.

* vk_gemm_sharded (single process, all visible GPUs, NCCL all-gather of C) -- needs >= 2 GPUs
  for the collective; with one GPU the ngpu = 1 path (no exchange) is still exercised.
* one process per GPU (torchrun): vibekernel_b200.dist_gemm.sharded_matmul with the CUDA kernel
  and torch.distributed NCCL all-gather, run by tests/_dist_gpu_worker.py.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import v0  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def vk():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    import vibekernel_b200 as vkm
    return vkm


def _sharded(vk, ngpu, m, n, k, allgather):
    A, B = v0.make_inputs(m, n, k, 4)
    off = vk.row_blocks(m, ngpu)
    A_parts = [torch.from_numpy(A[off[r]:off[r + 1]]).cuda(r) for r in range(ngpu)]
    B_parts = [torch.from_numpy(B).cuda(r) for r in range(ngpu)]
    C_parts = [torch.full((m, n), float("nan"), dtype=torch.float16, device=f"cuda:{r}") for r in range(ngpu)]
    t_compute, t_gather = vk.gemm_sharded(A_parts, B_parts, C_parts, m, n, k, allgather=allgather)
    g16, g32 = v0.v0_f16(A, B)
    return C_parts, off, g16, g32, t_compute, t_gather


def test_sharded_single_gpu_no_exchange(vk):
    C_parts, off, g16, g32, tc, tg = _sharded(vk, 1, 1000, 768, 512, allgather=False)
    c = C_parts[0].cpu().numpy()
    assert v0.max_elem_rel(c, g16) <= 2e-3
    assert tc > 0 and tg == 0


@pytest.mark.parametrize("m", [4096, 4001])  # even split (ncclAllGather) / uneven (broadcasts)
@pytest.mark.parametrize("mode", [True, "pipelined", "fused"], ids=["nccl", "pipelined", "fused"])  # nvls: test_nvls_gpu.py
def test_sharded_multi_gpu_allgather(vk, m, mode):
    ngpu = torch.cuda.device_count()
    if ngpu < 2:
        pytest.skip("needs >= 2 GPUs")
    C_parts, off, g16, g32, tc, tg = _sharded(vk, ngpu, m, 2048, 1024, allgather=mode)
    for r in range(ngpu):
        c = C_parts[r].cpu().numpy()
        assert not np.isnan(c.astype(np.float32)).any(), f"GPU {r} missing rows after the all-gather"
        assert v0.max_elem_rel(c, g16) <= 2e-3
    assert tg > 0


def test_sharded_multi_gpu_local_blocks_only(vk):
    ngpu = torch.cuda.device_count()
    if ngpu < 2:
        pytest.skip("needs >= 2 GPUs")
    m = 2048
    C_parts, off, g16, g32, tc, tg = _sharded(vk, ngpu, m, 1024, 1024, allgather=False)
    for r in range(ngpu):
        c = C_parts[r].cpu().numpy()
        blk = c[off[r]:off[r + 1]]
        assert v0.max_elem_rel(blk, g16[off[r]:off[r + 1]]) <= 2e-3
        outside = np.delete(c, np.s_[off[r]:off[r + 1]], axis=0)
        assert np.isnan(outside.astype(np.float32)).all(), "a GPU wrote outside its row block"


@pytest.mark.parametrize("big", [False, True], ids=["shapes", "cfg4a_16384"])
def test_torchrun_all_gpus(vk, big):
    """One rank per visible GPU: every gather mode (NCCL, copy engines, fused peer stores, NVLS), and
    BASELINE configs[4a] at full size."""
    ngpu = torch.cuda.device_count()
    if ngpu < 2:
        pytest.skip("needs >= 2 GPUs")
    env = dict(os.environ, PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "30", "420", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(ngpu), "--master-addr", "127.0.0.1", "--master-port", "29731" if big else "29733",
           os.path.join(ROOT, "tests", "_dist_gpu_worker.py")] + (["--big"] if big else [])
    res = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
    assert "rank0 ok" in res.stdout
