"""GPU: the NVLink SHARP (multicast) all-gather of the row-sharded GEMM and BASELINE configs[4a].

* vk_gemm_mc through a multicast buffer of this process (vk_mc_alloc): on one GPU the buffer has a
  single member, so the epilogue's multicast stores must reproduce vk_gemm bit for bit; on several
  GPUs vk_gemm_sharded(allgather_c = 4) must leave the full C on every GPU.
* configs[4a] (16384^3, seed 4) against the golden rows of the reference v0: one GPU, and M split
  over every visible GPU with the NCCL and the NVLS gathers.
Skipped where the GPUs have no NVLS multicast (vk_mc_supported).
"""
import os

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


def _mc_or_skip(vk, devices):
    for d in devices:
        if not vk.mc_supported(d):
            pytest.skip(f"device {d} has no NVLS multicast")


@pytest.mark.parametrize("m,n,k", [(1024, 1024, 512), (777, 512, 300), (4096, 4096, 4096)])
def test_mc_single_member_matches_vk_gemm(vk, m, n, k):
    _mc_or_skip(vk, [0])
    A, B = v0.make_inputs(m, n, k, 21)
    dA, dB = torch.from_numpy(A).cuda(0), torch.from_numpy(B).cuda(0)
    ref = vk.gemm(dA, dB)
    try:
        buf = vk.McBuffer([0], m, n, torch.float16)
    except vk.VkError as e:  # the driver may refuse a multicast team of one GPU
        pytest.skip(f"single-member multicast buffer refused: {e}")
    try:
        C = buf.views[0]
        C.fill_(float("nan"))
        for _ in range(2):  # twice: the second call overwrites a complete buffer
            vk.gemm(dA, dB, C, mc=buf.mc)
        torch.cuda.synchronize(0)
        assert vk.device_error(0) == 0
        got = C.cpu().numpy()
    finally:
        buf.free()
    assert np.array_equal(got.view(np.uint16), ref.cpu().numpy().view(np.uint16))
    g16, _ = v0.v0_f16(A, B)
    assert v0.max_elem_rel(got, g16) <= 2e-3


def test_mc_rejects_foreign_c(vk):
    ngpu = torch.cuda.device_count()
    devs = list(range(min(ngpu, 2)))
    _mc_or_skip(vk, devs)
    try:
        buf = vk.McBuffer(devs, 256, 256, torch.float16)
    except vk.VkError as e:
        pytest.skip(f"multicast buffer refused: {e}")
    try:
        A = torch.zeros((256, 64), dtype=torch.float16, device="cuda:0")
        B = torch.zeros((64, 256), dtype=torch.float16, device="cuda:0")
        C = torch.empty((256, 256), dtype=torch.float16, device="cuda:0")  # not in the multicast buffer
        with pytest.raises(vk.VkError):
            vk.gemm(A, B, C, mc=buf.mc)
        with pytest.raises(vk.VkError):  # n not a multiple of 8
            vk.gemm(A, B[:, :250], buf.views[0][:, :250], mc=buf.mc)
    finally:
        buf.free()


@pytest.mark.parametrize("m", [4096, 4001])
def test_sharded_nvls_allgather(vk, m):
    ngpu = torch.cuda.device_count()
    if ngpu < 2:
        pytest.skip("needs >= 2 GPUs")
    _mc_or_skip(vk, range(ngpu))
    n, k = 2048, 1024
    A, B = v0.make_inputs(m, n, k, 4)
    off = vk.row_blocks(m, ngpu)
    buf = vk.McBuffer(list(range(ngpu)), m, n, torch.float16)
    try:
        for r in range(ngpu):
            buf.views[r].fill_(float("nan"))
        A_parts = [torch.from_numpy(A[off[r]:off[r + 1]]).cuda(r) for r in range(ngpu)]
        B_parts = [torch.from_numpy(B).cuda(r) for r in range(ngpu)]
        for _ in range(2):
            tc, tg = vk.gemm_sharded(A_parts, B_parts, buf.views, m, n, k, allgather="nvls")
        got = [buf.views[r].cpu().numpy() for r in range(ngpu)]
    finally:
        buf.free()
    g16, _ = v0.v0_f16(A, B)
    for r in range(ngpu):
        assert not np.isnan(got[r].astype(np.float32)).any(), f"GPU {r} missing rows"
        assert v0.max_elem_rel(got[r], g16) <= 2e-3
        assert np.array_equal(got[r].view(np.uint16), got[0].view(np.uint16))
    assert tc > 0


# ------------------------------------------------------------------------------------------
# BASELINE configs[4a]: 16384^3, seed 4, against the golden rows of the reference v0
# ------------------------------------------------------------------------------------------
@pytest.fixture(scope="module")
def cfg4a():
    from vibekernel_b200 import testdata
    z = np.load(os.path.join(ROOT, "tests", "golden", "cfg4a_16384_seed4.npz"))
    A, B = testdata.make_inputs(16384, 16384, 16384, 4)
    return A, B, z["rows"], z["C"]


def _check_rows(C, rows, gold):
    """fp16 C rows against the fp16 golden rows.  At K = 16384 the tensor cores' fp32 accumulation
    (products aligned and summed with truncation inside each MMA) drifts by up to ~2e-3 absolute, so
    elements near zero exceed the per-element bound of the fp32-accumulate tier (2e-3 relative with
    a floor of 1e-2 RMS); the relative Frobenius error of the fp16 output (dominated by its own
    rounding, 2^-11 relative) is the bound here, with the fp32-copy check in test_cfg4a_one_gpu."""
    got = C[torch.from_numpy(rows).to(C.device)].cpu().numpy()
    assert not np.isnan(got.astype(np.float32)).any()
    assert v0.rel_frobenius(got, gold) <= 1e-3
    assert v0.max_elem_rel(got, gold) <= 1e-2


def test_cfg4a_one_gpu(vk, cfg4a):
    A, B, rows, gold = cfg4a
    dA, dB = torch.from_numpy(A).cuda(0), torch.from_numpy(B).cuda(0)
    C = torch.full((16384, 16384), float("nan"), dtype=torch.float16, device="cuda:0")
    C32 = torch.empty((16384, 16384), dtype=torch.float32, device="cuda:0")
    vk.gemm(dA, dB, C, c_f32=C32)
    torch.cuda.synchronize(0)
    _check_rows(C, rows, gold)
    # fp32-accumulate tier on the fp32 copy: relative Frobenius <= 1e-4 against the reference's fp32
    # sgemm of the same rows (recomputed here from the seeded inputs)
    _, g32 = v0.v0_f16(A[rows], B)
    got32 = C32[torch.from_numpy(rows).cuda(0)].cpu().numpy()
    assert v0.rel_frobenius(got32, g32) <= 1e-4


@pytest.mark.parametrize("mode", [True, "nvls"], ids=["nccl", "nvls"])
def test_cfg4a_sharded(vk, cfg4a, mode):
    ngpu = torch.cuda.device_count()
    if ngpu < 2:
        pytest.skip("needs >= 2 GPUs")
    if mode == "nvls":
        _mc_or_skip(vk, range(ngpu))
    A, B, rows, gold = cfg4a
    m = n = k = 16384
    off = vk.row_blocks(m, ngpu)
    A_parts = [torch.from_numpy(A[off[r]:off[r + 1]]).cuda(r) for r in range(ngpu)]
    B_parts = [torch.from_numpy(B).cuda(r) for r in range(ngpu)]
    buf = vk.McBuffer(list(range(ngpu)), m, n, torch.float16) if mode == "nvls" else None
    try:
        C_parts = buf.views if buf else [torch.empty((m, n), dtype=torch.float16, device=f"cuda:{r}")
                                         for r in range(ngpu)]
        for c in C_parts:
            c.fill_(float("nan"))
        vk.gemm_sharded(A_parts, B_parts, C_parts, m, n, k, allgather=mode)
        for r in range(ngpu):
            _check_rows(C_parts[r], rows, gold)
    finally:
        if buf:
            buf.free()
