"""GPU: the no-allocation entry point vk_gemm_noalloc, called through the C ABI.

It exists for callers that cannot call cudaMalloc (work recorded during CUDA graph capture,
device memory owned by a pool or framework allocator, fixed memory budgets).  Its scratch is a
fixed device array inside the library, so two calls in a row reuse the same array: the second
call must not see stale arrival counters or partials from the first.  Each call is checked
against the ordinary entry point vk_gemm on the same inputs and against the reference v0 (the
oracle), with the tolerances used throughout the GPU tests, and the device's free memory must not
move across calls made after the first one (which may load the library's device code), while an
ordinary vk_gemm visibly allocates its scratch.  The file name makes pytest collect
it last; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import v0  # noqa: E402

FROB, ELEM = 1e-4, 2e-3


@pytest.fixture(scope="module")
def vk():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    import vibekernel_b200 as vkm
    return vkm


def _args(vk, A, B, C, C32, acc):
    a = vk.GemmArgs()
    a.A, a.B, a.C, a.C_f32 = A.data_ptr(), B.data_ptr(), C.data_ptr(), C32.data_ptr()
    a.m, a.n, a.k = A.shape[0], B.shape[1], A.shape[1]
    a.dtype = vk.DTYPE_F16
    a.acc = vk.ACC_F32 if acc == "f32" else vk.ACC_F16
    a.algo = vk.ALGO_AUTO
    a.stream = torch.cuda.current_stream().cuda_stream or None
    return a


# 4096^3 and 1024^3 cut their last wave into k-slices (the path that needs scratch);
# 300 x 200 x 4096 is a single small tile cut into 8 slices.
@pytest.mark.parametrize("shape", [(4096, 4096, 4096), (1024, 1024, 1024), (300, 200, 4096)])
@pytest.mark.parametrize("acc", ["f32", "f16"])
def test_noalloc_matches_vk_gemm_on_two_calls_in_a_row(vk, shape, acc):
    m, n, k = shape
    A, B = v0.make_inputs(m, n, k, 90, lo=-0.5, hi=0.5)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()

    ref = torch.empty((m, n), dtype=torch.float16, device="cuda")
    ref32 = torch.empty((m, n), dtype=torch.float32, device="cuda")
    vk.check(vk.lib.vk_gemm(ctypes.byref(_args(vk, dA, dB, ref, ref32, acc))))

    outs = []
    for _ in range(2):
        C = torch.full((m, n), float("nan"), dtype=torch.float16, device="cuda")
        C32 = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        vk.check(vk.lib.vk_gemm_noalloc(ctypes.byref(_args(vk, dA, dB, C, C32, acc))))
        outs.append((C, C32))
    torch.cuda.synchronize()
    assert vk.device_error(0) == 0

    r32 = ref32.cpu().numpy()
    r16 = ref.cpu().numpy()
    g16, g32 = v0.v0_f16(A, B)  # the reference v0 (fp32 sgemm of the widened inputs)
    for C, C32 in outs:
        c32 = C32.cpu().numpy()
        c16 = C.cpu().numpy()
        assert not np.isnan(c32).any()
        assert v0.rel_frobenius(c32, r32) <= FROB
        assert v0.max_elem_rel(c32, r32) <= ELEM
        assert v0.max_elem_rel(c16, r16) <= ELEM
        if acc == "f32":  # fp32-accumulate tier against the oracle
            assert v0.rel_frobenius(c32, g32) <= FROB
            assert v0.max_elem_rel(c32, g32) <= ELEM
            assert v0.max_elem_rel(c16, g16) <= ELEM
        else:  # fp16-accumulate tier: relative Frobenius against the fp32 v0 result
            assert v0.rel_frobenius(c16, g32) <= 5e-3


def test_noalloc_allocates_nothing(vk):
    """Free device memory stays put across no-allocation calls on a fresh stream whose plan needs
    tail-split scratch, while vk_gemm (after vk_shutdown freed the library's scratch) allocates."""
    m = n = k = 4096  # last wave cut into k-slices: the path that needs scratch
    A, B = v0.make_inputs(m, n, k, 91)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    C = torch.empty((m, n), dtype=torch.float16, device="cuda")
    C32 = torch.empty((m, n), dtype=torch.float32, device="cuda")
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()

    def call(entry, stream):
        a = _args(vk, dA, dB, C, C32, "f32")
        a.stream = stream.cuda_stream
        vk.check(entry(ctypes.byref(a)))

    call(vk.lib.vk_gemm_noalloc, s1)  # the first call may load the library's device code
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        call(vk.lib.vk_gemm_noalloc, s1)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"no-allocation calls changed free device memory by {free0 - free1} bytes"
    g16, g32 = v0.v0_f16(A, B)
    assert v0.rel_frobenius(C32.cpu().numpy(), g32) <= FROB
    # control: after vk_shutdown has freed the library's scratch, the ordinary entry point allocates
    # its tail-split scratch again, and the same measurement sees it
    vk.check(vk.lib.vk_shutdown())
    torch.cuda.synchronize()
    free2, _ = torch.cuda.mem_get_info()
    call(vk.lib.vk_gemm, s2)
    torch.cuda.synchronize()
    free3, _ = torch.cuda.mem_get_info()
    assert free2 - free3 >= 16 << 20, "the measurement would not have seen an allocation"


def test_noalloc_rejects_what_it_cannot_run(vk):
    A = torch.zeros((64, 40), dtype=torch.float16, device="cuda")  # lda = 40 -> 80 bytes: fine
    B = torch.zeros((40, 36), dtype=torch.float16, device="cuda")  # ldb = 36 -> 72 bytes: not TMA-able
    C = torch.empty((64, 36), dtype=torch.float16, device="cuda")
    C32 = torch.empty((64, 36), dtype=torch.float32, device="cuda")
    rc = vk.lib.vk_gemm_noalloc(ctypes.byref(_args(vk, A, B, C, C32, "f32")))
    assert rc == vk.VK_ERR_ALIGNMENT
    a = _args(vk, A, B, C, C32, "f32")
    a.dtype = vk.DTYPE_F32
    assert vk.lib.vk_gemm_noalloc(ctypes.byref(a)) == vk.VK_ERR_UNSUPPORTED
    assert "fp16" in vk.last_error()
