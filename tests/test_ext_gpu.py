"""GPU: vk_gemm_ex -- transposed operand layouts and the fused epilogue, against the oracle.

op(A), op(B) are formed on the host from the stored matrices; the reference result is the v0
restatement on op(A), op(B), followed by act(alpha * . + beta * C_in + bias) in fp32.
Tolerances as in test_gemm_gpu.py (fp32 copy: rel-Frobenius <= 1e-4, per-element <= 2e-3)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import v0  # noqa: E402

FROB, ELEM = 1e-4, 2e-3
LAYOUTS = [(False, False), (False, True), (True, False), (True, True)]


@pytest.fixture(scope="module")
def vk():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    import vibekernel_b200 as vkm
    return vkm


def _stored(A, B, ta, tb):
    return (np.ascontiguousarray(A.T) if ta else A), (np.ascontiguousarray(B.T) if tb else B)


@pytest.mark.parametrize("ta,tb", LAYOUTS, ids=["NN", "NT", "TN", "TT"])
@pytest.mark.parametrize("algo,tile_n", [("tc2", 256), ("tc1", 256), ("tc2", 128), ("simt", 0)])
@pytest.mark.parametrize("shape", [(512, 768, 384), (200, 136, 72), (1024, 1024, 2048)])
def test_layouts(vk, ta, tb, algo, tile_n, shape):
    m, n, k = shape
    A, B = v0.make_inputs(m, n, k, 60)
    As, Bs = _stored(A, B, ta, tb)
    C32 = torch.empty((m, n), dtype=torch.float32, device="cuda")
    C = vk.gemm(torch.from_numpy(As).cuda(), torch.from_numpy(Bs).cuda(), trans_a=ta, trans_b=tb, algo=algo,
                tile_n=tile_n, c_f32=C32)
    torch.cuda.synchronize()
    g16, g32 = v0.v0_f16(A, B)
    c32 = C32.cpu().numpy()
    assert v0.rel_frobenius(c32, g32) <= FROB
    assert v0.max_elem_rel(c32, g32) <= ELEM
    assert v0.max_elem_rel(C.cpu().numpy(), g16) <= ELEM


@pytest.mark.parametrize("ta,tb", LAYOUTS, ids=["NN", "NT", "TN", "TT"])
def test_layouts_rubric_size_and_f16acc(vk, ta, tb):
    A, B = v0.make_inputs(4096, 4096, 4096, 61, lo=-0.5, hi=0.5)
    As, Bs = _stored(A, B, ta, tb)
    dA, dB = torch.from_numpy(As).cuda(), torch.from_numpy(Bs).cuda()
    C32 = torch.empty((4096, 4096), dtype=torch.float32, device="cuda")
    vk.gemm(dA, dB, trans_a=ta, trans_b=tb, c_f32=C32)
    C16 = vk.gemm(dA, dB, trans_a=ta, trans_b=tb, acc="f16")
    torch.cuda.synchronize()
    g32 = v0.v0_f16(A, B)[1]
    assert v0.rel_frobenius(C32.cpu().numpy(), g32) <= FROB
    assert v0.rel_frobenius(C16.cpu().numpy().astype(np.float32), g32) <= 5e-3


def test_unaligned_transposed_takes_predicated_kernel(vk):
    A, B = v0.make_inputs(37, 29, 21, 62)  # stored A^T: 21 x 37 (ld 37), B^T: 29 x 21 (ld 21)
    As, Bs = _stored(A, B, True, True)
    dA, dB = torch.from_numpy(As).cuda(), torch.from_numpy(Bs).cuda()
    with pytest.raises(vk.VkError):
        vk.gemm(dA, dB, trans_a=True, trans_b=True, algo="tc2")
    C = vk.gemm(dA, dB, trans_a=True, trans_b=True)
    torch.cuda.synchronize()
    assert v0.max_elem_rel(C.cpu().numpy(), v0.v0_f16(A, B)[0]) <= ELEM


def _fused_ref(g32, alpha, beta, cin, bias, act):
    r = alpha * g32.astype(np.float64)
    if beta != 0:
        r = r + beta * cin.astype(np.float64)
    if bias is not None:
        r = r + bias.astype(np.float64)[None, :]
    if act == "relu":
        r = np.maximum(r, 0)
    return r


@pytest.mark.parametrize("algo,tile_n", [("tc2", 256), ("tc1", 128), ("simt", 0)])
@pytest.mark.parametrize("shape", [(1024, 1024, 1024), (4096, 4096, 4096), (300, 264, 136)])
@pytest.mark.parametrize("opts", [dict(alpha=0.5), dict(beta=1.5), dict(bias=True), dict(act="relu"),
                                  dict(alpha=-2.0, beta=0.25, bias=True, act="relu")],
                         ids=["alpha", "beta", "bias", "relu", "all"])
def test_fused_epilogue_fp16(vk, algo, tile_n, shape, opts):
    m, n, k = shape
    A, B = v0.make_inputs(m, n, k, 63)
    rng = np.random.default_rng(64)
    cin = rng.uniform(-4, 4, size=(m, n)).astype(np.float16)
    bias = rng.uniform(-8, 8, size=(n,)).astype(np.float16) if opts.get("bias") else None
    alpha, beta, act = opts.get("alpha", 1.0), opts.get("beta", 0.0), opts.get("act")
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    C = torch.from_numpy(cin.copy()).cuda()  # in place: C_in is C
    C32 = torch.empty((m, n), dtype=torch.float32, device="cuda")
    vk.gemm(dA, dB, C, algo=algo, tile_n=tile_n, alpha=alpha, beta=beta, c_in=C if beta else None,
            bias=torch.from_numpy(bias).cuda() if bias is not None else None, act=act, c_f32=C32)
    torch.cuda.synchronize()
    ref = _fused_ref(v0.v0_f16(A, B)[1], alpha, beta, cin, bias, act)
    c32 = C32.cpu().numpy()
    assert v0.rel_frobenius(c32, ref) <= FROB
    assert v0.max_elem_rel(c32, ref) <= ELEM
    # The fp16 output is compared with one more fp16 ulp (2^-10) of slack: after cancellation
    # (alpha * A@B and bias of opposite sign) the GEMM's fp32 summation error plus two independent
    # roundings to fp16 can reach two ulps of a small result; the fp32 copy above keeps the 2e-3 bound.
    assert v0.max_elem_rel(C.cpu().numpy(), ref.astype(np.float16)) <= ELEM + 2.0 ** -10


@pytest.mark.parametrize("shape", [(1000, 1000, 1000), (300, 200, 20), (130, 131, 17)])
def test_fused_epilogue_fp32(vk, shape):
    m, n, k = shape
    A, B = v0.make_inputs(m, n, k, 65, dist="normal", dtype=np.float32)
    rng = np.random.default_rng(66)
    cin = rng.standard_normal((m, n)).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    C = torch.from_numpy(cin.copy()).cuda()
    vk.gemm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), C, alpha=0.75, beta=-1.25, c_in=C,
            bias=torch.from_numpy(bias).cuda(), act="relu")
    torch.cuda.synchronize()
    ref = _fused_ref(v0.v0_f32(A, B), 0.75, -1.25, cin, bias, "relu")
    assert v0.rel_frobenius(C.cpu().numpy(), ref) <= 1e-5


def test_fused_k_zero_and_fp32_transpose_rejected(vk):
    m, n = 64, 96
    cin = torch.full((m, n), 2.0, dtype=torch.float16, device="cuda")
    bias = torch.full((n,), -3.0, dtype=torch.float16, device="cuda")
    A = torch.empty((m, 0), dtype=torch.float16, device="cuda")
    B = torch.empty((0, n), dtype=torch.float16, device="cuda")
    C = vk.gemm(A, B, k=0, beta=2.0, c_in=cin, bias=bias)
    torch.cuda.synchronize()
    assert torch.all(C == 1.0)  # 2 * 2 - 3
    A32 = torch.zeros((8, 8), dtype=torch.float32, device="cuda")
    with pytest.raises(vk.VkError):
        vk.gemm(A32, A32, trans_a=True)
