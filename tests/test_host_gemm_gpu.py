"""GPU: vk_gemm_host -- C = A * B for host-resident A, B, C with the copies pipelined in row blocks."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import v0  # noqa: E402

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def vk():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    import vibekernel_b200 as vkm
    return vkm


def _pinned(a):
    t = torch.from_numpy(a).pin_memory()
    return t


def test_rubric_pinned_matches_reference_v0(vk):
    z = np.load(os.path.join(GOLD, "cfg1_4096_seed1.npz"))
    A, B = v0.make_inputs(4096, 4096, 4096, 1)
    C = torch.empty((4096, 4096), dtype=torch.float16).pin_memory()
    vk.gemm_host(_pinned(A), _pinned(B), C)
    c = C.numpy()
    assert v0.max_elem_rel(c[z["rows"]], z["C"]) <= 2e-3
    g16, _ = v0.v0_f16(A, B)
    assert v0.max_elem_rel(c, g16) <= 2e-3


@pytest.mark.parametrize("block_rows", [0, 1, 100, 1000, 5000])
def test_ragged_pageable_blocks(vk, block_rows):
    z = np.load(os.path.join(GOLD, "cfg5_ragged_4000x5120x3000_seed5.npz"))
    A, B = v0.make_inputs(4000, 5120, 3000, 5)
    c = vk.gemm_host(A, B, block_rows=block_rows)
    assert v0.max_elem_rel(c[z["rows"]], z["C"]) <= 2e-3


def test_f16acc_and_sgemm(vk):
    A, B = v0.make_inputs(1024, 768, 2048, 2, lo=-0.5, hi=0.5)
    c = vk.gemm_host(A, B, acc="f16")
    assert v0.rel_frobenius(c.astype(np.float32), v0.v0_f16(A, B)[1]) <= 5e-3
    A32, B32 = v0.make_inputs(1000, 520, 300, 3, dist="normal", dtype=np.float32)
    c32 = vk.gemm_host(A32, B32)
    assert v0.rel_frobenius(c32, v0.v0_f32(A32, B32)) <= 1e-5


def test_strided_host_operands_and_k_zero(vk):
    A, B = v0.make_inputs(300, 200, 136, 8)
    Abig = np.zeros((300, 200), dtype=np.float16)
    Abig[:, :136] = A
    Cbig = np.full((300, 264), 7, dtype=np.float16)
    vk.gemm_host(Abig[:, :136], B, Cbig[:, :200])
    assert v0.max_elem_rel(Cbig[:, :200], v0.v0_f16(A, B)[0]) <= 2e-3
    assert np.all(Cbig[:, 200:] == 7)
    Z = vk.gemm_host(np.zeros((64, 0), np.float16), np.zeros((0, 32), np.float16))
    assert Z.shape == (64, 32) and not Z.any()
