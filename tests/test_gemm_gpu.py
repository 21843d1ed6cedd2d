"""GPU parity: the sm_100a kernels, called through the C ABI, against the oracle.

Tolerances (never tuned per kernel):
  fp32-accumulate tier : rel-Frobenius(C32, v0 fp32) <= 1e-4 and per-element
                         |C32 - GT| / max(|GT|, tau) <= 2e-3, tau = 1e-2 * RMS(GT)
                         (the fp32 copy is used: fp16 output rounding alone is ~2e-4 Frobenius)
  fp16 output          : per-element (same tau) <= 2e-3 against the reference's fp16 v0 output
  fp16-accumulate tier : rel-Frobenius <= 5e-3 against the fp32 v0 result
  fp32 SGEMM           : rel-Frobenius <= 1e-5, per-element <= 2e-3
"""
import glob
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import v0  # noqa: E402

GOLD_DIR = os.path.join(os.path.dirname(__file__), "golden")
FROB_F32ACC, ELEM, FROB_F16ACC, FROB_SGEMM = 1e-4, 2e-3, 5e-3, 1e-5


@pytest.fixture(scope="module")
def vk():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    import vibekernel_b200 as vkm
    vkm.check(vkm.lib.vk_init(0))
    return vkm


def _golden(name):
    z = np.load(os.path.join(GOLD_DIR, name + ".npz"))
    dt = np.float16 if str(z["dtype"]) == "f16" else np.float32
    A, B = v0.make_inputs(int(z["m"]), int(z["n"]), int(z["k"]), int(z["seed"]), str(z["dist"]),
                          float(z["lo"]), float(z["hi"]), dt)
    return z, A, B


def _run16(vk, A, B, algo="auto", acc="f32", tile_n=0):
    dA = torch.from_numpy(A).cuda()
    dB = torch.from_numpy(B).cuda()
    m, n = A.shape[0], B.shape[1]
    C = torch.full((m, n), float("nan"), dtype=torch.float16, device="cuda")
    C32 = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    vk.gemm(dA, dB, C, acc=acc, algo=algo, c_f32=C32, tile_n=tile_n)
    torch.cuda.synchronize()
    assert vk.device_error(0) == 0
    return C.cpu().numpy(), C32.cpu().numpy()


def _check_f32acc(c16, c32, A, B, gold=None, rows=None):
    assert not np.isnan(c32).any() and not np.isnan(c16.astype(np.float32)).any()
    g16, g32 = v0.v0_f16(A, B)
    assert v0.rel_frobenius(c32, g32) <= FROB_F32ACC
    assert v0.max_elem_rel(c32, g32) <= ELEM
    assert v0.max_elem_rel(c16, g16) <= ELEM
    if gold is not None:
        assert v0.max_elem_rel(c16[rows], gold) <= ELEM


TC_VARIANTS = [("tc2", 256), ("tc2", 128), ("tc1", 256), ("tc1", 128)]


def test_device_is_sm100_and_library_loaded(vk):
    """The library is built for sm_100a only: the GPU under test is compute capability 10.0, and the
    library's own entry point (not a torch fallback) computes C."""
    assert torch.cuda.get_device_capability(0) == (10, 0)
    assert vk.lib.vk_init(0) == vk.VK_OK
    A = torch.ones((256, 64), dtype=torch.float16, device="cuda")
    B = torch.ones((64, 256), dtype=torch.float16, device="cuda")
    C = vk.gemm(A, B)
    torch.cuda.synchronize()
    assert bool((C == 64).all())


@pytest.mark.parametrize("algo,tile_n", TC_VARIANTS + [("simt", 0)])
def test_cfg0_1024_seed0_fp32acc(vk, algo, tile_n):
    z, A, B = _golden("cfg0_1024_seed0")
    c16, c32 = _run16(vk, A, B, algo=algo, tile_n=tile_n)
    _check_f32acc(c16, c32, A, B, z["C"], z["rows"])


@pytest.mark.parametrize("algo,tile_n", TC_VARIANTS)
def test_fp16acc_1024(vk, algo, tile_n):
    A, B = v0.make_inputs(1024, 1024, 1024, 2, lo=-0.5, hi=0.5)
    c16, c32 = _run16(vk, A, B, algo=algo, acc="f16", tile_n=tile_n)
    _, g32 = v0.v0_f16(A, B)
    assert not np.isnan(c32).any()
    assert v0.rel_frobenius(c16.astype(np.float32), g32) <= FROB_F16ACC
    # the fp16 output is the round-to-nearest of the fp32 copy (the copy is the exact widening of
    # the fp16 accumulator, or the fp32 sum of k-slices when the tail split cut the tile)
    assert np.array_equal(c32.astype(np.float16).view(np.uint16), c16.view(np.uint16))


def test_cfg1_rubric_4096_seed1(vk):
    z, A, B = _golden("cfg1_4096_seed1")
    c16, c32 = _run16(vk, A, B)
    _check_f32acc(c16, c32, A, B, z["C"], z["rows"])


def test_cfg2_fp16acc_4096_seed2(vk):
    z, A, B = _golden("cfg2_4096_seed2")
    c16, _ = _run16(vk, A, B, acc="f16")
    _, g32 = v0.v0_f16(A, B)
    assert v0.rel_frobenius(c16.astype(np.float32), g32) <= FROB_F16ACC
    assert v0.rel_frobenius(c16[z["rows"]].astype(np.float32), z["C"].astype(np.float32)) <= FROB_F16ACC


@pytest.mark.parametrize("algo,tile_n", [("auto", 0), ("tc1", 256), ("tc2", 128)])
def test_cfg5_ragged_4000x5120x3000(vk, algo, tile_n):
    z, A, B = _golden("cfg5_ragged_4000x5120x3000_seed5")
    c16, c32 = _run16(vk, A, B, algo=algo, tile_n=tile_n)
    _check_f32acc(c16, c32, A, B, z["C"], z["rows"])


@pytest.mark.parametrize("name", ["tiny_1x1x1", "tiny_7x13x5", "ragged_200x136x72", "ragged_129x264x520"])
def test_small_ragged_auto(vk, name):
    z, A, B = _golden(name)
    c16, c32 = _run16(vk, A, B)
    _check_f32acc(c16, c32, A, B, z["C"], z["rows"])


@pytest.mark.parametrize("algo,tile_n", TC_VARIANTS)
@pytest.mark.parametrize("shape", [(200, 136, 72), (129, 264, 520), (300, 64, 8), (513, 520, 1000), (8, 8, 8)])
def test_ragged_tc_variants(vk, algo, tile_n, shape):
    m, n, k = shape
    A, B = v0.make_inputs(m, n, k, 21)
    c16, c32 = _run16(vk, A, B, algo=algo, tile_n=tile_n)
    _check_f32acc(c16, c32, A, B)


def test_unaligned_strides_rejected_by_tc_and_taken_by_auto(vk):
    A, B = v0.make_inputs(33, 19, 21, 4)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    with pytest.raises(vk.VkError) as e:
        vk.gemm(dA, dB, algo="tc2")
    assert e.value.code == vk.VK_ERR_ALIGNMENT
    c16, c32 = _run16(vk, A, B, algo="auto")
    _check_f32acc(c16, c32, A, B)


@pytest.mark.parametrize("shape", [(1000, 999, 1001), (4095, 4097, 4093), (33, 19, 21), (7, 5, 3), (1, 1000, 4001)])
@pytest.mark.parametrize("repack", [1, 0], ids=["repack", "simt"])
@pytest.mark.parametrize("layout", [(False, False), (True, True)], ids=["NN", "TT"])
def test_unaligned_pitch_auto_paths(vk, shape, repack, layout):
    """Odd K/N (row pitch not a multiple of 16 bytes): AUTO repacks into a pitched buffer for the
    tensor cores, or (repack off) runs the predicated kernel; both match the oracle."""
    m, n, k = shape
    ta, tb = layout
    A, B = v0.make_inputs(m, n, k, 22)
    As = np.ascontiguousarray(A.T) if ta else A
    Bs = np.ascontiguousarray(B.T) if tb else B
    try:
        vk.set_option("repack", repack)
        C32 = torch.empty((m, n), dtype=torch.float32, device="cuda")
        C = vk.gemm(torch.from_numpy(As).cuda(), torch.from_numpy(Bs).cuda(), trans_a=ta, trans_b=tb, c_f32=C32)
        torch.cuda.synchronize()
    finally:
        vk.set_option("repack", 1)
    assert vk.device_error(0) == 0
    _check_f32acc(C.cpu().numpy(), C32.cpu().numpy(), A, B)


def test_unaligned_base_pointer_repack(vk):
    """Views whose first element is not 16-byte aligned (offset by one element)."""
    A, B = v0.make_inputs(512, 384, 256, 23)
    Abig = torch.zeros(512 * 256 + 1, dtype=torch.float16, device="cuda")
    Abig[1:].copy_(torch.from_numpy(A).cuda().reshape(-1))
    Av = Abig[1:].view(512, 256)
    C32 = torch.empty((512, 384), dtype=torch.float32, device="cuda")
    C = vk.gemm(Av, torch.from_numpy(B).cuda(), c_f32=C32)
    torch.cuda.synchronize()
    _check_f32acc(C.cpu().numpy(), C32.cpu().numpy(), A, B)


def test_sgemm_cfg3_4096_seed3(vk):
    A, B = v0.make_inputs(4096, 4096, 4096, 3, dist="normal", dtype=np.float32)
    C = vk.gemm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda())
    torch.cuda.synchronize()
    c = C.cpu().numpy()
    g = v0.v0_f32(A, B)
    assert v0.rel_frobenius(c, g) <= FROB_SGEMM
    assert v0.max_elem_rel(c, g) <= ELEM
    z, _, _ = _golden("cfg3_sgemm_1024_seed3")  # pins the 1024 fixture path below


@pytest.mark.parametrize("name", ["cfg3_sgemm_1024_seed3", "sgemm_ragged_67x45x33"])
def test_sgemm_golden(vk, name):
    z, A, B = _golden(name)
    C = vk.gemm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda())
    torch.cuda.synchronize()
    c = C.cpu().numpy()
    assert v0.rel_frobenius(c[z["rows"]], z["C"]) <= FROB_SGEMM
    assert v0.max_elem_rel(c[z["rows"]], z["C"]) <= ELEM


@pytest.mark.parametrize("shape", [(1, 1, 1), (130, 131, 17), (257, 129, 64), (128, 256, 1000), (300, 200, 20),
                                   (129, 260, 36), (1000, 1000, 4), (64, 4, 1004)])
def test_sgemm_ragged(vk, shape):
    m, n, k = shape
    A, B = v0.make_inputs(m, n, k, 31, dist="normal", dtype=np.float32)
    C = vk.gemm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda())
    torch.cuda.synchronize()
    c = C.cpu().numpy()
    g = v0.v0_f32(A, B)
    assert v0.rel_frobenius(c, g) <= FROB_SGEMM


@pytest.mark.parametrize("shape", [(4096, 4096, 4096), (1000, 1000, 1000), (300, 200, 20), (129, 260, 36),
                                   (64, 4, 1004), (1, 1, 1)])
def test_sgemm_paired_fma_bitwise(vk, shape):
    """Both paired-FMA SGEMMs (8 x 16 outputs per thread: default; 8 x 8) perform every element's
    fused multiply-adds in the same order as the scalar-FMA kernel: bitwise equal results."""
    m, n, k = shape
    A, B = v0.make_inputs(m, n, k, 33, dist="normal", dtype=np.float32)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    out = {}
    try:
        for variant in (1, 2, 0):
            vk.set_option("sgemm_paired", variant)
            out[variant] = vk.gemm(dA, dB)
    finally:
        vk.set_option("sgemm_paired", 1)
    torch.cuda.synchronize()
    for variant in (1, 2):
        assert torch.equal(out[variant].view(torch.int32), out[0].view(torch.int32)), variant
    assert v0.rel_frobenius(out[1].cpu().numpy(), v0.v0_f32(A, B)) <= FROB_SGEMM


@pytest.mark.parametrize("shape", [(4096, 4096, 4096), (1000, 1000, 1000), (300, 200, 20)])
def test_sgemm_v1_and_v2_agree(vk, shape):
    m, n, k = shape
    A, B = v0.make_inputs(m, n, k, 32, dist="normal", dtype=np.float32)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    c2 = vk.gemm(dA, dB)
    try:
        vk.set_option("sgemm_v2", 0)
        c1 = vk.gemm(dA, dB)
    finally:
        vk.set_option("sgemm_v2", 1)
    torch.cuda.synchronize()
    g = v0.v0_f32(A, B)
    for c in (c1, c2):
        assert v0.rel_frobenius(c.cpu().numpy(), g) <= FROB_SGEMM


@pytest.mark.parametrize("tma_store", [1, 0], ids=["tma-store", "lane-stores"])
@pytest.mark.parametrize("dtype", ["f16", "f32"])
def test_canary_and_strides(vk, dtype, tma_store):
    """C written through ldc > n inside a sentinel-filled buffer: nothing outside C changes (the
    fp16 C here is TMA-store eligible: 16-byte aligned, pitch a multiple of 8, ragged last box)."""
    m, n, k, pad = 300, 264, 136, 40
    if dtype == "f16":
        A, B = v0.make_inputs(m, n, k, 41)
        tdt = torch.float16
    else:
        A, B = v0.make_inputs(m, n, k, 41, dist="normal", dtype=np.float32)
        tdt = torch.float32
    big = torch.full((m + 2, n + pad), 7.0, dtype=tdt, device="cuda")
    C = big[1:m + 1, 8:8 + n]
    # A and B with row pitch > row length as well
    Abig = torch.zeros((m, k + 24), dtype=tdt, device="cuda")
    Abig[:, :k] = torch.from_numpy(A).cuda()
    vk.set_option("tma_store", tma_store)
    try:
        vk.gemm(Abig[:, :k], torch.from_numpy(B).cuda(), C)
        torch.cuda.synchronize()
    finally:
        vk.set_option("tma_store", 1)
    out = big.cpu().numpy().astype(np.float32)
    mask = np.ones_like(out, dtype=bool)
    mask[1:m + 1, 8:8 + n] = False
    assert np.all(out[mask] == 7.0), "write outside C"
    g = v0.v0_f16(A, B)[1] if dtype == "f16" else v0.v0_f32(A, B)
    assert v0.max_elem_rel(out[1:m + 1, 8:8 + n], g) <= ELEM


# (2048^3: 64 whole tiles, no split) (1024x1024x2048: 16 tiles cut into 4 k-slices)
# (4096x4096x1024: 3 full waves + 34 tiles cut into 2 k-slices)
@pytest.mark.parametrize("shape", [(2048, 2048, 2048), (1024, 1024, 2048), (4096, 4096, 1024), (256, 256, 4096)])
@pytest.mark.parametrize("acc", ["f32", "f16"])
def test_repeated_launches_are_bitwise_identical(vk, shape, acc):
    """The reference's race check: 110 consecutive launches compared (10 warm-up + 100).
    With the tail split this also proves the arrival counters return to zero every launch and
    that the slice sum does not depend on which slice arrives last (256x256x4096: 8 slices)."""
    m, n, k = shape
    A, B = v0.make_inputs(m, n, k, 51, lo=-0.5, hi=0.5)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    first = vk.gemm(dA, dB, acc=acc).clone()
    C = torch.empty_like(first)
    mismatches = 0
    for _ in range(110):
        C.fill_(float("nan"))
        vk.gemm(dA, dB, C, acc=acc)
        mismatches += int(not torch.equal(C.view(torch.int16), first.view(torch.int16)))
    torch.cuda.synchronize()
    assert mismatches == 0
    assert vk.device_error(0) == 0
    g32 = v0.v0_f16(A, B)[1]
    tol = FROB_F32ACC if acc == "f32" else FROB_F16ACC
    assert v0.rel_frobenius(first.cpu().numpy().astype(np.float32), g32) <= max(tol, 5e-4)


TAIL_DEFAULTS = {"tail_split": 1, "tail_nsplit": 1, "tail_first": 1}


@pytest.mark.parametrize("mode", [{"tail_split": 0}, {"tail_first": 1}, {"tail_first": 0, "tail_nsplit": 0},
                                  {"tail_first": 0, "tail_nsplit": 1}],
                         ids=["none", "ksplit-first", "ksplit-last", "nsplit"])
# (256, 21248, 4096): one full wave + 9 tiles -> 8 slices each; (512, 21248, 4096): two full waves +
# 18 tiles -> 4 slices each (run first); (2000, 3300, 3000): one full wave + 30 tiles -> 2 slices
# each, ragged M, N, K; (1000, 19000, 1000): ragged M, N, K
@pytest.mark.parametrize("shape", [(4096, 4096, 4096), (4000, 5120, 3000), (1024, 1024, 1024), (512, 768, 2048),
                                   (4096, 4096, 1024), (256, 21248, 4096), (512, 21248, 4096), (2000, 3300, 3000),
                                   (1000, 19000, 1000)])
@pytest.mark.parametrize("acc", ["f32", "f16"])
def test_tail_modes(vk, mode, shape, acc):
    """Whole-tile, k-sliced (before or after the whole tiles) and column-halved partial waves all
    agree with the oracle and are bitwise reproducible."""
    m, n, k = shape
    A, B = v0.make_inputs(m, n, k, 57, lo=-0.5, hi=0.5)
    try:
        for name, val in mode.items():
            vk.set_option(name, val)
        c16, c32 = _run16(vk, A, B, acc=acc)
        again, _ = _run16(vk, A, B, acc=acc)
    finally:
        for name, val in TAIL_DEFAULTS.items():
            vk.set_option(name, val)
    assert np.array_equal(c16.view(np.uint16), again.view(np.uint16))
    g32 = v0.v0_f16(A, B)[1]
    if acc == "f32":
        assert v0.rel_frobenius(c32, g32) <= FROB_F32ACC
        assert v0.max_elem_rel(c32, g32) <= ELEM
    else:
        assert v0.rel_frobenius(c16.astype(np.float32), g32) <= FROB_F16ACC


@pytest.mark.parametrize("shape", [(1024, 1024, 2048), (4096, 4096, 1024)], ids=["slices-only", "slices-first"])
def test_split_gemms_on_concurrent_streams(vk, shape):
    """Two k-sliced GEMMs in flight on different streams must not share tail-split scratch (and,
    with slices ahead of whole tiles, must not wait on each other's residency)."""
    m, n, k = shape
    A1, B1 = v0.make_inputs(m, n, k, 55)
    A2, B2 = v0.make_inputs(m, n, k, 56)
    d = [(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()) for A, B in ((A1, B1), (A2, B2))]
    ref = [vk.gemm(a, b).clone() for a, b in d]
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = [torch.empty_like(ref[0]), torch.empty_like(ref[1])]
    bad = 0
    for it in range(60):
        for i in (0, 1):
            with torch.cuda.stream(streams[i]):
                outs[i].fill_(float("nan"))
                vk.gemm(d[i][0], d[i][1], outs[i])
        if it % 10 == 9:
            torch.cuda.synchronize()
            bad += sum(int(not torch.equal(outs[i].view(torch.int16), ref[i].view(torch.int16))) for i in (0, 1))
    torch.cuda.synchronize()
    assert bad == 0
    assert vk.device_error(0) == 0


@pytest.mark.parametrize("shape", [(1024, 1024, 1024), (4096, 4096, 4096), (4000, 5120, 3000), (300, 200, 4096),
                                   (256, 256, 4096), (512, 768, 2048), (700, 1000, 1200)])
def test_tail_split_matches_unsplit(vk, shape):
    """Tail split on (default) and off give results within the fp32-accumulate tolerance."""
    m, n, k = shape
    A, B = v0.make_inputs(m, n, k, 52)
    try:
        vk.set_option("tail_split", 0)
        c16_off, c32_off = _run16(vk, A, B)
    finally:
        vk.set_option("tail_split", 1)
    c16_on, c32_on = _run16(vk, A, B)
    g32 = v0.v0_f16(A, B)[1]
    for c in (c32_off, c32_on):
        assert v0.rel_frobenius(c, g32) <= FROB_F32ACC
        assert v0.max_elem_rel(c, g32) <= ELEM


PIPELINE_OPTIONS = [{"bk_2sm256": 64}, {"bk_2sm256": 64, "tail_split": 0}, {"tail_split": 0}, {"tma_store": 0},
                    {"l2_evict_last": 0}]
_DEFAULTS = {"bk_2sm256": 128, "tail_split": 1, "tma_store": 1, "l2_evict_last": 1}


@pytest.mark.parametrize("opts", PIPELINE_OPTIONS, ids=["bk64", "bk64-nosplit", "bk128-nosplit", "lane-stores",
                                                        "no-l2-hint"])
@pytest.mark.parametrize("shape", [(1024, 1024, 1024), (4096, 4096, 4096), (4000, 5120, 3000), (200, 136, 72),
                                   (256, 256, 4096)])
@pytest.mark.parametrize("acc", ["f32", "f16"])
def test_pipeline_options(vk, opts, shape, acc):
    m, n, k = shape
    A, B = v0.make_inputs(m, n, k, 54, lo=-0.5, hi=0.5)
    try:
        for name, val in opts.items():
            vk.set_option(name, val)
        c16, c32 = _run16(vk, A, B, algo="tc2", tile_n=256, acc=acc)
    finally:
        for name in opts:
            vk.set_option(name, _DEFAULTS[name])
    g16, g32 = v0.v0_f16(A, B)
    if acc == "f32":
        _check_f32acc(c16, c32, A, B)
    else:
        assert v0.rel_frobenius(c16.astype(np.float32), g32) <= FROB_F16ACC


def test_options_reject_bad_values(vk):
    for name, val in [("raster_group", 0), ("bk_2sm256", 96), ("fwd_empty", 1), ("nope", 1)]:
        with pytest.raises(vk.VkError):
            vk.set_option(name, val)


def test_k_zero_and_empty(vk):
    A = torch.empty((64, 0), dtype=torch.float16, device="cuda")
    B = torch.empty((0, 96), dtype=torch.float16, device="cuda")
    C = torch.full((64, 96), 3.0, dtype=torch.float16, device="cuda")
    vk.gemm(A, B, C, k=0)
    torch.cuda.synchronize()
    assert torch.count_nonzero(C).item() == 0
    E = torch.empty((0, 32), dtype=torch.float16, device="cuda")
    out = vk.gemm(E, torch.zeros((32, 16), dtype=torch.float16, device="cuda"))
    assert out.shape == (0, 16)


def test_non_default_stream(vk):
    A, B = v0.make_inputs(512, 768, 320, 61)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    s = torch.cuda.Stream()
    C32 = torch.empty((512, 768), dtype=torch.float32, device="cuda")
    with torch.cuda.stream(s):
        C = vk.gemm(dA, dB, c_f32=C32)
    s.synchronize()
    assert v0.rel_frobenius(C32.cpu().numpy(), v0.v0_f16(A, B)[1]) <= FROB_F32ACC


@pytest.mark.parametrize("version", [1, 2, 3, 4])
def test_matmul_mirror_f16(vk, version):
    A, B = v0.make_inputs(256, 512, 384, 71)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    C = torch.empty((256, 512), dtype=torch.float16, device="cuda")
    vk.matmul(256, 512, 384, dA, dB, C, version=version)
    torch.cuda.synchronize()
    g16, g32 = v0.v0_f16(A, B)
    tol = FROB_F16ACC if version == 2 else 5e-4
    assert v0.rel_frobenius(C.cpu().numpy().astype(np.float32), g32) <= tol


def test_matmul_mirror_f32_and_bad_version(vk):
    A, B = v0.make_inputs(128, 128, 128, 72, dist="normal", dtype=np.float32)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    C = torch.empty((128, 128), dtype=torch.float32, device="cuda")
    vk.matmul(128, 128, 128, dA, dB, C, version=1)
    torch.cuda.synchronize()
    assert v0.rel_frobenius(C.cpu().numpy(), v0.v0_f32(A, B)) <= FROB_SGEMM
    with pytest.raises(vk.VkError):
        vk.matmul(128, 128, 128, dA, dB, C, version=0)


def test_bounded_wait_selftest(vk):
    """Failure detection without a fault: a wait nothing satisfies gives up and reports."""
    rc = vk.selftest_wait_timeout(0, 20000)
    assert rc == vk.VK_ERR_DEVICE_TIMEOUT, vk.last_error()
    assert vk.device_error(0) == 0  # the self-test clears its own record
    # the context is still usable
    A, B = v0.make_inputs(256, 256, 256, 81)
    c16, c32 = _run16(vk, A, B)
    _check_f32acc(c16, c32, A, B)


@pytest.mark.parametrize("opts", [{}, {"tma_store": 0}], ids=["tma-store", "lane-stores"])
@pytest.mark.parametrize("shape,acc", [((4096, 4096, 4096), "f32"), ((1000, 19000, 1000), "f32"),
                                       ((4000, 5120, 3000), "f32"), ((300, 264, 136), "f32"),
                                       ((4096, 4096, 1024), "f16"), ((1024, 1024, 8192), "f32")])
def test_peer_stores_copy_every_box(vk, shape, acc, opts):
    """vk_gemm_peers with a second buffer on the same device standing in for a peer GPU's C: the
    epilogue's box-by-box copy (whole tiles, k-slice reductions, column halves, ragged edges, TMA and
    per-lane store paths) lands exactly what the local C gets, and nothing outside the rows / columns
    of C is touched in either buffer."""
    m, n, k = shape
    A, B = v0.make_inputs(m, n, k, 71, lo=-0.5, hi=0.5)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    pad = 24
    bufs = [torch.full((m + 2, n + pad), 5.0, dtype=torch.float16, device="cuda") for _ in range(2)]
    C, P = bufs[0][1:m + 1, 8:8 + n], bufs[1][1:m + 1, 8:8 + n]
    try:
        for name, val in opts.items():
            vk.set_option(name, val)
        vk.gemm(dA, dB, C, acc=acc, peers=[P.data_ptr()])
        torch.cuda.synchronize()
    finally:
        vk.set_option("tma_store", 1)
    assert torch.equal(C.view(torch.int16), P.view(torch.int16))
    for b in bufs:
        out = b.cpu().numpy().astype(np.float32)
        mask = np.ones_like(out, dtype=bool)
        mask[1:m + 1, 8:8 + n] = False
        assert np.all(out[mask] == 5.0), "write outside C"
    g32 = v0.v0_f16(A, B)[1]
    c = C.cpu().numpy().astype(np.float32)
    if acc == "f32":
        assert v0.max_elem_rel(c, g32) <= ELEM + 2 ** -10
    else:
        assert v0.rel_frobenius(c, g32) <= FROB_F16ACC
    assert vk.device_error(0) == 0


def test_peer_stores_reject_paths_without_them(vk):
    A = torch.ones((64, 64), dtype=torch.float16, device="cuda")
    B = torch.ones((64, 64), dtype=torch.float16, device="cuda")
    P = torch.empty((64, 64), dtype=torch.float16, device="cuda")
    with pytest.raises(vk.VkError):
        vk.gemm(A, B, algo="simt", peers=[P])
    with pytest.raises(vk.VkError):
        vk.gemm(A[:, :0], B[:0], peers=[P])  # k == 0
