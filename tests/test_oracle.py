"""CPU: pin the oracle (oracle/v0.py) to the golden fixtures made by the reference's own v0.

The fixtures in tests/golden were produced by tests/golden/make_golden.py from the reference's
unmodified v0 sources (results/naive/src/matmul_f16/matmul_f16_v0_cblas.cpp:11-26 and
results/naive/src/matmul_f32/matmul_f32_v0_cblas.cpp:8-12) linked against OpenBLAS 0.3.15.
"""
import glob
import hashlib
import os

import numpy as np
import pytest

from oracle import v0

ALL_GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))
# The 16384^3 fixture (1 GiB of inputs) gets one test of its own that generates its inputs once.
BIG = [g for g in ALL_GOLDEN if "16384" in os.path.basename(g)]
GOLDEN = [g for g in ALL_GOLDEN if g not in BIG]
# Cases small enough to regenerate in well under a second each on one core.
FAST = [g for g in GOLDEN if not any(t in os.path.basename(g) for t in ("4096", "4000x5120", "16384"))]


def _load(path):
    z = np.load(path)
    dt = np.float16 if str(z["dtype"]) == "f16" else np.float32
    A, B = v0.make_inputs(int(z["m"]), int(z["n"]), int(z["k"]), int(z["seed"]), str(z["dist"]),
                          float(z["lo"]), float(z["hi"]), dt)
    return z, A, B


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_fixtures_present():
    names = {os.path.basename(g) for g in GOLDEN}
    assert "cfg0_1024_seed0.npz" in names and "cfg5_ragged_4000x5120x3000_seed5.npz" in names
    assert len(GOLDEN) >= 10 and len(BIG) == 1


@pytest.mark.parametrize("path", BIG, ids=[os.path.basename(g) for g in BIG])
def test_big_fixture(path):
    """configs[4a] (16384^3, seed 4): input digests, the restatement and the compiled reference."""
    from vibekernel_b200 import testdata  # same recipe as v0.make_inputs (tests/test_testdata.py), chunked
    z = np.load(path)
    A, B = testdata.make_inputs(int(z["m"]), int(z["n"]), int(z["k"]), int(z["seed"]), str(z["dist"]),
                                float(z["lo"]), float(z["hi"]), np.float16)
    assert _sha(A) == str(z["sha_A"]) and _sha(B) == str(z["sha_B"]), "input generator drifted"
    rows = z["rows"]
    gold = z["C"]
    c16, c32 = v0.v0_f16(A[rows], B)
    assert np.mean(c16.view(np.uint16) != gold.view(np.uint16)) < 0.01
    assert v0.max_elem_rel(c16, gold) < 2e-3
    if v0.ref_available() and v0.coretype_pinned():
        assert np.array_equal(v0.ref_v0_f16(A[rows], B).view(np.uint16), gold.view(np.uint16))


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(g) for g in GOLDEN])
def test_seeded_inputs_reproduce(path):
    z, A, B = _load(path)
    assert _sha(A) == str(z["sha_A"]), "input generator drifted"
    assert _sha(B) == str(z["sha_B"]), "input generator drifted"


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(g) for g in GOLDEN])
def test_restatement_matches_reference_v0(path):
    z, A, B = _load(path)
    rows = z["rows"]
    gold = z["C"]
    if str(z["dtype"]) == "f16":
        c16, c32 = v0.v0_f16(A[rows], B)
        # Same algorithm, different OpenBLAS build: the fp32 results agree to summation-order
        # noise (~1e-7 relative), so after rounding to fp16 only a small fraction of elements
        # differ (by one fp16 ulp, or by fp32 noise on entries near zero).
        assert np.mean(c16.view(np.uint16) != gold.view(np.uint16)) < 0.01
        assert v0.max_elem_rel(c16, gold) < 2e-3
        # fp16 rounding of gold alone: at most 2^-11 relative per element
        assert v0.rel_frobenius(c32, gold.astype(np.float32)) < 2.0 ** -11
    else:
        c = v0.v0_f32(A[rows], B)
        assert v0.rel_frobenius(c, gold) < 1e-6
        assert v0.max_elem_rel(c, gold) < 2e-3


@pytest.mark.skipif(not v0.ref_available(), reason="oracle/_ref not built (make -C oracle)")
@pytest.mark.parametrize("path", FAST, ids=[os.path.basename(g) for g in FAST])
def test_reference_build_reproduces_fixture(path):
    z, A, B = _load(path)
    rows = z["rows"]
    if str(z["dtype"]) == "f16":
        out = v0.ref_v0_f16(A[rows], B)
        if v0.coretype_pinned():
            # the fixtures' OpenBLAS kernel: bit for bit
            assert np.array_equal(out.view(np.uint16), z["C"].view(np.uint16))
        else:
            # another OpenBLAS kernel sums in another order: one fp16 ulp on a few elements
            assert np.mean(out.view(np.uint16) != z["C"].view(np.uint16)) < 0.01
            assert v0.max_elem_rel(out, z["C"]) < 2e-3
    else:
        out = v0.ref_v0_f32(A[rows], B)
        assert np.allclose(out, z["C"], rtol=0, atol=1e-4)


def test_oracle_against_fp64():
    A, B = v0.make_inputs(256, 192, 320, 7)
    _, c32 = v0.v0_f16(A, B)
    e = v0.exact_f64(A, B)
    assert v0.rel_frobenius(c32, e) < 1e-6
    assert v0.max_elem_rel(c32, e) < 1e-4


def test_metrics_on_planted_mistake():
    """A planted error in an oracle output must be caught by the parity metrics."""
    A, B = v0.make_inputs(64, 64, 64, 9)
    c16, c32 = v0.v0_f16(A, B)
    bad = c32.copy()
    bad[5, 7] += 1.0
    assert v0.max_elem_rel(bad, c32) > 2e-3
    bad2 = c32 * (1 + 1e-3)
    assert v0.rel_frobenius(bad2, c32) > 1e-4


def test_avg_err_matches_harness_definition():
    gt = np.array([1.0, 2.0, 0.0, -4.0], dtype=np.float16)
    c = np.array([1.0, 2.5, 3.0, -4.0], dtype=np.float16)
    # GT==0 term skipped, denominator is the full size (test_data.hpp:146-162 semantics)
    assert v0.avg_err(gt, c) == pytest.approx((0.5 / 2.0) / 4)
