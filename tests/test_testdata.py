"""The package's seeded data generator (used by bench.py) against the oracle's recipe and the
golden fixtures' input digests."""
import glob
import hashlib
import os

import numpy as np
import pytest

from oracle import v0
from vibekernel_b200 import testdata

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("dist,dtype", [("uniform", np.float16), ("normal", np.float32), ("uniform", np.float32)])
@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (37, 23, 29), (300, 70, 130)])
def test_full_matches_oracle(m, n, k, dist, dtype):
    A, B = testdata.make_inputs(m, n, k, 5, dist, -0.5, 0.5, dtype)
    A0, B0 = v0.make_inputs(m, n, k, 5, dist, -0.5, 0.5, dtype)
    assert np.array_equal(A, A0) and np.array_equal(B, B0)


@pytest.mark.parametrize("dist", ["uniform", "normal"])
@pytest.mark.parametrize("r0,r1", [(0, 0), (0, 17), (40, 97), (96, 97), (97, 97)])
def test_row_slices(dist, r0, r1, monkeypatch):
    monkeypatch.setattr(testdata, "_CHUNK_VALUES", 64)  # many chunks: chunking must not change the stream
    m, n, k = 97, 31, 33
    A0, B0 = v0.make_inputs(m, n, k, 9, dist, -1.0, 1.0, np.float16)
    A, B = testdata.make_inputs(m, n, k, 9, dist, -1.0, 1.0, np.float16, a_rows=(r0, r1))
    assert np.array_equal(A, A0[r0:r1]) and np.array_equal(B, B0)
    A, B = testdata.make_inputs(m, n, k, 9, dist, -1.0, 1.0, np.float16, a_rows=(r0, r1), with_b=False)
    assert B is None and np.array_equal(A, A0[r0:r1])


def test_bad_slice():
    with pytest.raises(ValueError):
        testdata.make_inputs(4, 4, 4, 0, a_rows=(3, 5))


@pytest.mark.parametrize("path", [p for p in sorted(glob.glob(os.path.join(HERE, "golden", "*.npz")))
                                  if os.path.getsize(p) < 4 << 20 and "16384" not in p])
def test_fixture_digests(path):
    z = np.load(path)
    m, n, k = int(z["m"]), int(z["n"]), int(z["k"])
    dt = np.float16 if str(z["dtype"]) == "f16" else np.float32
    A, B = testdata.make_inputs(m, n, k, int(z["seed"]), str(z["dist"]), float(z["lo"]), float(z["hi"]), dt)
    assert hashlib.sha256(A.tobytes()).hexdigest() == str(z["sha_A"])
    assert hashlib.sha256(B.tobytes()).hexdigest() == str(z["sha_B"])
