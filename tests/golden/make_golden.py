"""Generate the golden fixtures in this folder from the reference's own v0 ground truth.

Run where the reference tree is available (it builds ``oracle/_ref`` from the reference's
unmodified v0 sources first):

    make -C oracle && python tests/golden/make_golden.py [case names; default: all]

The reference's OpenBLAS selects its sgemm kernel by CPU model; ``oracle/v0.py`` pins the kernel the
fixtures were made with ("Cooperlake", AVX-512 BF16) wherever the CPU can run it, so regenerating
them on such a CPU reproduces the committed files bit for bit.

Each fixture is an ``.npz`` holding the seeded-input recipe, sha256 digests of the
generated inputs (so a drift of the generator is caught before any comparison), the
row indices sampled, and the reference v0 output on those rows (the full output for
small cases).  The reference publishes no golden vectors of its own; these are the
pins for the numpy restatement in ``oracle/v0.py`` and for the GPU parity tests.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import v0  # noqa: E402

# name, m, n, k, seed, dist, lo, hi, dtype, row_stride (1 = full output)
CASES = [
    ("cfg0_1024_seed0", 1024, 1024, 1024, 0, "uniform", -1.0, 1.0, "f16", 16),
    ("cfg1_4096_seed1", 4096, 4096, 4096, 1, "uniform", -1.0, 1.0, "f16", 128),
    ("cfg2_4096_seed2", 4096, 4096, 4096, 2, "uniform", -0.5, 0.5, "f16", 128),
    ("cfg3_sgemm_1024_seed3", 1024, 1024, 1024, 3, "normal", 0.0, 0.0, "f32", 32),
    ("cfg5_ragged_4000x5120x3000_seed5", 4000, 5120, 3000, 5, "uniform", -1.0, 1.0, "f16", 125),
    ("cfg3_sgemm_4096_seed3", 4096, 4096, 4096, 3, "normal", 0.0, 0.0, "f32", 128),
    ("cfg4a_16384_seed4", 16384, 16384, 16384, 4, "uniform", -1.0, 1.0, "f16", 512),
    ("tiny_1x1x1", 1, 1, 1, 11, "uniform", -1.0, 1.0, "f16", 1),
    ("tiny_7x13x5", 7, 13, 5, 12, "uniform", -1.0, 1.0, "f16", 1),
    ("ragged_200x136x72", 200, 136, 72, 13, "uniform", -1.0, 1.0, "f16", 1),
    ("ragged_129x264x520", 129, 264, 520, 14, "uniform", -1.0, 1.0, "f16", 1),
    ("sgemm_ragged_67x45x33", 67, 45, 33, 15, "normal", 0.0, 0.0, "f32", 1),
]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main(names: list[str]) -> None:
    for name, m, n, k, seed, dist, lo, hi, dt, stride in CASES:
        if names and name not in names:
            continue
        dtype = np.float16 if dt == "f16" else np.float32
        A, B = v0.make_inputs(m, n, k, seed, dist, lo, hi, dtype)
        rows = np.arange(0, m, stride, dtype=np.int64)
        if dt == "f16":
            C = v0.ref_v0_f16(A[rows], B)
        else:
            C = v0.ref_v0_f32(A[rows], B)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(
            path, m=m, n=n, k=k, seed=seed, dist=dist, lo=lo, hi=hi, dtype=dt,
            rows=rows, C=C, sha_A=sha(A), sha_B=sha(B))
        print(f"{name}: rows={rows.size} C={C.shape} -> {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main(sys.argv[1:])
