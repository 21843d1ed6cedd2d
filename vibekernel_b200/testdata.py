"""Seeded test data for the GEMM workloads (the harness's data layer, restated with seeds).

The reference harness draws its operands from ``std::random_device`` (unseeded N(0,1),
``results/naive_cycle4/include/playground/test_data.hpp:132-143``), so no two runs see the same
matrices.  The benchmark configurations fix a seed per workload instead; this module produces those
matrices: ``numpy.random.default_rng(seed)`` draws A[m, k] first, then B[k, n], row-major, each value
rounded to the operand type.  It is the recipe the golden fixtures (``tests/golden``) were made with,
so a benchmark can check its output against them.

For uniform draws every value consumes exactly one 64-bit output of the PCG64 generator, so a rank
that needs only rows [r0, r1) of A jumps straight to them (``PCG64.advance``) instead of drawing the
rows before; normal draws (ziggurat, a variable number of outputs) are drawn in sequence.  Matrices are
generated in row chunks, so the float64 intermediate stays small even at 16384 x 16384.
"""
from __future__ import annotations

import numpy as np

_CHUNK_VALUES = 1 << 24  # float64 values per generated chunk (128 MiB)


def _draw(gen: np.random.Generator, rows: int, cols: int, dist: str, lo: float, hi: float, dtype) -> np.ndarray:
    """rows x cols values, converted straight from float64 to ``dtype`` (one rounding).  One float64
    chunk buffer is reused: ``Generator.uniform(lo, hi)`` is ``lo + (hi - lo) * u`` for the generator's
    double u in [0, 1), which the in-place scale and shift below evaluate with the same two roundings."""
    if dist not in ("uniform", "normal"):
        raise ValueError(f"unknown dist {dist!r}")
    out = np.empty((rows, cols), dtype=dtype)
    step = max(1, _CHUNK_VALUES // max(cols, 1))
    buf = np.empty(min(rows, step) * cols, dtype=np.float64)
    for r in range(0, rows, step):
        n = min(step, rows - r)
        chunk = buf[:n * cols]
        if dist == "uniform":
            gen.random(out=chunk)
            chunk *= hi - lo
            chunk += lo
        else:
            gen.standard_normal(out=chunk)
        out[r:r + n] = chunk.reshape(n, cols)
    return out


def make_inputs(m: int, n: int, k: int, seed: int, dist: str = "uniform", lo: float = -1.0, hi: float = 1.0,
                dtype=np.float16, a_rows: tuple[int, int] | None = None, with_b: bool = True):
    """Returns (A, B): A[m, k] (or only rows ``a_rows`` = (r0, r1) of it) and B[k, n] (None when
    ``with_b`` is False), drawn from ``default_rng(seed)`` in the order A then B."""
    r0, r1 = (0, m) if a_rows is None else a_rows
    if not (0 <= r0 <= r1 <= m):
        raise ValueError(f"a_rows {a_rows} outside [0, {m}]")
    if dist == "uniform":
        bg = np.random.PCG64(seed)
        bg.advance(r0 * k)
        A = _draw(np.random.Generator(bg), r1 - r0, k, dist, lo, hi, dtype)
        B = None
        if with_b:
            bg = np.random.PCG64(seed)
            bg.advance(m * k)
            B = _draw(np.random.Generator(bg), k, n, dist, lo, hi, dtype)
        return A, B
    gen = np.random.default_rng(seed)
    if r0 > 0:
        _draw(gen, r0, k, dist, lo, hi, np.float32)  # drawn and dropped: rows before the slice
    A = _draw(gen, r1 - r0, k, dist, lo, hi, dtype)
    if not with_b:
        return A, None
    if r1 < m:
        _draw(gen, m - r1, k, dist, lo, hi, np.float32)
    return A, _draw(gen, k, n, dist, lo, hi, dtype)
