"""CPU oracle for the VibeKernel GEMM hot path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
legs of ``bench.py`` may import this module.  The product library never calls it and
has no CPU fallback.

What is restated here (reference paths relative to the VibeKernel project root):

* ``v0_f16`` follows ``results/naive/src/matmul_f16/matmul_f16_v0_cblas.cpp:11-26``:
  widen fp16 A, B to fp32 exactly (``:13-18``), ``cblas_sgemm(RowMajor, NoTrans,
  NoTrans, m, n, k, 1, A, k, B, n, 0, C, n)`` (``:22-23``), round the fp32 result to
  fp16 with round-to-nearest-even (``:25``).  ``numpy.matmul`` on float32 arrays is an
  OpenBLAS sgemm (numpy's bundled scipy-openblas), i.e. the same algorithm the
  reference calls; summation order may differ between OpenBLAS builds, which is why
  parity against the GPU uses error norms, not bit equality.
* ``v0_f32`` follows ``results/naive/src/matmul_f32/matmul_f32_v0_cblas.cpp:8-12``.
* ``avg_err`` follows ``results/naive_cycle4/include/playground/test_data.hpp:146-162``
  (mean |GT - C| / |GT| in fp32 over the stored-precision GT and C).  Terms whose GT
  is exactly 0 are skipped, the fix the reference harness later adopted for the
  1-in-12 inf abort it documents.
* ``ref_v0_f16`` / ``ref_v0_f32`` call the reference's own v0 sources, compiled
  unmodified into ``oracle/_ref/libv0ref.so`` by ``oracle/Makefile``.

Pinning: the reference ships no golden vectors (it seeds from ``std::random_device``,
``test_data.hpp:138-142``).  ``tests/golden/make_golden.py`` runs the reference's own
v0 (``oracle/_ref``) on seeded inputs and commits the outputs; ``tests/test_oracle.py``
checks this restatement against them.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
REF_LIB_PATH = os.path.join(_HERE, "_ref", "libv0ref.so")


# ----------------------------------------------------------------------------------
# Seeded inputs (uniform[lo,hi) or standard normal, rounded to dtype)
# ----------------------------------------------------------------------------------
def make_inputs(m: int, n: int, k: int, seed: int, dist: str = "uniform",
                lo: float = -1.0, hi: float = 1.0, dtype=np.float16):
    """Row-major A[m,k], B[k,n] drawn from ``numpy.random.default_rng(seed)``.

    A is drawn first, then B, from one generator, then rounded to ``dtype``.
    """
    rng = np.random.default_rng(seed)
    if dist == "uniform":
        a = rng.uniform(lo, hi, size=(m, k))
        b = rng.uniform(lo, hi, size=(k, n))
    elif dist == "normal":
        a = rng.standard_normal(size=(m, k))
        b = rng.standard_normal(size=(k, n))
    else:
        raise ValueError(f"unknown dist {dist!r}")
    return a.astype(dtype), b.astype(dtype)


# ----------------------------------------------------------------------------------
# v0 restatement
# ----------------------------------------------------------------------------------
def v0_f16(A: np.ndarray, B: np.ndarray):
    """fp16 v0: returns (C16, C32) where C32 is the fp32 sgemm result before rounding."""
    assert A.dtype == np.float16 and B.dtype == np.float16
    c32 = np.matmul(A.astype(np.float32), B.astype(np.float32))
    return c32.astype(np.float16), c32


def v0_f32(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    assert A.dtype == np.float32 and B.dtype == np.float32
    return np.matmul(A, B)


def exact_f64(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """fp64 product of the (exactly widened) inputs: bounds OpenBLAS version drift."""
    return np.matmul(A.astype(np.float64), B.astype(np.float64))


# ----------------------------------------------------------------------------------
# Error metrics
# ----------------------------------------------------------------------------------
TAU_FRACTION = 1e-2  # per-element floor tau = TAU_FRACTION * RMS(GT); fixed, never per-kernel


def rel_frobenius(c, gt) -> float:
    c = np.asarray(c, dtype=np.float64)
    gt = np.asarray(gt, dtype=np.float64)
    den = np.linalg.norm(gt)
    return float(np.linalg.norm(c - gt) / den) if den > 0 else float(np.linalg.norm(c))


def max_elem_rel(c, gt, tau_fraction: float = TAU_FRACTION) -> float:
    """max |C - GT| / max(|GT|, tau), tau = tau_fraction * RMS(GT)."""
    c = np.asarray(c, dtype=np.float64)
    gt = np.asarray(gt, dtype=np.float64)
    if gt.size == 0:
        return 0.0
    tau = tau_fraction * float(np.sqrt(np.mean(gt * gt)))
    den = np.maximum(np.abs(gt), max(tau, np.finfo(np.float64).tiny))
    return float(np.max(np.abs(c - gt) / den))


def avg_err(gt, c) -> float:
    """Harness metric: mean over GT!=0 of |GT - C| / |GT|, computed in fp32."""
    gt = np.asarray(gt).astype(np.float32).ravel()
    c = np.asarray(c).astype(np.float32).ravel()
    nz = gt != 0
    if gt.size == 0:
        return 0.0
    return float(np.sum(np.abs((gt[nz] - c[nz]) / gt[nz]), dtype=np.float32) / np.float32(gt.size))


# ----------------------------------------------------------------------------------
# The reference's own v0, compiled from its sources (oracle/_ref)
# ----------------------------------------------------------------------------------
_ref_lib = None


def ref_available() -> bool:
    return os.path.exists(REF_LIB_PATH)


# OpenBLAS picks its sgemm kernel by CPU model at load time, and kernels sum in different orders,
# so the same reference v0 gives fp16 outputs that differ by one ulp on ~0.2 % of elements between
# CPU generations.  The golden fixtures were produced with OpenBLAS's "Cooperlake" kernel (AVX-512
# with BF16); on any CPU that can run it, that kernel is pinned before the library loads, so the
# reference reproduces the fixtures bit for bit whatever the host.  Elsewhere the automatic choice
# stays and the fixture tests compare within one ulp instead.
PINNED_CORETYPE = "Cooperlake"


def _cpu_flags() -> set:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


def _pin_coretype() -> None:
    if "OPENBLAS_CORETYPE" not in os.environ and {"avx512f", "avx512_bf16"} <= _cpu_flags():
        os.environ["OPENBLAS_CORETYPE"] = PINNED_CORETYPE


def coretype_pinned() -> bool:
    """True when the reference library runs (or will run) the fixtures' OpenBLAS kernel."""
    if _ref_lib is None:
        _pin_coretype()
    return os.environ.get("OPENBLAS_CORETYPE") == PINNED_CORETYPE


def _ref():
    global _ref_lib
    if _ref_lib is None:
        if not ref_available():
            raise RuntimeError(f"{REF_LIB_PATH} is not built (make -C oracle)")
        _pin_coretype()
        lib = ctypes.CDLL(REF_LIB_PATH)
        sz = ctypes.c_size_t
        vp = ctypes.c_void_p
        lib.vk_ref_v0_f16.argtypes = [sz, sz, sz, vp, vp, vp]
        lib.vk_ref_v0_f16.restype = None
        lib.vk_ref_v0_f32.argtypes = [sz, sz, sz, vp, vp, vp]
        lib.vk_ref_v0_f32.restype = None
        _ref_lib = lib
    return _ref_lib


def ref_v0_f16(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    A = np.ascontiguousarray(A, dtype=np.float16)
    B = np.ascontiguousarray(B, dtype=np.float16)
    m, k = A.shape
    k2, n = B.shape
    assert k == k2
    C = np.zeros((m, n), dtype=np.float16)
    _ref().vk_ref_v0_f16(m, n, k, A.ctypes.data, B.ctypes.data, C.ctypes.data)
    return C


def ref_v0_f32(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    m, k = A.shape
    k2, n = B.shape
    assert k == k2
    C = np.zeros((m, n), dtype=np.float32)
    _ref().vk_ref_v0_f32(m, n, k, A.ctypes.data, B.ctypes.data, C.ctypes.data)
    return C


def set_ref_threads(n: int) -> None:
    """Thread count of the OpenBLAS under the reference v0 (openblas_set_num_threads)."""
    lib = _ref()
    fn = lib.openblas_set_num_threads  # resolved through the library's dependency (OpenBLAS)
    fn.argtypes = [ctypes.c_int]
    fn.restype = None
    fn(int(n))


def ref_threads() -> int:
    fn = _ref().openblas_get_num_threads
    fn.argtypes = []
    fn.restype = ctypes.c_int
    return int(fn())
