"""vibekernel_b200 -- Python side of the B200 GEMM library (libvkgemm.so, C ABI in include/vkgemm.h).

Mirrors the reference's plugin interface for the GEMM hot path,
``template<> void playground::matmul<DType, Version>(m, n, k, A, B, C)``
(``results/naive_cycle4/include/playground/matmul.hpp:11-23``), as :func:`matmul`, plus the
general entry point :func:`gemm` (strides, accumulate tier, kernel choice, fp32 copy, stream).

Device memory and streams come from PyTorch (plumbing only); all arithmetic runs in the
hand-written sm_100a kernels of ``libvkgemm.so``.  There is no CPU fallback: if the library is
missing, importing this package raises; if no B200 is present, every GPU call raises
:class:`VkError`.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libvkgemm.so")

VK_OK = 0
VK_ERR_INVALID_ARGUMENT = -1
VK_ERR_UNSUPPORTED = -2
VK_ERR_CUDA = -3
VK_ERR_DEVICE_TIMEOUT = -4
VK_ERR_NO_DEVICE = -5
VK_ERR_NCCL = -6
VK_ERR_ALIGNMENT = -7

DTYPE_F16, DTYPE_F32 = 0, 1
ACC_F32, ACC_F16 = 0, 1
ALGO_AUTO, ALGO_TC_2SM, ALGO_TC_1SM, ALGO_FFMA, ALGO_SIMT = 0, 1, 2, 3, 4

_ALGOS = {"auto": ALGO_AUTO, "tc2": ALGO_TC_2SM, "tc1": ALGO_TC_1SM, "ffma": ALGO_FFMA, "simt": ALGO_SIMT}
_ACCS = {"f32": ACC_F32, "f16": ACC_F16}

# The C-ABI symbols declared in include/vkgemm.h.
EXPORTED = (
    "vk_gemm", "vk_matmul_f16", "vk_matmul_f32", "vk_gemm_sharded", "vk_init", "vk_shutdown",
    "vk_last_error_string", "vk_version_string", "vk_device_error", "vk_selftest_wait_timeout",
    "vk_set_wait_timeout_ns", "vk_set_option", "vk_read_clock_probe", "vk_read_trace", "vk_gemm_noalloc",
    "vk_gemm_host", "vk_gemm_ex", "vk_read_trace_cta", "vk_ipc_export", "vk_ipc_import", "vk_ipc_release",
    "vk_copy_async", "vk_debug_schedule", "vk_gemm_peers", "vk_gemm_mc", "vk_mc_supported", "vk_mc_alloc",
    "vk_mc_free", "vk_mc_create", "vk_mc_import", "vk_mc_attach", "vk_mc_detach", "vk_debug_watchdog",
)


class VkError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"vkgemm error {code}: {msg}")
        self.code = code


class GemmArgs(ctypes.Structure):
    _fields_ = [
        ("A", ctypes.c_void_p), ("B", ctypes.c_void_p), ("C", ctypes.c_void_p), ("C_f32", ctypes.c_void_p),
        ("m", ctypes.c_int64), ("n", ctypes.c_int64), ("k", ctypes.c_int64),
        ("lda", ctypes.c_int64), ("ldb", ctypes.c_int64), ("ldc", ctypes.c_int64),
        ("dtype", ctypes.c_int32), ("acc", ctypes.c_int32), ("algo", ctypes.c_int32), ("tile_n", ctypes.c_int32),
        ("stream", ctypes.c_void_p),
    ]


class GemmExt(ctypes.Structure):
    _fields_ = [
        ("trans_a", ctypes.c_int32), ("trans_b", ctypes.c_int32), ("alpha", ctypes.c_float), ("beta", ctypes.c_float),
        ("C_in", ctypes.c_void_p), ("ldc_in", ctypes.c_int64), ("bias", ctypes.c_void_p), ("activation", ctypes.c_int32),
    ]


ACT_NONE, ACT_RELU = 0, 1


class ShardArgs(ctypes.Structure):
    _fields_ = [
        ("ngpu", ctypes.c_int32), ("devices", ctypes.POINTER(ctypes.c_int32)),
        ("A", ctypes.POINTER(ctypes.c_void_p)), ("B", ctypes.POINTER(ctypes.c_void_p)),
        ("C", ctypes.POINTER(ctypes.c_void_p)),
        ("m", ctypes.c_int64), ("n", ctypes.c_int64), ("k", ctypes.c_int64),
        ("dtype", ctypes.c_int32), ("acc", ctypes.c_int32), ("algo", ctypes.c_int32),
        ("allgather_c", ctypes.c_int32), ("times_ms", ctypes.POINTER(ctypes.c_float)),
    ]


class IpcHandle(ctypes.Structure):
    _fields_ = [("handle", ctypes.c_uint8 * 64), ("offset", ctypes.c_uint64)]


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is not built; run `python vibekernel_b200/build.py` (nvcc, sm_100a). "
            "There is no CPU fallback.")
    lib = ctypes.CDLL(LIB_PATH)
    lib.vk_gemm.argtypes = [ctypes.POINTER(GemmArgs)]
    lib.vk_gemm.restype = ctypes.c_int
    lib.vk_gemm_noalloc.argtypes = [ctypes.POINTER(GemmArgs)]
    lib.vk_gemm_noalloc.restype = ctypes.c_int
    lib.vk_gemm_host.argtypes = [ctypes.POINTER(GemmArgs), ctypes.c_int32]
    lib.vk_gemm_host.restype = ctypes.c_int
    lib.vk_gemm_ex.argtypes = [ctypes.POINTER(GemmArgs), ctypes.POINTER(GemmExt)]
    lib.vk_gemm_ex.restype = ctypes.c_int
    lib.vk_gemm_peers.argtypes = [ctypes.POINTER(GemmArgs), ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32]
    lib.vk_gemm_peers.restype = ctypes.c_int
    lib.vk_gemm_mc.argtypes = [ctypes.POINTER(GemmArgs), ctypes.c_void_p]
    lib.vk_gemm_mc.restype = ctypes.c_int
    vpp = ctypes.POINTER(ctypes.c_void_p)
    lib.vk_mc_supported.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
    lib.vk_mc_supported.restype = ctypes.c_int
    lib.vk_mc_alloc.argtypes = [ctypes.c_int32, ctypes.POINTER(ctypes.c_int32), ctypes.c_size_t, vpp, vpp]
    lib.vk_mc_alloc.restype = ctypes.c_int
    lib.vk_mc_free.argtypes = [ctypes.c_void_p]
    lib.vk_mc_free.restype = ctypes.c_int
    lib.vk_mc_create.argtypes = [ctypes.c_int, ctypes.c_int32, ctypes.c_size_t, vpp, ctypes.POINTER(ctypes.c_int64)]
    lib.vk_mc_create.restype = ctypes.c_int
    lib.vk_mc_import.argtypes = [ctypes.c_int, ctypes.c_int32, ctypes.POINTER(ctypes.c_int64), vpp]
    lib.vk_mc_import.restype = ctypes.c_int
    lib.vk_mc_attach.argtypes = [ctypes.c_void_p, vpp, vpp, ctypes.POINTER(ctypes.c_size_t)]
    lib.vk_mc_attach.restype = ctypes.c_int
    lib.vk_mc_detach.argtypes = [ctypes.c_void_p]
    lib.vk_mc_detach.restype = ctypes.c_int
    sz = ctypes.c_size_t
    lib.vk_matmul_f16.argtypes = [ctypes.c_int, sz, sz, sz, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.vk_matmul_f16.restype = ctypes.c_int
    lib.vk_matmul_f32.argtypes = [ctypes.c_int, sz, sz, sz, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.vk_matmul_f32.restype = ctypes.c_int
    lib.vk_gemm_sharded.argtypes = [ctypes.POINTER(ShardArgs)]
    lib.vk_gemm_sharded.restype = ctypes.c_int
    lib.vk_init.argtypes = [ctypes.c_int]
    lib.vk_init.restype = ctypes.c_int
    lib.vk_shutdown.argtypes = []
    lib.vk_shutdown.restype = ctypes.c_int
    lib.vk_last_error_string.argtypes = []
    lib.vk_last_error_string.restype = ctypes.c_char_p
    lib.vk_version_string.argtypes = []
    lib.vk_version_string.restype = ctypes.c_char_p
    lib.vk_device_error.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_uint64), ctypes.c_int]
    lib.vk_device_error.restype = ctypes.c_int
    lib.vk_selftest_wait_timeout.argtypes = [ctypes.c_int, ctypes.c_int64]
    lib.vk_selftest_wait_timeout.restype = ctypes.c_int
    lib.vk_set_wait_timeout_ns.argtypes = [ctypes.c_uint64]
    lib.vk_set_wait_timeout_ns.restype = ctypes.c_int
    lib.vk_set_option.argtypes = [ctypes.c_char_p, ctypes.c_int64]
    lib.vk_set_option.restype = ctypes.c_int
    lib.vk_read_clock_probe.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_uint64), ctypes.c_int]
    lib.vk_read_clock_probe.restype = ctypes.c_int
    lib.vk_read_trace.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_uint64)]
    lib.vk_read_trace.restype = ctypes.c_int
    lib.vk_read_trace_cta.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_uint64), ctypes.c_int]
    lib.vk_read_trace_cta.restype = ctypes.c_int
    lib.vk_ipc_export.argtypes = [ctypes.c_void_p, ctypes.POINTER(IpcHandle)]
    lib.vk_ipc_export.restype = ctypes.c_int
    lib.vk_ipc_import.argtypes = [ctypes.POINTER(IpcHandle), ctypes.POINTER(ctypes.c_void_p)]
    lib.vk_ipc_import.restype = ctypes.c_int
    lib.vk_ipc_release.argtypes = [ctypes.c_void_p]
    lib.vk_ipc_release.restype = ctypes.c_int
    lib.vk_copy_async.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.vk_copy_async.restype = ctypes.c_int
    i32p = ctypes.POINTER(ctypes.c_int32)
    lib.vk_debug_schedule.argtypes = [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, ctypes.c_int32,
                                      i32p, i32p, ctypes.c_int32]
    lib.vk_debug_schedule.restype = ctypes.c_int
    lib.vk_debug_watchdog.argtypes = [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, i32p,
                                      ctypes.POINTER(ctypes.c_int64)]
    lib.vk_debug_watchdog.restype = ctypes.c_int
    return lib


lib = _load()


def last_error() -> str:
    s = lib.vk_last_error_string()
    return s.decode() if s else ""


def check(rc: int) -> None:
    if rc != VK_OK:
        raise VkError(rc, last_error())


def version() -> str:
    return lib.vk_version_string().decode()


# ------------------------------------------------------------------------------------------
# Torch-facing helpers (torch is imported lazily: the C-ABI itself needs no torch)
# ------------------------------------------------------------------------------------------
def _stream_handle(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream or None
    return int(getattr(stream, "cuda_stream", stream)) or None


def _unit_col(t) -> bool:
    """Unit column stride; a dimension of size 1 may carry any stride."""
    return t.stride(1) == 1 or t.shape[1] <= 1


def _row_pitch(t) -> int:
    """Row pitch in elements; the stride of a single row does not matter, so use the row length."""
    return t.stride(0) if t.shape[0] > 1 else max(t.shape[1], 1)


def gemm(A, B, C=None, *, acc: str = "f32", algo: str = "auto", c_f32=None, tile_n: int = 0,
         stream=None, lda: int = 0, ldb: int = 0, ldc: int = 0, m: int | None = None,
         n: int | None = None, k: int | None = None, trans_a: bool = False, trans_b: bool = False,
         alpha: float = 1.0, beta: float = 0.0, c_in=None, bias=None, act: str | None = None, peers=None,
         mc: int | None = None):
    """C = act(alpha * op(A) @ op(B) + beta * c_in + bias) on the GPU (``vk_gemm`` / ``vk_gemm_ex``).

    A is [m, k] (or [k, m] with ``trans_a``) and B is [k, n] (or [n, k] with ``trans_b``), CUDA
    tensors (fp16, or fp32 for the FFMA kernel) with unit column stride; a row stride larger than
    the row length is passed on as lda/ldb.  Returns C (allocated if not given).  ``c_f32``:
    optional fp32 [m, n] tensor receiving the result before rounding (fp16 only).  ``act``: None
    or "relu".  Asynchronous on ``stream`` (default: torch's current stream).  ``peers``: addresses (ints)
    or tensors of up to 7 peer buffers that also receive C, box by box, at the same row / column offsets
    and ldc (``vk_gemm_peers``: the fused all-gather; fp16 tensor-core path, no epilogue extensions).
    ``mc``: address of the multicast view of C (``vk_gemm_mc``: C lies in a multicast buffer, see
    :class:`McBuffer` and ``dist_gemm.McRowGather``; every box is stored once through the NVSwitch into
    all member GPUs' C).
    """
    import torch
    if A.dtype not in (torch.float16, torch.float32) or B.dtype != A.dtype:
        raise TypeError("A and B must both be float16 or both float32")
    if not (A.is_cuda and B.is_cuda):
        raise ValueError("A and B must be CUDA tensors (no CPU fallback)")
    m = (A.shape[1] if trans_a else A.shape[0]) if m is None else m
    k = (A.shape[0] if trans_a else A.shape[1]) if k is None else k
    n = (B.shape[0] if trans_b else B.shape[1]) if n is None else n
    if A.dim() != 2 or B.dim() != 2 or not (_unit_col(A) and _unit_col(B)):
        raise ValueError("A and B must be 2-D with unit column stride")
    lda = lda or _row_pitch(A)
    ldb = ldb or _row_pitch(B)
    if C is None:
        C = torch.empty((m, n), dtype=A.dtype, device=A.device)
    if C.dim() != 2 or not _unit_col(C) or C.dtype != A.dtype:
        raise ValueError("C must be 2-D, unit column stride, same dtype as A")
    ldc = ldc or _row_pitch(C)
    if c_f32 is not None and (c_f32.dtype != torch.float32 or not c_f32.is_contiguous()):
        raise ValueError("c_f32 must be a contiguous float32 tensor")
    a = GemmArgs()
    a.A, a.B, a.C = A.data_ptr(), B.data_ptr(), C.data_ptr()
    a.C_f32 = c_f32.data_ptr() if c_f32 is not None else None
    a.m, a.n, a.k = m, n, k
    a.lda, a.ldb, a.ldc = max(lda, 1), max(ldb, 1), max(ldc, 1)
    a.dtype = DTYPE_F16 if A.dtype == torch.float16 else DTYPE_F32
    a.acc = _ACCS[acc]
    a.algo = _ALGOS[algo]
    a.tile_n = tile_n
    a.stream = _stream_handle(stream)
    extended = trans_a or trans_b or alpha != 1.0 or beta != 0.0 or bias is not None or act is not None
    with torch.cuda.device(A.device):
        if mc is not None:
            if extended or peers:
                raise ValueError("mc cannot be combined with peers, transposes or the fused epilogue")
            check(lib.vk_gemm_mc(ctypes.byref(a), ctypes.c_void_p(int(mc))))
            return C
        if peers is not None and len(peers) > 0:
            if extended:
                raise ValueError("peers cannot be combined with transposes or the fused epilogue")
            addrs = (ctypes.c_void_p * len(peers))(*[p if isinstance(p, int) else p.data_ptr() for p in peers])
            check(lib.vk_gemm_peers(ctypes.byref(a), addrs, len(peers)))
            return C
        if not extended:
            check(lib.vk_gemm(ctypes.byref(a)))
            return C
        x = GemmExt()
        x.trans_a, x.trans_b = int(bool(trans_a)), int(bool(trans_b))
        x.alpha, x.beta = float(alpha), float(beta)
        if c_in is not None:
            if c_in.dtype != C.dtype or c_in.dim() != 2 or c_in.stride(1) != 1:
                raise ValueError("c_in must be 2-D, unit column stride, same dtype as C")
            x.C_in, x.ldc_in = c_in.data_ptr(), c_in.stride(0)
        if bias is not None:
            if bias.dtype != C.dtype or not bias.is_contiguous() or bias.numel() < n:
                raise ValueError("bias must be a contiguous vector of length n with C's dtype")
            x.bias = bias.data_ptr()
        x.activation = {None: ACT_NONE, "relu": ACT_RELU}[act]
        check(lib.vk_gemm_ex(ctypes.byref(a), ctypes.byref(x)))
    return C


def gemm_host(A, B, C=None, *, acc: str = "f32", algo: str = "auto", block_rows: int = 0):
    """C = A @ B for HOST operands through ``vk_gemm_host`` (copies pipelined with the GEMM).

    A, B, C: CPU torch tensors (pin them for full PCIe bandwidth) or numpy arrays, row-major with
    unit column stride, fp16 or fp32.  Synchronous; returns C.
    """
    import numpy as np

    def info(t):
        if isinstance(t, np.ndarray):
            if t.ndim != 2:
                raise ValueError("2-D arrays only")
            if t.size == 0:  # numpy reports zero strides for empty arrays
                return t.ctypes.data, max(t.shape[1], 1), t.dtype == np.float16, t.shape
            if t.strides[1] != t.itemsize:
                raise ValueError("2-D arrays with unit column stride only")
            return t.ctypes.data, t.strides[0] // t.itemsize, t.dtype == np.float16, t.shape
        if t.is_cuda or t.dim() != 2 or t.stride(1) != 1:
            raise ValueError("CPU 2-D tensors with unit column stride only")
        import torch
        return t.data_ptr(), t.stride(0), t.dtype == torch.float16, tuple(t.shape)

    pa, lda, f16a, (m, k) = info(A)
    pb, ldb, f16b, (k2, n) = info(B)
    if k2 != k or f16a != f16b:
        raise ValueError("shape or dtype mismatch")
    if C is None:
        C = np.empty((m, n), dtype=np.float16 if f16a else np.float32)
    pc, ldc, f16c, shape_c = info(C)
    if shape_c != (m, n) or f16c != f16a:
        raise ValueError("C has the wrong shape or dtype")
    a = GemmArgs()
    a.A, a.B, a.C = pa, pb, pc
    a.m, a.n, a.k = m, n, k
    a.lda, a.ldb, a.ldc = max(lda, 1), max(ldb, 1), max(ldc, 1)
    a.dtype = DTYPE_F16 if f16a else DTYPE_F32
    a.acc = _ACCS[acc]
    a.algo = _ALGOS[algo]
    check(lib.vk_gemm_host(ctypes.byref(a), block_rows))
    return C


def matmul(m: int, n: int, k: int, A, B, C, version: int = 1) -> None:
    """Mirror of ``playground::matmul<DType, Version>(m, n, k, A, B, C)`` (default stream).

    DType follows the tensors (float16 -> ``vk_matmul_f16``, float32 -> ``vk_matmul_f32``).
    GPU versions: f16 1 = tcgen05 pair kernel (fp32 acc), 2 = fp16 acc, 3 = single-CTA tcgen05,
    4 = predicated CUDA-core kernel; f32 1 = FFMA SGEMM.  Version 0 is the reference's CPU
    ground truth and is not part of this library.
    """
    import torch
    with torch.cuda.device(A.device):
        if A.dtype == torch.float16:
            rc = lib.vk_matmul_f16(version, m, n, k, A.data_ptr(), B.data_ptr(), C.data_ptr())
        elif A.dtype == torch.float32:
            rc = lib.vk_matmul_f32(version, m, n, k, A.data_ptr(), B.data_ptr(), C.data_ptr())
        else:
            raise TypeError("float16 or float32 only")
    check(rc)


def device_error(device: int = 0, clear: bool = True) -> int:
    w = ctypes.c_uint64(0)
    check(lib.vk_device_error(device, ctypes.byref(w), 1 if clear else 0))
    return int(w.value)


def set_option(name: str, value: int) -> None:
    """Process-wide knob: tail_split, raster_group, bk_2sm256, clock_probe, trace, wait_timeout_ns."""
    check(lib.vk_set_option(name.encode(), int(value)))


def read_clock_probe(device: int = 0, clear: bool = True):
    """Returns (sm_mhz, launches) measured inside the tensor-core kernels since the last clear."""
    out = (ctypes.c_uint64 * 3)()
    check(lib.vk_read_clock_probe(device, out, 1 if clear else 0))
    cycles, ns, launches = int(out[0]), int(out[1]), int(out[2])
    return (cycles / ns * 1e3 if ns else None), launches


TRACE_FIELDS = ("cta0_entry", "prologue_done", "first_tma", "first_stage_full", "last_mma_commit",
                "first_acc_ready", "last_store", "cta0_exit", "min_entry", "max_entry", "min_exit", "max_exit")


def read_trace(device: int = 0) -> dict:
    """Timeline of the last traced launch, ns relative to the earliest CTA entry (and re-arm)."""
    out = (ctypes.c_uint64 * 16)()
    check(lib.vk_read_trace(device, out))
    v = [int(x) for x in out]
    t0 = v[8]
    return {name: (v[i] - t0) / 1e3 for i, name in enumerate(TRACE_FIELDS)}


def read_trace_cta(device: int = 0, ctas: int = 148):
    """Per-CTA timeline of the last traced launch: list of dicts (times in us from earliest entry)."""
    out = (ctypes.c_uint64 * (8 * ctas))()
    check(lib.vk_read_trace_cta(device, out, ctas))
    rows = [[int(out[8 * i + j]) for j in range(8)] for i in range(ctas)]
    t0 = min(r[0] for r in rows if r[0])

    def rel(v):
        return (v - t0) / 1e3 if v else None
    return [{"cta": i, "entry": rel(r[0]), "last_commit": rel(r[1]), "last_store": rel(r[2]), "exit": rel(r[3]),
             "smid": r[4], "units": r[5], "last_acc_ready": rel(r[6]), "tail_sync": rel(r[7])}
            for i, r in enumerate(rows)]


def set_wait_timeout_ns(ns: int) -> None:
    check(lib.vk_set_wait_timeout_ns(ns))


def selftest_wait_timeout(device: int = 0, timeout_us: int = 50000) -> int:
    """Runs the bounded-wait self-test; returns the status code (VK_ERR_DEVICE_TIMEOUT expected)."""
    return lib.vk_selftest_wait_timeout(device, timeout_us)


def gemm_sharded(A_parts, B_parts, C_parts, m: int, n: int, k: int, *, acc: str = "f32",
                 algo: str = "auto", allgather=True):
    """Single-process multi-GPU row-block GEMM through ``vk_gemm_sharded``.

    A_parts[r]: GPU r's row slice [rows_r, k]; B_parts[r]: full [k, n] on GPU r; C_parts[r]: full
    [m, n] buffer on GPU r.  ``allgather``: False, True (NCCL after the GEMMs), "pipelined" (peer
    copies of finished row chunks overlapped with the GEMM), "fused" (every GPU's epilogue also
    stores its C boxes into all peers' C) or "nvls" (C_parts are the views of one :class:`McBuffer`;
    every GPU's epilogue stores each box once to the multicast view).  Returns (compute_ms,
    gather_ms), each the max over GPUs.
    """
    import torch
    g = len(A_parts)
    devs = (ctypes.c_int32 * g)(*[t.device.index for t in A_parts])
    pa = (ctypes.c_void_p * g)(*[t.data_ptr() for t in A_parts])
    pb = (ctypes.c_void_p * g)(*[t.data_ptr() for t in B_parts])
    pc = (ctypes.c_void_p * g)(*[t.data_ptr() for t in C_parts])
    times = (ctypes.c_float * 2)()
    s = ShardArgs()
    s.ngpu = g
    s.devices = devs
    s.A, s.B, s.C = pa, pb, pc
    s.m, s.n, s.k = m, n, k
    s.dtype = DTYPE_F16 if A_parts[0].dtype == torch.float16 else DTYPE_F32
    s.acc = _ACCS[acc]
    s.algo = _ALGOS[algo]
    s.allgather_c = {"pipelined": 2, "fused": 3, "nvls": 4}.get(allgather, 1 if allgather else 0)
    s.times_ms = times
    check(lib.vk_gemm_sharded(ctypes.byref(s)))
    return float(times[0]), float(times[1])


# ------------------------------------------------------------------------------------------
# NVLS multicast buffers
# ------------------------------------------------------------------------------------------
def mc_supported(device: int = 0) -> bool:
    """True when ``device`` supports NVLink SHARP multicast (an NVSwitch system)."""
    v = ctypes.c_int(0)
    check(lib.vk_mc_supported(device, ctypes.byref(v)))
    return bool(v.value)


class _CudaArray:
    """__cuda_array_interface__ wrapper: lets torch view device memory the library mapped itself."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


def _view(ptr: int, shape, dtype, device):
    import torch
    typestr = {torch.float16: "<f2", torch.float32: "<f4"}[dtype]
    return torch.as_tensor(_CudaArray(ptr, shape, typestr), device=device)


class McBuffer:
    """One multicast buffer over several GPUs of this process (``vk_mc_alloc``).

    ``views[i]`` is a [rows, cols] tensor in GPU ``devices[i]``'s own memory; ``mc`` is the address
    of the multicast view.  Free with :meth:`free` after every GPU is done with it.
    """

    def __init__(self, devices, rows: int, cols: int, dtype):
        import torch
        esize = torch.tensor([], dtype=dtype).element_size()
        g = len(devices)
        devs = (ctypes.c_int32 * g)(*devices)
        ptrs = (ctypes.c_void_p * g)()
        mc = ctypes.c_void_p()
        check(lib.vk_mc_alloc(g, devs, rows * cols * esize, ptrs, ctypes.byref(mc)))
        self.devices = list(devices)
        self.mc = int(mc.value)
        self.views = [_view(ptrs[i], (rows, cols), dtype, torch.device("cuda", d)) for i, d in enumerate(devices)]

    def free(self) -> None:
        if self.mc:
            import torch
            for d in self.devices:
                torch.cuda.synchronize(d)
            self.views = []
            check(lib.vk_mc_free(ctypes.c_void_p(self.mc)))
            self.mc = 0


def ipc_export(tensor) -> bytes:
    """CUDA IPC handle (+ offset) of a device tensor's memory, as bytes to send to a peer process."""
    h = IpcHandle()
    check(lib.vk_ipc_export(ctypes.c_void_p(tensor.data_ptr()), ctypes.byref(h)))
    return bytes(ctypes.string_at(ctypes.addressof(h), ctypes.sizeof(h)))


def ipc_import(handle: bytes) -> int:
    """Maps a buffer exported by ANOTHER process (``ipc_export``) into this one; returns its address."""
    h = IpcHandle.from_buffer_copy(handle)
    p = ctypes.c_void_p()
    check(lib.vk_ipc_import(ctypes.byref(h), ctypes.byref(p)))
    return int(p.value)


def ipc_release(ptr: int) -> None:
    check(lib.vk_ipc_release(ctypes.c_void_p(ptr)))


def copy_async(dst: int, src: int, nbytes: int, stream=None) -> None:
    """Device-to-device copy of ``nbytes`` (peer addresses allowed) on ``stream`` (copy engines)."""
    check(lib.vk_copy_async(ctypes.c_void_p(dst), ctypes.c_void_p(src), nbytes,
                            ctypes.c_void_p(stream.cuda_stream if stream is not None else 0)))


def debug_schedule(tiles: int, num_kb: int, max_units: int, k: int, split: bool = True, nsplit: bool = True,
                   first: bool = True):
    """The persistent kernels' work units for a problem (host-side, no device): (plan dict, units list of
    (tile, kb0, kb1, tag)) with tag = slice index, 100 + column half, or -1 for a whole tile."""
    plan = (ctypes.c_int32 * 6)()
    flags = (1 if split else 0) | (2 if nsplit else 0) | (4 if first else 0)
    check(lib.vk_debug_schedule(tiles, num_kb, max_units, k, flags, plan, None, 0))
    n = int(plan[0])
    units = (ctypes.c_int32 * max(4 * n, 1))()
    check(lib.vk_debug_schedule(tiles, num_kb, max_units, k, flags, plan, units, n))
    keys = ("units", "full_units", "split", "nsplit", "tail_first", "grid_units")
    return dict(zip(keys, (int(x) for x in plan))), [tuple(int(units[4 * u + j]) for j in range(4)) for u in range(n)]


def row_blocks(m: int, parts: int):
    """Row offsets of the balanced split used by the sharded layer: GPU r owns [off[r], off[r+1])."""
    return [m * r // parts for r in range(parts + 1)]
