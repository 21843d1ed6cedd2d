"""CPU: the C-ABI library loads, exports every entry point the header declares, and rejects
bad arguments before touching a device."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "vkgemm.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(vk_\w+)\s*\(", text, re.M)))


def test_header_declares_the_boundary():
    names = _declared()
    for n in ("vk_gemm", "vk_matmul_f16", "vk_matmul_f32", "vk_gemm_sharded", "vk_last_error_string"):
        assert n in names


def test_library_exports_every_declared_symbol():
    import vibekernel_b200 as vk
    lib = ctypes.CDLL(vk.LIB_PATH)
    for name in _declared():
        assert hasattr(lib, name), f"{name} declared in include/vkgemm.h but not exported"
    assert set(_declared()) <= set(vk.EXPORTED)


def test_library_is_built_for_sm100a_only():
    """The build recipe compiles every source for exactly one target, sm_100a (no PTX for JIT, no
    other architecture), and the built library is newer than every source it depends on."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("vk_build", os.path.join(ROOT, "vibekernel_b200", "build.py"))
    build = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(build)
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]
    import vibekernel_b200 as vk
    assert os.path.abspath(vk.LIB_PATH) == os.path.abspath(build.LIB)
    assert not build._stale(), "libvkgemm.so is older than its sources; run python vibekernel_b200/build.py"


def test_argument_validation_without_gpu():
    import vibekernel_b200 as vk
    lib = vk.lib
    assert lib.vk_gemm(None) == vk.VK_ERR_INVALID_ARGUMENT
    a = vk.GemmArgs()
    a.m, a.n, a.k = -1, 4, 4
    assert lib.vk_gemm(ctypes.byref(a)) == vk.VK_ERR_INVALID_ARGUMENT
    assert "negative" in vk.last_error()
    a.m = 4
    a.dtype = 7
    assert lib.vk_gemm(ctypes.byref(a)) == vk.VK_ERR_INVALID_ARGUMENT
    a.dtype = vk.DTYPE_F32
    a.acc = vk.ACC_F16
    assert lib.vk_gemm(ctypes.byref(a)) == vk.VK_ERR_UNSUPPORTED
    a.acc = vk.ACC_F32
    a.algo = 99
    assert lib.vk_gemm(ctypes.byref(a)) == vk.VK_ERR_INVALID_ARGUMENT
    a.algo = 0
    a.lda = 2  # < k
    assert lib.vk_gemm(ctypes.byref(a)) == vk.VK_ERR_INVALID_ARGUMENT
    a.lda = 0
    a.tile_n = 96
    assert lib.vk_gemm(ctypes.byref(a)) == vk.VK_ERR_INVALID_ARGUMENT
    assert lib.vk_matmul_f16(0, 4, 4, 4, None, None, None) == vk.VK_ERR_INVALID_ARGUMENT
    assert lib.vk_matmul_f32(2, 4, 4, 4, None, None, None) == vk.VK_ERR_INVALID_ARGUMENT
    assert lib.vk_gemm_sharded(None) == vk.VK_ERR_INVALID_ARGUMENT
    assert lib.vk_set_wait_timeout_ns(0) == vk.VK_ERR_INVALID_ARGUMENT
    assert vk.version().startswith("vkgemm")


def test_no_device_is_an_error_not_a_fallback():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    import vibekernel_b200 as vk
    a = vk.GemmArgs()
    a.m = a.n = a.k = 8
    rc = vk.lib.vk_gemm(ctypes.byref(a))
    assert rc in (vk.VK_ERR_CUDA, vk.VK_ERR_NO_DEVICE)


def test_peer_plumbing_rejects_bad_arguments_without_gpu():
    """The IPC / peer-copy entry points validate their arguments before any CUDA call."""
    import vibekernel_b200 as vk
    lib = vk.lib
    h = vk.IpcHandle()
    assert lib.vk_ipc_export(None, ctypes.byref(h)) == vk.VK_ERR_INVALID_ARGUMENT
    assert lib.vk_ipc_export(ctypes.c_void_p(0x1000), None) == vk.VK_ERR_INVALID_ARGUMENT
    p = ctypes.c_void_p()
    assert lib.vk_ipc_import(None, ctypes.byref(p)) == vk.VK_ERR_INVALID_ARGUMENT
    assert lib.vk_ipc_import(ctypes.byref(h), None) == vk.VK_ERR_INVALID_ARGUMENT
    # only pointers handed out by vk_ipc_import may be released
    assert lib.vk_ipc_release(ctypes.c_void_p(0x1000)) == vk.VK_ERR_INVALID_ARGUMENT
    assert "vk_ipc_import" in vk.last_error()
    assert lib.vk_copy_async(None, None, 0, None) == vk.VK_OK  # nothing to copy
    assert lib.vk_copy_async(None, ctypes.c_void_p(0x1000), 16, None) == vk.VK_ERR_INVALID_ARGUMENT
    assert ctypes.sizeof(vk.IpcHandle) == 72  # 64-byte cudaIpcMemHandle_t + 8-byte offset


def test_peer_gemm_rejects_bad_arguments_without_gpu():
    import vibekernel_b200 as vk
    a = vk.GemmArgs()
    a.m = a.n = a.k = 8
    a.A = a.B = a.C = 0x1000
    peers = (ctypes.c_void_p * 8)(*([0x2000] * 8))
    assert vk.lib.vk_gemm_peers(ctypes.byref(a), peers, 8) == vk.VK_ERR_INVALID_ARGUMENT  # at most 7 peers
    assert vk.lib.vk_gemm_peers(ctypes.byref(a), None, 1) == vk.VK_ERR_INVALID_ARGUMENT
    nul = (ctypes.c_void_p * 2)(0x2000, None)
    assert vk.lib.vk_gemm_peers(ctypes.byref(a), nul, 2) == vk.VK_ERR_INVALID_ARGUMENT
    a.dtype = vk.DTYPE_F32
    assert vk.lib.vk_gemm_peers(ctypes.byref(a), peers, 1) == vk.VK_ERR_UNSUPPORTED


def test_multicast_entry_points_reject_bad_arguments_without_gpu():
    import ctypes

    import vibekernel_b200 as vk
    a = vk.GemmArgs()
    a.m = a.n = a.k = 16
    assert vk.lib.vk_gemm_mc(ctypes.byref(a), None) == vk.VK_ERR_INVALID_ARGUMENT
    assert "C_mc is NULL" in vk.last_error()
    assert vk.lib.vk_mc_supported(0, None) == vk.VK_ERR_INVALID_ARGUMENT
    ptrs = (ctypes.c_void_p * 1)()
    mc = ctypes.c_void_p()
    assert vk.lib.vk_mc_alloc(0, None, 1 << 20, ptrs, ctypes.byref(mc)) == vk.VK_ERR_INVALID_ARGUMENT
    assert vk.lib.vk_mc_free(ctypes.c_void_p(0x1234)) == vk.VK_ERR_INVALID_ARGUMENT
    assert "not a multicast pointer" in vk.last_error()
    assert vk.lib.vk_mc_detach(None) == vk.VK_ERR_INVALID_ARGUMENT
    assert vk.lib.vk_mc_attach(None, None, None, None) == vk.VK_ERR_INVALID_ARGUMENT
    team = ctypes.c_void_p()
    share = (ctypes.c_int64 * 3)()
    assert vk.lib.vk_mc_create(0, 0, 1 << 20, ctypes.byref(team), share) == vk.VK_ERR_INVALID_ARGUMENT
    assert vk.lib.vk_mc_import(0, 2, None, ctypes.byref(team)) == vk.VK_ERR_INVALID_ARGUMENT
