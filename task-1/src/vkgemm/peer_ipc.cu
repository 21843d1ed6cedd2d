// Peer-memory plumbing for one-process-per-GPU jobs (torchrun): export a device buffer as a CUDA IPC
// handle, map a peer process's buffer into this process, and push bytes into it with the copy
// engines.  The row-sharded GEMM uses it to overlap the all-gather of C with the GEMM: every rank
// computes its row block in chunks and, as each chunk finishes, copies it straight into every peer's
// full C buffer over NVLink (vibekernel_b200/dist_gemm.py).  The reference has no multi-GPU path
// (README.md:161); the single-process counterpart is the pipelined mode of vk_gemm_sharded.
//
// Only plain peer mappings are used (cudaIpcOpenMemHandle with lazy peer access): no multicast
// object, no TMA from peer memory.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <map>
#include <mutex>

#include "vkgemm.h"
#include "vk_internal.h"

namespace {

typedef CUresult (*GetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
GetAddressRangeFn g_range = nullptr;
std::mutex g_ipc_mu;
std::map<void*, void*> g_imported;  // pointer handed out by vk_ipc_import -> mapped allocation base

int cuda_err(cudaError_t e, const char* what)
{
    return vk::set_error(VK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(((vk_ipc_handle*)nullptr)->handle), "IPC handle size");

}  // namespace

extern "C" int vk_ipc_export(const void* ptr, vk_ipc_handle* out)
{
    if (ptr == nullptr || out == nullptr) return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_ipc_export: NULL");
    std::lock_guard<std::mutex> lk(g_ipc_mu);
    if (g_range == nullptr) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess) return cuda_err(e, "vk_ipc_export: cuMemGetAddressRange entry point");
        if (q != cudaDriverEntryPointSuccess || fn == nullptr)
            return vk::set_error(VK_ERR_CUDA, "vk_ipc_export: cuMemGetAddressRange not available");
        g_range = reinterpret_cast<GetAddressRangeFn>(fn);
    }
    // Allocators hand out pieces of larger allocations; the IPC handle names the whole allocation,
    // so the buffer's offset inside it travels with the handle.
    CUdeviceptr base = 0;
    size_t size = 0;
    const CUresult r = g_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
    if (r != CUDA_SUCCESS) return vk::set_error(VK_ERR_CUDA, "vk_ipc_export: cuMemGetAddressRange failed (%d)", (int)r);
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
    if (e != cudaSuccess) return cuda_err(e, "vk_ipc_export: cudaIpcGetMemHandle");
    memcpy(out->handle, &h, sizeof(h));
    out->offset = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
    return VK_OK;
}

extern "C" int vk_ipc_import(const vk_ipc_handle* h, void** out_ptr)
{
    if (h == nullptr || out_ptr == nullptr) return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_ipc_import: NULL");
    cudaIpcMemHandle_t ch;
    memcpy(&ch, h->handle, sizeof(ch));
    void* base = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&base, ch, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_err(e, "vk_ipc_import: cudaIpcOpenMemHandle");
    void* p = static_cast<char*>(base) + h->offset;
    std::lock_guard<std::mutex> lk(g_ipc_mu);
    g_imported[p] = base;
    *out_ptr = p;
    return VK_OK;
}

extern "C" int vk_ipc_release(void* ptr)
{
    void* base = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_ipc_mu);
        auto it = g_imported.find(ptr);
        if (it == g_imported.end())
            return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_ipc_release: pointer was not returned by vk_ipc_import");
        base = it->second;
        g_imported.erase(it);
    }
    const cudaError_t e = cudaIpcCloseMemHandle(base);
    if (e != cudaSuccess) return cuda_err(e, "vk_ipc_release: cudaIpcCloseMemHandle");
    return VK_OK;
}

extern "C" int vk_copy_async(void* dst, const void* src, size_t bytes, void* stream)
{
    if (bytes == 0) return VK_OK;
    if (dst == nullptr || src == nullptr) return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_copy_async: NULL");
    const cudaError_t e =
        cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_err(e, "vk_copy_async: cudaMemcpyAsync");
    return VK_OK;
}
