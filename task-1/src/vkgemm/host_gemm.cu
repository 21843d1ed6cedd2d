// Host-buffer GEMM (vk_gemm_host): C = A * B where A, B and C live in host memory, as in the
// reference harness's data flow (TestData: host A/B -> cudaMemcpy -> matmul -> cudaMemcpy back,
// results/naive_cycle4/include/playground/test_data.hpp:177-196).  Instead of three serial copies
// around one launch, the transfers are pipelined over two streams:
//   B host->device first (every row block needs all of it), then A in row blocks: block i is
//   copied in, multiplied (vk_gemm on its rows) and its C rows copied out on stream i % 2, so the
//   host->device copy of block i+1, the GEMM of block i and the device->host copy of block i-1
//   overlap (the two copy directions run on separate copy engines).
// Device staging buffers and the streams are per device, allocated on first use, grown as needed
// and released by vk_shutdown().  Synchronous: returns when C is in host memory.  Pinned host
// memory (cudaHostAlloc / cudaHostRegister) gives full PCIe bandwidth; pageable memory works too.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "vkgemm.h"
#include "vk_internal.h"

namespace {

struct HostPipe {
    bool ready = false;
    cudaStream_t s[2] = {nullptr, nullptr};
    cudaEvent_t b_ready = nullptr;
    void* dA = nullptr;
    void* dB = nullptr;
    void* dC = nullptr;
    size_t capA = 0, capB = 0, capC = 0;
};

constexpr int kMaxDev = 64;
std::mutex g_host_mu;
HostPipe g_pipe[kMaxDev];

int cuda_err(cudaError_t e, const char* what)
{
    return vk::set_error(VK_ERR_CUDA, "vk_gemm_host: %s: %s", what, cudaGetErrorString(e));
}

int ensure(void** p, size_t* cap, size_t bytes)
{
    if (*cap >= bytes) return VK_OK;
    if (*p != nullptr) {
        cudaFree(*p);
        *p = nullptr;
        *cap = 0;
    }
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) return cuda_err(e, "cudaMalloc staging buffer");
    *cap = bytes;
    return VK_OK;
}

}  // namespace

namespace vk {
void release_host_pipes()
{
    std::lock_guard<std::mutex> lk(g_host_mu);
    int prev = 0;
    cudaGetDevice(&prev);
    for (int d = 0; d < kMaxDev; ++d) {
        HostPipe& hp = g_pipe[d];
        if (!hp.ready) continue;
        cudaSetDevice(d);
        for (auto& st : hp.s) cudaStreamDestroy(st);
        cudaEventDestroy(hp.b_ready);
        cudaFree(hp.dA);
        cudaFree(hp.dB);
        cudaFree(hp.dC);
        hp = HostPipe();
    }
    cudaSetDevice(prev);
}
}  // namespace vk

extern "C" int vk_gemm_host(const vk_gemm_args* a, int32_t block_rows)
{
    if (a == nullptr) return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_host: args is NULL");
    if (a->m < 0 || a->n < 0 || a->k < 0)
        return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_host: negative size");
    if (a->dtype != VK_DTYPE_F16 && a->dtype != VK_DTYPE_F32)
        return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_host: unknown dtype %d", a->dtype);
    if (a->C_f32 != nullptr)
        return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_host: no fp32 copy for host outputs");
    if (block_rows < 0) return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_host: block_rows < 0");
    const int64_t m = a->m, n = a->n, k = a->k;
    const int64_t lda = a->lda ? a->lda : k, ldb = a->ldb ? a->ldb : n, ldc = a->ldc ? a->ldc : n;
    if (lda < k || ldb < n || ldc < n)
        return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_host: leading dimension smaller than the row length");
    if (m == 0 || n == 0) return VK_OK;
    if (a->C == nullptr || (k > 0 && (a->A == nullptr || a->B == nullptr)))
        return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_host: NULL buffer");
    const size_t es = a->dtype == VK_DTYPE_F16 ? 2 : 4;

    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_err(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDev) return vk::set_error(VK_ERR_NO_DEVICE, "vk_gemm_host: device %d", dev);

    std::lock_guard<std::mutex> lk(g_host_mu);  // one host GEMM per process at a time (shared staging)
    HostPipe& hp = g_pipe[dev];
    if (!hp.ready) {
        for (auto& st : hp.s) {
            e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
            if (e != cudaSuccess) return cuda_err(e, "cudaStreamCreate");
        }
        e = cudaEventCreateWithFlags(&hp.b_ready, cudaEventDisableTiming);
        if (e != cudaSuccess) return cuda_err(e, "cudaEventCreate");
        hp.ready = true;
    }
    int rc = ensure(&hp.dA, &hp.capA, static_cast<size_t>(m) * (k > 0 ? k : 1) * es);
    if (rc == VK_OK) rc = ensure(&hp.dB, &hp.capB, static_cast<size_t>(k > 0 ? k : 1) * n * es);
    if (rc == VK_OK) rc = ensure(&hp.dC, &hp.capC, static_cast<size_t>(m) * n * es);
    if (rc != VK_OK) return rc;

    // Row blocks: about 4 blocks (measured best at 4096^3 on B200 among 1-16 blocks), multiples of
    // 256 rows (one pair tile), at least 256 rows.
    int64_t rows = block_rows > 0 ? block_rows : ((m + 3) / 4 + 255) / 256 * 256;
    if (rows < 1) rows = 1;
    const int64_t nblk = (m + rows - 1) / rows;

    if (k > 0) {
        e = cudaMemcpy2DAsync(hp.dB, static_cast<size_t>(n) * es, a->B, static_cast<size_t>(ldb) * es,
                              static_cast<size_t>(n) * es, static_cast<size_t>(k), cudaMemcpyHostToDevice, hp.s[0]);
        if (e != cudaSuccess) return cuda_err(e, "copy B");
        e = cudaEventRecord(hp.b_ready, hp.s[0]);
        if (e != cudaSuccess) return cuda_err(e, "record B");
        e = cudaStreamWaitEvent(hp.s[1], hp.b_ready, 0);
        if (e != cudaSuccess) return cuda_err(e, "wait B");
    }
    for (int64_t b = 0; b < nblk && rc == VK_OK; ++b) {
        cudaStream_t st = hp.s[b & 1];
        const int64_t r0 = b * rows;
        const int64_t rb = (r0 + rows <= m) ? rows : m - r0;
        char* dA = static_cast<char*>(hp.dA) + static_cast<size_t>(r0) * k * es;
        char* dC = static_cast<char*>(hp.dC) + static_cast<size_t>(r0) * n * es;
        if (k > 0) {
            e = cudaMemcpy2DAsync(dA, static_cast<size_t>(k) * es,
                                  static_cast<const char*>(a->A) + static_cast<size_t>(r0) * lda * es,
                                  static_cast<size_t>(lda) * es, static_cast<size_t>(k) * es, static_cast<size_t>(rb),
                                  cudaMemcpyHostToDevice, st);
            if (e != cudaSuccess) {
                rc = cuda_err(e, "copy A block");
                break;
            }
        }
        vk_gemm_args g = *a;
        g.A = dA;
        g.B = hp.dB;
        g.C = dC;
        g.C_f32 = nullptr;
        g.m = rb;
        g.lda = k > 0 ? k : 1;
        g.ldb = n;
        g.ldc = n;
        g.stream = st;
        rc = vk_gemm(&g);
        if (rc != VK_OK) break;
        e = cudaMemcpy2DAsync(static_cast<char*>(a->C) + static_cast<size_t>(r0) * ldc * es,
                              static_cast<size_t>(ldc) * es, dC, static_cast<size_t>(n) * es,
                              static_cast<size_t>(n) * es, static_cast<size_t>(rb), cudaMemcpyDeviceToHost, st);
        if (e != cudaSuccess) rc = cuda_err(e, "copy C block");
    }
    for (auto& st : hp.s) {
        e = cudaStreamSynchronize(st);
        if (e != cudaSuccess && rc == VK_OK) rc = cuda_err(e, "synchronize");
    }
    return rc;
}
