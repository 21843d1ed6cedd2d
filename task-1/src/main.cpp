// Task-1 driver, re-created for this repository: results/naive_cycle6/src/main.cpp:1-127.
//
// Same CLI, same timing rubric (10 warm-up calls, then 100 calls each bracketed by CUDA events on the
// legacy default stream and followed by an event synchronize; v0 runs 10 rounds on the CPU timed with
// std::chrono), same error check and the same result line:
//   [Playground] Result >>> TFLOPS: X; Average Error: Y
// Additive lines follow it: the rel-Frobenius and per-element errors of an fp32 copy of C (from one
// extra verification launch of the same kernel), the SM clock the kernels ran at (in-kernel probe),
// the seed, and the fraction of the 2.25 PFLOP/s dense fp16 figure.
//
// Additive multi-GPU mode (--gpus P, GPU versions only): the same problem split into P row blocks of A
// and C over devices 0..P-1 with B copied to each, run through vk_gemm_sharded with the all-gather of C
// chosen by --allgather (none | nccl | pipelined | fused | nvls); the timed loop and the result line are
// those of one GPU, the time of a call is its slowest GPU's compute plus the gather.
#include <chrono>
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "playground/cli.hpp"
#include "playground/matmul.hpp"
#include "playground/system.hpp"
#include "playground/test_data.hpp"
#include "playground/vk_call.hpp"
#include "vkgemm.h"

#ifndef TARGET_BIN_OUTPUT_NAME
#define TARGET_BIN_OUTPUT_NAME "task1"
#endif

constexpr bool USING_CPU_MATMUL = playground::params::MatmulVersion == playground::PG_MATMUL_FP16_CBLAS;

namespace playground
{
PLAYGROUND_MATMUL_DEC(params::DataType, params::MatmulVersion, M, N, K, A, B, C);
}

namespace
{
using namespace playground;

// The kernel each fp16 GPU version runs (the mapping of vk_matmul_f16), for the verification launch
// that also writes an fp32 copy of C.
[[maybe_unused]] void verifyF32Copy(std::uint32_t m, std::uint32_t n, std::uint32_t k, const float16_t* dA, const float16_t* dB,
                   std::vector<float32_t>& out)
{
    vk_gemm_args a{};
    a.A = dA;
    a.B = dB;
    a.m = m;
    a.n = n;
    a.k = k;
    a.dtype = VK_DTYPE_F16;
    switch (params::MatmulVersion) {
        case 2: a.algo = VK_ALGO_TC_2SM; a.acc = VK_ACC_F16; break;
        case 3: a.algo = VK_ALGO_TC_1SM; a.acc = VK_ACC_F32; break;
        case 4: a.algo = VK_ALGO_SIMT; a.acc = VK_ACC_F32; break;
        default: a.algo = VK_ALGO_TC_2SM; a.acc = VK_ACC_F32; break;
    }
    CudaDeviceMemPtr<float16_t> c16(static_cast<size_t>(m) * n);
    CudaDeviceMemPtr<float32_t> c32(static_cast<size_t>(m) * n);
    a.C = c16.get();
    a.C_f32 = c32.get();
    vkCheck(vk_gemm(&a), "verification launch");
    out.resize(static_cast<size_t>(m) * n);
    PLAYGROUND_CHECK(cudaMemcpy(out.data(), c32.get(), out.size() * sizeof(float32_t), cudaMemcpyDeviceToHost) ==
                     cudaSuccess);
}

void test(std::uint32_t m, std::uint32_t n, std::uint32_t k, std::uint32_t nWarmupRound, std::uint32_t nTestRound,
          const DataOptions& opt, const std::string& jsonPath)
{
    TestData testData(m, n, k, opt);
    float32_t totalMilliSecs = 0.0f;
    std::printf("[Playground] Start Testing for GEMM Version %u with DType %s ...\n",
                static_cast<unsigned>(params::MatmulVersion), params::DataTypeName.data());

    params::DataType* Aptr = nullptr;
    params::DataType* Bptr = nullptr;
    params::DataType* Cptr = nullptr;
    auto matmulFn = [&Aptr, &Bptr, &Cptr, m, n, k]() {
        PLAYGOUND_MATMUL_CALL(params::MatmulVersion, m, n, k, Aptr, Bptr, Cptr);
    };

    double kernelMhz = 0.0;
    std::vector<float32_t> c32;
    if constexpr (!USING_CPU_MATMUL) {
        cudaEvent_t start, stop;
        cudaEventCreate(&start);
        cudaEventCreate(&stop);
        float32_t runtime = 0.0f;
        testData.initDeviceData();
        Aptr = testData.get_mutable_d_A_ptr();
        Bptr = testData.get_mutable_d_B_ptr();
        Cptr = testData.get_mutable_d_C_ptr();
        for (std::uint32_t i = 0; i < nWarmupRound; ++i) matmulFn();
        vk_set_option("clock_probe", 1);
        std::uint64_t probe[3];
        vk_read_clock_probe(0, probe, 1);
        for (std::uint32_t i = 0; i < nTestRound; ++i) {
            cudaEventRecord(start, nullptr);
            matmulFn();
            cudaEventRecord(stop, nullptr);
            cudaEventSynchronize(stop);
            cudaEventElapsedTime(&runtime, start, stop);
            totalMilliSecs += runtime;
        }
        if (vk_read_clock_probe(0, probe, 1) == VK_OK && probe[1] > 0)
            kernelMhz = static_cast<double>(probe[0]) / static_cast<double>(probe[1]) * 1e3;
        vk_set_option("clock_probe", 0);
        testData.copyResultD2H();
#if defined(TEST_FLOAT16)
        verifyF32Copy(m, n, k, Aptr, Bptr, c32);
#else
        const params::DataType* c = testData.get_mutable_C_ptr();
        c32.assign(c, c + static_cast<size_t>(m) * n);
#endif
        std::uint64_t word = 0;
        vkCheck(vk_device_error(0, &word, 1), "vk_device_error");
        PLAYGROUND_CHECK(word == 0);
        cudaEventDestroy(start);
        cudaEventDestroy(stop);
    } else {
        Aptr = testData.get_mutable_A_ptr();
        Bptr = testData.get_mutable_B_ptr();
        Cptr = testData.get_mutable_C_ptr();
        nTestRound = 10;  // the reference times 10 CPU rounds
        for (std::uint32_t i = 0; i < nTestRound; ++i) {
            auto t0 = std::chrono::high_resolution_clock::now();
            matmulFn();
            auto t1 = std::chrono::high_resolution_clock::now();
            totalMilliSecs += std::chrono::duration<float32_t, std::milli>(t1 - t0).count();
        }
        const params::DataType* c = testData.get_mutable_C_ptr();
        c32.resize(static_cast<size_t>(m) * n);
        for (size_t i = 0; i < c32.size(); ++i) c32[i] = static_cast<float32_t>(c[i]);
    }
    if constexpr (!USING_CPU_MATMUL) cudaDeviceSynchronize();
    std::printf("[Playground] Calculating Finished\n");

    const float32_t avgErr = testData.calculateAvgErr();
    const float32_t msecPerMatrixMul = totalMilliSecs / static_cast<float32_t>(nTestRound);
    const float64_t flopsPerMatrixMul = 2.0 * m * n * k;
    const float64_t tflops = (flopsPerMatrixMul * 1.0e-12) / (msecPerMatrixMul / 1000.0);
    std::printf("[Playground] Result >>> TFLOPS: %g; Average Error: %g\n", tflops, avgErr);

    const float64_t frob = testData.relFrobenius(c32);
    const float64_t elem = testData.maxElemRel(c32);
    std::printf("[Playground] Extra >>> RelFrobenius(fp32 copy): %.3e; MaxElemRel(tau=1e-2*RMS): %.3e; "
                "KernelSmMHz: %.0f; Seed: %llu; PctOf2250TF: %.4f\n",
                frob, elem, kernelMhz, static_cast<unsigned long long>(testData.seedUsed()), tflops / 2250.0);
    if (!jsonPath.empty()) {
        if (FILE* f = std::fopen(jsonPath.c_str(), "a")) {
            std::fprintf(f,
                         "{\"binary\": \"%s\", \"m\": %u, \"n\": %u, \"k\": %u, \"warmup\": %u, \"iters\": %u, "
                         "\"tflops\": %.4f, \"avg_err\": %.6g, \"rel_frobenius\": %.6g, \"max_elem_rel\": %.6g, "
                         "\"kernel_sm_mhz\": %.1f, \"seed\": %llu}\n",
                         TARGET_BIN_OUTPUT_NAME, m, n, k, nWarmupRound, nTestRound, tflops, avgErr, frob, elem,
                         kernelMhz, static_cast<unsigned long long>(testData.seedUsed()));
            std::fclose(f);
        }
    }
}
// vk_gemm_sharded's arguments for this build's version: dtype, accumulate tier and kernel.
void shardKind(vk_shard_args& a)
{
#if defined(TEST_FLOAT16)
    a.dtype = VK_DTYPE_F16;
    switch (params::MatmulVersion) {
        case 2: a.algo = VK_ALGO_TC_2SM; a.acc = VK_ACC_F16; break;
        case 3: a.algo = VK_ALGO_TC_1SM; a.acc = VK_ACC_F32; break;
        case 4: a.algo = VK_ALGO_SIMT; a.acc = VK_ACC_F32; break;
        default: a.algo = VK_ALGO_TC_2SM; a.acc = VK_ACC_F32; break;
    }
#else
    a.dtype = VK_DTYPE_F32;
    a.acc = VK_ACC_F32;
    a.algo = VK_ALGO_FFMA;
#endif
}

void testSharded(std::uint32_t m, std::uint32_t n, std::uint32_t k, std::uint32_t nWarmupRound, std::uint32_t nTestRound,
                 const DataOptions& opt, int gpus, const std::string& mode)
{
    int count = 0;
    PLAYGROUND_CHECK(cudaGetDeviceCount(&count) == cudaSuccess);
    if (gpus < 1 || gpus > count)
        throw std::invalid_argument("--gpus " + std::to_string(gpus) + ": " + std::to_string(count) + " GPU(s) visible");
    const int gather = mode == "none" ? 0 : mode == "nccl" ? 1 : mode == "pipelined" ? 2 : mode == "fused" ? 3
                     : mode == "nvls" ? 4 : -1;
    if (gather < 0) throw std::invalid_argument("--allgather must be none, nccl, pipelined, fused or nvls");
    TestData testData(m, n, k, opt);
    std::printf("[Playground] Start Testing for GEMM Version %u with DType %s on %d GPU(s), all-gather %s ...\n",
                static_cast<unsigned>(params::MatmulVersion), params::DataTypeName.data(), gpus, mode.c_str());
    const size_t es = sizeof(params::DataType);
    std::vector<int32_t> devs(gpus);
    std::vector<int64_t> off(gpus + 1);
    for (int r = 0; r <= gpus; ++r) off[r] = static_cast<int64_t>(m) * r / gpus;
    std::vector<void*> A(gpus), B(gpus), C(gpus);
    void* mc = nullptr;
    for (int r = 0; r < gpus; ++r) devs[r] = r;
    if (gather == 4) vkCheck(vk_mc_alloc(gpus, devs.data(), static_cast<size_t>(m) * n * es, C.data(), &mc), "vk_mc_alloc");
    for (int r = 0; r < gpus; ++r) {
        PLAYGROUND_CHECK(cudaSetDevice(r) == cudaSuccess);
        const size_t rows = static_cast<size_t>(off[r + 1] - off[r]);
        PLAYGROUND_CHECK(cudaMalloc(&A[r], std::max<size_t>(rows * k * es, 16)) == cudaSuccess);
        PLAYGROUND_CHECK(cudaMalloc(&B[r], static_cast<size_t>(k) * n * es) == cudaSuccess);
        if (gather != 4) PLAYGROUND_CHECK(cudaMalloc(&C[r], static_cast<size_t>(m) * n * es) == cudaSuccess);
        PLAYGROUND_CHECK(cudaMemcpy(A[r], testData.get_mutable_A_ptr() + off[r] * k, rows * k * es,
                                    cudaMemcpyHostToDevice) == cudaSuccess);
        PLAYGROUND_CHECK(cudaMemcpy(B[r], testData.get_mutable_B_ptr(), static_cast<size_t>(k) * n * es,
                                    cudaMemcpyHostToDevice) == cudaSuccess);
    }
    vk_shard_args a{};
    a.ngpu = gpus;
    a.devices = devs.data();
    a.A = A.data();
    a.B = B.data();
    a.C = C.data();
    a.m = m;
    a.n = n;
    a.k = k;
    shardKind(a);
    a.allgather_c = gather;
    float times[2] = {0.f, 0.f};
    a.times_ms = times;
    for (std::uint32_t i = 0; i < nWarmupRound; ++i) vkCheck(vk_gemm_sharded(&a), "vk_gemm_sharded");
    float32_t totalMilliSecs = 0.0f;
    for (std::uint32_t i = 0; i < nTestRound; ++i) {  // each call returns after every GPU (and the gather)
        vkCheck(vk_gemm_sharded(&a), "vk_gemm_sharded");
        totalMilliSecs += times[0] + times[1];
    }
    // C on the host: every GPU's own rows (without a gather), or GPU 0's full C (with one), and every
    // other GPU's full C must then be bitwise the same
    params::DataType* hC = testData.get_mutable_C_ptr();
    bool same = true;
    for (int r = 0; r < gpus; ++r) {
        PLAYGROUND_CHECK(cudaSetDevice(r) == cudaSuccess);
        if (gather == 0 || r == 0) {
            const size_t r0 = gather == 0 ? static_cast<size_t>(off[r]) : 0;
            const size_t rows = gather == 0 ? static_cast<size_t>(off[r + 1] - off[r]) : m;
            PLAYGROUND_CHECK(cudaMemcpy(hC + r0 * n, static_cast<char*>(C[r]) + r0 * n * es, rows * n * es,
                                        cudaMemcpyDeviceToHost) == cudaSuccess);
        } else {
            std::vector<params::DataType> other(static_cast<size_t>(m) * n);
            PLAYGROUND_CHECK(cudaMemcpy(other.data(), C[r], other.size() * es, cudaMemcpyDeviceToHost) == cudaSuccess);
            same = same && std::memcmp(other.data(), hC, other.size() * es) == 0;
        }
    }
    for (int r = 0; r < gpus; ++r) {
        cudaSetDevice(r);
        cudaFree(A[r]);
        cudaFree(B[r]);
        if (gather != 4) cudaFree(C[r]);
    }
    if (mc != nullptr) vkCheck(vk_mc_free(mc), "vk_mc_free");
    cudaSetDevice(0);
    std::printf("[Playground] Calculating Finished\n");
    const float32_t avgErr = testData.calculateAvgErr();
    const float32_t msecPerMatrixMul = totalMilliSecs / static_cast<float32_t>(nTestRound);
    const float64_t tflops = (2.0 * m * n * k * 1.0e-12) / (msecPerMatrixMul / 1000.0);
    std::printf("[Playground] Result >>> TFLOPS: %g; Average Error: %g\n", tflops, avgErr);
    std::printf("[Playground] Sharded >>> GPUs: %d; AllGather: %s; AllGpusEqual: %d; ComputeMs: %.4f; GatherMs: %.4f\n",
                gpus, mode.c_str(), same ? 1 : 0, times[0], times[1]);
    PLAYGROUND_CHECK(same);
}
}  // namespace

int main(int argc, const char* argv[])
{
    try {
        playground::Cli cli(argc, argv);
        if (cli.has("h")) {
            std::printf("%s\n%s", TARGET_BIN_OUTPUT_NAME, playground::Cli::usage());
            return 0;
        }
        playground::DataOptions opt;
        opt.seed = cli.i64("seed", -1);
        opt.dist = cli.str("dist", "normal");
        opt.lo = cli.f64("lo", -1.0);
        opt.hi = cli.f64("hi", 1.0);
        if (opt.dist != "normal" && opt.dist != "uniform") throw std::invalid_argument("--dist must be normal or uniform");
        if (cli.has("gpus")) {
            if constexpr (USING_CPU_MATMUL) throw std::invalid_argument("--gpus needs a GPU version (v >= 1)");
            testSharded(cli.u32("m", 4096), cli.u32("n", 4096), cli.u32("k", 4096), cli.u32("w", 10),
                        cli.u32("t", 100), opt, static_cast<int>(cli.u32("gpus", 1)), cli.str("allgather", "nccl"));
            return 0;
        }
        test(cli.u32("m", 4096), cli.u32("n", 4096), cli.u32("k", 4096), cli.u32("w", 10), cli.u32("t", 100), opt,
             cli.str("json", ""));
    } catch (const std::exception& e) {
        std::fprintf(stderr, "[Playground] %s\n%s", e.what(), playground::Cli::usage());
        return 2;
    }
    return 0;
}
