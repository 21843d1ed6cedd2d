// fp32 v0: the CPU ground truth, after results/naive/src/matmul_f32/matmul_f32_v0_cblas.cpp:8-12 (one
// row-major CBLAS sgemm, alpha = 1, beta = 0), written for this repository.
#include "playground/matmul.hpp"
#include "playground/system.hpp"

extern "C" void cblas_sgemm(int order, int transA, int transB, int m, int n, int k, float alpha, const float* A,
                            int lda, const float* B, int ldb, float beta, float* C, int ldc);

namespace playground
{
PLAYGROUND_MATMUL_DEC(float32_t, 0, m, n, k, A, B, C)
{
    cblas_sgemm(101, 111, 111, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), 1.0f, A,
                static_cast<int>(k), B, static_cast<int>(n), 0.0f, C, static_cast<int>(n));
}

// The fp16 helper is declared for every build of the harness; fp32 builds never call it.
void matmulF16GroundTruthF32(size_t, size_t, size_t, const float16_t*, const float16_t*, float32_t*) {}
}  // namespace playground
