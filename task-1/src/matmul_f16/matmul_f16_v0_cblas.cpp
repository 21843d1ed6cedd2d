// fp16 v0: the CPU ground truth of the harness, written for this repository after the reference's
// results/naive/src/matmul_f16/matmul_f16_v0_cblas.cpp:11-26: widen A and B exactly to fp32, one
// row-major single-precision GEMM through the CBLAS interface (alpha = 1, beta = 0), round each
// result to fp16 with round-to-nearest-even.  Linked against the OpenBLAS in this image.
#include <vector>

#include "playground/matmul.hpp"
#include "playground/system.hpp"

extern "C" void cblas_sgemm(int order, int transA, int transB, int m, int n, int k, float alpha, const float* A,
                            int lda, const float* B, int ldb, float beta, float* C, int ldc);

namespace playground
{
namespace
{
constexpr int kRowMajor = 101, kNoTrans = 111;  // CBLAS enumerator values

void sgemmF16Inputs(size_t m, size_t n, size_t k, const float16_t* A, const float16_t* B, float32_t* C32)
{
    std::vector<float32_t> a(m * k), b(k * n);
    for (size_t i = 0; i < a.size(); ++i) a[i] = __half2float(A[i]);
    for (size_t i = 0; i < b.size(); ++i) b[i] = __half2float(B[i]);
    cblas_sgemm(kRowMajor, kNoTrans, kNoTrans, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), 1.0f,
                a.data(), static_cast<int>(k), b.data(), static_cast<int>(n), 0.0f, C32, static_cast<int>(n));
}
}  // namespace

PLAYGROUND_MATMUL_DEC(float16_t, 0, m, n, k, A, B, C)
{
    std::vector<float32_t> c(m * n);
    sgemmF16Inputs(m, n, k, A, B, c.data());
    for (size_t i = 0; i < c.size(); ++i) C[i] = __float2half_rn(c[i]);
}

void matmulF16GroundTruthF32(size_t m, size_t n, size_t k, const float16_t* A, const float16_t* B, float32_t* C32)
{
    sgemmF16Inputs(m, n, k, A, B, C32);
}
}  // namespace playground
