// The versioned GEMM entry point of task-1 (plugin interface), re-created with the reference's names
// so that version files and drivers written for the reference compile unchanged:
// results/naive_cycle4/include/playground/matmul.hpp:11-39.
//   template <typename DType, uint8_t Version> void matmul(m, n, k, A, B, C) = delete;
//   PLAYGROUND_MATMUL_DEC  declares/defines one full specialisation;
//   PLAYGOUND_MATMUL_CALL  calls the specialisation for the element type of A (the reference's
//                          spelling, kept so existing callers compile).
// Row-major A[m x k], B[k x n], C[m x n]; C = A * B.  v0 takes host pointers, v>=1 device pointers.
#pragma once

#include <cstdint>
#include <type_traits>

#include "playground/system.hpp"

namespace playground
{
template <typename DType, std::uint8_t Version>
void matmul(size_t m, size_t n, size_t k, const DType* A, const DType* B, DType* C) = delete;

#define PLAYGROUND_MATMUL_DEC(DType, Version, m, n, k, A, B, C) \
    template <>                                                 \
    void matmul<DType, Version>(size_t m, size_t n, size_t k, const DType* A, const DType* B, DType* C)

#define PLAYGOUND_MATMUL_CALL(Version, m, n, k, A, B, C) \
    ::playground::matmul<::std::remove_cvref_t<decltype(*A)>, Version>(m, n, k, A, B, C)

constexpr std::uint8_t PG_MATMUL_FP16_CBLAS = 0;
constexpr std::uint8_t PG_MATMUL_FP32_CBLAS = 0;

// fp16 v0: widen to fp32, single-precision GEMM on the CPU, round to fp16.
PLAYGROUND_MATMUL_DEC(float16_t, PG_MATMUL_FP16_CBLAS, m, n, k, A, B, C);
// fp32 v0: single-precision GEMM on the CPU.
PLAYGROUND_MATMUL_DEC(float32_t, PG_MATMUL_FP32_CBLAS, m, n, k, A, B, C);

// fp32 result of the fp16 v0 before its final rounding (verification of the fp32 copy of C).
void matmulF16GroundTruthF32(size_t m, size_t n, size_t k, const float16_t* A, const float16_t* B,
                             float32_t* C32);
}  // namespace playground
