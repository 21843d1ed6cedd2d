// TEST INFRASTRUCTURE ONLY -- never linked into the product library.
//
// C-ABI shim around the reference's own v0 ground truth so Python tests and the
// bench's CPU arm can call it through ctypes.  The two specializations it calls,
// playground::matmul<float16_t,0> and playground::matmul<float32_t,0>, are compiled
// unmodified from the reference sources by oracle/Makefile:
//   results/naive/src/matmul_f16/matmul_f16_v0_cblas.cpp:11-26  (fp16 -> fp32 sgemm -> fp16)
//   results/naive/src/matmul_f32/matmul_f32_v0_cblas.cpp:8-12   (fp32 sgemm)
// The declarations come from the reference header results/naive_cycle4/include/playground/matmul.hpp:28-39.
#include <cstddef>
#include <cstdint>

#include "playground/matmul.hpp"

extern "C" {

void vk_ref_v0_f16(size_t m, size_t n, size_t k, const uint16_t* A, const uint16_t* B,
                   uint16_t* C)
{
    using playground::float16_t;
    playground::matmul<float16_t, playground::PG_MATMUL_FP16_CBLAS>(
        m, n, k, reinterpret_cast<const float16_t*>(A), reinterpret_cast<const float16_t*>(B),
        reinterpret_cast<float16_t*>(C));
}

void vk_ref_v0_f32(size_t m, size_t n, size_t k, const float* A, const float* B, float* C)
{
    playground::matmul<playground::float32_t, playground::PG_MATMUL_FP32_CBLAS>(m, n, k, A, B, C);
}

}  // extern "C"
