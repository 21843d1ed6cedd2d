// fp32 version 1: register-blocked CUDA-core SGEMM (FFMA), through the vkgemm C ABI.
#include "playground/matmul.hpp"
#include "playground/vk_call.hpp"

namespace playground
{
PLAYGROUND_MATMUL_DEC(float32_t, 1, m, n, k, A, B, C)
{
    vkCheck(vk_matmul_f32(1, m, n, k, A, B, C), "vk_matmul_f32");
}
}  // namespace playground
