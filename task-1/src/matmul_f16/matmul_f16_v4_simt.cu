// fp16 version 4: predicated CUDA-core kernel, fp32 accumulate, any alignment.
// One-line dispatcher into the vkgemm C ABI (include/vkgemm.h), in the reference's pattern of a thin
// version file over a shared kernel library.
#include "playground/matmul.hpp"
#include "playground/vk_call.hpp"

namespace playground
{
PLAYGROUND_MATMUL_DEC(float16_t, 4, m, n, k, A, B, C)
{
    vkCheck(vk_matmul_f16(4, m, n, k, A, B, C), "vk_matmul_f16");
}
}  // namespace playground
