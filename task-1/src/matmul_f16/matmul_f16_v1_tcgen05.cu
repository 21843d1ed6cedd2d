// fp16 version 1: tcgen05 pair kernel, fp32 accumulate (2 CTAs per 256x256 tile).
// One-line dispatcher into the vkgemm C ABI (include/vkgemm.h), in the reference's pattern of a thin
// version file over a shared kernel library.
#include "playground/matmul.hpp"
#include "playground/vk_call.hpp"

namespace playground
{
PLAYGROUND_MATMUL_DEC(float16_t, 1, m, n, k, A, B, C)
{
    vkCheck(vk_matmul_f16(1, m, n, k, A, B, C), "vk_matmul_f16");
}
}  // namespace playground
