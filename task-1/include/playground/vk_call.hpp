// Failure convention for version files that call the vkgemm C ABI: a non-zero status is reported
// with the library's message and ends the program, as PLAYGROUND_CHECK does in the reference.
#pragma once

#include <cstdio>
#include <cstdlib>

#include "vkgemm.h"

namespace playground
{
inline void vkCheck(int rc, const char* what)
{
    if (rc != VK_OK) {
        std::fprintf(stderr, "[Playground] %s failed (%d): %s\n", what, rc, vk_last_error_string());
        std::exit(EXIT_FAILURE);
    }
}
}  // namespace playground
