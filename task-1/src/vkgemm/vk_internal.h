// Internal helpers shared by the translation units of libvkgemm.so (not part of the C ABI).
#pragma once

#include <cstddef>

namespace vk {
// Most peer C buffers one launch of the fused all-gather (vk_gemm_peers) stores into: an 8-GPU node.
constexpr int kMaxPeers = 7;

// Records a thread-local error message (read back by vk_last_error_string) and returns `code`.
int set_error(int code, const char* fmt, ...);
// Frees per-device scratch owned by the library (vk_shutdown).
void release_device_state();
// Frees the host-buffer pipeline's staging buffers and streams (vk_shutdown).
void release_host_pipes();
// Multicast view of [ptr, ptr + bytes) on device `dev` when that range lies inside the unicast view of
// a live multicast team (vk_mc_alloc / vk_mc_attach), else nullptr.
void* mc_lookup(int dev, const void* ptr, size_t bytes);
// Host-side deadline of the NCCL all-gather in vk_gemm_sharded, milliseconds (option "gather_timeout_ms").
long long gather_timeout_ms();
}  // namespace vk
