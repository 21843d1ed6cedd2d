// Multi-GPU row-block sharding layer (vk_gemm_sharded) for single-process, multi-device callers
// such as the task-1 C++ driver.  The reference is single-GPU (README.md:161) and has no NCCL
// call anywhere; this layer is new.  GPU r computes C[off_r : off_r + rows_r, :] from its own A
// slice and a full copy of B with the same tensor-core kernel as one GPU (local loads only), on
// its own stream; the optional exchange is one NCCL all-gather of the C row blocks over NVLink
// (in place, since C is row-major and the blocks are contiguous), or one broadcast per block
// when the row split is uneven.  Processes-per-GPU callers (torchrun) shard in Python instead and
// use torch.distributed for the same all-gather.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#include "vkgemm.h"
#include "vk_internal.h"

namespace {

// NCCL is resolved lazily with dlopen so that loading the library never pins a libnccl.so.2 of
// its own: inside a PyTorch process the already-loaded (torch-bundled) NCCL is reused, and a
// single-GPU caller never needs NCCL at all.
struct NcclApi {
    bool loaded = false;
    ncclResult_t (*CommInitAll)(ncclComm_t*, int, const int*) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};
NcclApi g_nccl;

template <typename F>
bool bind(void* h, const char* name, F& fn)
{
    fn = reinterpret_cast<F>(dlsym(h, name));
    return fn != nullptr;
}

int load_nccl()
{
    if (g_nccl.loaded) return VK_OK;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) return vk::set_error(VK_ERR_NCCL, "cannot load libnccl.so.2: %s", dlerror());
    bool ok = bind(h, "ncclCommInitAll", g_nccl.CommInitAll) && bind(h, "ncclAllGather", g_nccl.AllGather) &&
              bind(h, "ncclBroadcast", g_nccl.Broadcast) && bind(h, "ncclGroupStart", g_nccl.GroupStart) &&
              bind(h, "ncclGroupEnd", g_nccl.GroupEnd) && bind(h, "ncclCommDestroy", g_nccl.CommDestroy) &&
              bind(h, "ncclCommAbort", g_nccl.CommAbort) &&
              bind(h, "ncclCommGetAsyncError", g_nccl.CommGetAsyncError) &&
              bind(h, "ncclGetErrorString", g_nccl.GetErrorString);
    if (!ok) return vk::set_error(VK_ERR_NCCL, "libnccl.so.2 lacks an expected symbol");
    g_nccl.loaded = true;
    return VK_OK;
}

struct ShardGroup {
    std::vector<int> devices;
    std::vector<ncclComm_t> comms;   // empty until the first all-gather
    std::vector<cudaStream_t> streams;
    std::vector<cudaEvent_t> ev_start, ev_compute, ev_gather;
    // pipelined gather (allgather_c == 2): a copy stream and one "chunk done" event per chunk per GPU
    bool peer_ready = false;
    std::vector<cudaStream_t> copy_streams;
    std::vector<std::vector<cudaEvent_t>> ev_chunk;
};

std::mutex g_shard_mu;
std::vector<ShardGroup*> g_groups;

int cuda_err(cudaError_t e, const char* what)
{
    return vk::set_error(VK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

ShardGroup* find_or_create(const int32_t* devs, int n, int* rc)
{
    for (ShardGroup* g : g_groups) {
        if (static_cast<int>(g->devices.size()) != n) continue;
        bool same = true;
        for (int i = 0; i < n; ++i) same = same && g->devices[i] == devs[i];
        if (same) return g;
    }
    ShardGroup* g = new ShardGroup();
    g->devices.assign(devs, devs + n);
    g->streams.resize(n);
    g->ev_start.resize(n);
    g->ev_compute.resize(n);
    g->ev_gather.resize(n);
    for (int i = 0; i < n; ++i) {
        cudaError_t e = cudaSetDevice(devs[i]);
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&g->streams[i], cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaEventCreate(&g->ev_start[i]);
        if (e == cudaSuccess) e = cudaEventCreate(&g->ev_compute[i]);
        if (e == cudaSuccess) e = cudaEventCreate(&g->ev_gather[i]);
        if (e != cudaSuccess) {
            *rc = cuda_err(e, "shard group setup");
            return nullptr;  // partially built group is leaked deliberately: it is never reused
        }
    }
    g_groups.push_back(g);
    return g;
}

constexpr int kGatherChunks = 2;

// Peer access between every pair of the group's GPUs and the copy streams/events of the pipelined
// gather, once per group.
int ensure_peer(ShardGroup* g)
{
    if (g->peer_ready) return VK_OK;
    const int n = static_cast<int>(g->devices.size());
    g->copy_streams.resize(n);
    g->ev_chunk.assign(n, std::vector<cudaEvent_t>(kGatherChunks));
    for (int i = 0; i < n; ++i) {
        cudaError_t e = cudaSetDevice(g->devices[i]);
        for (int j = 0; j < n && e == cudaSuccess; ++j) {
            if (j == i) continue;
            int can = 0;
            e = cudaDeviceCanAccessPeer(&can, g->devices[i], g->devices[j]);
            if (e == cudaSuccess && can) {
                e = cudaDeviceEnablePeerAccess(g->devices[j], 0);
                if (e == cudaErrorPeerAccessAlreadyEnabled) {
                    cudaGetLastError();  // clear the sticky "already enabled" status
                    e = cudaSuccess;
                }
            }
        }
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&g->copy_streams[i], cudaStreamNonBlocking);
        for (int q = 0; q < kGatherChunks && e == cudaSuccess; ++q)
            e = cudaEventCreateWithFlags(&g->ev_chunk[i][q], cudaEventDisableTiming);
        if (e != cudaSuccess) return cuda_err(e, "peer access / copy streams");
    }
    g->peer_ready = true;
    return VK_OK;
}

int ensure_comms(ShardGroup* g)
{
    if (!g->comms.empty()) return VK_OK;
    int rc = load_nccl();
    if (rc != VK_OK) return rc;
    const int n = static_cast<int>(g->devices.size());
    g->comms.resize(n);
    ncclResult_t r = g_nccl.CommInitAll(g->comms.data(), n, g->devices.data());
    if (r != ncclSuccess) {
        g->comms.clear();
        return vk::set_error(VK_ERR_NCCL, "ncclCommInitAll: %s", g_nccl.GetErrorString(r));
    }
    return VK_OK;
}

// Host-side watchdog of an enqueued collective: polls `query` (1 = complete, 0 = still running,
// -1 = failed) until it completes or `deadline_ms` passes; on a failure or at the deadline it calls
// `abort` once (ncclCommAbort on the real path, which makes the in-flight NCCL kernels give up) and
// returns VK_ERR_NCCL.  A rank that never joins the gather therefore costs the caller an error after
// the deadline instead of a hang.
int watch_collective(const std::function<int()>& query, const std::function<void()>& abort, long long deadline_ms,
                     const char* what, long long* polls_out)
{
    const auto t0 = std::chrono::steady_clock::now();
    long long polls = 0;
    int state = 0;
    while (true) {
        state = query();
        ++polls;
        if (state != 0) break;
        const long long waited =
            std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
        if (waited >= deadline_ms) break;
        std::this_thread::sleep_for(std::chrono::microseconds(polls < 64 ? 5 : 100));
    }
    if (polls_out) *polls_out = polls;
    if (state == 1) return VK_OK;
    abort();
    if (state < 0) return vk::set_error(VK_ERR_NCCL, "%s failed; communicators aborted", what);
    return vk::set_error(VK_ERR_NCCL, "%s did not complete within %lld ms; communicators aborted", what, deadline_ms);
}

}  // namespace

extern "C" int vk_debug_watchdog(int64_t deadline_ms, int32_t done_after_polls, int32_t fail_at_poll, int32_t* aborted,
                                 int64_t* polls)
{
    if (deadline_ms < 0 || aborted == nullptr) return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_debug_watchdog: bad args");
    *aborted = 0;
    long long n = 0;
    auto query = [&]() {
        ++n;
        if (fail_at_poll > 0 && n >= fail_at_poll) return -1;
        if (done_after_polls >= 0 && n > done_after_polls) return 1;
        return 0;
    };
    auto abort = [&]() { ++*aborted; };
    long long p = 0;
    const int rc = watch_collective(query, abort, deadline_ms, "fake collective", &p);
    if (polls) *polls = p;
    return rc;
}

extern "C" int vk_gemm_sharded(const vk_shard_args* a)
{
    if (a == nullptr) return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_sharded: args is NULL");
    if (a->ngpu < 1 || a->ngpu > 64 || a->devices == nullptr || a->A == nullptr || a->B == nullptr ||
        a->C == nullptr)
        return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_sharded: bad ngpu or NULL arrays");
    if (a->m < 0 || a->n < 0 || a->k < 0)
        return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_sharded: negative size");
    if (a->dtype != VK_DTYPE_F16 && a->dtype != VK_DTYPE_F32)
        return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_sharded: unknown dtype");
    const int n_gpu = a->ngpu;
    const size_t esize = a->dtype == VK_DTYPE_F16 ? 2 : 4;

    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) return cuda_err(e, "cudaGetDevice");

    std::lock_guard<std::mutex> lk(g_shard_mu);
    int rc = VK_OK;
    ShardGroup* g = find_or_create(a->devices, n_gpu, &rc);
    if (g == nullptr) {
        cudaSetDevice(prev);
        return rc;
    }
    if (a->allgather_c < 0 || a->allgather_c > 4) {
        cudaSetDevice(prev);
        return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_sharded: allgather_c must be 0..4");
    }
    const bool pipelined = a->allgather_c == 2 && n_gpu > 1;
    const bool gather = a->allgather_c == 1 && n_gpu > 1;
    const bool fused = a->allgather_c == 3 && n_gpu > 1;
    const bool nvls = a->allgather_c == 4 && n_gpu > 1;
    if (nvls && a->dtype != VK_DTYPE_F16) {
        cudaSetDevice(prev);
        return vk::set_error(VK_ERR_UNSUPPORTED, "vk_gemm_sharded: the NVLS gather takes fp16");
    }
    if (fused && (n_gpu - 1 > vk::kMaxPeers || a->dtype != VK_DTYPE_F16)) {
        cudaSetDevice(prev);
        return vk::set_error(VK_ERR_UNSUPPORTED, "vk_gemm_sharded: the fused gather takes fp16 and at most %d GPUs",
                             vk::kMaxPeers + 1);
    }
    if (pipelined || fused) {
        rc = ensure_peer(g);
        if (rc != VK_OK) {
            cudaSetDevice(prev);
            return rc;
        }
    }
    if (gather) {
        rc = ensure_comms(g);
        if (rc != VK_OK) {
            cudaSetDevice(prev);
            return rc;
        }
    }

    std::vector<int64_t> off(n_gpu + 1);
    for (int r = 0; r <= n_gpu; ++r) off[r] = a->m * r / n_gpu;
    bool even = true;
    for (int r = 0; r < n_gpu; ++r) even = even && (off[r + 1] - off[r] == off[1] - off[0]);

    for (int r = 0; r < n_gpu && rc == VK_OK; ++r) {
        e = cudaSetDevice(a->devices[r]);
        if (e == cudaSuccess) e = cudaEventRecord(g->ev_start[r], g->streams[r]);
        if (e != cudaSuccess) {
            rc = cuda_err(e, "shard start");
            break;
        }
        const int nchunks = pipelined ? kGatherChunks : 1;
        const int64_t rows = off[r + 1] - off[r];
        for (int q = 0; q < nchunks && rc == VK_OK; ++q) {
            // pipelined gather: the rows of chunk q go to every peer (copy engines, NVLink) while
            // chunk q+1 is computed
            const int64_t c0 = rows * q / nchunks, c1 = rows * (q + 1) / nchunks;
            vk_gemm_args ga = {};
            ga.A = static_cast<const char*>(a->A[r]) + static_cast<size_t>(c0) * a->k * esize;
            ga.B = a->B[r];
            ga.C = static_cast<char*>(a->C[r]) + static_cast<size_t>(off[r] + c0) * a->n * esize;
            ga.m = c1 - c0;
            ga.n = a->n;
            ga.k = a->k;
            ga.dtype = a->dtype;
            ga.acc = a->acc;
            ga.algo = a->algo;
            ga.stream = g->streams[r];
            if (nvls) {
                // NVLS gather: C[r] is GPU r's view of one multicast buffer (vk_mc_alloc); the epilogue
                // stores every finished box once to the multicast view of its rows and the switch
                // writes it into every GPU's C
                void* mc = vk::mc_lookup(a->devices[r], a->C[r], static_cast<size_t>(a->m) * a->n * esize);
                if (mc == nullptr) {
                    rc = vk::set_error(VK_ERR_INVALID_ARGUMENT,
                                       "vk_gemm_sharded: allgather_c 4 needs C[%d] from vk_mc_alloc", r);
                    break;
                }
                rc = ga.m > 0 ? vk_gemm_mc(&ga, static_cast<char*>(mc) + static_cast<size_t>(off[r] + c0) * a->n * esize)
                              : VK_OK;
            } else if (fused) {
                // fused gather: the epilogue also stores every finished box into the same rows of
                // every peer's C (peer access enabled by ensure_peer)
                void* peers[vk::kMaxPeers];
                int np = 0;
                for (int peer = 0; peer < n_gpu; ++peer)
                    if (peer != r)
                        peers[np++] = static_cast<char*>(a->C[peer]) + static_cast<size_t>(off[r] + c0) * a->n * esize;
                rc = ga.m > 0 ? vk_gemm_peers(&ga, peers, np) : VK_OK;
            } else {
                rc = vk_gemm(&ga);
            }
            if (rc != VK_OK || !pipelined) break;
            e = cudaEventRecord(g->ev_chunk[r][q], g->streams[r]);
            if (e == cudaSuccess) e = cudaStreamWaitEvent(g->copy_streams[r], g->ev_chunk[r][q], 0);
            const size_t bytes = static_cast<size_t>(c1 - c0) * a->n * esize;
            for (int peer = 0; peer < n_gpu && e == cudaSuccess; ++peer) {
                if (peer == r || bytes == 0) continue;
                e = cudaMemcpyPeerAsync(static_cast<char*>(a->C[peer]) + static_cast<size_t>(off[r] + c0) * a->n * esize,
                                        a->devices[peer], ga.C, a->devices[r], bytes, g->copy_streams[r]);
            }
            if (e != cudaSuccess) rc = cuda_err(e, "pipelined gather");
        }
        if (rc != VK_OK) break;
        e = cudaEventRecord(g->ev_compute[r], g->streams[r]);
        if (e != cudaSuccess) rc = cuda_err(e, "shard compute event");
    }

    if (rc == VK_OK && gather) {
        const ncclDataType_t dt = a->dtype == VK_DTYPE_F16 ? ncclHalf : ncclFloat;
        ncclResult_t nr = g_nccl.GroupStart();
        for (int r = 0; r < n_gpu && nr == ncclSuccess; ++r) {
            char* base = static_cast<char*>(a->C[r]);
            if (even) {
                const size_t count = static_cast<size_t>(off[1] - off[0]) * a->n;
                nr = g_nccl.AllGather(base + static_cast<size_t>(off[r]) * a->n * esize, base, count, dt, g->comms[r],
                                   g->streams[r]);
            } else {
                for (int root = 0; root < n_gpu && nr == ncclSuccess; ++root) {
                    const size_t count = static_cast<size_t>(off[root + 1] - off[root]) * a->n;
                    char* blk = base + static_cast<size_t>(off[root]) * a->n * esize;
                    nr = g_nccl.Broadcast(blk, blk, count, dt, root, g->comms[r], g->streams[r]);
                }
            }
        }
        ncclResult_t nr2 = g_nccl.GroupEnd();
        if (nr == ncclSuccess) nr = nr2;
        if (nr != ncclSuccess) rc = vk::set_error(VK_ERR_NCCL, "all-gather of C: %s", g_nccl.GetErrorString(nr));
    }

    float t_compute = 0.f, t_gather = 0.f;
    for (int r = 0; r < n_gpu; ++r) {
        cudaSetDevice(a->devices[r]);
        // the gather-done event follows this GPU's peer copies as well in the pipelined mode
        if (pipelined) cudaStreamWaitEvent(g->streams[r], g->ev_chunk[r][kGatherChunks - 1], 0);
        if (pipelined) {
            cudaEvent_t copies_done;
            if (cudaEventCreateWithFlags(&copies_done, cudaEventDisableTiming) == cudaSuccess) {
                cudaEventRecord(copies_done, g->copy_streams[r]);
                cudaStreamWaitEvent(g->streams[r], copies_done, 0);
                cudaEventDestroy(copies_done);
            }
        }
        if (fused || nvls) {  // C is complete on GPU r once every GPU's kernel (and its stores) finished
            for (int q = 0; q < n_gpu; ++q)
                if (q != r) cudaStreamWaitEvent(g->streams[r], g->ev_compute[q], 0);
        }
        cudaEventRecord(g->ev_gather[r], g->streams[r]);
    }
    if (rc == VK_OK && gather) {
        // NCCL gather under a deadline: every GPU's gather-done event, and no communicator error
        auto query = [&]() {
            int done = 1;
            for (int r = 0; r < n_gpu; ++r) {
                cudaSetDevice(a->devices[r]);
                const cudaError_t q = cudaEventQuery(g->ev_gather[r]);
                if (q == cudaErrorNotReady) {
                    done = 0;
                } else if (q != cudaSuccess) {
                    return -1;
                }
                ncclResult_t ae = ncclSuccess;
                if (g_nccl.CommGetAsyncError(g->comms[r], &ae) != ncclSuccess || ae != ncclSuccess) return -1;
            }
            return done;
        };
        auto abort = [&]() {
            for (ncclComm_t c : g->comms) g_nccl.CommAbort(c);
            g->comms.clear();  // the next call builds new communicators
        };
        rc = watch_collective(query, abort, vk::gather_timeout_ms(), "NCCL all-gather of C", nullptr);
    }
    for (int r = 0; r < n_gpu; ++r) {
        cudaSetDevice(a->devices[r]);
        e = cudaStreamSynchronize(g->streams[r]);
        if (e != cudaSuccess && rc == VK_OK) rc = cuda_err(e, "shard synchronize");
        if (rc == VK_OK) {
            float tc = 0.f, tg = 0.f;
            cudaEventElapsedTime(&tc, g->ev_start[r], g->ev_compute[r]);
            cudaEventElapsedTime(&tg, g->ev_compute[r], g->ev_gather[r]);
            if (tc > t_compute) t_compute = tc;
            if (tg > t_gather) t_gather = tg;
        }
    }
    cudaSetDevice(prev);
    if (rc == VK_OK && a->times_ms != nullptr) {
        a->times_ms[0] = t_compute;
        a->times_ms[1] = (gather || pipelined || fused || nvls) ? t_gather : 0.f;
    }
    return rc;
}

extern "C" int vk_shutdown(void)
{
    std::lock_guard<std::mutex> lk(g_shard_mu);
    int prev = 0;
    cudaGetDevice(&prev);
    for (ShardGroup* g : g_groups) {
        for (ncclComm_t c : g->comms) g_nccl.CommDestroy(c);
        for (size_t i = 0; i < g->devices.size(); ++i) {
            cudaSetDevice(g->devices[i]);
            if (g->peer_ready) {
                cudaStreamDestroy(g->copy_streams[i]);
                for (cudaEvent_t ev : g->ev_chunk[i]) cudaEventDestroy(ev);
            }
            cudaStreamDestroy(g->streams[i]);
            cudaEventDestroy(g->ev_start[i]);
            cudaEventDestroy(g->ev_compute[i]);
            cudaEventDestroy(g->ev_gather[i]);
        }
        delete g;
    }
    g_groups.clear();
    cudaSetDevice(prev);
    vk::release_device_state();
    vk::release_host_pipes();
    return VK_OK;
}
