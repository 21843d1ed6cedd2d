// C-ABI implementation of include/vkgemm.h: argument checking, kernel selection, TMA tensor-map
// encoding, persistent-grid sizing and launches.  Single translation unit for all device code
// (no relocatable device code needed).
//
// Host-side state mirrors what the reference kernels keep in function-static variables
// (results/ralph_loop_fable/src/matmul_f16/matmul_f16_v42_shfl2.cu:496-518: SM count, smem
// attribute, workspace) but is per device, mutex-protected, and released by vk_shutdown().
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "vkgemm.h"
#include "ptx.cuh"
#include "simt_gemm.cuh"
#include "tc_gemm.cuh"
#include "vk_internal.h"

namespace vk {

__global__ void selftest_wait_kernel(unsigned long long timeout_ns)
{
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);
        fence_mbar_init();
        // Nothing ever arrives: the bounded wait must give up and record kErrWaitSelftest.
        (void)mbar_wait(smem_u32(&bar), 0u, timeout_ns, kErrWaitSelftest, 0);
    }
}

// ------------------------------------------------------------------------------------------
// Errors
// ------------------------------------------------------------------------------------------
static thread_local std::string t_last_error;

int set_error(int code, const char* fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

static int cuda_fail(cudaError_t e, const char* what)
{
    return set_error(VK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define VK_CUDA_TRY(expr)                                  \
    do {                                                   \
        cudaError_t _e = (expr);                           \
        if (_e != cudaSuccess) return cuda_fail(_e, #expr); \
    } while (0)

// ------------------------------------------------------------------------------------------
// Per-device state
// ------------------------------------------------------------------------------------------
constexpr int kMaxDevices = 64;
constexpr int kMaxKernels = 32;

struct KernelSlot {
    const void* fn = nullptr;
    int max_clusters = 0;  // co-resident clusters (CG=2) or CTAs (CG=1) at this smem size
};

// Fixed scratch for vk_gemm_noalloc: the tail-split partials and arrival counters of one call,
// passed instead of the library's cudaMalloc'd workspace.
struct FixedScratch {
    float* ws;
    int* counters;
    size_t ws_bytes, ctr_bytes;
};

// One encoded tensor map, keyed by everything the encoding depends on.  A map holds only the base
// address, shape, pitch and box, so a hit stays valid even after the buffer is freed and another
// allocation reuses the address.
struct TmapEntry {
    const void* base = nullptr;
    int64_t rows = 0, cols = 0, ld = 0;
    uint32_t box_cols = 0, box_rows = 0;
    int kind = -1;  // 0 = operand (128-byte swizzle), 1 = C store map (64-byte swizzle)
    CUtensorMap map;
};

struct DeviceState {
    std::atomic<bool> ready{false};
    // Recently encoded tensor maps (round-robin replacement): the reference driver's loop calls
    // with the same pointers and shapes every iteration, and encoding costs host time that sits
    // between its start event and the kernel.
    static constexpr int kTmapCache = 16;
    std::mutex tmap_mu;
    TmapEntry tmaps[kTmapCache];
    int tmap_next = 0;
    // Device address of this file's static no-allocation scratch array, looked up once per device
    // by the first vk_gemm_noalloc call made with the device current.
    std::atomic<void*> noalloc_scratch{nullptr};
    int sm_count = 0;
    // Append-only table; num_kernels is published with release after the new slot is written, so
    // the lock-free scan in kernel_slot sees only complete slots.
    KernelSlot kernels[kMaxKernels];
    std::atomic<int> num_kernels{0};
    // Tail-split scratch, one per stream that launched a split GEMM (launches on different streams
    // may overlap on the GPU, so they must not share partials or counters), allocated on first
    // need: fp32 partials for at most one unit per persistent CTA (sm_count x 128 x 256 floats,
    // 19.4 MB on 148 SMs) and 4 arrival counters per CTA (zeroed at allocation; each reduction
    // leaves them zero again).
    struct StreamScratch {
        cudaStream_t stream = nullptr;
        float* ws = nullptr;
        int* counters = nullptr;
        // repack buffers for operands whose pitch breaks the TMA rule (grown on demand)
        void* pack[2] = {nullptr, nullptr};
        size_t pack_bytes[2] = {0, 0};
    };
    static constexpr int kMaxStreams = 32;
    StreamScratch scratch[kMaxStreams];
    int num_scratch = 0;
    size_t ws_bytes = 0, ctr_bytes = 0;
};

static std::mutex g_mu;
static DeviceState g_dev[kMaxDevices];
static std::atomic<unsigned long long> g_timeout_ns{2000000000ull};
static std::atomic<int> g_tail_split{1};
static std::atomic<int> g_tail_nsplit{1};
static std::atomic<int> g_tail_first{1};
static std::atomic<int> g_tma_store{1};
// Operand tiles are loaded with an L2 evict_last policy: they stay resident over the C stores,
// the k-slice partials and whatever the previous kernel left dirty in L2 (+0.4 to +1 % measured).
static std::atomic<int> g_l2_evict_last{1};
static std::atomic<int> g_raster_group{8};
// k depth per pipeline stage of the 256-column pair kernel.  Every stage ends with tcgen05.commit
// to both CTAs' "empty" barriers, and those commits measurably throttle the tensor pipe; 128-deep
// stages (3 x 64 KB) halve them per MMA and beat 64-deep ones (6 x 32 KB) at every size measured.
static std::atomic<int> g_bk_2sm256{128};
static std::atomic<int> g_sgemm_v2{1};
static std::atomic<int> g_sgemm_paired{1};
static std::atomic<int> g_repack{1};
static std::atomic<int> g_clock_probe_on{0};
// Two accumulation chains per unit (kernel template CH): 0 = never (default), 1 = when K > kChainsMinK,
// 2 = always.  Measured on B200: at 16384^3 the fp32 result's per-element error falls from 3.7e-3 to
// 1.9e-3 at no cost, but the 2048 x 16384 x 16384 shard of an 8-GPU split runs 19 % slower (the
// epilogue no longer overlaps the next tile), so it is opt-in.
static std::atomic<int> g_k_chains{0};
static constexpr long long kChainsMinK = 8192;
// Deadline of the NCCL all-gather in vk_gemm_sharded (after it, the communicators are aborted).
static std::atomic<long long> g_gather_timeout_ms{60000};
long long gather_timeout_ms() { return g_gather_timeout_ms.load(std::memory_order_relaxed); }
// Devices (bit per ordinal < 31) on which each SGEMM variant's shared-memory attribute is set.
static std::atomic<int> g_sgemm_attr_mask[3] = {{0}, {0}, {0}};
static std::atomic<int> g_trace_on{0};

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn g_encode = nullptr;

static int init_device_locked(int dev)
{
    DeviceState& st = g_dev[dev];
    if (st.ready.load(std::memory_order_acquire)) return VK_OK;
    cudaDeviceProp prop;
    VK_CUDA_TRY(cudaGetDeviceProperties(&prop, dev));
    if (prop.major != 10 || prop.minor != 0)
        return set_error(VK_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a only", dev,
                         prop.major, prop.minor);
    st.sm_count = prop.multiProcessorCount;
    if (g_encode == nullptr) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        VK_CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || fn == nullptr)
            return set_error(VK_ERR_CUDA, "cuTensorMapEncodeTiled not available from the driver");
        g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
    st.ready.store(true, std::memory_order_release);
    return VK_OK;
}

int current_device(int* dev_out, DeviceState** st_out)
{
    int dev = 0;
    VK_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return set_error(VK_ERR_NO_DEVICE, "device ordinal %d out of range", dev);
    DeviceState& st = g_dev[dev];
    if (!st.ready.load(std::memory_order_acquire)) {
        std::lock_guard<std::mutex> lk(g_mu);
        int rc = init_device_locked(dev);
        if (rc != VK_OK) return rc;
    }
    *dev_out = dev;
    if (st_out) *st_out = &st;
    return VK_OK;
}

// Sets the smem attribute once per (device, kernel) and caches the co-residency limit.
template <typename Kernel>
static int kernel_slot(DeviceState& st, Kernel fn, int smem, int threads, int cluster, int* max_units)
{
    const void* key = reinterpret_cast<const void*>(fn);
    const int seen = st.num_kernels.load(std::memory_order_acquire);
    for (int i = 0; i < seen; ++i) {
        if (st.kernels[i].fn == key) {
            *max_units = st.kernels[i].max_clusters;
            return VK_OK;
        }
    }
    std::lock_guard<std::mutex> lk(g_mu);
    const int count = st.num_kernels.load(std::memory_order_relaxed);
    for (int i = 0; i < count; ++i) {
        if (st.kernels[i].fn == key) {
            *max_units = st.kernels[i].max_clusters;
            return VK_OK;
        }
    }
    if (count >= kMaxKernels) return set_error(VK_ERR_UNSUPPORTED, "kernel table full");
    VK_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    int units = 0;
    if (cluster > 1) {
        VK_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 0));
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = cluster;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(cluster * st.sm_count, 1, 1);
        cfg.blockDim = dim3(threads, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        VK_CUDA_TRY(cudaOccupancyMaxActiveClusters(&units, fn, &cfg));
    } else {
        int per_sm = 0;
        VK_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem));
        units = per_sm * st.sm_count;
    }
    if (units <= 0) return set_error(VK_ERR_CUDA, "kernel cannot be resident (smem %d)", smem);
    KernelSlot& s = st.kernels[count];
    s.fn = key;
    s.max_clusters = units;
    st.num_kernels.store(count + 1, std::memory_order_release);
    *max_units = units;
    return VK_OK;
}

// Tail-split workspace of (current device, stream), allocated on first use; see DeviceState.
static int ensure_workspace(DeviceState& st, int dev, cudaStream_t stream, float** ws_out, int** ctr_out)
{
    std::lock_guard<std::mutex> lk(g_mu);
    for (int i = 0; i < st.num_scratch; ++i) {
        if (st.scratch[i].stream == stream) {
            *ws_out = st.scratch[i].ws;
            *ctr_out = st.scratch[i].counters;
            return VK_OK;
        }
    }
    if (st.num_scratch >= DeviceState::kMaxStreams)
        return set_error(VK_ERR_UNSUPPORTED,
                         "tail-split workspaces exist for %d streams on device %d; use fewer streams or "
                         "vk_set_option(\"tail_split\", 0)",
                         DeviceState::kMaxStreams, dev);
    const size_t ws_bytes = static_cast<size_t>(st.sm_count) * 128 * 256 * sizeof(float);
    const size_t ctr_bytes = static_cast<size_t>(st.sm_count) * 4 * 2 * sizeof(int);
    float* ws = nullptr;
    int* ctr = nullptr;
    cudaError_t e = cudaMalloc(&ws, ws_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&ctr, ctr_bytes);
    if (e == cudaSuccess) e = cudaMemset(ctr, 0, ctr_bytes);
    if (e != cudaSuccess) {
        if (ws) cudaFree(ws);
        if (ctr) cudaFree(ctr);
        return set_error(VK_ERR_CUDA, "tail-split workspace on device %d: %s", dev, cudaGetErrorString(e));
    }
    st.ctr_bytes = ctr_bytes;
    st.ws_bytes = ws_bytes;
    DeviceState::StreamScratch& s = st.scratch[st.num_scratch++];
    s.stream = stream;
    s.ws = ws;
    s.counters = ctr;
    *ws_out = ws;
    *ctr_out = ctr;
    return VK_OK;
}

// Repack buffer `which` (0 = A, 1 = B) of (current device, stream), at least `bytes` long.
static int ensure_pack(DeviceState& st, int dev, cudaStream_t stream, int which, size_t bytes, void** out)
{
    float* ws = nullptr;
    int* ctr = nullptr;
    int rc = ensure_workspace(st, dev, stream, &ws, &ctr);  // creates the stream's scratch slot
    if (rc != VK_OK) return rc;
    std::lock_guard<std::mutex> lk(g_mu);
    for (int i = 0; i < st.num_scratch; ++i) {
        DeviceState::StreamScratch& s = st.scratch[i];
        if (s.stream != stream) continue;
        if (s.pack_bytes[which] < bytes) {
            if (s.pack[which] != nullptr) {
                // the old buffer may still be read by work queued on this stream
                cudaError_t e = cudaStreamSynchronize(stream);
                if (e == cudaSuccess) e = cudaFree(s.pack[which]);
                if (e != cudaSuccess) return set_error(VK_ERR_CUDA, "repack buffer: %s", cudaGetErrorString(e));
                s.pack[which] = nullptr;
                s.pack_bytes[which] = 0;
            }
            cudaError_t e = cudaMalloc(&s.pack[which], bytes);
            if (e != cudaSuccess) return set_error(VK_ERR_CUDA, "repack buffer (%zu bytes): %s", bytes, cudaGetErrorString(e));
            s.pack_bytes[which] = bytes;
        }
        *out = s.pack[which];
        return VK_OK;
    }
    return set_error(VK_ERR_CUDA, "repack buffer: no scratch slot for the stream");
}

// Work decomposition of the persistent tensor-core kernels: whole tiles for the full waves,
// and the tiles of a partial last wave cut into k-slices (at least kMinSliceKb k-blocks each).
struct Schedule {
    int units, full_units, split, nsplit, tail_first, grid_units;
};

static constexpr int kMinSliceKb = 4;
static constexpr int kMaxSplit = 8;

// Tail policy.  With R tail tiles on C clusters, at least one full wave, S = C / R k-slices in
// 2..4 and K >= kFirstMinK, the tail tiles are cut into S k-slices that run FIRST (tail_first): the
// fp32 partials are published and reduced while the clusters' whole tiles keep the tensor pipes
// busy, and the MMAs keep the full-width tile shape (measured on B200: +2 to +5 % over column
// halves at 4096^3, 5120^3, 4000x5120x3000, 2048x8192x4096, even at 4096^2 x 3072; slower for
// K <= 2048 or S = 8, where the reduction outlasts the next tile's main loop).  Otherwise, when 2R <= C and the layout allows
// it, each tail tile is cut into two column halves (MMA N = BN/2, no partial sums; they move 1.5x
// the operand bytes per MMA cycle of a whole tile).  When R <= C/4 the tiles are cut into up to 8
// k-slices instead, which parallelises small problems more.
static constexpr long long kFirstMinK = 2560;
static constexpr int kFirstMaxSplit = 4;

static Schedule plan_schedule(long long tiles, int num_kb, int max_units, bool allow_split, bool allow_nsplit,
                              bool allow_first)
{
    Schedule sc;
    sc.units = static_cast<int>(tiles);
    sc.full_units = static_cast<int>(tiles);
    sc.split = 1;
    sc.nsplit = 0;
    sc.tail_first = 0;
    if (allow_split && tiles > 0) {
        const long long full_waves = tiles / max_units;
        const long long rem = tiles - full_waves * max_units;
        if (rem > 0) {
            long long s = max_units / rem;
            if (s > num_kb / kMinSliceKb) s = num_kb / kMinSliceKb;
            if (s > kMaxSplit) s = kMaxSplit;
            const bool ksplit_better = 4 * rem <= max_units && s >= 4;
            if (allow_first && full_waves >= 1 && s >= 2 && s <= kFirstMaxSplit) {
                sc.full_units = static_cast<int>(full_waves * max_units);
                sc.split = static_cast<int>(s);
                sc.tail_first = 1;
                sc.units = static_cast<int>(sc.full_units + rem * s);
            } else if (allow_nsplit && 2 * rem <= max_units && !ksplit_better) {
                sc.full_units = static_cast<int>(full_waves * max_units);
                sc.nsplit = 1;
                sc.units = static_cast<int>(sc.full_units + 2 * rem);
            } else if (s >= 2) {
                sc.full_units = static_cast<int>(full_waves * max_units);
                sc.split = static_cast<int>(s);
                sc.units = static_cast<int>(sc.full_units + rem * s);
            }
        }
    }
    sc.grid_units = sc.units < max_units ? sc.units : max_units;
    return sc;
}

// ------------------------------------------------------------------------------------------
// Tensor maps
// ------------------------------------------------------------------------------------------
// 2-D fp16 tensor map over a row-major matrix [rows x cols] with row pitch `ld` elements and a
// (box_cols x box_rows) box, 128-byte swizzle, zero fill outside the matrix.
static int make_tmap_f16(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld,
                         uint32_t box_cols, uint32_t box_rows)
{
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(VK_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) rows=%lld cols=%lld ld=%lld", (int)r,
                         (long long)rows, (long long)cols, (long long)ld);
    return VK_OK;
}

// 2-D fp16 tensor map for the TMA stores of C: 32 x 32 boxes in the 64-byte swizzle layout of the
// kernel's epilogue staging buffers.
static int make_tmap_c(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld)
{
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                          CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(VK_ERR_CUDA, "cuTensorMapEncodeTiled (C) failed (%d) rows=%lld cols=%lld ld=%lld", (int)r,
                         (long long)rows, (long long)cols, (long long)ld);
    return VK_OK;
}

// make_tmap_f16 (kind 0) / make_tmap_c (kind 1) through the device's cache.
static int cached_tmap(DeviceState& st, int kind, CUtensorMap* out, const void* base, int64_t rows, int64_t cols,
                       int64_t ld, uint32_t box_cols, uint32_t box_rows)
{
    std::lock_guard<std::mutex> lk(st.tmap_mu);
    for (const TmapEntry& e : st.tmaps) {
        if (e.kind == kind && e.base == base && e.rows == rows && e.cols == cols && e.ld == ld &&
            e.box_cols == box_cols && e.box_rows == box_rows) {
            *out = e.map;
            return VK_OK;
        }
    }
    const int rc = kind == 0 ? make_tmap_f16(out, base, rows, cols, ld, box_cols, box_rows)
                             : make_tmap_c(out, base, rows, cols, ld);
    if (rc != VK_OK) return rc;
    TmapEntry& e = st.tmaps[st.tmap_next];
    st.tmap_next = (st.tmap_next + 1) % DeviceState::kTmapCache;
    e.base = base;
    e.rows = rows;
    e.cols = cols;
    e.ld = ld;
    e.box_cols = box_cols;
    e.box_rows = box_rows;
    e.kind = kind;
    e.map = *out;
    return VK_OK;
}

// ------------------------------------------------------------------------------------------
// Launchers
// ------------------------------------------------------------------------------------------
struct Problem {
    const void* A;
    const void* B;
    void* C;
    float* C32;
    int64_t m, n, k, lda, ldb, ldc;
    cudaStream_t stream;
    int tile_n;
    // vk_gemm_ex extensions (all off for vk_gemm)
    int trans_a = 0, trans_b = 0;
    int ep = 0, act = 0;
    float alpha = 1.f, beta = 0.f;
    const void* Cin = nullptr;
    int64_t ldcin = 0;
    const void* bias = nullptr;
    // vk_gemm_peers: peer C buffers that also receive every finished box of C (tensor-core path only)
    int npeers = 0;
    void* peer_c[kMaxPeers] = {};
    // vk_gemm_mc: multicast view of C (tensor-core path only; C itself is written through it)
    void* mc_c = nullptr;
};

template <int CG, int BN, int STAGES, int KA, bool ACC_F32, int XG = 0, bool CH = false>
static int launch_tc(DeviceState& st, int dev, const Problem& pb, const FixedScratch* fixed)
{
    using Cfg = TcCfg<CG, BN, STAGES, KA, ACC_F32, XG>;
    auto fn = tc_gemm_kernel<CG, BN, STAGES, KA, ACC_F32, XG, CH>;
    int max_units = 0;
    int rc = kernel_slot(st, fn, Cfg::kSmemBytes, Cfg::kThreads, CG, &max_units);
    if (rc != VK_OK) return rc;

    CUtensorMap ta, tb;
    // A: K-major boxes of 64 k x 128 rows, or (A stored k x m) M-major boxes of 64 rows x BK k.
    // B: N-major boxes of 64 columns x BK k, or (B stored n x k) K-major boxes of 64 k x BN/CG rows.
    rc = pb.trans_a ? cached_tmap(st, 0, &ta, pb.A, pb.k, pb.m, pb.lda, 64, Cfg::kBK)
                    : cached_tmap(st, 0, &ta, pb.A, pb.m, pb.k, pb.lda, 64, Cfg::kBM);
    if (rc != VK_OK) return rc;
    rc = pb.trans_b ? cached_tmap(st, 0, &tb, pb.B, pb.n, pb.k, pb.ldb, 64, Cfg::kBNCta)
                    : cached_tmap(st, 0, &tb, pb.B, pb.k, pb.n, pb.ldb, 64, Cfg::kBK);
    if (rc != VK_OK) return rc;

    TcParams p;
    p.M = static_cast<int>(pb.m);
    p.N = static_cast<int>(pb.n);
    p.K = static_cast<int>(pb.k);
    p.tiles_m = static_cast<int>((pb.m + Cfg::kBM * CG - 1) / (Cfg::kBM * CG));
    p.tiles_n = static_cast<int>((pb.n + BN - 1) / BN);
    p.num_kb = static_cast<int>((pb.k + Cfg::kBK - 1) / Cfg::kBK);
    p.raster_group = g_raster_group.load(std::memory_order_relaxed);
    p.C = static_cast<__half*>(pb.C);
    p.ldc = pb.ldc;
    p.C32 = pb.C32;
    const bool c_vec = (reinterpret_cast<uintptr_t>(pb.C) % 16 == 0) && (pb.ldc % 8 == 0);
    const bool c32_vec = pb.C32 == nullptr || ((reinterpret_cast<uintptr_t>(pb.C32) % 16 == 0) && (pb.n % 4 == 0));
    bool peers_vec = true;
    p.l2_evict_last = g_l2_evict_last.load(std::memory_order_relaxed);
    p.npeers = pb.npeers;
    for (int q = 0; q < kMaxPeers; ++q) {
        p.peer_c[q] = q < pb.npeers ? static_cast<__half*>(pb.peer_c[q]) : nullptr;
        if (q < pb.npeers) peers_vec = peers_vec && reinterpret_cast<uintptr_t>(pb.peer_c[q]) % 16 == 0;
    }
    p.vec_ok = (c_vec && c32_vec && peers_vec) ? 1 : 0;
    p.mc_c = static_cast<__half*>(pb.mc_c);
    // TMA stores of C need a 16-byte aligned base and a pitch that is a multiple of 16 bytes; with a
    // multicast view every box goes through it instead of a local store
    CUtensorMap tc;
    memset(&tc, 0, sizeof(tc));
    p.c_tma = (XG != 2 && g_tma_store.load(std::memory_order_relaxed) && c_vec && pb.m > 0 && pb.n > 0 &&
               pb.ldc * 2 < (1LL << 40)) ? 1 : 0;
    if (p.c_tma) {
        rc = cached_tmap(st, 1, &tc, pb.C, pb.m, pb.n, pb.ldc, 32, 32);
        if (rc != VK_OK) return rc;
    }
    p.timeout_ns = g_timeout_ns.load(std::memory_order_relaxed);
    p.clock_probe = g_clock_probe_on.load(std::memory_order_relaxed);
    p.a_mn = pb.trans_a;
    p.b_k = pb.trans_b;
    p.ep = pb.ep;
    p.act = pb.act;
    p.alpha = pb.alpha;
    p.beta = pb.beta;
    p.Cin = static_cast<const __half*>(pb.Cin);
    p.ldcin = pb.ldcin;
    p.bias = static_cast<const __half*>(pb.bias);
    p.trace = g_trace_on.load(std::memory_order_relaxed);

    const long long tiles = static_cast<long long>(p.tiles_m) * p.tiles_n;
    // n-split halves need whole 64-column boxes per CTA and N-major B tiles
    const bool nsplit_ok = (Cfg::kBNCta / 2) % 64 == 0 && !pb.trans_b && g_tail_nsplit.load(std::memory_order_relaxed);
    const Schedule sc =
        plan_schedule(tiles, p.num_kb, max_units, g_tail_split.load(std::memory_order_relaxed) != 0, nsplit_ok,
                      g_tail_first.load(std::memory_order_relaxed) != 0 && pb.k >= kFirstMinK);
    p.units = sc.units;
    p.full_units = sc.full_units;
    p.split = sc.split;
    p.nsplit = sc.nsplit;
    p.tail_first = sc.tail_first;
    p.ws = nullptr;
    p.counters = nullptr;
    if (sc.split > 1 && fixed != nullptr) {
        // Caller-provided scratch: never allocate; refuse a plan that does not fit, and zero the
        // arrival counters this launch will use (the array keeps the previous call's contents).
        const size_t slots = static_cast<size_t>(sc.units - sc.full_units) * CG;
        const size_t ws_need = slots * Cfg::kBM * BN * sizeof(float);
        const size_t ctr_need = static_cast<size_t>(sc.units - sc.full_units) / sc.split * CG * 4 * 2 * sizeof(int);
        if (ws_need > fixed->ws_bytes || ctr_need > fixed->ctr_bytes)
            return set_error(VK_ERR_UNSUPPORTED,
                             "vk_gemm_noalloc: this problem needs %zu bytes of tail-split scratch and %zu bytes "
                             "of counters; the no-allocation array holds %zu and %zu",
                             ws_need, ctr_need, fixed->ws_bytes, fixed->ctr_bytes);
        VK_CUDA_TRY(cudaMemsetAsync(fixed->counters, 0, ctr_need, pb.stream));
        p.ws = fixed->ws;
        p.counters = fixed->counters;
    } else if (sc.split > 1) {
        rc = ensure_workspace(st, dev, pb.stream, &p.ws, &p.counters);
        if (rc != VK_OK) return rc;
    }
    const int clusters = sc.grid_units;

    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CG;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(CG * clusters, 1, 1);
    cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = pb.stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    VK_CUDA_TRY(cudaLaunchKernelEx(&cfg, fn, ta, tb, tc, p));
    return VK_OK;
}

// One tensor-core variant per (pair or single CTA, tile N, accumulate type, pipeline shape).
template <bool F32>
static int launch_tc_variant(DeviceState& st, int dev, const Problem& pb, int algo, const FixedScratch* fixed)
{
    const int tn = pb.tile_n ? pb.tile_n : 256;
    const bool pair_default = algo == VK_ALGO_TC_2SM && tn == 256 && g_bk_2sm256.load(std::memory_order_relaxed) == 128;
    // two accumulation chains: compiled into the default pair kernel (local and multicast epilogues);
    // every unit needs >= 2 k-blocks of 128 (slices have >= kMinSliceKb)
    const int kc = g_k_chains.load(std::memory_order_relaxed);
    const bool chains = pair_default && pb.k > 128 && (kc == 2 || (kc == 1 && pb.k > kChainsMinK));
    if (pb.mc_c != nullptr) {
        // the multicast epilogue is compiled into the default pair kernel only
        if (pair_default && chains) return launch_tc<2, 256, 3, 2, F32, 2, true>(st, dev, pb, fixed);
        if (pair_default) return launch_tc<2, 256, 3, 2, F32, 2>(st, dev, pb, fixed);
        return set_error(VK_ERR_UNSUPPORTED,
                         "vk_gemm_mc: multicast stores run on the default pair kernel only (algo AUTO or TC_2SM, "
                         "tile_n 256, bk_2sm256 128)");
    }
    if (pb.npeers > 0) {
        // the peer-storing epilogue is compiled into the default pair kernel only
        if (algo == VK_ALGO_TC_2SM && tn == 256 && g_bk_2sm256.load(std::memory_order_relaxed) == 128)
            return launch_tc<2, 256, 3, 2, F32, 1>(st, dev, pb, fixed);
        return set_error(VK_ERR_UNSUPPORTED,
                         "vk_gemm_peers: peer stores run on the default pair kernel only (algo AUTO or TC_2SM, "
                         "tile_n 256, bk_2sm256 128)");
    }
    if (algo == VK_ALGO_TC_2SM) {
        if (tn == 256) {
            if (chains) return launch_tc<2, 256, 3, 2, F32, 0, true>(st, dev, pb, fixed);
            if (g_bk_2sm256.load(std::memory_order_relaxed) == 128) return launch_tc<2, 256, 3, 2, F32>(st, dev, pb, fixed);
            return launch_tc<2, 256, 6, 1, F32>(st, dev, pb, fixed);
        }
        return launch_tc<2, 128, 8, 1, F32>(st, dev, pb, fixed);
    }
    if (tn == 256) return launch_tc<1, 256, 4, 1, F32>(st, dev, pb, fixed);
    return launch_tc<1, 128, 6, 1, F32>(st, dev, pb, fixed);
}

static int launch_sgemm(const Problem& pb)
{
    SgemmParams p;
    p.M = static_cast<int>(pb.m);
    p.N = static_cast<int>(pb.n);
    p.K = static_cast<int>(pb.k);
    p.A = static_cast<const float*>(pb.A);
    p.B = static_cast<const float*>(pb.B);
    p.C = static_cast<float*>(pb.C);
    p.lda = pb.lda;
    p.ldb = pb.ldb;
    p.ldc = pb.ldc;
    p.vec_a = (reinterpret_cast<uintptr_t>(pb.A) % 16 == 0) && (pb.lda % 4 == 0);
    p.vec_b = (reinterpret_cast<uintptr_t>(pb.B) % 16 == 0) && (pb.ldb % 4 == 0);
    p.vec_c = (reinterpret_cast<uintptr_t>(pb.C) % 16 == 0) && (pb.ldc % 4 == 0);
    p.ep = pb.ep;
    p.act = pb.act;
    p.alpha = pb.alpha;
    p.beta = pb.beta;
    p.Cin = static_cast<const float*>(pb.Cin);
    p.ldcin = pb.ldcin;
    p.bias = static_cast<const float*>(pb.bias);
    dim3 grid(static_cast<unsigned>((pb.n + kSgBN - 1) / kSgBN), static_cast<unsigned>((pb.m + kSgBM - 1) / kSgBM));
    if (grid.y > 65535u) return set_error(VK_ERR_UNSUPPORTED, "m too large for the SGEMM grid");
    if (p.vec_a && p.vec_b && g_sgemm_v2.load(std::memory_order_relaxed)) {
        // smem attribute set once per device (bit per ordinal < 31) and kernel.  Variants (all bitwise
        // equal): 1 (default) = paired FMAs, 8 x 16 outputs per thread (55.9 TFLOP/s at 4096^3 on B200);
        // 2 = paired FMAs, 8 x 8 per thread (49.8); 0 = scalar FMAs, 8 x 8 (42.2).  A variant that stored
        // the A tile pre-broadcast as (a, a) pairs (register-staged A) measured 10 % slower than the
        // register broadcast and was dropped.
        std::atomic<int>* attr_dev_mask = g_sgemm_attr_mask;
        const int variant = g_sgemm_paired.load(std::memory_order_relaxed);
        auto fn = variant == 1 ? sgemm_ffma_w16_kernel
                               : (variant == 2 ? sgemm_ffma_v2_kernel<true> : sgemm_ffma_v2_kernel<false>);
        const int threads = variant == 1 ? kSgW16Threads : kSgThreads;
        int dev = 0;
        VK_CUDA_TRY(cudaGetDevice(&dev));
        const int bit = 1 << (dev & 31);
        if (!(attr_dev_mask[variant].load() & bit)) {
            VK_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSg2SmemBytes));
            attr_dev_mask[variant].fetch_or(bit);
        }
        fn<<<grid, threads, kSg2SmemBytes, pb.stream>>>(p);
    } else {
        sgemm_ffma_kernel<<<grid, kSgThreads, 0, pb.stream>>>(p);
    }
    VK_CUDA_TRY(cudaGetLastError());
    return VK_OK;
}

static int launch_hgemm_simt(const Problem& pb)
{
    HgemmSimtParams p;
    p.M = static_cast<int>(pb.m);
    p.N = static_cast<int>(pb.n);
    p.K = static_cast<int>(pb.k);
    p.A = static_cast<const __half*>(pb.A);
    p.B = static_cast<const __half*>(pb.B);
    p.C = static_cast<__half*>(pb.C);
    p.lda = pb.lda;
    p.ldb = pb.ldb;
    p.ldc = pb.ldc;
    p.C32 = pb.C32;
    p.trans_a = pb.trans_a;
    p.trans_b = pb.trans_b;
    p.ep = pb.ep;
    p.act = pb.act;
    p.alpha = pb.alpha;
    p.beta = pb.beta;
    p.Cin = static_cast<const __half*>(pb.Cin);
    p.ldcin = pb.ldcin;
    p.bias = static_cast<const __half*>(pb.bias);
    dim3 grid(static_cast<unsigned>((pb.n + kHsTile - 1) / kHsTile), static_cast<unsigned>((pb.m + kHsTile - 1) / kHsTile));
    if (grid.y > 65535u) return set_error(VK_ERR_UNSUPPORTED, "m too large for the SIMT grid");
    hgemm_simt_kernel<<<grid, 256, 0, pb.stream>>>(p);
    VK_CUDA_TRY(cudaGetLastError());
    return VK_OK;
}

template <typename T>
static int launch_zero(DeviceState& st, const Problem& pb)
{
    const long long total = pb.m * pb.n;
    long long blocks = (total + 255) / 256;
    if (blocks > 8LL * st.sm_count) blocks = 8LL * st.sm_count;
    if (pb.ep) {
        // k == 0: the product is zero, the epilogue still applies (beta * C_in + bias, activation)
        epilogue_only_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, pb.stream>>>(
            static_cast<T*>(pb.C), pb.ldc, static_cast<int>(pb.m), static_cast<int>(pb.n), pb.C32,
            static_cast<const T*>(pb.Cin), pb.ldcin, pb.beta, static_cast<const T*>(pb.bias), pb.act);
    } else {
        fill_zero_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, pb.stream>>>(
            static_cast<T*>(pb.C), pb.ldc, static_cast<int>(pb.m), static_cast<int>(pb.n), pb.C32);
    }
    VK_CUDA_TRY(cudaGetLastError());
    return VK_OK;
}

static bool tma_ok_f16(const void* p, int64_t ld)
{
    return (reinterpret_cast<uintptr_t>(p) % 16 == 0) && ((ld * 2) % 16 == 0) && (ld * 2 < (1LL << 40));
}

int dispatch(DeviceState& st, int dev, const Problem& pb, int dtype, int acc, int algo);

// Frees every device's tail-split workspace and forgets its cached tensor maps (called from
// vk_shutdown).
void release_device_state()
{
    std::lock_guard<std::mutex> lk(g_mu);
    int prev = 0;
    cudaGetDevice(&prev);
    for (std::atomic<int>& m : g_sgemm_attr_mask) m.store(0);
    for (int d = 0; d < kMaxDevices; ++d) {
        DeviceState& st = g_dev[d];
        {
            std::lock_guard<std::mutex> tl(st.tmap_mu);
            for (TmapEntry& e : st.tmaps) e = TmapEntry();
            st.tmap_next = 0;
        }
        // Per-context facts cached on first use: the device address of the no-allocation array and
        // the kernels' shared-memory attributes.  A later cudaDeviceReset would make them stale, so
        // they are looked up again after vk_shutdown.
        st.noalloc_scratch.store(nullptr, std::memory_order_release);
        st.num_kernels.store(0, std::memory_order_release);
        for (KernelSlot& k : st.kernels) k = KernelSlot();
        if (st.num_scratch == 0) continue;
        cudaSetDevice(d);
        for (int i = 0; i < st.num_scratch; ++i) {
            cudaFree(st.scratch[i].ws);
            cudaFree(st.scratch[i].counters);
            for (void* pk : st.scratch[i].pack)
                if (pk != nullptr) cudaFree(pk);
            st.scratch[i] = DeviceState::StreamScratch();
        }
        st.num_scratch = 0;
        st.ws_bytes = st.ctr_bytes = 0;
    }
    cudaSetDevice(prev);
}

}  // namespace vk

// ==========================================================================================
// C ABI
// ==========================================================================================
using namespace vk;

static int gemm_entry(const vk_gemm_args* a, const vk_gemm_ext* x, const char* name, void* const* peers = nullptr,
                      int npeers = 0, void* mc_c = nullptr)
{
    if (a == nullptr) return set_error(VK_ERR_INVALID_ARGUMENT, "%s: args is NULL", name);
    if (a->m < 0 || a->n < 0 || a->k < 0)
        return set_error(VK_ERR_INVALID_ARGUMENT, "%s: negative size m=%lld n=%lld k=%lld", name, (long long)a->m,
                         (long long)a->n, (long long)a->k);
    const int64_t kMaxDim = (1LL << 31) - 1;
    if (a->m > kMaxDim || a->n > kMaxDim || a->k > kMaxDim)
        return set_error(VK_ERR_UNSUPPORTED, "%s: dimensions above 2^31-1 are not supported", name);
    if (a->dtype != VK_DTYPE_F16 && a->dtype != VK_DTYPE_F32)
        return set_error(VK_ERR_INVALID_ARGUMENT, "%s: unknown dtype %d", name, a->dtype);
    if (a->acc != VK_ACC_F32 && a->acc != VK_ACC_F16)
        return set_error(VK_ERR_INVALID_ARGUMENT, "%s: unknown acc %d", name, a->acc);
    if (a->algo < VK_ALGO_AUTO || a->algo > VK_ALGO_SIMT)
        return set_error(VK_ERR_INVALID_ARGUMENT, "%s: unknown algo %d", name, a->algo);
    if (x != nullptr) {
        if ((x->trans_a != 0 && x->trans_a != 1) || (x->trans_b != 0 && x->trans_b != 1))
            return set_error(VK_ERR_INVALID_ARGUMENT, "%s: trans_a and trans_b must be 0 or 1", name);
        if (x->activation != VK_ACT_NONE && x->activation != VK_ACT_RELU)
            return set_error(VK_ERR_INVALID_ARGUMENT, "%s: unknown activation %d", name, x->activation);
        if (x->beta != 0.f && x->C_in == nullptr)
            return set_error(VK_ERR_INVALID_ARGUMENT, "%s: beta != 0 needs C_in", name);
    }

    Problem pb;
    pb.A = a->A;
    pb.B = a->B;
    pb.C = a->C;
    pb.C32 = a->C_f32;
    pb.m = a->m;
    pb.n = a->n;
    pb.k = a->k;
    pb.trans_a = x ? x->trans_a : 0;
    pb.trans_b = x ? x->trans_b : 0;
    // row lengths of the stored matrices: A is m x k (k x m when transposed), B is k x n (n x k)
    const int64_t a_row = pb.trans_a ? a->m : a->k;
    const int64_t b_row = pb.trans_b ? a->k : a->n;
    pb.lda = a->lda ? a->lda : a_row;
    pb.ldb = a->ldb ? a->ldb : b_row;
    pb.ldc = a->ldc ? a->ldc : a->n;
    pb.stream = static_cast<cudaStream_t>(a->stream);
    pb.tile_n = a->tile_n;
    if (pb.lda < a_row || pb.ldb < b_row || pb.ldc < pb.n || pb.lda < 0 || pb.ldb < 0 || pb.ldc < 0)
        return set_error(VK_ERR_INVALID_ARGUMENT, "%s: leading dimension smaller than the row length", name);
    if (x != nullptr) {
        pb.ep = (x->alpha != 1.f || x->beta != 0.f || x->bias != nullptr || x->activation != VK_ACT_NONE) ? 1 : 0;
        pb.act = x->activation;
        pb.alpha = x->alpha;
        pb.beta = x->beta;
        pb.Cin = x->beta != 0.f ? x->C_in : nullptr;
        pb.ldcin = x->ldc_in ? x->ldc_in : pb.ldc;
        pb.bias = x->bias;
        if (pb.Cin != nullptr && pb.ldcin < pb.n)
            return set_error(VK_ERR_INVALID_ARGUMENT, "%s: ldc_in smaller than n", name);
    }
    if (a->dtype == VK_DTYPE_F32 && a->acc != VK_ACC_F32)
        return set_error(VK_ERR_UNSUPPORTED, "%s: fp32 GEMM supports fp32 accumulation only", name);
    if (a->dtype == VK_DTYPE_F32 && a->C_f32 != nullptr)
        return set_error(VK_ERR_INVALID_ARGUMENT, "%s: C_f32 copy is for fp16 output only", name);
    if (a->dtype == VK_DTYPE_F32 && (pb.trans_a || pb.trans_b))
        return set_error(VK_ERR_UNSUPPORTED, "%s: transposed operands are supported for fp16 only", name);
    if (a->tile_n != 0 && a->tile_n != 128 && a->tile_n != 256)
        return set_error(VK_ERR_INVALID_ARGUMENT, "%s: tile_n must be 0, 128 or 256", name);

    if (npeers < 0 || npeers > kMaxPeers)
        return set_error(VK_ERR_INVALID_ARGUMENT, "%s: npeers must be 0..%d", name, kMaxPeers);
    if (npeers > 0) {
        if (peers == nullptr) return set_error(VK_ERR_INVALID_ARGUMENT, "%s: peer_C is NULL", name);
        for (int q = 0; q < npeers; ++q) {
            if (peers[q] == nullptr) return set_error(VK_ERR_INVALID_ARGUMENT, "%s: peer_C[%d] is NULL", name, q);
            pb.peer_c[q] = peers[q];
        }
        if (a->dtype != VK_DTYPE_F16)
            return set_error(VK_ERR_UNSUPPORTED, "%s: peer stores are for the fp16 tensor-core kernels", name);
        pb.npeers = npeers;
    }

    int dev = 0;
    DeviceState* st = nullptr;
    int rc = current_device(&dev, &st);
    if (rc != VK_OK) return rc;
    if (mc_c != nullptr) {
        if (a->dtype != VK_DTYPE_F16)
            return set_error(VK_ERR_UNSUPPORTED, "%s: multicast stores are for the fp16 tensor-core kernels", name);
        if (pb.n % 8 != 0 || pb.ldc % 8 != 0 || reinterpret_cast<uintptr_t>(pb.C) % 16 != 0 ||
            reinterpret_cast<uintptr_t>(mc_c) % 16 != 0)
            return set_error(VK_ERR_ALIGNMENT, "%s: needs n and ldc multiples of 8 and 16-byte aligned C and C_mc",
                             name);
        // C_mc must be the multicast view of exactly this C (same offset inside a live team's buffer)
        if (pb.m > 0 && pb.n > 0) {
            const size_t extent = static_cast<size_t>((pb.m - 1) * pb.ldc + pb.n) * 2;
            if (mc_lookup(dev, pb.C, extent) != mc_c)
                return set_error(VK_ERR_INVALID_ARGUMENT,
                                 "%s: C is not inside a multicast buffer of this device, or C_mc is not its "
                                 "multicast view", name);
        }
        pb.mc_c = mc_c;
    }
    return dispatch(*st, dev, pb, a->dtype, a->acc, a->algo);
}

extern "C" int vk_gemm(const vk_gemm_args* a) { return gemm_entry(a, nullptr, "vk_gemm"); }

extern "C" int vk_gemm_ex(const vk_gemm_args* a, const vk_gemm_ext* x) { return gemm_entry(a, x, "vk_gemm_ex"); }

extern "C" int vk_gemm_peers(const vk_gemm_args* a, void* const* peer_C, int32_t npeers)
{
    return gemm_entry(a, nullptr, "vk_gemm_peers", peer_C, npeers);
}

extern "C" int vk_gemm_mc(const vk_gemm_args* a, void* C_mc)
{
    if (C_mc == nullptr) return set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_mc: C_mc is NULL");
    return gemm_entry(a, nullptr, "vk_gemm_mc", nullptr, 0, C_mc);
}

namespace vk {
int dispatch(DeviceState& st_ref, int dev, const Problem& pb, int dtype, int acc, int algo_in)
{
    DeviceState* st = &st_ref;
    if (pb.m == 0 || pb.n == 0) return VK_OK;
    if (pb.C == nullptr) return set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm: C is NULL");
    if (pb.npeers > 0 && (pb.k == 0 || algo_in == VK_ALGO_SIMT || algo_in == VK_ALGO_FFMA))
        return set_error(VK_ERR_UNSUPPORTED, "vk_gemm_peers: peer stores need the tensor-core kernels and k > 0");
    if (pb.mc_c != nullptr && (pb.k == 0 || algo_in == VK_ALGO_SIMT || algo_in == VK_ALGO_FFMA))
        return set_error(VK_ERR_UNSUPPORTED, "vk_gemm_mc: multicast stores need the tensor-core kernels and k > 0");
    if (pb.k == 0) return dtype == VK_DTYPE_F16 ? launch_zero<__half>(*st, pb) : launch_zero<float>(*st, pb);
    if (pb.A == nullptr || pb.B == nullptr) return set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm: A or B is NULL");

    if (dtype == VK_DTYPE_F32) {
        if (algo_in != VK_ALGO_AUTO && algo_in != VK_ALGO_FFMA)
            return set_error(VK_ERR_UNSUPPORTED, "vk_gemm: fp32 runs on the FFMA kernel only");
        return launch_sgemm(pb);
    }

    // fp16
    const bool a_ok = tma_ok_f16(pb.A, pb.lda), b_ok = tma_ok_f16(pb.B, pb.ldb);
    const bool tma_ok = a_ok && b_ok;
    int algo = algo_in;
    if (algo == VK_ALGO_FFMA) return set_error(VK_ERR_UNSUPPORTED, "vk_gemm: FFMA kernel is fp32 only");
    if (algo == VK_ALGO_AUTO && !tma_ok && g_repack.load(std::memory_order_relaxed)) {
        // Copy the operand(s) that break the TMA rule into a buffer whose row pitch is a multiple of
        // 16 bytes (one strided device copy each, ordered on the caller's stream), then run the
        // tensor-core kernel; C keeps its own pitch (the epilogue predicates its stores).
        Problem pk = pb;
        for (int which = 0; which < 2; ++which) {
            if (which == 0 ? a_ok : b_ok) continue;
            const void* src = which == 0 ? pb.A : pb.B;
            const int64_t ld = which == 0 ? pb.lda : pb.ldb;
            const bool trans = which == 0 ? pb.trans_a : pb.trans_b;
            // stored rows x cols of this operand
            const int64_t rows = which == 0 ? (trans ? pb.k : pb.m) : (trans ? pb.n : pb.k);
            const int64_t cols = which == 0 ? (trans ? pb.m : pb.k) : (trans ? pb.k : pb.n);
            const int64_t ld_new = (cols + 7) / 8 * 8;
            void* dst = nullptr;
            int rc2 = ensure_pack(*st, dev, pb.stream, which, static_cast<size_t>(rows) * ld_new * 2, &dst);
            if (rc2 != VK_OK) return rc2;
            VK_CUDA_TRY(cudaMemcpy2DAsync(dst, static_cast<size_t>(ld_new) * 2, src, static_cast<size_t>(ld) * 2,
                                          static_cast<size_t>(cols) * 2, static_cast<size_t>(rows),
                                          cudaMemcpyDeviceToDevice, pb.stream));
            if (which == 0) {
                pk.A = dst;
                pk.lda = ld_new;
            } else {
                pk.B = dst;
                pk.ldb = ld_new;
            }
        }
        return acc == VK_ACC_F32 ? launch_tc_variant<true>(*st, dev, pk, VK_ALGO_TC_2SM, nullptr)
                                 : launch_tc_variant<false>(*st, dev, pk, VK_ALGO_TC_2SM, nullptr);
    }
    if (algo == VK_ALGO_AUTO) algo = tma_ok ? VK_ALGO_TC_2SM : VK_ALGO_SIMT;
    if (algo == VK_ALGO_SIMT && (pb.npeers > 0 || pb.mc_c != nullptr))
        return set_error(VK_ERR_UNSUPPORTED,
                         "vk_gemm_peers: these operands need the predicated kernel (enable \"repack\"), which has no "
                         "peer stores");
    if (algo == VK_ALGO_SIMT) {
        if (acc != VK_ACC_F32)
            return set_error(VK_ERR_UNSUPPORTED, "vk_gemm: the predicated CUDA-core kernel accumulates in fp32 only");
        return launch_hgemm_simt(pb);
    }
    if (!tma_ok)
        return set_error(VK_ERR_ALIGNMENT,
                         "vk_gemm: tensor-core kernels need 16-byte aligned A/B and lda, ldb multiples of 8 "
                         "(use VK_ALGO_AUTO or VK_ALGO_SIMT)");
    return acc == VK_ACC_F32 ? launch_tc_variant<true>(*st, dev, pb, algo, nullptr)
                             : launch_tc_variant<false>(*st, dev, pb, algo, nullptr);
}
}  // namespace vk

// ------------------------------------------------------------------------------------------
// No-allocation entry point.  Some callers cannot call cudaMalloc at all: code running while a
// CUDA graph is being captured, applications whose memory is owned by a custom pool or a
// framework allocator that forbids side allocations, and hosts that budget every byte of device
// memory up front.  vk_gemm_noalloc runs the fp16 tensor-core kernel with its tail-split scratch
// taken from the fixed array below instead of the library's lazily cudaMalloc'd workspace.
// ------------------------------------------------------------------------------------------
namespace vk {
// 16 KiB of arrival counters followed by 20 MiB of fp32 partials: one 128 x 256 fp32 slot per
// persistent CTA on a GPU with up to 160 SMs (B200 has 148), so every problem fits on B200.
// Every GPU that loads this library holds the array until the process exits.
constexpr size_t kNoAllocCounterBytes = 16384;
constexpr size_t kNoAllocPartialBytes = 20u * 1024u * 1024u;
constexpr size_t kNoAllocScratchBytes = kNoAllocCounterBytes + kNoAllocPartialBytes;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Looks up (once per device, with that device current) the device address of the array: the
// host-side symbol is only a stand-in and must never be passed to a kernel.
static int noalloc_scratch(DeviceState& st, FixedScratch* out)
{
    void* ptr = st.noalloc_scratch.load(std::memory_order_acquire);
    if (ptr == nullptr) {
        std::lock_guard<std::mutex> lk(g_mu);
        ptr = st.noalloc_scratch.load(std::memory_order_acquire);
        if (ptr == nullptr) {
            cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
            if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
            st.noalloc_scratch.store(ptr, std::memory_order_release);
        }
    }
    unsigned char* base = static_cast<unsigned char*>(ptr);
    out->counters = reinterpret_cast<int*>(base);
    out->ctr_bytes = kNoAllocCounterBytes;
    out->ws = reinterpret_cast<float*>(base + kNoAllocCounterBytes);
    out->ws_bytes = kNoAllocPartialBytes;
    return VK_OK;
}
}  // namespace vk

extern "C" int vk_gemm_noalloc(const vk_gemm_args* a)
{
    if (a == nullptr) return set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_noalloc: args is NULL");
    if (a->m < 0 || a->n < 0 || a->k < 0)
        return set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_noalloc: negative size");
    const int64_t kMaxDim = (1LL << 31) - 1;
    if (a->m > kMaxDim || a->n > kMaxDim || a->k > kMaxDim)
        return set_error(VK_ERR_UNSUPPORTED, "vk_gemm_noalloc: dimensions above 2^31-1 are not supported");
    if (a->dtype != VK_DTYPE_F16)
        return set_error(VK_ERR_UNSUPPORTED, "vk_gemm_noalloc: fp16 tensor-core GEMM only");
    if (a->acc != VK_ACC_F32 && a->acc != VK_ACC_F16)
        return set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_noalloc: unknown acc %d", a->acc);
    if (a->algo != VK_ALGO_AUTO && a->algo != VK_ALGO_TC_2SM && a->algo != VK_ALGO_TC_1SM)
        return set_error(VK_ERR_UNSUPPORTED, "vk_gemm_noalloc: tensor-core kernels only (AUTO, TC_2SM, TC_1SM)");
    if (a->tile_n != 0 && a->tile_n != 128 && a->tile_n != 256)
        return set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_noalloc: tile_n must be 0, 128 or 256");
    Problem pb;
    pb.A = a->A;
    pb.B = a->B;
    pb.C = a->C;
    pb.C32 = a->C_f32;
    pb.m = a->m;
    pb.n = a->n;
    pb.k = a->k;
    pb.lda = a->lda ? a->lda : a->k;
    pb.ldb = a->ldb ? a->ldb : a->n;
    pb.ldc = a->ldc ? a->ldc : a->n;
    pb.stream = static_cast<cudaStream_t>(a->stream);
    pb.tile_n = a->tile_n;
    if (pb.lda < pb.k || pb.ldb < pb.n || pb.ldc < pb.n)
        return set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_noalloc: leading dimension smaller than the row length");

    int dev = 0;
    DeviceState* st = nullptr;
    int rc = current_device(&dev, &st);
    if (rc != VK_OK) return rc;
    if (pb.m == 0 || pb.n == 0) return VK_OK;
    if (pb.C == nullptr) return set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_noalloc: C is NULL");
    if (pb.k == 0) return launch_zero<__half>(*st, pb);
    if (pb.A == nullptr || pb.B == nullptr)
        return set_error(VK_ERR_INVALID_ARGUMENT, "vk_gemm_noalloc: A or B is NULL");
    if (!(tma_ok_f16(pb.A, pb.lda) && tma_ok_f16(pb.B, pb.ldb)))
        return set_error(VK_ERR_ALIGNMENT,
                         "vk_gemm_noalloc: needs 16-byte aligned A/B and lda, ldb multiples of 8");
    FixedScratch fx;
    rc = noalloc_scratch(*st, &fx);
    if (rc != VK_OK) return rc;
    const int algo = a->algo == VK_ALGO_TC_1SM ? VK_ALGO_TC_1SM : VK_ALGO_TC_2SM;
    return a->acc == VK_ACC_F32 ? launch_tc_variant<true>(*st, dev, pb, algo, &fx)
                                : launch_tc_variant<false>(*st, dev, pb, algo, &fx);
}

extern "C" int vk_matmul_f16(int version, size_t m, size_t n, size_t k, const void* A, const void* B, void* C)
{
    vk_gemm_args a;
    memset(&a, 0, sizeof(a));
    a.A = A;
    a.B = B;
    a.C = C;
    a.m = static_cast<int64_t>(m);
    a.n = static_cast<int64_t>(n);
    a.k = static_cast<int64_t>(k);
    a.dtype = VK_DTYPE_F16;
    switch (version) {
        case 1: a.algo = VK_ALGO_TC_2SM; a.acc = VK_ACC_F32; break;
        case 2: a.algo = VK_ALGO_TC_2SM; a.acc = VK_ACC_F16; break;
        case 3: a.algo = VK_ALGO_TC_1SM; a.acc = VK_ACC_F32; break;
        case 4: a.algo = VK_ALGO_SIMT; a.acc = VK_ACC_F32; break;
        default:
            return set_error(VK_ERR_INVALID_ARGUMENT,
                             "vk_matmul_f16: version %d is not a GPU version (1..4; v0 is the CPU ground truth)",
                             version);
    }
    return vk_gemm(&a);
}

extern "C" int vk_matmul_f32(int version, size_t m, size_t n, size_t k, const float* A, const float* B, float* C)
{
    if (version != 1)
        return set_error(VK_ERR_INVALID_ARGUMENT, "vk_matmul_f32: version %d is not a GPU version (1)", version);
    vk_gemm_args a;
    memset(&a, 0, sizeof(a));
    a.A = A;
    a.B = B;
    a.C = C;
    a.m = static_cast<int64_t>(m);
    a.n = static_cast<int64_t>(n);
    a.k = static_cast<int64_t>(k);
    a.dtype = VK_DTYPE_F32;
    a.acc = VK_ACC_F32;
    a.algo = VK_ALGO_FFMA;
    return vk_gemm(&a);
}

extern "C" int vk_init(int device)
{
    int prev = 0;
    VK_CUDA_TRY(cudaGetDevice(&prev));
    VK_CUDA_TRY(cudaSetDevice(device));
    int dev = 0;
    int rc = current_device(&dev, nullptr);
    cudaSetDevice(prev);
    return rc;
}

extern "C" const char* vk_last_error_string(void) { return t_last_error.c_str(); }

extern "C" const char* vk_version_string(void) { return "vkgemm 0.1.0 (sm_100a)"; }

// Test hook: the persistent kernels' work decomposition for a problem, computed on the host by the same
// planner (plan_schedule) and unit decoder (unit_info) the launches use, so CPU tests can check that
// every (tile, k-block) is covered exactly once.  No device is touched.
extern "C" int vk_debug_schedule(int64_t tiles, int32_t num_kb, int32_t max_units, int64_t k, int32_t flags,
                                 int32_t* out_plan, int32_t* out_units, int32_t max_units_out)
{
    if (tiles < 0 || num_kb < 1 || max_units < 1 || out_plan == nullptr)
        return set_error(VK_ERR_INVALID_ARGUMENT, "vk_debug_schedule: bad arguments");
    const bool first = (flags & 4) != 0 && k >= kFirstMinK;
    const Schedule sc = plan_schedule(tiles, num_kb, max_units, (flags & 1) != 0, (flags & 2) != 0, first);
    out_plan[0] = sc.units;
    out_plan[1] = sc.full_units;
    out_plan[2] = sc.split;
    out_plan[3] = sc.nsplit;
    out_plan[4] = sc.tail_first;
    out_plan[5] = sc.grid_units;
    if (out_units == nullptr) return VK_OK;
    if (sc.units > max_units_out)
        return set_error(VK_ERR_INVALID_ARGUMENT, "vk_debug_schedule: %d units, room for %d", sc.units, max_units_out);
    TcParams p;
    memset(&p, 0, sizeof(p));
    p.num_kb = num_kb;
    p.units = sc.units;
    p.full_units = sc.full_units;
    p.split = sc.split;
    p.nsplit = sc.nsplit;
    p.tail_first = sc.tail_first;
    for (int u = 0; u < sc.units; ++u) {
        const Unit w = unit_info(p, u);
        out_units[4 * u + 0] = w.tile;
        out_units[4 * u + 1] = w.kb0;
        out_units[4 * u + 2] = w.kb1;
        out_units[4 * u + 3] = w.slice >= 0 ? w.slice : (w.half >= 0 ? 100 + w.half : -1);
    }
    return VK_OK;
}

extern "C" int vk_set_option(const char* name, int64_t value)
{
    if (name == nullptr) return set_error(VK_ERR_INVALID_ARGUMENT, "vk_set_option: name is NULL");
    if (strcmp(name, "tail_split") == 0) {
        g_tail_split.store(value != 0 ? 1 : 0);
        return VK_OK;
    }
    if (strcmp(name, "tail_nsplit") == 0) {
        g_tail_nsplit.store(value != 0 ? 1 : 0);
        return VK_OK;
    }
    if (strcmp(name, "tail_first") == 0) {
        g_tail_first.store(value != 0 ? 1 : 0);
        return VK_OK;
    }
    if (strcmp(name, "l2_evict_last") == 0) {
        g_l2_evict_last.store(value != 0 ? 1 : 0);
        return VK_OK;
    }
    if (strcmp(name, "k_chains") == 0) {
        if (value < 0 || value > 2) return set_error(VK_ERR_INVALID_ARGUMENT, "k_chains must be 0, 1 or 2");
        g_k_chains.store(static_cast<int>(value));
        return VK_OK;
    }
    if (strcmp(name, "tma_store") == 0) {
        g_tma_store.store(value != 0 ? 1 : 0);
        return VK_OK;
    }
    if (strcmp(name, "raster_group") == 0) {
        if (value < 1 || value > 64) return set_error(VK_ERR_INVALID_ARGUMENT, "raster_group must be 1..64");
        g_raster_group.store(static_cast<int>(value));
        return VK_OK;
    }
    if (strcmp(name, "bk_2sm256") == 0) {
        if (value != 64 && value != 128) return set_error(VK_ERR_INVALID_ARGUMENT, "bk_2sm256 must be 64 or 128");
        g_bk_2sm256.store(static_cast<int>(value));
        return VK_OK;
    }
    if (strcmp(name, "repack") == 0) {
        g_repack.store(value != 0 ? 1 : 0);
        return VK_OK;
    }
    if (strcmp(name, "sgemm_v2") == 0) {
        g_sgemm_v2.store(value != 0 ? 1 : 0);
        return VK_OK;
    }
    if (strcmp(name, "sgemm_paired") == 0) {
        if (value < 0 || value > 2) return set_error(VK_ERR_INVALID_ARGUMENT, "sgemm_paired must be 0, 1 or 2");
        g_sgemm_paired.store(static_cast<int>(value));
        return VK_OK;
    }
    if (strcmp(name, "trace") == 0) {
        g_trace_on.store(value != 0 ? 1 : 0);
        return VK_OK;
    }
    if (strcmp(name, "clock_probe") == 0) {
        g_clock_probe_on.store(value != 0 ? 1 : 0);
        return VK_OK;
    }
    if (strcmp(name, "gather_timeout_ms") == 0) {
        if (value <= 0) return set_error(VK_ERR_INVALID_ARGUMENT, "gather_timeout_ms must be > 0");
        g_gather_timeout_ms.store(value);
        return VK_OK;
    }
    if (strcmp(name, "wait_timeout_ns") == 0) {
        if (value <= 0) return set_error(VK_ERR_INVALID_ARGUMENT, "wait_timeout_ns must be > 0");
        g_timeout_ns.store(static_cast<unsigned long long>(value));
        return VK_OK;
    }
    return set_error(VK_ERR_INVALID_ARGUMENT, "vk_set_option: unknown option '%s'", name);
}

extern "C" int vk_set_wait_timeout_ns(uint64_t ns)
{
    if (ns == 0) return set_error(VK_ERR_INVALID_ARGUMENT, "timeout must be > 0");
    g_timeout_ns.store(ns);
    return VK_OK;
}

extern "C" int vk_device_error(int device, uint64_t* out_word, int clear)
{
    if (out_word == nullptr) return set_error(VK_ERR_INVALID_ARGUMENT, "out_word is NULL");
    int prev = 0;
    VK_CUDA_TRY(cudaGetDevice(&prev));
    VK_CUDA_TRY(cudaSetDevice(device));
    unsigned long long w = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&w, g_device_error, sizeof(w));
    if (e == cudaSuccess && clear && w != 0) {
        const unsigned long long z = 0;
        e = cudaMemcpyToSymbol(g_device_error, &z, sizeof(z));
        // a kernel that gave up may have left tail-split arrival counters mid-count
        if (device >= 0 && device < kMaxDevices) {
            std::lock_guard<std::mutex> lk(g_mu);
            DeviceState& st = g_dev[device];
            for (int i = 0; i < st.num_scratch && e == cudaSuccess; ++i)
                e = cudaMemset(st.scratch[i].counters, 0, st.ctr_bytes);
        }
    }
    cudaSetDevice(prev);
    if (e != cudaSuccess) return cuda_fail(e, "vk_device_error");
    *out_word = w;
    return VK_OK;
}

extern "C" int vk_read_clock_probe(int device, uint64_t* out3, int clear)
{
    if (out3 == nullptr) return set_error(VK_ERR_INVALID_ARGUMENT, "out3 is NULL");
    int prev = 0;
    VK_CUDA_TRY(cudaGetDevice(&prev));
    VK_CUDA_TRY(cudaSetDevice(device));
    unsigned long long v[3] = {0, 0, 0};
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(v, g_clock_probe, sizeof(v));
    if (e == cudaSuccess && clear) {
        const unsigned long long z[3] = {0, 0, 0};
        e = cudaMemcpyToSymbol(g_clock_probe, z, sizeof(z));
    }
    cudaSetDevice(prev);
    if (e != cudaSuccess) return cuda_fail(e, "vk_read_clock_probe");
    out3[0] = v[0];
    out3[1] = v[1];
    out3[2] = v[2];
    return VK_OK;
}

extern "C" int vk_read_trace(int device, uint64_t* out16)
{
    if (out16 == nullptr) return set_error(VK_ERR_INVALID_ARGUMENT, "out16 is NULL");
    int prev = 0;
    VK_CUDA_TRY(cudaGetDevice(&prev));
    VK_CUDA_TRY(cudaSetDevice(device));
    unsigned long long v[16];
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(v, g_trace, sizeof(v));
    if (e == cudaSuccess) {
        // re-arm: min slots start high, everything else at zero
        unsigned long long z[16] = {0};
        z[8] = z[10] = ~0ull;
        e = cudaMemcpyToSymbol(g_trace, z, sizeof(z));
    }
    cudaSetDevice(prev);
    if (e != cudaSuccess) return cuda_fail(e, "vk_read_trace");
    for (int i = 0; i < 16; ++i) out16[i] = v[i];
    return VK_OK;
}

extern "C" int vk_read_trace_cta(int device, uint64_t* out, int max_ctas)
{
    if (out == nullptr || max_ctas <= 0) return set_error(VK_ERR_INVALID_ARGUMENT, "vk_read_trace_cta: bad buffer");
    const int n = max_ctas < 256 ? max_ctas : 256;
    int prev = 0;
    VK_CUDA_TRY(cudaGetDevice(&prev));
    VK_CUDA_TRY(cudaSetDevice(device));
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(out, g_trace_cta, sizeof(uint64_t) * 8 * n);
    cudaSetDevice(prev);
    if (e != cudaSuccess) return cuda_fail(e, "vk_read_trace_cta");
    return VK_OK;
}

extern "C" int vk_selftest_wait_timeout(int device, int64_t timeout_us)
{
    if (timeout_us <= 0 || timeout_us > 10000000) return set_error(VK_ERR_INVALID_ARGUMENT, "timeout_us out of range");
    int prev = 0;
    VK_CUDA_TRY(cudaGetDevice(&prev));
    VK_CUDA_TRY(cudaSetDevice(device));
    int dev = 0;
    int rc = current_device(&dev, nullptr);
    if (rc != VK_OK) {
        cudaSetDevice(prev);
        return rc;
    }
    const unsigned long long z = 0;
    unsigned long long w = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_device_error, &z, sizeof(z));
    if (e == cudaSuccess) {
        selftest_wait_kernel<<<1, 32>>>(static_cast<unsigned long long>(timeout_us) * 1000ull);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&w, g_device_error, sizeof(w));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_device_error, &z, sizeof(z));
    cudaSetDevice(prev);
    if (e != cudaSuccess) return cuda_fail(e, "vk_selftest_wait_timeout");
    if ((w >> 32) == kErrWaitSelftest)
        return set_error(VK_ERR_DEVICE_TIMEOUT, "self-test wait ran out after %lld us as designed",
                         (long long)timeout_us);
    return set_error(VK_ERR_CUDA, "self-test wait did not report a timeout (word=%llx)", w);
}
