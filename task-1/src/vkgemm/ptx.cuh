// Inline-PTX helpers for sm_100a: mbarriers, TMA bulk-tensor loads, tcgen05 (UMMA / TMEM),
// cluster addressing and bounded waits.  Everything here is hand-written against the
// public PTX ISA (8.7); no template library is used.
#pragma once

#include <cstdint>
#include <cuda.h>

namespace vk {

// ------------------------------------------------------------------------------------------
// Device error word.  Any bounded wait that gives up records (code << 32 | detail) here with
// atomicCAS (the first error wins) and the kernel unwinds; the host reads it back through
// vk_device_error().  Defined here because exactly one translation unit (vkgemm.cu) holds all
// device code of the library.
// ------------------------------------------------------------------------------------------
__device__ unsigned long long g_device_error = 0ull;

// Clock probe accumulators: [0] SM cycles, [1] nanoseconds, [2] launches (see vk_read_clock_probe).
__device__ unsigned long long g_clock_probe[3] = {0ull, 0ull, 0ull};

enum : uint32_t {
    kErrWaitProducer = 1,   // producer gave up waiting for a free stage
    kErrWaitMma = 2,        // MMA issuer gave up waiting for a loaded stage / free accumulator
    kErrWaitEpilogue = 3,   // epilogue gave up waiting for a finished accumulator
    kErrWaitTail = 4,       // drain at kernel end gave up
    kErrWaitSelftest = 5,   // the self-test wait (nothing ever arrives) ran out, as intended
};

__device__ __forceinline__ uint64_t globaltimer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Launch timeline (%globaltimer ns) written when the trace option is on (see vk_read_trace):
// [0] CTA 0 entry, [1] CTA 0 prologue done, [2] first TMA issued, [3] first stage full at the MMA,
// [4] last MMA commit, [5] first accumulator ready at the epilogue, [6] last epilogue store issued,
// [7] CTA 0 exit, [8] earliest CTA entry, [9] latest CTA entry, [10] earliest CTA exit,
// [11] latest CTA exit.
__device__ unsigned long long g_trace[16];
// Per-CTA timeline (trace option): for CTA b < 256, [b][0] entry, [b][1] last MMA commit (pair leader
// or single CTA), [b][2] last epilogue store, [b][3] exit, [b][4] SM id, [b][5] units processed,
// [b][6] last accumulator ready at the epilogue, [b][7] tail slice: partial published / others'
// partials all published (last arriver).
__device__ unsigned long long g_trace_cta[256][8];

__device__ __forceinline__ void trace_at(int trace, int slot)
{
    if (trace && blockIdx.x == 0) g_trace[slot] = globaltimer_ns();
}

__device__ __forceinline__ void record_error(uint32_t code, uint32_t detail)
{
    unsigned long long v = (static_cast<unsigned long long>(code) << 32) | detail;
    atomicCAS(&g_device_error, 0ull, v);
}

__device__ __forceinline__ bool device_error_set()
{
    return *reinterpret_cast<volatile unsigned long long*>(&g_device_error) != 0ull;
}

// ------------------------------------------------------------------------------------------
// Shared-memory addressing
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t cluster_ctarank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of the same shared variable in CTA `rank` of this cluster (shared::cluster window).
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank)
{
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync_all()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ------------------------------------------------------------------------------------------
// mbarrier
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Arrive on a barrier that may live in another CTA of the cluster (address from mapa_shared).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar)
{
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity.  Returns false (after recording the error)
// when `timeout_ns` of wall time passes, or as soon as another wait anywhere on the device has
// given up, so that every role of every CTA unwinds instead of spinning forever.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint64_t timeout_ns,
                                          uint32_t code, uint32_t detail)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (device_error_set()) return false;
        if (globaltimer_ns() - t0 > timeout_ns) {
            record_error(code, detail);
            return false;
        }
    }
}

// ------------------------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor): every load fills only the issuing CTA's own shared memory.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void prefetch_tmap(const void* map)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Tile load into this CTA's shared memory; completion bytes go to `bar` in this CTA.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* map, uint32_t bar, int32_t c0,
                                            int32_t c1)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
        : "memory");
}

// Tile load into this CTA's shared memory whose completion bytes are signalled on a barrier
// of either CTA of the pair (`bar_cluster` from mapa_shared): used so that the pair's leader
// sees one "stage full" event covering both CTAs' halves of the operands.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void* map, uint32_t bar_cluster,
                                                 int32_t c0, int32_t c1)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1)
        : "memory");
}

// L2 cache policy that keeps the lines a load brings in resident over others (evict_last).
__device__ __forceinline__ uint64_t l2_policy_evict_last()
{
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// tma_load_2d / tma_load_2d_pair with an L2 cache policy.
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const void* map, uint32_t bar, int32_t c0, int32_t c1,
                                                 uint64_t pol)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "l"(pol)
        : "memory");
}

__device__ __forceinline__ void tma_load_2d_pair_hint(uint32_t dst, const void* map, uint32_t bar_cluster, int32_t c0,
                                                      int32_t c1, uint64_t pol)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "l"(pol)
        : "memory");
}

// Contiguous bulk copy global -> this CTA's shared memory (no tensor map); both addresses 16-byte
// aligned, size a multiple of 16.  Completion bytes go to `bar` in this CTA.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
        : "memory");
}

// Orders this thread's generic-proxy global-memory accesses (and what it acquired) before later
// async-proxy ones (bulk copies reading global memory).
__device__ __forceinline__ void fence_proxy_async_global()
{
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Bounded wait until the counter at `addr` (global) reaches at least `target`, with acquire
// semantics; records (code, detail) and returns false when `timeout_ns` passes or another wait
// has already given up.
__device__ __forceinline__ bool wait_count_at_least(int* addr, int target, uint64_t timeout_ns, uint32_t code,
                                                    uint32_t detail)
{
    auto load = [&]() {
        int v;
        asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
        return v;
    };
    if (load() >= target) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i)
            if (load() >= target) return true;
        if (device_error_set()) return false;
        if (globaltimer_ns() - t0 > timeout_ns) {
            record_error(code, detail);
            return false;
        }
    }
}

// Orders this thread's generic-proxy shared-memory accesses before later async-proxy ones.
__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Tile store from this CTA's shared memory to global through a tensor map (out-of-range rows and
// columns of the box are not written), tracked in the issuing thread's bulk async-group.
__device__ __forceinline__ void tma_store_2d(const void* map, uint32_t src, int32_t c0, int32_t c1)
{
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(src), "r"(c0), "r"(c1)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Wait until at most N of this thread's bulk groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read()
{
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until all of this thread's bulk groups have completed (writes performed).
__device__ __forceinline__ void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ------------------------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, loads, fences
// ------------------------------------------------------------------------------------------
template <int CG>
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols)
{
    if constexpr (CG == 1)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                     "r"(ncols)
                     : "memory");
    else
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                     "r"(ncols)
                     : "memory");
}

template <int CG>
__device__ __forceinline__ void tmem_relinquish()
{
    if constexpr (CG == 1)
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    else
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

template <int CG>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    if constexpr (CG == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                     : "memory");
    else
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                     : "memory");
}

__device__ __forceinline__ void tc_fence_before()
{
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after()
{
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (fp16 or bf16 inputs, fp32 or fp16 accumulate).
template <int CG>
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate)
{
    if constexpr (CG == 1)
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    else
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
}

// Arrive once on `bar` (a shared::cluster address: this CTA's own or the peer's) when all
// tcgen05 operations issued so far by this thread have completed.
template <int CG>
__device__ __forceinline__ void umma_commit(uint32_t bar)
{
    if constexpr (CG == 1)
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                     : "memory");
    else
        asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                     : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives lane (base + i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_ld_wait()
{
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ------------------------------------------------------------------------------------------
// UMMA descriptors (PTX ISA "Shared memory descriptor" / "Instruction descriptor", sm_100)
// ------------------------------------------------------------------------------------------
// Shared-memory matrix descriptor, 128-byte swizzle:
//   [0,14) start address >> 4, [16,30) leading byte offset >> 4, [32,46) stride byte offset >> 4,
//   [46,48) version = 1, [49,52) base offset = 0 (stage buffers are 1024-byte aligned),
//   [52] LBO mode = 0, [61,64) layout = 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes)
{
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= 1ull << 46;
    d |= 2ull << 61;
    return d;
}

// Instruction descriptor for kind::f16 with fp16 A and B:
//   [4,6) D format (0 = f16, 1 = f32), [7,10) A format (0 = f16), [10,13) B format (0 = f16),
//   [15] A major (0 = K-major), [16] B major (1 = MN-major), [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool acc_f32, bool b_mn_major)
{
    return (static_cast<uint32_t>(acc_f32 ? 1 : 0) << 4) | (static_cast<uint32_t>(b_mn_major ? 1 : 0) << 16) |
           (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

}  // namespace vk
