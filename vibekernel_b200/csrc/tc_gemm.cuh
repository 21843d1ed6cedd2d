// Persistent, warp-specialised tcgen05 GEMM for sm_100a:  C[M,N] = A[M,K] * B[K,N], fp16 in,
// fp32 (or fp16) accumulate in tensor memory, fp16 out (+ optional fp32 copy).
//
// Replaces the A100 mma.sync/cp.async kernels behind playground::matmul<float16_t, V>
// (e.g. results/ralph_loop_fable/src/matmul_f16/matmul_f16_v42_shfl2.cu:104-490): same row-major
// NN contract, but the math is tcgen05.mma issued by one thread with accumulators in TMEM, the
// operands arrive by TMA into 128-byte-swizzled shared memory, and a pair of CTAs (cta_group::2)
// shares one 256-row tile.
//
// Roles (192 threads per CTA):
//   warp 0      TMA producer: one lane streams A (K-major) and B (N-major) k-blocks into a ring
//               of STAGES shared-memory stages guarded by full/empty mbarriers.
//   warp 1      TMEM allocator (whole warp) and, in the pair's leader CTA, the MMA issuer (one
//               lane).  Two accumulators (2 x BN TMEM columns) alternate between tiles, so the
//               epilogue of tile i overlaps the main loop of tile i+1.
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns at a time, convert, store to global.
//
// Pair mode (CG = 2): the two CTAs of a cluster each hold 128 rows of A and BN/2 columns of B
// per stage; the leader issues 256 x BN x 16 MMAs that read both CTAs' shared memory and write
// both CTAs' TMEM.  Both CTAs' TMA loads signal the leader's "full" barrier (.cta_group::2
// completion), and the leader's commits arrive on both CTAs' "empty" and "tmem full" barriers.
// Every CTA loads only its own operand tiles, so the same binary serves 1-GPU and multi-GPU runs.
//
// Ragged shapes: TMA zero-fills out-of-range rows/columns of A and B (M, N and the K tail);
// the epilogue predicates stores on row < M and col < N.
//
// Tail split (the reference's last-wave K-split, results/ralph_loop_fable/src/matmul_f16/
// matmul_f16_v23_wavesplit.cu:1-8 and matmul_f16_v42_shfl2.cu:182-189): with T tiles on C
// persistent clusters, the first F*C tiles (F = T / C full waves) run whole; each of the R = T - F*C
// tiles of the partial last wave is cut into S = C / R k-slices, so the last wave takes ~1/S of a
// tile.  Every slice writes its fp32 partial to a workspace and bumps a per-(tile, CTA, warp)
// arrival counter; the slice that arrives last sums all slices in slice order (its own from TMEM,
// the others from the workspace) -- the same order whoever arrives last, so results are
// bitwise reproducible -- writes C, and resets the counter.  Nobody waits on another CTA, so
// the tail cannot deadlock whatever the residency.
#pragma once

#include <cuda_fp16.h>

#include <type_traits>

#include "ptx.cuh"

namespace vk {

struct TcParams {
    int M, N, K;
    int tiles_m, tiles_n, num_kb;
    int raster_group;        // tiles along M per rasterisation group
    __half* C;
    long long ldc;
    float* C32;              // optional fp32 copy, ld = N
    int vec_ok;              // C / C32 alignment allows 16-byte stores
    unsigned long long timeout_ns;
    // work units: [0, full_units) are whole tiles, then (units - full_units) / split tail tiles
    // cut into `split` k-slices each
    int units, full_units, split;
    float* ws;               // split partials: [tail tile][slice][CTA rank][128 rows x BN] fp32
    int* counters;           // arrival counters: [tail tile][CTA rank][4 epilogue warps]
    int clock_probe;         // 1: CTA 0 accumulates (cycles, ns, launches) into g_clock_probe
    int trace;               // 1: record the launch timeline into g_trace
    // operand layouts: a_mn = A stored k x m (A^T row-major: M-major tiles); b_k = B stored n x k
    // (B^T row-major: K-major tiles).  Default (0, 0) is the reference's NN row-major convention.
    int a_mn, b_k;
    // fused epilogue (ep = 1): C = act(alpha * acc + beta * C_in + bias), act 0 = none, 1 = relu
    int ep, act;
    float alpha, beta;
    const __half* Cin;
    long long ldcin;
    const __half* bias;
};

// Fused epilogue for one row's 32 fp32 results at columns col .. col+31 (fp32 math, then round).
__device__ __forceinline__ void store_chunk_fused(const TcParams& p, int row, int col, float (&f)[32])
{
    if (row >= p.M) return;
    __half* crow = p.C + static_cast<long long>(row) * p.ldc;
    const __half* cin = p.Cin ? p.Cin + static_cast<long long>(row) * p.ldcin : nullptr;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        if (col + i < p.N) {
            float v = p.alpha * f[i];
            if (cin != nullptr && p.beta != 0.f) v = fmaf(p.beta, __half2float(cin[col + i]), v);
            if (p.bias != nullptr) v += __half2float(p.bias[col + i]);
            if (p.act == 1) v = fmaxf(v, 0.f);
            crow[col + i] = __float2half_rn(v);
            if (p.C32 != nullptr) p.C32[static_cast<long long>(row) * p.N + col + i] = v;
        }
    }
}

struct Unit {
    int tile, kb0, kb1, slice;  // slice < 0: whole tile
};

__device__ __forceinline__ Unit unit_info(const TcParams& p, int u)
{
    Unit w;
    if (u < p.full_units) {
        w.tile = u;
        w.kb0 = 0;
        w.kb1 = p.num_kb;
        w.slice = -1;
    } else {
        const int v = u - p.full_units;
        const int ti = v / p.split;
        w.slice = v - ti * p.split;
        w.tile = p.full_units + ti;
        w.kb0 = p.num_kb * w.slice / p.split;
        w.kb1 = p.num_kb * (w.slice + 1) / p.split;
    }
    return w;
}

template <int CG, int BN, int STAGES, int KA, bool ACC_F32>
struct TcCfg {
    static constexpr int kBM = 128;              // rows per CTA (TMEM lanes)
    static constexpr int kBK = 64 * KA;          // k per stage: KA 128-byte swizzle spans of fp16
    static constexpr int kBNCta = BN / CG;       // B columns held per CTA
    static constexpr int kABytes = kBM * kBK * 2;
    static constexpr int kBBytes = kBNCta * kBK * 2;
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kBBoxes = kBNCta / 64;  // 64-column TMA boxes of B per stage
    static constexpr int kABox = kBM * 64 * 2;   // bytes of one 64-wide k-span of K-major A (128 rows)
    static constexpr int kAMnBox = 64 * kBK * 2; // bytes of one 64-row box of M-major A (kBK k rows)
    static constexpr int kBBox = 64 * kBK * 2;   // bytes of one 64-column box of N-major B (kBK rows)
    static constexpr int kBKBox = kBNCta * 64 * 2; // bytes of one 64-wide k-span of K-major B
    static constexpr int kTmemCols = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128
                                   : (2 * BN <= 256) ? 256 : 512;
    static constexpr int kNumBars = 2 * STAGES + 4 + 4;  // + one reduction barrier per epilogue warp
    // The tail-split reduction stages other slices' partials in the (idle) pipeline buffers:
    // 48 KB per epilogue warp.
    static constexpr int kRedFloatsPerWarp = 12288;
    static constexpr int kSmemBytes = 1024 /*alignment slack*/ + STAGES * kStageBytes + kNumBars * 8 + 16;
    static constexpr int kThreads = 192;
    static_assert(CG == 1 || CG == 2, "cta group");
    static_assert(KA == 1 || KA == 2, "k spans per stage");
    static_assert(kBNCta % 64 == 0, "each CTA holds whole 64-column swizzle atoms of B");
    static_assert(BN % 16 == 0 && BN >= 64 && BN <= 256, "UMMA N");
    static_assert(2 * BN <= 512, "two accumulators must fit in TMEM");
    static_assert(kSmemBytes <= 232448, "shared memory per CTA");
    static_assert(STAGES * kStageBytes >= 4 * kRedFloatsPerWarp * 4, "reduction staging fits the stage area");
};

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int group, int& tm, int& tn)
{
    const int per_group = group * tiles_n;
    const int g = t / per_group;
    const int first_m = g * group;
    const int gsz = min(tiles_m - first_m, group);
    const int r = t - g * per_group;
    tm = first_m + r % gsz;
    tn = r / gsz;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi)
{
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Store one row's 32 consecutive results (r = raw TMEM words) at C[row, col .. col+31].
template <bool ACC_F32>
__device__ __forceinline__ void store_chunk(const TcParams& p, int row, int col, const uint32_t (&r)[32])
{
    if (row >= p.M) return;
    if (p.ep) {
        float f[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            if constexpr (ACC_F32)
                f[i] = __uint_as_float(r[i]);
            else
                f[i] = __half2float(__ushort_as_half(static_cast<unsigned short>(r[i])));
        }
        store_chunk_fused(p, row, col, f);
        return;
    }
    __half* crow = p.C + static_cast<long long>(row) * p.ldc;
    const bool full = (col + 32 <= p.N) && p.vec_ok;
    if (full) {
        uint4* dst = reinterpret_cast<uint4*>(crow + col);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint4 v;
            if constexpr (ACC_F32) {
                v.x = pack_half2(__uint_as_float(r[8 * j + 0]), __uint_as_float(r[8 * j + 1]));
                v.y = pack_half2(__uint_as_float(r[8 * j + 2]), __uint_as_float(r[8 * j + 3]));
                v.z = pack_half2(__uint_as_float(r[8 * j + 4]), __uint_as_float(r[8 * j + 5]));
                v.w = pack_half2(__uint_as_float(r[8 * j + 6]), __uint_as_float(r[8 * j + 7]));
            } else {
                // fp16 accumulators occupy the low 16 bits of each 32-bit TMEM column.
                v.x = __byte_perm(r[8 * j + 0], r[8 * j + 1], 0x5410);
                v.y = __byte_perm(r[8 * j + 2], r[8 * j + 3], 0x5410);
                v.z = __byte_perm(r[8 * j + 4], r[8 * j + 5], 0x5410);
                v.w = __byte_perm(r[8 * j + 6], r[8 * j + 7], 0x5410);
            }
            dst[j] = v;
        }
        if (p.C32 != nullptr) {
            float4* d32 = reinterpret_cast<float4*>(p.C32 + static_cast<long long>(row) * p.N + col);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float4 f;
                if constexpr (ACC_F32) {
                    f = make_float4(__uint_as_float(r[4 * j + 0]), __uint_as_float(r[4 * j + 1]),
                                    __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
                } else {
                    f = make_float4(__half2float(__ushort_as_half(static_cast<unsigned short>(r[4 * j + 0]))),
                                    __half2float(__ushort_as_half(static_cast<unsigned short>(r[4 * j + 1]))),
                                    __half2float(__ushort_as_half(static_cast<unsigned short>(r[4 * j + 2]))),
                                    __half2float(__ushort_as_half(static_cast<unsigned short>(r[4 * j + 3]))));
                }
                d32[j] = f;
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            if (col + i < p.N) {
                float f;
                __half h;
                if constexpr (ACC_F32) {
                    f = __uint_as_float(r[i]);
                    h = __float2half_rn(f);
                } else {
                    h = __ushort_as_half(static_cast<unsigned short>(r[i]));
                    f = __half2float(h);
                }
                crow[col + i] = h;
                if (p.C32 != nullptr) p.C32[static_cast<long long>(row) * p.N + col + i] = f;
            }
        }
    }
}

template <int CG, int BN, int STAGES, int KA, bool ACC_F32>
__global__ void __launch_bounds__(192, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   const TcParams p)
{
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
    using Cfg = TcCfg<CG, BN, STAGES, KA, ACC_F32>;
    constexpr int BM = Cfg::kBM;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * Cfg::kABytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * Cfg::kBBytes);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::kNumBars);

    const uint32_t bar0 = smem_u32(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
    auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
    auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
    auto red_bar = [&](int q) { return bar0 + 8u * (2 * STAGES + 4 + q); };

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (p.trace && threadIdx.x == 0) {
        const unsigned long long t = globaltimer_ns();
        if (blockIdx.x == 0) g_trace[0] = t;
        atomicMin(&g_trace[8], t);
        atomicMax(&g_trace[9], t);
    }
    const uint32_t rank = (CG == 2) ? cluster_ctarank() : 0u;
    const int cluster_id = blockIdx.x / CG;
    const int num_clusters = gridDim.x / CG;

    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), CG * 4);
        }
        for (int q = 0; q < 4; ++q) mbar_init(red_bar(q), 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc<CG>(smem_u32(tmem_slot), Cfg::kTmemCols);
        tmem_relinquish<CG>();
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (CG == 2) cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    if (threadIdx.x == 0) trace_at(p.trace, 1);
    uint64_t probe_t0 = 0, probe_c0 = 0;
    if (p.clock_probe && blockIdx.x == 0 && threadIdx.x == 0) {
        probe_t0 = globaltimer_ns();
        probe_c0 = clock64();
    }

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            trace_at(p.trace, 2);
            for (int u = cluster_id; ok && u < p.units; u += num_clusters) {
                const Unit w = unit_info(p, u);
                int tm, tn;
                tile_coords(w.tile, p.tiles_m, p.tiles_n, p.raster_group, tm, tn);
                const int m0 = tm * (BM * CG) + static_cast<int>(rank) * BM;
                const int n0 = tn * BN + static_cast<int>(rank) * Cfg::kBNCta;
                for (int kb = w.kb0; kb < w.kb1; ++kb) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.timeout_ns, kErrWaitProducer, stage)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = full_bar(stage);
                    const uint32_t a_dst = smem_u32(sA + stage * Cfg::kABytes);
                    const uint32_t b_dst = smem_u32(sB + stage * Cfg::kBBytes);
                    const int k0 = kb * Cfg::kBK;
                    uint32_t bar = fb;
                    if constexpr (CG == 1) {
                        mbar_arrive_expect_tx(fb, Cfg::kStageBytes);
                    } else {
                        if (rank == 0) mbar_arrive_expect_tx(fb, 2 * Cfg::kStageBytes);
                        bar = mapa_shared(fb, 0);
                    }
                    auto load = [&](uint32_t dst, const CUtensorMap* map, int c0, int c1) {
                        if constexpr (CG == 1)
                            tma_load_2d(dst, map, bar, c0, c1);
                        else
                            tma_load_2d_pair(dst, map, bar, c0, c1);
                    };
                    if (!p.a_mn) {
#pragma unroll
                        for (int a = 0; a < KA; ++a) load(a_dst + a * Cfg::kABox, &tmap_a, k0 + 64 * a, m0);
                    } else {
#pragma unroll
                        for (int j = 0; j < BM / 64; ++j) load(a_dst + j * Cfg::kAMnBox, &tmap_a, m0 + 64 * j, k0);
                    }
                    if (!p.b_k) {
#pragma unroll
                        for (int j = 0; j < Cfg::kBBoxes; ++j) load(b_dst + j * Cfg::kBBox, &tmap_b, n0 + 64 * j, k0);
                    } else {
#pragma unroll
                        for (int a = 0; a < KA; ++a) load(b_dst + a * Cfg::kBKBox, &tmap_b, k0 + 64 * a, n0);
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // Drain: every stage this CTA filled must be released by the MMA (whose commits may
            // arrive from the peer CTA) before the CTA may exit.
            if (ok) {
                for (int i = 0; i < STAGES; ++i) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.timeout_ns, kErrWaitTail, stage)) break;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        // One copy of the issue loop per operand layout, so the descriptor arithmetic of the
        // single issuing thread is resolved at compile time (its issue rate matters).
        auto mma_loop = [&](auto a_mn_tag, auto b_k_tag) {
            constexpr bool A_MN = decltype(a_mn_tag)::value;
            constexpr bool B_K = decltype(b_k_tag)::value;
            // M/N-major operands: 64-element atoms of BK rows x 128 B, LBO steps between atoms and
            // SBO between 8-row groups, k advances 16 rows (2 KB) per MMA.  K-major operands: rows
            // of 128 B in 8-row groups (SBO), k advances 32 B within a 64-wide span and a whole span
            // (box) every 4 MMAs.
            constexpr uint32_t kIdesc =
                idesc_f16(BM * CG, BN, ACC_F32, /*b_mn_major=*/!B_K) | (A_MN ? (1u << 15) : 0u);
            constexpr uint32_t kMnLbo = Cfg::kBK * 128;
            int stage = 0;
            uint32_t phase = 0;
            int it = 0;
            bool ok = true;
            for (int u = cluster_id; ok && u < p.units; u += num_clusters, ++it) {
                const Unit w = unit_info(p, u);
                const int acc = it & 1;
                const uint32_t acc_phase = static_cast<uint32_t>(it >> 1) & 1u;
                if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, p.timeout_ns, kErrWaitMma, 100 + acc)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = w.kb0; kb < w.kb1; ++kb) {
                    if (!mbar_wait(full_bar(stage), phase, p.timeout_ns, kErrWaitMma, stage)) {
                        ok = false;
                        break;
                    }
                    if (it == 0 && kb == w.kb0) trace_at(p.trace, 3);
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + stage * Cfg::kABytes);
                    const uint32_t b_addr = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
                    for (int kk = 0; kk < Cfg::kBK / 16; ++kk) {
                        const uint64_t a_desc =
                            A_MN ? smem_desc_sw128(a_addr + kk * 16 * 128, kMnLbo, 1024)
                                 : smem_desc_sw128(a_addr + (kk >> 2) * Cfg::kABox + (kk & 3) * 32, 16, 1024);
                        const uint64_t b_desc =
                            B_K ? smem_desc_sw128(b_addr + (kk >> 2) * Cfg::kBKBox + (kk & 3) * 32, 16, 1024)
                                : smem_desc_sw128(b_addr + kk * 16 * 128, kMnLbo, 1024);
                        umma_f16<CG>(d_tmem, a_desc, b_desc, kIdesc, (kb != w.kb0 || kk != 0) ? 1u : 0u);
                    }
                    const uint32_t eb = empty_bar(stage);
                    umma_commit<CG>(eb);
                    if constexpr (CG == 2) umma_commit<CG>(mapa_shared(eb, 1));
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                const uint32_t tb = tfull_bar(acc);
                umma_commit<CG>(tb);
                if constexpr (CG == 2) umma_commit<CG>(mapa_shared(tb, 1));
                trace_at(p.trace, 4);
            }
        };
        if (rank == 0 && lane == 0) {
            using T = std::true_type;
            using F = std::false_type;
            if (!p.a_mn && !p.b_k)
                mma_loop(F{}, F{});
            else if (!p.a_mn)
                mma_loop(F{}, T{});
            else if (!p.b_k)
                mma_loop(T{}, F{});
            else
                mma_loop(T{}, T{});
        }
    } else {
        // ------------------------------------------------------------------ epilogue
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        int it = 0;
        for (int u = cluster_id; u < p.units; u += num_clusters, ++it) {
            const Unit w = unit_info(p, u);
            const int acc = it & 1;
            const uint32_t acc_phase = static_cast<uint32_t>(it >> 1) & 1u;
            if (!mbar_wait(tfull_bar(acc), acc_phase, p.timeout_ns, kErrWaitEpilogue, acc)) break;
            if (it == 0 && warp == 2 && lane == 0) trace_at(p.trace, 5);
            tc_fence_after();
            int tm, tn;
            tile_coords(w.tile, p.tiles_m, p.tiles_n, p.raster_group, tm, tn);
            const int row = tm * (BM * CG) + static_cast<int>(rank) * BM + q * 32 + lane;
            const int col0 = tn * BN;
            const uint32_t tbase = tmem_base + static_cast<uint32_t>(acc * BN) + (static_cast<uint32_t>(q * 32) << 16);
            if (w.slice >= 0) {
                // Tail slice: publish this slice's fp32 partial (lane-major float4 runs, so each warp
                // store is one contiguous 512-byte span), then count arrivals; only the last slice
                // to arrive reduces and writes C.
                const int ti = w.tile - p.full_units;
                constexpr size_t kRegion = static_cast<size_t>(BM) * BN;
                const size_t warp_off = static_cast<size_t>(q) * 32 * BN;
                float* mine = p.ws + (static_cast<size_t>(ti * p.split + w.slice) * CG + rank) * kRegion + warp_off;
#pragma unroll 1
                for (int c = 0; c < BN; c += 32) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>(c), r);
                    tmem_ld_wait();
                    float4* dst = reinterpret_cast<float4*>(mine + c * 32);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        float4 f;
                        if constexpr (ACC_F32) {
                            f = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                            __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
                        } else {
                            f = make_float4(__half2float(__ushort_as_half(static_cast<unsigned short>(r[4 * j]))),
                                            __half2float(__ushort_as_half(static_cast<unsigned short>(r[4 * j + 1]))),
                                            __half2float(__ushort_as_half(static_cast<unsigned short>(r[4 * j + 2]))),
                                            __half2float(__ushort_as_half(static_cast<unsigned short>(r[4 * j + 3]))));
                        }
                        __stcg(dst + j * 32 + lane, f);
                    }
                }
                __threadfence();
                __syncwarp();
                int* ctr = p.counters + (ti * CG + static_cast<int>(rank)) * 4 + q;
                int old = 0;
                if (lane == 0) old = atomicAdd(ctr, 1);
                old = __shfl_sync(0xffffffffu, old, 0);
                if (old == p.split - 1) {
                    __threadfence();
                    // Columns per round so that the other (split - 1) slices' partials of this warp's
                    // 32 rows fit its 48 KB of staging: (split - 1) * cr <= 384.
                    int cr = BN;
                    while ((p.split - 1) * cr > Cfg::kRedFloatsPerWarp / 32) cr >>= 1;
                    float* red = reinterpret_cast<float*>(smem) + q * Cfg::kRedFloatsPerWarp;
                    uint32_t rphase = 0;
#pragma unroll 1
                    for (int c0 = 0; c0 < BN && col0 + c0 < p.N; c0 += cr) {
                        if (lane == 0) {
                            fence_proxy_async_smem();  // earlier reads of `red` precede the refill
                            mbar_arrive_expect_tx(red_bar(q), static_cast<uint32_t>((p.split - 1) * cr * 32 * 4));
                            int j = 0;
                            for (int s2 = 0; s2 < p.split; ++s2) {
                                if (s2 == w.slice) continue;
                                const float* src = p.ws + (static_cast<size_t>(ti * p.split + s2) * CG + rank) * kRegion +
                                                   warp_off + static_cast<size_t>(c0) * 32;
                                bulk_load(smem_u32(red + j * cr * 32), src, static_cast<uint32_t>(cr * 32 * 4), red_bar(q));
                                ++j;
                            }
                        }
                        if (!mbar_wait(red_bar(q), rphase, p.timeout_ns, kErrWaitEpilogue, 200 + q)) break;
                        rphase ^= 1u;
#pragma unroll 1
                        for (int c = c0; c < c0 + cr; c += 32) {
                            if (col0 + c >= p.N) break;
                            uint32_t r[32];
                            tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>(c), r);
                            tmem_ld_wait();
                            // f = ((p_0 + p_1) + p_2) + ... in slice order, p_own taken from TMEM
                            float f[32];
                            int j = 0;
#pragma unroll 1
                            for (int s2 = 0; s2 < p.split; ++s2) {
                                float4 v[8];
                                if (s2 == w.slice) {
#pragma unroll
                                    for (int jj = 0; jj < 8; ++jj) {
                                        if constexpr (ACC_F32) {
                                            v[jj] = make_float4(__uint_as_float(r[4 * jj]), __uint_as_float(r[4 * jj + 1]),
                                                                __uint_as_float(r[4 * jj + 2]), __uint_as_float(r[4 * jj + 3]));
                                        } else {
                                            v[jj] = make_float4(
                                                __half2float(__ushort_as_half(static_cast<unsigned short>(r[4 * jj]))),
                                                __half2float(__ushort_as_half(static_cast<unsigned short>(r[4 * jj + 1]))),
                                                __half2float(__ushort_as_half(static_cast<unsigned short>(r[4 * jj + 2]))),
                                                __half2float(__ushort_as_half(static_cast<unsigned short>(r[4 * jj + 3]))));
                                        }
                                    }
                                } else {
                                    const float4* src = reinterpret_cast<const float4*>(red + j * cr * 32 + (c - c0) * 32);
#pragma unroll
                                    for (int jj = 0; jj < 8; ++jj) v[jj] = src[jj * 32 + lane];
                                    ++j;
                                }
                                if (s2 == 0) {
#pragma unroll
                                    for (int jj = 0; jj < 8; ++jj) {
                                        f[4 * jj] = v[jj].x;
                                        f[4 * jj + 1] = v[jj].y;
                                        f[4 * jj + 2] = v[jj].z;
                                        f[4 * jj + 3] = v[jj].w;
                                    }
                                } else {
#pragma unroll
                                    for (int jj = 0; jj < 8; ++jj) {
                                        f[4 * jj] += v[jj].x;
                                        f[4 * jj + 1] += v[jj].y;
                                        f[4 * jj + 2] += v[jj].z;
                                        f[4 * jj + 3] += v[jj].w;
                                    }
                                }
                            }
                            uint32_t rr[32];
#pragma unroll
                            for (int i = 0; i < 32; ++i) rr[i] = __float_as_uint(f[i]);
                            store_chunk<true>(p, row, col0 + c, rr);
                        }
                        __syncwarp();
                    }
                    if (lane == 0) *ctr = 0;  // every slice has arrived: ready for the next launch
                }
            } else {
#pragma unroll 1
                for (int c = 0; c < BN; c += 32) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>(c), r);
                    tmem_ld_wait();
                    if (col0 + c < p.N) store_chunk<ACC_F32>(p, row, col0 + c, r);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (warp == 2 && lane == 0) trace_at(p.trace, 6);
            if (lane == 0) {
                if constexpr (CG == 1)
                    mbar_arrive(tempty_bar(acc));
                else
                    mbar_arrive_cluster(mapa_shared(tempty_bar(acc), 0));
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (p.clock_probe && blockIdx.x == 0 && threadIdx.x == 0) {
        // SM cycles and wall nanoseconds of CTA 0's persistent loop: their ratio is the SM clock
        // the kernel actually ran at (power capping moves it within a launch).
        atomicAdd(&g_clock_probe[0], static_cast<unsigned long long>(clock64() - probe_c0));
        atomicAdd(&g_clock_probe[1], static_cast<unsigned long long>(globaltimer_ns() - probe_t0));
        atomicAdd(&g_clock_probe[2], 1ull);
    }
    if constexpr (CG == 2) cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc<CG>(tmem_base, Cfg::kTmemCols);
    }
    if (p.trace && threadIdx.x == 0) {
        const unsigned long long t = globaltimer_ns();
        if (blockIdx.x == 0) g_trace[7] = t;
        atomicMin(&g_trace[10], t);
        atomicMax(&g_trace[11], t);
    }
#endif
}

}  // namespace vk
