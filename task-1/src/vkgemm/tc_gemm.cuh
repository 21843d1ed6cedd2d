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
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns at a time, fused epilogue, fp16 pack
//               into swizzled shared staging, TMA tile store of each 32 x 32 box (per-lane
//               coalesced stores when C cannot take TMA stores).
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
// persistent clusters, F*C tiles (F = T / C full waves) run whole; each of the R = T - F*C
// remaining tiles is cut into S <= C / R k-slices, so the partial wave takes ~1/S of a tile.
// With tail_first the slices run first (each cluster: at most one slice, then its whole tiles),
// so their epilogues overlap the next tile's main loop.  Every slice bumps a per-(tile, CTA, warp)
// arrival counter; all but the last arriver write their fp32 partial to a workspace and count
// themselves as published; the last arriver waits (bounded) for those publishers -- CTAs that have
// already arrived, so resident, and that wait on nobody: no deadlock whatever the residency --
// sums all slices in slice order (its own from TMEM, the others from the workspace) -- the same
// order whoever arrives last, so results are bitwise reproducible -- writes C, and resets the
// counters.  Alternatively (nsplit) each tail tile is cut into two column halves.
//
// Kernel instances beyond the default: XG = 1 / 2 add the all-gather of C to the epilogue (stores
// into every peer's C, or once into the NVLS multicast view of C, which replaces the local store);
// CH runs each unit's k range as two accumulation chains in the two accumulators (see the kernel).
#pragma once

#include <cuda_fp16.h>

#include <type_traits>

#include "ptx.cuh"
#include "vk_internal.h"

namespace vk {

struct TcParams {
    int M, N, K;
    int tiles_m, tiles_n, num_kb;
    int raster_group;        // tiles along M per rasterisation group
    __half* C;
    long long ldc;
    float* C32;              // optional fp32 copy, ld = N
    int vec_ok;              // C / C32 alignment allows 16-byte stores
    int c_tma;               // 1: fp16 C is written by TMA tile stores through the C tensor map
    // fused all-gather: every finished 32 x 32 box of fp16 C is also stored (plain 16-byte stores over
    // NVLink, never TMA) at the same row / column offsets into each peer GPU's C buffer (same ldc)
    int l2_evict_last;       // 1: operand tiles are loaded with an L2 evict_last policy
    int npeers;
    __half* peer_c[kMaxPeers];
    // fused all-gather through NVLS (XG = 2): the multicast address of C's first element (same ldc);
    // every finished box is stored once there and the switch writes it into every member GPU's C,
    // this GPU's included, so the local store is skipped
    __half* mc_c;
    unsigned long long timeout_ns;
    // work units: full_units whole tiles and the tail tiles, each cut either into two column
    // halves (nsplit = 1: BN/2-wide MMAs, no reduction) or into `split` k-slices; the whole tiles
    // come first ([0, full_units)) unless tail_first
    int units, full_units, split, nsplit;
    // tail_first = 1 (k-slices only): the slice units are numbered before the whole tiles, so each
    // cluster runs its slice first and the slice's publish / reduce epilogue overlaps the main loop
    // of the cluster's next tile instead of ending the launch
    int tail_first;
    float* ws;               // split partials: [tail tile][slice][CTA rank][128 rows x BN] fp32
    int* counters;           // [tail tile][CTA rank][4 epilogue warps][arrived, published]
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


struct Unit {
    int tile, kb0, kb1;
    int slice;  // k-slice index of a k-split tail tile, -1 otherwise
    int half;   // column half (0/1) of an n-split tail tile, -1 for the full width
};

__host__ __device__ __forceinline__ Unit unit_info(const TcParams& p, int u)
{
    Unit w;
    w.half = -1;
    if (p.tail_first) {
        // slice units [0, units - full_units) first, then whole tiles 0 .. full_units - 1
        const int tail_units = p.units - p.full_units;
        if (u >= tail_units) {
            w.tile = u - tail_units;
            w.kb0 = 0;
            w.kb1 = p.num_kb;
            w.slice = -1;
        } else {
            const int ti = u / p.split;
            w.slice = u - ti * p.split;
            w.tile = p.full_units + ti;
            w.kb0 = p.num_kb * w.slice / p.split;
            w.kb1 = p.num_kb * (w.slice + 1) / p.split;
        }
    } else if (u < p.full_units) {
        w.tile = u;
        w.kb0 = 0;
        w.kb1 = p.num_kb;
        w.slice = -1;
    } else if (p.nsplit) {
        const int v = u - p.full_units;
        w.tile = p.full_units + (v >> 1);
        w.half = v & 1;
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

// Epilogue staging per warp: two 2 KB buffers of 32 rows x 32 fp16 in the 64-byte swizzle layout of
// the C tensor map (TMA stores, double-buffered), or, when C cannot take TMA stores, one buffer of
// 32 rows at an 80-byte pitch (bank-conflict-free row writes, 64-byte runs read back).
constexpr int kEpiPitch = 80;
constexpr int kEpiBufBytes = 32 * 64;
constexpr int kEpiWarpBytes = 2 * kEpiBufBytes;
static_assert(kEpiWarpBytes >= 32 * kEpiPitch, "fallback staging fits the warp's area");
// Multicast epilogue (XG = 2): a warp stages up to kMcRunChunks adjacent 32-column chunks of its 32
// rows (32 rows x 256 bytes) and sends them as runs of up to 256 bytes per row.
constexpr int kMcRunChunks = 4;
constexpr int kMcRowBytes = kMcRunChunks * 64;
constexpr int kMcWarpBytes = 32 * kMcRowBytes;

template <int CG, int BN, int STAGES, int KA, bool ACC_F32, int XG = 0>
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
    static constexpr int kEpiWarp = XG == 2 ? kMcWarpBytes : kEpiWarpBytes;  // staging bytes per epilogue warp
    static constexpr int kSmemBytes =
        1024 /*alignment slack*/ + STAGES * kStageBytes + kNumBars * 8 + 32 + 1024 /*staging alignment*/ +
        4 * kEpiWarp;
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

// TMEM words of one 32-column chunk to fp32 values (fp16 accumulators sit in the low halves).
template <bool ACC_F32>
__device__ __forceinline__ void tmem_words_to_f32(const uint32_t (&r)[32], float (&f)[32])
{
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        if constexpr (ACC_F32)
            f[i] = __uint_as_float(r[i]);
        else
            f[i] = __half2float(__ushort_as_half(static_cast<unsigned short>(r[i])));
    }
}

// multimem store of 16 bytes to a multicast address: the NVSwitch replicates it into the same
// offset of every member GPU's buffer.
__device__ __forceinline__ void multimem_st_16(void* addr, const uint4& v)
{
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

// Fused all-gather through NVLS.  In this mode a warp's staging area holds 32 rows x 256 bytes: up
// to four adjacent 32-column chunks of its rows (16-byte slot j of row r at j ^ (r & 7), so the row
// writes and the run reads below are bank-conflict free).  The staged chunks leave together as runs of
// up to 256 bytes per row (16 lanes per row, 2 rows per store instruction): the NVSwitch replicates
// fewer, fuller packets than for 64-byte runs (measured on 8 GPUs: 64-byte runs 1.33 ms per 16384^3
// step, 128-byte runs 1.09 ms).  The host guarantees N and ldc are multiples of 8 and the view is
// 16-byte aligned, so every 16-byte segment with column < N is whole.
struct McRun {
    int col = -1;  // first column of the staged run (-1: nothing staged)
    int n = 0;     // 32-column chunks staged
};

__device__ __forceinline__ void mc_flush(const TcParams& p, const uint8_t* stg, int row0, int lane, McRun& run)
{
    if (run.n > 0) {
        const int spr = run.n * 4;  // 16-byte segments per row
#pragma unroll 1
        for (int idx = lane; idx < 32 * spr; idx += 32) {
            const int rr = idx / spr;
            const int seg = idx - rr * spr;
            const int grow = row0 + rr;
            const int gcol = run.col + seg * 8;
            if (grow < p.M && gcol < p.N) {
                const uint4 v = *reinterpret_cast<const uint4*>(stg + rr * kMcRowBytes + ((seg ^ (rr & 7)) * 16));
                multimem_st_16(p.mc_c + static_cast<long long>(grow) * p.ldc + gcol, v);
            }
        }
        __syncwarp();
    }
    run.col = -1;
    run.n = 0;
}

// Fused all-gather: one warp copies its staged 32 x 32 fp16 box (rows row0.., columns col..; row r's
// 64 bytes at `pitch`, 16-byte chunk j at j ^ ((r >> 1) & 3) when `swizzled`) into every peer's C,
// 4 lanes per row so each store instruction writes 64-byte runs of 8 rows.  Same bounds as the local
// stores (row < M, column < N); 16-byte stores only when the row segment is whole and aligned.
__device__ __forceinline__ void store_box_to_peers(const TcParams& p, const uint8_t* box, int pitch, bool swizzled,
                                                   int row0, int lane, int col)
{
    const int seg = lane & 3;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int rr = (lane >> 2) + 8 * j;
        const int grow = row0 + rr;
        const int gcol = col + seg * 8;
        if (grow >= p.M || gcol >= p.N) continue;
        const int chunk = swizzled ? (seg ^ ((rr >> 1) & 3)) : seg;
        const uint4 v = *reinterpret_cast<const uint4*>(box + rr * pitch + chunk * 16);
        const long long off = static_cast<long long>(grow) * p.ldc + gcol;
        const bool whole = gcol + 8 <= p.N && p.vec_ok;
#pragma unroll 1
        for (int q = 0; q < p.npeers; ++q) {
            __half* dst = p.peer_c[q] + off;
            if (whole) {
                *reinterpret_cast<uint4*>(dst) = v;
            } else {
                const __half* h = reinterpret_cast<const __half*>(&v);
                for (int e = 0; e < 8; ++e)
                    if (gcol + e < p.N) dst[e] = h[e];
            }
        }
    }
}

// One 32-column chunk of this warp's accumulator rows as fp32 values: the TMEM words at `taddr`, plus,
// with two accumulation chains (CH), the second chain's words at `taddr2`, added in fp32 (the second
// load reuses the first one's registers).
template <bool ACC_F32, bool CH>
__device__ __forceinline__ void acc_chunk(uint32_t taddr, uint32_t taddr2, float (&f)[32])
{
    uint32_t r[32];
    tmem_ld_32x32b_x32(taddr, r);
    tmem_ld_wait();
    tmem_words_to_f32<ACC_F32>(r, f);
    if constexpr (CH) {
        tmem_ld_32x32b_x32(taddr2, r);
        tmem_ld_wait();
        float g[32];
        tmem_words_to_f32<ACC_F32>(r, g);
#pragma unroll
        for (int i = 0; i < 32; ++i) f[i] += g[i];
    }
}

// One warp writes its 32 rows x 32 columns of C (this lane's row = row0 + lane, values f for
// columns col .. col+31): the fused epilogue and the fp32 copy are applied per row, then the fp16
// results go through the warp's staging buffer.  With a C tensor map (c_tma) lane 0 stores the
// 32 x 32 box with one TMA store (the box is clipped to M x N by the hardware); the two buffers
// alternate, and a buffer is rewritten only after the store issued from it two chunks earlier has
// read it.  Otherwise each global store instruction writes 64-byte runs of 8 rows (4 lanes per row)
// instead of 16 bytes of 32 different rows.
// XG (exchange of C with other GPUs): 0 = none; 1 = the box is also stored into every peer's C
// (vk_gemm_peers); 2 = the box is stored once to the multicast view of C instead of locally
// (vk_gemm_mc; the host turns TMA stores off).  Each value is its own kernel instance, so the
// default kernels' epilogue code stays exactly as it is without the exchange.
template <int XG>
__device__ __forceinline__ void store_rows(const TcParams& p, const CUtensorMap* tmap_c, uint8_t* stg, int row0,
                                           int lane, int col, float (&f)[32], uint32_t& nbuf, McRun& mc)
{
    const int row = row0 + lane;
    if (p.ep && row < p.M) {
        const __half* cin = p.Cin ? p.Cin + static_cast<long long>(row) * p.ldcin : nullptr;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            if (col + i < p.N) {
                float v = p.alpha * f[i];
                if (cin != nullptr && p.beta != 0.f) v = fmaf(p.beta, __half2float(cin[col + i]), v);
                if (p.bias != nullptr) v += __half2float(p.bias[col + i]);
                if (p.act == 1) v = fmaxf(v, 0.f);
                f[i] = v;
            }
        }
    }
    if (p.C32 != nullptr && row < p.M) {
        float* d32 = p.C32 + static_cast<long long>(row) * p.N + col;
        if (col + 32 <= p.N && p.vec_ok) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
                reinterpret_cast<float4*>(d32)[j] = make_float4(f[4 * j], f[4 * j + 1], f[4 * j + 2], f[4 * j + 3]);
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (col + i < p.N) d32[i] = f[i];
        }
    }
    if constexpr (XG == 2) {
        // a chunk that does not continue the staged run sends the run first
        if (mc.n > 0 && col != mc.col + 32 * mc.n) mc_flush(p, stg, row0, lane, mc);
        if (mc.n == 0) mc.col = col;
        uint4* srow = reinterpret_cast<uint4*>(stg + lane * kMcRowBytes);
        const int sw = lane & 7;
#pragma unroll
        for (int j = 0; j < 4; ++j)
            srow[(4 * mc.n + j) ^ sw] = make_uint4(pack_half2(f[8 * j], f[8 * j + 1]),
                                                   pack_half2(f[8 * j + 2], f[8 * j + 3]),
                                                   pack_half2(f[8 * j + 4], f[8 * j + 5]),
                                                   pack_half2(f[8 * j + 6], f[8 * j + 7]));
        __syncwarp();
        ++mc.n;
        if (mc.n == kMcRunChunks || col + 32 >= p.N) mc_flush(p, stg, row0, lane, mc);  // full, or row end
        return;
    }
    if (p.c_tma) {
        uint8_t* buf = stg + (nbuf & 1u) * kEpiBufBytes;
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
        // 64-byte swizzle: 16-byte chunk j of row r sits at chunk j ^ ((r >> 1) & 3)
        uint4* srow = reinterpret_cast<uint4*>(buf + lane * 64);
        const int sw = (lane >> 1) & 3;
#pragma unroll
        for (int j = 0; j < 4; ++j)
            srow[j ^ sw] = make_uint4(pack_half2(f[8 * j], f[8 * j + 1]), pack_half2(f[8 * j + 2], f[8 * j + 3]),
                                      pack_half2(f[8 * j + 4], f[8 * j + 5]), pack_half2(f[8 * j + 6], f[8 * j + 7]));
        fence_proxy_async_smem();  // the generic-proxy writes precede the TMA engine's reads
        __syncwarp();
        if (lane == 0 && row0 < p.M) {
            tma_store_2d(tmap_c, smem_u32(buf), col, row0);
            bulk_commit_group();
        }
        if constexpr (XG == 1) store_box_to_peers(p, buf, 64, true, row0, lane, col);
        ++nbuf;
        return;
    }
    uint4* srow = reinterpret_cast<uint4*>(stg + lane * kEpiPitch);
#pragma unroll
    for (int j = 0; j < 4; ++j)
        srow[j] = make_uint4(pack_half2(f[8 * j], f[8 * j + 1]), pack_half2(f[8 * j + 2], f[8 * j + 3]),
                             pack_half2(f[8 * j + 4], f[8 * j + 5]), pack_half2(f[8 * j + 6], f[8 * j + 7]));
    __syncwarp();
    if constexpr (XG == 1) store_box_to_peers(p, stg, kEpiPitch, false, row0, lane, col);
    const int seg = lane & 3;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int rr = (lane >> 2) + 8 * j;
        const int grow = row0 + rr;
        const int gcol = col + seg * 8;
        if (grow < p.M && gcol < p.N) {
            const uint4 v = *reinterpret_cast<const uint4*>(stg + rr * kEpiPitch + seg * 16);
            __half* dst = p.C + static_cast<long long>(grow) * p.ldc + gcol;
            if (gcol + 8 <= p.N && p.vec_ok) {
                *reinterpret_cast<uint4*>(dst) = v;
            } else {
                const __half* h = reinterpret_cast<const __half*>(&v);
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    if (gcol + e < p.N) dst[e] = h[e];
            }
        }
    }
    __syncwarp();
}

// CH (two accumulation chains): each unit's k range runs as two independent chains, the first half
// into TMEM accumulator 0 and the second into accumulator 1, summed in fp32 by the epilogue.  The MMA's
// fp32 accumulation truncates the aligned addends, so its error grows with the chain length; two
// half-length chains halve it (K = 16384: per-element error of the fp16 result 3.7e-3 -> see the
// parity tests).  Both accumulators serve one unit, so the epilogue no longer overlaps the next
// unit's main loop; units need >= 2 k-blocks (slices have >= 4).
template <int CG, int BN, int STAGES, int KA, bool ACC_F32, int XG = 0, bool CH = false>
__global__ void __launch_bounds__(192, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   const __grid_constant__ CUtensorMap tmap_c, const TcParams p)
{
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
    using Cfg = TcCfg<CG, BN, STAGES, KA, ACC_F32, XG>;
    constexpr int BM = Cfg::kBM;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * Cfg::kABytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * Cfg::kBBytes);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::kNumBars);
    // 1024-byte aligned: the 64-byte swizzle pattern of the TMA stores is a function of address bits
    uint8_t* epi_stage =
        reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tmem_slot) + 4 + 1023) & ~uintptr_t(1023));

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
        if (blockIdx.x < 256) {
            unsigned int smid;
            asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
            g_trace_cta[blockIdx.x][0] = t;
            g_trace_cta[blockIdx.x][4] = smid;
        }
    }
    const uint32_t rank = (CG == 2) ? cluster_ctarank() : 0u;
    const int cluster_id = blockIdx.x / CG;
    const int num_clusters = gridDim.x / CG;

    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
        if (p.c_tma) prefetch_tmap(&tmap_c);
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
            const uint64_t l2_pol = p.l2_evict_last ? l2_policy_evict_last() : 0ull;
            trace_at(p.trace, 2);
            for (int u = cluster_id; ok && u < p.units; u += num_clusters) {
                const Unit w = unit_info(p, u);
                int tm, tn;
                tile_coords(w.tile, p.tiles_m, p.tiles_n, p.raster_group, tm, tn);
                const int m0 = tm * (BM * CG) + static_cast<int>(rank) * BM;
                // an n-split half tile: BN/2 columns, BN/2/CG per CTA (whole 64-column boxes)
                const int bn_cta = w.half >= 0 ? Cfg::kBNCta / 2 : Cfg::kBNCta;
                const int n0 = tn * BN + (w.half > 0 ? BN / 2 : 0) + static_cast<int>(rank) * bn_cta;
                const uint32_t stage_bytes = Cfg::kABytes + static_cast<uint32_t>(bn_cta) * Cfg::kBK * 2;
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
                        mbar_arrive_expect_tx(fb, stage_bytes);
                    } else {
                        if (rank == 0) mbar_arrive_expect_tx(fb, 2 * stage_bytes);
                        bar = mapa_shared(fb, 0);
                    }
                    auto load = [&](uint32_t dst, const CUtensorMap* map, int c0, int c1) {
                        if (p.l2_evict_last) {
                            if constexpr (CG == 1)
                                tma_load_2d_hint(dst, map, bar, c0, c1, l2_pol);
                            else
                                tma_load_2d_pair_hint(dst, map, bar, c0, c1, l2_pol);
                        } else {
                            if constexpr (CG == 1)
                                tma_load_2d(dst, map, bar, c0, c1);
                            else
                                tma_load_2d_pair(dst, map, bar, c0, c1);
                        }
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
                        for (int j = 0; j < Cfg::kBBoxes; ++j)
                            if (j * 64 < bn_cta) load(b_dst + j * Cfg::kBBox, &tmap_b, n0 + 64 * j, k0);
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
            constexpr uint32_t kIdescHalf =
                idesc_f16(BM * CG, BN / 2, ACC_F32, /*b_mn_major=*/!B_K) | (A_MN ? (1u << 15) : 0u);
            constexpr uint32_t kMnLbo = Cfg::kBK * 128;
            int stage = 0;
            uint32_t phase = 0;
            int it = 0;
            bool ok = true;
            for (int u = cluster_id; ok && u < p.units; u += num_clusters, ++it) {
                const Unit w = unit_info(p, u);
                // alternate accumulators between units, or (chains) both for every unit, signalled on
                // the barriers of accumulator 0
                const int acc = CH ? 0 : (it & 1);
                const uint32_t acc_phase = CH ? (static_cast<uint32_t>(it) & 1u) : (static_cast<uint32_t>(it >> 1) & 1u);
                if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, p.timeout_ns, kErrWaitMma, 100 + acc)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                // first k-block of the second chain (w.kb1: no second chain); units have >= 2 k-blocks
                const int kmid = CH ? (w.kb0 + w.kb1 + 1) / 2 : w.kb1;
                const uint32_t idesc = w.half >= 0 ? kIdescHalf : kIdesc;
                for (int kb = w.kb0; kb < w.kb1; ++kb) {
                    if (!mbar_wait(full_bar(stage), phase, p.timeout_ns, kErrWaitMma, stage)) {
                        ok = false;
                        break;
                    }
                    if (it == 0 && kb == w.kb0) trace_at(p.trace, 3);
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + stage * Cfg::kABytes);
                    const uint32_t b_addr = smem_u32(sB + stage * Cfg::kBBytes);
                    // The last k-block of a ragged K holds zero-filled k-steps: issue only the
                    // 16-deep MMAs that touch k < K (K = 3000: 4 of 8).
                    const int kk_end = min(Cfg::kBK / 16, (p.K - kb * Cfg::kBK + 15) / 16);
#pragma unroll
                    for (int kk = 0; kk < Cfg::kBK / 16; ++kk) {
                        if (kk >= kk_end) break;
                        const uint64_t a_desc =
                            A_MN ? smem_desc_sw128(a_addr + kk * 16 * 128, kMnLbo, 1024)
                                 : smem_desc_sw128(a_addr + (kk >> 2) * Cfg::kABox + (kk & 3) * 32, 16, 1024);
                        const uint64_t b_desc =
                            B_K ? smem_desc_sw128(b_addr + (kk >> 2) * Cfg::kBKBox + (kk & 3) * 32, 16, 1024)
                                : smem_desc_sw128(b_addr + kk * 16 * 128, kMnLbo, 1024);
                        const uint32_t d = kb >= kmid ? tmem_base + static_cast<uint32_t>(BN) : d_tmem;
                        umma_f16<CG>(d, a_desc, b_desc, idesc, ((kb != w.kb0 && kb != kmid) || kk != 0) ? 1u : 0u);
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
                if (p.trace && blockIdx.x < 256) {
                    g_trace_cta[blockIdx.x][1] = globaltimer_ns();
                    g_trace_cta[blockIdx.x][5] = static_cast<unsigned long long>(it + 1);
                }
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
        uint32_t nbuf = 0;       // 32-column chunks stored so far (staging buffer parity)
        McRun mc;                // XG = 2: chunks staged for the next multicast run
        for (int u = cluster_id; u < p.units; u += num_clusters, ++it) {
            const Unit w = unit_info(p, u);
            const int acc = CH ? 0 : (it & 1);
            const uint32_t acc_phase = CH ? (static_cast<uint32_t>(it) & 1u) : (static_cast<uint32_t>(it >> 1) & 1u);
            if (!mbar_wait(tfull_bar(acc), acc_phase, p.timeout_ns, kErrWaitEpilogue, acc)) break;
            if (it == 0 && warp == 2 && lane == 0) trace_at(p.trace, 5);
            if (p.trace && warp == 2 && lane == 0 && blockIdx.x < 256) g_trace_cta[blockIdx.x][6] = globaltimer_ns();
            tc_fence_after();
            int tm, tn;
            tile_coords(w.tile, p.tiles_m, p.tiles_n, p.raster_group, tm, tn);
            const int row0 = tm * (BM * CG) + static_cast<int>(rank) * BM + q * 32;  // this warp's rows
            uint8_t* stg = epi_stage + q * Cfg::kEpiWarp;
            const int col0 = tn * BN + (w.half > 0 ? BN / 2 : 0);
            const int bn_eff = w.half >= 0 ? BN / 2 : BN;  // columns of this unit
            const uint32_t tbase = tmem_base + static_cast<uint32_t>(acc * BN) + (static_cast<uint32_t>(q * 32) << 16);
            const uint32_t tbase2 = tmem_base + static_cast<uint32_t>(BN) + (static_cast<uint32_t>(q * 32) << 16);
            if (w.slice >= 0) {
                // Tail slice.  Arrivals are counted first: every slice but the last to arrive publishes
                // its fp32 partial (lane-major float4 runs: each warp store is one contiguous 512-byte
                // span) and then counts itself as published; the last one waits (bounded) until the
                // others have published, adds them to its own accumulator in slice order and writes C.
                const int ti = w.tile - p.full_units;
                constexpr size_t kRegion = static_cast<size_t>(BM) * BN;
                const size_t warp_off = static_cast<size_t>(q) * 32 * BN;
                int* ctr = p.counters + ((ti * CG + static_cast<int>(rank)) * 4 + q) * 2;  // arrived, published
                int old = 0;
                if (lane == 0) old = atomicAdd(&ctr[0], 1);
                old = __shfl_sync(0xffffffffu, old, 0);
                if (old < p.split - 1) {
                    float* mine = p.ws + (static_cast<size_t>(ti * p.split + w.slice) * CG + rank) * kRegion + warp_off;
#pragma unroll 1
                    for (int c = 0; c < BN; c += 32) {
                        float f[32];
                        acc_chunk<ACC_F32, CH>(tbase + static_cast<uint32_t>(c), tbase2 + static_cast<uint32_t>(c), f);
                        float4* dst = reinterpret_cast<float4*>(mine + c * 32);
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            __stcg(dst + j * 32 + lane, make_float4(f[4 * j], f[4 * j + 1], f[4 * j + 2], f[4 * j + 3]));
                    }
                    __threadfence();
                    __syncwarp();
                    if (lane == 0) atomicAdd(&ctr[1], 1);
                    if (p.trace && warp == 2 && lane == 0 && blockIdx.x < 256) g_trace_cta[blockIdx.x][7] = globaltimer_ns();
                } else {
                    bool ok = true;
                    if (lane == 0) ok = wait_count_at_least(&ctr[1], p.split - 1, p.timeout_ns, kErrWaitEpilogue, 300 + q);
                    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
                    if (p.trace && warp == 2 && lane == 0 && blockIdx.x < 256) g_trace_cta[blockIdx.x][7] = globaltimer_ns();
                    // The pipeline buffers double as staging only when this slice is the cluster's last
                    // unit; otherwise the producer is already filling them for the next tile, and the
                    // partials are read straight from L2 (one contiguous 512-byte span per warp load).
                    const bool staged = u + num_clusters >= p.units;
                    if (ok && !staged) {
                        __threadfence();
                        // The partial of the first other slice is fetched one chunk ahead, so its L2
                        // latency overlaps the previous chunk's sums and stores.
                        const int first = w.slice == 0 ? 1 : 0;
                        const float4* first_src = reinterpret_cast<const float4*>(
                            p.ws + (static_cast<size_t>(ti * p.split + first) * CG + rank) * kRegion + warp_off);
                        float4 nxt[8];
#pragma unroll
                        for (int jj = 0; jj < 8; ++jj) nxt[jj] = __ldcg(first_src + jj * 32 + lane);
#pragma unroll 1
                        for (int c = 0; c < BN && col0 + c < p.N; c += 32) {
                            uint32_t r[32];
                            tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>(c), r);
                            float4 cur[8];
#pragma unroll
                            for (int jj = 0; jj < 8; ++jj) cur[jj] = nxt[jj];
                            if (c + 32 < BN && col0 + c + 32 < p.N) {
#pragma unroll
                                for (int jj = 0; jj < 8; ++jj) nxt[jj] = __ldcg(first_src + (c + 32) * 8 + jj * 32 + lane);
                            }
                            tmem_ld_wait();
                            float own[32];
                            tmem_words_to_f32<ACC_F32>(r, own);
                            if constexpr (CH) {
                                tmem_ld_32x32b_x32(tbase2 + static_cast<uint32_t>(c), r);
                                tmem_ld_wait();
                                float own2[32];
                                tmem_words_to_f32<ACC_F32>(r, own2);
#pragma unroll
                                for (int i = 0; i < 32; ++i) own[i] += own2[i];
                            }
                            // f = ((p_0 + p_1) + p_2) + ... in slice order, p_own taken from TMEM
                            float f[32];
#pragma unroll 1
                            for (int s2 = 0; s2 < p.split; ++s2) {
                                float4 v[8];
                                if (s2 == w.slice) {
#pragma unroll
                                    for (int jj = 0; jj < 8; ++jj)
                                        v[jj] = make_float4(own[4 * jj], own[4 * jj + 1], own[4 * jj + 2], own[4 * jj + 3]);
                                } else if (s2 == first) {
#pragma unroll
                                    for (int jj = 0; jj < 8; ++jj) v[jj] = cur[jj];
                                } else {
                                    const float4* src = reinterpret_cast<const float4*>(
                                        p.ws + (static_cast<size_t>(ti * p.split + s2) * CG + rank) * kRegion + warp_off +
                                        static_cast<size_t>(c) * 32);
#pragma unroll
                                    for (int jj = 0; jj < 8; ++jj) v[jj] = __ldcg(src + jj * 32 + lane);
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
                            store_rows<XG>(p, &tmap_c, stg, row0, lane, col0 + c, f, nbuf, mc);
                        }
                    } else if (ok) {
                        __threadfence();
                        if (lane == 0) fence_proxy_async_global();  // published partials precede the bulk reads
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
                                float own[32];
                                acc_chunk<ACC_F32, CH>(tbase + static_cast<uint32_t>(c), tbase2 + static_cast<uint32_t>(c),
                                                       own);
                                // f = ((p_0 + p_1) + p_2) + ... in slice order, p_own taken from TMEM
                                float f[32];
                                int j = 0;
#pragma unroll 1
                                for (int s2 = 0; s2 < p.split; ++s2) {
                                    float4 v[8];
                                    if (s2 == w.slice) {
#pragma unroll
                                        for (int jj = 0; jj < 8; ++jj)
                                            v[jj] = make_float4(own[4 * jj], own[4 * jj + 1], own[4 * jj + 2], own[4 * jj + 3]);
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
                                store_rows<XG>(p, &tmap_c, stg, row0, lane, col0 + c, f, nbuf, mc);
                            }
                            __syncwarp();
                        }
                    }
                    if (lane == 0) {  // every slice has arrived and published: ready for the next launch
                        ctr[0] = 0;
                        ctr[1] = 0;
                    }
                }
            } else {
#pragma unroll 1
                for (int c = 0; c < bn_eff; c += 32) {
                    float f[32];
                    acc_chunk<ACC_F32, CH>(tbase + static_cast<uint32_t>(c), tbase2 + static_cast<uint32_t>(c), f);
                    if (col0 + c < p.N) {
                        store_rows<XG>(p, &tmap_c, stg, row0, lane, col0 + c, f, nbuf, mc);
                    }
                }
            }
            if constexpr (XG == 2) mc_flush(p, stg, row0, lane, mc);
            tc_fence_before();
            __syncwarp();
            if (warp == 2 && lane == 0) {
                trace_at(p.trace, 6);
                if (p.trace && blockIdx.x < 256) g_trace_cta[blockIdx.x][2] = globaltimer_ns();
            }
            if (lane == 0) {
                if constexpr (CG == 1)
                    mbar_arrive(tempty_bar(acc));
                else
                    mbar_arrive_cluster(mapa_shared(tempty_bar(acc), 0));
            }
        }
        if (p.c_tma && lane == 0) bulk_wait_group_all();  // C written before the CTA exits
        // multicast stores are ordered at system scope before the kernel's completion is observed
        if constexpr (XG == 2) asm volatile("fence.acq_rel.sys;" ::: "memory");
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
        if (blockIdx.x < 256) g_trace_cta[blockIdx.x][3] = t;
        if (blockIdx.x == 0) g_trace[7] = t;
        atomicMin(&g_trace[10], t);
        atomicMax(&g_trace[11], t);
    }
#endif
}

}  // namespace vk
