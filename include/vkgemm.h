/*
 * vkgemm -- B200 (sm_100a) GEMM library behind a plain C ABI.
 *
 * This is the drop-in boundary for the GEMM hot path of VibeKernel's playground task-1.
 * The reference's plugin interface is the C++ template
 *
 *     template <> void playground::matmul<DType, Version>(size_t m, size_t n, size_t k,
 *                                                         const DType* A, const DType* B, DType* C);
 *
 * declared by PLAYGROUND_MATMUL_DEC and called by PLAYGOUND_MATMUL_CALL
 * (results/naive_cycle4/include/playground/matmul.hpp:11-23), with one full specialization per
 * version file `matmul_<dtype>_v<N>_*.cu` (results/naive_cycle6/src/CMakeLists.txt:27-50).  Every
 * v>=1 specialization in this repository (task-1/src/matmul_f16, task-1/src/matmul_f32) is a
 * one-line call into the entry points below.
 *
 * Conventions (same as the reference):
 *   - row-major A[m x k], B[k x n], C[m x n]; lda = k, ldb = n, ldc = n unless given;
 *   - C = A * B (alpha = 1, beta = 0; matmul_f16_v0_cblas.cpp:22-23);
 *   - device pointers, the call is asynchronous on the given stream (NULL = legacy default
 *     stream, which is what the reference driver uses, main.cpp:55-62).
 * Differences (by design): every entry point returns a vk_status instead of exiting; shapes
 * are int64; there is no CPU fallback -- an unsupported request is an error.
 */
#ifndef VKGEMM_H_
#define VKGEMM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes.  0 = success; negative = error (details in vk_last_error_string()). */
typedef enum vk_status {
    VK_OK = 0,
    VK_ERR_INVALID_ARGUMENT = -1, /* null pointer, negative size, ld too small, bad enum      */
    VK_ERR_UNSUPPORTED = -2,      /* combination not implemented (e.g. f32 with f16 acc)      */
    VK_ERR_CUDA = -3,             /* a CUDA runtime/driver call failed                        */
    VK_ERR_DEVICE_TIMEOUT = -4,   /* a bounded device-side wait ran out (see vk_device_error) */
    VK_ERR_NO_DEVICE = -5,        /* no sm_100 device / library built for another arch       */
    VK_ERR_NCCL = -6,             /* an NCCL call failed in the sharded layer                 */
    VK_ERR_ALIGNMENT = -7         /* explicitly requested kernel cannot take these strides    */
} vk_status;

typedef enum vk_dtype {
    VK_DTYPE_F16 = 0, /* IEEE binary16 in and out (playground::float16_t = half) */
    VK_DTYPE_F32 = 1  /* IEEE binary32 in and out                                */
} vk_dtype;

typedef enum vk_acc {
    VK_ACC_F32 = 0, /* fp32 accumulation (the rubric tier)                  */
    VK_ACC_F16 = 1  /* fp16 accumulation (tensor-core f16-accumulate tier)   */
} vk_acc;

typedef enum vk_algo {
    VK_ALGO_AUTO = 0,     /* pick the fastest kernel that can take the shape/strides          */
    VK_ALGO_TC_2SM = 1,   /* tcgen05 cta_group::2 pair kernel, 256-row tiles, persistent       */
    VK_ALGO_TC_1SM = 2,   /* tcgen05 cta_group::1 kernel, 128-row tiles, persistent            */
    VK_ALGO_FFMA = 3,     /* fp32 CUDA-core SGEMM (register-blocked FFMA)                      */
    VK_ALGO_SIMT = 4      /* predicated CUDA-core fp16 kernel: any strides/alignment           */
} vk_algo;

/* One GEMM: C[m x n] = A[m x k] * B[k x n], row-major with leading dimensions in elements. */
typedef struct vk_gemm_args {
    const void* A;
    const void* B;
    void* C;
    float* C_f32;   /* optional (may be NULL): fp32 copy of the result before rounding to fp16,
                       dense m x n (ld = n); used by the verification launch.  fp16 only. */
    int64_t m, n, k;
    int64_t lda, ldb, ldc; /* 0 = dense default (k, n, n) */
    int32_t dtype;         /* vk_dtype */
    int32_t acc;           /* vk_acc   */
    int32_t algo;          /* vk_algo  */
    int32_t tile_n;        /* 0 = default; TC kernels: 128 or 256 (pair tile N)               */
    void* stream;          /* cudaStream_t; NULL = legacy default stream                       */
} vk_gemm_args;

/* Replaces: playground::matmul<DType, Version> specialisations, matmul.hpp:16-23.
 * The general entry point.  Asynchronous; returns before the kernel finishes. */
int vk_gemm(const vk_gemm_args* args);

/* Extensions beyond the reference's NN, alpha = 1, beta = 0 contract (no counterpart in the
 * reference; the survey's "next" rows: generic layouts and epilogue fusion):
 *   C = act(alpha * op(A) * op(B) + beta * C_in + bias)
 * op(A) = A (stored m x k, lda >= k) or, with trans_a, A^T of a matrix stored k x m (lda >= m);
 * op(B) = B (stored k x n, ldb >= n) or, with trans_b, B^T of a matrix stored n x k (ldb >= k).
 * C_in (m x n, leading dimension ldc_in, 0 = ldc; may be C itself) is read when beta != 0; bias is
 * a length-n row vector broadcast over rows; both have C's element type.  The epilogue runs in
 * fp32 before the single rounding to the output type.  Transposed operands: fp16 only.  The
 * tensor-core kernels take all four layouts when the stored matrices meet the TMA rule (16-byte
 * aligned, leading dimension a multiple of 8); otherwise VK_ALGO_AUTO uses the predicated kernel. */
typedef enum vk_activation { VK_ACT_NONE = 0, VK_ACT_RELU = 1 } vk_activation;

typedef struct vk_gemm_ext {
    int32_t trans_a, trans_b;
    float alpha, beta;
    const void* C_in;
    int64_t ldc_in;
    const void* bias;
    int32_t activation; /* vk_activation */
} vk_gemm_ext;

/* vk_gemm with the extensions above; ext == NULL is exactly vk_gemm. */
int vk_gemm_ex(const vk_gemm_args* args, const vk_gemm_ext* ext);

/* Fused compute + all-gather (no counterpart in the reference): vk_gemm for the fp16 tensor-core
 * kernels that also stores every finished box of C, at the same row / column offsets and with the
 * same ldc, into each of the npeers (0..7) buffers peer_C[i] -- typically the matching rows of the
 * other GPUs' full C, mapped with peer access (one process) or vk_ipc_import (one process per GPU).
 * The peer stores are plain 16-byte stores over NVLink issued by the epilogue while the main loop
 * runs on (no TMA on peer memory).  The caller orders the peers' reads after this kernel (an event
 * or a collective).  fp16 only; operands that would need the predicated kernel are rejected. */
int vk_gemm_peers(const vk_gemm_args* args, void* const* peer_C, int32_t npeers);

/* Fused compute + all-gather through NVLink SHARP multicast (no counterpart in the reference): vk_gemm
 * for the fp16 tensor-core kernels whose epilogue stores every finished box of C ONCE, with
 * multimem.st, to C_mc -- the multicast view of the same bytes as C in a buffer from vk_mc_alloc
 * (one process) or vk_mc_attach (one process per GPU).  The NVSwitch writes each box into the same
 * offset of every member GPU's buffer, this GPU's included, so C is not stored locally as well and the
 * SMs issue 1/(P-1) of the bytes of vk_gemm_peers.  C must lie inside the calling device's view of a
 * live multicast buffer and C_mc must be its multicast address (checked); n and ldc multiples of 8.
 * The caller orders the other GPUs' reads after this kernel (an event join or a collective). */
int vk_gemm_mc(const vk_gemm_args* args, void* C_mc);

/* Multicast (NVLS) buffers, no counterpart in the reference.  A buffer has one view per member GPU
 * (that GPU's own memory, used as its full C) and one multicast view.  Needs an NVSwitch system
 * (vk_mc_supported).  Teardown rule: every member must have finished with the buffer (synchronise and
 * barrier) before any member frees / detaches it, and no member may exit while attached.
 *   vk_mc_supported  *out = 1 when `device` supports NVLS multicast.
 *   vk_mc_alloc      one process, ndev GPUs: ptrs[i] = device i's view (bytes, rounded up to the
 *                    multicast granularity), *mc_ptr = the multicast view; vk_mc_free(mc_ptr) frees.
 *   vk_mc_create     one process per GPU, on the owner: creates the object for `members` GPUs and
 *                    exports it; share[3] = {owner pid, descriptor, padded bytes} to send to the others.
 *   vk_mc_import     on every other member: fetches the owner's descriptor (pidfd_getfd, same node).
 *   vk_mc_attach     on every member (owner included), collectively: adds the device, creates and binds
 *                    its memory (blocks until every member has attached) and maps both views.
 *   vk_mc_detach     on every member, after a barrier: unmaps, unbinds and releases this member. */
typedef struct vk_mc_team vk_mc_team;
int vk_mc_supported(int device, int* out);
int vk_mc_alloc(int32_t ndev, const int32_t* devices, size_t bytes, void** ptrs, void** mc_ptr);
int vk_mc_free(void* mc_ptr);
int vk_mc_create(int device, int32_t members, size_t bytes, vk_mc_team** team, int64_t* share);
int vk_mc_import(int device, int32_t members, const int64_t* share, vk_mc_team** team);
int vk_mc_attach(vk_mc_team* team, void** local_ptr, void** mc_ptr, size_t* bytes);
int vk_mc_detach(vk_mc_team* team);

/* No counterpart in the reference.  Same contract as vk_gemm for the fp16 tensor-core kernels
 * (algo AUTO, TC_2SM or TC_1SM; 16-byte aligned A/B with lda, ldb multiples of 8), for callers
 * that cannot allocate device memory: code running during CUDA graph capture, applications whose
 * device memory belongs to a custom pool or framework allocator that forbids side allocations,
 * and hosts that budget every byte up front.  It calls no cudaMalloc/cudaFree: the scratch that
 * vk_gemm would cudaMalloc once (fp32 partials of the k-sliced last wave, plus arrival counters)
 * lives in a file-scope device array of 16 KiB + 20 MiB that every GPU loading the library holds
 * until exit.  Enough for any problem on B200 (148 SMs); a plan needing more is rejected with
 * VK_ERR_UNSUPPORTED and a message giving both sizes.  The first call on each device looks up the
 * array's device address (cudaGetSymbolAddress, with that device current): make that first call
 * before any stream capture.  Every call shares the one array and zeroes its counters on the
 * given stream first, so calls that overlap on the GPU (other streams, other threads) race: order
 * them on one stream.  The caller still passes A, B and C.  Asynchronous like vk_gemm. */
int vk_gemm_noalloc(const vk_gemm_args* args);

/* Replaces: the reference harness's host-side flow around one matmul call -- copy A and B to the
 * device, call, copy C back (test_data.hpp:177-196, main.cpp:46-62) -- for callers whose A, B and C
 * are in HOST memory.  Same fields as vk_gemm (A, B, C are host pointers; C_f32 must be NULL;
 * `stream` is ignored).  The copies are pipelined with the computation in row blocks of
 * `block_rows` rows (0 = automatic, about 4 blocks); device staging buffers are cached per device
 * (freed by vk_shutdown).  Synchronous: returns when C is in host memory.  Pinned host memory
 * gives full PCIe bandwidth.  Calls from several threads are serialised. */
int vk_gemm_host(const vk_gemm_args* args, int32_t block_rows);

/* Replaces: template<> matmul<float16_t, V>(m, n, k, A, B, C), matmul.hpp:16-19 with
 * DType = float16_t (system.hpp:25).  `version` selects the kernel exactly as the
 * `--ver N` file does in the reference build (CMakeLists.txt:31-33):
 *   1 = tcgen05 pair kernel, fp32 accumulate (default champion)
 *   2 = tcgen05 pair kernel, fp16 accumulate
 *   3 = tcgen05 single-CTA kernel, fp32 accumulate
 *   4 = predicated CUDA-core kernel, fp32 accumulate (any alignment)
 * Version 0 (the cBLAS CPU ground truth) is not part of this library. Default stream. */
int vk_matmul_f16(int version, size_t m, size_t n, size_t k, const void* A, const void* B, void* C);

/* Replaces: template<> matmul<float32_t, V>(m, n, k, A, B, C), matmul.hpp:16-19 with
 * DType = float32_t.  version 1 = FFMA SGEMM.  Default stream. */
int vk_matmul_f32(int version, size_t m, size_t n, size_t k, const float* A, const float* B, float* C);

/* Multi-GPU row-block sharding (no counterpart in the reference, which is single-GPU,
 * README.md:161; this is the layer BASELINE.json asks for).  GPU r of `ngpu` computes rows
 * [r*m/ngpu, (r+1)*m/ngpu) of C from its own A slice and a full copy of B; with
 * allgather_c != 0 an NCCL all-gather then leaves the full C on every GPU.  All pointers
 * are per-device arrays of length ngpu (A[r] holds only GPU r's rows, dense, ld = k;
 * B[r] the full k x n matrix; C[r] the full m x n output buffer on GPU r, of which GPU r
 * writes its own row block).  Synchronous: returns after every GPU finished. */
typedef struct vk_shard_args {
    int32_t ngpu;
    const int32_t* devices;   /* CUDA device ordinals, length ngpu */
    const void* const* A;     /* per GPU: its (m/ngpu) x k slice  */
    const void* const* B;     /* per GPU: full k x n              */
    void* const* C;           /* per GPU: full m x n buffer       */
    int64_t m, n, k;
    int32_t dtype, acc, algo; /* as in vk_gemm_args               */
    int32_t allgather_c;      /* 0 = local row block only; 1 = NCCL all-gather after the GEMMs;
                                 2 = pipelined: each GPU computes its rows in two chunks and pushes
                                 every finished chunk to all peers with peer-to-peer copies (copy
                                 engines over NVLink) while the next chunk is computed;
                                 3 = fused: each GPU's epilogue stores every finished box of C into
                                 all peers' C as well (vk_gemm_peers; fp16, at most 8 GPUs);
                                 4 = NVLS: C[r] are the views of one vk_mc_alloc buffer and each
                                 GPU's epilogue stores every box once to its multicast view
                                 (vk_gemm_mc; fp16) */
    float* times_ms;          /* optional, length 2: [0] compute max over GPUs, [1] all-gather */
} vk_shard_args;

int vk_gemm_sharded(const vk_shard_args* args);

/* Peer-memory plumbing for one-process-per-GPU jobs (torchrun), no counterpart in the reference:
 * the pipelined all-gather of the row-sharded GEMM (vibekernel_b200/dist_gemm.py) maps every
 * peer's full C buffer into its own process and pushes each finished chunk of its rows into them
 * with the copy engines over NVLink while the next chunk is computed.
 *   vk_ipc_export   CUDA IPC handle of the allocation holding device buffer `ptr`, plus the
 *                   buffer's byte offset inside it (allocators hand out pieces of allocations);
 *   vk_ipc_import   map a handle exported by ANOTHER process on this node into this process
 *                   (plain peer mapping, lazy peer access); *out_ptr = the peer's buffer;
 *   vk_ipc_release  unmap a pointer returned by vk_ipc_import;
 *   vk_copy_async   cudaMemcpyAsync of `bytes` device bytes on `stream` (peer pointers allowed). */
typedef struct vk_ipc_handle {
    uint8_t handle[64]; /* cudaIpcMemHandle_t */
    uint64_t offset;    /* byte offset of the buffer inside the exported allocation */
} vk_ipc_handle;

int vk_ipc_export(const void* ptr, vk_ipc_handle* out);
int vk_ipc_import(const vk_ipc_handle* handle, void** out_ptr);
int vk_ipc_release(void* ptr);
int vk_copy_async(void* dst, const void* src, size_t bytes, void* stream);

/* Device and library state. */
int vk_init(int device);                 /* optional: warm per-device state (SM count, attrs) */
int vk_shutdown(void);                   /* frees per-device state and NCCL communicators;
                                            call it before any cudaDeviceReset, since the library
                                            caches per-context facts (kernel attributes, the
                                            no-allocation array's address) until then            */
const char* vk_last_error_string(void);  /* thread-local message for the last failure        */
const char* vk_version_string(void);

/* Reads (and optionally clears) the device error word written by a bounded device-side wait
 * that gave up: 0 = no error, else (code << 32 | detail).  Synchronises the device. */
int vk_device_error(int device, uint64_t* out_word, int clear);

/* Failure-detection self-test: launches one block whose thread waits on an mbarrier that
 * nothing arrives on, with the same bounded wait the GEMM kernels use, for `timeout_us`
 * microseconds.  Returns VK_ERR_DEVICE_TIMEOUT when the wait ran out as designed (and
 * clears the device error word again), VK_OK never. */
int vk_selftest_wait_timeout(int device, int64_t timeout_us);

/* Per-call device-side wait limit for the GEMM kernels, nanoseconds (default 2e9). */
int vk_set_wait_timeout_ns(uint64_t ns);

/* Process-wide tuning knobs (no counterpart in the reference, whose versions hard-code them):
 *   "tail_split"      1 (default) = cut the tiles of a partial last wave (into column halves or
 *                     k-slices, see "tail_nsplit"), 0 = off
 *   "tail_nsplit"     1 (default) = prefer column halves for the last wave when it is at most half
 *                     full; 0 = k-slices only
 *   "tail_first"      1 (default) = when there is at least one full wave, k >= 2560 and the
 *                     leftover tiles can be cut into 2..4 k-slices, those slices run before the
 *                     whole tiles (their partial sums are reduced while the tensor pipes work on
 *                     whole tiles); 0 = leftover tiles run last, policy of "tail_nsplit"
 *   "k_chains"        0 (default) = off; 1 = when k > 8192, the default pair kernel runs each output tile's
 *                     k range as two accumulation chains (its two TMEM accumulators) summed in fp32 by the
 *                     epilogue: the tensor cores' truncating fp32 accumulation drifts about half as far
 *                     (16384^3: per-element error 3.7e-3 -> 1.9e-3), at the cost of the epilogue /
 *                     main-loop overlap (up to 19 % slower on short-M shapes); 2 = always (k > 128)
 *   "tma_store"       1 (default) = the tensor-core kernels write fp16 C with TMA tile stores when C
 *                     is 16-byte aligned with a pitch that is a multiple of 8 elements; 0 = always
 *                     per-lane coalesced stores (the path taken for any other C)
 *   "l2_evict_last"   1 (default) = the tensor-core kernels load A and B tiles with an L2
 *                     evict_last cache policy; 0 = default caching
 *   "raster_group"    tiles along M per rasterisation group of the persistent scheduler (8)
 *   "bk_2sm256"       k per pipeline stage of the 256-column pair kernel: 128 (default, 3 stages
 *                     of 64 KB) or 64 (6 stages of 32 KB)
 *   "wait_timeout_ns" same as vk_set_wait_timeout_ns
 *   "gather_timeout_ms" host-side deadline of vk_gemm_sharded's NCCL all-gather (60000): when it passes,
 *                     or NCCL reports an asynchronous error, the communicators are aborted
 *                     (ncclCommAbort) and the call returns VK_ERR_NCCL instead of waiting forever
 *   "repack"          1 (default) = VK_ALGO_AUTO copies an fp16 operand whose pitch or base breaks the
 *                     TMA rule into a 16-byte-pitched scratch buffer (cached per stream) and runs the
 *                     tensor-core kernel; 0 = such problems run on the predicated CUDA-core kernel
 *   "sgemm_v2"        1 (default) = fp32 GEMM uses the cp.async pipelined kernel when A and B are
 *                     16-byte aligned with lda, ldb multiples of 4; 0 = always the register-staged one
 *   "sgemm_paired"    inner product of that kernel: 1 (default) = paired fp32 FMAs of sm_100 (two
 *                     fused multiply-adds per instruction), 8 x 16 outputs per thread, 128 threads;
 *                     2 = paired FMAs, 8 x 8 per thread, 256 threads; 0 = scalar FMAs, 8 x 8.  All
 *                     three give bitwise the same results
 *   "clock_probe"     1 = the tensor-core kernels accumulate the SM cycles and nanoseconds of
 *                     their first CTA (read with vk_read_clock_probe); 0 (default) = off
 *   "trace"           1 = the tensor-core kernels record a launch timeline (vk_read_trace)
 * Returns VK_ERR_INVALID_ARGUMENT for an unknown name or value. */
int vk_set_option(const char* name, int64_t value);

/* Test hook (no counterpart in the reference; touches no device): the work decomposition the
 * persistent tensor-core kernels would use for `tiles` output tiles of `num_kb` k-blocks on
 * `max_units` co-resident clusters, from the same planner and unit decoder as the launches.
 * flags: 1 = tail split allowed, 2 = column halves allowed, 4 = slices-first allowed (also needs
 * k >= 2560).  out_plan[6] = {units, whole tiles, k-slices per tail tile, column halves (0/1),
 * slices first (0/1), clusters launched}; out_units (optional, 4 ints per unit, room for
 * max_units_out units) = {tile, first k-block, end k-block, slice index | 100 + column half | -1}. */
int vk_debug_schedule(int64_t tiles, int32_t num_kb, int32_t max_units, int64_t k, int32_t flags,
                      int32_t* out_plan, int32_t* out_units, int32_t max_units_out);

/* Test hook (no counterpart in the reference; touches no device): runs the host-side watchdog that
 * guards vk_gemm_sharded's NCCL all-gather against a fake completion query that reports "done" after
 * `done_after_polls` polls (< 0: never) or "failed" at poll `fail_at_poll` (<= 0: never).  *aborted counts
 * the abort calls, *polls the queries.  Returns VK_OK or VK_ERR_NCCL like the real gather. */
int vk_debug_watchdog(int64_t deadline_ms, int32_t done_after_polls, int32_t fail_at_poll, int32_t* aborted,
                      int64_t* polls);

/* Clock probe (no counterpart in the reference, whose scores were confounded by the unlogged
 * SM clock, README.md:160): out3 = {SM cycles, nanoseconds, launches} accumulated since the last
 * clear; cycles / ns is the SM clock in GHz that the kernels actually ran at.  Synchronises. */
int vk_read_clock_probe(int device, uint64_t* out3, int clear);

/* Launch timeline of the last tensor-core launch made with the "trace" option (no counterpart
 * in the reference), %globaltimer nanoseconds: [0] CTA 0 entry, [1] prologue done, [2] first
 * TMA issued, [3] first stage full at the MMA issuer, [4] last MMA commit, [5] first accumulator
 * ready at the epilogue, [6] last epilogue store issued, [7] CTA 0 exit, [8]/[9] earliest/latest
 * CTA entry, [10]/[11] earliest/latest CTA exit.  Read once, re-arm for the next launch first
 * (call it once before tracing).  Synchronises. */
int vk_read_trace(int device, uint64_t* out16);

/* Per-CTA part of the same timeline (no counterpart in the reference): for the first max_ctas CTAs
 * (at most 256), eight words each: entry, last MMA commit (pair leaders / single CTAs), last epilogue
 * store, exit (%globaltimer ns), SM id, units processed, last accumulator ready at the epilogue,
 * k-sliced tail: partial published / all other partials published.  Synchronises. */
int vk_read_trace_cta(int device, uint64_t* out, int max_ctas);

#ifdef __cplusplus
}
#endif

#endif /* VKGEMM_H_ */
