// gemm_sm100.cu -- persistent tcgen05 GEMM with the fused bias / HardSigmoid epilogue (sm_100a).
//
// Computes Y[M,N] = act(X[M,K] * W[N,K]^T + b[N]) in FP16 with FP32 accumulation in TMEM.
// It replaces the reference's per-output-tile NPU task chain
//   MM (first K tile) -> MM_ACC (each further K tile, FP16 ping-pong accumulators)
//   -> EW (bias) -> LUT (HardSigmoid)        research/custom-ops/src/linear_hardsigmoid.c:51-82
// with one launch. Two variants share the code (template CG = CTA group):
//   CG=2  a cluster of two CTAs on a TPC computes a 256x256 output tile with the 2-SM UMMA
//         (tcgen05.mma.cta_group::2, M=256 N=256 K=16): each CTA stages its own 128 rows of X and
//         128 rows of W per 64-wide K block (32 KB, 6-stage ring), so per SM the shared-memory
//         and L2 traffic per FLOP is two thirds of the single-SM tile. Used for M > 128.
//   CG=1  one CTA computes a 128x256 tile with tcgen05.mma.cta_group::1 (48 KB, 4-stage ring).
// Roles per CTA (384 threads):
//   warp 0      TMA producer (one thread): X and W boxes, 128-byte swizzle, into the ring; both
//               CTAs of a pair signal the leader's full barrier (.cta_group::2, no multicast)
//   warp 1      MMA issuer (one thread, leader CTA only): tcgen05.mma kind::f16 into one of two
//               256-column TMEM accumulators; tcgen05.commit (multicast to both CTAs of a pair)
//               frees ring stages and publishes finished accumulators
//   warp 2      TMEM allocator (512 columns)
//   warps 4-11  epilogue, each on its 32-lane TMEM quarter and 128-column half:
//                 - FP32 mode: tcgen05.ld, y = fp16(act(acc + b)) (+ residual);
//                 - tile-16 modes (the reference's FP16-K-TILING numerics): the MMA warp closes an
//                   accumulator every 256 K; the epilogue folds run = fp16(run + chunk) with packed
//                   FP32 adds into 64 registers (unrolled, the TMEM loads software-pipelined) and
//                   hands the accumulator straight back -- the last chunk's too -- then finishes
//                   the tile from registers (affine = fp16(run + b), HardSigmoid, residual, or the
//                   gate·up product of a packed gate|up weight) while the MMA warp starts the next
//                   tile: with only two accumulators a finish that held one would stall the MMAs;
//               FP16 results leave through one TMA tile store per warp and 32x32 box (staged in
//               2 KB of shared memory per warp), or per-thread 16-byte stores where Y does not
//               allow a tensor map.
// Tiles are scheduled persistently (cluster c takes tiles c, c + clusters, ...) so the TMA/MMA of
// the next tile overlaps the epilogue of the previous one through the two TMEM accumulators.
//
// Every mbarrier wait is bounded (globaltimer): on expiry the CTA raises the timeout flag, stops
// issuing work, waits (bounded) for its own TMA loads and MMAs in flight, frees TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string.h>

#include "common.cuh"
#include "gemm_sm100.h"
#include "mbarrier.cuh"

namespace b2 {
namespace gemm {

constexpr int BK = 64;
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 128 + EPI_WARPS * 32;
constexpr uint32_t SMEM_LIMIT = 232448;              // dynamic shared memory per CTA on sm_100
constexpr int TILE_N = 256;                          // output columns per tile

// Tile configuration: CG CTAs per cluster (1 or 2) and TN output columns per tile (64, 128 or 256;
// the 2-SM pair always 256).
template <int CG, int TN>
struct Cfg {
    static constexpr int BM = 128 * CG;                 // output rows per tile (per CTA: 128)
    static constexpr int B_ROWS = TN / CG;              // W rows staged by each CTA
    static constexpr uint32_t A_BYTES = 128 * BK * 2;
    static constexpr uint32_t B_BYTES = B_ROWS * BK * 2;
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
    // output staging of the TMA tile stores: one 32 x 32 FP16 box (2 KB) per epilogue warp
    static constexpr uint32_t OUT_BYTES = EPI_WARPS * 32 * 64;
    static constexpr int STAGES = (int)((SMEM_LIMIT - 1024 - 512 - OUT_BYTES) / STAGE_BYTES);
    static constexpr int NUM_BARS = 2 * STAGES + 2 + 2 + 1;
    static constexpr uint32_t SMEM_BYTES = STAGES * STAGE_BYTES + OUT_BYTES + 1024 + NUM_BARS * 8 + 16;
    static constexpr uint32_t TMEM_COLS = 2 * TN;       // two accumulators (power of two >= 32)
    // Instruction descriptor, kind::f16: D=F32 (bits 4-5 = 1), A=B=F16 (0), both K-major,
    // N>>3 at bits 17-22, M>>4 at bits 24-28.
    static constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(TN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
    static_assert(SMEM_BYTES <= SMEM_LIMIT, "shared memory");
};

// ----------------------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Address of the same shared variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
template <int CG>
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c0, int c1) {
    if constexpr (CG == 2) {
        // `bar` is the leader CTA's barrier (shared::cluster address); no multicast.
        asm volatile(
            "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
            " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
            "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
            : "memory");
    } else {
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
            " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
            "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
            : "memory");
    }
}
// One 3-D box of a cube view's map (8 channels x 128 rows x 8 channel groups) into shared memory.
template <int CG>
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c0, int c1,
                                            int c2) {
    if constexpr (CG == 2) {
        asm volatile(
            "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
            " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
            "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
            : "memory");
    } else {
        asm volatile(
            "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
            " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
            "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
            : "memory");
    }
}
// A tensor map in global memory that the host rewrote since the last launch: the tensormap proxy
// must not use a copy of its old contents.
__device__ __forceinline__ void tmap_acquire(const CUtensorMap *map) {
    asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(reinterpret_cast<uint64_t>(map))
                 : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

template <int CG>
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    if constexpr (CG == 2)
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                     : "memory");
    else
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                     : "memory");
}
template <int CG>
__device__ __forceinline__ void tmem_relinquish() {
    if constexpr (CG == 2)
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    else
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
template <int CG>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    if constexpr (CG == 2)
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
    else
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
template <int CG>
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    if constexpr (CG == 2)
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    else
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
}
// Completion of this thread's earlier MMAs arrives on `bar` (in both CTAs of a pair for CG=2).
template <int CG>
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    if constexpr (CG == 2) {
        const uint16_t both = 0x3;
        asm volatile(
            "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
            "h"(both)
            : "memory");
    } else {
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                     : "memory");
    }
}
template <int CG>
__device__ __forceinline__ void umma_commit_local(uint32_t bar) {
    if constexpr (CG == 2)
        asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                     : "memory");
    else
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                     : "memory");
}

// 32 consecutive FP32 columns of this thread's TMEM lane; the wait is in the same asm statement so
// the registers are valid when it returns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, 8-row core groups 1024 B
// apart (SBO), version 1 (sm_100), base offset 0 (stage buffers are 1024-byte aligned).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Shared-memory matrix descriptor of a cube stage: K-major without swizzle, [8 channel groups][128
// rows][8] FP16, i.e. 8-row x 16-byte core matrices 128 bytes apart along M (SBO) and 2048 bytes
// apart along K (LBO); version 1, base offset 0. One K = 16 step advances the start by 4096 bytes.
__device__ __forceinline__ uint64_t cube_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(2048 >> 4) << 16) | ((uint64_t)(128 >> 4) << 32) |
           ((uint64_t)1 << 46);
}
constexpr uint32_t CUBE_K16_STEP = 4096 >> 4;   // descriptor units (16 bytes) per K = 16 step

__device__ __forceinline__ float load_bias(const __half *bias, int col, int n) {
    return (bias && col < n) ? __half2float(bias[col]) : 0.0f;
}


// 32 bias values of columns [cb, cb+32) as floats (zero past n or without bias).
__device__ __forceinline__ void load_bias32(const __half *bias, int cb, int n, float (&b)[32]) {
    if (bias && cb + 32 <= n) {
        const uint4 *bp = reinterpret_cast<const uint4 *>(bias + cb);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint4 u = __ldg(bp + q);
            const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(h[e]);
                b[8 * q + 2 * e] = f.x;
                b[8 * q + 2 * e + 1] = f.y;
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) b[i] = load_bias(bias, cb + i, n);
    }
}

// 32 FP16 values of row `src` at columns [cb, cb+32) as floats (zero past n).
__device__ __forceinline__ void load_half32(const __half *src, int cb, int n, bool vec, float (&r)[32]) {
    if (vec && cb + 32 <= n) {
        const uint4 *sp = reinterpret_cast<const uint4 *>(src + cb);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint4 u = __ldg(sp + q);
            const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(h[e]);
                r[8 * q + 2 * e] = f.x;
                r[8 * q + 2 * e + 1] = f.y;
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = cb + i < n ? __half2float(src[cb + i]) : 0.0f;
    }
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// 32 FP16 results (16 packed pairs) to row `dst` at columns [cb, cb+32), clipped at n.
__device__ __forceinline__ void store32(__half *dst, int cb, int n, bool vec, const uint32_t (&pk)[16]) {
    if (vec && cb + 32 <= n) {
        uint4 *d = reinterpret_cast<uint4 *>(dst + cb);
#pragma unroll
        for (int q = 0; q < 4; ++q) d[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const __half2 h = *reinterpret_cast<const __half2 *>(&pk[i]);
            if (cb + 2 * i < n) dst[cb + 2 * i] = __low2half(h);
            if (cb + 2 * i + 1 < n) dst[cb + 2 * i + 1] = __high2half(h);
        }
    }
}

// 32 FP32 raw accumulators to row `dst` at columns [cb, cb+32), clipped at n.
__device__ __forceinline__ void store32f(float *dst, int cb, int n, bool vec, const float (&v)[32]) {
    if (vec && cb + 32 <= n) {
        float4 *d = reinterpret_cast<float4 *>(dst + cb);
#pragma unroll
        for (int q = 0; q < 8; ++q) d[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (cb + i < n) dst[cb + i] = v[i];
    }
}

// The tile-16 running sum of a thread's 128 columns is 64 half2 registers; piece j (a rolled loop)
// owns [16j, 16j+16). Reading and writing a piece through these selects (static indices only)
// keeps the array in registers -- indexed by j it would live in local memory, and with the ring
// holding 227 KB of shared memory the L1 is too small to keep it: every 256-K chunk would move
// 128 KB per CTA through L2.
template <int N>
__device__ __forceinline__ void run_get(const __half2 (&run)[N], int j, __half2 (&cur)[16]) {
#pragma unroll
    for (int q = 0; q < N / 16; ++q)
        if (q == j) {
#pragma unroll
            for (int i = 0; i < 16; ++i) cur[i] = run[16 * q + i];
        }
}
template <int N>
__device__ __forceinline__ void run_put(__half2 (&run)[N], int j, const __half2 (&cur)[16]) {
#pragma unroll
    for (int q = 0; q < N / 16; ++q)
        if (q == j) {
#pragma unroll
            for (int i = 0; i < 16; ++i) run[16 * q + i] = cur[i];
        }
}

// Two FP32 adds in one instruction (sm_100 packed FP32), each rounded to nearest like __fadd_rn.
__device__ __forceinline__ float2 fadd2_rn(float2 a, float2 b) {
    uint64_t x, y, r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a.x), "f"(a.y));
    asm("mov.b64 %0, {%1, %2};" : "=l"(y) : "f"(b.x), "f"(b.y));
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(x), "l"(y));
    float2 o;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(o.x), "=f"(o.y) : "l"(r));
    return o;
}

// 16 FP32 columns of this thread's TMEM lane, issued without waiting: the registers are valid only
// after tmem_wait16 on the same array (which names them as in/out operands, so no use of them can
// be scheduled before the wait).
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait16(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;\n"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                   "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
                   "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
}

// Folds 16 columns (8 packed pairs) of a 256-K chunk into run[8j, 8j+8).
template <int N>
__device__ __forceinline__ void fold16x(__half2 (&run)[N], int j, const uint32_t (&r)[16], bool first) {
    if (first) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
            run[8 * j + i] = __floats2half2_rn(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float2 s = fadd2_rn(__half22float2(run[8 * j + i]),
                                      make_float2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])));
            run[8 * j + i] = __floats2half2_rn(s.x, s.y);
        }
    }
}

// One fold-only 256-K chunk of the tile-16 modes over this thread's HALF columns: run =
// fp16(chunk) for the first chunk, else fp16(run + chunk) (fold16, two columns per packed add and
// one packing conversion). Unrolled, so every index into `run` is static, and software-pipelined:
// the TMEM load of the next 16 columns is in flight while the current ones are folded. The
// accumulator is handed back (release) as soon as its last columns are in registers.
template <int HALF, int N, typename Release>
__device__ __forceinline__ void fold_chunk(__half2 (&run)[N], uint32_t taddr, bool first, Release release) {
    constexpr int SUB = HALF / 16;
    uint32_t a[16], b[16];
    tmem_ld16_async(taddr, a);
    tmem_wait16(a);
#pragma unroll
    for (int j = 0; j < SUB; ++j) {
        uint32_t (&cur)[16] = (j & 1) ? b : a;
        uint32_t (&nxt)[16] = (j & 1) ? a : b;
        if (j + 1 < SUB) tmem_ld16_async(taddr + 16 * (j + 1), nxt);
        else release();
        fold16x(run, j, cur, first);
        if (j + 1 < SUB) tmem_wait16(nxt);
    }
}

// Hands a drained TMEM accumulator back to the MMA warp (the leader CTA's barrier for a pair).
template <int CG>
__device__ __forceinline__ void release_acc(int lane, uint32_t tempty_leader, uint32_t tempty0, uint32_t acc) {
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
        if constexpr (CG == 2) mbar_arrive_cluster(tempty_leader + 8 * acc);
        else mbar_arrive(tempty0 + 8 * acc);
    }
}

// 32 FP16 results of this thread's row at output columns [x, x+32) (n_out columns in all). With
// p.tma_y the warp writes its 32 rows into its 2 KB staging box (64-byte swizzle: 16-byte chunk q of
// row r at chunk q ^ ((r >> 1) & 3), so the eight rows of each store phase hit distinct banks) and
// one lane issues a TMA tile store of the box (coalesced 64-byte row writes, asynchronous; rows past
// M and columns past n_out are clipped by the tensor map). Otherwise each thread stores its row.
__device__ __forceinline__ void store_out(const Params &p, const CUtensorMap *tmap_y, uint32_t stage, int lane,
                                          int row, bool row_ok, int x, int n_out, const uint32_t (&pk)[16]) {
    if (p.y_cube) {
        // The tile's output cube: this thread's row, four 16-byte atoms (32 columns); consecutive lanes
        // are consecutive rows, so each atom store of the warp is 512 contiguous bytes. Padding rows
        // and columns of the cube receive zeros (the caller's cube must not keep stale values there).
        const CubeOut o = p.y_cube[(row >> 8) * p.y_cube_nt + (x >> 8)];
        const int r = row & 255, c0 = x & 255;
        if (r >= o.prow) return;
        const bool live = r < o.rows;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int a = (c0 >> 3) + q, keep = o.cols - 8 * a;   // channels of atom a inside the tile
            if (8 * a >= o.pcols) break;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (live && keep > 0) {
                v = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
                if (keep < 8) {
                    uint32_t *w = reinterpret_cast<uint32_t *>(&v);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        if (2 * j >= keep) w[j] = 0u;
                        else if (2 * j + 1 >= keep) w[j] &= 0x0000ffffu;
                    }
                }
            }
            *reinterpret_cast<uint4 *>(o.ptr + ((size_t)a * o.prow + r) * 8) = v;
        }
        return;
    }
    if (p.tma_y) {
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");   // box free again
        __syncwarp();
        const uint32_t base = stage + (uint32_t)lane * 64;
#pragma unroll
        for (int q = 0; q < 4; ++q)
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(base + ((q ^ ((lane >> 1) & 3)) << 4)),
                         "r"(pk[4 * q]), "r"(pk[4 * q + 1]), "r"(pk[4 * q + 2]), "r"(pk[4 * q + 3])
                         : "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        const int row0 = row - lane;
        if (lane == 0 && row0 < p.M && x < n_out) {
            asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                             reinterpret_cast<uint64_t>(tmap_y)),
                         "r"(x), "r"(row0), "r"(stage)
                         : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
    } else if (row_ok) {
        store32(p.y + (size_t)row * p.ldy, x, n_out, p.vec_y, pk);
    }
}

// Residual add of the graph's ADD node fused into the store: pk[i] = fp16(res + pk[i]) for the 32
// results of row `row` at columns [cb, cb+32) (the FP32 sum of two FP16 values, rounded once).
__device__ __forceinline__ void add_residual32(const Params &p, int row, int cb, uint32_t (&pk)[16], bool &bad) {
    float rv[32];
    load_half32(p.res + (size_t)row * p.ldr, cb, p.N, p.vec_r, rv);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float2 y = __half22float2(*reinterpret_cast<const __half2 *>(&pk[i]));
        const float s0 = __fadd_rn(rv[2 * i], y.x), s1 = __fadd_rn(rv[2 * i + 1], y.y);
        bad |= f16_overflows(s0) | f16_overflows(s1);
        pk[i] = pack_half2(s0, s1);
    }
}

// Output tile -> (m block, n block). With group_m > 0, tiles are walked in bands of group_m
// m-blocks so that the clusters running at the same time share X and W blocks in L2.
__device__ __forceinline__ void tile_coords(int tile, const Params &p, int &mb, int &nb) {
    if (p.group_m > 0) {
        const int per_group = p.group_m * p.num_n_blocks;
        const int g = tile / per_group, r = tile % per_group;
        const int gm0 = g * p.group_m;
        const int gsz = min(p.group_m, p.num_m_blocks - gm0);
        mb = gm0 + r % gsz;
        nb = r / gsz;
    } else {
        mb = tile % p.num_m_blocks;
        nb = tile / p.num_m_blocks;
    }
}

// Epilogue modes (one kernel instantiation each, so no mode branches in the hot code).
// EPI_GATED is the tile-16 fold with the gate·up product of a packed gate|up weight.
enum : int { EPI_FP32 = 0, EPI_TILE16 = 1, EPI_RAW16 = 2, EPI_RAW32 = 3, EPI_GATED = 4 };

// 16 bias values as packed pairs for columns [cb, cb+32) (zero past n or without bias).
__device__ __forceinline__ void load_bias_pairs(const __half *bias, int cb, int n, __half2 (&b)[16]) {
    if (bias && cb + 32 <= n) {
        const uint4 *bp = reinterpret_cast<const uint4 *>(bias + cb);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint4 u = __ldg(bp + q);
            const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
            for (int e = 0; e < 4; ++e) b[4 * q + e] = h[e];
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const __half lo = (bias && cb + 2 * i < n) ? bias[cb + 2 * i] : __float2half(0.0f);
            const __half hi = (bias && cb + 2 * i + 1 < n) ? bias[cb + 2 * i + 1] : __float2half(0.0f);
            b[i] = __halves2half2(lo, hi);
        }
    }
}

// FP32-mode finish of 32 accumulators: y = fp16(POST ? hsig(acc + b) : acc + b) (finish_fp32),
// specialised on POST for the same reason as finish_piece16.
template <bool POST>
__device__ __forceinline__ void finish_piece32(const float (&v)[32], const float (&b)[32], uint32_t (&pk)[16],
                                               bool &bad) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        float y0 = __fadd_rn(v[2 * i], b[2 * i]), y1 = __fadd_rn(v[2 * i + 1], b[2 * i + 1]);
        if constexpr (POST) {
            y0 = hsig(y0);
            y1 = hsig(y1);
        }
        bad |= f16_overflows(y0) | f16_overflows(y1);
        pk[i] = pack_half2(y0, y1);
    }
}

// Finish of 32 columns from their folded FP16 sums r, specialised on the operator's uniform choices
// so that no element evaluates a bias add or HardSigmoid it does not use (a per-element branch on
// them is if-converted into computing both sides): affine = BIAS ? fp16(run + b) : run, then
// POST ? fp16(hsig(affine)) : affine -- finish_tile16 of common.cuh.
template <bool BIAS, bool POST>
__device__ __forceinline__ void finish_piece16(const __half2 (&r)[16], const __half2 (&b)[16], uint32_t (&pk)[16],
                                               bool &bad) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        if constexpr (!BIAS && !POST) {
            pk[i] = *reinterpret_cast<const uint32_t *>(&r[i]);
            bad |= half_nonfinite(__low2half(r[i])) | half_nonfinite(__high2half(r[i]));
        } else {
            float2 s = __half22float2(r[i]);
            if constexpr (BIAS) {
                const float2 bb = __half22float2(b[i]);
                s = make_float2(round16(__fadd_rn(s.x, bb.x)), round16(__fadd_rn(s.y, bb.y)));
            }
            if constexpr (POST) s = make_float2(hsig(s.x), hsig(s.y));
            bad |= f16_overflows(s.x) | f16_overflows(s.y);
            pk[i] = pack_half2(s.x, s.y);
        }
    }
}

// The gate·up product of 32 hidden columns from their folded gate sums g and up sums u, each finished
// with its bias when it has one.
template <bool BG, bool BU>
__device__ __forceinline__ void gated_piece(const __half2 (&g)[16], const __half2 (&u)[16], const __half2 (&bg)[16],
                                            const __half2 (&bu)[16], const __half *table, int act, uint32_t (&pk)[16],
                                            bool &bad) {
    // the 32 gate-table reads of the piece are independent: all in flight at once (the table is an
    // L2 read: the shared-memory ring leaves little L1)
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        float2 gs = __half22float2(g[i]), us = __half22float2(u[i]);
        if constexpr (BG) {
            const float2 b = __half22float2(bg[i]);
            gs = make_float2(round16(__fadd_rn(gs.x, b.x)), round16(__fadd_rn(gs.y, b.y)));
        }
        if constexpr (BU) {
            const float2 b = __half22float2(bu[i]);
            us = make_float2(round16(__fadd_rn(us.x, b.x)), round16(__fadd_rn(us.y, b.y)));
        }
        const float y0 = gated16(table, gs.x, us.x, act), y1 = gated16(table, gs.y, us.y, act);
        bad |= f16_overflows(y0) | f16_overflows(y1);
        pk[i] = pack_half2(y0, y1);
    }
}

// The finish of a tile-16 tile from its folded FP16 sums in `run` (this thread's row, HALF columns
// from col0), after the last chunk's accumulator was handed back:
//   EPI_TILE16  y = fp16(hsig?(fp16(run + b))) (+ residual), the reference's EW bias then LUT
//   EPI_RAW16   y = run (the separate epilogue kernel finishes it)
//   EPI_GATED   pieces 2t / 2t+1 are the gate / up sums of 32 hidden columns:
//               y[hb + i] = fp16(fp16(g * fp16(gate(g))) * u), g and u finished with their biases
template <int MODE, int N>
__device__ __forceinline__ void finish_tile(const Params &p, const __half2 (&run)[N], int row, bool row_ok, int col0,
                                            bool &bad, const CUtensorMap *tmap_y, uint32_t stage, int lane) {
    constexpr int PIECES = N / 16;
#pragma unroll 1
    for (int j = 0; j < PIECES; ++j) {
        if constexpr (MODE == EPI_GATED)
            if (!(j & 1)) continue;   // each gate piece is finished together with its up piece
        __half2 r[16];
        run_get(run, j, r);
        uint32_t pk[16];
        if constexpr (MODE == EPI_GATED) {
            __half2 g[16], bg[16], bu[16];
            run_get(run, j - 1, g);
            const int hb = (col0 + 32 * (j - 1)) >> 1;
            load_bias_pairs(p.bias, hb, p.gate_n, bg);
            load_bias_pairs(p.bias2, hb, p.gate_n, bu);
            if (p.bias) {
                if (p.bias2) gated_piece<true, true>(g, r, bg, bu, p.gate_table, p.gate, pk, bad);
                else gated_piece<true, false>(g, r, bg, bu, p.gate_table, p.gate, pk, bad);
            } else {
                if (p.bias2) gated_piece<false, true>(g, r, bg, bu, p.gate_table, p.gate, pk, bad);
                else gated_piece<false, false>(g, r, bg, bu, p.gate_table, p.gate, pk, bad);
            }
            store_out(p, tmap_y, stage, lane, row, row_ok, hb, p.gate_n, pk);
        } else {
            const int cb = col0 + 32 * j;
            if constexpr (MODE == EPI_TILE16) {
                __half2 b[16];
                if (p.bias) {
                    load_bias_pairs(p.bias, cb, p.N, b);
                    if (p.post) finish_piece16<true, true>(r, b, pk, bad);
                    else finish_piece16<true, false>(r, b, pk, bad);
                } else {
                    if (p.post) finish_piece16<false, true>(r, b, pk, bad);
                    else finish_piece16<false, false>(r, b, pk, bad);
                }
                if (p.res != nullptr && row_ok) add_residual32(p, row, cb, pk, bad);
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) pk[i] = *reinterpret_cast<const uint32_t *>(&r[i]);
            }
            store_out(p, tmap_y, stage, lane, row, row_ok, cb, p.N, pk);
        }
    }
}

// Epilogue warps: drain the TMEM accumulator of each finished tile (or 256-K chunk) in four
// 32-column pieces, hand the accumulator back after the last piece is in registers, finish and
// store. The loops stay rolled so the code of the persistent kernel fits the instruction cache.
template <int CG, int TN, int MODE>
__device__ __forceinline__ void epilogue_role(const Params &p, int warp, int lane, uint32_t rank, int cluster_id,
                                              int num_clusters, int nchunks, uint32_t tmem_base, uint32_t tfull0,
                                              uint32_t tempty0, volatile int *abort_flag,
                                              const CUtensorMap *tmap_y, uint32_t stage) {
    using C = Cfg<CG, TN>;
    constexpr int HALF = TN / 2, PIECES = HALF / 32;
    const int quarter = warp & 3;          // TMEM lanes [32*quarter, 32*quarter + 32)
    const int half = (warp - 4) >> 2;      // columns [HALF*half, HALF*half + HALF) of the tile
    const uint32_t tempty_leader = CG == 2 ? map_to_rank(tempty0, 0) : tempty0;
    uint32_t acc_used = 0;
    bool ok = true, bad = false;
    __half2 run[HALF / 2];                 // per-256-K FP16 running sum (tile-16 modes)
    // routed raw output: the parity plane of this round (the signal step increments the counter)
    unsigned route_par = 0;
    if constexpr (MODE == EPI_RAW32)
        if (p.route_rows > 0) route_par = (*reinterpret_cast<const volatile unsigned *>(p.route_seq) + 1u) & 1u;
    for (int tile = cluster_id; ok && tile < p.num_tiles; tile += num_clusters) {
        int mb, nb;
        tile_coords(tile, p, mb, nb);
        const int row = mb * C::BM + (int)rank * 128 + quarter * 32 + lane;
        const bool row_ok = row < p.M;
        const int col0 = nb * TN + half * HALF;
        for (int c = 0; c < nchunks; ++c) {
            const uint32_t acc = acc_used & 1u, acc_ph = (acc_used >> 1) & 1u;
            int got = 1;
            if (lane == 0) got = wait_phase(tfull0 + 8 * acc, acc_ph, abort_flag, p.flags);
            got = __shfl_sync(0xffffffffu, got, 0);       // the warp stays converged
            if (!got) { ok = false; break; }
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * TN + half * HALF;
            const bool first = c == 0, last = c == nchunks - 1;
            if constexpr (MODE == EPI_TILE16 || MODE == EPI_RAW16 || MODE == EPI_GATED) {
                // Every 256-K chunk, the last included, is folded into `run` and its accumulator handed
                // back at once; the tile's finish then runs from registers while the MMA warp already
                // works on the next tile (with two accumulators it needs this one back within a chunk).
                fold_chunk<HALF>(run, taddr, first, [&] { release_acc<CG>(lane, tempty_leader, tempty0, acc); });
                if (last) finish_tile<MODE>(p, run, row, row_ok, col0, bad, tmap_y, stage, lane);
            } else {
#pragma unroll 1
            for (int j = 0; j < PIECES; ++j) {
                float v[32];
                tmem_ld32(taddr + j * 32, v);
                if (j == PIECES - 1) release_acc<CG>(lane, tempty_leader, tempty0, acc);   // drained into registers
                const int cb = col0 + 32 * j;
                if constexpr (MODE == EPI_RAW32) {
                    if (p.route_rows > 0) {
                        // Routed: the owner's slot is stored in 32-row panels, column by column
                        // ((r / 32) * 32 * ldp + c * 32 + r % 32), so each store instruction of the
                        // warp (32 consecutive rows of one column) is one 128-byte line over NVLink.
                        // route_rows is a multiple of 32: a warp's rows share one owner and panel.
                        if (row_ok) {
                            const int q = row / p.route_rows;
                            float *base = p.route_dst[0];
#pragma unroll
                            for (int i = 1; i < ROUTE_MAX; ++i)
                                if (i == q) base = p.route_dst[i];
                            const int r = row - q * p.route_rows;
                            float *dst = base + (size_t)route_par * p.route_plane + (size_t)(r >> 5) * 32 * p.ldp +
                                         (size_t)cb * 32 + (r & 31);
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                if (cb + i < p.N) dst[(size_t)i * 32] = v[i];
                        }
                    } else if (row_ok) {
                        store32f(p.partial + (size_t)row * p.ldp, cb, p.N, p.vec_p, v);
                    }
                } else {
                    float b[32];
                    load_bias32(p.bias, cb, p.N, b);
                    uint32_t pk[16];
                    if (p.post) finish_piece32<true>(v, b, pk, bad);
                    else finish_piece32<false>(v, b, pk, bad);
                    if (p.res != nullptr && row_ok) add_residual32(p, row, cb, pk, bad);
                    store_out(p, tmap_y, stage, lane, row, row_ok, cb, p.N, pk);
                }
            }
            }
            ++acc_used;
        }
    }
    if (p.tma_y && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");   // stores done
    if constexpr (MODE == EPI_RAW32)
        if (p.route_rows > 0) __threadfence_system();   // peer stores before the round's signal
    if (__any_sync(0xffffffffu, bad) && lane == 0) raise_flag(p.flags, FLAG_NONFINITE_OUTPUT);
}

// ----------------------------------------------------------------------------- the kernel
template <int CG, int TN, int MODE>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                const __grid_constant__ CUtensorMap tmap_y, const Params p) {
    using C = Cfg<CG, TN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~static_cast<uintptr_t>(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + C::STAGES * C::A_BYTES;
    uint8_t *sOut = smem + C::STAGES * C::STAGE_BYTES;   // 1024-byte aligned
    uint64_t *bars = reinterpret_cast<uint64_t *>(sOut + C::OUT_BYTES);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + C::NUM_BARS);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = CG == 2 ? cluster_rank() : 0;   // 0 = leader (issues the MMAs)
    const int cluster_id = (int)blockIdx.x / CG, num_clusters = (int)gridDim.x / CG;
    const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * C::STAGES;
    const uint32_t tfull0 = empty0 + 8 * C::STAGES, tempty0 = tfull0 + 16, drain_bar = tempty0 + 16;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull0 + 8 * a, 1);
            mbar_init(tempty0 + 8 * a, EPI_WARPS * CG);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (!p.a_maps) prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
        if (p.tma_y) prefetch_tmap(&tmap_y);
    }
    if (warp == 2) {
        tmem_alloc<CG>(smem_u32(tmem_slot), C::TMEM_COLS);
        tmem_relinquish<CG>();
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (CG == 2) cluster_sync();   // peer barriers initialised before any remote use
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int nchunks = (p.num_kb + p.kb_per_chunk - 1) / p.kb_per_chunk;

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------------------------ TMA producer
            uint32_t issued = 0;
            bool ok = true;
            const CUtensorMap *a_map_seen = nullptr;
            int a_oct = 0;
            for (int tile = cluster_id; ok && tile < p.num_tiles; tile += num_clusters) {
                int mb, nb;
                tile_coords(tile, p, mb, nb);
                const int row_a = mb * C::BM + (int)rank * 128, row_b = nb * TN + (int)rank * C::B_ROWS;
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    const uint32_t s = issued % C::STAGES, ph = (issued / C::STAGES) & 1u;
                    if (!wait_phase(empty0 + 8 * s, ph ^ 1u, abort_flag, p.flags)) { ok = false; break; }
                    uint32_t full_bar = full0 + 8 * s;
                    if constexpr (CG == 2) full_bar = map_to_rank(full_bar, 0);
                    if (rank == 0) mbar_arrive_expect_tx(full0 + 8 * s, C::STAGE_BYTES * CG);
                    if (p.a_maps) {
                        // X from the caller's cube view of this row band and K range (box rows past the
                        // view's rows and channel groups past its K arrive as zeros)
                        const int k = kb * BK;
                        const size_t view = (size_t)(row_a >> 8) * p.a_kviews + k / p.a_kview_k;
                        const CUtensorMap *am = p.a_maps + view;
                        if (am != a_map_seen) {
                            tmap_acquire(am);
                            a_map_seen = am;
                            a_oct = p.a_octets[view];
                        }
                        tma_load_3d<CG>(smem_u32(sA + s * C::A_BYTES), am, full_bar, 0,
                                        a_oct ? (row_a & 255) >> 3 : row_a & 255, (k % p.a_kview_k) / 8);
                    } else {
                        tma_load_2d<CG>(smem_u32(sA + s * C::A_BYTES), &tmap_a, full_bar, kb * BK, row_a);
                    }
                    tma_load_2d<CG>(smem_u32(sB + s * C::B_BYTES), &tmap_b, full_bar, kb * BK, row_b);
                    ++issued;
                }
            }
            if (!ok && rank == 0) {
                // Loads in flight land in the last STAGES slots; wait for each before exiting.
                const uint32_t first = issued > (uint32_t)C::STAGES ? issued - C::STAGES : 0;
                for (uint32_t i = first; i < issued; ++i)
                    drain_phase(full0 + 8 * (i % C::STAGES), (i / C::STAGES) & 1u);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // ------------------------------------------------------------------ MMA issuer
            uint32_t consumed = 0, acc_used = 0;
            bool ok = true;
            const bool cube_a = p.a_maps != nullptr;
            for (int tile = cluster_id; ok && tile < p.num_tiles; tile += num_clusters) {
                for (int c = 0; ok && c < nchunks; ++c) {
                    const uint32_t acc = acc_used & 1u, acc_ph = (acc_used >> 1) & 1u;
                    if (!wait_phase(tempty0 + 8 * acc, acc_ph ^ 1u, abort_flag, p.flags)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + acc * TN;
                    const int kb0 = c * p.kb_per_chunk;
                    const int kb1 = min(kb0 + p.kb_per_chunk, p.num_kb);
                    for (int kb = kb0; kb < kb1; ++kb) {
                        const uint32_t s = consumed % C::STAGES, ph = (consumed / C::STAGES) & 1u;
                        if (!wait_phase(full0 + 8 * s, ph, abort_flag, p.flags)) { ok = false; break; }
                        tc_fence_after();
                        const uint64_t adesc = cube_a ? cube_desc(smem_u32(sA + s * C::A_BYTES))
                                                      : sw128_desc(smem_u32(sA + s * C::A_BYTES));
                        const uint64_t bdesc = sw128_desc(smem_u32(sB + s * C::B_BYTES));
                        const uint32_t astep = cube_a ? CUBE_K16_STEP : 2u;
#pragma unroll
                        for (int k = 0; k < BK / 16; ++k)   // swizzled: +32 bytes along K = +2 in the desc
                            umma_f16<CG>(d_tmem, adesc + astep * k, bdesc + 2 * k, C::IDESC,
                                         (kb > kb0 || k > 0) ? 1u : 0u);
                        umma_commit<CG>(empty0 + 8 * s);
                        ++consumed;
                    }
                    if (!ok) break;
                    umma_commit<CG>(tfull0 + 8 * acc);
                    ++acc_used;
                }
            }
            // All MMAs issued by this thread complete before TMEM can be released (a commit is only
            // issued when this thread issued MMAs before it).
            if (consumed) {
                umma_commit_local<CG>(drain_bar);
                drain_phase(drain_bar, 0);
            }
        }
    } else if (warp >= 4) {
        epilogue_role<CG, TN, MODE>(p, warp, lane, rank, cluster_id, num_clusters, nchunks, tmem_base, tfull0,
                                tempty0, abort_flag, &tmap_y, smem_u32(sOut + (warp - 4) * 2048));
    }

    tc_fence_before();
    __syncthreads();
    if constexpr (CG == 2) cluster_sync();   // the leader's MMAs into this CTA's TMEM are done
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc<CG>(tmem_base, C::TMEM_COLS);
    }
}

// ----------------------------------------------------------------------------- host launcher
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    }
    return fn;
}

// 2-D FP16 tensor map over a row-major [rows, ld] matrix of which `inner` columns are valid.
// Columns >= inner and rows >= rows are outside the tensor: TMA fills them with zeros.
static bool make_map(CUtensorMap *map, const void *ptr, uint64_t inner, uint64_t rows, uint64_t ld,
                     uint32_t box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(ptr), dims, strides, box,
               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


bool make_cube_map(CUtensorMap *map, const void *ptr, unsigned rows, unsigned prow, unsigned cols, int *octets) {
    EncodeTiledFn enc = encode_fn();
    if (!enc || !rows || prow < rows || !cols || cols % 8 || (reinterpret_cast<uintptr_t>(ptr) & 15)) return false;
    const bool oct = rows % 8 == 0;
    cuuint64_t dims[3] = {oct ? 64u : 8u, oct ? rows / 8 : rows, cols / 8};
    cuuint64_t strides[2] = {oct ? 128u : 16u, (cuuint64_t)prow * 16};
    cuuint32_t box[3] = {oct ? 64u : 8u, oct ? 16u : 128u, 8};
    cuuint32_t estr[3] = {1, 1, 1};
    *octets = oct ? 1 : 0;
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int CG, int TN, int MODE>
static cudaError_t set_smem_attr() {
    return cudaFuncSetAttribute(gemm_kernel<CG, TN, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)Cfg<CG, TN>::SMEM_BYTES);
}

static cudaLaunchConfig_t cluster_config(int cg, unsigned grid, uint32_t smem, cudaStream_t stream,
                                         cudaLaunchAttribute *attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cg;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

// Co-resident clusters of a variant on the current device (2-SM clusters must fit inside a GPC,
// so this can be below sm_count / 2); queried once per device and variant.
template <int CG, int TN>
static int resident_clusters(int sm_count) {
    static int cached[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return sm_count / CG;
    if (cached[dev]) return cached[dev];
    int n = 0;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = cluster_config(CG, (unsigned)(sm_count / CG * CG), Cfg<CG, TN>::SMEM_BYTES, 0, attr);
    if (set_smem_attr<CG, TN, EPI_FP32>() != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&n, gemm_kernel<CG, TN, EPI_FP32>, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = sm_count / CG;
    }
    if (n > sm_count / CG) n = sm_count / CG;
    cached[dev] = n;
    return n;
}

static int clusters_for(int cg, int sm_count) {
    return cg == 2 ? resident_clusters<2, TILE_N>(sm_count) : resident_clusters<1, TILE_N>(sm_count);
}

// Column width of a 1-SM launch's tiles. TILE_N = 256 wherever the 256-wide tiles fill the GPU:
// narrower tiles need more operand traffic per FLOP and measured 0.55-0.65x the throughput there.
// A launch whose 256-wide tiles occupy at most a quarter (half) of the SMs takes 64- (128-) wide
// tiles instead: each CTA then stages a quarter (half) of the W rows and finishes a quarter (half)
// of the columns, so a latency-bound launch (M = 64, N = 256: one CTA) spreads over more SMs. The
// per-element arithmetic does not depend on the tile width. The gated epilogue pairs 32-column
// pieces inside a tile and keeps 256; cube operands and routed stores keep 256 as well.
static int choose_tn(int cg, int M, int N, int sm_count, const Params *p) {
    if (cg != 1 || (p && (p->gate || p->a_maps || p->y_cube || p->route_rows))) return TILE_N;
    const long long tiles = (long long)((M + 127) / 128) * ((N + TILE_N - 1) / TILE_N);
    if (4 * tiles <= sm_count) return 64;
    if (2 * tiles <= sm_count) return 128;
    return TILE_N;
}

// Picks the CTA group with fewer persistent waves of 256-wide tiles, preferring the 2-SM pair (less
// shared-memory traffic per FLOP); 2-SM tiles need M > 128. A launch whose 1-SM 256-wide tiles fill
// at most half of the SMs runs narrow 1-SM tiles instead (choose_tn): two or four times the CTAs of
// the 1-SM form, each with a half or a quarter of the MMA work (measured against the pair: 512 x 4096
// x 4096 tile-16 41.3 -> 34.9 us, 1000 x 1000 x 4096 41.0 -> 31.1 us, outputs bit-identical).
static int choose_cg(int M, int N, int sm_count) {
    if (M <= 128) return 1;
    if (2 * (long long)((M + 127) / 128) * ((N + TILE_N - 1) / TILE_N) <= sm_count) return 1;
    long long waves[3];
    for (int cg = 1; cg <= 2; ++cg) {
        const long long tiles = (long long)((M + 128 * cg - 1) / (128 * cg)) * ((N + TILE_N - 1) / TILE_N);
        const long long clusters = clusters_for(cg, sm_count);
        waves[cg] = (tiles + clusters - 1) / clusters;
    }
    return waves[1] < waves[2] ? 1 : 2;
}

static unsigned grid_for_tile(int cg, int tn, int M, int N, int sm_count) {
    const long long tiles = (long long)((M + 128 * cg - 1) / (128 * cg)) * ((N + tn - 1) / tn);
    const long long clusters = clusters_for(cg, sm_count);
    return (unsigned)((tiles < clusters ? tiles : clusters) * cg);
}

unsigned grid_for_variant(int cg, int M, int N, int sm_count) {
    return grid_for_tile(cg, choose_tn(cg, M, N, sm_count, nullptr), M, N, sm_count);
}

unsigned grid_for(int M, int N, int sm_count) {
    return grid_for_variant(choose_cg(M, N, sm_count), M, N, sm_count);
}

void config_for(int M, int N, int sm_count, unsigned *tile_m, unsigned *tile_n, unsigned *stages) {
    const int cg = choose_cg(M, N, sm_count);
    const int tn = choose_tn(cg, M, N, sm_count, nullptr);
    *tile_m = 128u * cg;
    *tile_n = (unsigned)tn;
    *stages = cg == 2 ? Cfg<2, TILE_N>::STAGES
                      : (tn == 64 ? Cfg<1, 64>::STAGES : tn == 128 ? Cfg<1, 128>::STAGES : Cfg<1, TILE_N>::STAGES);
}

template <int CG, int TN, int MODE>
static cudaError_t ensure_attr(int device) {
    static bool attr_done[64];
    if (!attr_done[device]) {
        const cudaError_t e = set_smem_attr<CG, TN, MODE>();
        if (e != cudaSuccess) return e;
        attr_done[device] = true;
    }
    return cudaSuccess;
}

// The shared-memory opt-in of every kernel a variant launches (narrow tiles have no gated form).
template <int CG, int TN>
static cudaError_t prepare_variant(int device, int sm_count) {
    resident_clusters<CG, TN>(sm_count);
    cudaError_t e = cudaSuccess;
    for (cudaError_t r : {ensure_attr<CG, TN, EPI_FP32>(device), ensure_attr<CG, TN, EPI_TILE16>(device),
                          ensure_attr<CG, TN, EPI_RAW16>(device), ensure_attr<CG, TN, EPI_RAW32>(device)})
        if (r != cudaSuccess) e = r;
    if constexpr (TN == TILE_N)
        if (ensure_attr<CG, TN, EPI_GATED>(device) != cudaSuccess) e = cudaErrorInvalidValue;
    return e;
}

cudaError_t prepare(int device, int sm_count) {
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    if (!encode_fn()) return cudaErrorNotSupported;
    cudaError_t e = cudaSuccess;
    for (cudaError_t r : {prepare_variant<1, TILE_N>(device, sm_count), prepare_variant<2, TILE_N>(device, sm_count),
                          prepare_variant<1, 64>(device, sm_count), prepare_variant<1, 128>(device, sm_count)})
        if (r != cudaSuccess && e == cudaSuccess) e = r;
    return e;
}

// Output tensor map of the TMA tile stores: FP16 [rows, ld] of which `cols` are valid, 32 x 32 boxes,
// 64-byte swizzle (the layout store_out writes into the staging box).
static bool make_store_map(CUtensorMap *map, const void *ptr, uint64_t cols, uint64_t rows, uint64_t ld) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int CG, int TN, int MODE>
static cudaError_t launch_mode(const CUtensorMap &ta, const CUtensorMap &tb, Params p, unsigned grid,
                               cudaStream_t stream, int device) {
    const cudaError_t e = ensure_attr<CG, TN, MODE>(device);
    if (e != cudaSuccess) return e;
    // FP16 outputs leave through TMA tile stores when Y allows a tensor map (16-byte aligned base and
    // pitch, at least one 32 x 32 box) whose row ends on a 16-byte boundary: a box crossing a ragged
    // row end was seen to write the rest of that row's last 16 bytes, i.e. into the pitch padding.
    // Otherwise each epilogue thread stores its row directly, clipped at the last column.
    CUtensorMap ty;
    memset(&ty, 0, sizeof(ty));
    const uint64_t n_out = MODE == EPI_GATED ? (uint64_t)p.gate_n : (uint64_t)p.N;
    p.tma_y = 0;
    if constexpr (MODE != EPI_RAW32)
        if (p.vec_y && n_out % 8 == 0 && n_out >= 32 && p.M >= 32 &&
            make_store_map(&ty, p.y, n_out, (uint64_t)p.M, (uint64_t)p.ldy))
            p.tma_y = 1;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = cluster_config(CG, grid, Cfg<CG, TN>::SMEM_BYTES, stream, attr);
    return cudaLaunchKernelEx(&cfg, gemm_kernel<CG, TN, MODE>, ta, tb, ty, p);
}

template <int CG, int TN>
static cudaError_t launch_tile(const Shape &s, Params p, cudaStream_t stream, int device, int sm_count,
                               unsigned *grid_out) {
    using C = Cfg<CG, TN>;
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    CUtensorMap ta, tb;
    memset(&ta, 0, sizeof(ta));   // unused when X comes from cube views (p.a_maps)
    if ((!p.a_maps && !make_map(&ta, s.x, (uint64_t)p.K, (uint64_t)p.M, s.ldx, 128)) ||
        !make_map(&tb, s.w, (uint64_t)p.K, (uint64_t)p.N, s.ldw, C::B_ROWS))
        return cudaErrorInvalidValue;
    if ((p.a_maps || p.y_cube) && (p.out_mode != OUT_FINAL || p.gate || p.res || p.route_rows ||
                                   (p.a_maps && (p.a_kviews < 1 || p.a_kview_k < BK || p.a_kview_k % BK))))
        return cudaErrorInvalidValue;
    p.num_m_blocks = (p.M + C::BM - 1) / C::BM;
    p.num_n_blocks = (p.N + TN - 1) / TN;
    p.num_tiles = p.num_m_blocks * p.num_n_blocks;
    p.num_kb = (p.K + BK - 1) / BK;
    p.kb_per_chunk = p.fold ? 256 / BK : p.num_kb;
    // Bands of 8 m-blocks keep a wave's X and W blocks L2-resident once X outgrows the L2.
    p.group_m = (p.num_m_blocks >= 16 && p.num_n_blocks >= 16 && (long long)p.M * p.K >= (64ll << 20)) ? 8 : 0;
    const unsigned grid = grid_for_tile(CG, TN, p.M, p.N, sm_count);
    if (grid_out) *grid_out = grid;
    if (p.out_mode == OUT_RAW32) return launch_mode<CG, TN, EPI_RAW32>(ta, tb, p, grid, stream, device);
    if (p.out_mode == OUT_RAW16) return launch_mode<CG, TN, EPI_RAW16>(ta, tb, p, grid, stream, device);
    if (p.gate) {
        if constexpr (TN != TILE_N) return cudaErrorInvalidValue;   // 32-column pairs need the 256-wide tile
        else {
            if (!p.fold || p.res || p.post || p.N != 2 * ((p.gate_n + 31) / 32 * 32)) return cudaErrorInvalidValue;
            return launch_mode<CG, TN, EPI_GATED>(ta, tb, p, grid, stream, device);
        }
    }
    if (p.fold) return launch_mode<CG, TN, EPI_TILE16>(ta, tb, p, grid, stream, device);
    return launch_mode<CG, TN, EPI_FP32>(ta, tb, p, grid, stream, device);
}

cudaError_t launch_variant(int cg, const Shape &s, const Params &p, cudaStream_t stream, int device,
                           int sm_count, unsigned *grid_out) {
    if (cg == 2) return launch_tile<2, TILE_N>(s, p, stream, device, sm_count, grid_out);
    if (cg != 1) return cudaErrorInvalidValue;
    const int tn = choose_tn(1, p.M, p.N, sm_count, &p);
    if (tn == 64) return launch_tile<1, 64>(s, p, stream, device, sm_count, grid_out);
    if (tn == 128) return launch_tile<1, 128>(s, p, stream, device, sm_count, grid_out);
    return launch_tile<1, TILE_N>(s, p, stream, device, sm_count, grid_out);
}

cudaError_t launch(const Shape &s, Params p, cudaStream_t stream, int device, int sm_count,
                   unsigned *grid_out) {
    return launch_variant(choose_cg(p.M, p.N, sm_count), s, p, stream, device, sm_count, grid_out);
}

}  // namespace gemm
}  // namespace b2
