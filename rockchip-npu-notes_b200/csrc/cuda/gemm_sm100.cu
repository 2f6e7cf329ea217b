// gemm_sm100.cu -- persistent tcgen05 GEMM with the fused bias / HardSigmoid epilogue (sm_100a).
//
// Computes Y[M,N] = act(X[M,K] * W[N,K]^T + b[N]) in FP16 with FP32 accumulation in TMEM.
// It replaces the reference's per-output-tile NPU task chain
//   MM (first K tile) -> MM_ACC (each further K tile, FP16 ping-pong accumulators)
//   -> EW (bias) -> LUT (HardSigmoid)        research/custom-ops/src/linear_hardsigmoid.c:51-82
// with one launch:
//   warp 0      TMA producer: 128x64 X and 256x64 W tiles (128-byte swizzle) into a 4-stage
//               shared-memory ring, mbarrier transaction counts
//   warp 1      MMA issuer (one thread): tcgen05.mma kind::f16, M=128 N=256 K=16 per instruction,
//               accumulating into one of two 256-column TMEM buffers; tcgen05.commit frees ring
//               stages and publishes finished accumulators
//   warp 2      TMEM allocator (512 columns)
//   warps 4-11  epilogue: tcgen05.ld of their 32-lane quarter and 128-column half, then either
//                 - FP32 mode: y = fp16(act(acc + b)), or
//                 - tile-16 mode (the reference's FP16-K-TILING numerics): the MMA warp closes an
//                   accumulator every 256 K, the epilogue folds run = fp16(run + chunk) in
//                   registers and finishes with affine = fp16(run + b), y = fp16(hsig(affine));
//               results are written with 16-byte stores.
// Tiles are scheduled persistently: CTA i takes output tiles i, i+grid, ... so the TMA/MMA of the
// next tile overlaps the epilogue of the previous one (two TMEM accumulators).
//
// Every mbarrier wait is bounded (globaltimer): on expiry the CTA raises the timeout flag, stops
// issuing work, waits (bounded) for its own TMA loads and MMAs in flight, frees TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"
#include "gemm_sm100.h"

namespace b2 {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 128 + EPI_WARPS * 32;
constexpr uint32_t A_BYTES = BM * BK * 2;
constexpr uint32_t B_BYTES = BN * BK * 2;
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr int NUM_BARS = 2 * STAGES + 2 + 2 + 1;
constexpr uint32_t SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + NUM_BARS * 8 + 16;
constexpr uint64_t WAIT_LIMIT_NS = 1000000000ull;   // 1 s per wait; a healthy wait is microseconds

// Instruction descriptor, kind::f16: D=F32 (bits 4-5 = 1), A=B=F16 (0), both K-major,
// N>>3 at bits 17-22, M>>4 at bits 24-28.
constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

// ----------------------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits for the phase of parity `parity` to complete. Returns false when the CTA is aborting or
// the wait exceeded WAIT_LIMIT_NS (then the timeout flag is raised and the CTA aborts).
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                           unsigned *flags) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_ns() - t0 > WAIT_LIMIT_NS) {
            *abort_flag = 1;
            raise_flag(flags, FLAG_TIMEOUT);
            return false;
        }
    }
}
// Bounded wait used only while draining after an abort (ignores the abort flag).
__device__ __forceinline__ void drain_phase(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity))
        if (global_ns() - t0 > WAIT_LIMIT_NS) return;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar,
                                            int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
        : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
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

__device__ __forceinline__ float load_bias(const __half *bias, int col, int n) {
    return (bias && col < n) ? __half2float(bias[col]) : 0.0f;
}

// ----------------------------------------------------------------------------- the kernel
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~static_cast<uintptr_t>(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * A_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + NUM_BARS);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * STAGES;
    const uint32_t tfull0 = empty0 + 8 * STAGES, tempty0 = tfull0 + 16, drain_bar = tempty0 + 16;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull0 + 8 * a, 1);
            mbar_init(tempty0 + 8 * a, EPI_WARPS);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
    }
    if (warp == 2) {
        tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int nchunks = (p.num_kb + p.kb_per_chunk - 1) / p.kb_per_chunk;

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------------------------ TMA producer
            uint32_t issued = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
                const int mb = tile % p.num_m_blocks, nb = tile / p.num_m_blocks;
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    const uint32_t s = issued % STAGES, ph = (issued / STAGES) & 1u;
                    if (!wait_phase(empty0 + 8 * s, ph ^ 1u, abort_flag, p.flags)) { ok = false; break; }
                    mbar_arrive_expect_tx(full0 + 8 * s, STAGE_BYTES);
                    tma_load_2d(smem_u32(sA + s * A_BYTES), &tmap_a, full0 + 8 * s, kb * BK, mb * BM);
                    tma_load_2d(smem_u32(sB + s * B_BYTES), &tmap_b, full0 + 8 * s, kb * BK, nb * BN);
                    ++issued;
                }
            }
            if (!ok) {
                // Loads in flight land in the last STAGES slots; wait for each before exiting.
                const uint32_t first = issued > STAGES ? issued - STAGES : 0;
                for (uint32_t i = first; i < issued; ++i)
                    drain_phase(full0 + 8 * (i % STAGES), (i / STAGES) & 1u);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------------------------------------------ MMA issuer
            uint32_t consumed = 0, acc_used = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
                for (int c = 0; ok && c < nchunks; ++c) {
                    const uint32_t acc = acc_used & 1u, acc_ph = (acc_used >> 1) & 1u;
                    if (!wait_phase(tempty0 + 8 * acc, acc_ph ^ 1u, abort_flag, p.flags)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + acc * BN;
                    const int kb0 = c * p.kb_per_chunk;
                    const int kb1 = min(kb0 + p.kb_per_chunk, p.num_kb);
                    for (int kb = kb0; kb < kb1; ++kb) {
                        const uint32_t s = consumed % STAGES, ph = (consumed / STAGES) & 1u;
                        if (!wait_phase(full0 + 8 * s, ph, abort_flag, p.flags)) { ok = false; break; }
                        tc_fence_after();
                        const uint64_t adesc = sw128_desc(smem_u32(sA + s * A_BYTES));
                        const uint64_t bdesc = sw128_desc(smem_u32(sB + s * B_BYTES));
#pragma unroll
                        for (int k = 0; k < BK / 16; ++k)   // +32 bytes along K = +2 in the desc
                            umma_f16(d_tmem, adesc + 2 * k, bdesc + 2 * k, (kb > kb0 || k > 0) ? 1u : 0u);
                        umma_commit(empty0 + 8 * s);
                        ++consumed;
                    }
                    if (!ok) break;
                    umma_commit(tfull0 + 8 * acc);
                    ++acc_used;
                }
            }
            // All MMAs issued by this thread complete before TMEM can be released.
            umma_commit(drain_bar);
            drain_phase(drain_bar, 0);
        }
    } else if (warp >= 4) {
        // ---------------------------------------------------------------------- epilogue
        const int quarter = warp & 3;          // TMEM lanes [32*quarter, 32*quarter + 32)
        const int half = (warp - 4) >> 2;      // columns [128*half, 128*half + 128) of the tile
        const bool has_bias = p.bias != nullptr;
        uint32_t acc_used = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
            const int mb = tile % p.num_m_blocks, nb = tile / p.num_m_blocks;
            const int row = mb * BM + quarter * 32 + lane;
            const int col0 = nb * BN + half * 128;
            __half2 out[64];      // 128 columns as FP16 pairs: the running sum, then the result
#pragma unroll
            for (int i = 0; i < 64; ++i) out[i] = __floats2half2_rn(0.0f, 0.0f);
            for (int c = 0; c < nchunks; ++c) {
                const uint32_t acc = acc_used & 1u, acc_ph = (acc_used >> 1) & 1u;
                if (!wait_phase(tfull0 + 8 * acc, acc_ph, abort_flag, p.flags)) { ok = false; break; }
                __syncwarp();
                tc_fence_after();
                const uint32_t taddr =
                    tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN + half * 128;
                const bool first = c == 0, last = c == nchunks - 1;
                if (p.out_mode == OUT_RAW32) {
                    // Raw FP32 accumulator straight from TMEM (K-split partials).
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        float v[32];
                        tmem_ld32(taddr + j * 32, v);
                        if (row < p.M) {
                            float *dst = p.partial + (size_t)row * p.ldp;
#pragma unroll
                            for (int g = 0; g < 8; ++g) {
                                const int col = col0 + j * 32 + g * 4;
                                if (p.vec_p && col + 4 <= p.N) {
                                    *reinterpret_cast<float4 *>(dst + col) =
                                        make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
                                } else {
#pragma unroll
                                    for (int e = 0; e < 4; ++e)
                                        if (col + e < p.N) dst[col + e] = v[4 * g + e];
                                }
                            }
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        float v[32];
                        tmem_ld32(taddr + j * 32, v);
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            float a0 = v[2 * i], a1 = v[2 * i + 1];
                            if (p.fold) {
                                const float2 r = __half22float2(out[j * 16 + i]);
                                a0 = fold16(r.x, a0, first);
                                a1 = fold16(r.y, a1, first);
                            } else if (p.out_mode == OUT_FINAL) {
                                // FP32 mode (a single chunk): finish from the exact accumulator.
                                const int col = col0 + j * 32 + 2 * i;
                                a0 = finish_fp32(a0, load_bias(p.bias, col, p.N), p.post);
                                a1 = finish_fp32(a1, load_bias(p.bias, col + 1, p.N), p.post);
                            }
                            out[j * 16 + i] = __floats2half2_rn(a0, a1);
                        }
                    }
                }
                // Accumulator drained into registers: hand it back to the MMA warp.
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(tempty0 + 8 * acc);
                ++acc_used;
                if (!last || p.out_mode == OUT_RAW32) continue;

                // ------------------------------------------------ finish and store 128 columns
                if (p.out_mode == OUT_FINAL) {
                    bool bad = false;
#pragma unroll
                    for (int i = 0; i < 64; ++i) {
                        if (p.fold) {   // tile-16 mode: bias and activation after the last fold
                            const int col = col0 + 2 * i;
                            const float2 a = __half22float2(out[i]);
                            out[i] = __floats2half2_rn(
                                finish_tile16(a.x, load_bias(p.bias, col, p.N), has_bias, p.post),
                                finish_tile16(a.y, load_bias(p.bias, col + 1, p.N), has_bias, p.post));
                        }
                        bad |= half_nonfinite(__low2half(out[i])) | half_nonfinite(__high2half(out[i]));
                    }
                    if (__any_sync(0xffffffffu, bad) && lane == 0) raise_flag(p.flags, FLAG_NONFINITE_OUTPUT);
                }
                if (row < p.M) {
                    __half *dst = p.y + (size_t)row * p.ldy;
#pragma unroll
                    for (int g = 0; g < 16; ++g) {
                        const int col = col0 + 8 * g;
                        if (p.vec_y && col + 8 <= p.N) {
                            uint4 v;
                            v.x = *reinterpret_cast<const uint32_t *>(&out[4 * g]);
                            v.y = *reinterpret_cast<const uint32_t *>(&out[4 * g + 1]);
                            v.z = *reinterpret_cast<const uint32_t *>(&out[4 * g + 2]);
                            v.w = *reinterpret_cast<const uint32_t *>(&out[4 * g + 3]);
                            *reinterpret_cast<uint4 *>(dst + col) = v;
                        } else {
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                if (col + 2 * e < p.N) dst[col + 2 * e] = __low2half(out[4 * g + e]);
                                if (col + 2 * e + 1 < p.N) dst[col + 2 * e + 1] = __high2half(out[4 * g + e]);
                            }
                        }
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

}  // namespace gemm
}  // namespace b2

// ----------------------------------------------------------------------------- host launcher
namespace b2 {
namespace gemm {

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
    cuuint32_t box[2] = {(cuuint32_t)TILE_K, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(ptr), dims, strides, box,
               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

unsigned grid_for(int M, int N, int sm_count) {
    long long tiles = (long long)((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    return (unsigned)(tiles < sm_count ? tiles : sm_count);
}

cudaError_t launch(const Shape &s, Params p, cudaStream_t stream, int device, int sm_count,
                   unsigned *grid_out) {
    static bool attr_done[64];
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    if (!attr_done[device]) {
        cudaError_t e = cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)SMEM_BYTES);
        if (e != cudaSuccess) return e;
        attr_done[device] = true;
    }
    CUtensorMap ta, tb;
    if (!make_map(&ta, s.x, (uint64_t)p.K, (uint64_t)p.M, s.ldx, BM) ||
        !make_map(&tb, s.w, (uint64_t)p.K, (uint64_t)p.N, s.ldw, BN))
        return cudaErrorInvalidValue;
    p.num_m_blocks = (p.M + BM - 1) / BM;
    p.num_n_blocks = (p.N + BN - 1) / BN;
    p.num_tiles = p.num_m_blocks * p.num_n_blocks;
    p.num_kb = (p.K + BK - 1) / BK;
    p.kb_per_chunk = p.fold ? 256 / BK : p.num_kb;
    unsigned grid = grid_for(p.M, p.N, sm_count);
    if (grid_out) *grid_out = grid;
    gemm_kernel<<<grid, THREADS, SMEM_BYTES, stream>>>(ta, tb, p);
    return cudaGetLastError();
}

}  // namespace gemm
}  // namespace b2
