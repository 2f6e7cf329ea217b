// gemv.cu -- memory-bound small-M Linear (M <= 8): y[r, n] = act(x[r, :] . W[n, :] + b[n]).
//
// The reference runs M=1 decode through the same NPU matmul with the row count padded to 12
// (research/scheduling/GEMM-GEMV-CONCURRENCY.md:24-30 in the reference project) and produces a
// decoder layer's Q/K/V projections from one input in one graph call
// (research/custom-ops/src/co_decoder.c:128-129). On B200 the small-M case is a weight stream,
// served by two kernels with the same per-element arithmetic:
//
// Streamed kernel (M <= 8, K <= 16384; every decode projection of a small decoder):
//   persistent CTAs. Lanes of warp 0 each own one 16 KB shared-memory slot of a copy ring and keep
//   it filled; consumer warp s takes the units landing in slot s and computes them on the tensor
//   cores (below). The launch's x rows are copied once per CTA into a shared table (problems that
//   share an input share the entry), filled by the consumer warps while the first weights are in
//   flight. Configurations (SCfg):
//   * whole-row (K <= 2048): a unit is whole W rows -- rows [n0, n0 + R) of a row-major [N, ldw]
//     matrix are one contiguous byte range, one cp.async.bulk copy. 12 slots and a 32 KB x table
//     per SM; launches whose x rows fit 12 KB run as half-SM CTAs (6 slots, two CTAs per SM) under
//     programmatic dependent launch, so the next launch's CTAs stream their weights while this
//     launch runs or drains (see half_sm). A launch covers a group of up to GROUP_MAX independent
//     projections (same M): units of R rows from all of them are spread over the CTAs.
//   * sliced (2048 < K <= 16384): a unit is one 512-wide K slice of a 16-row block, one 3-D TMA
//     copy (eight 2-D boxes when K is not a multiple of 64); each CTA takes a contiguous range of
//     units and the blocks' per-256-K tile sums are folded in K order by the block's owner
//     (deliver_slice). 11 slots and a 32 KB x table, or 8 slots and a 64 KB table when the x rows
//     need it (wide_x).
// Per-lane-load kernel (the other M <= 8 shapes): each warp owns one W row at a time and every
//   lane reads 16 bytes per 256-element K tile with read-only, L1-bypassing loads; several tiles'
//   loads are issued before any arithmetic. The grid is the number of co-resident CTAs.
//
// Arithmetic: the per-lane-load kernel sums each lane's 8 products with fmaf in element order,
// accumulates over K tiles and reduces across the warp; the streamed kernel sums on the tensor
// cores (mma.sync m16n8k16, FP16 inputs, FP32 accumulation: W rows as A, up to 8 x rows as B, so a
// batch of 8 costs what one x row does). Both accumulate in FP32 (tile-16 mode: per 256-K tile,
// then the FP16 fold of the reference's FP16-K-TILING) and finish with the bias/activation of
// common.cuh; they agree with each other and the oracle within the operator's tolerance, and one
// x row's result never depends on the other rows of the batch.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "common.cuh"
#include "gemv.h"
#include "mbarrier.cuh"

namespace b2 {
namespace gemv {

namespace {

// ----------------------------------------------------------------------------- shared arithmetic
// Dot product of 8 FP16 weights with 8 x values (as FP32); elements at index >= valid contribute
// nothing.
__device__ __forceinline__ float dot8(uint4 w, const float (&xv)[8], int valid) {
    const __half2 *hw = reinterpret_cast<const __half2 *>(&w);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 fw = __half22float2(hw[i]);
        if (2 * i < valid) s = fmaf(fw.x, xv[2 * i], s);
        if (2 * i + 1 < valid) s = fmaf(fw.y, xv[2 * i + 1], s);
    }
    return s;
}

__device__ __forceinline__ void widen8(uint4 v, float (&out)[8]) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        out[2 * i] = f.x;
        out[2 * i + 1] = f.y;
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Lane r writes output row r of column n. Returns true if a final FP16 output is not finite.
template <int MR>
__device__ __forceinline__ bool finish_row(int M, int lane, int n, int out_mode, int fold, int post,
                                           const __half *bias, __half *y, long long ldy, float *partial,
                                           long long ldp, const float (&acc)[MR], const float (&run)[MR]) {
    const bool has_bias = bias != nullptr;
    const float b = has_bias ? __half2float(bias[n]) : 0.0f;
    bool bad = false;
#pragma unroll
    for (int r = 0; r < MR; ++r) {
        if (r >= M) break;
        const float total = fold ? run[r] : warp_sum(acc[r]);
        if (lane != r) continue;
        if (out_mode == OUT_RAW32) {
            partial[(size_t)r * ldp + n] = total;
        } else if (out_mode == OUT_RAW16) {
            y[(size_t)r * ldy + n] = __float2half_rn(total);
        } else {
            const float v = fold ? finish_tile16(total, b, has_bias, post) : finish_fp32(total, b, post);
            const __half h = __float2half_rn(v);
            bad |= half_nonfinite(h);
            y[(size_t)r * ldy + n] = h;
        }
    }
    return bad;
}

// ----------------------------------------------------------------------------- per-lane-load kernel
constexpr int D_THREADS = 256;
constexpr int D_UNROLL = 4;

__device__ __forceinline__ uint4 ld_stream(const __half *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

template <int MR>
__global__ void __launch_bounds__(D_THREADS) gemv_direct_kernel(const Params p) {
    const int lane = threadIdx.x & 31;
    const int warps = (gridDim.x * D_THREADS) >> 5;
    const int nchunk = (p.K + 255) >> 8;
    bool bad = false;
    for (int n = (blockIdx.x * D_THREADS + threadIdx.x) >> 5; n < p.N; n += warps) {
        const __half *wrow = p.w + (size_t)n * p.ldw;
        float acc[MR], run[MR];
#pragma unroll
        for (int r = 0; r < MR; ++r) acc[r] = run[r] = 0.0f;
        for (int c0 = 0; c0 < nchunk; c0 += D_UNROLL) {
            uint4 wv[D_UNROLL];
#pragma unroll
            for (int u = 0; u < D_UNROLL; ++u) {
                const int k8 = (c0 + u) * 256 + lane * 8;
                wv[u] = (c0 + u < nchunk && k8 < p.K) ? ld_stream(wrow + k8) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < D_UNROLL; ++u) {
                const int c = c0 + u;
                if (c >= nchunk) break;                       // uniform across the warp
                const int k8 = c * 256 + lane * 8;
                const int valid = k8 < p.K ? min(8, p.K - k8) : 0;
#pragma unroll
                for (int r = 0; r < MR; ++r) {
                    if (r >= p.M) break;
                    float xv[8];
                    widen8(valid ? __ldg(reinterpret_cast<const uint4 *>(p.x + (size_t)r * p.ldx + k8))
                                 : make_uint4(0, 0, 0, 0),
                           xv);
                    const float s = dot8(wv[u], xv, valid);
                    if (p.fold) run[r] = fold16(run[r], warp_sum(s), c == 0);
                    else acc[r] += s;
                }
            }
        }
        bad |= finish_row<MR>(p.M, lane, n, p.out_mode, p.fold, p.post, p.bias, p.y, p.ldy, p.partial, p.ldp, acc,
                              run);
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) raise_flag(p.flags, FLAG_NONFINITE_OUTPUT);
}

// ----------------------------------------------------------------------------- streamed kernel
constexpr long long PDL_MAX_BYTES = 16ll << 20;      // weight bytes up to which launches start early
struct Meta {
    int prob, row0, rows, slice;   // prob < 0: no more units; slice: K slice of a sliced unit
};
// Sliced launches keep the FP32 tile sums of the 16-row blocks they own in a ring of B_RING
// shared-memory buffers of 16 rows x M x/K tiles (the host limits M x tiles to 64).
constexpr int B_RING = 4;
constexpr int TILES_PER_SLICE = STREAM_SLICE / 256;
constexpr int SWZ_BOX_K = 64;                        // K width of one 128-byte swizzled TMA box

// Shared-memory plan: ring of 16 KB slots (one consumer warp per slot) | x table | meta | full and
// empty barriers | abort flag | the group's problems (copied from the kernel parameter once per CTA:
// dynamically indexed parameter reads are slow) | sliced only: tile-sum buffers, their arrival
// counters and the block each buffer is open to. Whole-row launches use 12 slots; sliced launches
// (a single long-K problem) give the 12th slot's space to the tile-sum buffers, wide ones (WX) four
// slots to the 64 KB x table and the larger buffers.
// Half-SM whole-row launches (HF: see half_sm) use 6 slots and the small x table, ~110 KB in all,
// so two CTAs fit one SM: a CTA of the next launch on the stream (programmatic dependent launch)
// becomes resident while this launch's CTA still runs there and streams its own weights into its
// ring, hiding the launch's ramp-up and tail.
// Wide sliced launches (WX: x rows beyond 32 KB, e.g. M = 8 at K = 4096) use 8 slots, a 64 KB x
// table and buffers for M x tiles <= 128, so the batch streams W once.
// WX is the wide configuration of either kind: for sliced launches the 64 KB x table, for whole-row
// launches the 24 KB slots of long octet rows; both have 8 slots.
template <bool SL, bool HF = false, bool WX = false>
struct SCfg {
    static_assert(!(SL && HF), "half-SM launches are whole-row launches");
    static_assert(!(WX && HF), "the wide configurations are full-SM launches");
    static constexpr int STAGES = HF ? 6 : (WX ? 8 : (SL ? 11 : 12));
    static constexpr int THREADS = 32 * (1 + STAGES);
    static constexpr int MIN_BLOCKS = HF ? 2 : 1;
    static constexpr uint32_t STAGE_BYTES = (!SL && WX) ? STREAM_WIDE_ROW_BYTES : STREAM_ROW_BYTES;
    static constexpr int PROBS = SL ? 1 : GROUP_MAX;
    static constexpr uint32_t X_BYTES =
        HF ? STREAM_X_HALF_BYTES : ((SL && WX) ? STREAM_X_WIDE_BYTES : STREAM_X_BYTES);
    static constexpr int BUF_FL = 16 * ((SL && WX) ? STREAM_MAX_XTILES_WIDE : STREAM_MAX_XTILES);   // floats per buffer
    static constexpr uint32_t X_OFFSET = STAGES * STAGE_BYTES;
    static constexpr uint32_t META_OFFSET = X_OFFSET + X_BYTES;
    static constexpr uint32_t BAR_OFFSET = META_OFFSET + STAGES * sizeof(Meta);
    static constexpr uint32_t ABORT_OFFSET = BAR_OFFSET + 2 * STAGES * 8;   // [abort flag, x-table-ready flag]
    static constexpr uint32_t PROB_OFFSET = ABORT_OFFSET + 16;
    static constexpr uint32_t BUF_OFFSET = (PROB_OFFSET + PROBS * (uint32_t)sizeof(Problem) + 15u) & ~15u;
    static constexpr uint32_t CTL_OFFSET = BUF_OFFSET + (SL ? B_RING * BUF_FL * 4u : 0u);
    // sliced launches also reserve the room to align the ring to 1024 bytes (swizzle atom)
    static constexpr uint32_t SMEM_BYTES = CTL_OFFSET + (SL ? 2u * B_RING * 4u + 16u + 1024u : 0u);
};
static_assert(SCfg<false>::SMEM_BYTES <= 232448 && SCfg<true>::SMEM_BYTES <= 232448 &&
              SCfg<true, false, true>::SMEM_BYTES <= 232448, "shared memory");
static_assert(SCfg<true, false, true>::BAR_OFFSET % 8 == 0, "barrier alignment");
static_assert(SCfg<false, false, true>::SMEM_BYTES <= 232448 && SCfg<false, false, true>::BAR_OFFSET % 8 == 0 &&
                  SCfg<false, false, true>::PROB_OFFSET % 8 == 0 && STREAM_WIDE_ROW_BYTES % 16 == 0 &&
                  STREAM_OCTET_WIDE_MAX_K * 2 <= STREAM_WIDE_ROW_BYTES && STREAM_OCTET_WIDE_MAX_K * 2 <= STREAM_X_BYTES,
              "wide-slot whole-row configuration");
// two half-SM CTAs (each with the 1 KB the hardware reserves per CTA) in the SM's 228 KB
static_assert(2 * (SCfg<false, true>::SMEM_BYTES + 1024) <= 233472, "two half-SM CTAs per SM");
static_assert(SCfg<false>::STAGES <= 32 && SCfg<true>::STAGES <= 32, "one producer lane per slot");
static_assert(SCfg<false>::BAR_OFFSET % 8 == 0 && SCfg<true>::BAR_OFFSET % 8 == 0 &&
              SCfg<false, true>::BAR_OFFSET % 8 == 0, "barrier alignment");
static_assert(SCfg<false>::PROB_OFFSET % 8 == 0 && SCfg<false, true>::PROB_OFFSET % 8 == 0 &&
              sizeof(Problem) % 8 == 0, "problem table alignment");
static_assert(16 * STREAM_SLICE * 2 == STREAM_ROW_BYTES && STREAM_SLICE % 256 == 0, "a 16-row slice fills one slot");

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// One 2-D box of a tensor map into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_box(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
                 ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
                 : "memory");
}

// One 3-D box (64 K x 16 rows x 8 K chunks of 64) into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_box3(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

// Non-blocking test of an mbarrier phase (the producer polls all its slots without suspending).
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ void red_release_add(unsigned *p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// CTA-scope acquire load, release store and acquire-release add on shared-memory words (the
// ordering of the tile-sum buffers among the consumer warps of one CTA).
__device__ __forceinline__ int ld_acquire_cta(volatile int *p) {
    int v;
    asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];" : "=r"(v) : "r"(smem_u32(const_cast<int *>(p))) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_cta(volatile int *p, int v) {
    asm volatile("st.release.cta.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(const_cast<int *>(p))), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned atom_add_acq_rel_cta(unsigned *p) {
    unsigned old;
    asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;" : "=r"(old) : "r"(smem_u32(p)) : "memory");
    return old;
}

// D += A * B, m16n8k16, FP16 inputs, FP32 accumulation.
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The units of one CTA. Whole-row launches deal units round-robin (unit blockIdx.x + q * gridDim.x);
// sliced launches give each CTA one contiguous range [first, end) of the block-major unit order
// (unit = block * slices + slice), so a CTA sees every slice of most of its blocks and only the
// blocks at the ends of its range are shared with a neighbour.
struct Range {
    long long first, end;
};
__device__ __forceinline__ Range cta_range(int units) {
    return Range{(long long)blockIdx.x * units / gridDim.x, (long long)(blockIdx.x + 1) * units / gridDim.x};
}

// The producer warp of a sliced launch (one long-K problem): lane s < STAGES feeds ring slot s with
// the units rg.first + s, + STAGES, ... of the CTA's range, then an end marker. The problem's fields
// stay in registers and each lane steps its (block, slice) position without a division, and the
// next position is computed as soon as a copy is issued, so a freed slot costs the lane the meta
// store, the expect-tx and the copy: one 3-D box of 8 x (64 K x 16 rows) when map3, else eight
// 2-D boxes. Polling, abort and the bounded wait are those of produce().
template <bool HF, bool WX>
__device__ __forceinline__ void produce_sliced(const Group &g, const Problem *prob, uint8_t *smem, Meta *meta,
                                               uint32_t full0, uint32_t empty0, volatile int *abort_flag, int lane) {
    using C = SCfg<true, HF, WX>;
    const bool mine = lane < C::STAGES;
    const int slot = mine ? lane : 0;
    const uint32_t full = full0 + 8 * slot, empty = empty0 + 8 * slot;
    const uint32_t dst = smem_u32(smem + (size_t)slot * C::STAGE_BYTES);
    const Range rg = cta_range(g.units);
    const int S = prob[0].slices, N = prob[0].N, kslice = prob[0].kslice, K8 = (prob[0].K + 7) & ~7;
    const bool map3 = g.map3 != 0;
    long long u = rg.first + slot;
    const int uq = (int)(u - prob[0].unit_begin);
    int blk = uq / S, sl = uq - blk * S;
    uint32_t ph = 0;
    bool done = !mine, armed = false;
    uint64_t t0 = 0;
    for (uint32_t polls = 1;; ++polls) {
        if (!done && mbar_test_wait(empty, ph ^ 1u)) {
            if (u < rg.end) {
                const int row0 = blk * 16, k0 = sl * kslice;
                meta[slot] = Meta{0, row0, min(16, N - row0), sl};
                if (map3) {
                    // chunks past K arrive as zeros; the box's bytes are always counted in full
                    mbar_arrive_expect_tx(full, (uint32_t)C::STAGE_BYTES);
                    tma_box3(dst, &g.wmap, full, 0, row0, k0 / SWZ_BOX_K);
                } else {
                    // box b: rows [row0, row0 + 16) x K [k0 + 64b, k0 + 64b + 64); rows past N and
                    // columns past K arrive as zeros
                    const int boxes = min(kslice / SWZ_BOX_K, (K8 - k0 + SWZ_BOX_K - 1) / SWZ_BOX_K);
                    mbar_arrive_expect_tx(full, (uint32_t)boxes * 16u * SWZ_BOX_K * 2u);
                    for (int b = 0; b < boxes; ++b)
                        tma_box(dst + (uint32_t)b * 16u * SWZ_BOX_K * 2u, &g.wmap, full, k0 + SWZ_BOX_K * b, row0);
                }
                armed = true;
                ph ^= 1u;
                u += C::STAGES;
                sl += C::STAGES;
                while (sl >= S) {
                    sl -= S;
                    ++blk;
                }
            } else {
                meta[slot] = Meta{-1, 0, 0, 0};
                mbar_arrive(full);
                done = true;
            }
            t0 = 0;
        }
        if (__all_sync(0xffffffffu, done)) return;
        if ((polls & 255u) == 0) {   // the abort flag and the clock, every 256 polls
            bool stop = *abort_flag != 0;
            if (!stop && !done) {
                const uint64_t t = global_ns();
                if (!t0) {
                    t0 = t;
                } else if (t - t0 > WAIT_LIMIT_NS) {
                    *abort_flag = 1;
                    raise_flag(g.flags, FLAG_TIMEOUT);
                    stop = true;
                }
            }
            if (__any_sync(0xffffffffu, stop)) break;
        }
    }
    if (armed) drain_phase(full, ph ^ 1u);   // the last copy this lane issued
}

// The producer warp of a whole-row launch: lane s < STAGES feeds ring slot s with this CTA's local
// units q = s, s + STAGES, ... then an end marker. All lanes poll their slots' empty barriers
// together with a non-blocking test, so no lane's wait holds up another lane's copy. A unit is one
// bulk copy of its rows. After an abort or a wait that ran out, each lane waits (bounded) for its
// own copy in flight. (Sliced launches use produce_sliced.)
template <bool HF, bool WX>
__device__ __forceinline__ void produce(const Group &g, const Problem *prob, uint8_t *smem, Meta *meta, uint32_t full0,
                                        uint32_t empty0, volatile int *abort_flag, int lane) {
    using C = SCfg<false, HF, WX>;
    const int count = g.count, units = g.units;
    const bool mine = lane < C::STAGES;
    const int slot = mine ? lane : 0;
    const uint32_t full = full0 + 8 * slot, empty = empty0 + 8 * slot;
    const uint32_t dst = smem_u32(smem + (size_t)slot * C::STAGE_BYTES);
    uint32_t ph = 0;
    bool done = !mine, armed = false;
    int q = slot, pi = 0;
    const int hold = g.hold;
    uint64_t t0 = 0;
    for (uint32_t polls = 1;; ++polls) {
        // slots from `hold` on take their first unit once the consumers have issued the x loads
        const bool held = hold && q == slot && slot >= hold && abort_flag[1] == 0;
        if (!done && !held && mbar_test_wait(empty, ph ^ 1u)) {
            const long long u = (long long)blockIdx.x + (long long)q * gridDim.x;   // round-robin units
            if (u < (long long)units) {
                while (pi + 1 < count && u >= prob[pi + 1].unit_begin) ++pi;
                const Problem &p = prob[pi];
                const int row0 = ((int)u - p.unit_begin) * p.rows_per_unit;
                meta[slot] = Meta{pi, row0, min(p.rows_per_unit, p.N - row0), 0};
                const uint32_t bytes = (uint32_t)meta[slot].rows * (uint32_t)p.ldw * 2u;
                mbar_arrive_expect_tx(full, bytes);
                bulk_g2s(dst, p.w + (size_t)row0 * p.ldw, bytes, full);
                armed = true;
                ph ^= 1u;
                q += C::STAGES;
            } else {
                meta[slot] = Meta{-1, 0, 0, 0};
                mbar_arrive(full);
                done = true;
            }
            t0 = 0;
        }
        if (__all_sync(0xffffffffu, done)) return;
        if ((polls & 255u) == 0) {   // the abort flag and the clock, every 256 polls
            bool stop = *abort_flag != 0;
            if (!stop && !done) {
                const uint64_t t = global_ns();
                if (!t0) {
                    t0 = t;
                } else if (t - t0 > WAIT_LIMIT_NS) {
                    *abort_flag = 1;
                    raise_flag(g.flags, FLAG_TIMEOUT);
                    stop = true;
                }
            }
            if (__any_sync(0xffffffffu, stop)) break;
        }
    }
    if (armed) drain_phase(full, ph ^ 1u);   // the last copy this lane issued
}

// One 16-row block of W against up to 8 x rows, with the m16n8k16 MMA: the W rows as A (row-major)
// and the x rows (from the shared x table, zero past K) as B. Lane (g = lane/4, t = lane%4) supplies,
// per 32-wide K window, the 8 consecutive elements at window + 8t of W rows g and g+8 and of x row
// g; those 8 elements are the k-slots {2t, 2t+1, 2t+8, 2t+9} of two consecutive MMAs. The dot
// product only needs A and B to use the same k order, and this order depends on t alone. Four
// accumulators (one per 16-wide slice of a 64-wide step) keep consecutive MMAs independent; their
// sum is the tile sum (tile-16) or the row total (FP32). The accumulator of lane (g, t) holds rows
// g and g+8 for x rows 2t and 2t+1.
struct BlockAcc {
    float acc[4][4];
    float run[4];
};

__device__ __forceinline__ void block_reset(BlockAcc &s) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) s.acc[j][i] = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) s.run[i] = 0.0f;
}

// One 64-wide K window at kw: 4 MMAs over W rows wa / wc and x row xrow. With `tail`, chunks at or
// past K8 load as zeros (only the last window of a K that is not a multiple of 64).
template <bool TAIL>
__device__ __forceinline__ void block_window(const __half *wa, const __half *wc, const __half *xrow, int kw, int K8,
                                             int t4, BlockAcc &s) {
    const uint4 z = make_uint4(0, 0, 0, 0);
    const int k0 = kw + t4 * 8, k1 = k0 + 32;
    const bool l0 = !TAIL || k0 < K8, l1 = !TAIL || k1 < K8;
    const uint4 a0 = l0 ? *reinterpret_cast<const uint4 *>(wa + k0) : z;
    const uint4 a1 = l1 ? *reinterpret_cast<const uint4 *>(wa + k1) : z;
    const uint4 b0 = l0 ? *reinterpret_cast<const uint4 *>(wc + k0) : z;
    const uint4 b1 = l1 ? *reinterpret_cast<const uint4 *>(wc + k1) : z;
    const uint4 x0 = l0 ? *reinterpret_cast<const uint4 *>(xrow + k0) : z;
    const uint4 x1 = l1 ? *reinterpret_cast<const uint4 *>(xrow + k1) : z;
    mma16816(s.acc[0], a0.x, b0.x, a0.y, b0.y, x0.x, x0.y);
    mma16816(s.acc[1], a0.z, b0.z, a0.w, b0.w, x0.z, x0.w);
    mma16816(s.acc[2], a1.x, b1.x, a1.y, b1.y, x1.x, x1.y);
    mma16816(s.acc[3], a1.z, b1.z, a1.w, b1.w, x1.z, x1.w);
}

// Accumulates K positions [0, K8) of W rows wa / wc against x row xrow. Rows past the unit and x rows
// past M are given the pointer of a real row by the caller: they only feed outputs that are never
// stored, so every full window loads without predication. Tile-16 folds run = fp16(run + tile) at
// every 256-K tile (the first tile starts the running sum); FP32 keeps summing.
__device__ __forceinline__ void block_accumulate(const __half *wa, const __half *wc, const __half *xrow, int K8,
                                                 bool fold, int lane, BlockAcc &s) {
    const int t4 = lane & 3;
    const int full = K8 & ~63;   // K covered by full 64-wide windows
    for (int t0 = 0; t0 < K8; t0 += 256) {
        if (fold) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int i = 0; i < 4; ++i) s.acc[j][i] = 0.0f;
        }
        if (t0 + 256 <= full) {
#pragma unroll
            for (int w = 0; w < 4; ++w) block_window<false>(wa, wc, xrow, t0 + 64 * w, K8, t4, s);
        } else {
            const int kend = min(K8, t0 + 256);
            int kw = t0;
            for (; kw + 64 <= kend; kw += 64) block_window<false>(wa, wc, xrow, kw, K8, t4, s);
            if (kw < kend) block_window<true>(wa, wc, xrow, kw, K8, t4, s);
        }
        if (fold) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                s.run[i] = fold16(s.run[i], (s.acc[0][i] + s.acc[1][i]) + (s.acc[2][i] + s.acc[3][i]), t0 == 0);
        }
    }
}

// Writes one output: raw FP32 / raw FP16 / bias + activation. Returns true if a final FP16 output is
// not finite.
// `b` is bias[n] (0 without a bias), loaded by the caller ahead of the sums.
__device__ __forceinline__ float bias_at(const Problem &pr, int n, bool valid) {
    return (pr.bias && valid) ? __half2float(__ldg(pr.bias + n)) : 0.0f;
}
__device__ __forceinline__ bool store_out(const Problem &pr, int xr, int n, float total, float b) {
    if (pr.out_mode == OUT_RAW32) {
        pr.partial[(size_t)xr * pr.ldp + n] = total;
        return false;
    }
    if (pr.out_mode == OUT_RAW16) {
        pr.y[(size_t)xr * pr.ldy + n] = __float2half_rn(total);
        return false;
    }
    const bool has_bias = pr.bias != nullptr;
    const float v = pr.fold ? finish_tile16(total, b, has_bias, pr.post) : finish_fp32(total, b, pr.post);
    const __half h = __float2half_rn(v);
    pr.y[(size_t)xr * pr.ldy + n] = h;
    return half_nonfinite(h);
}

// Hands the warp's ring slot back to the producer: every lane's reads of it are complete (their
// values have been consumed by the instructions before the __syncwarp).
__device__ __forceinline__ void release_slot(uint32_t empty, int lane) {
    __syncwarp();
    if (lane == 0) mbar_arrive(empty);
}

// Writes the block's results: lane (g, t4) element 0 is row g / x row 2t4, 1 row g / x row 2t4+1,
// 2 and 3 the same for row g+8 (rows relative to the block's first row `n0`).
__device__ __forceinline__ bool block_finish(const Problem &pr, int M, int n0, int ra, int rc, int rows, int lane,
                                             const BlockAcc &s, float ba, float bc) {
    const int t4 = lane & 3;
    bool bad = false;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = (i < 2 ? ra : rc), xr = 2 * t4 + (i & 1);
        if (r >= rows || xr >= M) continue;
        const float total = pr.fold ? s.run[i] : (s.acc[0][i] + s.acc[1][i]) + (s.acc[2][i] + s.acc[3][i]);
        bad |= store_out(pr, xr, n0 + r, total, i < 2 ? ba : bc);
    }
    return bad;
}

// A whole-row unit: rows [0, rows) staged at `stage` (pitch ldw), all of K, in 16-row blocks. The
// slot is handed back (`empty`) once the last block's sums are in registers, before its outputs are
// finished and stored; the bias values are loaded before the sums.
__device__ __forceinline__ bool process_unit(const Problem &pr, int M, const __half *stage, const __half *xtab,
                                             int row0, int rows, int lane, uint32_t empty) {
    const int g = lane >> 2;
    const int K8 = (pr.K + 7) & ~7;
    // x rows past M read row M - 1 (their outputs are not stored)
    const __half *xrow = xtab + pr.x_off + (size_t)min(g, M - 1) * K8;
    const bool fin = pr.out_mode == OUT_FINAL;
    bool bad = false;
    for (int rb = 0; rb < rows; rb += 16) {
        const int ra = rb + g, rc = rb + g + 8;
        const float ba = bias_at(pr, row0 + ra, fin && ra < rows), bc = bias_at(pr, row0 + rc, fin && rc < rows);
        BlockAcc s;
        block_reset(s);
        // rows past the unit read its first row (their outputs are not stored)
        block_accumulate(stage + (size_t)(ra < rows ? ra : 0) * pr.ldw, stage + (size_t)(rc < rows ? rc : 0) * pr.ldw,
                         xrow, K8, pr.fold != 0, lane, s);
        if (rb + 16 >= rows) release_slot(empty, lane);
        bad |= block_finish(pr, M, row0, ra, rc, rows, lane, s, ba, bc);
    }
    return bad;
}

// An octet unit (long K, whole rows): W rows ra = 0 and rc = 1 (rc = 0 when the unit has one row)
// staged at `stage` (pitch ldw), against MR x rows (MR = 1, 2 or 4; x rows past M read row M - 1,
// their outputs are not stored).
// Octet o covers the 256-K tiles 8o .. 8o + 7. In its MMAs, A row i is W row (i < 8 ? ra : rc)
// restricted to tile 8o + i % 8 and B column j is tile 8o + j of one x row, so D[i][j] is a tile sum
// where i % 8 == j (the other outputs are discarded). Lane (g, t4) loads, per 64-wide window of its
// tile 8o + g, the 8 consecutive elements at window + 8 t4 (and + 32) of both W rows and of the x
// row: the k order of block_window, whose D[i][j] only needs A row i and B column j from the same
// lanes -- here both come from lanes (g, *). Lanes with odd g take the upper half of each window
// first (the 512-byte tile stride would otherwise put lanes g and g + 1 on the same banks); that
// swaps accumulators 0/1 with 2/3, and their sum (acc0 + acc1) + (acc2 + acc3) is unchanged because
// FP32 addition commutes. So every tile sum is the same bits as slice_sums gives, and the fold below
// is deliver_slice's: the result equals the sliced path's for any batch size.
// Tile (8o + g)'s sums land in lane 4g + g/2 (elements g % 2 and 2 + g % 2); after each octet they are
// gathered with shuffles and folded in K order into the running total of the lane that finishes
// that output. The slot is handed back after the last octet's reads.
// x rows [xb, xb + MR) of the batch (MR = 1 or 2; M = 3..4 runs two passes over the staged rows);
// the pass with `release` hands the slot back.
template <int MR>
__device__ __forceinline__ bool process_octet_unit(const Problem &pr, int M, const __half *stage, const __half *xtab,
                                                   int row0, int rows, int lane, uint32_t empty, int xb,
                                                   bool release) {
    const int g = lane >> 2, t4 = lane & 3;
    const int K8 = (pr.K + 7) & ~7, T = (K8 + 255) >> 8, O = (T + 7) >> 3;
    const __half *wa = stage;
    const __half *wc = stage + (size_t)(rows > 1 ? 1 : 0) * pr.ldw;
    const __half *xr[MR];
#pragma unroll
    for (int m = 0; m < MR; ++m) xr[m] = xtab + pr.x_off + (size_t)min(xb + m, M - 1) * K8;
    // output of this lane in the fold: lane L < 2 MR finishes W row L / MR, x row xb + L % MR
    const int orow = lane / MR, oxr = xb + lane % MR;
    const bool owner = lane < 2 * MR && orow < rows && oxr < M;
    const float b = bias_at(pr, row0 + orow, owner && pr.out_mode == OUT_FINAL);
    const int lo = (g & 1) ? 32 : 0, hi = 32 - lo;   // bank-spreading order of the two window halves
    const int e = g & 1;                              // element of D[g][g] in this lane's fragment
    const uint4 z = make_uint4(0, 0, 0, 0);
    float total = 0.0f;
#pragma unroll 1
    for (int o = 0; o < O; ++o) {
        const int kt = (o * 8 + g) * 256;   // this lane's tile; past K its chunks load as zeros
        float acc[MR][4][4];
#pragma unroll
        for (int m = 0; m < MR; ++m)
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[m][j][i] = 0.0f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const int k0 = kt + 64 * w + 8 * t4 + lo, k1 = kt + 64 * w + 8 * t4 + hi;
            const bool l0 = k0 < K8, l1 = k1 < K8;
            const uint4 a0 = l0 ? *reinterpret_cast<const uint4 *>(wa + k0) : z;
            const uint4 a1 = l1 ? *reinterpret_cast<const uint4 *>(wa + k1) : z;
            const uint4 c0 = l0 ? *reinterpret_cast<const uint4 *>(wc + k0) : z;
            const uint4 c1 = l1 ? *reinterpret_cast<const uint4 *>(wc + k1) : z;
#pragma unroll
            for (int m = 0; m < MR; ++m) {
                const uint4 x0 = l0 ? *reinterpret_cast<const uint4 *>(xr[m] + k0) : z;
                const uint4 x1 = l1 ? *reinterpret_cast<const uint4 *>(xr[m] + k1) : z;
                mma16816(acc[m][0], a0.x, c0.x, a0.y, c0.y, x0.x, x0.y);
                mma16816(acc[m][1], a0.z, c0.z, a0.w, c0.w, x0.z, x0.w);
                mma16816(acc[m][2], a1.x, c1.x, a1.y, c1.y, x1.x, x1.y);
                mma16816(acc[m][3], a1.z, c1.z, a1.w, c1.w, x1.z, x1.w);
            }
        }
        float ts[MR][2];
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            float s[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) s[i] = (acc[m][0][i] + acc[m][1][i]) + (acc[m][2][i] + acc[m][3][i]);
            ts[m][0] = e ? s[1] : s[0];   // W row ra, tile 8o + g
            ts[m][1] = e ? s[3] : s[2];   // W row rc, tile 8o + g
        }
        if (release && o == O - 1) release_slot(empty, lane);   // every read of the stage is done
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int t = o * 8 + j;
            if (t >= T) break;   // uniform
            const int src = j * 4 + (j >> 1);
            float mine = 0.0f;
#pragma unroll
            for (int r = 0; r < 2; ++r)
#pragma unroll
                for (int m = 0; m < MR; ++m) {
                    const float v = __shfl_sync(0xffffffffu, ts[m][r], src);
                    if (lane == r * MR + m) mine = v;
                }
            total = pr.fold ? fold16(total, mine, t == 0) : (t == 0 ? mine : total + mine);
        }
    }
    return owner ? store_out(pr, oxr, row0 + orow, total, b) : false;
}

// The FP32 sums of the (up to) two 256-K tiles of slice `sl` of a 16-row block, staged as eight
// 64 x 16 boxes with the 128-byte swizzle (16-byte chunk c of box row r sits at chunk c ^ (r & 7),
// so the eight rows a warp reads at once fall on different banks). Same products and summation
// order as block_accumulate: ts[tt][i] is tile 2sl + tt of lane element i.
__device__ __forceinline__ void slice_sums(const __half *stage, const __half *xrow, int sl, int K8, int lane,
                                           float (&ts)[TILES_PER_SLICE][4]) {
    const int g = lane >> 2, t4 = lane & 3;
    const uint4 z = make_uint4(0, 0, 0, 0);
    const int ca = (t4 ^ g) * 8, cb = ((t4 ^ g) ^ 4) * 8;   // swizzled chunk offsets (halves) of k0, k1
    const int kb = sl * STREAM_SLICE;
#pragma unroll
    for (int tt = 0; tt < TILES_PER_SLICE; ++tt) {
        float acc[4][4] = {};
#pragma unroll
        for (int st = 0; st < 256 / SWZ_BOX_K; ++st) {
            const int box = tt * (256 / SWZ_BOX_K) + st;
            const int kw = kb + box * SWZ_BOX_K;
            if (kw >= K8) break;   // past the end of K (uniform): the tile ends here
            const __half *bx = stage + box * 16 * SWZ_BOX_K;
            const int k0 = kw + t4 * 8, k1 = k0 + 32;
            // W: rows past N and columns past K of a loaded box arrive as zeros
            const uint4 a0 = *reinterpret_cast<const uint4 *>(bx + g * SWZ_BOX_K + ca);
            const uint4 a1 = *reinterpret_cast<const uint4 *>(bx + g * SWZ_BOX_K + cb);
            const uint4 b0 = *reinterpret_cast<const uint4 *>(bx + (g + 8) * SWZ_BOX_K + ca);
            const uint4 b1 = *reinterpret_cast<const uint4 *>(bx + (g + 8) * SWZ_BOX_K + cb);
            // x: only the box that crosses K8 has chunks past the x row
            const bool full = kw + SWZ_BOX_K <= K8;
            const uint4 x0 = (full || k0 < K8) ? *reinterpret_cast<const uint4 *>(xrow + k0) : z;
            const uint4 x1 = (full || k1 < K8) ? *reinterpret_cast<const uint4 *>(xrow + k1) : z;
            mma16816(acc[0], a0.x, b0.x, a0.y, b0.y, x0.x, x0.y);
            mma16816(acc[1], a0.z, b0.z, a0.w, b0.w, x0.z, x0.w);
            mma16816(acc[2], a1.x, b1.x, a1.y, b1.y, x1.x, x1.y);
            mma16816(acc[3], a1.z, b1.z, a1.w, b1.w, x1.z, x1.w);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) ts[tt][i] = (acc[0][i] + acc[1][i]) + (acc[2][i] + acc[3][i]);
    }
}

// Shared-memory state of a sliced launch's tile-sum buffers.
struct SliceCtl {
    float *buf;              // B_RING x buf_floats: [tile (T)][row (16)][x row (M)]
    unsigned *count;         // [B_RING] slices of the buffer's block that have arrived
    volatile int *open;      // [B_RING] local block index the buffer is open to
    unsigned *lead;          // slices handed on so far of the block owned by the previous CTA
    int buf_floats;          // floats per buffer (16 x the largest M x tiles of the configuration)
};

// Bounded spin of lane 0 until the buffer is open to local block lb (its previous block was folded).
__device__ __forceinline__ bool wait_open(const SliceCtl &ctl, int bb, int lb, volatile int *abort_flag,
                                          unsigned *flags) {
    uint64_t t0 = 0;
    for (uint32_t i = 1; ctl.open[bb] != lb; ++i) {
        if ((i & 255u) == 0) {
            if (*abort_flag) return false;
            const uint64_t t = global_ns();
            if (!t0) {
                t0 = t;
            } else if (t - t0 > WAIT_LIMIT_NS) {
                *abort_flag = 1;
                raise_flag(flags, FLAG_TIMEOUT);
                return false;
            }
        }
    }
    return true;
}

// Bounded wait of the whole warp (every lane acquires) until `expected` slices have arrived on the
// block counter from other CTAs.
__device__ __forceinline__ bool wait_remote(const unsigned *cnt, unsigned expected, volatile int *abort_flag,
                                            unsigned *flags) {
    uint64_t t0 = 0;
    for (uint32_t i = 1; !__all_sync(0xffffffffu, ld_acquire(cnt) >= expected); ++i) {
        if ((i & 63u) == 0) {
            bool stop = *abort_flag != 0;
            if (!stop) {
                const uint64_t t = global_ns();
                if (!t0) {
                    t0 = t;
                } else if (t - t0 > WAIT_LIMIT_NS) {
                    stop = true;
                }
            }
            if (__any_sync(0xffffffffu, stop)) {
                if ((threadIdx.x & 31) == 0 && !*abort_flag) {
                    *abort_flag = 1;
                    raise_flag(flags, FLAG_TIMEOUT);
                }
                return false;
            }
        }
    }
    return true;
}

// Hands one slice's tile sums on and finishes the block when they complete it. The owner of a
// block is the CTA whose range holds the block's slice 0. It meets every other slice of the block in
// its own range, except for the block at the end of its range, whose remaining slices open the
// ranges of the following CTAs (processed first there, so they are in by the time the owner needs
// them).
//   Owner: the sums go to the block's shared buffer (tile-major, so the folding lanes read
//   consecutive words). The warp that brings the block's last local slice folds the tile sums in K
//   order -- the fp16 fold of the tile-16 arithmetic, or their FP32 sum -- after a bounded wait for
//   the other CTAs' slices, writes Y and reopens the buffer.
//   Other CTAs: the sums go to the block's rows of the device scratch, counted as described below.
//   The owner resets the block counter.
// The bits are those of folding the same tile sums in one place. `fb` is the first block this CTA
// owns (the first whose slice 0 lies in its range).
__device__ __forceinline__ bool deliver_slice(const Group &grp, const Problem &pr, int M, const SliceCtl &ctl,
                                              const Range &rg, int fb, int row0, int rows, int sl, int lane,
                                              const float (&ts)[TILES_PER_SLICE][4], volatile int *abort_flag) {
    const int g = lane >> 2, t4 = lane & 3;
    const int K8 = (pr.K + 7) & ~7, T = (K8 + 255) >> 8, S = pr.slices;
    const int blk = row0 / 16;
    const long long b0 = (long long)blk * S;   // unit of the block's slice 0
    const int tiles = min(TILES_PER_SLICE, T - sl * TILES_PER_SLICE);
    unsigned *cnt = grp.scratch.tcount + blk;
    float *tg = grp.scratch.tsum + (size_t)row0 * M * T;   // the block's tile sums in the scratch
    if (b0 < rg.first) {
#pragma unroll
        for (int tt = 0; tt < TILES_PER_SLICE; ++tt) {
            if (tt >= tiles) break;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int r = i < 2 ? g : g + 8, xr = 2 * t4 + (i & 1);
                if (r < rows && xr < M) tg[((size_t)r * M + xr) * T + sl * TILES_PER_SLICE + tt] = ts[tt][i];
            }
        }
        // The CTA's slices of this block are the first units of its range: each counts itself in
        // shared memory (acquire-release), and the one that completes them publishes them all with one
        // GPU-scope release (cumulative over the sums the count has ordered before it).
        __syncwarp();   // the warp's sums are ordered before lane 0's count
        if (lane == 0) {
            const unsigned lead = (unsigned)(min(rg.end, b0 + S) - rg.first);
            if (atom_add_acq_rel_cta(ctl.lead) == lead - 1u) red_release_add(cnt, lead);
        }
        return false;
    }
    const int lb = blk - fb;   // local index among the blocks this CTA owns
    const int bb = lb & (B_RING - 1);
    float *buf = ctl.buf + bb * ctl.buf_floats;
    bool ok = true;
    if (lane == 0 && ld_acquire_cta(ctl.open + bb) != lb) {   // acquire: the buffer's previous reads are done
        ok = wait_open(ctl, bb, lb, abort_flag, grp.flags);
        __threadfence_block();
    }
    __syncwarp();   // ... and ordered before this warp's writes
    if (!__shfl_sync(0xffffffffu, ok, 0)) return false;
#pragma unroll
    for (int tt = 0; tt < TILES_PER_SLICE; ++tt) {
        if (tt >= tiles) break;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = i < 2 ? g : g + 8, xr = 2 * t4 + (i & 1);
            if (r < rows && xr < M) buf[(sl * TILES_PER_SLICE + tt) * 16 * M + r * M + xr] = ts[tt][i];
        }
    }
    const long long lend = min(rg.end, b0 + S);   // local slices of the block: [b0, lend)
    const unsigned local = (unsigned)(lend - b0), remote = (unsigned)S - local;
    __syncwarp();
    int last = 0;
    // release: this warp's sums before the count; acquire: the other warps' sums before the fold
    if (lane == 0) last = atom_add_acq_rel_cta(ctl.count + bb) == local - 1u;
    __syncwarp();
    if (!__shfl_sync(0xffffffffu, last, 0)) return false;
    if (remote && !wait_remote(cnt, remote, abort_flag, grp.flags)) return false;
    const int ltiles = (int)local * TILES_PER_SLICE;   // tiles [0, ltiles) are in the buffer
    bool bad = false;
    for (int o = lane; o < rows * M; o += 32) {
        const int r = o / M, xr = o - r * M;
        const float *pl = buf + r * M + xr;   // tile t at pl[16 M t]
        const float *pg = tg + ((size_t)r * M + xr) * T;
        const float b = bias_at(pr, row0 + r, pr.out_mode == OUT_FINAL);
        float total = 0.0f;
        for (int t0 = 0; t0 < T; t0 += 8) {   // eight tile sums loaded ahead of their fold
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int t = t0 + j;
                v[j] = t >= T ? 0.0f : t < ltiles ? pl[t * 16 * M] : __ldcg(pg + t);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int t = t0 + j;
                if (t < T) total = pr.fold ? fold16(total, v[j], t == 0) : (t == 0 ? v[j] : total + v[j]);
            }
        }
        bad |= store_out(pr, xr, row0 + r, total, b);
    }
    __syncwarp();
    if (lane == 0) {
        if (remote) *cnt = 0u;   // every other slice of this launch has arrived
        ctl.count[bb] = 0u;
        st_release_cta(ctl.open + bb, lb + B_RING);   // after the count reset and the warp's reads
    }
    return bad;
}

template <bool SL, bool HF, bool WX>
__global__ void __launch_bounds__(SCfg<SL, HF, WX>::THREADS, SCfg<SL, HF, WX>::MIN_BLOCKS)
    gemv_stream_kernel(const __grid_constant__ Group g) {
    using C = SCfg<SL, HF, WX>;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    // sliced launches read 128-byte-swizzled boxes, whose pattern repeats every 1024 bytes
    uint8_t *smem = SL ? reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                     ~static_cast<uintptr_t>(1023))
                       : smem_raw;
    Meta *meta = reinterpret_cast<Meta *>(smem + C::META_OFFSET);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFFSET);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + C::ABORT_OFFSET);
    Problem *prob = reinterpret_cast<Problem *>(smem + C::PROB_OFFSET);
    __half *xtab = reinterpret_cast<__half *>(smem + C::X_OFFSET);
    SliceCtl ctl{reinterpret_cast<float *>(smem + C::BUF_OFFSET), reinterpret_cast<unsigned *>(smem + C::CTL_OFFSET),
                 reinterpret_cast<volatile int *>(smem + C::CTL_OFFSET + 4 * B_RING),
                 reinterpret_cast<unsigned *>(smem + C::CTL_OFFSET + 8 * B_RING), C::BUF_FL};
    const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * C::STAGES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Programmatic dependent launch (when the launch allows it): the next kernel on the stream may
    // start as SMs free up. This kernel's producer only reads W, which no kernel writes; every read
    // of x and every global write happens in the consumer warps after griddepcontrol.wait (the
    // previous kernel has completed and its writes are visible), so neither a read-after-write nor
    // a write-after-read crosses. Without the attribute both instructions have no effect.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (warp == 0) {
        // Warp 0 sets up the barriers, the problem table and the tile-sum buffers' state, hands them
        // to the consumer warps with a non-blocking arrive on named barrier 2, and its producer lanes
        // start streaming at once.
        if (SL && lane == 0)
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&g.wmap)) : "memory");
        if (lane == 0) {
            for (int s = 0; s < C::STAGES; ++s) {
                mbar_init(full0 + 8 * s, 1);
                mbar_init(empty0 + 8 * s, 1);
            }
            abort_flag[0] = 0;
            abort_flag[1] = 0;   // x table ready
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        if (SL && lane < B_RING) {
            ctl.count[lane] = 0u;
            ctl.open[lane] = lane;
        }
        if (SL && lane == 0) *ctl.lead = 0u;
        const int words = g.count * (int)(sizeof(Problem) / 8);
        const unsigned long long *src = reinterpret_cast<const unsigned long long *>(g.prob);
        unsigned long long *dst = reinterpret_cast<unsigned long long *>(prob);
        for (int i = lane; i < words; i += 32) dst[i] = src[i];
        __syncwarp();
        asm volatile("bar.arrive 2, %0;" ::"r"(C::THREADS) : "memory");
        if constexpr (SL) produce_sliced<HF, WX>(g, prob, smem, meta, full0, empty0, abort_flag, lane);
        else produce<HF, WX>(g, prob, smem, meta, full0, empty0, abort_flag, lane);
        return;
    }
    asm volatile("bar.sync 2, %0;" ::"r"(C::THREADS) : "memory");   // barriers and problem table ready
    asm volatile("griddepcontrol.wait;" ::: "memory");              // the previous kernel is done

    // The consumer warps fill the x table (x rows, zero past K) while the producer streams W. Every
    // 16-byte chunk of every source is issued before any is waited for (cp.async, the bytes past K
    // zero-filled by the copy), so the fill costs one round trip however many inputs the launch has:
    // these loads queue behind the W stream already in flight.
    {
        const int ct = threadIdx.x - 32, nct = C::STAGES * 32;
        for (int e = 0; e < g.nx; ++e) {
            const XSource xs = g.xsrc[e];
            const int K8 = (xs.K + 7) & ~7, per_row = K8 / 8;
            for (int i = ct; i < g.M * per_row; i += nct) {
                const int r = i / per_row, k = (i - r * per_row) * 8;
                const uint32_t bytes = (uint32_t)min(8, xs.K - k) * 2u;   // k < K: at least one element
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                                 smem_u32(xtab + xs.off + (size_t)r * K8 + k)),
                             "l"(xs.x + (size_t)r * xs.ldx + k), "r"(bytes)
                             : "memory");
            }
        }
        // Once every x request is issued, the producer slots held back (see Group::hold) may queue
        // their W copies behind them: the stream keeps HBM busy while x is in flight (measured on
        // the 63.8 MB grouped decode set: 12.99 -> 12.72 us; the LM head alone unchanged).
        asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("bar.sync 1, %0;" ::"r"(nct) : "memory");
        if (threadIdx.x == 32) abort_flag[1] = 1;
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        asm volatile("bar.sync 1, %0;" ::"r"(nct) : "memory");
    }

    // Consumer warp c owns slot c and takes its units in order (the producer fills slot c with the
    // CTA's units c, c + STAGES, ...); it stops at the end marker.
    const int c = warp - 1;
    const uint32_t full = full0 + 8 * c, empty = empty0 + 8 * c;
    const __half *stage = reinterpret_cast<const __half *>(smem + (size_t)c * C::STAGE_BYTES);
    const Range rg = cta_range(g.units);
    const int fb = SL ? (int)((rg.first + prob[0].slices - 1) / prob[0].slices) : 0;
    bool bad = false;
    for (uint32_t ph = 0;; ph ^= 1u) {
        // Every lane waits (each gets the barrier's acquire); the warp leaves together.
        if (!__all_sync(0xffffffffu, wait_phase(full, ph, abort_flag, g.flags))) break;
        const Meta mt = meta[c];
        if (mt.prob < 0) break;
        const Problem &pr = prob[mt.prob];
        if (SL) {
            const int gq = lane >> 2, K8 = (pr.K + 7) & ~7;
            // x rows past M read row M - 1 (their outputs are not kept)
            const __half *xrow = xtab + pr.x_off + (size_t)min(gq, g.M - 1) * K8;
            float ts[TILES_PER_SLICE][4];
            slice_sums(stage, xrow, mt.slice, K8, lane, ts);
            __syncwarp();
            if (lane == 0) mbar_arrive(empty);   // the slot refills while the sums are handed on
            bad |= deliver_slice(g, pr, g.M, ctl, rg, fb, mt.row0, mt.rows, mt.slice, lane, ts, abort_flag);
        } else if (pr.octet) {
            if (g.M == 1) {
                bad |= process_octet_unit<1>(pr, g.M, stage, xtab, mt.row0, mt.rows, lane, empty, 0, true);
            } else {
                const bool two = g.M > 2;   // a half-SM launch's 12 KB table holds two long-K x rows at most
                bad |= process_octet_unit<2>(pr, g.M, stage, xtab, mt.row0, mt.rows, lane, empty, 0, HF || !two);
                if (!HF && two)
                    bad |= process_octet_unit<2>(pr, g.M, stage, xtab, mt.row0, mt.rows, lane, empty, 2, true);
            }
        } else {
            bad |= process_unit(pr, g.M, stage, xtab, mt.row0, mt.rows, lane, empty);
        }
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) raise_flag(g.flags, FLAG_NONFINITE_OUTPUT);
}

// ----------------------------------------------------------------------------- host helpers
int device_index() {
    int dev = 0;
    cudaGetDevice(&dev);
    return dev;
}

cudaError_t stream_attr() {
    static bool done[64] = {};
    const int dev = device_index();
    if (dev >= 0 && dev < 64 && done[dev]) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(gemv_stream_kernel<false, false, false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SCfg<false>::SMEM_BYTES);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemv_stream_kernel<true, false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)SCfg<true>::SMEM_BYTES);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemv_stream_kernel<true, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)SCfg<true, false, true>::SMEM_BYTES);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemv_stream_kernel<false, true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)SCfg<false, true>::SMEM_BYTES);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemv_stream_kernel<false, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)SCfg<false, false, true>::SMEM_BYTES);
    if (e == cudaSuccess && dev >= 0 && dev < 64) done[dev] = true;
    return e;
}

template <int MR>
int direct_blocks_per_sm() {
    static int cached = 0;
    if (!cached) {
        int b = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, gemv_direct_kernel<MR>, D_THREADS, 0) != cudaSuccess ||
            b < 1) {
            cudaGetLastError();
            b = 1;
        }
        cached = b;
    }
    return cached;
}

int direct_blocks(int M) {
    if (M <= 1) return direct_blocks_per_sm<1>();
    if (M <= 2) return direct_blocks_per_sm<2>();
    if (M <= 4) return direct_blocks_per_sm<4>();
    return direct_blocks_per_sm<MAX_M>();
}

unsigned direct_grid(int M, int N, int sm_count) {
    const long long need = ((long long)N + (D_THREADS / 32) - 1) / (D_THREADS / 32);
    const long long cap = (long long)sm_count * direct_blocks(M);
    return (unsigned)(need < cap ? need : cap);
}

// Long-K whole-row (octet) units: 2048 < K <= 8192 with the row in one slot, M <= 4, and the M x rows
// within the 32 KB x table; or, at M = 1, rows up to K = 12288 in the wide slots.
bool octet(int M, int K, long long ldw) {
    const long long k8 = ((long long)K + 7) & ~7ll;
    if (k8 <= STREAM_WHOLE_K) return false;
    if (k8 <= STREAM_OCTET_MAX_K && ldw * 2 <= (long long)STREAM_ROW_BYTES && M >= 1 && M <= STREAM_OCTET_MAX_M &&
        (long long)M * k8 * 2 <= STREAM_X_BYTES)
        return true;
    return M == 1 && k8 <= STREAM_OCTET_WIDE_MAX_K && ldw * 2 <= (long long)STREAM_WIDE_ROW_BYTES;
}

// Rows longer than a 16 KB slot (octet units of the wide-slot configuration).
bool wide_rows(long long ldw) { return ldw * 2 > (long long)STREAM_ROW_BYTES; }

// Whole-row problems: rows per unit spread the group's weight bytes over about two units per SM, one
// slot at most. Octet problems: one or two whole rows per unit. Other long-K problems (or rows wider
// than a slot): 16-row units streamed in K slices.
void plan_units(Group &g, int sm_count) {
    long long total = 0;
    for (int i = 0; i < g.count; ++i) total += (long long)g.prob[i].N * g.prob[i].ldw * 2;
    long long target = total / (2LL * (sm_count > 0 ? sm_count : 1));
    if (target > (long long)STREAM_ROW_BYTES) target = STREAM_ROW_BYTES;
    int units = 0;
    for (int i = 0; i < g.count; ++i) {
        Problem &p = g.prob[i];
        const int k8 = (p.K + 7) & ~7;
        p.octet = 0;
        if (octet(g.M, p.K, p.ldw)) {
            // two rows per unit while they fit a slot (the A rows of an octet MMA hold two W rows)
            p.octet = 1;
            p.kslice = 0;
            p.slices = 1;
            p.rows_per_unit = 2 * p.ldw * 2 <= (long long)STREAM_ROW_BYTES ? 2 : 1;
            p.unit_begin = units;
            units += (p.N + p.rows_per_unit - 1) / p.rows_per_unit;
            continue;
        }
        if (k8 > STREAM_WHOLE_K || p.ldw * 2 > (long long)STREAM_ROW_BYTES) {
            p.kslice = STREAM_SLICE;
            p.slices = (k8 + STREAM_SLICE - 1) / STREAM_SLICE;
            p.rows_per_unit = 16;
            p.unit_begin = units;
            units += (p.N + 15) / 16 * p.slices;
            continue;
        }
        p.kslice = 0;
        p.slices = 1;
        const long long row_bytes = p.ldw * 2;
        long long r = target / row_bytes;
        const long long rmax = (long long)STREAM_ROW_BYTES / row_bytes;
        if (r < 1) r = 1;
        if (r > rmax) r = rmax;
        p.rows_per_unit = (int)r;
        p.unit_begin = units;
        units += (int)((p.N + r - 1) / r);
    }
    g.units = units;
}

}  // namespace

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

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

// W [N, ldw] of which K columns are valid, as 64 (K) x 16 (rows) boxes with the 128-byte swizzle:
// the layout slice_sums reads. Columns >= K and rows >= N arrive as zeros.
static bool make_wmap(CUtensorMap *map, const __half *w, int K, int N, long long ldw) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
    cuuint64_t strides[1] = {(cuuint64_t)ldw * 2};
    cuuint32_t box[2] = {(cuuint32_t)SWZ_BOX_K, 16};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(w), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// W [N, ldw] with K a multiple of 64, as one 3-D box per unit: dimension 0 is 64 K elements,
// dimension 1 the rows (stride ldw), dimension 2 the K chunks of 64 (stride 128 bytes), box 64 x 16 x 8
// with the 128-byte swizzle. Shared memory receives the eight 64 x 16 boxes of make_wmap back to back.
// Every element read lies inside its row ([0, K)), so the map reads nothing past W; chunks past K
// arrive as zeros.
static bool make_wmap3(CUtensorMap *map, const __half *w, int K, int N, long long ldw) {
    EncodeTiledFn enc = encode_fn();
    if (!enc || K % SWZ_BOX_K) return false;
    cuuint64_t dims[3] = {(cuuint64_t)SWZ_BOX_K, (cuuint64_t)N, (cuuint64_t)(K / SWZ_BOX_K)};
    cuuint64_t strides[2] = {(cuuint64_t)ldw * 2, (cuuint64_t)SWZ_BOX_K * 2};
    cuuint32_t box[3] = {(cuuint32_t)SWZ_BOX_K, 16, (cuuint32_t)(STREAM_SLICE / SWZ_BOX_K)};
    cuuint32_t estr[3] = {1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half *>(w), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t prepare() {
    for (int m = 1; m <= MAX_M; m *= 2) direct_blocks(m);
    if (!encode_fn()) return cudaErrorNotSupported;
    return stream_attr();
}

bool sliced(int M, int K, long long ldw) {
    const long long k8 = ((long long)K + 7) & ~7ll;
    return (k8 > STREAM_WHOLE_K || ldw * 2 > (long long)STREAM_ROW_BYTES) && !octet(M, K, ldw);
}

// Half-SM CTAs (6 slots, two CTAs per SM) serve the whole-row launches whose x rows fit the small
// table, with programmatic dependent launch:
//   * up to PDL_MAX_BYTES of weights, one CTA per SM: the next launch's CTA becomes resident beside
//     this one and prefetches its weights while this one runs (1.8 MB projection 3.3 -> 2.6 us);
//   * larger launches, two CTAs per SM (192 KB in flight per SM, as with full-SM CTAs; one 96 KB CTA
//     per SM streamed the 56 MB LM head in 13.9 us against 12.4 us): each CTA of the next launch takes
//     the place of one that exits and streams during this launch's drain (LM head 12.4 -> 11.5 us).
static bool half_sm(bool sl, long long x_elems) { return !sl && x_elems * 2 <= STREAM_X_HALF_BYTES; }
static unsigned stream_grid(bool hf, long long wbytes, int units, int sm_count) {
    const int ctas = hf && wbytes > PDL_MAX_BYTES ? 2 * sm_count : sm_count;
    return (unsigned)(units < ctas ? units : ctas);
}

// A sliced launch of M x rows needs the wide configuration when its x rows exceed the 32 KB table or
// its M x tiles exceed the standard block buffers.
static bool wide_x(int M, int K) {
    const long long k8 = ((long long)K + 7) & ~7ll;
    return (long long)M * k8 * 2 > STREAM_X_BYTES || (long long)M * ((k8 + 255) / 256) > STREAM_MAX_XTILES;
}

// x rows of one launch: as many as the x table holds (and, for a sliced problem, as many as the
// scratch holds the tile sums of); 0 when not even one fits.
static long long rows_that_fit(int M, int N, int K, long long ldw) {
    const long long k8 = ((long long)K + 7) & ~7ll;
    if (octet(M, K, ldw)) return (long long)STREAM_X_BYTES / (k8 * 2);
    const bool sl = sliced(M, K, ldw);
    long long fit = (long long)(sl ? STREAM_X_WIDE_BYTES : STREAM_X_BYTES) / (k8 * 2);
    if (sl) {
        if ((N + 15) / 16 > TCOUNT_WORDS) return 0;
        const long long tiles = (k8 + 255) / 256;
        const long long per_row = ((long long)N + 15) / 16 * 16 * tiles;
        const long long fs = TSUM_FLOATS / per_row, fb = STREAM_MAX_XTILES_WIDE / tiles;
        if (fs < fit) fit = fs;
        if (fb < fit) fit = fb;
    }
    return fit;
}

int stream_stages(int M, int N, int K, long long ldw) {
    if (!stream_launches(M, N, K, ldw)) return 0;
    if (sliced(M, K, ldw)) return wide_x(M, K) ? SCfg<true, false, true>::STAGES : SCfg<true>::STAGES;
    if (wide_rows(ldw)) return SCfg<false, false, true>::STAGES;
    const long long xelems = (long long)M * (((long long)K + 7) & ~7ll);
    return half_sm(false, xelems) ? SCfg<false, true>::STAGES : SCfg<false>::STAGES;
}

int stream_launches(int M, int N, int K, long long ldw) {
    if (M < 1 || M > STREAM_MAX_M || K < 1 || N < 1 || ldw < K) return 0;
    const long long fit = rows_that_fit(M, N, K, ldw);
    if (fit < 1) return 0;
    return (int)((M + fit - 1) / fit);
}

bool streamed(int M, int N, int K, long long ldw) { return stream_launches(M, N, K, ldw) == 1; }

namespace {

// Assigns x-table offsets to problems [first, last) of `all` (sharing entries for the same x, ldx
// and K) and copies them into `g`. Returns the index after the last problem that fits.
int pack_group(const Group &all, int first, Group &g) {
    g.count = 0;
    g.nx = 0;
    g.M = all.M;
    g.flags = all.flags;
    g.scratch = all.scratch;
    int used = 0;
    int i = first;
    for (; i < all.count; ++i) {
        Problem p = all.prob[i];
        // a sliced problem uses the whole tile-sum scratch: it runs in a launch of its own
        if (sliced(all.M, p.K, p.ldw) && g.count > 0) break;
        if (g.count == 1 && sliced(all.M, g.prob[0].K, g.prob[0].ldw)) break;
        int e = 0;
        while (e < g.nx && !(g.xsrc[e].x == p.x && g.xsrc[e].ldx == p.ldx && g.xsrc[e].K == p.K)) ++e;
        if (e == g.nx) {
            const int need = all.M * ((p.K + 7) & ~7);
            if ((used + need) * 2 > (sliced(all.M, p.K, p.ldw) ? STREAM_X_WIDE_BYTES : STREAM_X_BYTES)) break;
            g.xsrc[g.nx++] = XSource{p.x, p.ldx, p.K, used};
            used += need;
        }
        p.x_off = g.xsrc[e].off;
        g.prob[g.count++] = p;
    }
    return i;
}

}  // namespace

cudaError_t launch_group(Group &all, cudaStream_t stream, int sm_count, unsigned *grid_out, unsigned *launches) {
    if (launches) *launches = 0;
    if (all.count < 1 || all.count > GROUP_MAX || all.M < 1 || all.M > STREAM_MAX_M) return cudaErrorInvalidValue;
    for (int i = 0; i < all.count; ++i) {
        const Problem &p = all.prob[i];
        if (!streamed(all.M, p.N, p.K, p.ldw) || p.ldw % 8 ||
            p.ldx < p.K || p.ldx % 8 || (reinterpret_cast<uintptr_t>(p.w) & 15) ||
            (reinterpret_cast<uintptr_t>(p.x) & 15))
            return cudaErrorInvalidValue;
    }
    const cudaError_t e = stream_attr();
    if (e != cudaSuccess) return e;
    for (int first = 0; first < all.count;) {
        Group g{};
        const int next = pack_group(all, first, g);
        if (next == first) return cudaErrorInvalidValue;   // one problem always fits the table
        plan_units(g, sm_count);
        if (g.prob[0].kslice) {
            const Problem &p0 = g.prob[0];
            g.map3 = make_wmap3(&g.wmap, p0.w, p0.K, p0.N, p0.ldw) ? 1 : 0;
            if (!g.map3 && !make_wmap(&g.wmap, p0.w, p0.K, p0.N, p0.ldw)) return cudaErrorInvalidValue;
        }
        const bool sl = g.prob[0].kslice != 0;   // a sliced problem is alone in its launch
        int xused = 0;                           // FP16 elements of the x table this launch fills
        for (int e = 0; e < g.nx; ++e) {
            const int end = g.xsrc[e].off + g.M * ((g.xsrc[e].K + 7) & ~7);
            if (end > xused) xused = end;
        }
        long long wbytes = 0;
        for (int i = 0; i < g.count; ++i) wbytes += (long long)g.prob[i].N * g.prob[i].ldw * 2;
        bool wr = false;                         // octet rows longer than a 16 KB slot: wide slots
        for (int i = 0; i < g.count; ++i) wr = wr || (!sl && wide_rows(g.prob[i].ldw));
        const bool hf = half_sm(sl, xused) && !wr;
        const unsigned grid = stream_grid(hf, wbytes, g.units, sm_count);
        // Two half-SM CTAs per SM keep ~28 MB of weights in flight across the GPU, and loads queue
        // behind them: the x rows the consumers need first would wait ~2-4 us. In those launches
        // each producer fills half its ring, then the rest once its CTA has issued its x loads (measured:
        // LM head 12.7 -> 11.6 us, 63.8 MB grouped decode set 15.7 -> 14.4 us, 4096 x 4096 at K =
        // 4096 9.3 -> 8.8 us; a 7 MB launch with one CTA per SM was slower with it).
        g.hold = hf && grid > (unsigned)sm_count ? SCfg<false, true>::STAGES / 2 : 0;
        if (grid_out) *grid_out = grid;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        const bool wx = sl && wide_x(g.M, g.prob[0].K);
        cfg.blockDim = dim3(sl   ? (wx ? SCfg<true, false, true>::THREADS : SCfg<true>::THREADS)
                            : wr ? SCfg<false, false, true>::THREADS
                                 : (hf ? SCfg<false, true>::THREADS : SCfg<false>::THREADS));
        cfg.dynamicSmemBytes = sl   ? (wx ? SCfg<true, false, true>::SMEM_BYTES : SCfg<true>::SMEM_BYTES)
                               : wr ? SCfg<false, false, true>::SMEM_BYTES
                                    : (hf ? SCfg<false, true>::SMEM_BYTES : SCfg<false>::SMEM_BYTES);
        cfg.stream = stream;
        // Early start of the next kernel: always for half-SM launches (half_sm); full-SM launches
        // (whose next CTAs cannot become resident before this launch's exit) allow it where the fixed
        // per-launch cost dominates (it hid 0.6-0.7 us of a 1.8 MB projection), up to PDL_MAX_BYTES
        // of weights (it had slowed 56 MB full-SM launches with M >= 4 by ~10 %).
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = (hf || wbytes <= PDL_MAX_BYTES) ? 1 : 0;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const cudaError_t le0 = sl   ? (wx ? cudaLaunchKernelEx(&cfg, gemv_stream_kernel<true, false, true>, g)
                                           : cudaLaunchKernelEx(&cfg, gemv_stream_kernel<true, false, false>, g))
                                : wr ? cudaLaunchKernelEx(&cfg, gemv_stream_kernel<false, false, true>, g)
                                : hf ? cudaLaunchKernelEx(&cfg, gemv_stream_kernel<false, true, false>, g)
                                     : cudaLaunchKernelEx(&cfg, gemv_stream_kernel<false, false, false>, g);
        if (le0 != cudaSuccess) return le0;
        const cudaError_t le = cudaGetLastError();
        if (le != cudaSuccess) return le;
        if (launches) ++*launches;
        first = next;
    }
    return cudaSuccess;
}

unsigned grid_for(int M, int N, int K, long long ldw, int sm_count) {
    const int nl = stream_launches(M, N, K, ldw);
    if (!nl) return direct_grid(M, N, sm_count);
    Group g = {};
    g.count = 1;
    g.M = (M + nl - 1) / nl;   // x rows of the first launch
    g.prob[0].N = N;
    g.prob[0].K = K;
    g.prob[0].ldw = ldw;
    plan_units(g, sm_count);
    const bool hf = half_sm(sliced(g.M, K, ldw), (long long)g.M * (((long long)K + 7) & ~7ll));
    return stream_grid(hf, (long long)N * ldw * 2, g.units, sm_count);
}

cudaError_t launch(const Params &p, cudaStream_t stream, int sm_count, unsigned *grid_out) {
    if (p.M < 1 || p.M > MAX_M) return cudaErrorInvalidValue;
    const int nl = stream_launches(p.M, p.N, p.K, p.ldw);
    if (nl > 0) {
        const int per = (p.M + nl - 1) / nl;   // x rows per launch, balanced
        for (int r0 = 0; r0 < p.M; r0 += per) {
            Group g = {};
            g.count = 1;
            g.M = p.M - r0 < per ? p.M - r0 : per;
            g.flags = p.flags;
            g.scratch = p.scratch;
            g.prob[0] = Problem{p.x + (size_t)r0 * p.ldx, p.ldx, p.w, p.ldw, p.bias,
                                p.y ? p.y + (size_t)r0 * p.ldy : nullptr, p.ldy,
                                p.partial ? p.partial + (size_t)r0 * p.ldp : nullptr, p.ldp,
                                p.N, p.K, p.out_mode, p.post, p.fold, 0, 0, 0, 0, 0, 0};
            const cudaError_t e = launch_group(g, stream, sm_count, grid_out, nullptr);
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    }
    const unsigned grid = direct_grid(p.M, p.N, sm_count);
    if (grid_out) *grid_out = grid;
    if (p.M <= 1) gemv_direct_kernel<1><<<grid, D_THREADS, 0, stream>>>(p);
    else if (p.M <= 2) gemv_direct_kernel<2><<<grid, D_THREADS, 0, stream>>>(p);
    else if (p.M <= 4) gemv_direct_kernel<4><<<grid, D_THREADS, 0, stream>>>(p);
    else gemv_direct_kernel<MAX_M><<<grid, D_THREADS, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace gemv
}  // namespace b2
