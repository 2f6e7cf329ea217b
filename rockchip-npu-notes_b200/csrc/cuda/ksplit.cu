// ksplit.cu -- fused K-split across GPUs: GEMM partials routed to their owner over NVLink, a
// round signal, and the owner's reduction + bias/activation epilogue.
//
// The reference accumulates K slices on one NPU through FP16 ping-pong partials
// (research/custom-ops/src/custom_ops.c:297-330). Across B200s each rank r holds X[:, Kr] and
// W[:, Kr] and computes the FP32 partial X_r W_r^T; output row block q (rows [q*R, (q+1)*R)) is
// owned by rank q. One round is three launches on the rank's stream:
//   1. the tcgen05 GEMM in raw-FP32 mode with routed output: its epilogue stores row block q of
//      the partial straight into rank q's receive buffer (plain stores through a CUDA IPC mapping,
//      no TMA), slot r of parity plane (round & 1), overlapping the transfer with later tiles'
//      MMAs; then a system-scope fence;
//   2. signal (one thread): round = ++seq; store `round` into every rank's flag word [r];
//   3. reduce: wait (bounded) until every rank's flag word for this rank has reached `round`, then
//      y = fp16(act(sum over ranks q = 0..world-1 of slot q + b)) for the owned rows (FP32 adds in
//      rank order, so every run gives the same bits).
// Two parity planes keep a fast rank from overwriting data its owner is still reducing: rank q can
// only start round n+2 after its own round-n+1 reduce, which waited for this rank's round-n+1
// signal, which follows this rank's round-n reduce on its stream.
//
// Buffer of each rank (one cudaMalloc, exported by CUDA IPC): [flags: 64 words][seq][pad] at 0,
// the planes at PLANES_OFFSET: [2][world][R][ldp] FP32, each [R][ldp] slot in 32-row panels
// stored column by column (element (r, c) at (r/32)*32*ldp + c*32 + r%32; R is a multiple of 32)
// so that the GEMM's stores and the reduction's loads are whole 128-byte lines.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "ksplit.h"
#include "mbarrier.cuh"

namespace b2 {
namespace ksplit {

namespace {

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void signal_kernel(SignalParams p) {
    unsigned *seq = p.seq;
    const unsigned round = *seq + 1u;
    *seq = round;
    __threadfence_system();
    for (int q = 0; q < p.world; ++q) st_release_sys(p.peer_flag[q], round);
}

constexpr int THREADS = 256;

__global__ void __launch_bounds__(THREADS) reduce_kernel(ReduceParams p) {
    __shared__ int ok;
    __shared__ unsigned round;
    if (threadIdx.x == 0) {
        const unsigned target = *reinterpret_cast<const volatile unsigned *>(p.seq);
        int good = 1;
        for (int q = 0; q < p.world && good; ++q) {
            const uint64_t t0 = global_ns();
            while ((int)(ld_acquire_sys(p.flags + q) - target) < 0) {
                if (global_ns() - t0 > WAIT_LIMIT_NS) {   // a rank never signalled this round
                    raise_flag(p.status, FLAG_TIMEOUT);
                    good = 0;
                    break;
                }
            }
        }
        ok = good;
        round = target;
    }
    __syncthreads();
    if (!ok) return;
    const float *plane = p.planes + (size_t)(round & 1u) * p.plane_floats;
    const size_t slot = (size_t)p.rows_per_rank * p.ldp;
    const bool has_bias = p.bias != nullptr;
    bool bad = false;
    // Thread (row r, 8 columns from c0): consecutive threads take consecutive rows of a 32-row
    // panel, so every load (one column of 32 rows) is one 128-byte line; each thread writes 16
    // bytes of its Y row.
    const int groups = (p.n + 7) / 8;
    const int panels = (p.rows + 31) / 32;
    const long long total = (long long)panels * groups * 32;
    for (long long i = blockIdx.x * (long long)THREADS + threadIdx.x; i < total; i += (long long)gridDim.x * THREADS) {
        const int lane = (int)(i & 31);
        const long long pg = i >> 5;
        const int g = (int)(pg % groups), panel = (int)(pg / groups);
        const int r = panel * 32 + lane, c0 = g * 8;
        if (r >= p.rows) continue;
        const float *src = plane + (size_t)panel * 32 * p.ldp + (size_t)c0 * 32 + lane;
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            if (c0 + e >= p.n) { v[e] = 0.0f; continue; }
            float s = __ldcg(src + e * 32);
            for (int q = 1; q < p.world; ++q) s += __ldcg(src + q * slot + e * 32);
            v[e] = s;
        }
        __half h[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float b = (has_bias && c0 + e < p.n) ? __half2float(p.bias[c0 + e]) : 0.0f;
            h[e] = __float2half_rn(finish_fp32(v[e], b, p.post));
            if (c0 + e < p.n) bad |= half_nonfinite(h[e]);
        }
        __half *yrow = p.y + (size_t)r * p.ldy + c0;
        if (c0 + 8 <= p.n && p.vec) {
            *reinterpret_cast<uint4 *>(yrow) = *reinterpret_cast<const uint4 *>(h);
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e)
                if (c0 + e < p.n) yrow[e] = h[e];
        }
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) raise_flag(p.status, FLAG_NONFINITE_OUTPUT);
}

}  // namespace

cudaError_t signal(const SignalParams &p, cudaStream_t stream) {
    if (p.world < 1 || p.world > MAX_WORLD) return cudaErrorInvalidValue;
    signal_kernel<<<1, 1, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t reduce(const ReduceParams &p, cudaStream_t stream, int sm_count) {
    if (p.world < 1 || p.world > MAX_WORLD || p.rows < 0 || p.n < 1 || p.rows_per_rank % 32) return cudaErrorInvalidValue;
    if (p.rows == 0) return cudaSuccess;
    const long long work = (long long)((p.rows + 31) / 32) * ((p.n + 7) / 8) * 32;
    long long blocks = (work + THREADS - 1) / THREADS;
    // every block waits for the flags on its own: keep the grid resident in one wave, so a rank that
    // never signals costs one wait limit, not one per wave
    const long long cap = (long long)sm_count * 4;
    if (blocks > cap) blocks = cap;
    reduce_kernel<<<(unsigned)blocks, THREADS, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace ksplit
}  // namespace b2
