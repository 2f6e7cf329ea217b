// gemv.cu -- memory-bound small-M Linear (M <= 8): y[r, n] = act(x[r, :] . W[n, :] + b[n]).
//
// The reference runs M=1 decode through the same NPU matmul with the row count padded to 12
// (research/scheduling/GEMM-GEMV-CONCURRENCY.md:24-30 in the reference project); on B200 the
// M<=8 case is a weight stream: each warp owns one W row at a time and every lane reads 16 bytes
// (8 FP16) per 256-element K tile with read-only, L1-bypassing loads, so one K tile of the
// reference's FP16-K-TILING scheme is exactly one load per lane. The x rows are re-read from
// L1/L2 (tiny). Per-tile FP16 folding (tile-16 mode) reduces each tile across the warp with
// shuffles before the fold; FP32 mode reduces once per row. Several tiles' loads are issued
// before any arithmetic to keep enough bytes in flight to saturate HBM.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "gemv.h"

namespace b2 {
namespace gemv {

constexpr int THREADS = 256;
constexpr int UNROLL = 4;

__device__ __forceinline__ uint4 ld_stream(const __half *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Dot product of 8 FP16 pairs; elements at index >= valid contribute nothing.
__device__ __forceinline__ float dot8(uint4 a, uint4 b, int valid) {
    const __half2 *ha = reinterpret_cast<const __half2 *>(&a);
    const __half2 *hb = reinterpret_cast<const __half2 *>(&b);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 fa = __half22float2(ha[i]), fb = __half22float2(hb[i]);
        if (2 * i < valid) s = fmaf(fa.x, fb.x, s);
        if (2 * i + 1 < valid) s = fmaf(fa.y, fb.y, s);
    }
    return s;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <int MR>
__global__ void __launch_bounds__(THREADS) gemv_kernel(const Params p) {
    const int lane = threadIdx.x & 31;
    const int warps = (gridDim.x * THREADS) >> 5;
    const int nchunk = (p.K + 255) >> 8;
    const bool has_bias = p.bias != nullptr;
    bool bad = false;
    for (int n = (blockIdx.x * THREADS + threadIdx.x) >> 5; n < p.N; n += warps) {
        const __half *wrow = p.w + (size_t)n * p.ldw;
        float acc[MR], run[MR];
#pragma unroll
        for (int r = 0; r < MR; ++r) acc[r] = run[r] = 0.0f;
        for (int c0 = 0; c0 < nchunk; c0 += UNROLL) {
            uint4 wv[UNROLL];
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                const int k8 = (c0 + u) * 256 + lane * 8;
                wv[u] = (c0 + u < nchunk && k8 < p.K) ? ld_stream(wrow + k8) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                const int c = c0 + u;
                if (c >= nchunk) break;                       // uniform across the warp
                const int k8 = c * 256 + lane * 8;
                const int valid = k8 < p.K ? min(8, p.K - k8) : 0;
#pragma unroll
                for (int r = 0; r < MR; ++r) {
                    if (r >= p.M) break;
                    const uint4 xv = valid ? __ldg(reinterpret_cast<const uint4 *>(p.x + (size_t)r * p.ldx + k8))
                                           : make_uint4(0, 0, 0, 0);
                    const float s = dot8(wv[u], xv, valid);
                    if (p.fold) run[r] = fold16(run[r], warp_sum(s), c == 0);
                    else acc[r] += s;
                }
            }
        }
        const float b = has_bias ? __half2float(p.bias[n]) : 0.0f;
#pragma unroll
        for (int r = 0; r < MR; ++r) {
            if (r >= p.M) break;
            const float total = p.fold ? run[r] : warp_sum(acc[r]);
            if (lane != r) continue;
            if (p.out_mode == OUT_RAW32) {
                p.partial[(size_t)r * p.ldp + n] = total;
            } else if (p.out_mode == OUT_RAW16) {
                p.y[(size_t)r * p.ldy + n] = __float2half_rn(total);
            } else {
                const float v = p.fold ? finish_tile16(total, b, has_bias, p.post) : finish_fp32(total, b, p.post);
                const __half h = __float2half_rn(v);
                bad |= half_nonfinite(h);
                p.y[(size_t)r * p.ldy + n] = h;
            }
        }
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) raise_flag(p.flags, FLAG_NONFINITE_OUTPUT);
}

unsigned grid_for(int N, int sm_count) {
    const long long need = ((long long)N + (THREADS / 32) - 1) / (THREADS / 32);
    const long long cap = (long long)sm_count * 8;
    return (unsigned)(need < cap ? need : cap);
}

cudaError_t launch(const Params &p, cudaStream_t stream, int sm_count, unsigned *grid_out) {
    const unsigned grid = grid_for(p.N, sm_count);
    if (grid_out) *grid_out = grid;
    if (p.M <= 1) gemv_kernel<1><<<grid, THREADS, 0, stream>>>(p);
    else if (p.M <= 2) gemv_kernel<2><<<grid, THREADS, 0, stream>>>(p);
    else if (p.M <= 4) gemv_kernel<4><<<grid, THREADS, 0, stream>>>(p);
    else if (p.M <= MAX_M) gemv_kernel<MAX_M><<<grid, THREADS, 0, stream>>>(p);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

}  // namespace gemv
}  // namespace b2
