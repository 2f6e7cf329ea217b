// graph_kernels.cu -- the static graph's node kernels other than Linear (sm_100a).
//
// They replace the NPU programs research/custom-ops/src/co_graph.c:293-313 emits per 256x256
// tile and the hybrid row operator of co_row_ops.c:150-224:
//   elementwise    ADD / MUL: y = fp16(a op b) (co_emit_ew); HSIG: fp16(hsig(a)) (co_emit_lut);
//                  SILU / GELU: y = fp16(a * fp16(gate(a))) (a LUT pass into a gate buffer, then
//                  co_emit_ew multiply), the gate read from the handle's table of every FP16 input
//                  (fill_gate_table: common.cuh's double-precision gate16, once per handle). One
//                  FP32 operation on two FP16 values rounded once to FP16
//                  is the correctly rounded FP16 result (24 >= 2*11 + 2 bits), so these match the
//                  reference's double-precision restatement bit for bit.
//   rmsnorm        per row: each 256-column tile's sum of FP16 squares fp16(x*x), summed exactly
//                  (64-bit fixed point: every FP16 square is a multiple of 2^-24 below 2^16) and
//                  rounded once to FP32 -- the NPU's FP32 matmul-with-ones statistic; a tile sum
//                  >= 65504 or not finite rejects the row (co_row_ops.c:190-195); the tile sums are
//                  added in double, coefficient c_j = fp16(gamma_j / sqrt(sum / cols + eps)) in
//                  double (co_row_ops.c:207-211), a non-finite coefficient rejects the row, and
//                  y = fp16(x * c). A rejected row raises the non-finite-input status (the
//                  reference's ROCKET_E_SHAPE; the run then publishes nothing).
//   gated_combine  the gate·up product of a packed gate|up Linear whose FP16 sums were written
//                  unfinished (small M, or the unfused arm): the same arithmetic as the GEMM's
//                  fused gated epilogue.
// One thread handles 8 consecutive columns (one 16-byte vector); grids are sized in multiples of
// the SM count. All are HBM-bound: the traffic is the bytes read plus the bytes written.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "graph_kernels.h"

namespace b2 {
namespace graph {

constexpr int THREADS = 256;

static unsigned grid_cap(size_t work, int sm_count, int per_sm) {
    const size_t blocks = (work + THREADS - 1) / THREADS;
    const size_t cap = (size_t)sm_count * per_sm;
    return (unsigned)(blocks < 1 ? 1 : (blocks < cap ? blocks : cap));
}

__device__ __forceinline__ void unpack8(const uint4 &u, float (&f)[8]) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float2 t = __half22float2(h[e]);
        f[2 * e] = t.x;
        f[2 * e + 1] = t.y;
    }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
    uint4 u;
    __half2 *h = reinterpret_cast<__half2 *>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(f[2 * e], f[2 * e + 1]);
    return u;
}

// Stores 8 results at columns [c, c+8) of a row, clipped at n (the pitch padding stays untouched).
__device__ __forceinline__ void store8(__half *row, int c, int n, const float (&f)[8]) {
    if (c + 8 <= n) {
        *reinterpret_cast<uint4 *>(row + c) = pack8(f);
    } else {
#pragma unroll
        for (int e = 0; e < 8; ++e)
            if (c + e < n) row[c + e] = __float2half_rn(f[e]);
    }
}

// ----------------------------------------------------------------------------- elementwise
template <int OP>
__global__ void __launch_bounds__(THREADS) ew_kernel(EwParams p) {
    const int groups = (p.cols + 7) / 8;
    const long long total = (long long)p.rows * groups;
    bool bad = false;
    for (long long i = (long long)blockIdx.x * THREADS + threadIdx.x; i < total; i += (long long)gridDim.x * THREADS) {
        const int r = (int)(i / groups), c = (int)(i % groups) * 8;
        // a full vector is inside the row's pitch even when it crosses `cols`
        float a[8], y[8];
        unpack8(__ldg(reinterpret_cast<const uint4 *>(p.a + (size_t)r * p.lda + c)), a);
        if constexpr (OP == EW_ADD || OP == EW_MUL) {
            float b[8];
            unpack8(__ldg(reinterpret_cast<const uint4 *>(p.b + (size_t)r * p.ldb + c)), b);
#pragma unroll
            for (int e = 0; e < 8; ++e) y[e] = OP == EW_ADD ? __fadd_rn(a[e], b[e]) : __fmul_rn(a[e], b[e]);
        } else if constexpr (OP == EW_HSIG) {
#pragma unroll
            for (int e = 0; e < 8; ++e) y[e] = hsig(a[e]);
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) y[e] = gated_act16(p.gate_table, a[e], OP == EW_GELU ? GATE_GELU : GATE_SIGMOID);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e)
            if (c + e < p.cols) bad |= f16_overflows(y[e]);
        store8(p.y + (size_t)r * p.ldy, c, p.cols, y);
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) raise_flag(p.flags, FLAG_NONFINITE_OUTPUT);
}

cudaError_t elementwise(const EwParams &p, cudaStream_t s, int sm_count) {
    if (p.rows <= 0 || p.cols <= 0) return cudaSuccess;
    const unsigned grid = grid_cap((size_t)p.rows * ((p.cols + 7) / 8), sm_count, 8);
    switch (p.op) {
        case EW_ADD: ew_kernel<EW_ADD><<<grid, THREADS, 0, s>>>(p); break;
        case EW_MUL: ew_kernel<EW_MUL><<<grid, THREADS, 0, s>>>(p); break;
        case EW_SILU: ew_kernel<EW_SILU><<<grid, THREADS, 0, s>>>(p); break;
        case EW_GELU: ew_kernel<EW_GELU><<<grid, THREADS, 0, s>>>(p); break;
        case EW_HSIG: ew_kernel<EW_HSIG><<<grid, THREADS, 0, s>>>(p); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

// ----------------------------------------------------------------------------- gated combine
// Thread (row r, hidden columns [j, j+8)): gate sums at packed columns 64*(j/32) + j%32 + e, up sums
// 32 columns further; each is finished with its own bias like the Linear epilogue (fp16(run + b)
// when the half has a bias), then y = fp16(fp16(g * fp16(gate(g))) * u).
// The biases of columns [j, j + 8) as FP32 (zero past n or without a bias): one 16-byte load when
// the 8 columns are inside n and 16-byte aligned, else element loads.
__device__ __forceinline__ void bias8(const __half *b, int j, int n, float (&out)[8]) {
    if (b && j + 8 <= n && (reinterpret_cast<uintptr_t>(b + j) & 15) == 0) {
        unpack8(__ldg(reinterpret_cast<const uint4 *>(b + j)), out);
        return;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) out[e] = (b && j + e < n) ? __half2float(b[j + e]) : 0.0f;
}

__global__ void __launch_bounds__(THREADS) gated_kernel(GatedParams p) {
    const int groups = (p.gate_n + 7) / 8;
    const long long total = (long long)p.rows * groups;
    bool bad = false;
    for (long long i = (long long)blockIdx.x * THREADS + threadIdx.x; i < total; i += (long long)gridDim.x * THREADS) {
        const int r = (int)(i / groups), j = (int)(i % groups) * 8;
        const __half *row = p.src + (size_t)r * p.lds + 64 * (j >> 5) + (j & 31);
        float g[8], u[8], y[8], bgv[8], buv[8];
        unpack8(__ldg(reinterpret_cast<const uint4 *>(row)), g);
        unpack8(__ldg(reinterpret_cast<const uint4 *>(row + 32)), u);
        bias8(p.bias_gate, j, p.gate_n, bgv);
        bias8(p.bias_up, j, p.gate_n, buv);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const bool in = j + e < p.gate_n;
            const float bg = bgv[e], bu = buv[e];
            const float gv = finish_tile16(g[e], bg, p.bias_gate != nullptr, false);
            const float uv = finish_tile16(u[e], bu, p.bias_up != nullptr, false);
            y[e] = gated16(p.gate_table, gv, uv, p.act);
            if (in) bad |= f16_overflows(y[e]);
        }
        store8(p.y + (size_t)r * p.ldy, j, p.gate_n, y);
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) raise_flag(p.flags, FLAG_NONFINITE_OUTPUT);
}

cudaError_t gated_combine(const GatedParams &p, cudaStream_t s, int sm_count) {
    if (p.rows <= 0 || p.gate_n <= 0) return cudaSuccess;
    if (p.act != GATE_SIGMOID && p.act != GATE_GELU) return cudaErrorInvalidValue;
    gated_kernel<<<grid_cap((size_t)p.rows * ((p.gate_n + 7) / 8), sm_count, 8), THREADS, 0, s>>>(p);
    return cudaGetLastError();
}

// ----------------------------------------------------------------------------- gate table
__global__ void __launch_bounds__(THREADS) gate_table_kernel(__half *table) {
    const int i = blockIdx.x * THREADS + threadIdx.x;
    if (i >= GATE_TABLE_ENTRIES) return;
    const float a = __half2float(__ushort_as_half((unsigned short)(i & 0xffff)));
    table[i] = __float2half_rn(gate16(a, i < 65536 ? GATE_SIGMOID : GATE_GELU));   // exact: already FP16
}

cudaError_t fill_gate_table(__half *table, cudaStream_t s) {
    gate_table_kernel<<<(GATE_TABLE_ENTRIES + THREADS - 1) / THREADS, THREADS, 0, s>>>(table);
    return cudaGetLastError();
}

// ----------------------------------------------------------------------------- rmsnorm
// One warp per row. A 256-column tile is exactly one 8-column vector per lane, so each tile's
// statistic is one warp reduction of 64-bit integers (exact) in units of 2^-24.
__global__ void __launch_bounds__(THREADS) rmsnorm_kernel(NormParams p) {
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (THREADS / 32);
    const int tiles = (p.cols + 255) / 256;
    bool rejected = false;
    for (int r = blockIdx.x * (THREADS / 32) + (threadIdx.x >> 5); r < p.rows; r += warps) {
        const __half *xr = p.x + (size_t)r * p.ldx;
        double sum = 0.0;
        bool bad = false;
        for (int t = 0; t < tiles; ++t) {
            const int c = t * 256 + lane * 8;
            long long q = 0;
            if (c < p.cols) {
                float x[8];
                unpack8(__ldg(reinterpret_cast<const uint4 *>(xr + c)), x);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    if (c + e >= p.cols) continue;
                    const float s = round16(__fmul_rn(x[e], x[e]));
                    if (f16_overflows(s)) bad = true;                          // an infinite square
                    else q += __float2ll_rn(__fmul_rn(s, 16777216.0f));         // exact: s * 2^24
                }
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
            const float stat = __fmul_rn(__ll2float_rn(q), 5.9604644775390625e-8f);   // RN(q) * 2^-24
            if (!(stat < 65504.0f)) bad = true;
            sum += (double)stat;
        }
        bad = __any_sync(0xffffffffu, bad);
        if (!bad) {
            const double scale = sqrt(sum / (double)p.cols + (double)p.eps);
            for (int c = lane * 8; c < p.cols && !bad; c += 256) {
                float x[8], y[8];
                unpack8(__ldg(reinterpret_cast<const uint4 *>(xr + c)), x);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float g = c + e < p.cols ? __half2float(p.gamma[c + e]) : 0.0f;
                    const float coeff = round16_from_double((double)g / scale);
                    if (c + e < p.cols && f16_overflows(coeff)) bad = true;
                    y[e] = round16(__fmul_rn(x[e], coeff));
                }
                if (!bad) store8(p.y + (size_t)r * p.ldy, c, p.cols, y);
            }
            bad = __any_sync(0xffffffffu, bad);
        }
        rejected |= bad;
    }
    if (rejected && lane == 0) raise_flag(p.flags, FLAG_NONFINITE_INPUT);
}

cudaError_t rmsnorm(const NormParams &p, cudaStream_t s, int sm_count) {
    if (p.rows <= 0 || p.cols <= 0) return cudaSuccess;
    const size_t blocks = ((size_t)p.rows + THREADS / 32 - 1) / (THREADS / 32);
    const size_t cap = (size_t)sm_count * 8;
    rmsnorm_kernel<<<(unsigned)(blocks < cap ? blocks : cap), THREADS, 0, s>>>(p);
    return cudaGetLastError();
}

}  // namespace graph
}  // namespace b2
