// common.cuh -- device helpers shared by the sm_100a kernels of the Linear path.
//
// Epilogue arithmetic (one definition, used by the fused GEMM/GEMV epilogues and by the separate
// epilogue kernel, so CO_CHAIN and CO_SEPARATE runs give identical bytes):
//   per-256-K fold   run = fp16(chunk) for the first K tile, run = fp16(run + chunk) afterwards
//                    (research/custom-ops/src/linear_hardsigmoid.c:51-62, co_emit_mm/_acc)
//   tile-16 finish   affine = bias ? fp16(run + b) : run;  y = post ? fp16(hsig(affine)) : affine
//                    (linear_hardsigmoid.c:63-79, co_emit_ew bias then co_emit_lut HardSigmoid)
//   FP32 finish      y = fp16(post ? hsig(acc + b) : acc + b), single rounding
//   hsig(v)          clamp(v / 6 + 0.5, 0, 1): the function the reference's 513-entry LUT
//                    samples (research/custom-ops/src/custom_ops.c:357-369), evaluated in FP32
//                    instead of an interpolated Q0.15 table. v / 6 is the correctly rounded
//                    quotient, obtained with Markstein's division-by-constant step: q = v * RN(1/6),
//                    r = v - 6q exactly (one FMA), q' = q + r * RN(1/6) (one FMA) -- three flops
//                    instead of a full division, checked against IEEE division on all FP32 inputs.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace b2 {

// Status flag slots (host-mapped pinned memory; one word per kind, written with plain stores so
// no system-scope atomics are needed). Host side maps them to the B2_STATUS_* bits.
// FLAG_SCAN_OUTPUT: a finiteness scan of a caller-visible result (the graph's outputs) found a
// non-finite value; kept apart from FLAG_NONFINITE_OUTPUT, which any kernel raises on an overflow.
enum : int { FLAG_TIMEOUT = 0, FLAG_NONFINITE_OUTPUT = 1, FLAG_NONFINITE_INPUT = 2, FLAG_GUARD = 3,
             FLAG_SCAN_OUTPUT = 4, FLAG_COUNT = 5 };

__device__ __forceinline__ void raise_flag(unsigned *flags, int idx) {
    volatile unsigned *p = flags + idx;
    *p = 1u;
    __threadfence_system();
}

// Correctly rounded v / 6 (Markstein: one exact remainder, one corrective FMA).
__device__ __forceinline__ float div6(float v) {
    const float y = 0.16666667f;          // RN(1/6) = 0x3E2AAAAB
    const float q = __fmul_rn(v, y);
    const float r = __fmaf_rn(-q, 6.0f, v);
    return __fmaf_rn(r, y, q);
}

// clamp(v/6 + 0.5, 0, 1). Exactly 1 for v >= 3 and 0 for v <= -3 (this also covers infinities,
// for which the remainder step of div6 is undefined); NaN gives 0 like fmax(0, NaN).
__device__ __forceinline__ float hsig(float v) {
    if (v >= 3.0f) return 1.0f;
    if (v <= -3.0f) return 0.0f;
    const float r = __fadd_rn(div6(v), 0.5f);
    return fminf(fmaxf(r, 0.0f), 1.0f);
}

// True if v does not round to a finite FP16 (NaN or |v| >= 65520).
__device__ __forceinline__ bool f16_overflows(float v) { return !(fabsf(v) < 65520.0f); }

__device__ __forceinline__ float round16(float v) { return __half2float(__float2half_rn(v)); }

// One fold step of the reference's per-K-tile FP16 running sum.
__device__ __forceinline__ float fold16(float run, float chunk, bool first) {
    return first ? round16(chunk) : round16(__fadd_rn(run, chunk));
}

__device__ __forceinline__ float finish_tile16(float run, float b, bool has_bias, bool post) {
    float a = has_bias ? round16(__fadd_rn(run, b)) : run;
    return post ? hsig(a) : a;
}

__device__ __forceinline__ float finish_fp32(float acc, float b, bool post) {
    float a = __fadd_rn(acc, b);
    return post ? hsig(a) : a;
}

__device__ __forceinline__ bool half_nonfinite(__half h) {
    return (__half_as_ushort(h) & 0x7c00u) == 0x7c00u;
}

// Activation gates of the graph's SiLU / GELU nodes (research/custom-ops/src/co_graph.c:303-307:
// a LUT pass x -> gate, then an elementwise multiply x * gate). The reference's 513-entry LUTs
// sample these functions (custom_ops.c:357-369); here each FP16 input gets the function itself,
// evaluated in double and rounded once to FP16:
//   GATE_SIGMOID  1 / (1 + exp(-a))
//   GATE_GELU     0.5 * (1 + erf(a / sqrt 2))
enum : int { GATE_SIGMOID = 1, GATE_GELU = 2 };

__device__ __forceinline__ float round16_from_double(double g) {
    unsigned short h;
    asm("cvt.rn.f16.f64 %0, %1;" : "=h"(h) : "d"(g));
    return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ float gate16(float a, int act) {
    const double v = (double)a;
    const double g = act == GATE_GELU ? 0.5 * (1.0 + erf(v / 1.4142135623730951)) : 1.0 / (1.0 + exp(-v));
    return round16_from_double(g);
}

// The kernels read the gate of an FP16 input from a table of all 65536 inputs, one per activation
// (GATE_SIGMOID at [0, 65536), GATE_GELU at [65536, 131072)), filled once per device handle with
// gate16 itself: the same bits as evaluating it, without double-precision math per element.
constexpr int GATE_TABLE_ENTRIES = 2 * 65536;

__device__ __forceinline__ float gate16_lut(const __half *table, float a, int act) {
    const unsigned idx = (unsigned)__half_as_ushort(__float2half_rn(a)) + (act == GATE_GELU ? 65536u : 0u);
    return __half2float(__ldg(table + idx));
}

// SiLU / GELU node value of an FP16 a: fp16(a * fp16(gate(a))).
__device__ __forceinline__ float gated_act16(const __half *table, float a, int act) {
    return round16(__fmul_rn(a, gate16_lut(table, a, act)));
}

// The fused gate·up product: fp16(act16(g) * u) for FP16 g, u (the graph's MUL node).
__device__ __forceinline__ float gated16(const __half *table, float g, float u, int act) {
    return round16(__fmul_rn(gated_act16(table, g, act), u));
}

}  // namespace b2
