// graph_kernels.h -- launchers of the graph's non-Linear node kernels (graph_kernels.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>

namespace b2 {
namespace graph {

enum EwOp : int { EW_ADD = 0, EW_MUL = 1, EW_SILU = 2, EW_GELU = 3, EW_HSIG = 4 };

// Every FP16 matrix here is row-major with a pitch (elements) that is a multiple of 8 and a
// 16-byte aligned base, so rows are read and written as 16-byte vectors.
struct EwParams {
    int op, rows, cols;
    const __half *a; long long lda;
    const __half *b; long long ldb;      // ADD / MUL only
    __half *y; long long ldy;
    const __half *gate_table;            // SILU / GELU: the gate of every FP16 input
    unsigned *flags;
};

struct NormParams {
    int rows, cols;
    const __half *x; long long ldx;
    const __half *gamma;                 // [cols]
    float eps;
    __half *y; long long ldy;
    unsigned *flags;
};

struct GatedParams {
    int rows, gate_n, act;
    const __half *src; long long lds;    // folded FP16 sums, packed gate|up 64-column blocks
    const __half *bias_gate, *bias_up;   // [gate_n] or nullptr
    __half *y; long long ldy;
    const __half *gate_table;
    unsigned *flags;
};

cudaError_t elementwise(const EwParams &p, cudaStream_t s, int sm_count);
cudaError_t rmsnorm(const NormParams &p, cudaStream_t s, int sm_count);
cudaError_t gated_combine(const GatedParams &p, cudaStream_t s, int sm_count);
// Fills table[GATE_TABLE_ENTRIES] (common.cuh) with gate16 of every FP16 input, both activations.
cudaError_t fill_gate_table(__half *table, cudaStream_t s);

}  // namespace graph
}  // namespace b2
