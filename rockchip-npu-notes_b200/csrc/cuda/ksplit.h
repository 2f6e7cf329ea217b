// ksplit.h -- signal and reduce launches of the fused K-split (ksplit.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace b2 {
namespace ksplit {

constexpr int MAX_WORLD = 8;
constexpr size_t FLAGS_OFFSET = 0;      // [64] round words, one per rank
constexpr size_t SEQ_OFFSET = 256;      // this rank's round counter
constexpr size_t PLANES_OFFSET = 512;   // [2][world][rows_per_rank][ldp] FP32 in 32-row panels

struct SignalParams {
    unsigned *seq;                      // this rank's counter
    unsigned *peer_flag[MAX_WORLD];     // rank q's flag word for this rank (q = 0..world-1)
    int world;
};

struct ReduceParams {
    const unsigned *seq;                // this rank's counter (already advanced by the signal)
    const unsigned *flags;              // this rank's flag words, [world]
    const float *planes;                // this rank's two parity planes
    long long plane_floats;
    int world, rows_per_rank, rows;     // rows: the owned rows of this round (<= rows_per_rank)
    int n;
    long long ldp;
    int vec;                            // Y rows are 16-byte aligned with ldy % 8 == 0
    const __half *bias;                 // [n] or nullptr
    int post;
    __half *y;                          // first owned row of Y
    long long ldy;
    unsigned *status;
};

cudaError_t signal(const SignalParams &p, cudaStream_t stream);
cudaError_t reduce(const ReduceParams &p, cudaStream_t stream, int sm_count);

}  // namespace ksplit
}  // namespace b2
