// gemv.h -- parameters and launcher of the small-M kernel (gemv.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace b2 {
namespace gemv {

constexpr int MAX_M = 8;
enum OutMode : int { OUT_FINAL = 0, OUT_RAW16 = 1, OUT_RAW32 = 2 };

struct Params {
    int M, N, K;
    const __half *x; long long ldx;     // [M, ldx], 16-byte aligned rows
    const __half *w; long long ldw;     // [N, ldw], 16-byte aligned rows
    const __half *bias;                 // [N] or nullptr
    __half *y; long long ldy;
    float *partial; long long ldp;
    int out_mode, post, fold;
    unsigned *flags;
};

cudaError_t launch(const Params &p, cudaStream_t stream, int sm_count, unsigned *grid_out);
unsigned grid_for(int N, int sm_count);

}  // namespace gemv
}  // namespace b2
