// gemv.h -- parameters and launchers of the small-M kernels (gemv.cu).
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

// Bulk-copy streamed kernel: one launch serves up to GROUP_MAX independent projections that share
// the row count M (for example the Q/K/V or gate/up projections of one decoder layer).
constexpr int GROUP_MAX = 16;
constexpr int STREAM_MAX_M = 8;         // x rows: the n8 dimension of the m16n8k16 MMA
constexpr int STREAM_MAX_K = 2048;      // 8 x rows of 2048 fill the 32 KB x table
constexpr int STREAM_X_BYTES = 32768;   // shared-memory table of the launch's distinct x rows

struct Problem {
    const __half *x; long long ldx;
    const __half *w; long long ldw;
    const __half *bias;
    __half *y; long long ldy;
    float *partial; long long ldp;
    int N, K, out_mode, post, fold;
    int rows_per_unit, unit_begin;      // filled in by launch_group
    int x_off;                          // element offset of this problem's x rows in the x table
    int pad;
};

// One distinct x (problems that share x and K share the entry): M rows of K, pitch ldx in
// global memory, stored with pitch round8(K) from element `off` of the table.
struct XSource {
    const __half *x; long long ldx;
    int K, off;
};

struct Group {
    Problem prob[GROUP_MAX];
    XSource xsrc[GROUP_MAX];
    int count, M, units, nx;
    unsigned *flags;
};

// True when the streamed kernel serves this shape (M <= 8, K <= 2048).
bool streamed(int M, int K);

// Picks the kernel for p (streamed when eligible, else the per-lane-load kernel) and launches it.
cudaError_t launch(const Params &p, cudaStream_t stream, int sm_count, unsigned *grid_out);
// Runs the launchers' one-time device setup (shared-memory limits, occupancy queries) now, so that
// a later launch issues no such call (a launch recorded into a CUDA graph must not).
cudaError_t prepare();
// Launches the streamed kernel over g.count problems (each must satisfy streamed(g.M, K)): one
// launch, or more when the problems' distinct x rows exceed the x table (*launches gets the count).
cudaError_t launch_group(Group &g, cudaStream_t stream, int sm_count, unsigned *grid_out, unsigned *launches);
unsigned grid_for(int M, int N, int K, long long ldw, int sm_count);

}  // namespace gemv
}  // namespace b2
