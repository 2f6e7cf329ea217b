// aux_kernels.h -- launchers of the auxiliary kernels (aux_kernels.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>

namespace b2 {
namespace aux {

constexpr unsigned MAX_TILES = 64;   // tiles per launch (kept in the kernel parameters)

struct CubeTile {
    void *ptr;
    unsigned rows, cols, physical_rows, physical_cols, row0, col0;
};
struct CubeTiles {
    CubeTile tile[MAX_TILES];
    unsigned count;
};
struct GuardList {
    const void *base[MAX_TILES];
    size_t payload[MAX_TILES];
    unsigned count;
};
struct EpilogueParams {
    int M, N;
    const float *partial; long long ldp;   // FP32 source, or nullptr: in place on y (FP16 run)
    const __half *bias;
    __half *y; long long ldy;
    int post;
    unsigned *flags;
};

cudaError_t scan_nonfinite(const void *p, size_t rows, size_t cols, size_t ld, unsigned *flags, int flag,
                           cudaStream_t s, int sm_count);
cudaError_t cube_gather(const CubeTiles &t, void *dst, size_t ld, cudaStream_t s, int sm_count);
cudaError_t cube_scatter(const void *src, size_t ld, const CubeTiles &t, cudaStream_t s, int sm_count);
cudaError_t guard_check(const GuardList &g, size_t slack, size_t guard, unsigned *flags, cudaStream_t s);
cudaError_t epilogue(const EpilogueParams &p, cudaStream_t s, int sm_count);

}  // namespace aux
}  // namespace b2
