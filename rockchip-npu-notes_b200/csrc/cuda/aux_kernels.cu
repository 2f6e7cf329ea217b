// aux_kernels.cu -- the small HBM-bound kernels around the GEMM.
//
//   scan_nonfinite   finiteness of the host entry's X after upload (the reference rejects
//                    non-finite inputs with ROCKET_E_SHAPE before any work:
//                    research/custom-ops/src/linear_hardsigmoid.c:174,255)
//   cube_gather      C2=8 cube tiles -> row-major staging (device-cube entries; the layout is
//   cube_scatter     research/custom-ops/src/custom_ops.c:80-85) and row-major -> cube tiles
//   guard_check      slack/guard integrity of caller buffers (custom_ops.c:196-221)
//   epilogue         bias + HardSigmoid on an FP32 partial or, in place, on the folded FP16 sum:
//                    the separate (unfused) arm of the reference's CO_SEPARATE mode
// Each kernel reads and writes with 16-byte accesses where the layout allows and sizes its grid
// in multiples of the SM count.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "aux_kernels.h"
#include "common.cuh"

namespace b2 {
namespace aux {

constexpr int THREADS = 256;

static unsigned grid_cap(size_t work, int sm_count, int per_sm) {
    const size_t blocks = (work + THREADS - 1) / THREADS;
    const size_t cap = (size_t)sm_count * per_sm;
    return (unsigned)(blocks < 1 ? 1 : (blocks < cap ? blocks : cap));
}

// ----------------------------------------------------------------------------- finiteness scan
__global__ void __launch_bounds__(THREADS) scan_kernel(const __half *p, size_t rows, size_t cols, size_t ld,
                                                       unsigned *flags, int flag) {
    const size_t vecs_per_row = (cols + 7) / 8;
    const size_t total = rows * vecs_per_row;
    bool bad = false;
    for (size_t i = (size_t)blockIdx.x * THREADS + threadIdx.x; i < total; i += (size_t)gridDim.x * THREADS) {
        const size_t r = i / vecs_per_row, c = (i % vecs_per_row) * 8;
        const uint4 v = __ldg(reinterpret_cast<const uint4 *>(p + r * ld + c));
        const uint16_t *h = reinterpret_cast<const uint16_t *>(&v);
#pragma unroll
        for (int e = 0; e < 8; ++e)
            if (c + e < cols && (h[e] & 0x7c00u) == 0x7c00u) bad = true;
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) raise_flag(flags, flag);
}

cudaError_t scan_nonfinite(const void *p, size_t rows, size_t cols, size_t ld, unsigned *flags, int flag,
                           cudaStream_t s, int sm_count) {
    const size_t work = rows * ((cols + 7) / 8);
    scan_kernel<<<grid_cap(work, sm_count, 8), THREADS, 0, s>>>(static_cast<const __half *>(p), rows, cols,
                                                                 ld, flags, flag);
    return cudaGetLastError();
}

// ----------------------------------------------------------------------------- cube <-> row-major
// One 16-byte atom = 8 consecutive channels of one row. Atom a of a tile walks rows fastest, so a
// warp reads (gather) or writes (scatter) 512 contiguous cube bytes.
__global__ void __launch_bounds__(THREADS) gather_kernel(CubeTiles t, __half *dst, size_t ld) {
    const CubeTile &c = t.tile[blockIdx.y];
    const unsigned groups = (c.cols + 7) / 8;
    const size_t atoms = (size_t)groups * c.rows;
    const uint4 *src = static_cast<const uint4 *>(c.ptr);
    for (size_t a = (size_t)blockIdx.x * THREADS + threadIdx.x; a < atoms; a += (size_t)gridDim.x * THREADS) {
        const unsigned g = (unsigned)(a / c.rows), r = (unsigned)(a % c.rows);
        const uint4 v = src[(size_t)g * c.physical_rows + r];
        *reinterpret_cast<uint4 *>(dst + (size_t)(c.row0 + r) * ld + c.col0 + 8 * g) = v;
    }
}

__global__ void __launch_bounds__(THREADS) scatter_kernel(CubeTiles t, const __half *src, size_t ld) {
    const CubeTile &c = t.tile[blockIdx.y];
    const unsigned groups = c.physical_cols / 8;
    const size_t atoms = (size_t)groups * c.physical_rows;
    uint4 *dst = static_cast<uint4 *>(c.ptr);
    for (size_t a = (size_t)blockIdx.x * THREADS + threadIdx.x; a < atoms; a += (size_t)gridDim.x * THREADS) {
        const unsigned g = (unsigned)(a / c.physical_rows), r = (unsigned)(a % c.physical_rows);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < c.rows && 8 * g < c.cols) {
            v = *reinterpret_cast<const uint4 *>(src + (size_t)(c.row0 + r) * ld + c.col0 + 8 * g);
            const unsigned keep = c.cols - 8 * g;       // channels of this atom inside the tile
            if (keep < 8) {
                uint16_t *h = reinterpret_cast<uint16_t *>(&v);
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    if ((unsigned)e >= keep) h[e] = 0;
            }
        }
        dst[(size_t)g * c.physical_rows + r] = v;
    }
}

cudaError_t cube_gather(const CubeTiles &t, void *dst, size_t ld, cudaStream_t s, int sm_count) {
    if (!t.count) return cudaSuccess;
    const unsigned bx = (unsigned)((sm_count * 4 + t.count - 1) / t.count);
    gather_kernel<<<dim3(bx < 1 ? 1 : (bx > 64 ? 64 : bx), t.count), THREADS, 0, s>>>(t, static_cast<__half *>(dst), ld);
    return cudaGetLastError();
}

cudaError_t cube_scatter(const void *src, size_t ld, const CubeTiles &t, cudaStream_t s, int sm_count) {
    if (!t.count) return cudaSuccess;
    const unsigned bx = (unsigned)((sm_count * 4 + t.count - 1) / t.count);
    scatter_kernel<<<dim3(bx < 1 ? 1 : (bx > 64 ? 64 : bx), t.count), THREADS, 0, s>>>(
        t, static_cast<const __half *>(src), ld);
    return cudaGetLastError();
}

// ----------------------------------------------------------------------------- guard check
// Buffer blockIdx.x, its slack + guard split over gridDim.y blocks: 16-byte loads when the region
// starts on a 16-byte boundary and both lengths are multiples of 16 (every buffer of this library),
// else byte loads.
constexpr unsigned GUARD_SPLIT = 8;
__global__ void __launch_bounds__(THREADS) guard_kernel(GuardList g, size_t slack, size_t guard, unsigned *flags) {
    const unsigned char *base = static_cast<const unsigned char *>(g.base[blockIdx.x]) + g.payload[blockIdx.x];
    const size_t total = slack + guard, stride = (size_t)gridDim.y * THREADS;
    bool bad = false;
    if ((reinterpret_cast<uintptr_t>(base) & 15) == 0 && (slack & 15) == 0 && (guard & 15) == 0) {
        const uint4 *v = reinterpret_cast<const uint4 *>(base);
        const size_t nv = total >> 4, ns = slack >> 4;
        for (size_t i = (size_t)blockIdx.y * THREADS + threadIdx.x; i < nv; i += stride) {
            const uint4 w = __ldcg(v + i);
            const unsigned want = i < ns ? 0u : 0xa5a5a5a5u;
            bad |= ((w.x ^ want) | (w.y ^ want) | (w.z ^ want) | (w.w ^ want)) != 0u;
        }
    } else {
        for (size_t i = (size_t)blockIdx.y * THREADS + threadIdx.x; i < total; i += stride) {
            const unsigned char want = i < slack ? 0x00 : 0xa5;
            if (base[i] != want) bad = true;
        }
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) raise_flag(flags, FLAG_GUARD);
}

cudaError_t guard_check(const GuardList &g, size_t slack, size_t guard, unsigned *flags, cudaStream_t s) {
    if (!g.count) return cudaSuccess;
    guard_kernel<<<dim3(g.count, GUARD_SPLIT), THREADS, 0, s>>>(g, slack, guard, flags);
    return cudaGetLastError();
}

// ----------------------------------------------------------------------------- separate epilogue
// FP32 partial -> y (FP32 finish) or folded FP16 run in y -> y (tile-16 finish, in place).
__global__ void __launch_bounds__(THREADS) epilogue_kernel(EpilogueParams p) {
    const size_t total = (size_t)p.M * p.N;
    const bool has_bias = p.bias != nullptr;
    bool bad = false;
    for (size_t i = (size_t)blockIdx.x * THREADS + threadIdx.x; i < total; i += (size_t)gridDim.x * THREADS) {
        const size_t r = i / p.N, c = i % p.N;
        const float b = has_bias ? __half2float(p.bias[c]) : 0.0f;
        float v;
        if (p.partial) v = finish_fp32(p.partial[r * p.ldp + c], b, p.post);
        else v = finish_tile16(__half2float(p.y[r * p.ldy + c]), b, has_bias, p.post);
        const __half h = __float2half_rn(v);
        bad |= half_nonfinite(h);
        p.y[r * p.ldy + c] = h;
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) raise_flag(p.flags, FLAG_NONFINITE_OUTPUT);
}

cudaError_t epilogue(const EpilogueParams &p, cudaStream_t s, int sm_count) {
    epilogue_kernel<<<grid_cap((size_t)p.M * p.N, sm_count, 8), THREADS, 0, s>>>(p);
    return cudaGetLastError();
}

}  // namespace aux
}  // namespace b2
