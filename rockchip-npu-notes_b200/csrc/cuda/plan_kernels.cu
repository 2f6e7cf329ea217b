// plan_kernels.cu -- the plan (RKPlan) runtime's device work on sm_100a.
//
// A plan is a schedule of small tiles (at most 256 x 256, K at most 256 for a matmul) in the
// reference's NPU layouts. Three kernels run it on B200:
//   pack     every per-run upload of the schedule in one launch: the caller's FP16 windows (copied
//            to HBM once per binding) are packed into the destination views' physical layouts,
//            padding zeroed (research/custom-ops/src/rk_plan_runtime.c:244-339).
//   task     one device task (or a chain of contraction tasks whose intermediate results nothing else
//            reads, as one launch): the NPU program's arithmetic as the reference's host model of the NPU
//            states it (research/custom-ops/tests/mock/npu_mock.c:392-537): a matmul-shaped pass
//            s(r, c) = sum over q of x[r][q] * w[c][q] accumulated in double in q order (every
//            FP16 product is exact in double, so an FMA equals the separate multiply and add), the
//            template's epilogue in double, one round-to-nearest-even to FP16 (cvt.rn.f16.f64);
//            LUT templates evaluate their function in double per element and round once.
//   unpack   every download in one launch: the views' logical elements into row-major staging
//            placed at the publish offsets of each output binding.
// The tiles are small and latency-bound; the double-precision contraction keeps the results
// bit-identical to the reference's model (the Linear path itself runs on the tcgen05 GEMM, not
// here).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "plan_kernels.h"

namespace b2 {
namespace rkplan {

constexpr int THREADS = 256;

__device__ __forceinline__ size_t tile_index(const b2k_rk_tile &t, unsigned r, unsigned c) {
    if (t.layout == B2K_RK_LINEAR) return (size_t)r * t.physical_cols + c;
    if (t.layout == B2K_RK_WEIGHT)
        return (((size_t)(r / 16) * (t.physical_cols / 32) + c / 32) * 16 + r % 16) * 32 + c % 32;
    return ((size_t)(c / 8) * t.physical_rows + r) * 8 + c % 8;
}

__device__ __forceinline__ double load_f64(const b2k_rk_tile &t, unsigned r, unsigned c) {
    const unsigned short h = static_cast<const unsigned short *>(t.ptr)[tile_index(t, r, c)];
    return (double)__half2float(__ushort_as_half(h));
}

__device__ __forceinline__ unsigned short round_f16(double v) {
    unsigned short h;
    asm("cvt.rn.f16.f64 %0, %1;" : "=h"(h) : "d"(v));
    return h;
}

// Physical vector v (8 consecutive physical elements) of a tile -> its row and first column.
// Every layout keeps 8 consecutive physical elements in one row at consecutive columns.
__device__ __forceinline__ void vector_origin(const b2k_rk_tile &t, size_t v, unsigned &r, unsigned &c) {
    if (t.layout == B2K_RK_LINEAR) {
        r = 0;
        c = (unsigned)(v * 8);
    } else if (t.layout == B2K_RK_WEIGHT) {
        const size_t ct = t.physical_cols / 32;
        const size_t block = v / 64;                  // one 16 x 32 block holds 64 vectors
        r = (unsigned)((block / ct) * 16 + (v / 4) % 16);
        c = (unsigned)((block % ct) * 32 + (v % 4) * 8);
    } else {
        r = (unsigned)(v % t.physical_rows);
        c = (unsigned)((v / t.physical_rows) * 8);
    }
}

// ----------------------------------------------------------------------------------- pack
__global__ void __launch_bounds__(THREADS) pack_kernel(const __grid_constant__ PackTable t) {
    const b2k_rk_pack &it = t.item[blockIdx.y];
    const b2k_rk_tile &d = it.dst;
    const size_t elements = (size_t)d.physical_rows * d.physical_cols;
    const size_t vectors = (elements + 7) / 8;
    const unsigned short *src = static_cast<const unsigned short *>(it.src);
    unsigned short *dst = static_cast<unsigned short *>(d.ptr);
    for (size_t v = (size_t)blockIdx.x * THREADS + threadIdx.x; v < vectors; v += (size_t)gridDim.x * THREADS) {
        unsigned r, c;
        vector_origin(d, v, r, c);
        const bool row_in = r >= it.r0 && r - it.r0 < it.rows;
        const bool any_in = row_in && c + 8 > it.c0 && c < it.c0 + it.cols;
        if (!any_in && !it.clear) continue;
        unsigned short out[8];
        const bool full = v * 8 + 8 <= elements;
        if (!it.clear && full) {
            const uint4 old = reinterpret_cast<const uint4 *>(dst)[v];
            memcpy(out, &old, 16);
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) out[k] = 0;
        }
        if (any_in) {
            const unsigned i = r - it.r0;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const unsigned cc = c + k;
                if (cc < it.c0 || cc - it.c0 >= it.cols) continue;
                const unsigned j = cc - it.c0;
                size_t at;
                if (it.mode == B2K_RK_SRC_SCALAR) at = 0;
                else if (it.mode == B2K_RK_SRC_CHANNEL) at = j;
                else at = it.transpose ? (size_t)j * it.ld + i : (size_t)i * it.ld + j;
                out[k] = src[at];
            }
        }
        if (full) {
            uint4 u;
            memcpy(&u, out, 16);
            reinterpret_cast<uint4 *>(dst)[v] = u;
        } else {
            for (size_t k = 0; v * 8 + k < elements; ++k)
                if (it.clear || (row_in && c + k >= it.c0 && c + k - it.c0 < it.cols)) dst[v * 8 + k] = out[k];
        }
    }
}

// ----------------------------------------------------------------------------------- tasks
// A block computes 8 output rows x 32 output columns. K (x's physical columns) is at most 256 for
// every contraction template, so the block stages its 8 x rows and 32 W rows over the whole of K in
// shared memory in one load phase, converted to double once there, and each thread then runs its
// element's sum in q order with nothing but the FMA on the dependency chain.
// The W rows are padded by one double so the 32 threads of a warp, reading W rows tx at one q, fall
// on different banks; the x row is a broadcast.
constexpr int TR = 8, TC = 32, KMAX = 256, WPITCH = KMAX + 1, CTHREADS = TR * TC;
constexpr size_t CONTRACT_SMEM = (size_t)(TR * KMAX + TC * WPITCH) * sizeof(double);

__global__ void __launch_bounds__(CTHREADS) contract_kernel(const __grid_constant__ b2k_rk_task t) {
    extern __shared__ double sm[];
    double *xs = sm;                  // [TR][KMAX]
    double *ws = sm + TR * KMAX;      // [TC][WPITCH]
    const unsigned tx = threadIdx.x % TC, ty = threadIdx.x / TC;
    const unsigned r0 = blockIdx.y * TR, c0 = blockIdx.x * TC;
    const unsigned K = t.x.physical_cols;
    const unsigned short *xg = static_cast<const unsigned short *>(t.x.ptr);
    const unsigned short *wg = static_cast<const unsigned short *>(t.w.ptr);
    // Thread (ty, tx) stages x row ty and W rows ty + 8 i (i < 4) at q = tx + 32 j: all 40 loads
    // are issued before any is used, so the phase costs one memory round trip.
    constexpr int J = KMAX / 32;
    unsigned short xv[J], wv[TC / TR][J];
    const unsigned r = r0 + ty;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const unsigned q = tx + 32 * j;
        xv[j] = (r < t.x.physical_rows && q < K) ? xg[tile_index(t.x, r, q)] : (unsigned short)0;
    }
#pragma unroll
    for (int i = 0; i < TC / TR; ++i) {
        const unsigned c = c0 + ty + TR * i;
#pragma unroll
        for (int j = 0; j < J; ++j) {
            const unsigned q = tx + 32 * j;
            wv[i][j] = (c < t.w.physical_rows && q < K) ? wg[tile_index(t.w, c, q)] : (unsigned short)0;
        }
    }
#pragma unroll
    for (int j = 0; j < J; ++j) xs[ty * KMAX + tx + 32 * j] = (double)__half2float(__ushort_as_half(xv[j]));
#pragma unroll
    for (int i = 0; i < TC / TR; ++i)
#pragma unroll
        for (int j = 0; j < J; ++j)
            ws[(ty + TR * i) * WPITCH + tx + 32 * j] = (double)__half2float(__ushort_as_half(wv[i][j]));
    __syncthreads();
    const unsigned c = c0 + tx;
    if (r >= t.y.physical_rows || c >= t.y.physical_cols) return;
    const double *xr = xs + ty * KMAX, *wr = ws + tx * WPITCH;
    double s = 0.0;
#pragma unroll 16
    for (unsigned q = 0; q < K; ++q) s = __fma_rn(xr[q], wr[q], s);
    double v = s;
    if (t.op != 1) {                                          // every op but MM reads aux
        const double b = load_f64(t.aux, r, c);
        switch (t.op) {
        case 2: case 3: v = __dadd_rn(s, b); break;          // MM_ACC, EW_ADD
        case 4: v = __dmul_rn(s, b); break;                   // EW_MUL
        case 8: v = fmax(s, b); break;                        // EW_MAX
        default: v = fmax(__dadd_rn(s, b), 0.0); break;       // EW_ADD_RELU
        }
    }
    static_cast<unsigned short *>(t.y.ptr)[tile_index(t.y, r, c)] = round_f16(v);
}

// A chain: block (bx, by, z) stages chunk z's operands exactly as contract_kernel does and leaves its
// 8 x 32 chunk sums in the scratch; the block that takes the last ticket of its output block folds
// the n sums in chunk order (MM, then MM_ACC: fp16 after each), applies the LUT and stores y. The
// partial stores, a fence and the ticket are the usual last-block hand-off; the folding block
// reads the partials from L2 and puts the ticket back to zero for the next launch.
__device__ __forceinline__ double lut(unsigned op, double v);

__global__ void __launch_bounds__(CTHREADS) chain_kernel(const __grid_constant__ b2k_rk_chain t) {
    extern __shared__ double sm[];
    __shared__ unsigned ticket;
    double *xs = sm;                  // [TR][KMAX]
    double *ws = sm + TR * KMAX;      // [TC][WPITCH]
    const unsigned tx = threadIdx.x % TC, ty = threadIdx.x / TC, z = blockIdx.z;
    const unsigned r0 = blockIdx.y * TR, c0 = blockIdx.x * TC;
    const b2k_rk_tile &X = t.x[z], &W = t.w[z];
    const unsigned K = X.physical_cols;
    const unsigned short *xg = static_cast<const unsigned short *>(X.ptr);
    const unsigned short *wg = static_cast<const unsigned short *>(W.ptr);
    constexpr int J = KMAX / 32;
    unsigned short xv[J], wv[TC / TR][J];
    const unsigned r = r0 + ty;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const unsigned q = tx + 32 * j;
        xv[j] = (r < X.physical_rows && q < K) ? xg[tile_index(X, r, q)] : (unsigned short)0;
    }
#pragma unroll
    for (int i = 0; i < TC / TR; ++i) {
        const unsigned c = c0 + ty + TR * i;
#pragma unroll
        for (int j = 0; j < J; ++j) {
            const unsigned q = tx + 32 * j;
            wv[i][j] = (c < W.physical_rows && q < K) ? wg[tile_index(W, c, q)] : (unsigned short)0;
        }
    }
#pragma unroll
    for (int j = 0; j < J; ++j) xs[ty * KMAX + tx + 32 * j] = (double)__half2float(__ushort_as_half(xv[j]));
#pragma unroll
    for (int i = 0; i < TC / TR; ++i)
#pragma unroll
        for (int j = 0; j < J; ++j)
            ws[(ty + TR * i) * WPITCH + tx + 32 * j] = (double)__half2float(__ushort_as_half(wv[i][j]));
    __syncthreads();
    const unsigned c = c0 + tx;
    const bool live = r < t.y.physical_rows && c < t.y.physical_cols;
    double s = 0.0;
    if (live) {
        const double *xr = xs + ty * KMAX, *wr = ws + tx * WPITCH;
#pragma unroll 16
        for (unsigned q = 0; q < K; ++q) s = __fma_rn(xr[q], wr[q], s);
    }
    const size_t blk = (size_t)blockIdx.y * gridDim.x + blockIdx.x;
    const size_t stride = (size_t)gridDim.x * gridDim.y * CTHREADS;   // doubles per chunk
    t.scratch[z * stride + blk * CTHREADS + threadIdx.x] = s;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) ticket = atomicAdd(&t.tickets[blk], 1u);
    __syncthreads();
    if (ticket != t.n - 1) return;
    __threadfence();
    if (live) {
        const double *part = t.scratch + blk * CTHREADS + threadIdx.x;
        unsigned short run = round_f16(__ldcg(part));
        for (unsigned i = 1; i < t.n; ++i)
            run = round_f16(__dadd_rn(__ldcg(part + i * stride), (double)__half2float(__ushort_as_half(run))));
        if (t.lut) run = round_f16(lut(t.lut, (double)__half2float(__ushort_as_half(run))));
        static_cast<unsigned short *>(t.y.ptr)[tile_index(t.y, r, c)] = run;
    }
    if (threadIdx.x == 0) t.tickets[blk] = 0u;
}

__device__ __forceinline__ double lut(unsigned op, double v) {
    switch (op) {
    case 5: return __ddiv_rn(1.0, __dadd_rn(1.0, exp(-v)));                          // sigmoid
    case 6: return fmin(1.0, fmax(0.0, __dadd_rn(__ddiv_rn(v, 6.0), 0.5)));         // hardsigmoid
    case 7: return __dmul_rn(0.5, __dadd_rn(1.0, erf(__ddiv_rn(v, 1.4142135623730951))));  // GELU gate
    default: return __ddiv_rn(1.0, __dsqrt_rn(fmax(0.125, v)));                      // rsqrt
    }
}

// x and y share one geometry, so physical element e of x maps to physical element e of y.
__global__ void __launch_bounds__(THREADS) lut_kernel(const __grid_constant__ b2k_rk_task t) {
    const size_t n = (size_t)t.y.physical_rows * t.y.physical_cols;
    const unsigned short *x = static_cast<const unsigned short *>(t.x.ptr);
    unsigned short *y = static_cast<unsigned short *>(t.y.ptr);
    for (size_t e = (size_t)blockIdx.x * THREADS + threadIdx.x; e < n; e += (size_t)gridDim.x * THREADS)
        y[e] = round_f16(lut(t.op, (double)__half2float(__ushort_as_half(x[e]))));
}

// ----------------------------------------------------------------------------------- unpack
__global__ void __launch_bounds__(THREADS) unpack_kernel(const __grid_constant__ UnpackTable t) {
    const b2k_rk_unpack &it = t.item[blockIdx.y];
    const size_t n = (size_t)it.src.rows * it.src.cols;
    const unsigned short *src = static_cast<const unsigned short *>(it.src.ptr);
    unsigned short *dst = static_cast<unsigned short *>(it.dst);
    for (size_t e = (size_t)blockIdx.x * THREADS + threadIdx.x; e < n; e += (size_t)gridDim.x * THREADS) {
        const unsigned r = (unsigned)(e / it.src.cols), c = (unsigned)(e % it.src.cols);
        dst[(size_t)r * it.ld + c] = src[tile_index(it.src, r, c)];
    }
}

static unsigned blocks_for(size_t work, int sm_count) {
    const size_t b = (work + THREADS - 1) / THREADS;
    const size_t cap = (size_t)(sm_count > 0 ? sm_count : 148) * 4;
    return (unsigned)(b < 1 ? 1 : (b < cap ? b : cap));
}

cudaError_t prepare() {
    const cudaError_t e =
        cudaFuncSetAttribute(contract_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)CONTRACT_SMEM);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)CONTRACT_SMEM);
}

cudaError_t pack(const PackTable &t, size_t max_vectors, cudaStream_t s, int sm_count) {
    if (!t.count) return cudaSuccess;
    pack_kernel<<<dim3(blocks_for(max_vectors, sm_count), t.count), THREADS, 0, s>>>(t);
    return cudaGetLastError();
}

cudaError_t task(const b2k_rk_task &t, cudaStream_t s, int sm_count) {
    if ((t.op >= 5 && t.op <= 7) || t.op == 10) {
        lut_kernel<<<blocks_for((size_t)t.y.physical_rows * t.y.physical_cols, sm_count), THREADS, 0, s>>>(t);
    } else {
        const dim3 grid((t.y.physical_cols + TC - 1) / TC, (t.y.physical_rows + TR - 1) / TR);
        contract_kernel<<<grid, CTHREADS, CONTRACT_SMEM, s>>>(t);
    }
    return cudaGetLastError();
}

cudaError_t chain(const b2k_rk_chain &t, cudaStream_t s) {
    const dim3 grid((t.y.physical_cols + TC - 1) / TC, (t.y.physical_rows + TR - 1) / TR, t.n);
    chain_kernel<<<grid, CTHREADS, CONTRACT_SMEM, s>>>(t);
    return cudaGetLastError();
}

cudaError_t unpack(const UnpackTable &t, size_t max_elements, cudaStream_t s, int sm_count) {
    if (!t.count) return cudaSuccess;
    unpack_kernel<<<dim3(blocks_for(max_elements, sm_count), t.count), THREADS, 0, s>>>(t);
    return cudaGetLastError();
}

}  // namespace rkplan
}  // namespace b2
