// gemm_sm100.h -- parameters and host launcher of the tcgen05 GEMM (gemm_sm100.cu).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>

namespace b2 {
namespace gemm {

enum OutMode : int {
    OUT_FINAL = 0,   // y = FP16 result with bias and activation
    OUT_RAW16 = 1,   // y = the per-256-K folded FP16 running sum (no bias, no activation)
    OUT_RAW32 = 2,   // partial = the FP32 accumulator over the whole K
};

constexpr int ROUTE_MAX = 8;   // ranks a routed raw output can address

// Output tile of the cube store (the device-cube entries): the caller's C2=8 cube holding rows x cols
// of the 256 x 256 output tile (mt, nt), element (r, c) at ptr + ((c / 8) * prow + r) * 8 + c % 8;
// rows [rows, prow) and columns [cols, pcols) of the cube are padding and receive zeros.
struct CubeOut {
    __half *ptr;
    int prow, rows, cols, pcols;
    int pad[2];
};

struct Params {
    int M, N, K;
    int num_m_blocks, num_n_blocks, num_tiles, num_kb, kb_per_chunk;
    const __half *bias;          // [N] or nullptr
    __half *y;                   // [M, ldy]
    long long ldy;
    float *partial;              // [M, ldp]
    long long ldp;
    int out_mode, post, fold, vec_y, vec_p;
    int group_m;                 // tile raster: bands of group_m m-blocks (0 = column-major)
    unsigned *flags;             // status flag words (common.cuh)
    // Routed raw output (fused K-split, out_mode OUT_RAW32): with route_rows > 0 (a multiple of 32),
    // accumulator row r goes to owner q = r / route_rows, as row r' = r - q * route_rows of parity
    // plane ((*route_seq + 1) & 1) at route_dst[q] (another GPU's memory for q != this rank,
    // written with plain stores over NVLink), element (r', c) at (r'/32)*32*ldp + c*32 + r'%32;
    // route_rows == 0 writes `partial` row-major.
    float *route_dst[ROUTE_MAX];
    long long route_plane;       // floats between the two parity planes
    const unsigned *route_seq;   // this rank's round counter, read by the epilogue
    int route_rows;
    // Residual (OUT_FINAL): y = fp16(res + fp16(result)), res FP16 [M, ldr]; nullptr for none.
    const __half *res;
    long long ldr;
    int vec_r;
    // Gated output (OUT_FINAL with fold, gate != 0): W is packed in 64-row blocks, rows
    // [64t, 64t+32) = gate rows [32t, 32t+32) and rows [64t+32, 64t+64) = up rows [32t, 32t+32),
    // so N = 2 * roundup(gate_n, 32). Each FP16 sum is finished with its own bias (bias: gate,
    // bias2: up; [gate_n] or nullptr) and y[r, j] = fp16(fp16(g * fp16(gate(g))) * u), j < gate_n.
    int gate;                    // 0 none, GATE_SIGMOID (SiLU) or GATE_GELU (common.cuh)
    int gate_n;
    const __half *bias2;
    const __half *gate_table;    // the gate of every FP16 input (common.cuh GATE_TABLE_ENTRIES)
    int tma_y;                   // FP16 output stored through TMA tile stores (set by the launcher)
    // Cube operands (the device-cube entries; OUT_FINAL only). With a_maps, X comes from the caller's
    // C2=8 cube views: a_maps (global memory, 64-byte aligned) holds one 3-D tensor map per view
    // (make_cube_map), view (row / 256) * a_kviews + k / a_kview_k holding rows [256 (row / 256), +256)
    // and K [k - k % a_kview_k, + a_kview_k) of X; shared memory receives [8 channel groups][128
    // rows][8] without swizzle. With y_cube (global memory, [M bands of 256][y_cube_nt]), each output
    // tile goes to its cube, padding included, and y is not written.
    const CUtensorMap *a_maps;
    const unsigned char *a_octets;   // [views] 1: the map addresses rows in octets (make_cube_map)
    int a_kviews, a_kview_k;
    const CubeOut *y_cube;
    int y_cube_nt;
};

struct Shape {
    const void *x; size_t ldx;   // FP16 [M, ldx]
    const void *w; size_t ldw;   // FP16 [N, ldw]
};

constexpr int TILE_K = 64;

// Launches one persistent GEMM on `stream` with the tile shape chosen for (M, N).
// `p` carries M/N/K, epilogue and output fields; the block counts are filled in here. Returns
// the CUDA error of the launch.
cudaError_t launch(const Shape &s, Params p, cudaStream_t stream, int device, int sm_count,
                   unsigned *grid_out);
// A specific variant: cg CTAs per cluster (1 = 128x256 tiles, 2 = 256x256 tiles per CTA pair).
cudaError_t launch_variant(int cg, const Shape &s, const Params &p, cudaStream_t stream, int device,
                           int sm_count, unsigned *grid_out);
// 3-D tensor map of a C2=8 FP16 cube view for Params::a_maps: rows x cols logical (cols % 8 == 0),
// prow physical rows, no swizzle, zeros outside the logical extent. When rows % 8 == 0 the map is
// (64 = 8 rows x 8 channels, rows / 8 row octets, cols / 8 groups) with box 64 x 16 x 8, so every
// request is 128 contiguous bytes (*octets = 1); otherwise (8 channels, rows, groups) with box
// 8 x 128 x 8 (16-byte requests). Both land [8 groups][128 rows][8] in shared memory. False when
// the view cannot be described.
bool make_cube_map(CUtensorMap *map, const void *ptr, unsigned rows, unsigned prow, unsigned cols, int *octets);
// Runs the launchers' one-time device setup (tensor-map encoder lookup, shared-memory limits,
// co-resident cluster counts) now, so that a later launch issues no such call (a launch recorded
// into a CUDA graph must not).
cudaError_t prepare(int device, int sm_count);
// Grid (CTAs) the launch would use, and its tile shape and ring depth (for reporting).
unsigned grid_for(int M, int N, int sm_count);
void config_for(int M, int N, int sm_count, unsigned *tile_m, unsigned *tile_n, unsigned *stages);

}  // namespace gemm
}  // namespace b2
