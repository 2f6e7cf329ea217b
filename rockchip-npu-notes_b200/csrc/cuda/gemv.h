// gemv.h -- parameters and launchers of the small-M kernels (gemv.cu).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace b2 {
namespace gemv {

constexpr int MAX_M = 8;
enum OutMode : int { OUT_FINAL = 0, OUT_RAW16 = 1, OUT_RAW32 = 2 };

// Per-handle device scratch of the long-K (sliced) streamed launches: FP32 sums of the 256-K tiles
// of a (W row, x row) that a CTA computes for a block another CTA finishes, and one arrival counter
// per 16-row block (zero between launches: the CTA that finishes the block resets it).
constexpr long long TSUM_FLOATS = 2ll << 20;   // 8 MB
constexpr int TCOUNT_WORDS = 1 << 16;
struct Scratch {
    float *tsum;
    unsigned *tcount;
};

struct Params {
    int M, N, K;
    const __half *x; long long ldx;     // [M, ldx], 16-byte aligned rows
    const __half *w; long long ldw;     // [N, ldw], 16-byte aligned rows
    const __half *bias;                 // [N] or nullptr
    __half *y; long long ldy;
    float *partial; long long ldp;
    int out_mode, post, fold;
    unsigned *flags;
    Scratch scratch;                    // tile sums of long-K problems (from the device handle)
};

// Bulk-copy streamed kernel: one launch serves up to GROUP_MAX independent projections that share
// the row count M (for example the Q/K/V or gate/up projections of one decoder layer).
constexpr int GROUP_MAX = 16;
constexpr int STREAM_MAX_M = 8;         // x rows: the n8 dimension of the m16n8k16 MMA
constexpr int STREAM_X_BYTES = 32768;   // shared-memory table of the launch's distinct x rows
constexpr int STREAM_X_HALF_BYTES = 12288; // the x table of half-SM launches (two CTAs per SM)
constexpr int STREAM_ROW_BYTES = 16384; // one copy slot
// A unit of a problem with K <= STREAM_WHOLE_K is whole W rows (as many as fill a slot). Above it:
// * octet units (K <= STREAM_OCTET_MAX_K, M <= STREAM_OCTET_MAX_M, the M x rows within the 32 KB
//   table): one or two whole W rows, and every m16n8k16 MMA pairs 16 (W row, 256-K tile) rows of A
//   with 8 consecutive x tiles as the columns of B, so a W element always meets its own x element
//   and D[i][i % 8] is a 256-K tile sum. Units are independent: no tile sums cross CTAs.
// * otherwise a unit is one K slice of STREAM_SLICE of a 16-row block, so the 16 W rows of every
//   m16n8k16 MMA are real rows however long K is. Each CTA takes a contiguous range of the
//   block-major unit order and finishes the blocks whose first slice it holds.
// Both compute every tile sum with the same products in the same MMA slots and fold them in K
// order, so a row's result is the same bits either way.
constexpr int STREAM_WHOLE_K = 2048;
constexpr int STREAM_OCTET_MAX_K = 8192;
constexpr int STREAM_OCTET_MAX_M = 4;
// Octet units of one row up to K = STREAM_OCTET_WIDE_MAX_K at M = 1 run in the wide-slot
// configuration (8 slots of STREAM_WIDE_ROW_BYTES, one CTA per SM), so rows longer than a 16 KB
// slot still stream whole instead of as K slices.
constexpr int STREAM_WIDE_ROW_BYTES = 24576;
constexpr int STREAM_OCTET_WIDE_MAX_K = 12288;
constexpr int STREAM_SLICE = 512;       // 16 rows x 512 FP16 = one slot; a multiple of the 256-K tile
constexpr int STREAM_MAX_XTILES = 64;   // sliced launches: M x (256-K tiles) per block buffer
// Wide sliced launches (x rows beyond 32 KB, e.g. M = 8 at K = 4096): 8 ring slots, a 64 KB x table
// and block buffers for M x tiles <= 128, so the batch streams W once instead of once per row group.
constexpr int STREAM_X_WIDE_BYTES = 65536;
constexpr int STREAM_MAX_XTILES_WIDE = 128;

struct Problem {
    const __half *x; long long ldx;
    const __half *w; long long ldw;
    const __half *bias;
    __half *y; long long ldy;
    float *partial; long long ldp;
    int N, K, out_mode, post, fold;
    int rows_per_unit, unit_begin;      // filled in by launch_group
    int x_off;                          // element offset of this problem's x rows in the x table
    int kslice;                         // 0: whole-row units; else K slice of the 16-row units
    int slices;                         // K slices of a sliced problem (units = blocks x slices)
    int octet;                          // 1: long-K whole-row units with the octet MMA mapping
};

// One distinct x (problems that share x and K share the entry): M rows of K, pitch ldx in
// global memory, stored with pitch round8(K) from element `off` of the table.
struct XSource {
    const __half *x; long long ldx;
    int K, off;
};

struct Group {
    CUtensorMap wmap;                   // W of a sliced problem (alone in its launch), see map3
    Problem prob[GROUP_MAX];
    XSource xsrc[GROUP_MAX];
    int count, M, units, nx;
    int map3;                           // wmap is 3-D (one copy per 16-row x 512-K unit), else 2-D 64 x 16 boxes
    int hold;                           // whole-row launches: slots a producer fills before the x loads are issued (0: all)
    unsigned *flags;
    Scratch scratch;
};

// The streamed kernel serves M <= 8 when the M x rows fit the x table (M * roundup(K, 8) FP16):
// whole-row problems (K <= 2048) in 32 KB; long-K problems in 64 KB (K <= 16384 for M = 2, 8192 for
// M = 4, 4096 for M = 8), with M x (K/256 tiles) <= STREAM_MAX_XTILES_WIDE, their tile sums
// (N * M * K/256 floats) and block counters (N / 16) fitting the scratch.
bool streamed(int M, int N, int K, long long ldw);
// Streamed launches that serve a single problem in `launch`: 1 when streamed(), else M is split into
// row groups whose x rows fit the table (each group streams all of W; every row's result is the same
// as in a one-launch run); 0 when no row group fits: the per-lane kernel serves it.
int stream_launches(int M, int N, int K, long long ldw);

// Ring slots of the streamed kernel that would serve this shape (long K: 11, or 8 in a wide launch;
// 6 for a half-SM launch, whose x rows fit STREAM_X_HALF_BYTES; else 12); 0 when the per-lane-load
// kernel serves it.
int stream_stages(int M, int N, int K, long long ldw);

// Picks the kernel for p (streamed when eligible, else the per-lane-load kernel) and launches it.
cudaError_t launch(const Params &p, cudaStream_t stream, int sm_count, unsigned *grid_out);
// Runs the launchers' one-time device setup (shared-memory limits, occupancy queries) now, so that
// a later launch issues no such call (a launch recorded into a CUDA graph must not).
cudaError_t prepare();
// Launches the streamed kernel over g.count problems (each must satisfy streamed(g.M, K, ldw)): one
// launch, or more when the problems' distinct x rows exceed the x table (*launches gets the count).
cudaError_t launch_group(Group &g, cudaStream_t stream, int sm_count, unsigned *grid_out, unsigned *launches);
unsigned grid_for(int M, int N, int K, long long ldw, int sm_count);
// True when a problem of this K streams in K slices (16-row units) for a batch of M x rows; false
// for whole-row and octet units.
bool sliced(int M, int K, long long ldw);

}  // namespace gemv
}  // namespace b2
