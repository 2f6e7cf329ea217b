/* b2_device.h -- internal seam between the host C layer and the CUDA layer.
 *
 * Host code (the C files under csrc/host) reaches the GPU only through these functions; the
 * CUDA files under csrc/cuda implement them with the CUDA runtime and hand-written sm_100a kernels. The host C tests link
 * a CPU stand-in of this seam instead (tests/c/mock_device.c), the way the reference's host tests
 * wrap its BO and submit calls (research/custom-ops/tests/c/multitile_host_test.c:14-58): that
 * stand-in exists only in test binaries; the shipped library has no CPU compute path.
 *
 * Only plain C types cross this boundary. FP16 data is opaque (uint16_t bits).
 */
#ifndef B2_DEVICE_H
#define B2_DEVICE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct b2_dev b2_dev;

/* Status bits returned by b2d_status (the same values as B2_STATUS_* in b2_linear.h). */
enum {
    B2D_ST_TIMEOUT = 1u,
    B2D_ST_NONFINITE_OUTPUT = 2u,
    B2D_ST_NONFINITE_INPUT = 4u,
    B2D_ST_GUARD = 8u,
    B2D_ST_SCAN_OUTPUT = 16u,       /* internal: a graph output scan found a non-finite value */
};

/* Largest M served by the weight-streaming small-M kernel; larger M uses the tcgen05 GEMM. */
#define B2D_GEMV_MAX_M 8u

int b2d_device_count(void);
int b2d_open(int ordinal, b2_dev **out);
void b2d_close(b2_dev *);
int b2d_set_stream(b2_dev *, void *stream);
void *b2d_stream(b2_dev *);
int b2d_sm_count(b2_dev *);

/* Zero-filled device allocation; returns ROCKET_E_NOMEM on failure. */
int b2d_malloc(b2_dev *, size_t bytes, void **out);
void b2d_free(b2_dev *, void *ptr);
void *b2d_host_alloc(size_t bytes);
void b2d_host_free(void *ptr);

enum { B2D_H2D = 0, B2D_D2H = 1, B2D_D2D = 2 };
/* Pitched copy of `rows` rows of `width` bytes, asynchronous on the handle's stream. */
int b2d_copy_2d(b2_dev *, void *dst, size_t dpitch, const void *src, size_t spitch,
                size_t width, size_t rows, int kind);
/* The same copy on the handle's side stream, ordered after all work issued so far on the handle's
 * stream, then recorded under side event `ev` (< B2D_SIDE_EVENTS): an input copy in row bands that
 * kernels on the handle's stream consume band by band (b2d_wait_side). Without a side stream the
 * copy goes to the handle's stream. */
#define B2D_SIDE_EVENTS 8u
int b2d_copy_side(b2_dev *, void *dst, size_t dpitch, const void *src, size_t spitch,
                  size_t width, size_t rows, int kind, unsigned ev);
/* Work issued on the handle's stream after this call waits for the copy recorded under `ev`. */
int b2d_wait_side(b2_dev *, unsigned ev);
int b2d_memset(b2_dev *, void *ptr, int value, size_t bytes);
/* Waits for the handle's stream; ROCKET_E_DEVICE if CUDA reported an error. */
int b2d_sync(b2_dev *);
/* Device status word (B2_STATUS_* bits) written by kernels; read after b2d_sync. */
uint32_t b2d_status(b2_dev *, int clear);
/* ORs `bits` into the status word (restores bits a synchronous entry read out early). */
void b2d_status_merge(b2_dev *, uint32_t bits);

/* ---------------------------------------------------------------------- Linear launches */
typedef struct {
    unsigned m, n, k;
    const void *x; size_t ldx;      /* FP16 [m, ldx], 16-byte aligned, ldx % 8 == 0 */
    const void *w; size_t ldw;      /* FP16 [n, ldw], 16-byte aligned, ldw % 8 == 0 */
    const void *bias;               /* FP16 [n] or NULL */
    void *y; size_t ldy;            /* FP16 [m, ldy] */
    float *partial; size_t ldp;     /* FP32 [m, ldp]: raw-accumulator destination / workspace */
    int post;                       /* 0 none, 1 HardSigmoid */
    int acc;                        /* 0 per-256-K FP16 fold (reference), 1 FP32 */
    int fused;                      /* 1: epilogue in the GEMM; 0: raw to `partial`, then epilogue */
    int raw_only;                   /* 1: stop after writing the raw accumulator to `partial` */
    /* Residual (graph ADD of this output): y = fp16(res + fp16(result)); FP16 [m, ldr], 16-byte
     * aligned, ldr % 8 == 0; y must then be 16-byte aligned with ldy % 8 == 0. NULL for none. */
    const void *res; size_t ldr;
    /* Gated Linear (graph SiLU/GELU of one Linear times another Linear of the same input):
     * gate = 1 SiLU, 2 GELU; w packed in 64-row blocks [32 gate rows | 32 up rows] with
     * n = 2 * roundup(gate_n, 32); bias = gate bias [gate_n], bias2 = up bias [gate_n] (either
     * NULL); y [m, ldy >= gate_n] receives fp16(fp16(g * fp16(gate(g))) * u). Requires acc = 0,
     * post = 0, no residual. Where the GEMM cannot fuse it (m <= B2D_GEMV_MAX_M, or fused = 0)
     * the folded sums go to tmp (FP16 [m, ldt >= n], 16-byte aligned, ldt % 8 == 0) and a
     * second kernel combines them. */
    int gate;
    unsigned gate_n;
    const void *bias2;
    void *tmp; size_t ldt;
} b2k_linear;

typedef struct {
    unsigned kernel;                /* 0 tcgen05 GEMM, 1 GEMV */
    unsigned tile_m, tile_n, tile_k, stages, grid;
} b2k_config;

/* Picks the kernel for the shape and launches it (plus the separate epilogue when !fused).
 * *launches receives the number of kernels launched. */
int b2d_linear(b2_dev *, const b2k_linear *, unsigned *launches);
int b2d_linear_config(b2_dev *, const b2k_linear *, b2k_config *);
/* Runs `count` (<= B2D_GROUP_MAX) independent fused Linears with the same m. Those the streamed
 * small-M kernel serves with whole-row units (m <= 8 with k <= 2048, or m <= 4 with k <= 8192, the
 * m x k input within its 32 KB x table) share one launch (or several when their distinct inputs
 * exceed the table); a long-K member streamed in K slices runs in a launch of its own; any other
 * runs as b2d_linear.
 * Every op must have fused = 1 and raw_only = 0. */
#define B2D_GROUP_MAX 16u
int b2d_linear_group(b2_dev *, const b2k_linear *ops, unsigned count, unsigned *launches);
/* y = act(partial + bias) with the same arithmetic as the fused epilogue of mode `acc`. */
int b2d_epilogue(b2_dev *, unsigned m, unsigned n, const float *partial, size_t ldp,
                 const void *bias, int post, int acc, void *y, size_t ldy);

/* ---------------------------------------------------------------------- graph node kernels
 * FP16 row-major operands with 16-byte aligned bases and pitches (elements) that are multiples
 * of 8; otherwise ROCKET_E_SHAPE. A result that overflows FP16 sets B2D_ST_NONFINITE_OUTPUT. */
enum { B2D_EW_ADD = 0, B2D_EW_MUL = 1, B2D_EW_SILU = 2, B2D_EW_GELU = 3, B2D_EW_HSIG = 4 };
/* y = fp16(a + b), fp16(a * b), fp16(a * fp16(sigmoid(a))), fp16(a * fp16(gelu_gate(a))) or
 * fp16(hsig(a)); b only for ADD/MUL. y may be a or b (same pitch). */
int b2d_elementwise(b2_dev *, int op, unsigned rows, unsigned cols, const void *a, size_t lda,
                    const void *b, size_t ldb, void *y, size_t ldy);
/* RMSNorm of each row with FP16 gamma [cols] and epsilon eps (> 0). A row whose 256-column
 * square sum reaches 65504 or whose coefficient overflows FP16 sets B2D_ST_NONFINITE_INPUT. */
int b2d_rmsnorm(b2_dev *, unsigned rows, unsigned cols, const void *x, size_t ldx,
                const void *gamma, float eps, void *y, size_t ldy);

/* ---------------------------------------------------------------------- CUDA graphs
 * Launches issued between b2d_capture_begin and b2d_capture_end on this handle's stream are
 * recorded (not run) into an executable graph; b2d_exec_launch replays it on the handle's
 * stream. capture_begin returns ROCKET_E_UNSUPPORTED where capture is not available; after a
 * failed launch inside the capture, capture_end still ends it and returns an error. */
typedef struct b2_exec b2_exec;
int b2d_capture_begin(b2_dev *);
int b2d_capture_end(b2_dev *, b2_exec **out, unsigned *kernels);
int b2d_exec_launch(b2_dev *, b2_exec *);
void b2d_exec_destroy(b2_exec *);

/* Sets status `bit` if any of rows x cols FP16 elements (row pitch ld elements) is not finite. */
int b2d_scan_nonfinite(b2_dev *, const void *p, size_t rows, size_t cols, size_t ld, uint32_t bit);

/* One C2=8 FP16 cube tile placed at (row0, col0) of a row-major matrix. */
typedef struct {
    void *ptr;                      /* device address of the cube view */
    unsigned rows, cols;            /* logical extent */
    unsigned physical_rows, physical_cols;
    unsigned row0, col0;            /* position in the row-major matrix */
} b2k_cube_tile;
#define B2K_MAX_CUBE_TILES 64
/* Gather cube tiles into row-major dst [*, ld] (logical elements and their atoms). */
int b2d_cube_to_rowmajor(b2_dev *, const b2k_cube_tile *tiles, unsigned count, void *dst, size_t ld);
/* Scatter row-major src into cube tiles: logical elements, padding zeroed (within each view). */
int b2d_rowmajor_to_cube(b2_dev *, const void *src, size_t ld, const b2k_cube_tile *tiles,
                         unsigned count);

/* The fused Linear (a->fused, no residual or gate, m > B2D_GEMV_MAX_M) reading X straight from the
 * caller's C2=8 cube views and writing the output cubes (padding zeroed): the gather/scatter-free
 * form of the cube entries. in[mb * kviews + kt] holds rows [256 mb, +256) and K [kt * kview_k,
 * + kview_k) of X (kviews = 1: all of K), its logical cols a multiple of 8; out[mt * ntiles + nt]
 * is the 256 x 256 output tile (mt, nt). a->x and a->y are ignored. The views' tensor maps are
 * encoded on the host and copied to a per-handle table before the launch. ROCKET_E_UNSUPPORTED when
 * the shape or a view does not qualify (the caller then gathers and scatters). */
#define B2D_CUBE_MAX_VIEWS 256u
typedef struct {
    const b2k_cube_tile *in; unsigned nin, kviews, kview_k;
    const b2k_cube_tile *out; unsigned nout, ntiles;
} b2k_cube_io;
int b2d_linear_cube(b2_dev *, const b2k_linear *a, const b2k_cube_io *io, unsigned *launches);

/* ---------------------------------------------------------------------- peer memory (CUDA IPC) */
#define B2D_IPC_HANDLE_BYTES 64
/* Exports a b2d_malloc'ed allocation for other processes on this node. */
int b2d_ipc_export(b2_dev *, const void *ptr, unsigned char out[B2D_IPC_HANDLE_BYTES]);
/* Maps another process's exported allocation into this device's address space (peer access over
 * NVLink); b2d_ipc_close unmaps it. */
int b2d_ipc_open(b2_dev *, const unsigned char in[B2D_IPC_HANDLE_BYTES], void **ptr);
int b2d_ipc_close(b2_dev *, void *ptr);

/* One fused K-split round (ksplit.cu): the routed raw-FP32 GEMM of `a` (a->fused = 0,
 * a->raw_only = 1), the round signal to every rank, and the reduction + epilogue of the owned
 * rows into y_own. `bufs[q]` is rank q's buffer as mapped here (bufs[rank] = the local one). */
typedef struct b2_timer b2_timer;
typedef struct {
    unsigned world, rank, rows_per_rank, own_rows;
    size_t ldp;
    void *bufs[8];
    const void *bias;
    int post;
    void *y_own; size_t ldy;
    b2_timer *timer;                /* NULL, or marks 0..3: round start, GEMM done, signal done, reduce done */
} b2k_ksplit;
int b2d_ksplit_round(b2_dev *, const b2k_linear *a, const b2k_ksplit *ks, unsigned *launches);

/* ---------------------------------------------------------------------- event timer
 * B2D_TIMER_MARKS CUDA timing events of one handle: b2d_timer_mark records mark i on the handle's
 * stream; b2d_timer_ms waits for mark `to` and returns the device time from mark `from` to it. */
#define B2D_TIMER_MARKS 8u
int b2d_timer_create(b2_dev *, b2_timer **out);
void b2d_timer_destroy(b2_timer *);
int b2d_timer_mark(b2_dev *, b2_timer *, unsigned mark);
int b2d_timer_ms(b2_timer *, unsigned from, unsigned to, float *ms);

/* Ordinal of the CUDA device behind a handle (-1 for NULL). */
int b2d_ordinal(b2_dev *);

/* Fixed FP32 scratch of B2D_NOALLOC_SCRATCH_BYTES in every device's static memory (noalloc.cu).
 * The first call on a device looks its address up (cudaGetSymbolAddress); nothing is allocated. */
#define B2D_NOALLOC_SCRATCH_BYTES (8u << 20)
int b2d_noalloc_scratch(b2_dev *, float **ptr, size_t *bytes);

/* Guard regions: [payload, payload+slack) must be zero, [payload+slack, +guard) 0xA5. */
int b2d_guard_init(b2_dev *, void *base, size_t payload, size_t slack, size_t guard);
/* Checks up to B2K_MAX_CUBE_TILES buffers; sets B2_STATUS_GUARD on any mismatch. */
int b2d_guard_check(b2_dev *, void *const *bases, const size_t *payloads, unsigned count,
                    size_t slack, size_t guard);

/* ---------------------------------------------------------------------- plan (RKPlan) tiles
 * A device tile of a plan view: FP16 at `ptr` (16-byte aligned) in one of the three layouts
 * (values of enum rk_layout): CUBE [pcols/8][prows][8], WEIGHT [prows/16][pcols/32][16][32],
 * LINEAR [pcols] (prows 1). */
enum { B2K_RK_CUBE = 1, B2K_RK_WEIGHT = 2, B2K_RK_LINEAR = 3 };
typedef struct {
    void *ptr;
    unsigned layout, rows, cols, physical_rows, physical_cols;
} b2k_rk_tile;

/* Upload packing: the destination logical rectangle [r0, r0+rows) x [c0, c0+cols) of `dst`
 * receives, for its element (r0+i, c0+j),
 *   MATRIX   src[(transpose ? j : i) * ld + (transpose ? i : j)]
 *   SCALAR   src[0]
 *   CHANNEL  src[j]
 * and, with `clear`, every other physical element of the tile becomes 0. src is device FP16. */
enum { B2K_RK_SRC_MATRIX = 0, B2K_RK_SRC_SCALAR = 1, B2K_RK_SRC_CHANNEL = 2 };
typedef struct {
    b2k_rk_tile dst;
    unsigned r0, c0, rows, cols;
    unsigned clear, mode, transpose;
    const void *src;
    size_t ld;
} b2k_rk_pack;
#define B2K_RK_MAX_PACK 40u     /* items per b2d_rk_pack launch (kernel parameter space) */
int b2d_rk_pack(b2_dev *, const b2k_rk_pack *items, unsigned count);

/* One device task (op = an rk_template_id value) over the tiles' whole physical extents:
 *   contraction ops (MM, MM_ACC, EW_*): s(r, c) = sum over q < x.physical_cols, in order, of
 *     double(x[r][q]) * double(w[c][q]) (w = the identity operand for EW_*), then
 *     MM fp16(s); MM_ACC fp16(s + aux); EW_ADD fp16(s + aux); EW_MUL fp16(s * aux);
 *     EW_MAX fp16(fmax(s, aux)); EW_ADD_RELU fp16(fmax(s + aux, 0)), for r < y.physical_rows,
 *     c < y.physical_cols (aux has y's geometry);
 *   LUT ops: y[e] = fp16(f(double(x[e]))) for each physical element (x and y same geometry) with
 *     f = 1/(1+exp(-v)), clamp(v/6+0.5, 0, 1), 0.5(1+erf(v/sqrt 2)) or 1/sqrt(max(v, 0.125)).
 * Every fp16() is one round-to-nearest-even of the double. ROCKET_E_SHAPE for an unknown op, a
 * contraction over more than 256 physical columns, or tiles whose extents do not fit together. */
typedef struct {
    unsigned op;
    b2k_rk_tile x, w, aux, y;
} b2k_rk_task;
int b2d_rk_task(b2_dev *, const b2k_rk_task *task);

/* A contraction chain of tasks whose intermediate results nothing else reads: MM over (x[0], w[0]),
 * then MM_ACC over (x[i], w[i]) with the previous result as the prior for 0 < i < n, and with
 * lut != 0 (an rk_template_id LUT value) that LUT on the last result. Only y (the last task's
 * output) is written; every element gets the same arithmetic as the separate tasks (each chunk sum
 * in q order in double, fp16 after every task). The n chunk sums run in parallel: `scratch` holds
 * n * B * 256 doubles and `tickets` B words, zero on entry and left at zero, where B =
 * ceil(y.physical_rows / 8) * ceil(y.physical_cols / 32). */
#define B2K_RK_CHAIN_MAX 16u
typedef struct {
    b2k_rk_tile x[B2K_RK_CHAIN_MAX], w[B2K_RK_CHAIN_MAX], y;
    unsigned n, lut;
    double *scratch;
    unsigned *tickets;
} b2k_rk_chain;
int b2d_rk_chain(b2_dev *, const b2k_rk_chain *chain);

/* Download unpacking: the logical rows x cols of `src` into row-major device FP16 at dst with a
 * pitch of ld elements. */
typedef struct {
    b2k_rk_tile src;
    void *dst;
    size_t ld;
} b2k_rk_unpack;
#define B2K_RK_MAX_UNPACK 64u
int b2d_rk_unpack(b2_dev *, const b2k_rk_unpack *items, unsigned count);

#ifdef __cplusplus
}
#endif
#endif
