/* b2_linear.h -- extended entry points of the B200 Linear path.
 *
 * The reference caps M, N, K at 4096 (research/custom-ops/include/custom_ops.h:20,145-146) and
 * only offers host-array and device-cube entries. The B200 build keeps those limits on the
 * co_* API (custom_ops.h) and adds, here:
 *   - explicit device selection and caller-supplied CUDA streams (one handle per GPU);
 *   - operators up to B2_MAX_DIM in M, N and K (the SmolLM LM head N=49152, K=16384 cases);
 *   - full-K FP32 accumulation as an alternative to the reference's per-256-K FP16 narrowing;
 *   - asynchronous row-major device-pointer entries (inputs already resident in HBM);
 *   - raw FP32 partial accumulators and a separate bias/activation epilogue, used for K-split
 *     across GPUs (partials reduced with NCCL between the two calls);
 *   - an allocation-free run of the unfused FP32 arm;
 *   - a grouped small-M run (a decoder layer's decode projections in one launch);
 *   - the per-GPU shard of N or K (b2_shard_range) and a fused K-split across GPUs whose GEMM
 *     writes its partials straight into the owner's memory over NVLink (b2_ksplit_*);
 *   - a host-side fault-injection seam for failure-path tests.
 * An operator created here is the same object type as a co_linear and accepts every co_* run
 * entry whose shape limits it meets.
 */
#ifndef B2_LINEAR_H
#define B2_LINEAR_H
#include "custom_ops.h"

#ifdef __cplusplus
extern "C" {
#endif

#define B2_MAX_DIM (1u << 20)

typedef struct co_linear_hsig b2_linear;

/* Accumulation of the K reduction. */
enum b2_accumulate {
    B2_ACC_TILE16 = 0,  /* reference: FP32 per 256-wide K tile, running sum narrowed to FP16 */
    B2_ACC_FP32 = 1,    /* FP32 over the whole K, FP32 bias/activation, one FP16 rounding */
};

/* Device status bits (accumulated per handle by asynchronous entries). */
#define B2_STATUS_TIMEOUT           0x1u   /* a bounded device wait expired; kernel bailed out */
#define B2_STATUS_NONFINITE_OUTPUT  0x2u
#define B2_STATUS_NONFINITE_INPUT   0x4u
#define B2_STATUS_GUARD             0x8u   /* a buffer's slack or guard bytes were overwritten */

/* ----------------------------------------------------------------------- devices and streams */
int b2_device_count(void);
/* Opens CUDA device `ordinal` with a new non-blocking stream; returns a handle (fd) >= 0. */
int b2_open_device(int ordinal);
/* Streams work submitted through `fd` onto `stream` (a cudaStream_t); NULL restores the
 * handle's own stream. The caller keeps ownership of the stream. */
int b2_set_stream(int fd, void *stream);
void *b2_get_stream(int fd);
int b2_sync(int fd);
/* Returns the accumulated B2_STATUS_* bits of asynchronous calls on `fd`; clears them if asked. */
unsigned b2_status(int fd, int clear);
/* Number of streaming multiprocessors of the handle's device (0 on error). */
int b2_sm_count(int fd);
/* Pinned host memory (for end-to-end transfers at full PCIe rate). */
void *b2_host_alloc(size_t bytes);
void b2_host_free(void *p);

/* ----------------------------------------------------------------------- extended operator */
/* Like co_linear_create without the 4096 caps: 1 <= m,k,n <= B2_MAX_DIM. `m` sizes the host
 * staging used by co_linear_run; device entries take their own row count. */
int b2_linear_create(int fd, unsigned m, unsigned k, unsigned n,
                     const _Float16 *weights, const _Float16 *optional_bias,
                     enum co_linear_post post, enum co_mode mode,
                     enum b2_accumulate acc, b2_linear **out);
int b2_linear_set_accumulate(b2_linear *, enum b2_accumulate);
/* X: device row-major [m, ldx] FP16, Y: device row-major [m, ldy] FP16, both 16-byte aligned,
 * ldx and ldy multiples of 8 elements. Asynchronous on the handle's stream: returns after the
 * launches; errors raised by the device appear in b2_status(). */
int b2_linear_run_device(b2_linear *, unsigned m, const void *x, size_t ldx, void *y, size_t ldy);
/* Raw accumulator only: P[m, ldp] FP32 = X * W^T (no bias, no activation, FP32 accumulation). */
int b2_linear_partial_device(b2_linear *, unsigned m, const void *x, size_t ldx,
                             float *partial, size_t ldp);
/* Y[m, ldy] FP16 = act(P + b) using this operator's bias and post-op (FP32 arithmetic). */
int b2_linear_epilogue_device(b2_linear *, unsigned m, const float *partial, size_t ldp,
                              void *y, size_t ldy);

/* No counterpart in the reference: an allocation-free way to run the unfused FP32 arm.
 *
 * Some callers must not allocate GPU memory once they are running -- for instance a serving loop
 * whose device memory is planned up front, where a cudaMalloc/cudaFree in the middle of a request
 * would synchronise the device, add latency, or fail under memory pressure. The other entries
 * that run the unfused FP32 arm (CO_SEPARATE mode with B2_ACC_FP32) allocate their M x N FP32
 * workspace with cudaMalloc on first use. This entry instead uses a fixed scratch array that the
 * library keeps in static device memory: B2_NOALLOC_SCRATCH_BYTES (8 MiB) on every GPU that
 * loads the library, held until the process exits.
 *
 * Computes Y[m, ldy] = act(X W^T + b) like b2_linear_run_device, with FP32 accumulation over the
 * whole K (the operator must use B2_ACC_FP32, else ROCKET_E_UNSUPPORTED), as two launches: the
 * GEMM writes the raw FP32 accumulator into the scratch, then the epilogue kernel writes Y.
 * The caller passes device X and Y (same rules as b2_linear_run_device). Nothing is allocated:
 * no cudaMalloc/cudaFree and no allocating library call.
 *
 * Limits and rules:
 *   - m * roundup(n, 4) * 4 bytes must fit in B2_NOALLOC_SCRATCH_BYTES, else ROCKET_E_TILING
 *     (for example n = 4096 allows m <= 512).
 *   - The first call on a device looks up the scratch address (cudaGetSymbolAddress) and caches
 *     it; make that first call before any stream capture. The lookup switches the calling
 *     thread's current CUDA device to the handle's device and back; the call leaves the current
 *     device as it found it.
 *   - m <= 8 runs the weight-streaming small-M kernel, which writes the raw FP32 sums into the
 *     same scratch (its long-K tile-sum buffers belong to the handle and were allocated when the
 *     handle was opened), so that route allocates nothing either.
 *   - All calls on a device share the one scratch array and it keeps the last call's contents.
 *     No clearing is needed (each call writes every scratch element it later reads), but calls
 *     whose work overlaps on the GPU -- two streams, or two operators at once -- race on it.
 *   - Asynchronous on the handle's stream, like b2_linear_run_device. */
#define B2_NOALLOC_SCRATCH_BYTES (8u << 20)
int b2_linear_run_device_noalloc(b2_linear *, unsigned m, const void *x, size_t ldx, void *y, size_t ldy);

/* Grouped small-M run: Y_i[m, ldy_i] = act_i(X_i W_i^T + b_i) for `count` independent operators on
 * the same handle (same GPU), for example the Q/K/V or gate/up projections of one decoder layer at
 * decode time. It replaces the projection step of the reference's multi-output graph call
 * (research/custom-ops/src/co_decoder.c:128-129, co_graph_run_many in
 * research/custom-ops/include/co_graph.h:77), which produces Q, K and V from one input.
 * Operators with m <= 8 whose m x k input fits the weight-streaming GEMV's 32 KB shared-memory
 * table (m * roundup(k, 8) * 2 bytes; k <= 8192 at m <= 2, 4096 at m = 4, 2048 at m = 8) share ONE
 * kernel launch as long as their distinct inputs (members passing the same X share it) fit the
 * table together; otherwise they are packed in order into consecutive launches that each fit.
 * A member whose K is streamed in slices (k > 2048 at m > 4, k > 8192) runs in a launch of its
 * own, and any other member as its own b2_linear_run_device launch. Each result is bit-identical
 * to that operator's own b2_linear_run_device (CO_SEPARATE operators are finished in the same
 * launch with the same arithmetic as their separate epilogue). X_i and Y_i follow
 * b2_linear_run_device's rules; the X_i may alias (a shared input). Asynchronous on the handle's
 * stream.
 * 1 <= count <= B2_GROUP_MAX, else ROCKET_E_SHAPE; operators on different handles: ROCKET_E_SHAPE. */
#define B2_GROUP_MAX 16u
int b2_linear_group_run_device(b2_linear *const *ops, unsigned count, unsigned m,
                               const void *const *x, const size_t *ldx, void *const *y,
                               const size_t *ldy);

typedef struct {
    unsigned m, k, n;
    unsigned kernel;             /* 0 = tcgen05 GEMM, 1 = GEMV (small M) */
    unsigned tile_m, tile_n, tile_k;   /* GEMM tile_n: 256, or 128 / 64 for 1-SM launches whose 256-wide
                                           tiles would fill at most half / a quarter of the SMs */
    unsigned stages;             /* GEMM: TMA ring depth; streamed GEMV: copy slots (6, 11 or 12); else 0 */
    unsigned grid;               /* CTAs of the main kernel for the create-time m */
    unsigned launches_per_run;   /* CUDA launches of one co_linear_run (scan + GEMM per row band when a
                                    large input is copied in bands) */
    enum b2_accumulate acc;
    size_t device_bytes;         /* HBM held by the operator */
} b2_linear_info;
int b2_linear_get_info(const b2_linear *, b2_linear_info *);

/* ----------------------------------------------------------------------- multi-GPU partition */
/* Shard `index` of `parts` over [0, total): contiguous ranges whose interior boundaries fall on
 * multiples of `align` (256 keeps output tiles and 256-wide K tiles whole), sizes differing by
 * at most one `align` block; trailing shards may be empty when total is small. This is the
 * per-GPU work split of the column-parallel (N) and K-split layouts, replacing the reference's
 * per-submit NPU core assignment (research/custom-ops/src/co_schedule.c). Returns 0 or
 * ROCKET_E_SHAPE for bad arguments. */
int b2_shard_range(unsigned long long total, unsigned parts, unsigned index, unsigned align,
                   unsigned long long *begin, unsigned long long *end);

/* ----------------------------------------------------------------------- fused K-split */
/* K-split of one Linear over `world` GPUs of a node, one process per GPU, with the partial sums
 * added in the owner's memory. Replaces the reference's in-operator K accumulation
 * (research/custom-ops/src/custom_ops.c:297-330, FP16 ping-pong partials on one NPU) for shapes
 * whose N is too small to split by columns. Rank r creates its operator over W[:, k0:k1] (the
 * b2_shard_range of K, FP32 accumulation) and a b2_ksplit; ranks exchange the blobs of
 * b2_ksplit_export (any host channel, e.g. torch.distributed) and pass all of them, in rank order,
 * to b2_ksplit_connect. A round (b2_ksplit_run, every rank, same m):
 *   - the rank's GEMM stores row block q of its FP32 partial straight into rank q's buffer over
 *     NVLink (rows [q*R, (q+1)*R), R = ceil(m_max / world) rounded up to a multiple of 32);
 *   - it signals the round to every rank;
 *   - it waits (at most 1 s, then B2_STATUS_TIMEOUT) for every rank's signal and writes
 *     Y[rows of this rank] = act(sum of the world partials in rank order + b) in FP16.
 * Y is the caller's full [m, ldy] device matrix; only this rank's rows (b2_ksplit_rows) are
 * written. Three launches, asynchronous on the operator's handle stream; every rank must run the
 * same number of rounds. m > 8 (the routed output is a GEMM epilogue), m <= m_max. All ranks must
 * use the same world, m_max and N: b2_ksplit_connect checks the declared layouts and returns
 * ROCKET_E_SHAPE on any mismatch. The first round after connecting is also when peer access is
 * enabled. world = 1 needs no connect (a local reduction). A rank that misses a round makes the
 * others' round end with B2_STATUS_TIMEOUT after at most a second (their Y rows are not written);
 * the ranks' round counters are then out of step, so every rank destroys and re-creates its
 * b2_ksplit before the next round. */
#define B2_KSPLIT_MAX_WORLD 8u
#define B2_KSPLIT_BLOB_BYTES 96u
typedef struct b2_ksplit b2_ksplit;
int b2_ksplit_create(b2_linear *op, unsigned world, unsigned rank, unsigned m_max, b2_ksplit **out);
int b2_ksplit_export(const b2_ksplit *, unsigned char blob[B2_KSPLIT_BLOB_BYTES]);
int b2_ksplit_connect(b2_ksplit *, const unsigned char *blobs /* world x B2_KSPLIT_BLOB_BYTES */);
/* First row and row count of Y that this rank writes for a round of m rows. */
int b2_ksplit_rows(const b2_ksplit *, unsigned m, unsigned *row0, unsigned *rows);
int b2_ksplit_run(b2_ksplit *, unsigned m, const void *x, size_t ldx, void *y, size_t ldy);
/* Phase timing of rounds (no counterpart in the reference; the reference's probes time whole
 * submits). While enabled, every b2_ksplit_run records four CUDA timing events on the handle's
 * stream: round start, GEMM done (including its stores into the owners' memory), signal done,
 * reduction done. b2_ksplit_phase_ms waits for the last round's reduction and returns the three
 * device intervals in milliseconds: ms[0] GEMM + NVLink stores, ms[1] signal, ms[2] the wait for
 * every rank's signal + the reduction and epilogue of the owned rows. Disabling frees the events. */
int b2_ksplit_set_timing(b2_ksplit *, int enable);
int b2_ksplit_phase_ms(b2_ksplit *, float ms[3]);
void b2_ksplit_destroy(b2_ksplit *);

/* ----------------------------------------------------------------------- fault injection */
enum b2_fault {
    B2_FAULT_NONE = 0,
    B2_FAULT_ALLOC = 1,      /* the nth device allocation from now fails (ROCKET_E_NOMEM) */
    B2_FAULT_LAUNCH = 2,     /* the nth kernel launch from now is refused (ROCKET_E_DEVICE) */
    B2_FAULT_NAN_OUTPUT = 3, /* the nth op run from now reports a non-finite output */
};
/* Host-side seam only: nothing is done to the GPU. nth >= 1; kind NONE disarms. */
void b2_fault_inject(enum b2_fault kind, unsigned nth);

#ifdef __cplusplus
}
#endif
#endif
