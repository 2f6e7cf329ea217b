/* custom_ops.h -- operator-level C API of the FP16 Linear / fused HardSigmoid path, B200 build.
 *
 * Drop-in for the Linear subset of research/custom-ops/include/custom_ops.h (reference project):
 * the same enums, descriptor structs, limits, plan functions, tensor/view helpers and the
 * co_linear_* / co_linear_hsig_* entry points, with the same argument meaning and the same
 * status codes. Each declaration below cites the reference declaration it replaces.
 *
 * Numerics: Y[M,N] = act(X[M,K] * W[N,K]^T + b[N]), FP16 in and out. The default accumulation is
 * the reference's shipped one: every 256-wide K tile is reduced (here in FP32 on the tensor
 * cores), the running sum is narrowed to FP16 after each tile, bias is added with an FP16 result,
 * then HardSigmoid clamp(v/6 + 0.5, 0, 1) is applied and rounded to FP16
 * (reference custom_ops.h:131-138). b2_linear.h selects full-K FP32
 * accumulation instead.
 *
 * Layouts: host matrices are row-major little-endian IEEE FP16. Device "cubes" keep the
 * reference's C2=8 layout [ceil32(cols)/8][physical_rows][8] (custom_ops.c:18-33,80-85).
 *
 * Differences from the reference (by design, B200-first):
 *   - Buffers live in HBM; a co_view may sit anywhere in the device address space (the
 *     reference's 32-bit DMA window does not apply). Views must still be 16-byte aligned.
 *   - One op run is a handful of CUDA launches on the handle's stream, not one chained submit
 *     per output tile; the plan's task/submit counts are kept as metadata.
 *   - co_linear_plan.device_bytes is the HBM the B200 context actually allocates (weights,
 *     bias, staging); the budget check keeps the reference's semantics against that number.
 */
#ifndef CUSTOM_OPS_H
#define CUSTOM_OPS_H
#include "rocket_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* reference custom_ops.h:11-14 */
enum co_type { CO_F16, CO_F32 };
enum co_layout { CO_CUBE, CO_WEIGHT, CO_LINEAR };
enum co_act { CO_HARDSIGMOID, CO_SIGMOID, CO_GELU_GATE, CO_EXP_BOUNDED, CO_RSQRT_BOUNDED, CO_EXP_NEG4 };
enum co_mode { CO_SEPARATE, CO_CHAIN };

/* reference custom_ops.h:15-24 */
#define CO_MAX_WORDS 2048
#define CO_MAX_PROGRAMS 64
#define CO_MAX_K 4096u
#define CO_K_TILE 256u
#define CO_K_TILES ((CO_MAX_K + CO_K_TILE - 1u) / CO_K_TILE)
#define CO_SLACK 32768u
#define CO_GUARD 64u

/* reference custom_ops.h:26-33 */
typedef struct {
    enum co_type type;
    enum co_layout layout;
    unsigned rows, cols;                 /* logical rows / columns */
    unsigned physical_rows, physical_cols;
    unsigned atom;                       /* 8 fp16 or 4 fp32 elements */
    size_t bytes;
} co_tensor;

/* reference custom_ops.h:35-36 */
typedef struct { rocket_bo bo; int fd; size_t payload; } co_buffer;
typedef struct { co_buffer *buffer; size_t offset; co_tensor tensor; } co_view;

/* reference custom_ops.h:44-75: descriptors, buffers, views, host<->device transfers */
int co_tensor_matrix(co_tensor *, unsigned rows, unsigned cols, enum co_type);
int co_tensor_input(co_tensor *, unsigned rows, unsigned cols);
int co_tensor_weight(co_tensor *, unsigned outputs, unsigned inputs);
unsigned co_k_tiles(unsigned k);
unsigned co_k_tile_length(unsigned k, unsigned index);
size_t co_k_tile_offset(const co_tensor *full, unsigned k0);
int co_tensor_input_slice(co_tensor *slice, const co_tensor *full,
                          unsigned k0, unsigned kt, size_t *offset);
int co_tensor_spatial(co_tensor *, unsigned channels, unsigned h, unsigned w);
int co_tensor_linear(co_tensor *, unsigned elements);
size_t co_index(const co_tensor *, unsigned row, unsigned col);
/* Device buffer of `payload` bytes plus CO_SLACK zero bytes and a CO_GUARD tail of 0xA5. */
int co_buffer_alloc(int fd, size_t payload, co_buffer *);
void co_buffer_free(co_buffer *);
int co_view_init(co_view *, co_buffer *, size_t offset, const co_tensor *);
/* Row-major host FP16 -> device view layout (padding zeroed), synchronous. */
int co_upload_f16(co_view *, const _Float16 *row_major);
/* Device view -> row-major host (FP16 or FP32 per tensor.type), synchronous. */
int co_download(co_view *, void *row_major);
int co_sentinel(co_buffer *);                /* payload=NaN bits, tail guard=0xA5 */
int co_guard_check(co_buffer *);             /* slack all zero and guard intact, else E_DEVICE */
int co_copy(co_view *dst, co_view *src);
int co_bias_upload(co_view *, const _Float16 *per_column_bias);
int co_identity_upload(co_view *weights);
int co_ones_upload(co_view *weights, unsigned logical_k, int mean);

/* reference custom_ops.h:145-168: shape limits and plan */
#define CO_MAX_M 4096u
#define CO_MAX_N 4096u
#define CO_LINEAR_DEVICE_BUDGET (256u * 1024u * 1024u)
typedef struct {
    unsigned m, k, n, mtiles, ktiles, ntiles, output_tiles;
    unsigned has_bias, post;
    unsigned row_classes; /* one full row shape plus an optional ragged tail */
    size_t device_bytes;
    unsigned long long tasks, chain_submits;
} co_linear_plan;
typedef struct {
    unsigned m0, n0, rows, cols, ktiles, programs;
} co_linear_tile_info;
int co_linear_plan_init(co_linear_plan *, unsigned m, unsigned k, unsigned n,
                        size_t device_budget);
int co_linear_plan_tile(const co_linear_plan *, unsigned index, co_linear_tile_info *);
enum co_linear_post { CO_LINEAR_NONE, CO_LINEAR_HSIG };
int co_linear_plan_init_ex(co_linear_plan *, unsigned m, unsigned k, unsigned n,
                           int has_bias, enum co_linear_post, size_t device_budget);

/* reference custom_ops.h:169-183: generic Linear */
typedef struct co_linear_hsig co_linear;
int co_linear_create(int fd, unsigned m, unsigned k, unsigned n,
                     const _Float16 *weights, const _Float16 *optional_bias,
                     enum co_linear_post, enum co_mode, co_linear **out);
/* Host row-major X[M,K] -> Y[M,N]; Y is written only when the whole run succeeded. */
int co_linear_run(co_linear *, const _Float16 *x, _Float16 *y);
/* inputs[mtiles*ktiles]: co_tensor_matrix(tile_rows, k_tile_len, F16) cubes, row-block-major;
 * outputs[mtiles*ntiles]: co_tensor_matrix(tile_rows, tile_cols, F16) cubes. */
int co_linear_run_tiled(co_linear *, const co_view *inputs, unsigned ninputs,
                        const co_view *outputs, unsigned noutputs);
int co_linear_update_weights(co_linear *, const _Float16 *weights, const _Float16 *bias);
void co_linear_destroy(co_linear *);

/* reference custom_ops.h:184-206: HardSigmoid operator (bias required) */
typedef struct co_linear_hsig co_linear_hsig;
int co_linear_hsig_create(int fd, unsigned m, unsigned k, unsigned n,
                          const _Float16 *weights, const _Float16 *bias,
                          enum co_mode mode, co_linear_hsig **out);
int co_linear_hsig_run(co_linear_hsig *, const _Float16 *x, _Float16 *y);
/* Single-output-tile cube entry (M,N <= 256), else ROCKET_E_UNSUPPORTED. x: co_tensor_input(M,K)
 * cube; y: co_tensor_matrix(M,N,F16) cube. */
int co_linear_hsig_run_cube(co_linear_hsig *, co_view x, co_view y);
/* inputs[mtiles]: co_tensor_input(rows,K); outputs[output_tiles]: co_tensor_matrix(rows,cols),
 * M-major/N-minor. All views and aliases are checked before any launch. */
int co_linear_hsig_run_tiles(co_linear_hsig *, const co_view *inputs, unsigned ninputs,
                             const co_view *outputs, unsigned noutputs);
void co_linear_hsig_destroy(co_linear_hsig *);

#ifdef __cplusplus
}
#endif
#endif
