/* co_graph.h -- static FP16 graph compiler over the Linear path, B200 build.
 *
 * Drop-in for research/custom-ops/include/co_graph.h (reference project): the same node, desc,
 * plan and input/output structs, the same limits, functions, argument meaning and status codes
 * for the node kinds built here:
 *   INPUT, LINEAR (Y = X W^T + b with the per-256-K FP16 fold of co_linear_*), ADD, MUL,
 *   SILU / GELU (y = fp16(x * fp16(gate(x)))), HSIG, RMSNORM.
 * SOFTMAX, ROPE and ATTENTION nodes (the reference's hybrid row, rotary and attention operators)
 * are not built: a graph that reaches one is rejected by planning with ROCKET_E_UNSUPPORTED.
 *
 * B200 design instead of 256x256 NPU tiles and per-tile programs:
 *   - every tensor is one row-major FP16 matrix in HBM with a 16-byte row pitch; slots are reused
 *     by liveness with the reference's rule (a slot is free once its tensor's last use is
 *     strictly earlier);
 *   - CO_CHAIN compiles a fused program: a SiLU/GELU of one Linear multiplied by another Linear of
 *     the same input (the SwiGLU/GeGLU FFN) runs as ONE tcgen05 GEMM over the packed gate|up
 *     weight whose epilogue forms fp16(fp16(g * fp16(gate(g))) * u); a Linear whose only use is
 *     an ADD runs with the residual added in its epilogue; the program is recorded once as a CUDA
 *     graph and replayed per run. CO_SEPARATE runs one kernel (or Linear) per node. Both give the
 *     same bytes;
 *   - RMSNorm runs on the device (no host statistics round trip).
 * Plan fields that describe NPU resources keep their names with the B200 meaning noted below.
 */
#ifndef CO_GRAPH_H
#define CO_GRAPH_H
#include "custom_ops.h"

#ifdef __cplusplus
extern "C" {
#endif

/* reference co_rope.h:5 (the graph node carries it) */
#ifndef CO_ROPE_STYLE_DEFINED
#define CO_ROPE_STYLE_DEFINED
enum co_rope_style { CO_ROPE_INTERLEAVED, CO_ROPE_SPLIT_HALF };
#endif

/* reference co_graph.h:6-39 */
#define CO_GRAPH_MAX_NODES 64u
#define CO_GRAPH_NO_NODE UINT32_MAX
enum co_graph_op { CO_GRAPH_INPUT, CO_GRAPH_LINEAR, CO_GRAPH_ADD, CO_GRAPH_MUL,
                   CO_GRAPH_SILU, CO_GRAPH_GELU, CO_GRAPH_HSIG,
                   CO_GRAPH_RMSNORM, CO_GRAPH_SOFTMAX, CO_GRAPH_ROPE, CO_GRAPH_ATTENTION };
#define CO_GRAPH_ALLOW_NEG_INF 1u /* Input only; Softmax scores or Attention mask only */
typedef struct {
    enum co_graph_op op;
    unsigned a, b, rows, cols;
    unsigned c, mask_node, has_mask;
    const _Float16 *weights, *bias;       /* Linear: row-major [cols, in], optional bias [cols] */
    const _Float16 *gamma;                /* RMSNorm gamma[cols], copied at compile */
    float epsilon;                        /* RMSNorm: finite and positive */
    unsigned flags;
    unsigned heads, kv_heads, head_dim, rotary_dim;
    float theta, scale;
    enum co_rope_style rope_style;
    uint32_t position_base;
    int causal;
    unsigned window;
} co_graph_node;
typedef struct {
    const co_graph_node *nodes;
    unsigned count, output;
    size_t device_budget;                 /* 0 = default 256 MiB (CO_LINEAR_DEVICE_BUDGET) */
} co_graph_desc;
/* Per tensor: rows, cols; tiles = its 256x256 tile count (kept for callers that size per-tile
 * work); slot; first/last step; bytes = rows * roundup(cols, 8) * 2 (row-major in HBM). */
typedef struct {
    unsigned rows, cols, tiles, slot, first, last;
    size_t bytes;
} co_graph_tensor_plan;
/* B200 meanings: tensor_bytes = slots (+ CO_SLACK zero bytes and a CO_GUARD tail each);
 * linear_bytes = Linear weights (rows padded to 32) and biases; rowop_bytes = RMSNorm gammas;
 * workspace_bytes = the FP16 scratch of a gated Linear served by the small-M kernel;
 * rope/attention bytes, hybrid_nodes, host transfers beyond the inputs/outputs, identity_mask and
 * gate_bytes are 0 (nothing runs on the host); tasks = kernel launches of one CO_SEPARATE run,
 * chain_submits = kernels of one CO_CHAIN run (replayed as one CUDA graph). */
typedef struct {
    unsigned steps, inputs, slots, order[CO_GRAPH_MAX_NODES];
    unsigned noutputs, outputs[CO_GRAPH_MAX_NODES];
    co_graph_tensor_plan tensors[CO_GRAPH_MAX_NODES];
    size_t slot_bytes[CO_GRAPH_MAX_NODES];
    size_t tensor_bytes, linear_bytes, rowop_bytes, rope_bytes, attention_bytes, workspace_bytes, device_bytes;
    unsigned hybrid_nodes;
    unsigned long long host_upload_calls, statistic_download_calls, activation_download_calls;
    size_t host_activation_reads, statistic_downloads, activation_downloads, host_uploads;
    unsigned identity_mask;
    size_t gate_bytes;
    unsigned long long tasks, chain_submits;
} co_graph_plan;

/* reference co_graph.h:40-45: pure analysis (topology, shapes, liveness/slot reuse, HBM bytes);
 * no data reads, no device calls. */
int co_graph_plan_init(const co_graph_desc *, co_graph_plan *);
int co_graph_plan_many(const co_graph_desc *, const unsigned *outputs, unsigned count, co_graph_plan *);

/* reference co_graph.h:46-50 */
typedef struct co_graph co_graph;
int co_graph_compile(int fd, const co_graph_desc *, enum co_mode, co_graph **);
int co_graph_compile_many(int fd, const co_graph_desc *, const unsigned *outputs, unsigned count,
                          enum co_mode, co_graph **);
void co_graph_destroy(co_graph *);

/* reference co_graph.h:51-63: bind each reachable input exactly once (finite data, else
 * ROCKET_E_SHAPE before any work); outputs are published only after the whole run succeeded
 * (all finite, else ROCKET_E_DEVICE). RMSNorm rejecting a row (square sum >= 65504 in a 256-column
 * tile, or an FP16 coefficient overflow) fails the run with ROCKET_E_SHAPE. Synchronous. */
typedef struct { unsigned node; const _Float16 *data; } co_graph_input;
int co_graph_run(co_graph *, const co_graph_input *, unsigned count, _Float16 *output);
typedef struct { unsigned node; _Float16 *data; } co_graph_output;
int co_graph_run_many(co_graph *, const co_graph_input *, unsigned ninputs,
                      const co_graph_output *, unsigned noutputs);

/* ---------------------------------------------------------------------- B200 additions */
/* Device address and row pitch (elements) of a planned node's tensor in HBM. */
int b2_graph_tensor(const co_graph *, unsigned node, void **device_ptr, size_t *ld);
/* Enqueues one run of the compiled program on the handle's stream, reading the input tensors
 * where b2_graph_tensor places them: no host transfers, no wait, no checks (b2_sync, then
 * b2_graph_status). */
int b2_graph_launch(co_graph *);
/* After b2_sync: 0, or the status a synchronous run would have returned (and clears it). */
int b2_graph_status(co_graph *);
typedef struct {
    unsigned gated;          /* gate·up Linear pairs fused into one GEMM (CO_CHAIN) */
    unsigned residual;       /* Linears with the following ADD fused into the epilogue (CO_CHAIN) */
    unsigned kernels;        /* kernels per run */
    unsigned captured;       /* 1 while runs replay a recorded CUDA graph */
} b2_graph_info;
int b2_graph_get_info(const co_graph *, b2_graph_info *);

#ifdef __cplusplus
}
#endif
#endif
