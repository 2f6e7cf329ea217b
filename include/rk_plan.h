/* rk_plan.h -- the plan/workspace ABI (RKPlan) on B200.
 *
 * Replaces research/custom-ops/include/rk_plan.h (reference project), the second drop-in surface
 * of the reference's custom-ops library: a planner describes values (caller bindings), buffers
 * (device allocations grouped in slots), views (tensor geometry inside a buffer), actions (host
 * uploads, device tasks, downloads), submits (groups of device tasks) and publish entries (where
 * each downloaded tile lands in an output binding). rk_plan_create verifies the description,
 * rk_workspace_create allocates and fills constants, rk_workspace_run executes it and publishes the
 * outputs only after every check passed.
 *
 * The descriptor structs, enum values and status codes are the reference's (rk_plan.h:11-374),
 * so descriptors built for the reference load unchanged. On B200:
 *   - a device task runs as one CUDA kernel over its views' physical layouts (C2=8 cube, 16x32
 *     weight blocks, linear), with the numerics of the reference's host model of the NPU
 *     (research/custom-ops/tests/mock/npu_mock.c): matmuls sum in double over the physical K
 *     and round once to FP16; element-wise ops and activations are exact and round once;
 *   - submits group tasks for accounting; tasks run in plan order on the device handle's stream;
 *   - the fd is a device handle from rocket_open();
 *   - implemented: plan create/destroy, workspace create/run/run_ex/run_group/destroy, the
 *     persistent-upload helpers, rk_abi_version, rk_target_check; the NPU-specific diagnostics
 *     (command-buffer decode, program and multi-submit caches, shared packed constants, board
 *     compatible strings) return RK_E_UNSUPPORTED.
 */
#ifndef RK_PLAN_H
#define RK_PLAN_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RK_ABI_VERSION 1u
#define RK_SCHEMA_VERSION 2u
#define RK_MAX_SUBMIT_TASKS 64u
#define RK_MAX_PROGRAMS_PER_SUBMIT 64u
#define RK_MAX_WORDS_PER_PROGRAM 2048u
#define RK_MAX_INDEPENDENT_MM_TASKS 32u
#define RK_INDEPENDENT_MM_ROWS 16u
#define RK_INDEPENDENT_MM_COLS 16u
#define RK_INDEPENDENT_MM_K 16u
#define RK_INDEPENDENT_MM_PHYS_COLS 32u
#define RK_MAX_WRITERS_PER_BUFFER 64u
#define RK_MAX_ACTION_ARGS 8u
#define RK_MAX_ACTION_DEPS 64u
#define RK_MAX_BUFFERS_PER_SLOT 64u
#define RK_DIAG_STAGE_LEN 32u
#define RK_DIAG_MESSAGE_LEN 512u
#define RK_DIAG_SOURCE_LEN 128u
#define RK_DIAG_PROFILE_LEN 64u
#define RK_ORIGIN_LEN 64u

enum rk_status {
    RK_E_INVALID = -1,
    RK_E_UNSUPPORTED = -2,
    RK_E_SHAPE = -3,
    RK_E_NUMERIC_CONTRACT = -4,
    RK_E_BUDGET = -5,
    RK_E_TARGET_MISMATCH = -6,
    RK_E_ALIAS = -7,
    RK_E_NOMEM = -8,
    RK_E_DEVICE = -9,
    RK_E_BUSY = -10,
    RK_E_POISONED = -11,
    RK_E_SCHEMA = -12,
    RK_E_DOMAIN = -13
};

enum rk_role {
    RK_ROLE_INPUT = 0,
    RK_ROLE_CONSTANT = 1,
    RK_ROLE_OUTPUT = 2,
    RK_ROLE_SCRATCH = 3,
    RK_ROLE_INPUT_SLICE = 4,
    RK_ROLE_WEIGHT = 5,
    RK_ROLE_ACCUMULATOR = 6,
    RK_ROLE_GATE = 7,
    RK_ROLE_IDENTITY = 8,
    RK_ROLE_STATE = 9
};

enum rk_dtype { RK_DTYPE_F16 = 0 };
enum rk_layout { RK_LAYOUT_CUBE_F16 = 1, RK_LAYOUT_WEIGHT_F16 = 2, RK_LAYOUT_LINEAR_F16 = 3 };
enum rk_action_kind {
    RK_ACTION_HOST_PACK = 1,
    RK_ACTION_HOST_EXPAND = 2,
    RK_ACTION_HOST_CHECK = 3,
    RK_ACTION_UPLOAD = 4,
    RK_ACTION_NPU_TASK = 5,
    RK_ACTION_DOWNLOAD = 6,
    RK_ACTION_HOST_COMPUTE = 7,
    RK_ACTION_COMMIT = 8
};
enum rk_template_id {
    RK_TEMPLATE_MM_F16 = 1,           /* y = x w^T                      inputs (x cube, w weight)      */
    RK_TEMPLATE_MM_ACC_F16 = 2,       /* y = x w^T + acc                inputs (x, w, acc cube)        */
    RK_TEMPLATE_EW_ADD_F16 = 3,       /* y = x + operand                inputs (x, operand, identity)  */
    RK_TEMPLATE_EW_MUL_F16 = 4,       /* y = x * operand                                               */
    RK_TEMPLATE_LUT_SIGMOID_F16 = 5,  /* y = 1 / (1 + exp(-x))          input x                        */
    RK_TEMPLATE_LUT_HARDSIGMOID_F16 = 6,
    RK_TEMPLATE_LUT_GELU_GATE_F16 = 7,
    RK_TEMPLATE_EW_MAX_F16 = 8,
    RK_TEMPLATE_EW_ADD_RELU_F16 = 9,
    RK_TEMPLATE_LUT_RSQRT_F16 = 10    /* y = 1 / sqrt(max(x, 0.125))                                   */
};
enum rk_act_kind { RK_ACT_NONE = 0, RK_ACT_SIGMOID = 1, RK_ACT_HARDSIGMOID = 2, RK_ACT_GELU_GATE = 3 };
enum rk_submit_mode { RK_SUBMIT_CHAIN = 0, RK_SUBMIT_SEPARATE = 1 };
enum rk_core_policy { RK_CORE_SINGLE = 0, RK_CORE_AUTO = 1 };

/* Action flags. */
#define RK_ACTION_FLAG_TRANSPOSE_SOURCE 1u   /* upload: destination (r, c) reads source (c, r) */
#define RK_ACTION_FLAG_CACHE_CONSTANT 2u     /* upload of a constant: packed once, at workspace creation */
#define RK_ACTION_FLAG_BROADCAST_SCALAR 4u   /* upload: the one-element source fills the destination */
#define RK_ACTION_FLAG_BROADCAST_CHANNEL 8u  /* upload: source element col_offset + c fills column c */
#define RK_ACTION_FLAG_DATA_REUSE 16u        /* NPU register hints: accepted, no effect on B200 */
#define RK_ACTION_FLAG_WEIGHT_REUSE 32u

/* ------------------------------------------------------------------ descriptors (rk_plan.h:110-243)
 * Every struct starts with abi_version = RK_ABI_VERSION and struct_size = sizeof(struct). */
typedef struct rk_diag {
    uint32_t abi_version;
    uint32_t struct_size;
    int32_t code;                      /* the rk_status returned, 0 on success */
    int32_t native_status;             /* the ROCKET_E_* / CUDA-side status behind it, if any */
    uint32_t action_id;
    uint32_t has_action;
    char stage[RK_DIAG_STAGE_LEN];     /* "validate", "workspace_create", "run", ... */
    char message[RK_DIAG_MESSAGE_LEN];
    char source[RK_DIAG_SOURCE_LEN];   /* the failing action's origin string */
    char profile[RK_DIAG_PROFILE_LEN];
} rk_diag;

/* A caller binding: rank 2 [rows, cols] for inputs and outputs; constants may be rank 0 (one
 * element) or rank 1 [N] when an upload broadcasts them. */
typedef struct rk_value_desc {
    uint32_t abi_version;
    uint32_t struct_size;
    uint32_t id;                       /* == index in the values array */
    uint32_t role;                     /* RK_ROLE_INPUT / CONSTANT / OUTPUT (others: internal) */
    uint32_t dtype;
    uint32_t rank;
    uint32_t shape[2];                 /* each <= 4096 */
    uint64_t nbytes;
    const char *name;                  /* not NUL terminated; unique within the plan */
    uint32_t name_len;
    uint32_t reserved;
} rk_value_desc;

/* Geometry of one device tile, exactly as co_tensor_matrix / co_tensor_weight /
 * co_tensor_linear produce it:
 *   CUBE    atom 8,  physical_rows = round4(max(rows, 12)), physical_cols = round32(cols) <= 4096
 *   WEIGHT  atom 32, physical_rows = round32(rows),        physical_cols = round32(cols)
 *   LINEAR  atom 1,  physical_rows = 1,                    physical_cols = cols
 * bytes = physical_rows * physical_cols * 2. */
typedef struct rk_tensor_desc {
    uint32_t abi_version;
    uint32_t struct_size;
    uint32_t dtype;
    uint32_t layout;
    uint32_t rows;
    uint32_t cols;
    uint32_t physical_rows;
    uint32_t physical_cols;
    uint32_t atom;
    uint32_t reserved;
    uint64_t bytes;
} rk_tensor_desc;

/* A logical device buffer: [offset, offset + capacity) of allocation slot slot_id. Buffers that
 * share a slot must have disjoint live ranges. */
typedef struct rk_buffer_desc {
    uint32_t abi_version;
    uint32_t struct_size;
    uint32_t id;
    uint32_t role;
    uint32_t slot_id;
    uint32_t alignment;                /* power of two >= 16 */
    uint32_t layout_id;
    uint32_t padding_state;
    uint32_t lifetime_first;
    uint32_t lifetime_last;
    uint64_t offset;
    uint64_t capacity;
} rk_buffer_desc;

typedef struct rk_view_desc {
    uint32_t abi_version;
    uint32_t struct_size;
    uint32_t id;
    uint32_t buffer_id;
    uint64_t offset_bytes;             /* multiple of 16 */
    uint32_t valid_region[4];          /* row0, rows, col0, cols */
    rk_tensor_desc tensor;
} rk_view_desc;

/* UPLOAD: no inputs, one output view; packs the source binding's window (source_row_offset,
 *         source_col_offset, row stride source_row_stride elements) into the view.
 * NPU_TASK: template_id with its inputs (see enum rk_template_id) and one output view.
 * DOWNLOAD: one input view, published into output binding source_binding. */
typedef struct rk_action_desc {
    uint32_t abi_version;
    uint32_t struct_size;
    uint32_t id;                       /* == index; actions run in id order */
    uint32_t kind;
    uint32_t template_id;
    uint32_t ninputs;
    uint32_t noutputs;
    uint32_t ndeps;                    /* deps[i] < id */
    uint32_t source_binding;
    uint32_t source_row_offset;
    uint32_t source_col_offset;
    uint32_t source_row_stride;
    uint32_t source_k0;
    uint32_t source_k_index;
    uint32_t source_k_count;
    uint32_t flags;
    uint32_t act_kind;
    const uint32_t *inputs;
    const uint32_t *outputs;
    const uint32_t *deps;
    char origin[RK_ORIGIN_LEN];        /* NUL terminated */
} rk_action_desc;

/* A group of device tasks: an ascending, contiguous run of NPU_TASK action ids. */
typedef struct rk_submit_desc {
    uint32_t abi_version;
    uint32_t struct_size;
    uint32_t id;
    uint32_t mode;
    uint32_t core_policy;
    uint32_t ntask_ids;
    uint32_t ndeps;
    const uint32_t *task_ids;
    const uint32_t *deps;
} rk_submit_desc;

/* One downloaded tile of an output binding: the view's logical rows x cols land at
 * (dst_row_offset, dst_col_offset) of the row-major output. The tiles of a binding do not
 * overlap and cover it exactly. */
typedef struct rk_publish_desc {
    uint32_t abi_version;
    uint32_t struct_size;
    uint32_t binding_id;
    uint32_t view_id;
    uint32_t dst_row_offset;
    uint32_t dst_col_offset;
    uint32_t rows;
    uint32_t cols;
} rk_publish_desc;

typedef struct rk_plan_desc {
    uint32_t abi_version;
    uint32_t struct_size;
    uint32_t schema_version;           /* RK_SCHEMA_VERSION */
    uint32_t flags;
    uint64_t profile_hash;
    uint64_t source_hash;
    const rk_value_desc *values;
    uint32_t nvalues;
    uint32_t reserved0;
    const rk_buffer_desc *buffers;
    uint32_t nbuffers;
    uint32_t reserved1;
    const rk_view_desc *views;
    uint32_t nviews;
    uint32_t reserved2;
    const rk_action_desc *actions;
    uint32_t nactions;
    uint32_t reserved3;
    const rk_submit_desc *submits;
    uint32_t nsubmits;
    uint32_t reserved4;
    const rk_publish_desc *publish;
    uint32_t npublish;
    uint32_t reserved5;
    uint64_t device_budget_bytes;      /* 0: no budget */
    uint64_t host_budget_bytes;
    uint64_t claimed_device_bytes;     /* must cover slots + slack/guard + task descriptors */
    uint64_t claimed_host_bytes;       /* must cover bindings + staging + run scratch */
    uint32_t runtime_abi_version;      /* == RK_ABI_VERSION of the loaded library */
    uint32_t reserved6;
} rk_plan_desc;

typedef struct rk_binding {
    uint32_t abi_version;
    uint32_t struct_size;
    uint32_t id;                       /* value id */
    uint32_t dtype;
    uint32_t rank;
    uint32_t shape[2];
    const void *data;                  /* host memory, row-major FP16 */
    uint64_t nbytes;
} rk_binding;

/* ------------------------------------------------------------------ run reports (rk_plan.h:245-390)
 * rk_workspace_run writes exactly sizeof(rk_run_report). The _ex and _group entries require
 * struct_size within [V1 size, sizeof] and write only that many bytes. Times are host envelopes
 * in microseconds; on B200 pack_us covers the host-to-device copies and the pack kernel launch,
 * submit_wait_us the device schedule up to its completion, download_us the device-to-host copy
 * and the finiteness scan, emit_us / command_us / submit_alloc_us are 0 (no command buffers). */
typedef struct rk_run_report {
    uint32_t abi_version;
    uint32_t struct_size;
    uint32_t task_count;               /* device tasks of the plan (sum over submits) */
    uint32_t submit_count;             /* submits executed */
    uint32_t fail_action_id;           /* UINT32_MAX unless an action failed */
    uint32_t numeric_mode;             /* 1: FP16 storage, exact accumulation rounded once */
    uint64_t upload_calls;             /* per-run uploads executed (constants are not re-run) */
    uint64_t upload_bytes;             /* packed destination bytes */
    uint64_t download_calls;
    uint64_t download_bytes;           /* physical bytes of the downloaded views */
    double pack_us;
    double emit_us;
    double submit_wait_us;
    double output_sync_us;
} rk_run_report;

typedef struct rk_run_attribution {
    uint32_t abi_version;
    uint32_t struct_size;
    uint32_t task_count;
    uint32_t submit_count;
    uint32_t fail_action_id;
    uint32_t numeric_mode;
    uint64_t upload_calls;
    uint64_t upload_bytes;
    uint64_t download_calls;
    uint64_t download_bytes;
    double validate_us;
    double pack_us;
    double emit_us;
    double command_us;
    double submit_alloc_us;
    double submit_wait_us;
    double output_sync_us;
    double download_us;
    double guard_us;
    double publish_us;
    double alloc_us;
    double total_us;
    double clock_us;
    double pack_prep_us;
    double pack_clear_us;
    double pack_layout_us;
    double pack_fini_us;
    uint64_t pack_prep_calls;
    uint64_t pack_fini_calls;
    uint32_t upload_coalesce;
    uint32_t upload_fast_pack;
    uint32_t upload_policy_reserved[2];
} rk_run_attribution;

#define RK_RUN_ATTRIBUTION_V1_SIZE \
    ((uint32_t)(offsetof(rk_run_attribution, clock_us) + sizeof(double)))
#define RK_RUN_ATTRIBUTION_V2_SIZE \
    ((uint32_t)(offsetof(rk_run_attribution, upload_coalesce)))
#define RK_RUN_ATTRIBUTION_V3_SIZE ((uint32_t)sizeof(rk_run_attribution))

typedef struct rk_group_report {
    uint32_t abi_version;
    uint32_t struct_size;
    uint32_t repeat_count;
    uint32_t repeat_completed;
    uint32_t fail_repeat;
    uint32_t fail_action_id;
    uint32_t task_count;
    uint32_t submit_count;
    uint32_t numeric_mode;
    uint32_t reserved0;
    uint64_t upload_calls;
    uint64_t upload_bytes;
    uint64_t download_calls;
    uint64_t download_bytes;
    double validate_us;
    double pack_us;
    double emit_us;
    double command_us;
    double submit_alloc_us;
    double submit_wait_us;
    double output_sync_us;
    double download_us;
    double guard_us;
    double publish_us;
    double alloc_us;
    double total_us;
    double clock_us;
} rk_group_report;

#define RK_GROUP_REPORT_V1_SIZE \
    ((uint32_t)(offsetof(rk_group_report, clock_us) + sizeof(double)))

typedef struct rk_plan rk_plan;
typedef struct rk_workspace rk_workspace;

/* rk_plan.h:396-414: command/program cache state of the NPU runtime. On B200 every field is
 * 0 except nsubmits, device_bytes (slot allocations) and host_bytes (workspace host scratch). */
typedef struct {
    uint32_t nsubmits;
    uint32_t program_cache_requested;
    uint32_t program_cache_ready;
    uint32_t command_cache_requested;
    uint32_t command_cache_ready;
    uint32_t multi_submit_requested;
    uint32_t multi_submit_ready;
    uint32_t multi_submit_cached;
    uint32_t program_cache_submit;
    uint32_t program_cache_tasks;
    uint32_t command_plan_present;
    uint32_t submit_cache_present;
    uint64_t host_bytes;
    uint64_t device_bytes;
    uint32_t skipped_budget;
    uint32_t skipped_static;
} rk_workspace_cache_info;

typedef struct {
    uint32_t action_id;
    uint32_t task_count;
    uint32_t cbuf_writes;
    uint32_t data_reuse_tasks;
    uint32_t weight_reuse_tasks;
    uint32_t first_reuse_task;
    uint32_t first_cbuf_con0;
} rk_task_cbuf_info;

typedef struct rk_shared_constant rk_shared_constant;
typedef struct rk_shared_constant_binding {
    uint32_t action_id;
    uint32_t reserved;
    rk_shared_constant *constant;
} rk_shared_constant_binding;

#define RK_STATE_SOURCE_TRANSPOSE 1u
typedef struct rk_state_source {
    const void *data;
    uint64_t nbytes;
    uint32_t row_stride;               /* elements */
    uint32_t flags;                    /* RK_STATE_SOURCE_TRANSPOSE or 0 */
} rk_state_source;

/* ------------------------------------------------------------------ entry points (rk_plan.h:396-572) */

/* RK_ABI_VERSION of this library. */
uint32_t rk_abi_version(void);
/* Target identity: 0 when a CUDA device is visible to the process, else RK_E_TARGET_MISMATCH
 * (the reference compares the board's compatible string and driver version). */
int rk_target_check(rk_diag *diag);
/* The board compatible-string parser of the NPU build: RK_E_UNSUPPORTED. */
int rk_target_validate_text(const char *compat, size_t compat_len, const char *version,
                            rk_diag *diag);

/* Verifies `desc` and deep-copies it (the caller's arrays may be freed afterwards). On failure
 * *out = NULL and diag names the stage, the rule and the action. Codes: RK_E_SCHEMA (ids,
 * structure, ordering), RK_E_SHAPE (geometry, coverage), RK_E_ALIAS (overlapping writers, slots
 * shared by live buffers), RK_E_BUDGET, RK_E_UNSUPPORTED (action kinds), RK_E_NUMERIC_CONTRACT. */
int rk_plan_create(const rk_plan_desc *desc, rk_plan **out, rk_diag *diag);
void rk_plan_destroy(rk_plan *plan);

/* Allocates one HBM region per slot (capacity + CO_SLACK zero bytes + CO_GUARD guard bytes) on
 * device handle `fd` (rocket_open) and packs every constant-sourced upload once. `constants`
 * holds exactly the plan's constant values (finite FP16). */
int rk_workspace_create(int fd, const rk_plan *plan, const rk_binding *constants,
                        uint32_t nconstants, rk_workspace **out, rk_diag *diag);
/* Shared packed constants are an NPU buffer-object cache: RK_E_UNSUPPORTED when nshared > 0,
 * otherwise rk_workspace_create. */
int rk_workspace_create_shared(int fd, const rk_plan *plan, const rk_binding *constants,
                               uint32_t nconstants, const rk_shared_constant_binding *shared,
                               uint32_t nshared, rk_workspace **out, rk_diag *diag);

/* One run: checks the bindings (count, shape, finiteness of inputs, host-range overlap), uploads,
 * runs the device tasks in action order, downloads, checks every downloaded logical element is
 * finite and every slot's slack/guard bytes are intact, and only then writes the outputs.
 * On any failure no output byte is written. RK_E_BUSY when another run holds the workspace,
 * RK_E_POISONED after a device error. */
int rk_workspace_run(rk_workspace *ws, const rk_binding *inputs, uint32_t ninputs,
                     const rk_binding *outputs, uint32_t noutputs, rk_run_report *report,
                     rk_diag *diag);
/* nrepeat binding sets (inputs then outputs, each in value-id order) in one call; outputs are
 * published only after every repeat succeeded and the guard gate passed. */
int rk_workspace_run_group(rk_workspace *ws, const rk_binding *bindings, uint32_t nrepeat,
                           rk_group_report *report, rk_diag *diag);
int rk_workspace_run_ex(rk_workspace *ws, const rk_binding *inputs, uint32_t ninputs,
                        const rk_binding *outputs, uint32_t noutputs,
                        rk_run_attribution *envelope, rk_diag *diag);
int rk_workspace_destroy(rk_workspace *ws, rk_diag *diag);

/* Persistent uploads: the nominated upload action is no longer re-packed by each run; the
 * caller fills its destination with update_upload_region (source rectangle -> destination
 * logical rectangle, same transpose convention, untouched bytes kept) and zeroes it with
 * clear_upload_destination. */
int rk_workspace_set_persistent_upload(rk_workspace *ws, uint32_t action_id, rk_diag *diag);
int rk_workspace_update_upload_region(rk_workspace *ws, uint32_t action_id,
                                      const rk_state_source *source, uint32_t src_row,
                                      uint32_t src_col, uint32_t dst_row, uint32_t dst_col,
                                      uint32_t rows, uint32_t cols, rk_diag *diag);
int rk_workspace_clear_upload_destination(rk_workspace *ws, uint32_t action_id, rk_diag *diag);

int rk_workspace_get_cache_info(rk_workspace *ws, rk_workspace_cache_info *out, rk_diag *diag);
/* NPU command-buffer decode: RK_E_UNSUPPORTED. */
int rk_workspace_task_cbuf(rk_workspace *ws, uint32_t action_id, uint32_t *values,
                           uint32_t capacity, rk_task_cbuf_info *out, rk_diag *diag);

/* NPU shared packed-constant cache: get_or_create returns RK_E_UNSUPPORTED, the others are
 * no-ops / 0. */
int rk_shared_constant_get_or_create(int fd, const rk_plan *plan, uint32_t action_id,
                                     const rk_binding *source, const char *key,
                                     rk_shared_constant **out, uint32_t *created, rk_diag *diag);
void rk_shared_constant_retain(rk_shared_constant *constant);
void rk_shared_constant_release(rk_shared_constant *constant);
uint64_t rk_shared_constant_bytes(const rk_shared_constant *constant);
uint32_t rk_shared_constant_live(void);

#ifdef __cplusplus
}
#endif
#endif
