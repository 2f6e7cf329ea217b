/* rkplan.c -- the plan/workspace ABI (include/rk_plan.h) on B200: verifier, plan copy, workspaces
 * and the run.
 *
 * Replaces research/custom-ops/src/rk_plan_validate.c (the verifier and clone) and
 * rk_plan_runtime.c (workspaces, runs, publication gate) of the reference project.
 *
 * The verifier enforces the reference's descriptor contract rule for rule, with the same status
 * codes and diagnostic messages (callers match on both): ABI/struct sizes, ids, value and tensor
 * geometry (rk_plan_validate.c:59-86, 913-1000), upload/download/template arity and shapes
 * (:191-463), submits as ascending contiguous task runs in submit order (:540-600), dependency
 * ancestry of every read's producer and exact byte coverage of each read by earlier declared
 * writers (:600-850), host/device writer separation and overlapping-writer addressing (:730-780),
 * slot sharing only between buffers with disjoint live ranges (:860-905), publish tiles that cover
 * each output exactly once (:1566-1640) and the device/host budget claims (:1641-1740). Left out by
 * design: the NPU's submit whitelist of hardware-validated task chains and its independent-MM
 * geometry domain (:1107-1520) -- B200 runs any verified order of tasks with the same results, so
 * those plans are accepted; CBUF reuse flags keep their structural check and have no effect.
 *
 * The run (rk_plan_runtime.c:1580-2150): binding checks (count, shape, finiteness of every input,
 * host-range overlap) before any device work; the input bindings through pinned staging as one
 * host-to-device copy into HBM; then, on the device handle's stream and in action order, one pack launch per run of
 * consecutive uploads, one launch per task and one unpack launch per run of consecutive downloads
 * (slots may be shared by buffers with disjoint live ranges, so each transfer runs at its own
 * position), replayed as one CUDA graph when the handle supports capture, the slack/guard check
 * of every slot, one device-to-host copy of the outputs; only when every downloaded element is finite and every
 * guard is intact are the caller's output buffers written. Constant uploads run once, at
 * workspace creation.
 */
#define _GNU_SOURCE
#include <math.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "b2_host.h"
#include "custom_ops.h"
#include "rk_plan.h"

/* ------------------------------------------------------------------------------ diagnostics */
static void diag_clear(rk_diag *d) {
    if (!d) return;
    memset(d, 0, sizeof(*d));
    d->abi_version = RK_ABI_VERSION;
    d->struct_size = sizeof(*d);
    d->action_id = UINT32_MAX;
}

static int diag_set(rk_diag *d, int code, const char *stage, const char *msg, uint32_t action,
                    const char *source, int native) {
    if (!d) return code;
    d->abi_version = RK_ABI_VERSION;
    d->struct_size = sizeof(*d);
    d->code = code;
    d->native_status = native;
    d->action_id = action;
    d->has_action = action != UINT32_MAX;
    snprintf(d->stage, sizeof(d->stage), "%s", stage ? stage : "");
    snprintf(d->message, sizeof(d->message), "%s", msg ? msg : "");
    snprintf(d->source, sizeof(d->source), "%s", source ? source : "");
    return code;
}

#define VFAIL(code, msg) diag_set(diag, (code), "validate", (msg), UINT32_MAX, NULL, 0)
#define AFAIL(code, msg, a) diag_set(diag, (code), "validate", (msg), (a)->id, (a)->origin, 0)

static double now_us(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return (double)t.tv_sec * 1e6 + (double)t.tv_nsec / 1e3;
}

/* ------------------------------------------------------------------------------ descriptor rules */
static int struct_ok(uint32_t abi, uint32_t size, size_t expected) {
    return abi == RK_ABI_VERSION && size == expected;
}

static uint32_t round_up32(uint32_t v, uint32_t m) { return (v + m - 1u) / m * m; }
static int is_pow2(uint32_t v) { return v && !(v & (v - 1u)); }
static int valid_layout(uint32_t l) {
    return l == RK_LAYOUT_CUBE_F16 || l == RK_LAYOUT_WEIGHT_F16 || l == RK_LAYOUT_LINEAR_F16;
}

/* The geometry co_tensor_matrix / co_tensor_weight / co_tensor_linear produce, nothing else. */
static int tensor_valid(const rk_tensor_desc *t) {
    if (!struct_ok(t->abi_version, t->struct_size, sizeof(*t))) return 0;
    if (t->dtype != RK_DTYPE_F16 || !valid_layout(t->layout)) return 0;
    if (!t->rows || !t->cols || !t->physical_rows || !t->physical_cols) return 0;
    if (t->rows > t->physical_rows || t->cols > t->physical_cols) return 0;
    if (t->physical_rows > 256 || t->physical_cols > 65520) return 0;
    if (t->layout == RK_LAYOUT_LINEAR_F16) {
        if (t->atom != 1 || t->physical_rows != 1 || t->physical_cols != t->cols) return 0;
    } else if (t->layout == RK_LAYOUT_WEIGHT_F16) {
        if (t->atom != 32 || t->physical_rows != round_up32(t->rows, 32) ||
            t->physical_cols != round_up32(t->cols, 32))
            return 0;
    } else {
        const uint32_t rows = t->rows < 12u ? 12u : t->rows;
        if (t->atom != 8 || t->physical_cols > CO_MAX_K || t->physical_rows != round_up32(rows, 4) ||
            t->physical_cols != round_up32(t->cols, 32))
            return 0;
    }
    if (t->physical_cols % t->atom) return 0;
    return t->bytes == (uint64_t)t->physical_rows * t->physical_cols * 2u;
}

static int same_tensor(const rk_tensor_desc *a, const rk_tensor_desc *b) {
    return a->dtype == b->dtype && a->layout == b->layout && a->rows == b->rows && a->cols == b->cols &&
           a->physical_rows == b->physical_rows && a->physical_cols == b->physical_cols && a->atom == b->atom &&
           a->bytes == b->bytes;
}

static int same_addressing(const rk_tensor_desc *a, const rk_tensor_desc *b) {
    return a->layout == b->layout && a->atom == b->atom && a->physical_rows == b->physical_rows &&
           a->physical_cols == b->physical_cols;
}

static int same_geometry(const rk_tensor_desc *a, const rk_tensor_desc *b) {
    return a->layout == b->layout && a->rows == b->rows && a->cols == b->cols &&
           a->physical_rows == b->physical_rows && a->physical_cols == b->physical_cols;
}

static const rk_value_desc *value_at(const rk_plan_desc *p, uint32_t id) {
    return p->values && id < p->nvalues ? &p->values[id] : NULL;
}
static const rk_buffer_desc *buffer_at(const rk_plan_desc *p, uint32_t id) {
    return p->buffers && id < p->nbuffers ? &p->buffers[id] : NULL;
}
static const rk_view_desc *view_at(const rk_plan_desc *p, uint32_t id) {
    return p->views && id < p->nviews ? &p->views[id] : NULL;
}

static int check_upload(const rk_plan_desc *p, const rk_action_desc *a, rk_diag *diag) {
    if (a->ninputs != 0 || a->noutputs != 1 || !a->outputs)
        return AFAIL(RK_E_SHAPE, "upload requires zero inputs and one output view", a);
    const rk_view_desc *out = view_at(p, a->outputs[0]);
    const rk_value_desc *src = value_at(p, a->source_binding);
    if (!out || !src) return AFAIL(RK_E_SCHEMA, "upload references missing view or binding", a);
    if (src->role != RK_ROLE_INPUT && src->role != RK_ROLE_CONSTANT)
        return AFAIL(RK_E_SHAPE, "upload source binding must be input or constant", a);
    if (src->dtype != RK_DTYPE_F16 || src->rank > 2)
        return AFAIL(RK_E_NUMERIC_CONTRACT, "upload source must be rank-0/1/2 FP16", a);
    if (!tensor_valid(&out->tensor)) return AFAIL(RK_E_SHAPE, "upload destination tensor is invalid", a);
    const int transpose = (a->flags & RK_ACTION_FLAG_TRANSPOSE_SOURCE) != 0;
    const int scalar = (a->flags & RK_ACTION_FLAG_BROADCAST_SCALAR) != 0;
    const int channel = (a->flags & RK_ACTION_FLAG_BROADCAST_CHANNEL) != 0;
    if (scalar && channel) return AFAIL(RK_E_SCHEMA, "conflicting broadcast flags", a);
    if (scalar || channel) {
        if (src->role != RK_ROLE_CONSTANT)
            return AFAIL(RK_E_UNSUPPORTED,
                         "only constants may be broadcast-expanded; runtime tensor broadcast is not supported", a);
        if (transpose || a->source_row_offset || a->source_row_stride)
            return AFAIL(RK_E_SHAPE, "broadcast upload cannot transpose or use a source row offset/stride", a);
        if (scalar) {
            if (a->source_col_offset || src->rank != 0 || src->shape[0] || src->shape[1] || src->nbytes != 2u)
                return AFAIL(RK_E_SHAPE, "scalar broadcast source must be rank-0 with one FP16 element", a);
        } else {
            if (src->rank != 1 || src->shape[1] || src->nbytes != (uint64_t)src->shape[0] * 2u)
                return AFAIL(RK_E_SHAPE, "channel broadcast source must be a rank-1 FP16 vector", a);
            if ((uint64_t)a->source_col_offset + out->tensor.cols > src->shape[0])
                return AFAIL(RK_E_SHAPE, "channel broadcast window exceeds source N", a);
        }
        return 0;
    }
    if (src->rank != 2) return AFAIL(RK_E_UNSUPPORTED, "rank-0/1 uploads require an explicit broadcast flag", a);
    if (a->source_row_stride != src->shape[1])
        return AFAIL(RK_E_SHAPE, "upload source_row_stride must equal the binding row length", a);
    const uint64_t sr = transpose ? out->tensor.cols : out->tensor.rows;
    const uint64_t sc = transpose ? out->tensor.rows : out->tensor.cols;
    if (a->source_row_offset + sr > src->shape[0] || a->source_col_offset + sc > src->shape[1])
        return AFAIL(RK_E_SHAPE, "upload source region exceeds binding shape", a);
    const uint64_t last = (a->source_row_offset + sr - 1u) * (uint64_t)a->source_row_stride +
                          a->source_col_offset + sc - 1u;
    if (src->nbytes % 2u || last >= src->nbytes / 2u)
        return AFAIL(RK_E_SHAPE, "upload source element range exceeds the binding nbytes", a);
    return 0;
}

static int check_download(const rk_plan_desc *p, const rk_action_desc *a, rk_diag *diag) {
    if (a->ninputs != 1 || a->noutputs != 0 || !a->inputs)
        return AFAIL(RK_E_SHAPE, "download requires one input view", a);
    const rk_view_desc *src = view_at(p, a->inputs[0]);
    const rk_value_desc *dst = value_at(p, a->source_binding);
    if (!src || !dst) return AFAIL(RK_E_SCHEMA, "download references missing view or output binding", a);
    if (dst->role != RK_ROLE_OUTPUT) return AFAIL(RK_E_SHAPE, "download target binding must be output", a);
    if (!tensor_valid(&src->tensor)) return AFAIL(RK_E_SHAPE, "download view tensor is invalid", a);
    if (src->valid_region[0] || src->valid_region[2] || src->valid_region[1] != src->tensor.rows ||
        src->valid_region[3] != src->tensor.cols)
        return AFAIL(RK_E_SHAPE, "download view must expose its full logical tile", a);
    return 0;
}

static int template_arity(uint32_t t, uint32_t *nin, uint32_t *nout) {
    *nout = 1;
    switch (t) {
    case RK_TEMPLATE_MM_F16: *nin = 2; return 0;
    case RK_TEMPLATE_MM_ACC_F16:
    case RK_TEMPLATE_EW_ADD_F16:
    case RK_TEMPLATE_EW_MUL_F16:
    case RK_TEMPLATE_EW_MAX_F16:
    case RK_TEMPLATE_EW_ADD_RELU_F16: *nin = 3; return 0;
    case RK_TEMPLATE_LUT_SIGMOID_F16:
    case RK_TEMPLATE_LUT_HARDSIGMOID_F16:
    case RK_TEMPLATE_LUT_GELU_GATE_F16:
    case RK_TEMPLATE_LUT_RSQRT_F16: *nin = 1; return 0;
    default: return -1;
    }
}

static int is_ew(uint32_t t) {
    return t == RK_TEMPLATE_EW_ADD_F16 || t == RK_TEMPLATE_EW_MUL_F16 || t == RK_TEMPLATE_EW_MAX_F16 ||
           t == RK_TEMPLATE_EW_ADD_RELU_F16;
}

/* Per-template operand rules (rk_plan_validate.c:312-463). The arity is bounded before any
 * input/output id is read. */
static int check_task(const rk_plan_desc *p, const rk_action_desc *a, rk_diag *diag) {
    if (!a->inputs || !a->outputs) return AFAIL(RK_E_SCHEMA, "NPU task has null input/output array", a);
    uint32_t nin, nout;
    if (template_arity(a->template_id, &nin, &nout)) return AFAIL(RK_E_SCHEMA, "unknown NPU task template", a);
    if (a->ninputs != nin || a->noutputs != nout)
        return AFAIL(RK_E_SCHEMA, "NPU task argument counts do not match its template", a);
    for (uint32_t i = 0; i < nin; i++)
        if (!view_at(p, a->inputs[i])) return AFAIL(RK_E_SCHEMA, "NPU task references missing input view", a);
    if (!view_at(p, a->outputs[0])) return AFAIL(RK_E_SCHEMA, "NPU task references missing output view", a);
    const rk_view_desc *x = view_at(p, a->inputs[0]), *o = view_at(p, a->outputs[0]);
    const rk_tensor_desc *xt = &x->tensor, *ot = &o->tensor;
    if (a->template_id == RK_TEMPLATE_MM_F16 || a->template_id == RK_TEMPLATE_MM_ACC_F16) {
        const int acc = a->template_id == RK_TEMPLATE_MM_ACC_F16;
        const rk_view_desc *w = view_at(p, a->inputs[1]);
        const rk_view_desc *pr = acc ? view_at(p, a->inputs[2]) : NULL;
        const rk_tensor_desc *wt = &w->tensor;
        if (!acc) {
            if (!tensor_valid(xt) || !tensor_valid(wt) || !tensor_valid(ot) || xt->layout != RK_LAYOUT_CUBE_F16 ||
                wt->layout != RK_LAYOUT_WEIGHT_F16 || ot->layout != RK_LAYOUT_CUBE_F16)
                return AFAIL(RK_E_SHAPE, "mm layout mismatch", a);
            if (xt->rows > 256 || xt->cols > CO_K_TILE || wt->rows > 256 || wt->cols > CO_K_TILE)
                return AFAIL(RK_E_SHAPE, "mm primitive exceeds 256", a);
            if (xt->rows != ot->rows || xt->cols != wt->cols || wt->rows != ot->cols)
                return AFAIL(RK_E_SHAPE, "mm extents mismatch", a);
            if (x->buffer_id == o->buffer_id || w->buffer_id == o->buffer_id)
                return AFAIL(RK_E_ALIAS, "mm output aliases an input", a);
            return 0;
        }
        if (!tensor_valid(xt) || !tensor_valid(wt) || !tensor_valid(&pr->tensor) || !tensor_valid(ot))
            return AFAIL(RK_E_SHAPE, "mm_acc has invalid tensor", a);
        if (xt->layout != RK_LAYOUT_CUBE_F16 || wt->layout != RK_LAYOUT_WEIGHT_F16 ||
            pr->tensor.layout != RK_LAYOUT_CUBE_F16 || ot->layout != RK_LAYOUT_CUBE_F16)
            return AFAIL(RK_E_SHAPE, "mm_acc layout mismatch", a);
        if (!same_tensor(&pr->tensor, ot)) return AFAIL(RK_E_SHAPE, "mm_acc prior/output tensors differ", a);
        if (xt->rows != ot->rows || xt->cols != wt->cols || wt->rows != ot->cols)
            return AFAIL(RK_E_SHAPE, "mm_acc extents mismatch", a);
        if (xt->cols > CO_K_TILE || wt->cols > CO_K_TILE || xt->physical_cols > CO_K_TILE ||
            wt->physical_cols > CO_K_TILE)
            return AFAIL(RK_E_SHAPE, "mm_acc K extent exceeds one 256-wide tile", a);
        if (xt->physical_rows != ot->physical_rows || xt->physical_cols != wt->physical_cols ||
            wt->physical_rows != ot->physical_cols)
            return AFAIL(RK_E_SHAPE, "mm_acc physical geometry mismatch", a);
        if (pr->buffer_id == o->buffer_id) return AFAIL(RK_E_ALIAS, "mm_acc prior/output alias", a);
        const rk_buffer_desc *pb = buffer_at(p, pr->buffer_id), *ob = buffer_at(p, o->buffer_id);
        if (!pb || !ob || pb->slot_id == ob->slot_id) return AFAIL(RK_E_ALIAS, "mm_acc prior/output share a BO", a);
        if (x->buffer_id == o->buffer_id || w->buffer_id == o->buffer_id)
            return AFAIL(RK_E_ALIAS, "mm_acc output aliases x/weight", a);
        return 0;
    }
    if (is_ew(a->template_id)) {
        const rk_view_desc *y = view_at(p, a->inputs[1]), *id = view_at(p, a->inputs[2]);
        const rk_tensor_desc *yt = &y->tensor, *it = &id->tensor;
        if (!tensor_valid(xt) || !tensor_valid(yt) || !tensor_valid(it) || !tensor_valid(ot))
            return AFAIL(RK_E_SHAPE, "EW has invalid tensor", a);
        if (xt->rows != yt->rows || xt->cols != yt->cols || xt->physical_rows != yt->physical_rows ||
            xt->physical_cols != yt->physical_cols || xt->rows != ot->rows || xt->cols != ot->cols ||
            xt->physical_rows != ot->physical_rows || xt->physical_cols != ot->physical_cols)
            return AFAIL(RK_E_SHAPE, "EW requires exact shapes", a);
        if (xt->layout != RK_LAYOUT_CUBE_F16 || yt->layout != RK_LAYOUT_CUBE_F16 || ot->layout != RK_LAYOUT_CUBE_F16)
            return AFAIL(RK_E_SHAPE, "EW operands and output must be CUBE tiles", a);
        if (xt->atom != yt->atom || xt->atom != ot->atom || xt->bytes != yt->bytes || xt->bytes != ot->bytes)
            return AFAIL(RK_E_SHAPE, "EW operands and output must be the same tile", a);
        if (it->layout != RK_LAYOUT_WEIGHT_F16 || it->rows != xt->physical_cols || it->cols != xt->physical_cols)
            return AFAIL(RK_E_SHAPE, "EW identity weight geometry mismatch", a);
        if (it->physical_rows != xt->physical_cols || it->physical_cols != xt->physical_cols)
            return AFAIL(RK_E_SHAPE, "EW identity weight physical geometry mismatch", a);
        if (x->buffer_id == o->buffer_id || y->buffer_id == o->buffer_id)
            return AFAIL(RK_E_ALIAS, "EW output aliases an operand", a);
        return 0;
    }
    /* LUT */
    if (!tensor_valid(xt) || !tensor_valid(ot) || xt->bytes != ot->bytes)
        return AFAIL(RK_E_SHAPE, "LUT physical sizes mismatch", a);
    if (!same_tensor(xt, ot)) return AFAIL(RK_E_SHAPE, "LUT input and output must be the same tile", a);
    if (x->buffer_id == o->buffer_id) return AFAIL(RK_E_ALIAS, "LUT input/output alias", a);
    if (xt->layout == RK_LAYOUT_CUBE_F16) {
        if ((uint64_t)xt->physical_rows * xt->physical_cols > 65528)
            return AFAIL(RK_E_SHAPE, "LUT view exceeds 65528 elements", a);
    } else if (xt->layout != RK_LAYOUT_LINEAR_F16) {
        return AFAIL(RK_E_SHAPE, "LUT layout mismatch", a);
    }
    return 0;
}

/* A cube reader may read an atom-aligned column slice of a wider cube written by one plain host
 * upload (rk_plan_validate.c:117-147), and a device writer may produce an atom-aligned slice of a
 * wider cube read in one piece (:149-172): the slice is a contiguous byte range of the canonical
 * [K/8][Mp][8] layout when the physical row geometry agrees. */
static int cube_slice_of(const rk_view_desc *outer, const rk_view_desc *inner) {
    const rk_tensor_desc *o = &outer->tensor, *i = &inner->tensor;
    if (o->layout != RK_LAYOUT_CUBE_F16 || i->layout != RK_LAYOUT_CUBE_F16 || o->atom != 8 || i->atom != 8 ||
        o->physical_rows != i->physical_rows || o->rows != i->rows || outer->offset_bytes > inner->offset_bytes)
        return 0;
    if (outer->offset_bytes + o->bytes < inner->offset_bytes + i->bytes) return 0;
    const uint64_t row_stride = (uint64_t)o->physical_rows * 2u;
    const uint64_t delta = inner->offset_bytes - outer->offset_bytes;
    if (!row_stride || delta % row_stride) return 0;
    const uint64_t column = delta / row_stride;
    if (column % 8u || column > o->cols || i->cols > (uint64_t)o->cols - column) return 0;
    return inner->offset_bytes % 16u == 0;
}

static int upload_slice_covers(const rk_action_desc *wa, const rk_view_desc *w, const rk_view_desc *r) {
    if (wa->kind != RK_ACTION_UPLOAD ||
        (wa->flags & (RK_ACTION_FLAG_TRANSPOSE_SOURCE | RK_ACTION_FLAG_BROADCAST_SCALAR |
                      RK_ACTION_FLAG_BROADCAST_CHANNEL)))
        return 0;
    return cube_slice_of(w, r) && w->offset_bytes % 16u == 0;
}

static int device_slice_covers(const rk_action_desc *wa, const rk_view_desc *w, const rk_view_desc *r) {
    return wa->kind != RK_ACTION_UPLOAD && cube_slice_of(r, w);
}

/* seen[j] = 1 for every action j that `consumer` reaches through declared dependencies. */
static void mark_ancestors(const rk_plan_desc *p, uint32_t consumer, unsigned char *seen, uint32_t *stack) {
    memset(seen, 0, p->nactions);
    uint32_t top = 0;
    stack[top++] = consumer;
    while (top) {
        const rk_action_desc *a = &p->actions[stack[--top]];
        for (uint32_t d = 0; d < a->ndeps; d++) {
            const uint32_t dep = a->deps[d];
            if (dep < p->nactions && !seen[dep]) {
                seen[dep] = 1;
                stack[top++] = dep;
            }
        }
    }
}

static int writer_contributes(const rk_plan_desc *p, uint32_t writer, const rk_view_desc *wv,
                              const rk_view_desc *rd) {
    return rd->tensor.layout == RK_LAYOUT_LINEAR_F16 || wv->tensor.layout == RK_LAYOUT_LINEAR_F16 ||
           (wv->offset_bytes == rd->offset_bytes && same_addressing(&wv->tensor, &rd->tensor)) ||
           upload_slice_covers(&p->actions[writer], wv, rd) || device_slice_covers(&p->actions[writer], wv, rd);
}

/* The schedule the runtime executes is the action order itself (submits are ascending contiguous
 * runs of tasks in submit order), so sequence position == action id. Checks, per
 * rk_plan_validate.c:508-911: submit runs; one writer class (host or device) per buffer and at
 * most RK_MAX_WRITERS_PER_BUFFER writes; every read has an earlier overlapping writer that is a
 * declared ancestor; overlapping writers agree on addressing and never mix host and device;
 * every read's byte range is covered by earlier contributing ancestor writes; every buffer is
 * accessed; constant buffers own their slot; buffers sharing a slot have disjoint live ranges. */
static int check_schedule(const rk_plan_desc *p, rk_diag *diag) {
    const uint32_t na = p->nactions, nb = p->nbuffers;
    int rc = 0;
    uint32_t *cls = calloc(nb, sizeof(uint32_t)), *count = calloc(nb, sizeof(uint32_t));
    uint32_t *first = malloc(nb * sizeof(uint32_t)), *last = calloc(nb, sizeof(uint32_t));
    unsigned char *persistent = calloc(nb, 1), *seen = malloc(na);
    uint32_t *stack = malloc((size_t)na * sizeof(uint32_t));
    if (!cls || !count || !first || !last || !persistent || !seen || !stack) {
        rc = VFAIL(RK_E_NOMEM, "out of memory");
        goto done;
    }
    for (uint32_t b = 0; b < nb; b++) first[b] = UINT32_MAX;
    for (uint32_t s = 0; s < p->nsubmits; s++) {
        const rk_submit_desc *sub = &p->submits[s];
        if (!sub->ntask_ids || !sub->task_ids) { rc = VFAIL(RK_E_SHAPE, "submit has no task list"); goto done; }
        for (uint32_t t = 1; t < sub->ntask_ids; t++)
            if (sub->task_ids[t] <= sub->task_ids[t - 1]) {
                rc = VFAIL(RK_E_SCHEMA, "submit tasks must be listed in ascending emission order");
                goto done;
            }
        const uint32_t lo = sub->task_ids[0], hi = sub->task_ids[sub->ntask_ids - 1];
        for (uint32_t id = lo; id <= hi; id++)
            if (id >= na || p->actions[id].kind != RK_ACTION_NPU_TASK) {
                rc = VFAIL(RK_E_SCHEMA, "a host action is interleaved inside a task group");
                goto done;
            }
        if (hi - lo + 1u != sub->ntask_ids) {
            rc = VFAIL(RK_E_SCHEMA, "another submit's task is interleaved inside a task group; a submit must "
                                    "own a contiguous run of tasks");
            goto done;
        }
        if (s > 0) {
            const rk_submit_desc *prev = &p->submits[s - 1];
            if (lo <= prev->task_ids[prev->ntask_ids - 1]) {
                rc = VFAIL(RK_E_SCHEMA, "submit task runs must appear in submit order");
                goto done;
            }
        }
    }
    /* writers */
    for (uint32_t i = 0; i < na; i++) {
        const rk_action_desc *a = &p->actions[i];
        const uint32_t c = a->kind == RK_ACTION_UPLOAD ? 1u : 2u;
        for (uint32_t o = 0; o < a->noutputs; o++) {
            const uint32_t b = p->views[a->outputs[o]].buffer_id;
            if (cls[b] && cls[b] != c) {
                rc = AFAIL(RK_E_SCHEMA, "buffer is written by both the host and the device", a);
                goto done;
            }
            cls[b] = c;
            if (a->kind == RK_ACTION_UPLOAD &&
                ((a->flags & RK_ACTION_FLAG_CACHE_CONSTANT) || p->values[a->source_binding].role == RK_ROLE_CONSTANT))
                persistent[b] = 1;
            if (++count[b] > RK_MAX_WRITERS_PER_BUFFER) {
                rc = AFAIL(RK_E_SCHEMA, "too many writers for one logical buffer", a);
                goto done;
            }
        }
    }
    /* reads: latest overlapping earlier writer must be an ancestor */
    for (uint32_t i = 0; i < na; i++) {
        const rk_action_desc *a = &p->actions[i];
        if (a->ninputs) mark_ancestors(p, i, seen, stack);
        for (uint32_t n = 0; n < a->ninputs; n++) {
            const rk_view_desc *rd = &p->views[a->inputs[n]];
            const uint64_t s0 = rd->offset_bytes, s1 = rd->offset_bytes + rd->tensor.bytes;
            uint32_t producer = UINT32_MAX;
            for (uint32_t j = 0; j < i; j++) {
                const rk_action_desc *w = &p->actions[j];
                for (uint32_t o = 0; o < w->noutputs; o++) {
                    const rk_view_desc *wv = &p->views[w->outputs[o]];
                    if (wv->buffer_id == rd->buffer_id && wv->offset_bytes < s1 && s0 < wv->offset_bytes + wv->tensor.bytes)
                        producer = j;
                }
            }
            if (producer == UINT32_MAX) {
                rc = AFAIL(RK_E_SHAPE, "read of a buffer that no action writes before it", a);
                goto done;
            }
            if (!seen[producer]) {
                rc = AFAIL(RK_E_SCHEMA, "the producer of a read is not a declared dependency of the consumer", a);
                goto done;
            }
        }
    }
    /* overlapping writers of one buffer */
    for (uint32_t i = 0; i < na; i++) {
        const rk_action_desc *a = &p->actions[i];
        for (uint32_t o = 0; o < a->noutputs; o++) {
            const rk_view_desc *va = &p->views[a->outputs[o]];
            for (uint32_t j = i; j < na; j++) {
                const rk_action_desc *b = &p->actions[j];
                for (uint32_t q = (j == i ? o + 1 : 0); q < b->noutputs; q++) {
                    const rk_view_desc *vb = &p->views[b->outputs[q]];
                    if (vb->buffer_id != va->buffer_id || !(va->offset_bytes < vb->offset_bytes + vb->tensor.bytes &&
                                                            vb->offset_bytes < va->offset_bytes + va->tensor.bytes))
                        continue;
                    const int ha = a->kind == RK_ACTION_UPLOAD, hb = b->kind == RK_ACTION_UPLOAD;
                    if (ha && hb) {
                        rc = AFAIL(RK_E_ALIAS, "overlapping host uploads of one buffer are ambiguous; slices must be "
                                               "disjoint", b);
                        goto done;
                    }
                    if (ha || hb) {
                        rc = AFAIL(RK_E_ALIAS, "a host upload and a device write must not overlap in one buffer", b);
                        goto done;
                    }
                    if (!same_addressing(&va->tensor, &vb->tensor)) {
                        rc = AFAIL(RK_E_ALIAS, "overlapping writers of one buffer use different physical addressing",
                                   b);
                        goto done;
                    }
                }
            }
        }
    }
    /* coverage of every read by earlier contributing ancestor writes */
    for (uint32_t i = 0; i < na; i++) {
        const rk_action_desc *a = &p->actions[i];
        if (a->ninputs) mark_ancestors(p, i, seen, stack);
        for (uint32_t n = 0; n < a->ninputs; n++) {
            const rk_view_desc *rd = &p->views[a->inputs[n]];
            const uint64_t need0 = rd->offset_bytes, need1 = rd->offset_bytes + rd->tensor.bytes;
            uint64_t cursor = need0;
            int usable = 0;
            for (;;) {
                uint64_t best = cursor;
                for (uint32_t j = 0; j < i; j++) {
                    const rk_action_desc *w = &p->actions[j];
                    for (uint32_t o = 0; o < w->noutputs; o++) {
                        const rk_view_desc *wv = &p->views[w->outputs[o]];
                        const uint64_t w0 = wv->offset_bytes, w1 = wv->offset_bytes + wv->tensor.bytes;
                        if (wv->buffer_id != rd->buffer_id || w1 <= need0 || w0 >= need1) continue;
                        if (!writer_contributes(p, j, wv, rd)) continue;
                        if (!seen[j]) {
                            rc = AFAIL(RK_E_SCHEMA, "a producer covering this read is not a declared dependency of "
                                                    "the consumer", a);
                            goto done;
                        }
                        usable = 1;
                        if (w0 <= cursor && w1 > best) best = w1;
                    }
                }
                if (!usable) {
                    rc = AFAIL(RK_E_SHAPE, "no write before this read produces the consumed range", a);
                    goto done;
                }
                if (cursor >= need1) break;
                if (best <= cursor) {
                    rc = AFAIL(RK_E_SHAPE, "the writes that precede this read do not cover the consumed range", a);
                    goto done;
                }
                cursor = best;
            }
        }
    }
    /* live ranges and slots */
    for (uint32_t i = 0; i < na; i++) {
        const rk_action_desc *a = &p->actions[i];
        for (uint32_t n = 0; n < a->ninputs + a->noutputs; n++) {
            const uint32_t v = n < a->ninputs ? a->inputs[n] : a->outputs[n - a->ninputs];
            const uint32_t b = p->views[v].buffer_id;
            if (i < first[b]) first[b] = i;
            if (i > last[b]) last[b] = i;
        }
    }
    for (uint32_t b = 0; b < nb; b++)
        if (first[b] == UINT32_MAX) {
            rc = VFAIL(RK_E_SHAPE, "logical buffer is never accessed");
            goto done;
        }
    for (uint32_t b = 0; b < nb; b++) {
        uint32_t peers = 0;
        for (uint32_t c = 0; c < nb; c++)
            if (p->buffers[c].slot_id == p->buffers[b].slot_id && ++peers > RK_MAX_BUFFERS_PER_SLOT) {
                rc = VFAIL(RK_E_SCHEMA, "too many buffers share one slot");
                goto done;
            }
        if (persistent[b] && peers != 1u) {
            rc = VFAIL(RK_E_ALIAS, "a constant workspace buffer must own its slot for the whole workspace lifetime");
            goto done;
        }
        for (uint32_t c = b + 1; c < nb; c++)
            if (p->buffers[c].slot_id == p->buffers[b].slot_id && !(last[b] < first[c] || last[c] < first[b])) {
                rc = VFAIL(RK_E_ALIAS, "buffers sharing a slot have overlapping live ranges");
                goto done;
            }
    }
done:
    free(cls); free(count); free(first); free(last); free(persistent); free(seen); free(stack);
    return rc;
}

/* Per-submit-task host bytes the B200 runtime keeps (one task descriptor); the NPU runtime counts
 * one command program here. */
#define RK_HOST_TASK_BYTES ((uint64_t)sizeof(b2k_rk_task))

static int check_budgets(const rk_plan_desc *p, rk_diag *diag) {
    uint64_t *slot_end = calloc(p->nbuffers, sizeof(uint64_t));
    if (!slot_end) return VFAIL(RK_E_NOMEM, "out of memory");
    for (uint32_t i = 0; i < p->nbuffers; i++) {
        const rk_buffer_desc *b = &p->buffers[i];
        if (b->capacity > UINT64_MAX - b->offset) {
            free(slot_end);
            return VFAIL(RK_E_BUDGET, "buffer range overflow");
        }
        if (b->offset + b->capacity > slot_end[b->slot_id]) slot_end[b->slot_id] = b->offset + b->capacity;
    }
    uint64_t device = 0;
    for (uint32_t i = 0; i < p->nbuffers; i++) {
        if (!slot_end[i]) continue;
        if (slot_end[i] > UINT64_MAX - CO_SLACK - CO_GUARD || device > UINT64_MAX - (slot_end[i] + CO_SLACK + CO_GUARD)) {
            free(slot_end);
            return VFAIL(RK_E_BUDGET, "slot capacity overflow");
        }
        device += slot_end[i] + CO_SLACK + CO_GUARD;
    }
    free(slot_end);
    uint32_t max_tasks = 0;
    for (uint32_t i = 0; i < p->nsubmits; i++)
        if (p->submits[i].ntask_ids > max_tasks) max_tasks = p->submits[i].ntask_ids;
    const uint64_t command = (uint64_t)max_tasks * CO_MAX_WORDS * 8u;
    if (device > UINT64_MAX - command) return VFAIL(RK_E_BUDGET, "device request overflow");
    device += command;
    if (!p->claimed_device_bytes) return VFAIL(RK_E_BUDGET, "claimed_device_bytes must be stated (0 is not a bypass)");
    if (p->claimed_device_bytes < device)
        return VFAIL(RK_E_BUDGET, "claimed device bytes understate slots/command workspace");
    if (p->device_budget_bytes && device > p->device_budget_bytes) return VFAIL(RK_E_BUDGET, "device budget exceeded");
    uint64_t host = 0, largest = 0, outputs = 0, nout = 0;
    for (uint32_t i = 0; i < p->nvalues; i++) {
        const rk_value_desc *v = &p->values[i];
        if (v->role != RK_ROLE_INPUT && v->role != RK_ROLE_CONSTANT && v->role != RK_ROLE_OUTPUT) continue;
        host += v->nbytes;                         /* shapes are <= 4096 x 4096: no overflow */
        if (v->role == RK_ROLE_OUTPUT) {
            outputs += v->nbytes;
            nout++;
            if (v->nbytes > largest) largest = v->nbytes;
        }
    }
    const uint64_t staging = outputs > 65536u ? outputs : 65536u;
    host += staging + (uint64_t)max_tasks * RK_HOST_TASK_BYTES + largest +
            nout * (uint64_t)(sizeof(size_t) + sizeof(uint32_t));
    if (!p->claimed_host_bytes) return VFAIL(RK_E_BUDGET, "claimed_host_bytes must be stated (0 is not a bypass)");
    if (p->claimed_host_bytes < host) return VFAIL(RK_E_BUDGET, "claimed host bytes understate bindings and staging");
    if (p->host_budget_bytes && p->claimed_host_bytes > p->host_budget_bytes)
        return VFAIL(RK_E_BUDGET, "host budget exceeded");
    return 0;
}

static int check_publish(const rk_plan_desc *p, rk_diag *diag) {
    for (uint32_t i = 0; i < p->npublish; i++) {
        const rk_publish_desc *t = &p->publish[i];
        if (!struct_ok(t->abi_version, t->struct_size, sizeof(*t)))
            return VFAIL(RK_E_SCHEMA, "publish descriptor ABI/size mismatch");
        const rk_value_desc *v = value_at(p, t->binding_id);
        const rk_view_desc *view = view_at(p, t->view_id);
        if (!v || !view || v->role != RK_ROLE_OUTPUT) return VFAIL(RK_E_SCHEMA, "publish target invalid");
        if (!t->rows || !t->cols || (uint64_t)t->dst_row_offset + t->rows > v->shape[0] ||
            (uint64_t)t->dst_col_offset + t->cols > v->shape[1])
            return VFAIL(RK_E_SHAPE, "publish tile exceeds the output binding");
        if (t->rows != view->tensor.rows || t->cols != view->tensor.cols)
            return VFAIL(RK_E_SHAPE, "publish tile must publish the whole view");
        for (uint32_t j = 0; j < i; j++) {
            const rk_publish_desc *q = &p->publish[j];
            if (q->binding_id != t->binding_id) continue;
            if (q->view_id == t->view_id) return VFAIL(RK_E_SCHEMA, "the same view cannot be published twice");
            if (q->dst_row_offset < t->dst_row_offset + t->rows && t->dst_row_offset < q->dst_row_offset + q->rows &&
                q->dst_col_offset < t->dst_col_offset + t->cols && t->dst_col_offset < q->dst_col_offset + q->cols)
                return VFAIL(RK_E_SHAPE, "publish tiles overlap");
        }
        int downloaded = 0;
        for (uint32_t j = 0; j < p->nactions && !downloaded; j++) {
            const rk_action_desc *a = &p->actions[j];
            downloaded = a->kind == RK_ACTION_DOWNLOAD && a->source_binding == t->binding_id && a->ninputs == 1 &&
                         a->inputs[0] == t->view_id;
        }
        if (!downloaded) return VFAIL(RK_E_SCHEMA, "publish view has no matching download action");
    }
    for (uint32_t i = 0; i < p->nvalues; i++) {
        const rk_value_desc *v = &p->values[i];
        if (v->role != RK_ROLE_OUTPUT) continue;
        uint64_t area = 0;
        for (uint32_t j = 0; j < p->npublish; j++)
            if (p->publish[j].binding_id == i) area += (uint64_t)p->publish[j].rows * p->publish[j].cols;
        if (area != (uint64_t)v->shape[0] * v->shape[1])
            return VFAIL(RK_E_SHAPE, "publish tiles do not cover the output binding exactly");
    }
    for (uint32_t i = 0; i < p->nactions; i++) {
        const rk_action_desc *a = &p->actions[i];
        if (a->kind != RK_ACTION_DOWNLOAD) continue;
        uint32_t matches = 0;
        for (uint32_t j = 0; j < p->npublish; j++)
            matches += p->publish[j].binding_id == a->source_binding && p->publish[j].view_id == a->inputs[0];
        if (matches != 1) return AFAIL(RK_E_SCHEMA, "every download must map to exactly one publish tile", a);
    }
    return 0;
}

/* ------------------------------------------------------------------------------ the verifier */
static int validate_desc(const rk_plan_desc *p, rk_diag *diag) {
    if (!p) return VFAIL(RK_E_INVALID, "null plan descriptor");
    if (!struct_ok(p->abi_version, p->struct_size, sizeof(*p))) return VFAIL(RK_E_SCHEMA, "rk_plan_desc ABI/size mismatch");
    if (p->schema_version != RK_SCHEMA_VERSION) return VFAIL(RK_E_SCHEMA, "unsupported plan schema version");
    if (p->runtime_abi_version != RK_ABI_VERSION)
        return VFAIL(RK_E_SCHEMA, "descriptor runtime_abi_version does not match this library");
    if (!p->values || !p->nvalues || p->nvalues > 1000000) return VFAIL(RK_E_SCHEMA, "invalid values array");
    if (!p->nbuffers || p->nbuffers > 1000000 || !p->nviews || p->nviews > 1000000 || !p->nactions ||
        p->nactions > 1000000 || !p->nsubmits || p->nsubmits > 1000000 || !p->npublish || p->npublish > 1000000)
        return VFAIL(RK_E_SCHEMA, "missing or excessive plan arrays");
    if (!p->buffers || !p->views || !p->actions || !p->submits || !p->publish)
        return VFAIL(RK_E_SCHEMA, "null array with non-zero count");
    for (uint32_t i = 0; i < p->nvalues; i++) {
        const rk_value_desc *v = &p->values[i];
        if (!struct_ok(v->abi_version, v->struct_size, sizeof(*v)))
            return VFAIL(RK_E_SCHEMA, "value descriptor ABI/size mismatch");
        if (v->id != i || v->role > RK_ROLE_IDENTITY || v->dtype != RK_DTYPE_F16 || v->rank > 2 ||
            (v->rank != 2 && v->role != RK_ROLE_CONSTANT))
            return VFAIL(RK_E_SCHEMA, "value id/role/dtype/rank invalid");
        if (!v->name || !v->name_len || v->name_len > 128) return VFAIL(RK_E_SCHEMA, "value name invalid");
        if (v->rank == 0) {
            if (v->shape[0] || v->shape[1] || v->nbytes != 2u) return VFAIL(RK_E_SHAPE, "scalar value shape/bytes invalid");
        } else if (v->rank == 1) {
            if (!v->shape[0] || v->shape[0] > 4096 || v->shape[1] || v->nbytes != (uint64_t)v->shape[0] * 2u)
                return VFAIL(RK_E_SHAPE, "channel value shape/bytes invalid");
        } else {
            if (!v->shape[0] || !v->shape[1] || v->shape[0] > 4096 || v->shape[1] > 4096)
                return VFAIL(RK_E_SHAPE, "value shape out of range");
            if (v->nbytes != (uint64_t)v->shape[0] * v->shape[1] * 2u) return VFAIL(RK_E_SHAPE, "value byte size mismatch");
        }
        for (uint32_t j = 0; j < i; j++)
            if (p->values[j].name_len == v->name_len && !memcmp(p->values[j].name, v->name, v->name_len))
                return VFAIL(RK_E_SCHEMA, "duplicate value name");
    }
    for (uint32_t i = 0; i < p->nbuffers; i++) {
        const rk_buffer_desc *b = &p->buffers[i];
        if (!struct_ok(b->abi_version, b->struct_size, sizeof(*b)))
            return VFAIL(RK_E_SCHEMA, "buffer descriptor ABI/size mismatch");
        if (b->id != i || b->role > RK_ROLE_IDENTITY || !valid_layout(b->layout_id))
            return VFAIL(RK_E_SCHEMA, "buffer id/role/layout invalid");
        if (b->alignment < 16 || !is_pow2(b->alignment) || b->offset % b->alignment || !b->capacity)
            return VFAIL(RK_E_SHAPE, "buffer alignment/capacity invalid");
        if (b->lifetime_first > b->lifetime_last || b->lifetime_last >= p->nactions)
            return VFAIL(RK_E_SHAPE, "buffer lifetime invalid");
        if (b->slot_id >= p->nbuffers) return VFAIL(RK_E_SHAPE, "buffer slot id out of range");
        if (b->offset > UINT64_MAX - b->capacity) return VFAIL(RK_E_SHAPE, "buffer range overflows");
    }
    for (uint32_t i = 0; i < p->nviews; i++) {
        const rk_view_desc *v = &p->views[i];
        if (!struct_ok(v->abi_version, v->struct_size, sizeof(*v)))
            return VFAIL(RK_E_SCHEMA, "view descriptor ABI/size mismatch");
        if (v->id != i || !tensor_valid(&v->tensor)) return VFAIL(RK_E_SHAPE, "view id/tensor invalid");
        const rk_buffer_desc *b = buffer_at(p, v->buffer_id);
        if (!b) return VFAIL(RK_E_SCHEMA, "view references missing buffer");
        if (v->offset_bytes % 16 || v->offset_bytes > b->capacity || v->tensor.bytes > b->capacity - v->offset_bytes)
            return VFAIL(RK_E_SHAPE, "view exceeds buffer capacity");
        const uint32_t *vr = v->valid_region;
        if (vr[0] > v->tensor.rows || vr[1] > v->tensor.rows || vr[2] > v->tensor.cols || vr[3] > v->tensor.cols ||
            vr[0] + vr[1] > v->tensor.rows || vr[2] + vr[3] > v->tensor.cols)
            return VFAIL(RK_E_SHAPE, "view valid_region invalid");
    }
    for (uint32_t i = 0; i < p->nactions; i++) {
        const rk_action_desc *a = &p->actions[i];
        if (!struct_ok(a->abi_version, a->struct_size, sizeof(*a)))
            return VFAIL(RK_E_SCHEMA, "action descriptor ABI/size mismatch");
        if (a->id != i || a->kind < RK_ACTION_HOST_PACK || a->kind > RK_ACTION_COMMIT)
            return VFAIL(RK_E_SCHEMA, "action id/kind invalid");
        if (!memchr(a->origin, 0, sizeof(a->origin))) return VFAIL(RK_E_SCHEMA, "action origin is not NUL terminated");
        if (a->ninputs > RK_MAX_ACTION_ARGS || a->noutputs > RK_MAX_ACTION_ARGS || a->ndeps > RK_MAX_ACTION_DEPS)
            return AFAIL(RK_E_SCHEMA, "action argument count exceeds the ABI bound", a);
        if (a->ninputs && !a->inputs) return AFAIL(RK_E_SCHEMA, "action inputs pointer/count mismatch", a);
        if (a->noutputs && !a->outputs) return AFAIL(RK_E_SCHEMA, "action outputs pointer/count mismatch", a);
        if (a->ndeps && !a->deps) return AFAIL(RK_E_SCHEMA, "action deps pointer/count mismatch", a);
        for (uint32_t j = 0; j < a->ndeps; j++)
            if (a->deps[j] >= i) return AFAIL(RK_E_SCHEMA, "action dependency not topological", a);
        int rc;
        if (a->kind == RK_ACTION_UPLOAD) rc = check_upload(p, a, diag);
        else if (a->kind == RK_ACTION_DOWNLOAD) rc = check_download(p, a, diag);
        else if (a->kind == RK_ACTION_NPU_TASK) rc = check_task(p, a, diag);
        else if (a->kind == RK_ACTION_HOST_COMPUTE) rc = AFAIL(RK_E_UNSUPPORTED, "hidden host compute is forbidden", a);
        else rc = AFAIL(RK_E_UNSUPPORTED, "unsupported action kind", a);
        if (rc) return rc;
    }
    uint32_t *owner = malloc((size_t)p->nactions * sizeof(uint32_t));
    if (!owner) return VFAIL(RK_E_NOMEM, "out of memory");
    for (uint32_t i = 0; i < p->nactions; i++) owner[i] = UINT32_MAX;
    int rc = 0;
    for (uint32_t i = 0; i < p->nsubmits && !rc; i++) {
        const rk_submit_desc *s = &p->submits[i];
        if (!struct_ok(s->abi_version, s->struct_size, sizeof(*s))) { rc = VFAIL(RK_E_SCHEMA, "submit descriptor ABI/size mismatch"); break; }
        if (s->id != i || s->mode > RK_SUBMIT_SEPARATE || s->core_policy > RK_CORE_AUTO || !s->ntask_ids ||
            s->ntask_ids > RK_MAX_SUBMIT_TASKS || !s->task_ids || (s->ndeps && !s->deps)) {
            rc = VFAIL(RK_E_SHAPE, "submit metadata invalid");
            break;
        }
        for (uint32_t j = 0; j < s->ndeps && !rc; j++)
            if (s->deps[j] >= i) rc = VFAIL(RK_E_SCHEMA, "submit dependency not topological");
        for (uint32_t j = 0; j < s->ntask_ids && !rc; j++) {
            const uint32_t t = s->task_ids[j];
            if (t >= p->nactions) rc = VFAIL(RK_E_SCHEMA, "submit task id is out of range");
            else if (p->actions[t].kind != RK_ACTION_NPU_TASK) rc = VFAIL(RK_E_SCHEMA, "submit contains non-NPU task");
            else if (owner[t] != UINT32_MAX) rc = VFAIL(RK_E_SCHEMA, "task assigned to multiple submits");
            else owner[t] = i;
        }
        /* CBUF reuse hints: structural rule only (rk_plan_validate.c:1075-1104) */
        for (uint32_t j = 0; j < s->ntask_ids && !rc; j++) {
            const rk_action_desc *a = &p->actions[s->task_ids[j]];
            if (!(a->flags & (RK_ACTION_FLAG_DATA_REUSE | RK_ACTION_FLAG_WEIGHT_REUSE))) continue;
            if (s->mode != RK_SUBMIT_CHAIN || j == 0) {
                rc = AFAIL(RK_E_SCHEMA, "CBUF reuse requires a chained submit and non-first task", a);
                break;
            }
            const rk_action_desc *prev = &p->actions[s->task_ids[j - 1]];
            if (prev->source_k_index != a->source_k_index) rc = AFAIL(RK_E_SCHEMA, "CBUF reuse crosses a K boundary", a);
            else if ((a->flags & RK_ACTION_FLAG_DATA_REUSE) &&
                     (prev->inputs[0] != a->inputs[0] ||
                      !same_geometry(&p->views[prev->inputs[0]].tensor, &p->views[a->inputs[0]].tensor)))
                rc = AFAIL(RK_E_SCHEMA, "data_reuse predecessor input view/geometry mismatch", a);
            else if ((a->flags & RK_ACTION_FLAG_WEIGHT_REUSE) &&
                     (prev->ninputs < 2 || a->ninputs < 2 || prev->inputs[1] != a->inputs[1] ||
                      !same_geometry(&p->views[prev->inputs[1]].tensor, &p->views[a->inputs[1]].tensor)))
                rc = AFAIL(RK_E_SCHEMA, "weight_reuse predecessor weight view/geometry mismatch", a);
        }
    }
    for (uint32_t i = 0; i < p->nactions && !rc; i++)
        if (p->actions[i].kind == RK_ACTION_NPU_TASK && owner[i] == UINT32_MAX)
            rc = AFAIL(RK_E_SCHEMA, "unassigned NPU task", &p->actions[i]);
    free(owner);
    if (rc) return rc;
    for (uint32_t i = 0; i < p->nactions; i++) {
        const rk_action_desc *a = &p->actions[i];
        if (a->kind != RK_ACTION_NPU_TASK) continue;
        const rk_view_desc *ov = &p->views[a->outputs[0]];
        for (uint32_t n = 0; n < a->ninputs; n++) {
            const rk_view_desc *iv = &p->views[a->inputs[n]];
            if (iv->buffer_id == ov->buffer_id || p->buffers[iv->buffer_id].slot_id == p->buffers[ov->buffer_id].slot_id)
                return AFAIL(RK_E_ALIAS, "NPU output aliases/shared BO with an input", a);
        }
    }
    for (uint32_t i = 0; i < p->nvalues; i++) {
        const rk_value_desc *v = &p->values[i];
        if (v->role != RK_ROLE_INPUT && v->role != RK_ROLE_CONSTANT && v->role != RK_ROLE_OUTPUT) continue;
        int found = 0;
        for (uint32_t j = 0; j < p->nactions && !found; j++) {
            const rk_action_desc *a = &p->actions[j];
            found = a->source_binding == v->id &&
                    (v->role == RK_ROLE_OUTPUT ? a->kind == RK_ACTION_DOWNLOAD : a->kind == RK_ACTION_UPLOAD);
        }
        if (!found) return VFAIL(RK_E_SCHEMA, "binding has no matching host boundary action");
    }
    rc = check_schedule(p, diag);
    if (!rc) rc = check_publish(p, diag);
    if (!rc) rc = check_budgets(p, diag);
    return rc;
}

/* ------------------------------------------------------------------------------ plans */
/* A verified, immutable deep copy: `d` points only into memory the plan owns. */
struct rk_plan {
    rk_plan_desc d;
    rk_value_desc *values;
    char **names;
    rk_buffer_desc *buffers;
    rk_view_desc *views;
    rk_action_desc *actions;
    uint32_t **action_lists;     /* [3 * nactions]: inputs, outputs, deps */
    rk_submit_desc *submits;
    uint32_t **submit_lists;     /* [2 * nsubmits]: task ids, deps */
    rk_publish_desc *publish;
};

static void plan_free(rk_plan *p) {
    if (!p) return;
    if (p->names)
        for (uint32_t i = 0; i < p->d.nvalues; i++) free(p->names[i]);
    if (p->action_lists)
        for (uint32_t i = 0; i < 3u * p->d.nactions; i++) free(p->action_lists[i]);
    if (p->submit_lists)
        for (uint32_t i = 0; i < 2u * p->d.nsubmits; i++) free(p->submit_lists[i]);
    free(p->names); free(p->values); free(p->buffers); free(p->views); free(p->actions); free(p->action_lists);
    free(p->submits); free(p->submit_lists); free(p->publish);
    free(p);
}

static uint32_t *copy_ids(const uint32_t *src, uint32_t n, int *nomem) {
    if (!n) return NULL;
    uint32_t *out = malloc((size_t)n * sizeof(uint32_t));
    if (!out) *nomem = 1;
    else memcpy(out, src, (size_t)n * sizeof(uint32_t));
    return out;
}

static int plan_copy(const rk_plan_desc *src, rk_plan **out) {
    rk_plan *p = calloc(1, sizeof(*p));
    if (!p) return RK_E_NOMEM;
    p->d = *src;
    p->d.nvalues = src->nvalues;
    p->values = calloc(src->nvalues, sizeof(*p->values));
    p->names = calloc(src->nvalues, sizeof(char *));
    p->buffers = malloc((size_t)src->nbuffers * sizeof(*p->buffers));
    p->views = malloc((size_t)src->nviews * sizeof(*p->views));
    p->actions = malloc((size_t)src->nactions * sizeof(*p->actions));
    p->action_lists = calloc(3u * (size_t)src->nactions, sizeof(uint32_t *));
    p->submits = malloc((size_t)src->nsubmits * sizeof(*p->submits));
    p->submit_lists = calloc(2u * (size_t)src->nsubmits, sizeof(uint32_t *));
    p->publish = malloc((size_t)src->npublish * sizeof(*p->publish));
    int nomem = !p->values || !p->names || !p->buffers || !p->views || !p->actions || !p->action_lists ||
                !p->submits || !p->submit_lists || !p->publish;
    if (nomem) {
        p->d.nactions = p->d.nsubmits = p->d.nvalues = 0;
        plan_free(p);
        return RK_E_NOMEM;
    }
    for (uint32_t i = 0; i < src->nvalues; i++) {
        p->values[i] = src->values[i];
        p->names[i] = malloc((size_t)src->values[i].name_len + 1u);
        if (!p->names[i]) { nomem = 1; continue; }
        memcpy(p->names[i], src->values[i].name, src->values[i].name_len);
        p->names[i][src->values[i].name_len] = 0;
        p->values[i].name = p->names[i];
    }
    memcpy(p->buffers, src->buffers, (size_t)src->nbuffers * sizeof(*p->buffers));
    memcpy(p->views, src->views, (size_t)src->nviews * sizeof(*p->views));
    for (uint32_t i = 0; i < src->nactions; i++) {
        const rk_action_desc *a = &src->actions[i];
        p->actions[i] = *a;
        p->action_lists[3 * i] = copy_ids(a->inputs, a->ninputs, &nomem);
        p->action_lists[3 * i + 1] = copy_ids(a->outputs, a->noutputs, &nomem);
        p->action_lists[3 * i + 2] = copy_ids(a->deps, a->ndeps, &nomem);
        p->actions[i].inputs = p->action_lists[3 * i];
        p->actions[i].outputs = p->action_lists[3 * i + 1];
        p->actions[i].deps = p->action_lists[3 * i + 2];
    }
    for (uint32_t i = 0; i < src->nsubmits; i++) {
        const rk_submit_desc *s = &src->submits[i];
        p->submits[i] = *s;
        p->submit_lists[2 * i] = copy_ids(s->task_ids, s->ntask_ids, &nomem);
        p->submit_lists[2 * i + 1] = copy_ids(s->deps, s->ndeps, &nomem);
        p->submits[i].task_ids = p->submit_lists[2 * i];
        p->submits[i].deps = p->submit_lists[2 * i + 1];
    }
    memcpy(p->publish, src->publish, (size_t)src->npublish * sizeof(*p->publish));
    p->d.values = p->values;
    p->d.buffers = p->buffers;
    p->d.views = p->views;
    p->d.actions = p->actions;
    p->d.submits = p->submits;
    p->d.publish = p->publish;
    if (nomem) {
        plan_free(p);
        return RK_E_NOMEM;
    }
    *out = p;
    return 0;
}

uint32_t rk_abi_version(void) { return RK_ABI_VERSION; }

int rk_plan_create(const rk_plan_desc *desc, rk_plan **out, rk_diag *diag) {
    diag_clear(diag);
    if (!out) return diag_set(diag, RK_E_INVALID, "create", "null out pointer", UINT32_MAX, NULL, 0);
    *out = NULL;
    int rc = validate_desc(desc, diag);
    if (rc) return rc;
    rc = plan_copy(desc, out);
    if (rc) return diag_set(diag, rc, "create", "out of memory", UINT32_MAX, NULL, 0);
    return 0;
}

void rk_plan_destroy(rk_plan *plan) { plan_free(plan); }

int rk_target_check(rk_diag *diag) {
    if (b2d_device_count() > 0) return 0;
    return diag_set(diag, RK_E_TARGET_MISMATCH, "target", "no CUDA device is visible to this process", UINT32_MAX,
                    NULL, 0);
}

int rk_target_validate_text(const char *compat, size_t compat_len, const char *version, rk_diag *diag) {
    diag_clear(diag);
    return diag_set(diag, RK_E_UNSUPPORTED, "target", "board compatible strings do not apply to a CUDA device",
                    UINT32_MAX, NULL, 0);
}

/* ------------------------------------------------------------------------------ workspaces */
struct rk_workspace {
    int fd;
    b2_dev *dev;
    rk_plan *plan;                   /* the workspace's own copy */
    co_buffer *slots;                /* [nbuffers]: one HBM allocation per used slot id */
    b2k_rk_tile *tiles;              /* [nviews] */
    void *in_dev, *in_host;          /* the input bindings in HBM and their pinned host staging */
    size_t in_bytes;
    uint64_t *in_off;                /* [nvalues] */
    unsigned char *in_needed;        /* [nvalues]: a per-run upload reads this input */
    void *out_dev, *out_host;        /* output staging: HBM and pinned host, per-value offsets */
    size_t out_bytes;
    uint64_t *out_off;               /* [nvalues] */
    b2k_rk_pack *packs;              /* per-run uploads */
    uint32_t npacks;
    b2k_rk_task *tasks;              /* device tasks in action order */
    uint32_t ntasks;
    b2k_rk_unpack *unpacks;          /* downloads in action order */
    uint32_t nunpacks;
    struct rk_step { uint32_t kind, first, count; } *steps;   /* the run, in action order */
    b2k_rk_chain *chains;            /* fused contraction chains (find_chains) */
    uint32_t nchains;
    uint32_t *chain_head;            /* [nactions]: chain index + 1 where a chain starts, else 0 */
    unsigned char *chain_member;     /* [nactions]: a task folded into the chain before it */
    void *chain_scratch, *chain_tickets;
    size_t chain_scratch_bytes, chain_ticket_bytes;
    uint32_t nsteps;
    void **guard_base;               /* allocated slots for the guard check */
    size_t *guard_payload;
    uint32_t nguard;
    b2_exec *exec;                   /* the device schedule as a CUDA graph; NULL: eager launches */
    unsigned char *persistent;       /* [nactions] */
    void *scratch_dev;               /* region-update source staging */
    size_t scratch_bytes;
    uint32_t ninputs, noutputs, nconstants, task_count;
    uint64_t upload_calls, upload_bytes, download_bytes;
    uint64_t device_bytes;
    atomic_int busy, poisoned;
};

#define WS_FAIL(stage, code, msg) diag_set(diag, (code), (stage), (msg), UINT32_MAX, NULL, 0)

static size_t align256(size_t x) { return (x + 255u) & ~(size_t)255u; }

static const rk_binding *find_binding(const rk_binding *arr, uint32_t n, uint32_t id) {
    const rk_binding *found = NULL;
    for (uint32_t i = 0; i < n; i++)
        if (arr[i].id == id) {
            if (found) return NULL;          /* duplicated */
            found = &arr[i];
        }
    return found;
}

static int binding_matches(const rk_value_desc *v, const rk_binding *b, const char *stage, rk_diag *diag) {
    if (!b) return WS_FAIL(stage, RK_E_SHAPE, "missing binding");
    if (b->abi_version != RK_ABI_VERSION || b->struct_size < sizeof(*b) || b->dtype != v->dtype ||
        b->rank != v->rank || b->shape[0] != v->shape[0] || b->shape[1] != v->shape[1] || b->nbytes != v->nbytes ||
        (v->nbytes && !b->data))
        return WS_FAIL(stage, RK_E_SHAPE, "binding dtype/rank/shape/nbytes mismatch or null data");
    return 0;
}

/* Index of the first non-finite FP16 (exponent all ones) among n, or n. Four halves per 64-bit
 * word: a lane is non-finite when its exponent bits equal 0x7c00, i.e. (w & E) ^ E has a zero lane. */
static size_t first_nonfinite(const void *data, size_t n) {
    const unsigned char *p = data;
    const uint64_t E = 0x7c007c007c007c00ull, ONE = 0x0001000100010001ull, HI = 0x8000800080008000ull;
    size_t i = 0;
    for (; i + 4 <= n; i += 4) {
        uint64_t w;
        memcpy(&w, p + 2 * i, 8);
        const uint64_t u = (w & E) ^ E;
        if ((u - ONE) & ~u & HI) break;
    }
    for (; i < n; i++) {
        uint16_t h;
        memcpy(&h, p + 2 * i, 2);
        if ((h & 0x7c00u) == 0x7c00u) return i;
    }
    return n;
}

static b2k_rk_tile tile_of(const rk_workspace *ws, uint32_t view) {
    const rk_view_desc *v = &ws->plan->views[view];
    const rk_buffer_desc *b = &ws->plan->buffers[v->buffer_id];
    b2k_rk_tile t;
    t.ptr = (char *)ws->slots[b->slot_id].bo.ptr + b->offset + v->offset_bytes;
    t.layout = v->tensor.layout;
    t.rows = v->tensor.rows;
    t.cols = v->tensor.cols;
    t.physical_rows = v->tensor.physical_rows;
    t.physical_cols = v->tensor.physical_cols;
    return t;
}

/* The pack item of upload action `a` reading its source from `src_base` (the value's first
 * element in HBM). */
static b2k_rk_pack pack_of(const rk_workspace *ws, const rk_action_desc *a, const char *src_base) {
    b2k_rk_pack it;
    memset(&it, 0, sizeof(it));
    it.dst = ws->tiles[a->outputs[0]];
    it.rows = it.dst.rows;
    it.cols = it.dst.cols;
    it.clear = 1;
    if (a->flags & RK_ACTION_FLAG_BROADCAST_SCALAR) {
        it.mode = B2K_RK_SRC_SCALAR;
        it.src = src_base;
    } else if (a->flags & RK_ACTION_FLAG_BROADCAST_CHANNEL) {
        it.mode = B2K_RK_SRC_CHANNEL;
        it.src = src_base + 2u * (size_t)a->source_col_offset;
    } else {
        it.mode = B2K_RK_SRC_MATRIX;
        it.transpose = (a->flags & RK_ACTION_FLAG_TRANSPOSE_SOURCE) != 0;
        it.src = src_base + 2u * ((size_t)a->source_row_offset * a->source_row_stride + a->source_col_offset);
        it.ld = a->source_row_stride;
    }
    return it;
}

static int is_constant_upload(const rk_plan *p, const rk_action_desc *a) {
    return a->kind == RK_ACTION_UPLOAD && p->values[a->source_binding].role == RK_ROLE_CONSTANT;
}

/* ------------------------------------------------------------------------------ task chains
 * A chain is MM, then MM_ACC tasks that each take the previous result as their prior, then
 * optionally a LUT task on the last result: consecutive actions whose intermediate results nothing
 * else reads. It runs as one launch that computes the chunk sums in parallel and stores only the
 * final result (b2d_rk_chain), with the separate tasks' arithmetic. An intermediate result is
 * "dead" after its reader when no later action reads any of its bytes before a task output or an
 * upload (uploads rewrite their whole destination view) covers all of them; a LUT reader that writes
 * in place ends the life of its input itself. */
static void view_range(const rk_workspace *ws, uint32_t v, uintptr_t *lo, uintptr_t *hi) {
    *lo = (uintptr_t)ws->tiles[v].ptr;
    *hi = *lo + ws->plan->views[v].tensor.bytes;
}

static int views_overlap(const rk_workspace *ws, uint32_t a, uint32_t b) {
    uintptr_t alo, ahi, blo, bhi;
    view_range(ws, a, &alo, &ahi);
    view_range(ws, b, &blo, &bhi);
    return alo < bhi && blo < ahi;
}

static int same_view(const rk_workspace *ws, uint32_t a, uint32_t b) {
    return ws->tiles[a].ptr == ws->tiles[b].ptr &&
           same_geometry(&ws->plan->views[a].tensor, &ws->plan->views[b].tensor);
}

static int dead_after(const rk_workspace *ws, uint32_t v, uint32_t reader) {
    const rk_plan *p = ws->plan;
    uintptr_t lo, hi;
    view_range(ws, v, &lo, &hi);
    for (uint32_t j = reader; j < p->d.nactions; j++) {
        const rk_action_desc *a = &p->actions[j];
        for (uint32_t k = 0; k < a->ninputs && j > reader; k++)   /* the reader's own reads are checked by the caller */
            if (views_overlap(ws, a->inputs[k], v)) return 0;
        if ((a->kind == RK_ACTION_NPU_TASK || a->kind == RK_ACTION_UPLOAD) && a->noutputs) {
            uintptr_t wlo, whi;
            view_range(ws, a->outputs[0], &wlo, &whi);
            if (wlo <= lo && hi <= whi) return 1;
        }
    }
    return 1;
}

static int is_lut_template(uint32_t t) {
    return t == RK_TEMPLATE_LUT_SIGMOID_F16 || t == RK_TEMPLATE_LUT_HARDSIGMOID_F16 ||
           t == RK_TEMPLATE_LUT_GELU_GATE_F16 || t == RK_TEMPLATE_LUT_RSQRT_F16;
}

/* Finds the chains; returns the scratch doubles and ticket words the largest one needs. */
static void find_chains(rk_workspace *ws, size_t *scratch_doubles, size_t *tickets) {
    const rk_plan *p = ws->plan;
    const uint32_t na = p->d.nactions;
    *scratch_doubles = *tickets = 0;
    ws->nchains = 0;
    for (uint32_t i = 0; i < na; i++) {
        const rk_action_desc *a = &p->actions[i];
        if (a->kind != RK_ACTION_NPU_TASK || a->template_id != RK_TEMPLATE_MM_F16) continue;
        b2k_rk_chain ch;
        memset(&ch, 0, sizeof(ch));
        ch.x[0] = ws->tiles[a->inputs[0]];
        ch.w[0] = ws->tiles[a->inputs[1]];
        ch.n = 1;
        uint32_t out = a->outputs[0], end = i;
        void *lut_dst = NULL;
        while (end + 1 < na && !ch.lut) {
            const uint32_t j = end + 1;
            const rk_action_desc *b = &p->actions[j];
            if (b->kind != RK_ACTION_NPU_TASK) break;
            if (b->template_id == RK_TEMPLATE_MM_ACC_F16 && ch.n < B2K_RK_CHAIN_MAX) {
                if (!same_view(ws, b->inputs[2], out) ||
                    !same_geometry(&p->views[out].tensor, &p->views[b->outputs[0]].tensor) ||
                    views_overlap(ws, b->inputs[0], out) || views_overlap(ws, b->inputs[1], out) ||
                    !dead_after(ws, out, j))
                    break;
                ch.x[ch.n] = ws->tiles[b->inputs[0]];
                ch.w[ch.n] = ws->tiles[b->inputs[1]];
                ch.n++;
            } else if (is_lut_template(b->template_id)) {
                /* element-wise over physical elements: its input must be exactly the bytes of the
                 * last result (in any layout of the same size) and its output as many bytes, so the
                 * final tile is the last result's geometry at the LUT's destination */
                if (ws->tiles[b->inputs[0]].ptr != ws->tiles[out].ptr ||
                    p->views[b->inputs[0]].tensor.bytes != p->views[out].tensor.bytes ||
                    p->views[b->outputs[0]].tensor.bytes != p->views[out].tensor.bytes || !dead_after(ws, out, j))
                    break;
                ch.lut = b->template_id;
                lut_dst = ws->tiles[b->outputs[0]].ptr;
                end = j;
                break;
            } else {
                break;
            }
            out = b->outputs[0];
            end = j;
        }
        if (end == i) continue;
        ch.y = ws->tiles[out];
        if (lut_dst) ch.y.ptr = lut_dst;
        const size_t blocks = (size_t)((ch.y.physical_rows + 7) / 8) * ((ch.y.physical_cols + 31) / 32);
        if (ch.n * blocks * 256 > *scratch_doubles) *scratch_doubles = ch.n * blocks * 256;
        if (blocks > *tickets) *tickets = blocks;
        ws->chains[ws->nchains] = ch;
        ws->chain_head[i] = ++ws->nchains;
        for (uint32_t j = i + 1; j <= end; j++) ws->chain_member[j] = 1;
        i = end;
    }
}

/* The per-run device schedule, in action order: a run of consecutive per-run uploads (neither
 * constant nor persistent) is one pack launch, each task (or chain) one launch, a run of
 * consecutive downloads one unpack launch. Order matters: a plan may map buffers with disjoint live
 * ranges to one slot, so an upload or download may only run at its own position. */
enum { STEP_PACK = 0, STEP_TASK = 1, STEP_UNPACK = 2, STEP_CHAIN = 3 };

static void build_schedule(rk_workspace *ws) {
    const rk_plan *p = ws->plan;
    uint32_t task = 0, unpack = 0;
    ws->npacks = ws->nsteps = 0;
    ws->upload_calls = ws->upload_bytes = 0;
    memset(ws->in_needed, 0, p->d.nvalues);
    for (uint32_t i = 0; i < p->d.nactions; i++) {
        const rk_action_desc *a = &p->actions[i];
        struct rk_step *last = ws->nsteps ? &ws->steps[ws->nsteps - 1] : NULL;
        if (a->kind == RK_ACTION_UPLOAD) {
            if (is_constant_upload(p, a) || ws->persistent[i]) continue;
            if (!last || last->kind != STEP_PACK) ws->steps[ws->nsteps++] = (struct rk_step){STEP_PACK, ws->npacks, 0};
            ws->steps[ws->nsteps - 1].count++;
            ws->packs[ws->npacks++] = pack_of(ws, a, (const char *)ws->in_dev + ws->in_off[a->source_binding]);
            ws->in_needed[a->source_binding] = 1;
            ws->upload_calls++;
            ws->upload_bytes += p->views[a->outputs[0]].tensor.bytes;
        } else if (a->kind == RK_ACTION_NPU_TASK) {
            if (ws->chain_head[i]) ws->steps[ws->nsteps++] = (struct rk_step){STEP_CHAIN, ws->chain_head[i] - 1, 1};
            else if (!ws->chain_member[i]) ws->steps[ws->nsteps++] = (struct rk_step){STEP_TASK, task, 1};
            task++;
        } else if (a->kind == RK_ACTION_DOWNLOAD) {
            if (!last || last->kind != STEP_UNPACK) ws->steps[ws->nsteps++] = (struct rk_step){STEP_UNPACK, unpack, 0};
            ws->steps[ws->nsteps - 1].count++;
            unpack++;
        }
    }
}

/* The steps, then the guard check of every slot, on the handle's stream. */
static int issue_schedule(rk_workspace *ws) {
    int rc = 0;
    for (uint32_t i = 0; i < ws->nsteps && !rc; i++) {
        const struct rk_step *st = &ws->steps[i];
        if (st->kind == STEP_PACK) rc = b2d_rk_pack(ws->dev, ws->packs + st->first, st->count);
        else if (st->kind == STEP_TASK) rc = b2d_rk_task(ws->dev, &ws->tasks[st->first]);
        else if (st->kind == STEP_CHAIN) rc = b2d_rk_chain(ws->dev, &ws->chains[st->first]);
        else rc = b2d_rk_unpack(ws->dev, ws->unpacks + st->first, st->count);
    }
    for (uint32_t g = 0; g < ws->nguard && !rc; g += B2K_MAX_CUBE_TILES) {
        const uint32_t n = ws->nguard - g < B2K_MAX_CUBE_TILES ? ws->nguard - g : B2K_MAX_CUBE_TILES;
        rc = b2d_guard_check(ws->dev, ws->guard_base + g, ws->guard_payload + g, n, CO_SLACK, CO_GUARD);
    }
    return rc;
}

/* Records the schedule as a CUDA graph when the handle supports capture. */
static int capture_schedule(rk_workspace *ws) {
    if (ws->exec) {
        b2d_exec_destroy(ws->exec);
        ws->exec = NULL;
    }
    int rc = b2d_capture_begin(ws->dev);
    if (rc == ROCKET_E_UNSUPPORTED) return 0;
    if (rc) return rc;
    const int issued = issue_schedule(ws);
    unsigned kernels = 0;
    rc = b2d_capture_end(ws->dev, &ws->exec, &kernels);
    return issued ? issued : rc;
}

static void workspace_free(rk_workspace *ws) {
    if (!ws) return;
    if (ws->exec) b2d_exec_destroy(ws->exec);
    if (ws->slots && ws->plan)
        for (uint32_t s = 0; s < ws->plan->d.nbuffers; s++) co_buffer_free(&ws->slots[s]);
    b2h_free(ws->fd, ws->in_dev, ws->in_bytes);
    b2h_free(ws->fd, ws->out_dev, ws->out_bytes);
    b2h_free(ws->fd, ws->scratch_dev, ws->scratch_bytes);
    b2h_free(ws->fd, ws->chain_scratch, ws->chain_scratch_bytes);
    b2h_free(ws->fd, ws->chain_tickets, ws->chain_ticket_bytes);
    b2d_host_free(ws->out_host);
    b2d_host_free(ws->in_host);
    free(ws->slots); free(ws->tiles); free(ws->in_off); free(ws->in_needed); free(ws->out_off);
    free(ws->packs); free(ws->tasks); free(ws->unpacks); free(ws->steps); free(ws->guard_base);
    free(ws->guard_payload);
    free(ws->persistent);
    free(ws->chains); free(ws->chain_head); free(ws->chain_member);
    plan_free(ws->plan);
    free(ws);
}

/* Packs every constant-sourced upload once: the constants are copied to a temporary HBM buffer,
 * packed in one launch and the buffer is released after the stream drained. */
static int upload_constants(rk_workspace *ws, const rk_binding *constants, uint32_t n, rk_diag *diag) {
    const rk_plan *p = ws->plan;
    uint64_t *off = calloc(p->d.nvalues, sizeof(uint64_t));
    b2k_rk_pack *items = malloc((size_t)p->d.nactions * sizeof(b2k_rk_pack));
    if (!off || !items) {
        free(off); free(items);
        return WS_FAIL("workspace_create", RK_E_NOMEM, "out of memory");
    }
    size_t bytes = 0;
    for (uint32_t i = 0; i < p->d.nvalues; i++)
        if (p->values[i].role == RK_ROLE_CONSTANT) {
            off[i] = bytes;
            bytes = align256(bytes + p->values[i].nbytes);
        }
    void *stage = NULL;
    int rc = bytes ? b2h_malloc(ws->fd, bytes, &stage) : 0;
    uint32_t count = 0;
    for (uint32_t i = 0; i < p->d.nvalues && !rc; i++) {
        if (p->values[i].role != RK_ROLE_CONSTANT) continue;
        const rk_binding *b = find_binding(constants, n, i);
        rc = b2d_copy_2d(ws->dev, (char *)stage + off[i], b->nbytes, b->data, b->nbytes, b->nbytes, 1, B2D_H2D);
    }
    for (uint32_t i = 0; i < p->d.nactions && !rc; i++)
        if (is_constant_upload(p, &p->actions[i]))
            items[count++] = pack_of(ws, &p->actions[i], (const char *)stage + off[p->actions[i].source_binding]);
    if (!rc) rc = b2d_rk_pack(ws->dev, items, count);
    const int sync = b2d_sync(ws->dev);
    if (!rc) rc = sync;
    b2h_free(ws->fd, stage, bytes);
    free(off);
    free(items);
    if (rc) return diag_set(diag, rc == ROCKET_E_NOMEM ? RK_E_NOMEM : RK_E_DEVICE, "workspace_create",
                            "constant upload failed", UINT32_MAX, NULL, rc);
    return 0;
}

static int workspace_create_impl(int fd, const rk_plan *plan, const rk_binding *constants, uint32_t nconstants,
                                 rk_workspace **out, rk_diag *diag) {
    diag_clear(diag);
    if (!out) return RK_E_INVALID;
    *out = NULL;
    if (!plan || fd < 0)
        return WS_FAIL("workspace_create", RK_E_INVALID, "fd>=0 and a validated plan are required");
    int rc = rk_target_check(diag);
    if (rc) return rc;
    b2_dev *dev = b2h_dev(fd);
    if (!dev) return WS_FAIL("workspace_create", RK_E_DEVICE, "fd is not an open device handle");
    if ((nconstants && !constants) || nconstants > plan->d.nvalues)
        return WS_FAIL("workspace_create", RK_E_SCHEMA, "constant pointer/count mismatch");
    uint32_t nconst_values = 0;
    for (uint32_t i = 0; i < plan->d.nvalues; i++) nconst_values += plan->values[i].role == RK_ROLE_CONSTANT;
    if (nconstants != nconst_values) return WS_FAIL("workspace_create", RK_E_SHAPE, "constant binding count mismatch");
    for (uint32_t i = 0; i < plan->d.nvalues; i++) {
        if (plan->values[i].role != RK_ROLE_CONSTANT) continue;
        const rk_binding *b = find_binding(constants, nconstants, i);
        rc = binding_matches(&plan->values[i], b, "workspace_create", diag);
        if (rc) return rc;
        if (first_nonfinite(b->data, b->nbytes / 2u) != b->nbytes / 2u)
            return WS_FAIL("workspace_create", RK_E_NUMERIC_CONTRACT,
                           "non-finite FP16 input/constant is rejected before upload");
    }
    rk_workspace *ws = calloc(1, sizeof(*ws));
    if (!ws) return WS_FAIL("workspace_create", RK_E_NOMEM, "out of memory");
    ws->fd = fd;
    ws->dev = dev;
    atomic_init(&ws->busy, 0);
    atomic_init(&ws->poisoned, 0);
    if (plan_copy(&plan->d, &ws->plan)) {
        free(ws);
        return WS_FAIL("workspace_create", RK_E_NOMEM, "out of memory");
    }
    const rk_plan *p = ws->plan;
    const uint32_t nv = p->d.nvalues, na = p->d.nactions, nb = p->d.nbuffers;
    ws->slots = calloc(nb, sizeof(co_buffer));
    ws->tiles = calloc(p->d.nviews, sizeof(b2k_rk_tile));
    ws->in_off = calloc(nv, sizeof(uint64_t));
    ws->in_needed = calloc(nv, 1);
    ws->out_off = calloc(nv, sizeof(uint64_t));
    ws->packs = calloc(na, sizeof(b2k_rk_pack));
    ws->tasks = calloc(na, sizeof(b2k_rk_task));
    ws->unpacks = calloc(na, sizeof(b2k_rk_unpack));
    ws->steps = calloc(na, sizeof(*ws->steps));
    ws->guard_base = calloc(nb, sizeof(void *));
    ws->guard_payload = calloc(nb, sizeof(size_t));
    ws->persistent = calloc(na, 1);
    ws->chains = calloc(na ? na : 1, sizeof(b2k_rk_chain));
    ws->chain_head = calloc(na ? na : 1, sizeof(uint32_t));
    ws->chain_member = calloc(na ? na : 1, 1);
    if (!ws->slots || !ws->tiles || !ws->in_off || !ws->in_needed || !ws->out_off || !ws->packs || !ws->tasks ||
        !ws->unpacks || !ws->steps || !ws->guard_base || !ws->guard_payload || !ws->persistent || !ws->chains ||
        !ws->chain_head || !ws->chain_member) {
        workspace_free(ws);
        return WS_FAIL("workspace_create", RK_E_NOMEM, "out of memory");
    }
    /* slots: one allocation of the largest end offset of the buffers mapped to it */
    uint64_t *slot_end = calloc(nb, sizeof(uint64_t));
    if (!slot_end) {
        workspace_free(ws);
        return WS_FAIL("workspace_create", RK_E_NOMEM, "out of memory");
    }
    for (uint32_t i = 0; i < nb; i++) {
        const rk_buffer_desc *b = &p->buffers[i];
        if (b->offset + b->capacity > slot_end[b->slot_id]) slot_end[b->slot_id] = b->offset + b->capacity;
    }
    for (uint32_t s = 0; s < nb && !rc; s++) {
        if (!slot_end[s]) continue;
        rc = co_buffer_alloc(fd, (size_t)slot_end[s], &ws->slots[s]);
        if (!rc) {
            ws->guard_base[ws->nguard] = ws->slots[s].bo.ptr;
            ws->guard_payload[ws->nguard++] = ws->slots[s].payload;
            ws->device_bytes += slot_end[s] + CO_SLACK + CO_GUARD;
        }
    }
    free(slot_end);
    if (rc) {
        workspace_free(ws);
        return diag_set(diag, rc == ROCKET_E_NOMEM ? RK_E_NOMEM : RK_E_DEVICE, "workspace_create",
                        "co_buffer_alloc failed", UINT32_MAX, NULL, rc);
    }
    for (uint32_t v = 0; v < p->d.nviews; v++) ws->tiles[v] = tile_of(ws, v);
    /* input and output staging */
    for (uint32_t i = 0; i < nv; i++) {
        const rk_value_desc *v = &p->values[i];
        if (v->role == RK_ROLE_INPUT) {
            ws->ninputs++;
            ws->in_off[i] = ws->in_bytes;
            ws->in_bytes = align256(ws->in_bytes + v->nbytes);
        } else if (v->role == RK_ROLE_OUTPUT) {
            ws->noutputs++;
            ws->out_off[i] = ws->out_bytes;
            ws->out_bytes = align256(ws->out_bytes + v->nbytes);
        } else if (v->role == RK_ROLE_CONSTANT) {
            ws->nconstants++;
        }
    }
    if (ws->in_bytes) {
        rc = b2h_malloc(fd, ws->in_bytes, &ws->in_dev);
        if (!rc && !(ws->in_host = b2d_host_alloc(ws->in_bytes))) rc = ROCKET_E_NOMEM;
    }
    if (!rc) rc = b2h_malloc(fd, ws->out_bytes, &ws->out_dev);
    if (!rc && !(ws->out_host = b2d_host_alloc(ws->out_bytes))) rc = ROCKET_E_NOMEM;
    if (rc) {
        workspace_free(ws);
        return diag_set(diag, rc == ROCKET_E_NOMEM ? RK_E_NOMEM : RK_E_DEVICE, "workspace_create",
                        "staging allocation failed", UINT32_MAX, NULL, rc);
    }
    ws->device_bytes += ws->in_bytes + ws->out_bytes;
    /* the schedule */
    for (uint32_t i = 0; i < na; i++) {
        const rk_action_desc *a = &p->actions[i];
        if (a->kind == RK_ACTION_NPU_TASK) {
            b2k_rk_task *t = &ws->tasks[ws->ntasks++];
            memset(t, 0, sizeof(*t));
            t->op = a->template_id;
            t->x = ws->tiles[a->inputs[0]];
            t->y = ws->tiles[a->outputs[0]];
            if (a->template_id == RK_TEMPLATE_MM_F16 || a->template_id == RK_TEMPLATE_MM_ACC_F16) {
                t->w = ws->tiles[a->inputs[1]];
                if (a->template_id == RK_TEMPLATE_MM_ACC_F16) t->aux = ws->tiles[a->inputs[2]];
            } else if (is_ew(a->template_id)) {
                t->w = ws->tiles[a->inputs[2]];          /* the identity operand */
                t->aux = ws->tiles[a->inputs[1]];
            }
        } else if (a->kind == RK_ACTION_DOWNLOAD) {
            const rk_publish_desc *pub = NULL;
            for (uint32_t q = 0; q < p->d.npublish && !pub; q++)
                if (p->publish[q].binding_id == a->source_binding && p->publish[q].view_id == a->inputs[0])
                    pub = &p->publish[q];
            const rk_value_desc *v = &p->values[a->source_binding];
            b2k_rk_unpack *u = &ws->unpacks[ws->nunpacks++];
            u->src = ws->tiles[a->inputs[0]];
            u->dst = (char *)ws->out_dev + ws->out_off[a->source_binding] +
                     2u * ((size_t)pub->dst_row_offset * v->shape[1] + pub->dst_col_offset);
            u->ld = v->shape[1];
            ws->download_bytes += p->views[a->inputs[0]].tensor.bytes;
        }
    }
    for (uint32_t s = 0; s < p->d.nsubmits; s++) ws->task_count += p->submits[s].ntask_ids;
    size_t chain_doubles = 0, chain_words = 0;
    find_chains(ws, &chain_doubles, &chain_words);
    if (ws->nchains) {
        ws->chain_scratch_bytes = chain_doubles * sizeof(double);
        ws->chain_ticket_bytes = chain_words * sizeof(unsigned);
        rc = b2h_malloc(fd, ws->chain_scratch_bytes, &ws->chain_scratch);
        if (!rc) rc = b2h_malloc(fd, ws->chain_ticket_bytes, &ws->chain_tickets);
        if (rc) {
            workspace_free(ws);
            return diag_set(diag, rc == ROCKET_E_NOMEM ? RK_E_NOMEM : RK_E_DEVICE, "workspace_create",
                            "chain scratch allocation failed", UINT32_MAX, NULL, rc);
        }
        ws->device_bytes += ws->chain_scratch_bytes + ws->chain_ticket_bytes;
        for (uint32_t c = 0; c < ws->nchains; c++) {
            ws->chains[c].scratch = ws->chain_scratch;
            ws->chains[c].tickets = ws->chain_tickets;
        }
    }
    build_schedule(ws);
    rc = upload_constants(ws, constants, nconstants, diag);
    if (rc) {
        workspace_free(ws);
        return rc;
    }
    rc = capture_schedule(ws);
    if (rc) {
        workspace_free(ws);
        return diag_set(diag, RK_E_DEVICE, "workspace_create", "recording the device schedule failed", UINT32_MAX,
                        NULL, rc);
    }
    *out = ws;
    return 0;
}

int rk_workspace_create(int fd, const rk_plan *plan, const rk_binding *constants, uint32_t nconstants,
                        rk_workspace **out, rk_diag *diag) {
    return workspace_create_impl(fd, plan, constants, nconstants, out, diag);
}

int rk_workspace_create_shared(int fd, const rk_plan *plan, const rk_binding *constants, uint32_t nconstants,
                               const rk_shared_constant_binding *shared, uint32_t nshared, rk_workspace **out,
                               rk_diag *diag) {
    if (nshared) {
        diag_clear(diag);
        if (out) *out = NULL;
        return WS_FAIL("workspace_create", RK_E_UNSUPPORTED,
                       "shared packed constants are an NPU buffer-object cache; pass them as constants");
    }
    return workspace_create_impl(fd, plan, constants, nconstants, out, diag);
}

/* ------------------------------------------------------------------------------ runs */
typedef struct {
    double validate_us, pack_us, wait_us, download_us, guard_us, publish_us, alloc_us;
    uint32_t completed, fail_repeat, fail_action;
    uint32_t prior_status;           /* status bits of earlier work on the handle, restored after */
} run_stats;

static int run_gate(rk_workspace *ws, const char *stage, rk_diag *diag) {
    if (atomic_exchange(&ws->busy, 1)) return WS_FAIL(stage, RK_E_BUSY, "workspace is already running");
    if (atomic_load(&ws->poisoned)) {
        atomic_store(&ws->busy, 0);
        return WS_FAIL(stage, RK_E_POISONED, "workspace is poisoned after an unclassified device error");
    }
    return 0;
}

static int ranges_overlap(const void *a, uint64_t an, const void *b, uint64_t bn) {
    const uintptr_t x = (uintptr_t)a, y = (uintptr_t)b;
    return an && bn && x < y + bn && y < x + an;
}

/* Binding checks of one repeat (rk_plan_runtime.c:1700-1760), before any device work. */
static int check_bindings(rk_workspace *ws, const rk_binding *in, uint32_t nin, const rk_binding *out, uint32_t nout,
                          rk_diag *diag) {
    const rk_plan *p = ws->plan;
    if (nin != ws->ninputs || nout != ws->noutputs || (nin && !in) || (nout && !out))
        return WS_FAIL("run", RK_E_SHAPE, "input/output binding count mismatch");
    for (uint32_t i = 0; i < p->d.nvalues; i++) {
        const rk_value_desc *v = &p->values[i];
        if (v->role != RK_ROLE_INPUT && v->role != RK_ROLE_OUTPUT) continue;
        const int input = v->role == RK_ROLE_INPUT;
        const rk_binding *b = find_binding(input ? in : out, input ? nin : nout, i);
        int rc = binding_matches(v, b, "run", diag);
        if (rc) return rc;
        if (!input) continue;
        int seen = 0;
        for (uint32_t j = 0; j < i && !seen; j++) {
            if (p->values[j].role != RK_ROLE_INPUT) continue;
            const rk_binding *o = find_binding(in, nin, j);
            seen = o->data == b->data && o->nbytes == b->nbytes;
        }
        if (!seen && first_nonfinite(b->data, b->nbytes / 2u) != b->nbytes / 2u)
            return WS_FAIL("run", RK_E_NUMERIC_CONTRACT, "non-finite FP16 input/constant is rejected before upload");
    }
    for (uint32_t i = 0; i < nin; i++)
        for (uint32_t j = 0; j < nout; j++)
            if (ranges_overlap(in[i].data, in[i].nbytes, out[j].data, out[j].nbytes))
                return WS_FAIL("run", RK_E_ALIAS, "input and output host ranges overlap");
    for (uint32_t i = 0; i < nout; i++)
        for (uint32_t j = 0; j < i; j++)
            if (ranges_overlap(out[i].data, out[i].nbytes, out[j].data, out[j].nbytes))
                return WS_FAIL("run", RK_E_ALIAS, "output host ranges overlap");
    return 0;
}

/* The download action whose published tile holds element (r, c) of output value v. */
static uint32_t download_at(const rk_plan *p, uint32_t v, uint32_t r, uint32_t c) {
    for (uint32_t q = 0; q < p->d.npublish; q++) {
        const rk_publish_desc *t = &p->publish[q];
        if (t->binding_id != v || r < t->dst_row_offset || r - t->dst_row_offset >= t->rows || c < t->dst_col_offset ||
            c - t->dst_col_offset >= t->cols)
            continue;
        for (uint32_t i = 0; i < p->d.nactions; i++)
            if (p->actions[i].kind == RK_ACTION_DOWNLOAD && p->actions[i].source_binding == v &&
                p->actions[i].inputs[0] == t->view_id)
                return i;
    }
    return UINT32_MAX;
}

/* One repeat on the device: inputs to HBM, the schedule, outputs to `staged` (host, out_bytes),
 * then the finiteness check of every published element. */
static int run_once(rk_workspace *ws, const rk_binding *in, uint32_t nin, void *staged, run_stats *st,
                    rk_diag *diag) {
    const rk_plan *p = ws->plan;
    double t0 = now_us();
    int rc = 0;
    /* the inputs the schedule reads, through pinned staging, as one asynchronous copy (the previous
     * run's copy finished at its sync) */
    size_t end = 0;
    for (uint32_t i = 0; i < p->d.nvalues; i++) {
        if (!ws->in_needed[i]) continue;
        const rk_binding *b = find_binding(in, nin, i);
        memcpy((char *)ws->in_host + ws->in_off[i], b->data, b->nbytes);
        if (ws->in_off[i] + b->nbytes > end) end = ws->in_off[i] + b->nbytes;
    }
    if (end) rc = b2d_copy_2d(ws->dev, ws->in_dev, end, ws->in_host, end, end, 1, B2D_H2D);
    double t1 = now_us();
    st->pack_us += t1 - t0;
    if (!rc) rc = ws->exec ? b2d_exec_launch(ws->dev, ws->exec) : issue_schedule(ws);
    if (!rc) rc = b2d_copy_2d(ws->dev, ws->out_host, ws->out_bytes, ws->out_dev, ws->out_bytes, ws->out_bytes, 1,
                              B2D_D2H);
    if (!rc) rc = b2d_sync(ws->dev);
    double t2 = now_us();
    st->wait_us += t2 - t1;
    if (rc) {
        atomic_store(&ws->poisoned, 1);
        return diag_set(diag, RK_E_DEVICE, "run", "device schedule failed; workspace is poisoned", UINT32_MAX, NULL,
                        rc);
    }
    if (staged != ws->out_host) memcpy(staged, ws->out_host, ws->out_bytes);
    for (uint32_t i = 0; i < p->d.nvalues; i++) {
        const rk_value_desc *v = &p->values[i];
        if (v->role != RK_ROLE_OUTPUT) continue;
        const size_t n = v->nbytes / 2u, bad = first_nonfinite((const char *)staged + ws->out_off[i], n);
        if (bad == n) continue;
        const uint32_t a = download_at(p, i, (uint32_t)(bad / v->shape[1]), (uint32_t)(bad % v->shape[1]));
        st->fail_action = a;
        st->download_us += now_us() - t2;
        return diag_set(diag, RK_E_NUMERIC_CONTRACT, "run", "downloaded output tile is not finite; refusing to publish",
                        a, a != UINT32_MAX ? p->actions[a].origin : NULL, 0);
    }
    st->download_us += now_us() - t2;
    return 0;
}

/* Slack/guard bytes of every slot, as the schedule's guard check left them (status bit). */
static int publication_gate(rk_workspace *ws, run_stats *st, rk_diag *diag) {
    const double t0 = now_us();
    const uint32_t bits = b2d_status(ws->dev, 1);
    b2d_status_merge(ws->dev, st->prior_status | (bits & ~(uint32_t)B2D_ST_GUARD));
    st->guard_us += now_us() - t0;
    if (bits & B2D_ST_GUARD) {
        atomic_store(&ws->poisoned, 1);
        return WS_FAIL("run", RK_E_DEVICE, "data BO slack/guard check failed; refusing to publish");
    }
    return 0;
}

static void publish(rk_workspace *ws, const rk_binding *out, uint32_t nout, const void *staged) {
    for (uint32_t j = 0; j < nout; j++)
        memcpy((void *)out[j].data, (const char *)staged + ws->out_off[out[j].id], out[j].nbytes);
}

/* The shared body of run, run_ex and run_group: repeat r reads ins[r] and publishes into outs[r]. */
static int run_body(rk_workspace *ws, const rk_binding *const *ins, const rk_binding *const *outs, uint32_t nrepeat,
                    run_stats *st, rk_diag *diag) {
    st->fail_repeat = st->fail_action = UINT32_MAX;
    double t0 = now_us();
    for (uint32_t r = 0; r < nrepeat; r++) {
        int rc = check_bindings(ws, ins[r], ws->ninputs, outs[r], ws->noutputs, diag);
        if (rc) {
            st->fail_repeat = r;
            st->validate_us += now_us() - t0;
            return rc;
        }
    }
    double t1 = now_us();
    st->validate_us += t1 - t0;
    void *staged = ws->out_host;
    if (nrepeat > 1 && !(staged = malloc((size_t)nrepeat * ws->out_bytes)))
        return WS_FAIL("run", RK_E_NOMEM, "out of memory");
    st->alloc_us += now_us() - t1;
    st->prior_status = b2d_status(ws->dev, 1);
    int rc = 0;
    for (uint32_t r = 0; r < nrepeat && !rc; r++) {
        rc = run_once(ws, ins[r], ws->ninputs, (char *)staged + (nrepeat > 1 ? (size_t)r * ws->out_bytes : 0), st,
                      diag);
        if (rc) st->fail_repeat = r;
        else st->completed++;
    }
    if (!rc) rc = publication_gate(ws, st, diag);
    else b2d_status_merge(ws->dev, st->prior_status);
    if (!rc) {
        const double p0 = now_us();
        for (uint32_t r = 0; r < nrepeat; r++)
            publish(ws, outs[r], ws->noutputs, (char *)staged + (nrepeat > 1 ? (size_t)r * ws->out_bytes : 0));
        st->publish_us += now_us() - p0;
    }
    if (staged != ws->out_host) free(staged);
    return rc;
}

int rk_workspace_run(rk_workspace *ws, const rk_binding *inputs, uint32_t ninputs, const rk_binding *outputs,
                     uint32_t noutputs, rk_run_report *report, rk_diag *diag) {
    diag_clear(diag);
    if (!ws) return WS_FAIL("run", RK_E_INVALID, "null workspace");
    int rc = run_gate(ws, "run", diag);
    if (rc) return rc;
    run_stats st;
    memset(&st, 0, sizeof(st));
    if (ninputs != ws->ninputs || noutputs != ws->noutputs || (ninputs && !inputs) || (noutputs && !outputs))
        rc = WS_FAIL("run", RK_E_SHAPE, "input/output binding count mismatch");
    else
        rc = run_body(ws, &inputs, &outputs, 1, &st, diag);
    if (report) {
        memset(report, 0, sizeof(*report));
        report->abi_version = RK_ABI_VERSION;
        report->struct_size = sizeof(*report);
        report->fail_action_id = st.fail_action;
        report->numeric_mode = 1;
        if (st.completed) {
            report->task_count = ws->task_count;
            report->submit_count = ws->plan->d.nsubmits;
            report->upload_calls = ws->upload_calls;
            report->upload_bytes = ws->upload_bytes;
            report->download_calls = ws->nunpacks;
            report->download_bytes = ws->download_bytes;
        }
        report->pack_us = st.pack_us;
        report->submit_wait_us = st.wait_us;
        report->output_sync_us = st.download_us;
    }
    atomic_store(&ws->busy, 0);
    return rc;
}

int rk_workspace_run_ex(rk_workspace *ws, const rk_binding *inputs, uint32_t ninputs, const rk_binding *outputs,
                        uint32_t noutputs, rk_run_attribution *envelope, rk_diag *diag) {
    diag_clear(diag);
    if (!ws) return WS_FAIL("run", RK_E_INVALID, "null workspace");
    if (!envelope || envelope->struct_size < RK_RUN_ATTRIBUTION_V1_SIZE ||
        envelope->struct_size > sizeof(rk_run_attribution))
        return WS_FAIL("run", RK_E_SCHEMA, "rk_run_attribution struct_size is missing or unusable");
    const uint32_t size = envelope->struct_size;
    const double t0 = now_us();
    int rc = run_gate(ws, "run", diag);
    if (rc) return rc;
    run_stats st;
    memset(&st, 0, sizeof(st));
    if (ninputs != ws->ninputs || noutputs != ws->noutputs || (ninputs && !inputs) || (noutputs && !outputs))
        rc = WS_FAIL("run", RK_E_SHAPE, "input/output binding count mismatch");
    else
        rc = run_body(ws, &inputs, &outputs, 1, &st, diag);
    rk_run_attribution a;
    memset(&a, 0, sizeof(a));
    a.abi_version = RK_ABI_VERSION;
    a.struct_size = size;
    a.fail_action_id = st.fail_action;
    a.numeric_mode = 1;
    if (st.completed) {
        a.task_count = ws->task_count;
        a.submit_count = ws->plan->d.nsubmits;
        a.upload_calls = ws->upload_calls;
        a.upload_bytes = ws->upload_bytes;
        a.download_calls = ws->nunpacks;
        a.download_bytes = ws->download_bytes;
    }
    a.validate_us = st.validate_us;
    a.pack_us = a.pack_layout_us = st.pack_us;
    a.submit_wait_us = st.wait_us;
    a.download_us = st.download_us;
    a.guard_us = st.guard_us;
    a.publish_us = st.publish_us;
    a.alloc_us = st.alloc_us;
    a.upload_coalesce = 1;
    a.upload_fast_pack = 1;
    const double t1 = now_us();
    a.clock_us = now_us() - t1;
    a.total_us = t1 - t0;
    memcpy(envelope, &a, size);
    atomic_store(&ws->busy, 0);
    return rc;
}

int rk_workspace_run_group(rk_workspace *ws, const rk_binding *bindings, uint32_t nrepeat, rk_group_report *report,
                           rk_diag *diag) {
    diag_clear(diag);
    if (!ws) return WS_FAIL("run_group", RK_E_INVALID, "null workspace");
    if (!report || report->struct_size < RK_GROUP_REPORT_V1_SIZE || report->struct_size > sizeof(rk_group_report))
        return WS_FAIL("run_group", RK_E_SCHEMA, "rk_group_report struct_size is missing or unusable");
    const uint32_t size = report->struct_size;
    if (!nrepeat || nrepeat > 65536u || !bindings)
        return WS_FAIL("run_group", RK_E_SHAPE, "a group needs 1..65536 repeats and their bindings");
    const double t0 = now_us();
    int rc = run_gate(ws, "run_group", diag);
    if (rc) return rc;
    const uint32_t per = ws->ninputs + ws->noutputs;
    const rk_binding **ins = malloc((size_t)nrepeat * sizeof(*ins)), **outs = malloc((size_t)nrepeat * sizeof(*outs));
    run_stats st;
    memset(&st, 0, sizeof(st));
    if (!ins || !outs) {
        rc = WS_FAIL("run_group", RK_E_NOMEM, "out of memory");
    } else {
        for (uint32_t r = 0; r < nrepeat; r++) {
            ins[r] = bindings + (size_t)r * per;
            outs[r] = bindings + (size_t)r * per + ws->ninputs;
        }
        rc = run_body(ws, ins, outs, nrepeat, &st, diag);
    }
    free(ins);
    free(outs);
    rk_group_report g;
    memset(&g, 0, sizeof(g));
    g.abi_version = RK_ABI_VERSION;
    g.struct_size = size;
    g.repeat_count = nrepeat;
    g.repeat_completed = st.completed;
    g.fail_repeat = st.fail_repeat;
    g.fail_action_id = st.fail_action;
    g.task_count = ws->task_count * st.completed;
    g.submit_count = ws->plan->d.nsubmits * st.completed;
    g.numeric_mode = 1;
    g.upload_calls = ws->upload_calls * st.completed;
    g.upload_bytes = ws->upload_bytes * st.completed;
    g.download_calls = (uint64_t)ws->nunpacks * st.completed;
    g.download_bytes = ws->download_bytes * st.completed;
    g.validate_us = st.validate_us;
    g.pack_us = st.pack_us;
    g.submit_wait_us = st.wait_us;
    g.download_us = st.download_us;
    g.guard_us = st.guard_us;
    g.publish_us = st.publish_us;
    g.alloc_us = st.alloc_us;
    g.total_us = now_us() - t0;
    memcpy(report, &g, size);
    atomic_store(&ws->busy, 0);
    return rc;
}

int rk_workspace_destroy(rk_workspace *ws, rk_diag *diag) {
    diag_clear(diag);
    if (!ws) return 0;
    if (atomic_exchange(&ws->busy, 1))
        return WS_FAIL("workspace_destroy", RK_E_BUSY, "destroy raced a running workspace");
    /* A poisoned workspace is released once its stream drained; if the device no longer answers,
     * nothing is freed that it may still touch and the handle stays the caller's. */
    if (b2d_sync(ws->dev) && atomic_load(&ws->poisoned)) {
        atomic_store(&ws->busy, 0);
        return WS_FAIL("workspace_destroy", RK_E_POISONED, "workspace is poisoned; process-level recovery required");
    }
    workspace_free(ws);
    return 0;
}

/* ------------------------------------------------------------------------------ persistent uploads */
static int state_gate(rk_workspace *ws, rk_diag *diag) {
    if (!ws) return WS_FAIL("state", RK_E_INVALID, "null workspace");
    if (atomic_exchange(&ws->busy, 1)) return WS_FAIL("state", RK_E_BUSY, "workspace is already running or destroying");
    if (atomic_load(&ws->poisoned)) {
        atomic_store(&ws->busy, 0);
        return WS_FAIL("state", RK_E_POISONED, "workspace is poisoned; state mutation refused");
    }
    return 0;
}

#define STATE_FAIL(code, msg, a) diag_set(diag, (code), "state", (msg), (a), NULL, 0)

int rk_workspace_set_persistent_upload(rk_workspace *ws, uint32_t action_id, rk_diag *diag) {
    diag_clear(diag);
    int rc = state_gate(ws, diag);
    if (rc) return rc;
    const rk_plan *p = ws->plan;
    if (action_id >= p->d.nactions) rc = STATE_FAIL(RK_E_SCHEMA, "invalid persistent upload action", action_id);
    else if (p->actions[action_id].kind != RK_ACTION_UPLOAD || p->actions[action_id].noutputs != 1)
        rc = STATE_FAIL(RK_E_SCHEMA, "persistent state requires a single-output upload action", action_id);
    else if (!ws->persistent[action_id]) {
        ws->persistent[action_id] = 1;
        build_schedule(ws);
        rc = capture_schedule(ws);
        if (rc) {
            atomic_store(&ws->poisoned, 1);
            rc = diag_set(diag, RK_E_DEVICE, "state", "recording the device schedule failed", action_id, NULL, rc);
        }
    }
    atomic_store(&ws->busy, 0);
    return rc;
}

int rk_workspace_update_upload_region(rk_workspace *ws, uint32_t action_id, const rk_state_source *source,
                                      uint32_t src_row, uint32_t src_col, uint32_t dst_row, uint32_t dst_col,
                                      uint32_t rows, uint32_t cols, rk_diag *diag) {
    diag_clear(diag);
    int rc = state_gate(ws, diag);
    if (rc) return rc;
    const rk_plan *p = ws->plan;
    if (action_id >= p->d.nactions || !ws->persistent[action_id]) {
        rc = STATE_FAIL(RK_E_SCHEMA, "region update requires a persistent upload action", action_id);
        goto out;
    }
    if (!source || !source->data || !source->nbytes || !rows || !cols || !source->row_stride) {
        rc = STATE_FAIL(RK_E_SCHEMA, "invalid state source or upload action", action_id);
        goto out;
    }
    const b2k_rk_tile dst = ws->tiles[p->actions[action_id].outputs[0]];
    if ((uint64_t)dst_row + rows > dst.rows || (uint64_t)dst_col + cols > dst.cols) {
        rc = STATE_FAIL(RK_E_SHAPE, "state region is outside the destination tensor", action_id);
        goto out;
    }
    const int transpose = (source->flags & RK_STATE_SOURCE_TRANSPOSE) != 0;
    const uint64_t srows = transpose ? cols : rows, scols = transpose ? rows : cols;
    if (((uint64_t)src_row + srows - 1u) * source->row_stride + src_col + scols - 1u >= source->nbytes / 2u) {
        rc = STATE_FAIL(RK_E_SHAPE, "state source region exceeds the supplied buffer", action_id);
        goto out;
    }
    const size_t need = (size_t)(srows * scols * 2u);
    if (need > ws->scratch_bytes) {
        b2h_free(ws->fd, ws->scratch_dev, ws->scratch_bytes);
        ws->scratch_dev = NULL;
        ws->scratch_bytes = 0;
        rc = b2h_malloc(ws->fd, align256(need), &ws->scratch_dev);
        if (rc) {
            rc = diag_set(diag, RK_E_NOMEM, "state", "out of memory", action_id, NULL, rc);
            goto out;
        }
        ws->scratch_bytes = align256(need);
    }
    const char *window = (const char *)source->data + 2u * ((size_t)src_row * source->row_stride + src_col);
    rc = b2d_copy_2d(ws->dev, ws->scratch_dev, (size_t)scols * 2u, window, (size_t)source->row_stride * 2u,
                     (size_t)scols * 2u, (size_t)srows, B2D_H2D);
    b2k_rk_pack it;
    memset(&it, 0, sizeof(it));
    it.dst = dst;
    it.r0 = dst_row;
    it.c0 = dst_col;
    it.rows = rows;
    it.cols = cols;
    it.mode = B2K_RK_SRC_MATRIX;
    it.transpose = transpose;
    it.src = ws->scratch_dev;
    it.ld = scols;
    if (!rc) rc = b2d_rk_pack(ws->dev, &it, 1);
    const int sync = b2d_sync(ws->dev);
    if (!rc) rc = sync;
    if (rc) {
        atomic_store(&ws->poisoned, 1);
        rc = diag_set(diag, RK_E_DEVICE, "state", "state region upload failed", action_id, NULL, rc);
    }
out:
    atomic_store(&ws->busy, 0);
    return rc;
}

int rk_workspace_clear_upload_destination(rk_workspace *ws, uint32_t action_id, rk_diag *diag) {
    diag_clear(diag);
    int rc = state_gate(ws, diag);
    if (rc) return rc;
    if (action_id >= ws->plan->d.nactions || !ws->persistent[action_id]) {
        rc = STATE_FAIL(RK_E_SCHEMA, "clear requires a persistent upload action", action_id);
    } else {
        b2k_rk_pack it;
        memset(&it, 0, sizeof(it));
        it.dst = ws->tiles[ws->plan->actions[action_id].outputs[0]];
        it.clear = 1;
        rc = b2d_rk_pack(ws->dev, &it, 1);
        const int sync = b2d_sync(ws->dev);
        if (!rc) rc = sync;
        if (rc) {
            atomic_store(&ws->poisoned, 1);
            rc = diag_set(diag, RK_E_DEVICE, "state", "clearing the destination failed", action_id, NULL, rc);
        }
    }
    atomic_store(&ws->busy, 0);
    return rc;
}

/* ------------------------------------------------------------------------------ diagnostics entries */
int rk_workspace_get_cache_info(rk_workspace *ws, rk_workspace_cache_info *out, rk_diag *diag) {
    diag_clear(diag);
    if (!ws || !out) return WS_FAIL("cache_info", RK_E_INVALID, "null workspace or output");
    memset(out, 0, sizeof(*out));
    out->nsubmits = ws->plan->d.nsubmits;
    out->device_bytes = ws->device_bytes;
    out->host_bytes = ws->out_bytes + sizeof(*ws) +
                      (uint64_t)ws->plan->d.nactions * (sizeof(b2k_rk_pack) + sizeof(b2k_rk_task) + sizeof(b2k_rk_unpack));
    return 0;
}

int rk_workspace_task_cbuf(rk_workspace *ws, uint32_t action_id, uint32_t *values, uint32_t capacity,
                           rk_task_cbuf_info *out, rk_diag *diag) {
    diag_clear(diag);
    return diag_set(diag, RK_E_UNSUPPORTED, "task_cbuf", "NPU command-buffer registers do not exist on a CUDA device",
                    action_id, NULL, 0);
}

int rk_shared_constant_get_or_create(int fd, const rk_plan *plan, uint32_t action_id, const rk_binding *source,
                                     const char *key, rk_shared_constant **out, uint32_t *created, rk_diag *diag) {
    diag_clear(diag);
    if (out) *out = NULL;
    if (created) *created = 0;
    return diag_set(diag, RK_E_UNSUPPORTED, "shared_constant",
                    "shared packed constants are an NPU buffer-object cache; pass them as constants", action_id, NULL,
                    0);
}
void rk_shared_constant_retain(rk_shared_constant *constant) { (void)constant; }
void rk_shared_constant_release(rk_shared_constant *constant) { (void)constant; }
uint64_t rk_shared_constant_bytes(const rk_shared_constant *constant) { return 0; }
uint32_t rk_shared_constant_live(void) { return 0; }
