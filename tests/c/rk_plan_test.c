/* rk_plan_test.c -- the plan/workspace ABI (include/rk_plan.h) end to end.
 *
 * Built two ways (tests/test_rk_plan.py): against the library's host sources and the CPU stand-in
 * of the device seam (tests/c/mock_device.c, -DRK_TEST_MOCK), and against the built library on a
 * B200. It restates the cases of the reference's plan test
 * (research/custom-ops/tests/c/rk_plan_host_test.c): the multi-tile MM published into one output
 * at two row offsets (:64-377) with its overlap / missing-tile / shared-slot rejections, input
 * finiteness rechecked every call and a non-finite result never published; plus K accumulation
 * (MM then MM_ACC), the element-wise and LUT templates, broadcast constants, persistent uploads,
 * run_group / run_ex envelopes and a table of descriptor rejections with their status codes and
 * diagnostic messages. Every expected value is computed here from the templates' definitions
 * (double sums of the FP16 products rounded once, then the epilogue), independently of the
 * oracle the mock runs.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "b2_linear.h"
#include "rk_plan.h"
#include "rocket_b200.h"

#ifdef RK_TEST_MOCK
extern int mock_rk_inject;
size_t b2h_live_bytes(void);
#endif

static unsigned checks, failures;
static int mentions(const char *message, const char *needle) { return !needle || strstr(message, needle); }
#define EXPECT(e) do { checks++; if (!(e)) { failures++; fprintf(stderr, "FAIL line %d: %s\n", __LINE__, #e); } } while (0)
#define EXPECT_CODE(call, want_, needle_) do { \
    checks++; \
    int rc_ = (call); \
    if (rc_ != (want_) || diag.code != (want_) || !mentions(diag.message, (needle_))) { \
        failures++; \
        fprintf(stderr, "FAIL line %d: %s -> rc=%d diag.code=%d \"%s\"\n", __LINE__, #call, rc_, diag.code, \
                diag.message); \
    } \
} while (0)

/* ------------------------------------------------------------------------------ plan builder */
typedef struct {
    rk_value_desc values[8];
    uint32_t nvalues;
    rk_buffer_desc buffers[64];
    uint32_t nbuffers;
    rk_view_desc views[64];
    uint32_t nviews;
    rk_action_desc actions[128];
    uint32_t nactions;
    uint32_t ins[128][3], outs[128][1], deps[128][4];
    rk_submit_desc submits[32];
    uint32_t nsubmits;
    uint32_t tasks[32][16];
    rk_publish_desc publish[64];
    uint32_t npublish;
    const char *names[8];
} pb;

static uint32_t up32(uint32_t v, uint32_t m) { return (v + m - 1) / m * m; }

static uint32_t pb_value(pb *b, uint32_t role, uint32_t rank, uint32_t s0, uint32_t s1, const char *name) {
    rk_value_desc *v = &b->values[b->nvalues];
    memset(v, 0, sizeof(*v));
    v->abi_version = RK_ABI_VERSION;
    v->struct_size = sizeof(*v);
    v->id = b->nvalues;
    v->role = role;
    v->dtype = RK_DTYPE_F16;
    v->rank = rank;
    v->shape[0] = s0;
    v->shape[1] = s1;
    v->nbytes = 2ull * (rank == 0 ? 1 : rank == 1 ? s0 : (uint64_t)s0 * s1);
    v->name = name;
    v->name_len = (uint32_t)strlen(name);
    return b->nvalues++;
}

static rk_tensor_desc tensor(uint32_t layout, uint32_t rows, uint32_t cols) {
    rk_tensor_desc t;
    memset(&t, 0, sizeof(t));
    t.abi_version = RK_ABI_VERSION;
    t.struct_size = sizeof(t);
    t.dtype = RK_DTYPE_F16;
    t.layout = layout;
    t.rows = rows;
    t.cols = cols;
    if (layout == RK_LAYOUT_CUBE_F16) {
        t.physical_rows = up32(rows < 12 ? 12 : rows, 4);
        t.physical_cols = up32(cols, 32);
        t.atom = 8;
    } else if (layout == RK_LAYOUT_WEIGHT_F16) {
        t.physical_rows = up32(rows, 32);
        t.physical_cols = up32(cols, 32);
        t.atom = 32;
    } else {
        t.physical_rows = 1;
        t.physical_cols = cols;
        t.atom = 1;
    }
    t.bytes = 2ull * t.physical_rows * t.physical_cols;
    return t;
}

/* A view over a new buffer in its own slot. */
static uint32_t pb_view(pb *b, uint32_t layout, uint32_t rows, uint32_t cols, uint32_t role) {
    const uint32_t id = b->nbuffers;
    rk_buffer_desc *bu = &b->buffers[id];
    rk_view_desc *v = &b->views[b->nviews];
    memset(bu, 0, sizeof(*bu));
    memset(v, 0, sizeof(*v));
    v->tensor = tensor(layout, rows, cols);
    bu->abi_version = RK_ABI_VERSION;
    bu->struct_size = sizeof(*bu);
    bu->id = id;
    bu->role = role;
    bu->slot_id = id;
    bu->alignment = 16;
    bu->layout_id = layout;
    bu->capacity = v->tensor.bytes;
    v->abi_version = RK_ABI_VERSION;
    v->struct_size = sizeof(*v);
    v->id = b->nviews;
    v->buffer_id = id;
    v->valid_region[1] = rows;
    v->valid_region[3] = cols;
    b->nbuffers++;
    return b->nviews++;
}

static rk_action_desc *pb_action(pb *b, uint32_t kind) {
    const uint32_t id = b->nactions++;
    rk_action_desc *a = &b->actions[id];
    memset(a, 0, sizeof(*a));
    a->abi_version = RK_ABI_VERSION;
    a->struct_size = sizeof(*a);
    a->id = id;
    a->kind = kind;
    a->inputs = b->ins[id];
    a->outputs = b->outs[id];
    a->deps = b->deps[id];
    snprintf(a->origin, sizeof(a->origin), "case:%u", id);
    return a;
}

static uint32_t pb_upload(pb *b, uint32_t value, uint32_t view, uint32_t row_off, uint32_t col_off, uint32_t flags) {
    rk_action_desc *a = pb_action(b, RK_ACTION_UPLOAD);
    a->source_binding = value;
    a->source_row_offset = row_off;
    a->source_col_offset = col_off;
    a->source_row_stride = b->values[value].rank == 2 ? b->values[value].shape[1] : 0;
    a->flags = flags;
    a->noutputs = 1;
    b->outs[a->id][0] = view;
    return a->id;
}

static uint32_t pb_task(pb *b, uint32_t tpl, const uint32_t *in, uint32_t nin, uint32_t out, const uint32_t *dep,
                        uint32_t ndep) {
    rk_action_desc *a = pb_action(b, RK_ACTION_NPU_TASK);
    a->template_id = tpl;
    a->ninputs = nin;
    a->noutputs = 1;
    a->ndeps = ndep;
    memcpy(b->ins[a->id], in, nin * sizeof(uint32_t));
    b->outs[a->id][0] = out;
    memcpy(b->deps[a->id], dep, ndep * sizeof(uint32_t));
    return a->id;
}

static uint32_t pb_download(pb *b, uint32_t value, uint32_t view, uint32_t dep, uint32_t row, uint32_t col) {
    rk_action_desc *a = pb_action(b, RK_ACTION_DOWNLOAD);
    a->source_binding = value;
    a->ninputs = 1;
    a->ndeps = 1;
    b->ins[a->id][0] = view;
    b->deps[a->id][0] = dep;
    rk_publish_desc *p = &b->publish[b->npublish++];
    memset(p, 0, sizeof(*p));
    p->abi_version = RK_ABI_VERSION;
    p->struct_size = sizeof(*p);
    p->binding_id = value;
    p->view_id = view;
    p->dst_row_offset = row;
    p->dst_col_offset = col;
    p->rows = b->views[view].tensor.rows;
    p->cols = b->views[view].tensor.cols;
    return a->id;
}

/* One submit per contiguous run [first, first + n). */
static void pb_submit(pb *b, uint32_t first, uint32_t n) {
    rk_submit_desc *s = &b->submits[b->nsubmits];
    memset(s, 0, sizeof(*s));
    s->abi_version = RK_ABI_VERSION;
    s->struct_size = sizeof(*s);
    s->id = b->nsubmits;
    s->mode = RK_SUBMIT_CHAIN;
    s->ntask_ids = n;
    for (uint32_t i = 0; i < n; i++) b->tasks[b->nsubmits][i] = first + i;
    s->task_ids = b->tasks[b->nsubmits];
    b->nsubmits++;
}

static uint64_t device_claim(const pb *b) {
    uint64_t end[48] = {0}, total = 0;
    uint32_t max_tasks = 0;
    for (uint32_t i = 0; i < b->nbuffers; i++)
        if (b->buffers[i].offset + b->buffers[i].capacity > end[b->buffers[i].slot_id])
            end[b->buffers[i].slot_id] = b->buffers[i].offset + b->buffers[i].capacity;
    for (uint32_t i = 0; i < b->nbuffers; i++)
        if (end[i]) total += end[i] + CO_SLACK + CO_GUARD;
    for (uint32_t s = 0; s < b->nsubmits; s++)
        if (b->submits[s].ntask_ids > max_tasks) max_tasks = b->submits[s].ntask_ids;
    return total + (uint64_t)max_tasks * CO_MAX_WORDS * 8u;
}

static rk_plan_desc pb_desc(pb *b) {
    for (uint32_t i = 0; i < b->nbuffers; i++) b->buffers[i].lifetime_last = b->nactions - 1;
    rk_plan_desc d;
    memset(&d, 0, sizeof(d));
    d.abi_version = RK_ABI_VERSION;
    d.struct_size = sizeof(d);
    d.schema_version = RK_SCHEMA_VERSION;
    d.values = b->values;
    d.nvalues = b->nvalues;
    d.buffers = b->buffers;
    d.nbuffers = b->nbuffers;
    d.views = b->views;
    d.nviews = b->nviews;
    d.actions = b->actions;
    d.nactions = b->nactions;
    d.submits = b->submits;
    d.nsubmits = b->nsubmits;
    d.publish = b->publish;
    d.npublish = b->npublish;
    d.claimed_device_bytes = d.device_budget_bytes = device_claim(b);
    d.claimed_host_bytes = 1u << 24;
    d.host_budget_bytes = 1u << 25;
    d.runtime_abi_version = RK_ABI_VERSION;
    return d;
}

static rk_binding binding(const rk_value_desc *v, const void *data) {
    rk_binding b;
    memset(&b, 0, sizeof(b));
    b.abi_version = RK_ABI_VERSION;
    b.struct_size = sizeof(b);
    b.id = v->id;
    b.dtype = RK_DTYPE_F16;
    b.rank = v->rank;
    b.shape[0] = v->shape[0];
    b.shape[1] = v->shape[1];
    b.data = data;
    b.nbytes = v->nbytes;
    return b;
}

/* The reference test's data pattern (rk_plan_host_test.c:38-40). */
static _Float16 pattern(unsigned i, unsigned seed) { return (_Float16)(((int)((i * 17u + seed) % 31u) - 15) / 64.0); }

static int all_bytes(const void *p, size_t n, unsigned char v) {
    for (size_t i = 0; i < n; i++)
        if (((const unsigned char *)p)[i] != v) return 0;
    return 1;
}

/* ------------------------------------------------------------------------------ multi-tile MM */
/* Y[257, 32] = A[257, 256] * B[256, 32]: A uploaded as a 256-row tile and a 1-row tail, B a cached
 * constant uploaded transposed into the weight layout, one MM per tile in its own submit, both
 * tiles published into the one output (rk_plan_host_test.c:64-377). */
enum { MM = 257, KK = 256, NN = 32 };

static void build_multitile(pb *b) {
    memset(b, 0, sizeof(*b));
    const uint32_t A = pb_value(b, RK_ROLE_INPUT, 2, MM, KK, "A");
    const uint32_t B = pb_value(b, RK_ROLE_CONSTANT, 2, KK, NN, "B");
    const uint32_t Y = pb_value(b, RK_ROLE_OUTPUT, 2, MM, NN, "Y");
    const uint32_t x0 = pb_view(b, RK_LAYOUT_CUBE_F16, 256, KK, RK_ROLE_INPUT_SLICE);
    const uint32_t x1 = pb_view(b, RK_LAYOUT_CUBE_F16, 1, KK, RK_ROLE_INPUT_SLICE);
    const uint32_t w = pb_view(b, RK_LAYOUT_WEIGHT_F16, NN, KK, RK_ROLE_WEIGHT);
    const uint32_t y0 = pb_view(b, RK_LAYOUT_CUBE_F16, 256, NN, RK_ROLE_OUTPUT);
    const uint32_t y1 = pb_view(b, RK_LAYOUT_CUBE_F16, 1, NN, RK_ROLE_OUTPUT);
    const uint32_t u0 = pb_upload(b, A, x0, 0, 0, 0);
    const uint32_t u1 = pb_upload(b, A, x1, 256, 0, 0);
    const uint32_t uw = pb_upload(b, B, w, 0, 0, RK_ACTION_FLAG_TRANSPOSE_SOURCE | RK_ACTION_FLAG_CACHE_CONSTANT);
    const uint32_t d0[] = {u0, uw}, d1[] = {u1, uw};
    const uint32_t t0 = pb_task(b, RK_TEMPLATE_MM_F16, (uint32_t[]){x0, w}, 2, y0, d0, 2);
    const uint32_t t1 = pb_task(b, RK_TEMPLATE_MM_F16, (uint32_t[]){x1, w}, 2, y1, d1, 2);
    pb_download(b, Y, y0, t0, 0, 0);
    pb_download(b, Y, y1, t1, 256, 0);
    pb_submit(b, t0, 1);
    pb_submit(b, t1, 1);
}

static void multitile_case(int fd) {
    pb b;
    build_multitile(&b);
    rk_plan_desc desc = pb_desc(&b);
    rk_diag diag;
    rk_plan *plan = NULL;
    EXPECT(rk_plan_create(&desc, &plan, &diag) == 0 && plan);
    if (!plan) {
        fprintf(stderr, "  create: %s\n", diag.message);
        return;
    }
    /* the tiles may not cover each other */
    rk_publish_desc overlap[2] = {b.publish[0], b.publish[1]};
    overlap[1].dst_row_offset = 255;
    rk_plan_desc bad = desc;
    bad.publish = overlap;
    rk_plan *badplan = (rk_plan *)1;
    EXPECT(rk_plan_create(&bad, &badplan, &diag) != 0 && badplan == NULL);
    /* without the tail tile the binding is not covered */
    bad = desc;
    bad.npublish = 1;
    EXPECT_CODE(rk_plan_create(&bad, &badplan, &diag), RK_E_SHAPE, "cover the output binding");
    /* the two output tiles are live at the same time: they cannot share a slot */
    rk_buffer_desc shared[64];
    memcpy(shared, b.buffers, sizeof(shared));
    shared[4].slot_id = shared[3].slot_id;
    bad = desc;
    bad.buffers = shared;
    EXPECT_CODE(rk_plan_create(&bad, &badplan, &diag), RK_E_ALIAS, "overlapping live ranges");

    _Float16 *x = malloc((size_t)MM * KK * 2), *w = malloc((size_t)KK * NN * 2);
    _Float16 *y = malloc((size_t)MM * NN * 2), *ref = malloc((size_t)MM * NN * 2);
    for (size_t i = 0; i < (size_t)MM * KK; i++) x[i] = pattern((unsigned)i, 5);
    for (size_t i = 0; i < (size_t)KK * NN; i++) w[i] = pattern((unsigned)i, 13);
    for (unsigned r = 0; r < MM; r++)
        for (unsigned c = 0; c < NN; c++) {
            double s = 0;
            for (unsigned q = 0; q < KK; q++) s += (double)x[(size_t)r * KK + q] * (double)w[(size_t)q * NN + c];
            ref[(size_t)r * NN + c] = (_Float16)s;
        }
    rk_binding constants[] = {binding(&b.values[1], w)};
    rk_workspace *ws = NULL;
    EXPECT(rk_workspace_create(fd, plan, constants, 1, &ws, &diag) == 0 && ws);
    if (!ws) {
        fprintf(stderr, "  workspace: %s\n", diag.message);
        return;
    }
    rk_binding inputs[] = {binding(&b.values[0], x)};
    rk_binding outputs[] = {binding(&b.values[2], y)};
    rk_run_report report;
    memset(y, 0x23, (size_t)MM * NN * 2);
    EXPECT(rk_workspace_run(ws, inputs, 1, outputs, 1, &report, &diag) == 0);
    EXPECT(report.task_count == 2 && report.submit_count == 2 && report.download_calls == 2);
    EXPECT(report.upload_calls == 2 && report.fail_action_id == UINT32_MAX);
    EXPECT(!memcmp(y, ref, (size_t)MM * NN * 2));

    /* input finiteness is rechecked on every call; nothing is published */
    const _Float16 nonfinite[] = {(_Float16)NAN, (_Float16)INFINITY, (_Float16)-INFINITY};
    for (int k = 0; k < 3; k++) {
        memset(y, 0x23, (size_t)MM * NN * 2);
        x[(size_t)k * 977] = nonfinite[k];
        EXPECT_CODE(rk_workspace_run(ws, inputs, 1, outputs, 1, &report, &diag), RK_E_NUMERIC_CONTRACT,
                    "non-finite FP16 input");
        EXPECT(all_bytes(y, (size_t)MM * NN * 2, 0x23));
        x[(size_t)k * 977] = pattern((unsigned)k * 977, 5);
    }
    /* a result that overflows FP16 is never published: the download names its action */
    {
        _Float16 keep = x[(size_t)256 * KK];
        for (unsigned q = 0; q < KK; q++) x[(size_t)256 * KK + q] = (_Float16)(w[(size_t)q * NN] >= 0 ? 60000.0 : -60000.0);
        memset(y, 0x23, (size_t)MM * NN * 2);
        EXPECT_CODE(rk_workspace_run(ws, inputs, 1, outputs, 1, &report, &diag), RK_E_NUMERIC_CONTRACT,
                    "not finite; refusing to publish");
        EXPECT(report.fail_action_id == 6 && diag.action_id == 6 && diag.has_action);
        EXPECT(all_bytes(y, (size_t)MM * NN * 2, 0x23));
        for (unsigned q = 0; q < KK; q++) x[(size_t)256 * KK + q] = pattern(256u * KK + q, 5);
        (void)keep;
    }
#ifdef RK_TEST_MOCK
    mock_rk_inject = 1;
    memset(y, 0x23, (size_t)MM * NN * 2);
    EXPECT_CODE(rk_workspace_run(ws, inputs, 1, outputs, 1, &report, &diag), RK_E_NUMERIC_CONTRACT, NULL);
    EXPECT(all_bytes(y, (size_t)MM * NN * 2, 0x23));
    mock_rk_inject = 0;
#endif
    memset(y, 0x23, (size_t)MM * NN * 2);
    EXPECT(rk_workspace_run(ws, inputs, 1, outputs, 1, &report, &diag) == 0);
    EXPECT(!memcmp(y, ref, (size_t)MM * NN * 2));

    /* latency of one synchronous run (host copies in, the device schedule, the copy out, the
     * checks and the publish), printed for the record */
    {
#ifdef RK_TEST_MOCK
        enum { RUNS = 3 };
#else
        enum { RUNS = 200 };
#endif
        struct timespec t0, t1;
        double wait = 0;
        clock_gettime(CLOCK_MONOTONIC, &t0);
        for (int i = 0; i < RUNS; i++) {
            EXPECT(rk_workspace_run(ws, inputs, 1, outputs, 1, &report, &diag) == 0);
            wait += report.submit_wait_us;
        }
        clock_gettime(CLOCK_MONOTONIC, &t1);
        const double us = ((double)(t1.tv_sec - t0.tv_sec) * 1e6 + (double)(t1.tv_nsec - t0.tv_nsec) / 1e3) / RUNS;
        printf("rk_plan multitile [257x256]x[256x32]: %.1f us per run, %.1f us device schedule + copy out\n", us,
               wait / RUNS);
    }
    /* binding checks */
    rk_binding wrong = outputs[0];
    wrong.shape[0] = 256;
    EXPECT_CODE(rk_workspace_run(ws, inputs, 1, &wrong, 1, &report, &diag), RK_E_SHAPE, "binding");
    EXPECT_CODE(rk_workspace_run(ws, inputs, 0, outputs, 1, &report, &diag), RK_E_SHAPE, "count mismatch");
    rk_binding aliased = outputs[0];
    aliased.data = x;
    EXPECT_CODE(rk_workspace_run(ws, inputs, 1, &aliased, 1, &report, &diag), RK_E_ALIAS, "overlap");

    /* run_ex: the envelope's size is checked before anything is written */
    rk_run_attribution env;
    memset(&env, 0x5c, sizeof(env));
    env.struct_size = 8;
    EXPECT_CODE(rk_workspace_run_ex(ws, inputs, 1, outputs, 1, &env, &diag), RK_E_SCHEMA, NULL);
    memset(&env, 0x5c, sizeof(env));
    env.struct_size = RK_RUN_ATTRIBUTION_V1_SIZE;
    memset(y, 0x23, (size_t)MM * NN * 2);
    EXPECT(rk_workspace_run_ex(ws, inputs, 1, outputs, 1, &env, &diag) == 0);
    EXPECT(env.task_count == 2 && env.download_calls == 2 && env.total_us > 0);
    EXPECT(all_bytes((const char *)&env + RK_RUN_ATTRIBUTION_V1_SIZE, sizeof(env) - RK_RUN_ATTRIBUTION_V1_SIZE, 0x5c));
    EXPECT(!memcmp(y, ref, (size_t)MM * NN * 2));

    /* run_group: three repeats; a failing repeat publishes nothing for any repeat */
    {
        _Float16 *xs[3], *ys[3], *refs[3];
        rk_binding set[6];
        for (int r = 0; r < 3; r++) {
            xs[r] = malloc((size_t)MM * KK * 2);
            ys[r] = malloc((size_t)MM * NN * 2);
            refs[r] = malloc((size_t)MM * NN * 2);
            for (size_t i = 0; i < (size_t)MM * KK; i++) xs[r][i] = pattern((unsigned)i, 7 + 3 * r);
            set[2 * r] = binding(&b.values[0], xs[r]);
            set[2 * r + 1] = binding(&b.values[2], ys[r]);
            rk_binding one_in = set[2 * r], one_out = binding(&b.values[2], refs[r]);
            EXPECT(rk_workspace_run(ws, &one_in, 1, &one_out, 1, &report, &diag) == 0);
            memset(ys[r], 0x23, (size_t)MM * NN * 2);
        }
        rk_group_report g;
        memset(&g, 0, sizeof(g));
        g.struct_size = RK_GROUP_REPORT_V1_SIZE;
        EXPECT(rk_workspace_run_group(ws, set, 3, &g, &diag) == 0);
        EXPECT(g.repeat_completed == 3 && g.task_count == 6 && g.download_calls == 6 && g.fail_repeat == UINT32_MAX);
        for (int r = 0; r < 3; r++) EXPECT(!memcmp(ys[r], refs[r], (size_t)MM * NN * 2));
        for (int r = 0; r < 3; r++) memset(ys[r], 0x23, (size_t)MM * NN * 2);
        for (unsigned q = 0; q < KK; q++) xs[2][(size_t)7 * KK + q] = (_Float16)(w[(size_t)q * NN] >= 0 ? 60000.0 : -60000.0);
        EXPECT_CODE(rk_workspace_run_group(ws, set, 3, &g, &diag), RK_E_NUMERIC_CONTRACT, NULL);
        EXPECT(g.fail_repeat == 2 && g.repeat_completed == 2);
        for (int r = 0; r < 3; r++) EXPECT(all_bytes(ys[r], (size_t)MM * NN * 2, 0x23));
        g.struct_size = 4;
        EXPECT_CODE(rk_workspace_run_group(ws, set, 3, &g, &diag), RK_E_SCHEMA, NULL);
        for (int r = 0; r < 3; r++) {
            free(xs[r]);
            free(ys[r]);
            free(refs[r]);
        }
    }
#ifdef RK_TEST_MOCK
    /* an overwritten slack byte fails the publication gate and poisons the workspace */
    mock_rk_inject = 2;
    memset(y, 0x23, (size_t)MM * NN * 2);
    EXPECT_CODE(rk_workspace_run(ws, inputs, 1, outputs, 1, &report, &diag), RK_E_DEVICE, "guard");
    EXPECT(all_bytes(y, (size_t)MM * NN * 2, 0x23));
    mock_rk_inject = 0;
    EXPECT_CODE(rk_workspace_run(ws, inputs, 1, outputs, 1, &report, &diag), RK_E_POISONED, NULL);
#endif
    EXPECT(rk_workspace_destroy(ws, &diag) == 0);
    rk_plan_destroy(plan);
    free(x); free(w); free(y); free(ref);
}

/* ------------------------------------------------------------------------------ K accumulation */
/* Y[40, 48] = X[40, 300] * W[48, 300]^T in two K tiles (256 + a ragged 44): MM into a partial,
 * MM_ACC adds the second tile's sum to it (fp16(sum1 + fp16(sum0))). */
static void kacc_case(int fd) {
    enum { M = 40, K = 300, N = 48 };
    pb b;
    memset(&b, 0, sizeof(b));
    const uint32_t X = pb_value(&b, RK_ROLE_INPUT, 2, M, K, "X");
    const uint32_t W = pb_value(&b, RK_ROLE_CONSTANT, 2, N, K, "W");
    const uint32_t Y = pb_value(&b, RK_ROLE_OUTPUT, 2, M, N, "Y");
    const uint32_t x0 = pb_view(&b, RK_LAYOUT_CUBE_F16, M, 256, RK_ROLE_INPUT_SLICE);
    const uint32_t x1 = pb_view(&b, RK_LAYOUT_CUBE_F16, M, K - 256, RK_ROLE_INPUT_SLICE);
    const uint32_t w0 = pb_view(&b, RK_LAYOUT_WEIGHT_F16, N, 256, RK_ROLE_WEIGHT);
    const uint32_t w1 = pb_view(&b, RK_LAYOUT_WEIGHT_F16, N, K - 256, RK_ROLE_WEIGHT);
    const uint32_t ya = pb_view(&b, RK_LAYOUT_CUBE_F16, M, N, RK_ROLE_ACCUMULATOR);
    const uint32_t yb = pb_view(&b, RK_LAYOUT_CUBE_F16, M, N, RK_ROLE_OUTPUT);
    const uint32_t ux0 = pb_upload(&b, X, x0, 0, 0, 0), ux1 = pb_upload(&b, X, x1, 0, 256, 0);
    const uint32_t uw0 = pb_upload(&b, W, w0, 0, 0, RK_ACTION_FLAG_CACHE_CONSTANT);
    const uint32_t uw1 = pb_upload(&b, W, w1, 0, 256, RK_ACTION_FLAG_CACHE_CONSTANT);
    const uint32_t t0 = pb_task(&b, RK_TEMPLATE_MM_F16, (uint32_t[]){x0, w0}, 2, ya, (uint32_t[]){ux0, uw0}, 2);
    const uint32_t t1 = pb_task(&b, RK_TEMPLATE_MM_ACC_F16, (uint32_t[]){x1, w1, ya}, 3, yb,
                                (uint32_t[]){ux1, uw1, t0}, 3);
    b.actions[t0].source_k_count = b.actions[t1].source_k_count = 2;
    b.actions[t1].source_k_index = 1;
    pb_download(&b, Y, yb, t1, 0, 0);
    pb_submit(&b, t0, 2);
    rk_plan_desc desc = pb_desc(&b);
    rk_diag diag;
    rk_plan *plan = NULL;
    EXPECT(rk_plan_create(&desc, &plan, &diag) == 0);
    if (!plan) {
        fprintf(stderr, "  kacc create: %s\n", diag.message);
        return;
    }
    /* the accumulator's prior and output may not share a slot */
    rk_buffer_desc shared[64];
    memcpy(shared, b.buffers, sizeof(shared));
    shared[5].slot_id = shared[4].slot_id;
    rk_plan_desc bad = desc;
    bad.buffers = shared;
    rk_plan *badplan = NULL;
    EXPECT_CODE(rk_plan_create(&bad, &badplan, &diag), RK_E_ALIAS, "share a BO");

    _Float16 x[M * K], w[N * K], y[M * N], ref[M * N];
    for (int i = 0; i < M * K; i++) x[i] = (_Float16)((double)pattern((unsigned)i, 3) * 4.0);
    for (int i = 0; i < N * K; i++) w[i] = pattern((unsigned)i, 11);
    for (int r = 0; r < M; r++)
        for (int c = 0; c < N; c++) {
            double s0 = 0, s1 = 0;
            for (int q = 0; q < 256; q++) s0 += (double)x[r * K + q] * (double)w[c * K + q];
            for (int q = 256; q < K; q++) s1 += (double)x[r * K + q] * (double)w[c * K + q];
            ref[r * N + c] = (_Float16)(s1 + (double)(_Float16)s0);
        }
    rk_binding constants[] = {binding(&b.values[W], w)};
    rk_workspace *ws = NULL;
    EXPECT(rk_workspace_create(fd, plan, constants, 1, &ws, &diag) == 0);
    if (ws) {
        rk_binding in[] = {binding(&b.values[X], x)}, out[] = {binding(&b.values[Y], y)};
        rk_run_report report;
        memset(y, 0x23, sizeof(y));
        EXPECT(rk_workspace_run(ws, in, 1, out, 1, &report, &diag) == 0);
        EXPECT(!memcmp(y, ref, sizeof(y)));
        EXPECT(report.task_count == 2 && report.submit_count == 1 && report.upload_calls == 2);
        EXPECT(rk_workspace_destroy(ws, &diag) == 0);
    }
    rk_plan_destroy(plan);
}

/* The same K accumulation with the MM partial also downloaded after the MM_ACC: the partial is
 * read after its chain reader, so the two tasks must run separately and both outputs hold their
 * own results (a chain would leave the partial unwritten; the CPU seam writes only a chain's final
 * tile, like the device). */
static void kacc_observed_case(int fd) {
    enum { M = 40, K = 300, N = 48 };
    static pb b;
    memset(&b, 0, sizeof(b));
    const uint32_t X = pb_value(&b, RK_ROLE_INPUT, 2, M, K, "X");
    const uint32_t W = pb_value(&b, RK_ROLE_CONSTANT, 2, N, K, "W");
    const uint32_t Y = pb_value(&b, RK_ROLE_OUTPUT, 2, M, N, "Y");
    const uint32_t P = pb_value(&b, RK_ROLE_OUTPUT, 2, M, N, "P");
    const uint32_t x0 = pb_view(&b, RK_LAYOUT_CUBE_F16, M, 256, RK_ROLE_INPUT_SLICE);
    const uint32_t x1 = pb_view(&b, RK_LAYOUT_CUBE_F16, M, K - 256, RK_ROLE_INPUT_SLICE);
    const uint32_t w0 = pb_view(&b, RK_LAYOUT_WEIGHT_F16, N, 256, RK_ROLE_WEIGHT);
    const uint32_t w1 = pb_view(&b, RK_LAYOUT_WEIGHT_F16, N, K - 256, RK_ROLE_WEIGHT);
    const uint32_t ya = pb_view(&b, RK_LAYOUT_CUBE_F16, M, N, RK_ROLE_ACCUMULATOR);
    const uint32_t yb = pb_view(&b, RK_LAYOUT_CUBE_F16, M, N, RK_ROLE_OUTPUT);
    const uint32_t ux0 = pb_upload(&b, X, x0, 0, 0, 0), ux1 = pb_upload(&b, X, x1, 0, 256, 0);
    const uint32_t uw0 = pb_upload(&b, W, w0, 0, 0, RK_ACTION_FLAG_CACHE_CONSTANT);
    const uint32_t uw1 = pb_upload(&b, W, w1, 0, 256, RK_ACTION_FLAG_CACHE_CONSTANT);
    const uint32_t t0 = pb_task(&b, RK_TEMPLATE_MM_F16, (uint32_t[]){x0, w0}, 2, ya, (uint32_t[]){ux0, uw0}, 2);
    const uint32_t t1 = pb_task(&b, RK_TEMPLATE_MM_ACC_F16, (uint32_t[]){x1, w1, ya}, 3, yb,
                                (uint32_t[]){ux1, uw1, t0}, 3);
    b.actions[t0].source_k_count = b.actions[t1].source_k_count = 2;
    b.actions[t1].source_k_index = 1;
    pb_download(&b, Y, yb, t1, 0, 0);
    pb_download(&b, P, ya, t1, 0, 0);
    pb_submit(&b, t0, 2);
    rk_plan_desc desc = pb_desc(&b);
    rk_diag diag;
    rk_plan *plan = NULL;
    EXPECT(rk_plan_create(&desc, &plan, &diag) == 0);
    if (!plan) {
        fprintf(stderr, "  kacc observed create: %s\n", diag.message);
        return;
    }
    static _Float16 x[M * K], w[N * K], y[M * N], part[M * N], ref[M * N], pref[M * N];
    for (int i = 0; i < M * K; i++) x[i] = (_Float16)((double)pattern((unsigned)i, 5) * 4.0);
    for (int i = 0; i < N * K; i++) w[i] = pattern((unsigned)i, 13);
    for (int r = 0; r < M; r++)
        for (int c = 0; c < N; c++) {
            double s0 = 0, s1 = 0;
            for (int q = 0; q < 256; q++) s0 += (double)x[r * K + q] * (double)w[c * K + q];
            for (int q = 256; q < K; q++) s1 += (double)x[r * K + q] * (double)w[c * K + q];
            pref[r * N + c] = (_Float16)s0;
            ref[r * N + c] = (_Float16)(s1 + (double)(_Float16)s0);
        }
    rk_binding constants[] = {binding(&b.values[W], w)};
    rk_workspace *ws = NULL;
    EXPECT(rk_workspace_create(fd, plan, constants, 1, &ws, &diag) == 0);
    if (ws) {
        rk_binding in[] = {binding(&b.values[X], x)};
        rk_binding out[] = {binding(&b.values[Y], y), binding(&b.values[P], part)};
        rk_run_report report;
        memset(y, 0x23, sizeof(y));
        memset(part, 0x23, sizeof(part));
        EXPECT(rk_workspace_run(ws, in, 1, out, 2, &report, &diag) == 0);
        EXPECT(!memcmp(y, ref, sizeof(y)));
        EXPECT(!memcmp(part, pref, sizeof(part)));
        EXPECT(rk_workspace_destroy(ws, &diag) == 0);
    }
    rk_plan_destroy(plan);
}

/* ------------------------------------------------------------------------------ EW, LUT, broadcast */
enum { EM = 20, EN = 72, EP = 96, ETILES = 10 };

static double lut_ref(int tpl, double v) {
    switch (tpl) {
    case RK_TEMPLATE_LUT_SIGMOID_F16: return 1.0 / (1.0 + exp(-v));
    case RK_TEMPLATE_LUT_HARDSIGMOID_F16: return fmin(1.0, fmax(0.0, v / 6.0 + 0.5));
    case RK_TEMPLATE_LUT_GELU_GATE_F16: return 0.5 * (1.0 + erf(v / sqrt(2.0)));
    default: return 1.0 / sqrt(fmax(0.125, v));
    }
}

typedef struct {
    pb b;
    uint32_t A, B, ID, BIAS, SCALE, Y;
    uint32_t uploadB;
} ew_plan;

static void build_ew(ew_plan *e) {
    pb *b = &e->b;
    memset(e, 0, sizeof(*e));
    e->A = pb_value(b, RK_ROLE_INPUT, 2, EM, EN, "A");
    e->B = pb_value(b, RK_ROLE_INPUT, 2, EM, EN, "B");
    e->ID = pb_value(b, RK_ROLE_CONSTANT, 2, EP, EP, "I");
    e->BIAS = pb_value(b, RK_ROLE_CONSTANT, 1, EN, 0, "bias");
    e->SCALE = pb_value(b, RK_ROLE_CONSTANT, 0, 0, 0, "scale");
    e->Y = pb_value(b, RK_ROLE_OUTPUT, 2, EM, EN * ETILES, "Y");
    const uint32_t va = pb_view(b, RK_LAYOUT_CUBE_F16, EM, EN, RK_ROLE_INPUT_SLICE);
    const uint32_t vb = pb_view(b, RK_LAYOUT_CUBE_F16, EM, EN, RK_ROLE_INPUT_SLICE);
    const uint32_t vi = pb_view(b, RK_LAYOUT_WEIGHT_F16, EP, EP, RK_ROLE_IDENTITY);
    const uint32_t vbias = pb_view(b, RK_LAYOUT_CUBE_F16, EM, EN, RK_ROLE_CONSTANT);
    const uint32_t vscale = pb_view(b, RK_LAYOUT_CUBE_F16, EM, EN, RK_ROLE_CONSTANT);
    uint32_t out[ETILES];
    for (int i = 0; i < ETILES; i++) out[i] = pb_view(b, RK_LAYOUT_CUBE_F16, EM, EN, RK_ROLE_SCRATCH);
    const uint32_t ua = pb_upload(b, e->A, va, 0, 0, 0);
    e->uploadB = pb_upload(b, e->B, vb, 0, 0, 0);
    const uint32_t ui = pb_upload(b, e->ID, vi, 0, 0, RK_ACTION_FLAG_CACHE_CONSTANT);
    const uint32_t ubias = pb_upload(b, e->BIAS, vbias, 0, 0, RK_ACTION_FLAG_BROADCAST_CHANNEL);
    const uint32_t uscale = pb_upload(b, e->SCALE, vscale, 0, 0, RK_ACTION_FLAG_BROADCAST_SCALAR);
    const uint32_t ew[4] = {RK_TEMPLATE_EW_ADD_F16, RK_TEMPLATE_EW_MUL_F16, RK_TEMPLATE_EW_MAX_F16,
                            RK_TEMPLATE_EW_ADD_RELU_F16};
    uint32_t task[ETILES];
    for (int i = 0; i < 4; i++)
        task[i] = pb_task(b, ew[i], (uint32_t[]){va, vb, vi}, 3, out[i], (uint32_t[]){ua, e->uploadB, ui}, 3);
    task[4] = pb_task(b, RK_TEMPLATE_EW_ADD_F16, (uint32_t[]){va, vbias, vi}, 3, out[4], (uint32_t[]){ua, ubias, ui}, 3);
    task[5] = pb_task(b, RK_TEMPLATE_EW_MUL_F16, (uint32_t[]){va, vscale, vi}, 3, out[5], (uint32_t[]){ua, uscale, ui}, 3);
    const uint32_t lut[4] = {RK_TEMPLATE_LUT_SIGMOID_F16, RK_TEMPLATE_LUT_HARDSIGMOID_F16,
                             RK_TEMPLATE_LUT_GELU_GATE_F16, RK_TEMPLATE_LUT_RSQRT_F16};
    for (int i = 0; i < 4; i++)
        task[6 + i] = pb_task(b, lut[i], (uint32_t[]){out[0]}, 1, out[6 + i], (uint32_t[]){task[0]}, 1);
    for (int i = 0; i < ETILES; i++) pb_submit(b, task[i], 1);
    for (int i = 0; i < ETILES; i++) pb_download(b, e->Y, out[i], task[i], 0, (uint32_t)(EN * i));
}

/* Expected Y for A, B (row-major [EM][EN]), bias [EN], scale. */
static void ew_expect(const _Float16 *a, const _Float16 *bv, const _Float16 *bias, _Float16 scale, _Float16 *y) {
    for (int r = 0; r < EM; r++)
        for (int c = 0; c < EN; c++) {
            const double x = a[r * EN + c], o = bv[r * EN + c];
            _Float16 t[ETILES];
            t[0] = (_Float16)(x + o);
            t[1] = (_Float16)(x * o);
            t[2] = (_Float16)fmax(x, o);
            t[3] = (_Float16)fmax(x + o, 0.0);
            t[4] = (_Float16)(x + (double)bias[c]);
            t[5] = (_Float16)(x * (double)scale);
            for (int i = 0; i < 4; i++) t[6 + i] = (_Float16)lut_ref((int)RK_TEMPLATE_LUT_SIGMOID_F16 + (i == 3 ? 5 : i),
                                                                     (double)t[0]);
            for (int i = 0; i < ETILES; i++) y[(size_t)r * EN * ETILES + (size_t)EN * i + c] = t[i];
        }
}

static void ew_case(int fd) {
    ew_plan e;
    build_ew(&e);
    rk_plan_desc desc = pb_desc(&e.b);
    rk_diag diag;
    rk_plan *plan = NULL;
    EXPECT(rk_plan_create(&desc, &plan, &diag) == 0);
    if (!plan) {
        fprintf(stderr, "  ew create: %s\n", diag.message);
        return;
    }
    static _Float16 a[EM * EN], bv[EM * EN], zero[EM * EN], id[EP * EP], bias[EN], y[EM * EN * ETILES],
        ref[EM * EN * ETILES], bt[EN * EM];
    const _Float16 scale = (_Float16)-1.375;
    for (int i = 0; i < EM * EN; i++) {
        a[i] = (_Float16)((double)pattern((unsigned)i, 2) * 12.0);
        bv[i] = (_Float16)((double)pattern((unsigned)i, 19) * 5.0);
    }
    for (int r = 0; r < EM; r++)
        for (int c = 0; c < EN; c++) bt[c * EM + r] = bv[r * EN + c];
    for (int i = 0; i < EP * EP; i++) id[i] = (_Float16)(i / EP == i % EP ? 1.0 : 0.0);
    for (int c = 0; c < EN; c++) bias[c] = (_Float16)(c * 0.125 - 4.0);
    rk_binding constants[] = {binding(&e.b.values[e.ID], id), binding(&e.b.values[e.BIAS], bias),
                              binding(&e.b.values[e.SCALE], &scale)};
    rk_workspace *ws = NULL;
    EXPECT(rk_workspace_create(fd, plan, constants, 3, &ws, &diag) == 0);
    if (!ws) {
        fprintf(stderr, "  ew workspace: %s\n", diag.message);
        rk_plan_destroy(plan);
        return;
    }
    rk_binding in[] = {binding(&e.b.values[e.A], a), binding(&e.b.values[e.B], bv)};
    rk_binding out[] = {binding(&e.b.values[e.Y], y)};
    rk_run_report report;
    ew_expect(a, bv, bias, scale, ref);
    EXPECT(rk_workspace_run(ws, in, 2, out, 1, &report, &diag) == 0);
    EXPECT(!memcmp(y, ref, sizeof(y)));
    for (int t = 0; t < ETILES; t++) {
        int bad = 0;
        for (int r = 0; r < EM && !bad; r++)
            for (int c = 0; c < EN && !bad; c++) {
                const size_t i = (size_t)r * EN * ETILES + (size_t)EN * t + c;
                if (memcmp(&y[i], &ref[i], 2)) {
                    bad = 1;
                    fprintf(stderr, "  ew tile %d (%d,%d): got %.8g want %.8g\n", t, r, c, (double)y[i], (double)ref[i]);
                }
            }
    }
    EXPECT(report.task_count == ETILES && report.upload_calls == 2 && report.download_calls == ETILES);

    /* persistent upload of B: runs no longer pack it; the caller fills and clears it */
    EXPECT(rk_workspace_set_persistent_upload(ws, e.uploadB, &diag) == 0);
    EXPECT_CODE(rk_workspace_set_persistent_upload(ws, 7 + ETILES, &diag), RK_E_SCHEMA, "single-output upload");
    EXPECT(rk_workspace_clear_upload_destination(ws, e.uploadB, &diag) == 0);
    EXPECT(rk_workspace_run(ws, in, 2, out, 1, &report, &diag) == 0);
    EXPECT(report.upload_calls == 1);
    ew_expect(a, zero, bias, scale, ref);
    EXPECT(!memcmp(y, ref, sizeof(y)));
    rk_state_source src = {bt, sizeof(bt), EM, RK_STATE_SOURCE_TRANSPOSE};
    EXPECT(rk_workspace_update_upload_region(ws, e.uploadB, &src, 0, 0, 0, 0, EM, EN, &diag) == 0);
    EXPECT(rk_workspace_run(ws, in, 2, out, 1, &report, &diag) == 0);
    ew_expect(a, bv, bias, scale, ref);
    EXPECT(!memcmp(y, ref, sizeof(y)));
    /* a partial region over a cleared destination */
    static _Float16 part[EM * EN];
    for (int r = 0; r < EM; r++)
        for (int c = 0; c < EN; c++) part[r * EN + c] = (r >= 5 && r < 10 && c >= 8 && c < 40) ? bv[r * EN + c] : 0;
    EXPECT(rk_workspace_clear_upload_destination(ws, e.uploadB, &diag) == 0);
    rk_state_source rowmajor = {bv, sizeof(bv), EN, 0};
    EXPECT(rk_workspace_update_upload_region(ws, e.uploadB, &rowmajor, 5, 8, 5, 8, 5, 32, &diag) == 0);
    EXPECT(rk_workspace_run(ws, in, 2, out, 1, &report, &diag) == 0);
    ew_expect(a, part, bias, scale, ref);
    EXPECT(!memcmp(y, ref, sizeof(y)));
    EXPECT_CODE(rk_workspace_update_upload_region(ws, e.uploadB, &rowmajor, 0, 0, 16, 0, 5, 8, &diag), RK_E_SHAPE,
                "outside the destination");
    EXPECT_CODE(rk_workspace_update_upload_region(ws, e.uploadB, &rowmajor, 19, 70, 0, 0, 1, 3, &diag), RK_E_SHAPE,
                "exceeds the supplied buffer");
    EXPECT_CODE(rk_workspace_update_upload_region(ws, 0, &rowmajor, 0, 0, 0, 0, 1, 1, &diag), RK_E_SCHEMA,
                "persistent upload");
    EXPECT(rk_workspace_destroy(ws, &diag) == 0);

    /* workspace creation: constants are counted, shaped and finite */
    EXPECT_CODE(rk_workspace_create(fd, plan, constants, 2, &ws, &diag), RK_E_SHAPE, "constant binding count");
    _Float16 badbias[EN];
    memcpy(badbias, bias, sizeof(bias));
    badbias[EN - 1] = (_Float16)INFINITY;
    rk_binding badconst[] = {constants[0], binding(&e.b.values[e.BIAS], badbias), constants[2]};
    EXPECT_CODE(rk_workspace_create(fd, plan, badconst, 3, &ws, &diag), RK_E_NUMERIC_CONTRACT, "non-finite");
    EXPECT(ws == NULL);
    /* every failing allocation of workspace creation is reported and leaks nothing */
#ifdef RK_TEST_MOCK
    const size_t live = b2h_live_bytes();
#endif
    for (unsigned nth = 1; nth <= 12; nth++) {
        b2_fault_inject(B2_FAULT_ALLOC, nth);
        ws = NULL;
        const int rc = rk_workspace_create(fd, plan, constants, 3, &ws, &diag);
        b2_fault_inject(B2_FAULT_NONE, 1);
        if (rc == 0) {
            EXPECT(ws != NULL);
            EXPECT(rk_workspace_destroy(ws, &diag) == 0);
            break;
        }
        EXPECT(ws == NULL && (rc == RK_E_NOMEM || rc == RK_E_DEVICE));
#ifdef RK_TEST_MOCK
        EXPECT(b2h_live_bytes() == live);
#endif
    }
    rk_plan_destroy(plan);
}

/* ------------------------------------------------------------------------------ rejections */
typedef struct {
    const char *what;
    int code;
    const char *needle;
} reject_case;

/* Applies mutation i to a fresh multi-tile plan; returns its expectation. */
static reject_case mutate(int i, pb *b, rk_plan_desc *d) {
    build_multitile(b);
    switch (i) {
    case 0: *d = pb_desc(b); d->abi_version = 0; return (reject_case){"abi", RK_E_SCHEMA, "ABI/size"};
    case 1: *d = pb_desc(b); d->schema_version = 1; return (reject_case){"schema", RK_E_SCHEMA, "schema version"};
    case 2: *d = pb_desc(b); d->runtime_abi_version = 2; return (reject_case){"runtime abi", RK_E_SCHEMA, "runtime_abi"};
    case 3: b->values[1].id = 0; break;
    case 4: b->values[1].name = "A"; b->values[1].name_len = 1; break;
    case 5: b->buffers[0].alignment = 24; break;
    case 6: b->views[0].offset_bytes = 8; break;
    case 7: b->views[0].tensor.physical_rows = 260; break;
    case 8: b->actions[0].source_row_stride = 128; break;
    case 9: b->actions[1].source_row_offset = 257; break;
    case 10: b->actions[5].source_binding = 0; break;
    case 11: b->ins[3][1] = 0; break;
    case 12: b->actions[3].ndeps = 1; break;
    case 13: b->deps[3][0] = 3; break;
    case 14: b->tasks[0][0] = 0; break;
    case 15: b->tasks[1][0] = 3; break;
    case 16: b->nsubmits = 1; break;
    case 17: *d = pb_desc(b); d->claimed_device_bytes = 0; return (reject_case){"no device claim", RK_E_BUDGET, "claimed_device_bytes"};
    case 18: *d = pb_desc(b); d->claimed_device_bytes -= 1; d->device_budget_bytes = 0; return (reject_case){"device claim", RK_E_BUDGET, "understate"};
    case 19: *d = pb_desc(b); d->claimed_host_bytes = 1000; return (reject_case){"host claim", RK_E_BUDGET, "host bytes understate"};
    case 20: b->actions[0].kind = RK_ACTION_HOST_COMPUTE; break;
    case 21: memset(b->actions[2].origin, 'x', sizeof(b->actions[2].origin)); break;
    case 22: b->views[3].valid_region[1] = 255; break;
    case 23: b->outs[3][0] = 4; break;
    case 24: b->actions[3].flags = RK_ACTION_FLAG_DATA_REUSE; break;
    case 25: b->views[2].tensor.physical_rows = 64; break;
    default: return (reject_case){NULL, 0, NULL};
    }
    *d = pb_desc(b);
    static const reject_case expect[] = {
        {0}, {0}, {0},
        {"value id", RK_E_SCHEMA, "value id"},
        {"duplicate name", RK_E_SCHEMA, "duplicate value name"},
        {"alignment", RK_E_SHAPE, "alignment"},
        {"view offset", RK_E_SHAPE, "view exceeds buffer capacity"},
        {"tensor geometry", RK_E_SHAPE, "view id/tensor invalid"},
        {"row stride", RK_E_SHAPE, "source_row_stride"},
        {"source window", RK_E_SHAPE, "source region exceeds"},
        {"download target", RK_E_SHAPE, "download target binding must be output"},
        {"mm operand layout", RK_E_SHAPE, "mm layout mismatch"},
        {"missing dependency", RK_E_SCHEMA, "not a declared dependency"},
        {"self dependency", RK_E_SCHEMA, "not topological"},
        {"upload in a submit", RK_E_SCHEMA, "non-NPU"},
        {"task in two submits", RK_E_SCHEMA, "multiple submits"},
        {"unassigned task", RK_E_SCHEMA, "unassigned NPU task"},
        {0}, {0}, {0},
        {"host compute", RK_E_UNSUPPORTED, "hidden host compute"},
        {"origin", RK_E_SCHEMA, "origin is not NUL terminated"},
        {"partial download view", RK_E_SHAPE, "full logical tile"},
        {"output extents", RK_E_SHAPE, "mm extents mismatch"},
        {"cbuf reuse", RK_E_SCHEMA, "CBUF reuse"},
        {"weight geometry", RK_E_SHAPE, "view id/tensor invalid"},
    };
    return expect[i];
}

static void rejection_cases(void) {
    for (int i = 0;; i++) {
        pb b;
        rk_plan_desc d;
        const reject_case want = mutate(i, &b, &d);
        if (!want.what) break;
        rk_diag diag;
        rk_plan *plan = (rk_plan *)1;
        const int rc = rk_plan_create(&d, &plan, &diag);
        checks++;
        if (rc != want.code || diag.code != want.code || plan != NULL || !strstr(diag.message, want.needle)) {
            failures++;
            fprintf(stderr, "FAIL reject %d (%s): rc=%d diag.code=%d \"%s\"\n", i, want.what, rc, diag.code,
                    diag.message);
        }
        if (plan && plan != (rk_plan *)1) rk_plan_destroy(plan);
    }
    rk_diag diag;
    rk_plan *plan = (rk_plan *)1;
    EXPECT_CODE(rk_plan_create(NULL, &plan, &diag), RK_E_INVALID, NULL);
    EXPECT(plan == NULL);
    EXPECT(rk_abi_version() == RK_ABI_VERSION);
    EXPECT_CODE(rk_target_validate_text("x", 1, "y", &diag), RK_E_UNSUPPORTED, NULL);
}

/* ------------------------------------------------------------------------------ many uploads */
/* 50 uploads of 12-row slices of one input (more than one pack launch holds), a sigmoid task on
 * the first slice and 50 downloads back into one output (the reference's many-upload case,
 * rk_plan_host_test.c:1493-1695, in its own form). */
static void many_uploads_case(int fd) {
    enum { TILES = 50, TR = 12, C = 32 };
    static pb b;
    memset(&b, 0, sizeof(b));
    const uint32_t A = pb_value(&b, RK_ROLE_INPUT, 2, TILES * TR, C, "A");
    const uint32_t Y = pb_value(&b, RK_ROLE_OUTPUT, 2, TILES * TR, C, "Y");
    uint32_t v[TILES], u[TILES];
    for (int i = 0; i < TILES; i++) v[i] = pb_view(&b, RK_LAYOUT_CUBE_F16, TR, C, RK_ROLE_INPUT_SLICE);
    const uint32_t vs = pb_view(&b, RK_LAYOUT_CUBE_F16, TR, C, RK_ROLE_SCRATCH);
    for (int i = 0; i < TILES; i++) u[i] = pb_upload(&b, A, v[i], (uint32_t)(TR * i), 0, 0);
    const uint32_t t = pb_task(&b, RK_TEMPLATE_LUT_SIGMOID_F16, (uint32_t[]){v[0]}, 1, vs, (uint32_t[]){u[0]}, 1);
    pb_submit(&b, t, 1);
    pb_download(&b, Y, vs, t, 0, 0);
    for (int i = 1; i < TILES; i++) pb_download(&b, Y, v[i], u[i], (uint32_t)(TR * i), 0);
    rk_plan_desc desc = pb_desc(&b);
    rk_diag diag;
    rk_plan *plan = NULL;
    EXPECT(rk_plan_create(&desc, &plan, &diag) == 0);
    if (!plan) {
        fprintf(stderr, "  many uploads create: %s\n", diag.message);
        return;
    }
    static _Float16 a[TILES * TR * C], y[TILES * TR * C], ref[TILES * TR * C];
    for (int i = 0; i < TILES * TR * C; i++) a[i] = (_Float16)((double)pattern((unsigned)i, 29) * 9.0);
    for (int i = 0; i < TILES * TR * C; i++)
        ref[i] = i < TR * C ? (_Float16)(1.0 / (1.0 + exp(-(double)a[i]))) : a[i];
    rk_workspace *ws = NULL;
    EXPECT(rk_workspace_create(fd, plan, NULL, 0, &ws, &diag) == 0);
    if (ws) {
        rk_binding in[] = {binding(&b.values[A], a)}, out[] = {binding(&b.values[Y], y)};
        rk_run_report report;
        EXPECT(rk_workspace_run(ws, in, 1, out, 1, &report, &diag) == 0);
        EXPECT(report.upload_calls == TILES && report.download_calls == TILES && report.task_count == 1);
        EXPECT(!memcmp(y, ref, sizeof(y)));
        EXPECT(rk_workspace_destroy(ws, &diag) == 0);
    }
    rk_plan_destroy(plan);
}

/* A writer that touches a buffer does not cover a wider reader: 12 uploaded rows under a 13-row
 * view of the same buffer are refused (the reference's partial-coverage case,
 * rk_plan_host_test.c:379-540). */
static void partial_coverage_case(void) {
    static pb b;
    memset(&b, 0, sizeof(b));
    const uint32_t A = pb_value(&b, RK_ROLE_INPUT, 2, 13, 32, "A");
    const uint32_t Y = pb_value(&b, RK_ROLE_OUTPUT, 2, 13, 32, "Y");
    const uint32_t up = pb_view(&b, RK_LAYOUT_CUBE_F16, 12, 32, RK_ROLE_INPUT_SLICE);
    /* a 13-row reader over the uploaded view's buffer (physical rows 16 against 12) */
    const uint32_t rd = b.nviews++;
    b.views[rd] = b.views[up];
    b.views[rd].id = rd;
    b.views[rd].tensor = tensor(RK_LAYOUT_CUBE_F16, 13, 32);
    b.views[rd].valid_region[1] = 13;
    b.buffers[b.views[up].buffer_id].capacity = b.views[rd].tensor.bytes;
    const uint32_t out = pb_view(&b, RK_LAYOUT_CUBE_F16, 13, 32, RK_ROLE_SCRATCH);
    const uint32_t u = pb_upload(&b, A, up, 0, 0, 0);
    const uint32_t t = pb_task(&b, RK_TEMPLATE_LUT_HARDSIGMOID_F16, (uint32_t[]){rd}, 1, out, (uint32_t[]){u}, 1);
    pb_submit(&b, t, 1);
    pb_download(&b, Y, out, t, 0, 0);
    rk_plan_desc desc = pb_desc(&b);
    rk_diag diag;
    rk_plan *plan = (rk_plan *)1;
    EXPECT_CODE(rk_plan_create(&desc, &plan, &diag), RK_E_SHAPE, "no write before this read");
    EXPECT(plan == NULL);
}

int main(void) {
    rejection_cases();
    partial_coverage_case();
    const int fd = rocket_open();
    if (fd < 0) {
        printf("rk_plan_test: no device (%d); %u checks, %u failures\n", fd, checks, failures);
        return failures ? 1 : 77;
    }
    rk_diag diag;
    EXPECT(rk_target_check(&diag) == 0);
    multitile_case(fd);
    kacc_case(fd);
    kacc_observed_case(fd);
    ew_case(fd);
    many_uploads_case(fd);
    rocket_close(fd);
    printf("rk_plan_test: %u checks, %u failures\n", checks, failures);
    return failures ? 1 : 0;
}
