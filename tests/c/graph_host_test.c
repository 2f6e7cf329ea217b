/* graph_host_test.c -- the graph compiler (csrc/host/graph.c) against the CPU stand-in of the device
 * seam (tests/c/mock_device.c).
 *
 * TEST INFRASTRUCTURE ONLY. Restates the checks of the reference's graph host test
 * (research/custom-ops/tests/c/graph_host_test.c) for the node kinds built here:
 *   main:91-104 / :404-420   forward references, double binding, shape mismatch, cycle, bad
 *                            operand, unknown op -> UNSUPPORTED
 *   execution_case :61-131   SwiGLU FFN plan (7 steps, 1 input, slot reuse, x live to the end),
 *                            resident bytes == plan.device_bytes, wrong binding refused before any
 *                            work, a failed launch leaves the output untouched, re-runs with new
 *                            inputs, budget - 1 -> TILING, every allocation failure -> NOMEM with
 *                            nothing leaked
 *   row_case :132-200        RMSNorm: results, non-finite input refused, square overflow -> SHAPE
 *                            with the output untouched, bad epsilon / flagged input / NaN gamma
 *   multiple_outputs :317-340  co_graph_run_many: three outputs, overlap refused, publish after
 *                            success only
 * plus the B200 additions: CO_CHAIN's fused gated pair and residual (b2_graph_get_info), the
 * small-M workspace, GELU with biases on both halves, SOFTMAX/ROPE -> UNSUPPORTED.
 * Expected values come from the oracle's C restatement (oracle/linear_oracle.c TILE16_EXACT for
 * Linear, oracle/graph_oracle.c for the other nodes), so they are compared bit for bit.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "b2_host.h"
#include "co_graph.h"

int oracle_linear(int mode, unsigned m, unsigned k, unsigned n, const uint16_t *x, const uint16_t *w,
                  const uint16_t *bias, int post, uint16_t *y16, double *act, double *raw, int threads);
uint16_t oracle_f16_from_double(double d);
double oracle_f16_to_double(uint16_t h);
uint16_t oracle_ew16(int op, uint16_t a, uint16_t b);
uint16_t oracle_act16(int act, uint16_t a);
unsigned oracle_rmsnorm(unsigned rows, unsigned cols, const uint16_t *x, const uint16_t *gamma, float eps,
                        uint16_t *y);

static int checks, failures;
static int FD;
#define EXPECT(e)                                                   \
    do {                                                            \
        ++checks;                                                   \
        if (!(e)) {                                                 \
            ++failures;                                             \
            printf("FAIL %s:%d %s\n", __FILE__, __LINE__, #e);      \
        }                                                           \
    } while (0)

typedef uint16_t h16;
#define F(p) ((const _Float16 *)(p))

static h16 fillv(unsigned i, unsigned seed) { return oracle_f16_from_double((((int)((i * 17 + seed) % 31)) - 15) / 128.0); }
static h16 *alloc16(size_t n) { return calloc(n ? n : 1, 2); }

static void linear_ref(unsigned m, unsigned k, unsigned n, const h16 *x, const h16 *w, const h16 *b, h16 *y) {
    EXPECT(oracle_linear(0, m, k, n, x, w, b, 0, y, NULL, NULL, 1) == 0);
}

/* Y = X + Linear(act(Linear(X, Wg, bg)) * Linear(X, Wu, bu), Wd) */
static void ffn_ref(unsigned m, unsigned d, unsigned h, int act, const h16 *x, const h16 *wg, const h16 *bg,
                    const h16 *wu, const h16 *bu, const h16 *wd, h16 *ref) {
    h16 *gate = alloc16((size_t)m * h), *up = alloc16((size_t)m * h);
    linear_ref(m, d, h, x, wg, bg, gate);
    linear_ref(m, d, h, x, wu, bu, up);
    for (size_t i = 0; i < (size_t)m * h; i++) gate[i] = oracle_ew16(1, oracle_act16(act, gate[i]), up[i]);
    linear_ref(m, h, d, gate, wd, NULL, ref);
    for (size_t i = 0; i < (size_t)m * d; i++) ref[i] = oracle_ew16(0, ref[i], x[i]);
    free(gate);
    free(up);
}

static int untouched(const void *p, size_t bytes) {
    for (size_t i = 0; i < bytes; i++)
        if (((const unsigned char *)p)[i] != 0x23) return 0;
    return 1;
}

static void execution_case(unsigned m, unsigned d, unsigned h, int gelu, int up_bias) {
    h16 *x = alloc16((size_t)m * d), *wg = alloc16((size_t)h * d), *wu = alloc16((size_t)h * d);
    h16 *wd = alloc16((size_t)d * h), *bias = alloc16(h), *bias2 = alloc16(h);
    h16 *ref = alloc16((size_t)m * d), *y = alloc16((size_t)m * d);
    for (size_t i = 0; i < (size_t)m * d; i++) x[i] = fillv((unsigned)i, 2);
    for (size_t i = 0; i < (size_t)h * d; i++) {
        wg[i] = fillv((unsigned)i, 3);
        wu[i] = fillv((unsigned)i, 7);
    }
    for (size_t i = 0; i < (size_t)d * h; i++) wd[i] = fillv((unsigned)i, 11);
    for (unsigned i = 0; i < h; i++) {
        bias[i] = fillv(i, 17);
        bias2[i] = fillv(i, 5);
    }
    const int act = gelu ? 2 : 1;
    co_graph_node nodes[8];
    memset(nodes, 0, sizeof(nodes));
    nodes[0] = (co_graph_node){.op = CO_GRAPH_INPUT, .rows = m, .cols = d};
    nodes[1] = (co_graph_node){.op = CO_GRAPH_LINEAR, .a = 0, .cols = h, .weights = F(wg), .bias = F(bias)};
    nodes[2] = (co_graph_node){.op = CO_GRAPH_LINEAR, .a = 0, .cols = h, .weights = F(wu),
                               .bias = up_bias ? F(bias2) : NULL};
    nodes[3] = (co_graph_node){.op = gelu ? CO_GRAPH_GELU : CO_GRAPH_SILU, .a = 1};
    nodes[4] = (co_graph_node){.op = CO_GRAPH_MUL, .a = 3, .b = 2};
    nodes[5] = (co_graph_node){.op = CO_GRAPH_LINEAR, .a = 4, .cols = d, .weights = F(wd)};
    nodes[6] = (co_graph_node){.op = CO_GRAPH_ADD, .a = 5, .b = 0};
    nodes[7].op = (enum co_graph_op)99;   /* unreachable: eliminated, not rejected */
    co_graph_desc desc = {nodes, 8, 6, 0};
    co_graph_plan p;
    EXPECT(!co_graph_plan_init(&desc, &p));
    EXPECT(p.steps == 7 && p.inputs == 1 && p.slots < 7);
    EXPECT(p.tensors[0].last == 6 && p.tensors[0].slot != p.tensors[5].slot);
    EXPECT(p.chain_submits < p.tasks);
    EXPECT((m <= B2D_GEMV_MAX_M) == (p.workspace_bytes > 0));
    ffn_ref(m, d, h, act, x, wg, bias, wu, up_bias ? bias2 : NULL, wd, ref);
    for (unsigned mode = 0; mode < 2; mode++) {
        const size_t live = b2h_live_bytes();
        co_graph *g = NULL;
        EXPECT(!co_graph_compile(FD, &desc, (enum co_mode)mode, &g));
        if (!g) exit(1);
        EXPECT(b2h_live_bytes() - live == p.device_bytes);
        b2_graph_info info;
        EXPECT(!b2_graph_get_info(g, &info));
        EXPECT(info.gated == (mode == CO_CHAIN) && info.residual == (mode == CO_CHAIN) && !info.captured);
        co_graph_input input = {0, F(x)};
        EXPECT(!co_graph_run(g, &input, 1, (_Float16 *)y));
        EXPECT(!memcmp(y, ref, (size_t)m * d * 2));
        uint64_t before = rocket_launch_count();
        input.node = 1;
        EXPECT(co_graph_run(g, &input, 1, (_Float16 *)y) == ROCKET_E_SHAPE);
        EXPECT(rocket_launch_count() == before);
        input.node = 0;
        memset(y, 0x23, (size_t)m * d * 2);
        b2_fault_inject(B2_FAULT_LAUNCH, 2);
        EXPECT(co_graph_run(g, &input, 1, (_Float16 *)y) == ROCKET_E_DEVICE);
        b2_fault_inject(B2_FAULT_NONE, 1);
        EXPECT(untouched(y, (size_t)m * d * 2));
        EXPECT(!co_graph_run(g, &input, 1, (_Float16 *)y));
        EXPECT(!memcmp(y, ref, (size_t)m * d * 2));
        /* a re-run with other inputs gives their result: the plan is re-runnable */
        h16 *x2 = alloc16((size_t)m * d), *ref2 = alloc16((size_t)m * d);
        for (size_t i = 0; i < (size_t)m * d; i++) x2[i] = oracle_f16_from_double(oracle_f16_to_double(x[i]) * 0.5 + 0.125);
        ffn_ref(m, d, h, act, x2, wg, bias, wu, up_bias ? bias2 : NULL, wd, ref2);
        input.data = F(x2);
        EXPECT(!co_graph_run(g, &input, 1, (_Float16 *)y));
        EXPECT(!memcmp(y, ref2, (size_t)m * d * 2));
        EXPECT(memcmp(ref2, ref, (size_t)m * d * 2));
        memset(y, 0x23, (size_t)m * d * 2);
        b2_fault_inject(B2_FAULT_NAN_OUTPUT, 1);
        EXPECT(co_graph_run(g, &input, 1, (_Float16 *)y) == ROCKET_E_DEVICE);
        b2_fault_inject(B2_FAULT_NONE, 1);
        EXPECT(untouched(y, (size_t)m * d * 2));
        /* device-resident entry: the input tensor written in place, one launch, status */
        void *xin = NULL, *yout = NULL;
        size_t ldx = 0, ldy = 0;
        EXPECT(!b2_graph_tensor(g, 0, &xin, &ldx) && !b2_graph_tensor(g, 6, &yout, &ldy));
        EXPECT(ldx % 8 == 0 && ldx >= d && b2_graph_tensor(g, 7, &xin, &ldx) == ROCKET_E_SHAPE);
        EXPECT(!b2_graph_tensor(g, 0, &xin, &ldx));
        for (unsigned r = 0; r < m; r++) memcpy((h16 *)xin + (size_t)r * ldx, x + (size_t)r * d, (size_t)d * 2);
        EXPECT(!b2_graph_launch(g) && !b2_sync(FD) && !b2_graph_status(g));
        int same = 1;
        for (unsigned r = 0; r < m; r++) same &= !memcmp((h16 *)yout + (size_t)r * ldy, ref + (size_t)r * d, (size_t)d * 2);
        EXPECT(same);
        free(x2);
        free(ref2);
        co_graph_destroy(g);
        EXPECT(b2h_live_bytes() == live);
    }
    desc.device_budget = p.device_bytes - 1;
    EXPECT(co_graph_plan_init(&desc, &p) == ROCKET_E_TILING);
    desc.device_budget = 0;
    for (unsigned mode = 0; mode < 2; mode++)
        for (unsigned nth = 1; nth <= 32; nth++) {
            const size_t live = b2h_live_bytes();
            co_graph *g = (co_graph *)1;
            b2_fault_inject(B2_FAULT_ALLOC, nth);
            int rc = co_graph_compile(FD, &desc, (enum co_mode)mode, &g);
            b2_fault_inject(B2_FAULT_NONE, 1);
            if (!rc) {   /* past the last allocation */
                EXPECT(nth > 4);
                co_graph_destroy(g);
                break;
            }
            EXPECT(rc == ROCKET_E_NOMEM && !g && b2h_live_bytes() == live);
        }
    free(x);
    free(wg);
    free(wu);
    free(wd);
    free(bias);
    free(bias2);
    free(ref);
    free(y);
}

static void rmsnorm_case(unsigned m, unsigned n) {
    h16 *x = alloc16((size_t)m * n), *y = alloc16((size_t)m * n), *gamma = alloc16(n), *ref = alloc16((size_t)m * n);
    for (unsigned c = 0; c < n; c++) gamma[c] = oracle_f16_from_double(0.5 + (c % 5) * 0.125);
    for (unsigned r = 0; r < m; r++)
        for (unsigned c = 0; c < n; c++)
            x[(size_t)r * n + c] = oracle_f16_from_double(r % 3 ? (((int)(c % 17)) - 8) / 8.0 : 0.0);
    co_graph_node nodes[2];
    memset(nodes, 0, sizeof(nodes));
    nodes[0] = (co_graph_node){.op = CO_GRAPH_INPUT, .rows = m, .cols = n};
    nodes[1] = (co_graph_node){.op = CO_GRAPH_RMSNORM, .a = 0, .gamma = F(gamma), .epsilon = 1e-5f};
    co_graph_desc d = {nodes, 2, 1, 0};
    co_graph_plan p;
    EXPECT(!co_graph_plan_init(&d, &p));
    EXPECT(p.hybrid_nodes == 0 && p.statistic_downloads == 0 && p.rowop_bytes == (size_t)((n + 7) / 8 * 8) * 2);
    EXPECT(oracle_rmsnorm(m, n, x, gamma, 1e-5f, ref) == 0);
    /* the reference's own tolerance check (graph_host_test.c:174-186): x * gamma / sqrt(mean(x^2) + eps) */
    int close = 1;
    for (unsigned r = 0; r < m; r++) {
        double sum = 0;
        for (unsigned c = 0; c < n; c++) sum += oracle_f16_to_double(x[(size_t)r * n + c]) * oracle_f16_to_double(x[(size_t)r * n + c]);
        for (unsigned c = 0; c < n; c++) {
            double e = oracle_f16_to_double(x[(size_t)r * n + c]) * oracle_f16_to_double(gamma[c]) / sqrt(sum / n + 1e-5);
            close &= fabs(oracle_f16_to_double(ref[(size_t)r * n + c]) - e) < 0.004;
        }
    }
    EXPECT(close);
    for (unsigned mode = 0; mode < 2; mode++) {
        const size_t live = b2h_live_bytes();
        co_graph *g = NULL;
        EXPECT(!co_graph_compile(FD, &d, (enum co_mode)mode, &g));
        if (!g) exit(1);
        EXPECT(b2h_live_bytes() - live == p.device_bytes);
        co_graph_input in = {0, F(x)};
        EXPECT(!co_graph_run(g, &in, 1, (_Float16 *)y));
        EXPECT(!memcmp(y, ref, (size_t)m * n * 2));
        h16 saved = x[0];
        x[0] = 0x7c00u;
        uint64_t before = rocket_launch_count();
        EXPECT(co_graph_run(g, &in, 1, (_Float16 *)y) == ROCKET_E_SHAPE && rocket_launch_count() == before);
        x[0] = saved;
        b2_fault_inject(B2_FAULT_LAUNCH, 1);
        memset(y, 0x23, (size_t)m * n * 2);
        EXPECT(co_graph_run(g, &in, 1, (_Float16 *)y) == ROCKET_E_DEVICE);
        b2_fault_inject(B2_FAULT_NONE, 1);
        EXPECT(untouched(y, (size_t)m * n * 2));
        co_graph_destroy(g);
        EXPECT(b2h_live_bytes() == live);
    }
    nodes[1].epsilon = 0;
    EXPECT(co_graph_plan_init(&d, &p) == ROCKET_E_SHAPE);
    nodes[1].epsilon = NAN;
    EXPECT(co_graph_plan_init(&d, &p) == ROCKET_E_SHAPE);
    nodes[1].epsilon = 1e-5f;
    nodes[0].flags = CO_GRAPH_ALLOW_NEG_INF;
    EXPECT(co_graph_plan_init(&d, &p) == ROCKET_E_SHAPE);
    nodes[0].flags = 0;
    /* a square that overflows FP16 (256^2) is refused and the output is untouched */
    co_graph *overflow = NULL;
    EXPECT(!co_graph_compile(FD, &d, CO_CHAIN, &overflow));
    memset(x, 0, (size_t)m * n * 2);
    x[0] = oracle_f16_from_double(256.0);
    memset(y, 0x23, (size_t)m * n * 2);
    co_graph_input oin = {0, F(x)};
    EXPECT(co_graph_run(overflow, &oin, 1, (_Float16 *)y) == ROCKET_E_SHAPE);
    EXPECT(untouched(y, (size_t)m * n * 2));
    /* so is a coefficient that overflows FP16 */
    x[0] = 0;
    co_graph_destroy(overflow);
    for (unsigned c = 0; c < n; c++) gamma[c] = oracle_f16_from_double(65504.0);
    EXPECT(!co_graph_compile(FD, &d, CO_CHAIN, &overflow));
    EXPECT(co_graph_run(overflow, &oin, 1, (_Float16 *)y) == ROCKET_E_SHAPE);
    EXPECT(untouched(y, (size_t)m * n * 2));
    co_graph_destroy(overflow);
    gamma[0] = 0x7e00u;
    co_graph *g = (co_graph *)1;
    EXPECT(co_graph_compile(FD, &d, CO_CHAIN, &g) == ROCKET_E_SHAPE && !g);
    free(x);
    free(y);
    free(gamma);
    free(ref);
}

static void multiple_outputs_case(void) {
    enum { R = 13, C = 33 };
    h16 x[R * C], a[R * C], b[R * C], c[R * C];
    for (unsigned i = 0; i < R * C; i++) x[i] = fillv(i, 3);
    co_graph_node nodes[4];
    memset(nodes, 0, sizeof(nodes));
    nodes[0] = (co_graph_node){.op = CO_GRAPH_INPUT, .rows = R, .cols = C};
    nodes[1] = (co_graph_node){.op = CO_GRAPH_HSIG, .a = 0};
    nodes[2] = (co_graph_node){.op = CO_GRAPH_ADD, .a = 1, .b = 0};
    nodes[3] = (co_graph_node){.op = CO_GRAPH_MUL, .a = 1, .b = 1};
    co_graph_desc desc = {nodes, 4, 1, 0};
    unsigned ids[] = {1, 2, 3};
    co_graph_plan p;
    EXPECT(!co_graph_plan_many(&desc, ids, 3, &p));
    EXPECT(p.steps == 4 && p.noutputs == 3);
    for (unsigned i = 1; i < 4; i++) EXPECT(p.tensors[i].last == p.steps);
    co_graph *g = NULL;
    const size_t live = b2h_live_bytes();
    EXPECT(!co_graph_compile_many(FD, &desc, ids, 3, CO_CHAIN, &g));
    if (!g) exit(1);
    EXPECT(b2h_live_bytes() - live == p.device_bytes);
    co_graph_input input = {0, F(x)};
    co_graph_output outputs[] = {{3, (_Float16 *)c}, {1, (_Float16 *)a}, {2, (_Float16 *)b}};
    EXPECT(!co_graph_run_many(g, &input, 1, outputs, 3));
    int ok = 1;
    for (unsigned i = 0; i < R * C; i++) {
        h16 v = oracle_f16_from_double(oracle_f16_to_double(x[i]) / 6.0 + 0.5);
        ok &= a[i] == v && b[i] == oracle_ew16(0, v, x[i]) && c[i] == oracle_ew16(1, v, v);
    }
    EXPECT(ok);
    uint64_t before = rocket_launch_count();
    outputs[0].data = (_Float16 *)a;
    EXPECT(co_graph_run_many(g, &input, 1, outputs, 3) == ROCKET_E_SHAPE && rocket_launch_count() == before);
    outputs[0].data = (_Float16 *)c;
    memset(a, 0x23, sizeof(a));
    memset(b, 0x23, sizeof(b));
    memset(c, 0x23, sizeof(c));
    b2_fault_inject(B2_FAULT_LAUNCH, (unsigned)p.chain_submits);
    EXPECT(co_graph_run_many(g, &input, 1, outputs, 3) == ROCKET_E_DEVICE);
    b2_fault_inject(B2_FAULT_NONE, 1);
    EXPECT(untouched(a, sizeof(a)) && untouched(b, sizeof(b)) && untouched(c, sizeof(c)));
    EXPECT(co_graph_run(g, &input, 1, (_Float16 *)a) == ROCKET_E_SHAPE);
    co_graph_destroy(g);
    EXPECT(b2h_live_bytes() == live);
    ids[2] = 1;
    EXPECT(co_graph_plan_many(&desc, ids, 3, &p) == ROCKET_E_SHAPE);
}

static void topology_case(void) {
    enum { R = 13, C = 33 };
    co_graph_node nodes[3];
    memset(nodes, 0, sizeof(nodes));
    nodes[0] = (co_graph_node){.op = CO_GRAPH_ADD, .a = 1, .b = 2};
    nodes[1] = (co_graph_node){.op = CO_GRAPH_INPUT, .rows = R, .cols = C};
    nodes[2] = (co_graph_node){.op = CO_GRAPH_INPUT, .rows = R, .cols = C};
    co_graph_desc desc = {nodes, 3, 0, 0};
    co_graph_plan p;
    EXPECT(!co_graph_plan_init(&desc, &p));
    EXPECT(p.order[2] == 0 && p.inputs == 2);
    h16 a[R * C], b[R * C], y[R * C];
    for (unsigned i = 0; i < R * C; i++) {
        a[i] = fillv(i, 2);
        b[i] = fillv(i, 9);
    }
    co_graph *g = NULL;
    EXPECT(!co_graph_compile(FD, &desc, CO_CHAIN, &g));
    if (!g) exit(1);
    co_graph_input inputs[] = {{2, F(b)}, {1, F(a)}};
    EXPECT(!co_graph_run(g, inputs, 2, (_Float16 *)y));
    int ok = 1;
    for (unsigned i = 0; i < R * C; i++) ok &= y[i] == oracle_ew16(0, a[i], b[i]);
    EXPECT(ok);
    uint64_t before = rocket_launch_count();
    inputs[0].node = 1;
    EXPECT(co_graph_run(g, inputs, 2, (_Float16 *)y) == ROCKET_E_SHAPE && rocket_launch_count() == before);
    co_graph_destroy(g);
    nodes[2].cols = 32;
    EXPECT(co_graph_plan_init(&desc, &p) == ROCKET_E_SHAPE);
    nodes[2].cols = 33;
    nodes[1].op = CO_GRAPH_SILU;
    nodes[1].a = 0;
    EXPECT(co_graph_plan_init(&desc, &p) == ROCKET_E_SHAPE);   /* cycle */
    nodes[1].a = 3;
    EXPECT(co_graph_plan_init(&desc, &p) == ROCKET_E_SHAPE);   /* operand out of range */
    nodes[1].op = (enum co_graph_op)99;
    EXPECT(co_graph_plan_init(&desc, &p) == ROCKET_E_UNSUPPORTED);
    /* the reference's hybrid row / rotary / attention operators are not built here */
    nodes[1] = (co_graph_node){.op = CO_GRAPH_INPUT, .rows = R, .cols = C};
    nodes[0] = (co_graph_node){.op = CO_GRAPH_SOFTMAX, .a = 1};
    desc.count = 2;
    EXPECT(co_graph_plan_init(&desc, &p) == ROCKET_E_UNSUPPORTED);
    nodes[0] = (co_graph_node){.op = CO_GRAPH_ROPE, .a = 1, .heads = 1, .head_dim = C, .rotary_dim = 32};
    EXPECT(co_graph_plan_init(&desc, &p) == ROCKET_E_UNSUPPORTED);
    nodes[0] = (co_graph_node){.op = CO_GRAPH_LINEAR, .a = 1, .cols = 5};
    EXPECT(co_graph_plan_init(&desc, &p) == ROCKET_E_SHAPE);   /* Linear without weights */
    nodes[0] = (co_graph_node){.op = CO_GRAPH_HSIG, .a = 1, .cols = 5};
    EXPECT(co_graph_plan_init(&desc, &p) == ROCKET_E_SHAPE);   /* cols only on Linear */
    nodes[1].rows = CO_MAX_M + 1;
    nodes[0].cols = 0;
    EXPECT(co_graph_plan_init(&desc, &p) == ROCKET_E_SHAPE);
}

/* A large input (4 MiB): a NaN or an infinity at the start, on either side of a 1 MiB boundary and at
 * the end is refused with no launch and the output untouched, and the all-finite input runs. */
static void large_input_case(void) {
    enum { R = 1024, C = 2048 };
    const size_t n = (size_t)R * C;
    h16 *x = malloc(n * 2), *y = malloc(n * 2);
    if (!x || !y) exit(1);
    for (size_t i = 0; i < n; i++) x[i] = fillv((unsigned)i, 5);
    co_graph_node nodes[2];
    memset(nodes, 0, sizeof(nodes));
    nodes[0] = (co_graph_node){.op = CO_GRAPH_INPUT, .rows = R, .cols = C};
    nodes[1] = (co_graph_node){.op = CO_GRAPH_HSIG, .a = 0};
    co_graph_desc desc = {nodes, 2, 1, 0};
    co_graph *g = NULL;
    EXPECT(!co_graph_compile(FD, &desc, CO_CHAIN, &g));
    if (!g) exit(1);
    co_graph_input in = {0, F(x)};
    const size_t at[] = {0, (1u << 19) - 1, 1u << 19, 3u << 19, n - 1};
    for (unsigned i = 0; i < sizeof(at) / sizeof(at[0]); i++) {
        const h16 saved = x[at[i]];
        x[at[i]] = (i & 1) ? 0xfc00u : 0x7e00u;   /* -inf, NaN */
        memset(y, 0x23, n * 2);
        uint64_t before = rocket_launch_count();
        EXPECT(co_graph_run(g, &in, 1, (_Float16 *)y) == ROCKET_E_SHAPE && rocket_launch_count() == before);
        EXPECT(untouched(y, n * 2));
        x[at[i]] = saved;
    }
    EXPECT(!co_graph_run(g, &in, 1, (_Float16 *)y));
    int ok = 1;
    for (size_t i = 0; i < n; i++) ok &= y[i] == oracle_ew16(4, x[i], 0);   /* HardSigmoid */
    EXPECT(ok);
    co_graph_destroy(g);
    free(x);
    free(y);
}

int main(void) {
    FD = rocket_open();
    EXPECT(FD >= 0);
    if (FD < 0) return 1;
    topology_case();
    execution_case(13, 257, 289, 0, 0);
    execution_case(257, 17, 33, 0, 0);
    execution_case(5, 70, 40, 0, 1);      /* small M: the gated pair through the workspace */
    execution_case(40, 96, 72, 1, 1);     /* GELU, biases on both halves */
    rmsnorm_case(257, 513);
    multiple_outputs_case();
    large_input_case();
    rocket_close(FD);
    EXPECT(b2h_live_bytes() == 0);
    printf("graph_host_test: %d checks, %d failures\n", checks, failures);
    return failures ? 1 : 0;
}
