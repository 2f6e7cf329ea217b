/* graph.c -- static FP16 graph compiler and executor (co_graph_*), host side.
 *
 * Restates the public behaviour of research/custom-ops/src/co_graph.c (reference):
 *   visit / operands              :14-41    depth-first topology, cycle and operand checks,
 *                                           flags only on inputs, unknown op -> UNSUPPORTED
 *   co_graph_plan_many            :53-173   shape inference, Linear plan per node, operand flag
 *                                           rule, outputs live to the end, slot reuse with a
 *                                           strictly earlier last use, budget -> TILING
 *   co_graph_compile_many         :196-257  copies nodes, allocates slots and per-node state;
 *                                           any failure frees everything
 *   co_graph_run_many             :315-376  output binding checks, input binding/finiteness
 *                                           checks before any work, execution in plan order,
 *                                           guard checks, finite outputs, publish after success
 * B200 design: tensors are row-major FP16 matrices in HBM (16-byte row pitch) instead of 256x256
 * cube tiles; Linear nodes run the tcgen05 GEMM / streamed GEMV directly on the slots; the other
 * nodes are single kernels (graph_kernels.cu). A mode-independent fusion analysis finds
 *   gated pairs   MUL(SILU|GELU(LINEAR g), LINEAR u) with g, u on the same input and each of
 *                 g, u and the activation used once -> one GEMM over the packed gate|up weight
 *                 whose epilogue forms the product (CO_CHAIN),
 *   residuals     ADD(LINEAR l, r) with l used once -> the ADD in l's epilogue (CO_CHAIN),
 * and extends the liveness of the fused op's inputs to the step that consumes its result, so
 * one slot plan serves both modes. CO_CHAIN records the program as a CUDA graph at its first
 * run and replays it; CO_SEPARATE launches one kernel (Linear: GEMM + epilogue) per node.
 */
#include "b2_host.h"
#include "co_graph.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define MAXN CO_GRAPH_MAX_NODES

enum { F_NONE = 0, F_GATED = 1, F_RESIDUAL = 2, F_MEMBER = 3 };

/* Fusion groups, indexed by the root node (the MUL of a gated pair, the ADD of a residual). */
struct fusion {
    unsigned kind[MAXN];
    unsigned g[MAXN], u[MAXN], act[MAXN];   /* gated: gate Linear, up Linear, SILU/GELU node */
    unsigned l[MAXN], r[MAXN];              /* residual: the Linear and the other operand */
    unsigned ngated, nresidual;
    unsigned uses[MAXN];
};

struct co_graph {
    int fd;
    enum co_mode mode;
    unsigned count;
    co_graph_node nodes[MAXN];      /* data pointers cleared after compile */
    co_graph_plan plan;
    struct fusion f;
    void *slot[MAXN];
    size_t slot_alloc[MAXN];
    size_t ld[MAXN];                /* row pitch (elements) of each planned tensor */
    void *w[MAXN];                  /* Linear weight [roundup(cols, 32), ldw]; packed gate|up at a gated root */
    size_t w_bytes[MAXN], ldw[MAXN];
    void *bias[MAXN];               /* [roundup(cols, 32)] or NULL */
    size_t bias_bytes[MAXN];
    void *gamma[MAXN];
    size_t gamma_bytes[MAXN];
    void *tmp; size_t tmp_bytes;     /* FP16 sums of a gated pair served by the small-M kernel */
    b2_exec *exec;
    int no_capture;
    unsigned kernels;
};

static unsigned blocks256(unsigned n) { return (n + 255) / 256; }
static int binary(enum co_graph_op op) { return op == CO_GRAPH_ADD || op == CO_GRAPH_MUL; }
static int gated_op(enum co_graph_op op) { return op == CO_GRAPH_SILU || op == CO_GRAPH_GELU; }
static size_t pitch(unsigned cols) { return b2h_round_up(cols, 8); }
static size_t rows32(unsigned n) { return b2h_round_up(n, 32); }

/* reference co_graph.c:14-19 */
static unsigned operands(const co_graph_node *n, unsigned refs[4]) {
    if (n->op == CO_GRAPH_INPUT) return 0;
    refs[0] = n->a;
    if (n->op == CO_GRAPH_ATTENTION) {
        refs[1] = n->b;
        refs[2] = n->c;
        refs[3] = n->mask_node;
        return 3 + n->has_mask;
    }
    if (binary(n->op)) {
        refs[1] = n->b;
        return 2;
    }
    return 1;
}

/* The per-node checks made when the walk first reaches a node (reference co_graph.c:29-41): an op
 * past ATTENTION is unsupported; flags other than ALLOW_NEG_INF, flags on a non-INPUT node and a
 * mask count above one are shape errors. */
static int node_ok(const co_graph_node *n) {
    if ((unsigned)n->op > (unsigned)CO_GRAPH_ATTENTION) return ROCKET_E_UNSUPPORTED;
    if ((n->flags & ~CO_GRAPH_ALLOW_NEG_INF) || (n->flags && n->op != CO_GRAPH_INPUT)) return ROCKET_E_SHAPE;
    return n->op == CO_GRAPH_ATTENTION && n->has_mask > 1 ? ROCKET_E_SHAPE : 0;
}

enum { NODE_UNSEEN = 0, NODE_OPEN = 1, NODE_PLACED = 2 };
struct walk_frame {
    unsigned id, next, nrefs, refs[4];
};

/* Opens node `id` on the walk stack, unless it is already placed. Reaching an open node again
 * closes a cycle; an id past the graph is not a node: both ROCKET_E_SHAPE. */
static int open_node(const co_graph_desc *d, unsigned id, unsigned char *state, struct walk_frame *stack,
                     unsigned *depth) {
    if (id >= d->count || state[id] == NODE_OPEN) return ROCKET_E_SHAPE;
    if (state[id] == NODE_PLACED) return 0;
    const int rc = node_ok(&d->nodes[id]);
    if (rc) return rc;
    state[id] = NODE_OPEN;
    struct walk_frame *f = &stack[(*depth)++];
    f->id = id;
    f->next = 0;
    f->nrefs = operands(&d->nodes[id], f->refs);
    return 0;
}

/* Places `root` and everything it reads into p->order, operands before their consumer and in operand
 * order (a depth-first post-order, walked with an explicit stack: each node is open at most once, so
 * the stack never holds more than the graph's nodes). */
static int place(const co_graph_desc *d, unsigned root, unsigned char *state, co_graph_plan *p) {
    struct walk_frame stack[MAXN];
    unsigned depth = 0;
    int rc = open_node(d, root, state, stack, &depth);
    while (!rc && depth) {
        struct walk_frame *top = &stack[depth - 1];
        if (top->next < top->nrefs) {
            rc = open_node(d, top->refs[top->next++], state, stack, &depth);
            continue;
        }
        state[top->id] = NODE_PLACED;
        p->order[p->steps++] = top->id;
        depth--;
    }
    return rc;
}

static int tensor_size(unsigned rows, unsigned cols, size_t *bytes, unsigned *tiles) {
    if (!rows || rows > CO_MAX_M || !cols || cols > CO_MAX_N) return ROCKET_E_SHAPE;
    *bytes = (size_t)rows * pitch(cols) * 2;
    *tiles = blocks256(rows) * blocks256(cols);
    return 0;
}

static size_t linear_weight_bytes(unsigned in, unsigned cols) { return rows32(cols) * pitch(in) * 2; }
static size_t linear_bias_bytes(unsigned cols) { return rows32(cols) * 2; }

/* Gated pairs first, then residual Linears, in plan order; each node joins at most one group. */
static void find_fusions(const co_graph_desc *d, const co_graph_plan *p, struct fusion *f) {
    memset(f, 0, sizeof(*f));
    for (unsigned s = 0; s < p->steps; s++) {
        unsigned refs[4], nr = operands(&d->nodes[p->order[s]], refs);
        for (unsigned i = 0; i < nr; i++) f->uses[refs[i]]++;
    }
    for (unsigned i = 0; i < p->noutputs; i++) f->uses[p->outputs[i]]++;
    for (unsigned s = 0; s < p->steps; s++) {
        unsigned id = p->order[s];
        const co_graph_node *m = &d->nodes[id];
        if (m->op != CO_GRAPH_MUL) continue;
        for (unsigned side = 0; side < 2; side++) {
            unsigned sa = side ? m->b : m->a, ua = side ? m->a : m->b;
            const co_graph_node *act = &d->nodes[sa], *up = &d->nodes[ua];
            if (!gated_op(act->op) || up->op != CO_GRAPH_LINEAR) continue;
            unsigned ga = act->a;
            const co_graph_node *gate = &d->nodes[ga];
            if (gate->op != CO_GRAPH_LINEAR || ga == ua || gate->a != up->a || gate->cols != up->cols) continue;
            if (f->uses[sa] != 1 || f->uses[ga] != 1 || f->uses[ua] != 1) continue;
            if (f->kind[sa] || f->kind[ga] || f->kind[ua]) continue;
            f->kind[id] = F_GATED;
            f->g[id] = ga;
            f->u[id] = ua;
            f->act[id] = sa;
            f->kind[sa] = f->kind[ga] = f->kind[ua] = F_MEMBER;
            f->ngated++;
            break;
        }
    }
    for (unsigned s = 0; s < p->steps; s++) {
        unsigned id = p->order[s];
        const co_graph_node *add = &d->nodes[id];
        if (add->op != CO_GRAPH_ADD || f->kind[id]) continue;
        for (unsigned side = 0; side < 2; side++) {
            unsigned la = side ? add->b : add->a, ra = side ? add->a : add->b;
            if (la == ra || d->nodes[la].op != CO_GRAPH_LINEAR || f->uses[la] != 1 || f->kind[la]) continue;
            f->kind[id] = F_RESIDUAL;
            f->l[id] = la;
            f->r[id] = ra;
            f->kind[la] = F_MEMBER;
            f->nresidual++;
            break;
        }
    }
}

/* Kernels one node adds to a run (fused: CO_CHAIN program; else CO_SEPARATE). */
static unsigned node_kernels(const co_graph_node *n, const struct fusion *f, unsigned id, unsigned rows, int fused) {
    const int small = rows <= B2D_GEMV_MAX_M;
    if (fused) {
        if (f->kind[id] == F_MEMBER) return 0;
        if (f->kind[id] == F_GATED || f->kind[id] == F_RESIDUAL) return small ? 2 : 1;
        if (n->op == CO_GRAPH_LINEAR) return 1;
    } else if (n->op == CO_GRAPH_LINEAR) {
        return 2;   /* GEMM/GEMV to the FP16 fold, then the separate epilogue */
    }
    return n->op == CO_GRAPH_INPUT ? 0 : 1;
}

/* reference co_graph.c:53-173, with the B200 sizes and the fusion groups' liveness. */
static int analyze(const co_graph_desc *d, const unsigned *outputs, unsigned noutputs, co_graph_plan *out,
                   struct fusion *fo) {
    if (!out) return ROCKET_E_SHAPE;
    memset(out, 0, sizeof(*out));
    if (!d || !d->nodes || !d->count || d->count > MAXN || !outputs || !noutputs || noutputs > MAXN)
        return ROCKET_E_SHAPE;
    co_graph_plan p;
    memset(&p, 0, sizeof(p));
    unsigned char state[MAXN] = {0};
    p.noutputs = noutputs;
    for (unsigned i = 0; i < noutputs; i++) {
        if (outputs[i] >= d->count) return ROCKET_E_SHAPE;
        for (unsigned j = 0; j < i; j++)
            if (outputs[j] == outputs[i]) return ROCKET_E_SHAPE;
        p.outputs[i] = outputs[i];
        int rc = place(d, outputs[i], state, &p);
        if (rc) return rc;
    }
    for (unsigned step = 0; step < p.steps; step++) {
        unsigned id = p.order[step];
        const co_graph_node *node = &d->nodes[id];
        co_graph_tensor_plan *t = &p.tensors[id];
        t->first = step;
        t->last = step;
        if (node->op == CO_GRAPH_INPUT) {
            t->rows = node->rows;
            t->cols = node->cols;
            p.inputs++;
        } else {
            if (node->op == CO_GRAPH_SOFTMAX || node->op == CO_GRAPH_ROPE || node->op == CO_GRAPH_ATTENTION)
                return ROCKET_E_UNSUPPORTED;
            const co_graph_tensor_plan *a = &p.tensors[node->a];
            t->rows = a->rows;
            t->cols = a->cols;
            if (node->rows) return ROCKET_E_SHAPE;
            if (node->op == CO_GRAPH_LINEAR) {
                if (!node->weights) return ROCKET_E_SHAPE;
                t->cols = node->cols;
                co_linear_plan lp;
                int rc = co_linear_plan_init_ex(&lp, t->rows, a->cols, t->cols, node->bias != NULL, CO_LINEAR_NONE,
                                                SIZE_MAX);
                if (rc) return rc;
                p.linear_bytes += linear_weight_bytes(a->cols, t->cols) + (node->bias ? linear_bias_bytes(t->cols) : 0);
            } else {
                if (node->cols) return ROCKET_E_SHAPE;
                if (node->op == CO_GRAPH_RMSNORM &&
                    (!node->gamma || !isfinite(node->epsilon) || node->epsilon <= 0))
                    return ROCKET_E_SHAPE;
                if (binary(node->op)) {
                    const co_graph_tensor_plan *b = &p.tensors[node->b];
                    if (a->rows != b->rows || a->cols != b->cols) return ROCKET_E_SHAPE;
                }
            }
            unsigned refs[4], nr = operands(node, refs);
            for (unsigned i = 0; i < nr; i++) p.tensors[refs[i]].last = step;
        }
        int rc = tensor_size(t->rows, t->cols, &t->bytes, &t->tiles);
        if (rc) return rc;
        if (node->op == CO_GRAPH_RMSNORM) p.rowop_bytes += pitch(t->cols) * 2;
    }
    /* reference co_graph.c:141-150: -inf inputs only feed Softmax scores / an Attention mask */
    for (unsigned step = 0; step < p.steps; step++) {
        const co_graph_node *n = &d->nodes[p.order[step]];
        unsigned refs[4], nr = operands(n, refs);
        for (unsigned i = 0; i < nr; i++)
            if (d->nodes[refs[i]].flags &&
                !((n->op == CO_GRAPH_SOFTMAX && i == 0) || (n->op == CO_GRAPH_ATTENTION && n->has_mask && i == 3)))
                return ROCKET_E_SHAPE;
    }
    for (unsigned i = 0; i < noutputs; i++) {
        if (d->nodes[outputs[i]].flags) return ROCKET_E_SHAPE;
        p.tensors[outputs[i]].last = p.steps;
    }
    struct fusion f;
    find_fusions(d, &p, &f);
    size_t tmp_bytes = 0;
    for (unsigned step = 0; step < p.steps; step++) {
        unsigned id = p.order[step];
        unsigned src = f.kind[id] == F_GATED ? d->nodes[f.g[id]].a : f.kind[id] == F_RESIDUAL ? d->nodes[f.l[id]].a
                                                                                             : MAXN;
        if (src < MAXN && p.tensors[src].last < step) p.tensors[src].last = step;   /* read at the root's step */
        if (f.kind[id] == F_GATED && p.tensors[id].rows <= B2D_GEMV_MAX_M) {
            size_t b = (size_t)p.tensors[id].rows * 2 * rows32(p.tensors[id].cols) * 2;
            if (b > tmp_bytes) tmp_bytes = b;
        }
        p.tasks += node_kernels(&d->nodes[id], &f, id, p.tensors[id].rows, 0);
        p.chain_submits += node_kernels(&d->nodes[id], &f, id, p.tensors[id].rows, 1);
    }
    /* Strictly earlier last use is required: never overwrite a live operand (co_graph.c:151). */
    unsigned slot_end[MAXN] = {0};
    for (unsigned step = 0; step < p.steps; step++) {
        co_graph_tensor_plan *t = &p.tensors[p.order[step]];
        unsigned chosen = MAXN;
        size_t best = SIZE_MAX;
        for (unsigned s = 0; s < p.slots; s++)
            if (slot_end[s] < step) {
                size_t cost = p.slot_bytes[s] > t->bytes ? p.slot_bytes[s] : t->bytes;
                if (cost < best) {
                    best = cost;
                    chosen = s;
                }
            }
        if (chosen == MAXN) chosen = p.slots++;
        t->slot = chosen;
        slot_end[chosen] = t->last;
        if (t->bytes > p.slot_bytes[chosen]) p.slot_bytes[chosen] = t->bytes;
    }
    for (unsigned s = 0; s < p.slots; s++) p.tensor_bytes += p.slot_bytes[s] + CO_SLACK + CO_GUARD;
    p.workspace_bytes = tmp_bytes;
    p.tasks += 1 + p.noutputs;           /* the guard check of every slot, a scan of each output */
    p.chain_submits += 1 + p.noutputs;
    p.device_bytes = p.tensor_bytes + p.linear_bytes + p.rowop_bytes + p.workspace_bytes;
    if (p.device_bytes > (d->device_budget ? d->device_budget : CO_LINEAR_DEVICE_BUDGET)) return ROCKET_E_TILING;
    *out = p;
    if (fo) *fo = f;
    return 0;
}

int co_graph_plan_many(const co_graph_desc *d, const unsigned *outputs, unsigned noutputs, co_graph_plan *out) {
    return analyze(d, outputs, noutputs, out, NULL);
}

int co_graph_plan_init(const co_graph_desc *d, co_graph_plan *out) {
    return co_graph_plan_many(d, d ? &d->output : NULL, 1, out);
}

/* 1 if no FP16 value of v[0, n) is infinite or NaN: four values per 64-bit word at a time (an
 * exponent field of all ones plus one carries into the lane's sign bit). */
static int finite16(const _Float16 *v, size_t n) {
    const uint16_t *b = (const uint16_t *)v;
    size_t i = 0;
    if (((uintptr_t)b & 7u) == 0) {
        const uint64_t *w = (const uint64_t *)b;
        uint64_t any = 0;
        for (size_t j = 0; j < n / 4; j++) any |= ((w[j] & 0x7c007c007c007c00ull) + 0x0400040004000400ull);
        if (any & 0x8000800080008000ull) return 0;
        i = n / 4 * 4;
    }
    for (; i < n; i++)
        if ((b[i] & 0x7c00u) == 0x7c00u) return 0;
    return 1;
}

void co_graph_destroy(co_graph *g) {
    if (!g) return;
    b2_dev *d = b2h_dev(g->fd);
    if (d) b2d_sync(d);
    b2d_exec_destroy(g->exec);
    for (unsigned i = 0; i < MAXN; i++) {
        b2h_free(g->fd, g->slot[i], g->slot_alloc[i]);
        b2h_free(g->fd, g->w[i], g->w_bytes[i]);
        b2h_free(g->fd, g->bias[i], g->bias_bytes[i]);
        b2h_free(g->fd, g->gamma[i], g->gamma_bytes[i]);
    }
    b2h_free(g->fd, g->tmp, g->tmp_bytes);
    free(g);
}

static int alloc_into(co_graph *g, size_t bytes, void **ptr, size_t *held) {
    int rc = b2h_malloc(g->fd, bytes, ptr);
    if (!rc) *held = bytes;
    return rc;
}

/* W [cols, in] row-major on the host -> [roundup(cols, 32), pitch(in)] in HBM, padding rows zero. */
static int upload_rows(b2_dev *d, void *dst, size_t ldw, const _Float16 *src, unsigned in, unsigned rows) {
    if (!rows) return 0;
    return b2d_copy_2d(d, dst, ldw * 2, src, (size_t)in * 2, (size_t)in * 2, rows, B2D_H2D);
}

/* Gate and up weights interleaved in 64-row blocks: block t holds gate rows [32t, 32t+32) and
 * then up rows [32t, 32t+32), so one 256-column GEMM tile carries 128 hidden columns of both. */
static int upload_packed(b2_dev *d, void *dst, size_t ldw, const _Float16 *wg, const _Float16 *wu, unsigned in,
                         unsigned h) {
    for (unsigned t = 0; t * 32 < h; t++) {
        unsigned rows = h - t * 32 < 32 ? h - t * 32 : 32;
        char *blk = (char *)dst + (size_t)t * 64 * ldw * 2;
        int rc = upload_rows(d, blk, ldw, wg + (size_t)t * 32 * in, in, rows);
        if (!rc) rc = upload_rows(d, blk + (size_t)32 * ldw * 2, ldw, wu + (size_t)t * 32 * in, in, rows);
        if (rc) return rc;
    }
    return 0;
}

static int upload_vec(b2_dev *d, void *dst, const _Float16 *src, unsigned n) {
    return b2d_copy_2d(d, dst, (size_t)n * 2, src, (size_t)n * 2, (size_t)n * 2, 1, B2D_H2D);
}

static int compile_nodes(co_graph *g, const co_graph_desc *desc) {
    b2_dev *d = b2h_dev(g->fd);
    const co_graph_plan *p = &g->plan;
    const int fuse = g->mode == CO_CHAIN;
    int rc = 0;
    for (unsigned s = 0; s < p->slots; s++) {
        rc = alloc_into(g, p->slot_bytes[s] + CO_SLACK + CO_GUARD, &g->slot[s], &g->slot_alloc[s]);
        if (!rc) rc = b2d_guard_init(d, g->slot[s], p->slot_bytes[s], CO_SLACK, CO_GUARD);
        if (rc) return rc;
    }
    if (p->workspace_bytes) {
        rc = alloc_into(g, p->workspace_bytes, &g->tmp, &g->tmp_bytes);
        if (rc) return rc;
    }
    for (unsigned step = 0; step < p->steps; step++) {
        unsigned id = p->order[step];
        const co_graph_node *n = &desc->nodes[id];
        const co_graph_tensor_plan *t = &p->tensors[id];
        g->ld[id] = pitch(t->cols);
        if (n->op == CO_GRAPH_LINEAR) {
            unsigned in = p->tensors[n->a].cols;
            g->ldw[id] = pitch(in);
            if (n->bias) {
                rc = alloc_into(g, linear_bias_bytes(t->cols), &g->bias[id], &g->bias_bytes[id]);
                if (!rc) rc = upload_vec(d, g->bias[id], n->bias, t->cols);
                if (rc) return rc;
            }
            if (fuse && g->f.kind[id] == F_MEMBER) {
                int in_gated = 0;   /* a gated pair's weights live packed at the root */
                for (unsigned r = 0; r < MAXN && !in_gated; r++)
                    in_gated = g->f.kind[r] == F_GATED && (g->f.g[r] == id || g->f.u[r] == id);
                if (in_gated) continue;
            }
            rc = alloc_into(g, linear_weight_bytes(in, t->cols), &g->w[id], &g->w_bytes[id]);
            if (!rc) rc = upload_rows(d, g->w[id], g->ldw[id], n->weights, in, t->cols);
            if (rc) return rc;
        } else if (n->op == CO_GRAPH_RMSNORM) {
            rc = alloc_into(g, pitch(t->cols) * 2, &g->gamma[id], &g->gamma_bytes[id]);
            if (!rc) rc = upload_vec(d, g->gamma[id], n->gamma, t->cols);
            if (rc) return rc;
        } else if (fuse && g->f.kind[id] == F_GATED) {
            const co_graph_node *gn = &desc->nodes[g->f.g[id]], *un = &desc->nodes[g->f.u[id]];
            unsigned in = p->tensors[gn->a].cols, h = gn->cols;
            g->ldw[id] = pitch(in);
            rc = alloc_into(g, 2 * linear_weight_bytes(in, h), &g->w[id], &g->w_bytes[id]);
            if (!rc) rc = upload_packed(d, g->w[id], g->ldw[id], gn->weights, un->weights, in, h);
            if (rc) return rc;
        }
    }
    return b2d_sync(d);
}

int co_graph_compile_many(int fd, const co_graph_desc *desc, const unsigned *outputs, unsigned noutputs,
                          enum co_mode mode, co_graph **out) {
    if (!out) return ROCKET_E_SHAPE;
    *out = NULL;
    if (fd < 0 || !b2h_valid_fd(fd) || (mode != CO_CHAIN && mode != CO_SEPARATE)) return ROCKET_E_SHAPE;
    co_graph_plan plan;
    struct fusion f;
    int rc = analyze(desc, outputs, noutputs, &plan, &f);
    if (rc) return rc;
    if (mode == CO_CHAIN && !rocket_batched_submit_supported()) return ROCKET_E_UNSUPPORTED;
    /* model data is checked before any allocation (co_linear_create / co_rowop_create reject it) */
    for (unsigned step = 0; step < plan.steps; step++) {
        const co_graph_node *n = &desc->nodes[plan.order[step]];
        const co_graph_tensor_plan *t = &plan.tensors[plan.order[step]];
        if (n->op == CO_GRAPH_LINEAR &&
            (!finite16(n->weights, (size_t)t->cols * plan.tensors[n->a].cols) || (n->bias && !finite16(n->bias, t->cols))))
            return ROCKET_E_SHAPE;
        if (n->op == CO_GRAPH_RMSNORM && !finite16(n->gamma, t->cols)) return ROCKET_E_SHAPE;
    }
    co_graph *g = calloc(1, sizeof(*g));
    if (!g) return ROCKET_E_NOMEM;
    g->fd = fd;
    g->mode = mode;
    g->count = desc->count;
    g->plan = plan;
    g->f = f;
    memcpy(g->nodes, desc->nodes, desc->count * sizeof(*desc->nodes));
    rc = compile_nodes(g, desc);
    if (rc) {
        co_graph_destroy(g);
        return rc;
    }
    for (unsigned i = 0; i < g->count; i++) {
        g->nodes[i].weights = NULL;
        g->nodes[i].bias = NULL;
        g->nodes[i].gamma = NULL;
    }
    g->kernels = (unsigned)(mode == CO_CHAIN ? plan.chain_submits : plan.tasks);
    *out = g;
    return 0;
}

int co_graph_compile(int fd, const co_graph_desc *desc, enum co_mode mode, co_graph **out) {
    return co_graph_compile_many(fd, desc, desc ? &desc->output : NULL, 1, mode, out);
}

/* ------------------------------------------------------------------------------ execution */
static void *tensor_ptr(const co_graph *g, unsigned id) { return g->slot[g->plan.tensors[id].slot]; }

static int launch_linear(co_graph *g, unsigned id, const b2k_linear *a, unsigned *launches) {
    (void)id;
    if (b2h_fault(B2_FAULT_LAUNCH)) return ROCKET_E_DEVICE;
    unsigned l = 0;
    int rc = b2d_linear(b2h_dev(g->fd), a, &l);
    *launches += l;
    return rc;
}

static b2k_linear linear_desc(const co_graph *g, unsigned id, int fused) {
    const co_graph_node *n = &g->nodes[id];
    const co_graph_tensor_plan *t = &g->plan.tensors[id];
    b2k_linear a;
    memset(&a, 0, sizeof(a));
    a.m = t->rows;
    a.n = t->cols;
    a.k = g->plan.tensors[n->a].cols;
    a.x = tensor_ptr(g, n->a);
    a.ldx = g->ld[n->a];
    a.w = g->w[id];
    a.ldw = g->ldw[id];
    a.bias = g->bias[id];
    a.y = tensor_ptr(g, id);
    a.ldy = g->ld[id];
    a.acc = 0;            /* the reference's per-256-K FP16 fold */
    a.fused = fused;
    return a;
}

/* One node of the program (CO_CHAIN: the fused program, members of a group skipped). */
static int exec_node(co_graph *g, unsigned id, unsigned *launches) {
    b2_dev *d = b2h_dev(g->fd);
    const co_graph_node *n = &g->nodes[id];
    const co_graph_tensor_plan *t = &g->plan.tensors[id];
    const int fuse = g->mode == CO_CHAIN;
    const unsigned kind = fuse ? g->f.kind[id] : F_NONE;
    if (n->op == CO_GRAPH_INPUT || kind == F_MEMBER) return 0;
    if (kind == F_GATED) {
        unsigned gi = g->f.g[id], ui = g->f.u[id];
        const co_graph_node *gn = &g->nodes[gi];
        b2k_linear a = linear_desc(g, gi, 1);
        a.n = (unsigned)(2 * rows32(gn->cols));
        a.w = g->w[id];
        a.ldw = g->ldw[id];
        a.bias = g->bias[gi];
        a.bias2 = g->bias[ui];
        a.gate = g->nodes[g->f.act[id]].op == CO_GRAPH_GELU ? 2 : 1;
        a.gate_n = gn->cols;
        a.y = tensor_ptr(g, id);
        a.ldy = g->ld[id];
        a.tmp = g->tmp;
        a.ldt = a.n;
        return launch_linear(g, id, &a, launches);
    }
    if (kind == F_RESIDUAL) {
        unsigned li = g->f.l[id], ri = g->f.r[id];
        b2k_linear a = linear_desc(g, li, 1);
        a.y = tensor_ptr(g, id);
        a.ldy = g->ld[id];
        a.res = tensor_ptr(g, ri);
        a.ldr = g->ld[ri];
        return launch_linear(g, id, &a, launches);
    }
    if (n->op == CO_GRAPH_LINEAR) {
        b2k_linear a = linear_desc(g, id, fuse);
        return launch_linear(g, id, &a, launches);
    }
    if (b2h_fault(B2_FAULT_LAUNCH)) return ROCKET_E_DEVICE;
    int rc;
    if (n->op == CO_GRAPH_RMSNORM) {
        rc = b2d_rmsnorm(d, t->rows, t->cols, tensor_ptr(g, n->a), g->ld[n->a], g->gamma[id], n->epsilon,
                         tensor_ptr(g, id), g->ld[id]);
    } else {
        int op = n->op == CO_GRAPH_ADD ? B2D_EW_ADD : n->op == CO_GRAPH_MUL ? B2D_EW_MUL
               : n->op == CO_GRAPH_SILU ? B2D_EW_SILU : n->op == CO_GRAPH_GELU ? B2D_EW_GELU : B2D_EW_HSIG;
        const int bin = binary(n->op);
        rc = b2d_elementwise(d, op, t->rows, t->cols, tensor_ptr(g, n->a), g->ld[n->a],
                             bin ? tensor_ptr(g, n->b) : NULL, bin ? g->ld[n->b] : 0, tensor_ptr(g, id), g->ld[id]);
    }
    if (!rc) *launches += 1;
    return rc;
}

/* Every node in plan order, then the guard check of every slot. */
static int exec_program(co_graph *g, unsigned *launches) {
    for (unsigned step = 0; step < g->plan.steps; step++) {
        int rc = exec_node(g, g->plan.order[step], launches);
        if (rc) return rc;
    }
    size_t payload[MAXN];
    for (unsigned s = 0; s < g->plan.slots; s++) payload[s] = g->plan.slot_bytes[s];
    if (b2h_fault(B2_FAULT_LAUNCH)) return ROCKET_E_DEVICE;
    int rc = b2d_guard_check(b2h_dev(g->fd), g->slot, payload, g->plan.slots, CO_SLACK, CO_GUARD);
    if (rc) return rc;
    *launches += 1;
    /* every output must be finite before any is published (co_graph.c:366-367) */
    for (unsigned i = 0; i < g->plan.noutputs; i++) {
        unsigned id = g->plan.outputs[i];
        const co_graph_tensor_plan *t = &g->plan.tensors[id];
        if (b2h_fault(B2_FAULT_LAUNCH)) return ROCKET_E_DEVICE;
        rc = b2d_scan_nonfinite(b2h_dev(g->fd), tensor_ptr(g, id), t->rows, t->cols, g->ld[id], B2D_ST_SCAN_OUTPUT);
        if (rc) return rc;
        *launches += 1;
    }
    return 0;
}

/* One run of the program on the handle's stream: the recorded CUDA graph in CO_CHAIN (recorded at
 * the first run; where recording is unavailable the launches are issued directly). */
static int launch_program(co_graph *g, unsigned *launches) {
    b2_dev *d = b2h_dev(g->fd);
    *launches = 0;
    if (g->mode == CO_CHAIN && !g->exec && !g->no_capture) {
        int rc = b2d_capture_begin(d);
        if (rc == ROCKET_E_UNSUPPORTED) {
            g->no_capture = 1;
        } else if (rc) {
            return rc;
        } else {
            unsigned recorded = 0, kernels = 0;
            rc = exec_program(g, &recorded);
            b2_exec *x = NULL;
            int end = b2d_capture_end(d, &x, &kernels);
            if (rc || end) {
                b2d_exec_destroy(x);
                return rc ? rc : end;
            }
            g->exec = x;
            g->kernels = recorded;
        }
    }
    if (g->exec) {
        if (b2h_fault(B2_FAULT_LAUNCH)) return ROCKET_E_DEVICE;
        int rc = b2d_exec_launch(d, g->exec);
        if (!rc) *launches = g->kernels;
        return rc;
    }
    return exec_program(g, launches);
}

static int status_rc(uint32_t st) {
    if (st & (B2_STATUS_TIMEOUT | B2_STATUS_GUARD)) return ROCKET_E_DEVICE;
    if (st & B2_STATUS_NONFINITE_INPUT) return ROCKET_E_SHAPE;
    if (st & B2D_ST_SCAN_OUTPUT) return ROCKET_E_DEVICE;
    return 0;   /* an FP16 overflow inside the graph matters only where it reaches an output */
}

static void count_run(const co_graph *g, unsigned launches) {
    b2h_count_run(g->mode == CO_CHAIN ? g->plan.chain_submits : g->plan.tasks, g->plan.tasks, launches);
}

/* reference co_graph.c:315-376 */
int co_graph_run_many(co_graph *g, const co_graph_input *inputs, unsigned count, const co_graph_output *outputs,
                      unsigned noutputs) {
    if (!g || !inputs || !outputs || count != g->plan.inputs || noutputs != g->plan.noutputs) return ROCKET_E_SHAPE;
    _Float16 *targets[MAXN] = {0};
    for (unsigned i = 0; i < noutputs; i++) {
        unsigned id = outputs[i].node;
        int found = 0;
        for (unsigned j = 0; j < g->plan.noutputs; j++)
            if (id == g->plan.outputs[j]) found = 1;
        if (!found || !outputs[i].data || targets[id]) return ROCKET_E_SHAPE;
        size_t bytes = (size_t)g->plan.tensors[id].rows * g->plan.tensors[id].cols * 2;
        uintptr_t a = (uintptr_t)outputs[i].data;
        if (a > UINTPTR_MAX - bytes) return ROCKET_E_SHAPE;
        for (unsigned j = 0; j < i; j++) {
            const co_graph_tensor_plan *t = &g->plan.tensors[outputs[j].node];
            size_t bb = (size_t)t->rows * t->cols * 2;
            uintptr_t b = (uintptr_t)outputs[j].data;
            if (a < b + bb && b < a + bytes) return ROCKET_E_SHAPE;
        }
        targets[id] = outputs[i].data;
    }
    const _Float16 *bindings[MAXN] = {0};
    for (unsigned i = 0; i < count; i++) {
        unsigned id = inputs[i].node;
        if (id >= g->count || g->nodes[id].op != CO_GRAPH_INPUT || !g->ld[id] || bindings[id] || !inputs[i].data ||
            !finite16(inputs[i].data, (size_t)g->plan.tensors[id].rows * g->plan.tensors[id].cols))
            return ROCKET_E_SHAPE;
        bindings[id] = inputs[i].data;
    }
    b2_dev *d = b2h_dev(g->fd);
    if (!d) return ROCKET_E_SHAPE;
    int rc = b2d_sync(d);
    if (rc) return rc;
    uint32_t prior = b2d_status(d, 1);
    for (unsigned i = 0; i < count && !rc; i++) {
        unsigned id = inputs[i].node;
        const co_graph_tensor_plan *t = &g->plan.tensors[id];
        rc = b2d_copy_2d(d, tensor_ptr(g, id), g->ld[id] * 2, inputs[i].data, (size_t)t->cols * 2,
                         (size_t)t->cols * 2, t->rows, B2D_H2D);
    }
    unsigned launches = 0;
    if (!rc) rc = launch_program(g, &launches);
    int sync_rc = b2d_sync(d);
    if (!rc) rc = sync_rc;
    uint32_t st = b2d_status(d, 1);
    b2d_status_merge(d, prior);
    if (!rc && b2h_fault(B2_FAULT_NAN_OUTPUT)) st |= B2D_ST_SCAN_OUTPUT;
    if (!rc) rc = status_rc(st);
    /* the run succeeded and every output is finite: publish them */
    for (unsigned i = 0; i < g->plan.noutputs && !rc; i++) {
        unsigned id = g->plan.outputs[i];
        const co_graph_tensor_plan *t = &g->plan.tensors[id];
        rc = b2d_copy_2d(d, targets[id], (size_t)t->cols * 2, tensor_ptr(g, id), g->ld[id] * 2, (size_t)t->cols * 2,
                         t->rows, B2D_D2H);
    }
    if (!rc) rc = b2d_sync(d);
    if (launches) count_run(g, launches);
    return rc;
}

int co_graph_run(co_graph *g, const co_graph_input *inputs, unsigned count, _Float16 *out) {
    if (!g || g->plan.noutputs != 1) return ROCKET_E_SHAPE;
    co_graph_output output = {g->plan.outputs[0], out};
    return co_graph_run_many(g, inputs, count, &output, 1);
}

/* ------------------------------------------------------------------------------ B200 entries */
int b2_graph_tensor(const co_graph *g, unsigned node, void **ptr, size_t *ld) {
    if (!g || !ptr || !ld || node >= g->count || !g->ld[node]) return ROCKET_E_SHAPE;
    *ptr = tensor_ptr(g, node);
    *ld = g->ld[node];
    return 0;
}

int b2_graph_launch(co_graph *g) {
    if (!g || !b2h_dev(g->fd)) return ROCKET_E_SHAPE;
    unsigned launches = 0;
    int rc = launch_program(g, &launches);
    if (launches) count_run(g, launches);
    return rc;
}

int b2_graph_status(co_graph *g) {
    if (!g || !b2h_dev(g->fd)) return ROCKET_E_SHAPE;
    return status_rc(b2d_status(b2h_dev(g->fd), 1));
}

int b2_graph_get_info(const co_graph *g, b2_graph_info *info) {
    if (!g || !info) return ROCKET_E_SHAPE;
    memset(info, 0, sizeof(*info));
    if (g->mode == CO_CHAIN) {
        info->gated = g->f.ngated;
        info->residual = g->f.nresidual;
    }
    info->kernels = g->kernels;
    info->captured = g->exec != NULL;
    return 0;
}
