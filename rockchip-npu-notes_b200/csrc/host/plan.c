/* plan.c -- deterministic shape decomposition and HBM budget preflight.
 *
 * Restates research/custom-ops/src/linear_plan.c (reference project):
 *   co_linear_plan_init_ex  :10-46  validation, M/N/K tile counts, row classes, task and
 *                                   chain-submit accounting, budget check
 *   co_linear_plan_tile     :48-62  geometry of output tile `index` (M-major, N-minor)
 *   co_linear_plan_init     :64-66  HardSigmoid with bias
 * The tile counts, task formula (per output tile: ceil(K/256) + has_bias + LUT chunks, where a
 * LUT task covers at most 32768 physical elements), row classes and chain-submit count are the
 * reference's: they are the contract its file gate checks. device_bytes differs by design: it is
 * the HBM this B200 context allocates (resident FP16 weights with a 16-byte row pitch, bias, and
 * the row-major X/Y staging used by the host entry), and the budget is checked against it.
 *
 * The GPU's own schedule (CTA tiles over the 148 SMs) is chosen per launch by the CUDA layer;
 * the 256x256 plan tiles here are only the reference's accounting unit.
 */
#include "b2_host.h"

#include <string.h>

static unsigned extent(unsigned total, unsigned i) {
    unsigned left = total - i * 256u;
    return left > 256u ? 256u : left;
}

static unsigned lut_chunks(unsigned rows, unsigned cols) {
    unsigned pr = (rows < 12 ? 12 : rows + 3) / 4 * 4, pc = (cols + 31) / 32 * 32;
    return (unsigned)(((size_t)pr * pc + 32767) / 32768);
}

/* HBM held by a context for (m, k, n): FP16 W[n, k8] + bias[n] + X[m, k8] + Y[m, n8]. */
size_t b2h_context_bytes(unsigned m, unsigned k, unsigned n, int has_bias) {
    size_t k8 = b2h_round_up(k, 8), n8 = b2h_round_up(n, 8);
    return (size_t)n * k8 * 2 + (has_bias ? (size_t)n * 2 : 0) + (size_t)m * k8 * 2 +
           (size_t)m * n8 * 2;
}

int b2h_plan(co_linear_plan *out, unsigned m, unsigned k, unsigned n, int has_bias,
             enum co_linear_post post, size_t budget, unsigned max_dim, int compat) {
    if (!out) return ROCKET_E_SHAPE;
    memset(out, 0, sizeof(*out));
    unsigned max_m = compat ? CO_MAX_M : max_dim, max_k = compat ? CO_MAX_K : max_dim,
             max_n = compat ? CO_MAX_N : max_dim;
    if ((has_bias != 0 && has_bias != 1) || (post != CO_LINEAR_NONE && post != CO_LINEAR_HSIG) ||
        !m || m > max_m || !k || k > max_k || !n || n > max_n)
        return ROCKET_E_SHAPE;
    co_linear_plan p = {.m = m, .k = k, .n = n, .mtiles = (m + 255) / 256, .ktiles = co_k_tiles(k),
                        .ntiles = (n + 255) / 256, .has_bias = (unsigned)has_bias,
                        .post = (unsigned)post};
    p.output_tiles = p.mtiles * p.ntiles;
    p.row_classes = (p.mtiles > 1 && m % 256) ? 2 : 1;
    p.chain_submits = p.output_tiles;
    /* Tiles fall in at most four shape classes (full/tail rows x full/tail cols). */
    unsigned row_ext[2] = {m >= 256 ? 256u : m, m % 256}, col_ext[2] = {n >= 256 ? 256u : n, n % 256};
    unsigned long long row_cnt[2] = {m >= 256 ? m / 256 : 1, m >= 256 && m % 256 ? 1 : 0};
    unsigned long long col_cnt[2] = {n >= 256 ? n / 256 : 1, n >= 256 && n % 256 ? 1 : 0};
    for (int a = 0; a < 2; a++)
        for (int b = 0; b < 2; b++) {
            if (!row_cnt[a] || !col_cnt[b]) continue;
            unsigned programs = p.ktiles + (unsigned)has_bias +
                                (post == CO_LINEAR_HSIG ? lut_chunks(row_ext[a], col_ext[b]) : 0);
            if (compat && programs > CO_MAX_PROGRAMS) return ROCKET_E_TILING;
            p.tasks += row_cnt[a] * col_cnt[b] * programs;
        }
    p.device_bytes = b2h_context_bytes(m, k, n, has_bias);
    if (p.device_bytes > (budget ? budget : CO_LINEAR_DEVICE_BUDGET)) return ROCKET_E_TILING;
    *out = p;
    return 0;
}

int co_linear_plan_init_ex(co_linear_plan *out, unsigned m, unsigned k, unsigned n, int has_bias,
                           enum co_linear_post post, size_t budget) {
    return b2h_plan(out, m, k, n, has_bias, post, budget, CO_MAX_K, 1);
}

int co_linear_plan_tile(const co_linear_plan *p, unsigned index, co_linear_tile_info *out) {
    if (!p || !out) return ROCKET_E_SHAPE;
    co_linear_plan canonical;
    if (co_linear_plan_init_ex(&canonical, p->m, p->k, p->n, (int)p->has_bias,
                               (enum co_linear_post)p->post, SIZE_MAX) ||
        p->mtiles != canonical.mtiles || p->ntiles != canonical.ntiles ||
        p->ktiles != canonical.ktiles || p->output_tiles != canonical.output_tiles ||
        index >= canonical.output_tiles)
        return ROCKET_E_SHAPE;
    unsigned mi = index / p->ntiles, ni = index % p->ntiles;
    unsigned rows = extent(p->m, mi), cols = extent(p->n, ni);
    *out = (co_linear_tile_info){mi * 256, ni * 256, rows, cols, p->ktiles,
                                 p->ktiles + p->has_bias +
                                     (p->post == CO_LINEAR_HSIG ? lut_chunks(rows, cols) : 0)};
    return 0;
}

int co_linear_plan_init(co_linear_plan *out, unsigned m, unsigned k, unsigned n, size_t budget) {
    return co_linear_plan_init_ex(out, m, k, n, 1, CO_LINEAR_HSIG, budget);
}

/* ------------------------------------------------------------------------------ GPU shards */
int b2_shard_range(unsigned long long total, unsigned parts, unsigned index, unsigned align,
                   unsigned long long *begin, unsigned long long *end) {
    if (!begin || !end || !parts || index >= parts || !align) return ROCKET_E_SHAPE;
    const unsigned long long blocks = (total + align - 1) / align;
    const unsigned long long base = blocks / parts, extra = blocks % parts;
    const unsigned long long b0 = index * base + (index < extra ? index : extra);
    const unsigned long long nb = base + (index < extra ? 1 : 0);
    unsigned long long lo = b0 * align, hi = (b0 + nb) * align;
    if (lo > total) lo = total;
    if (hi > total) hi = total;
    *begin = lo;
    *end = hi;
    return 0;
}
