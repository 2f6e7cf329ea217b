/* linear.c -- the Linear / HardSigmoid operator context and its entry points.
 *
 * Restates the public behaviour of research/custom-ops/src/linear_hardsigmoid.c (reference):
 *   co_linear_create            :219-252  argument order of checks, plan, finite W/b, copy-in
 *   co_linear_hsig_run          :254-275  host entry; result published only if the run succeeded
 *   co_linear_hsig_run_tiles    :285-306  device-cube collection entry; every view and alias is
 *                                         validated before the first launch
 *   co_linear_hsig_run_cube     :308-312  single-tile cube entry (else ROCKET_E_UNSUPPORTED)
 *   co_linear_hsig_create       :314-319  bias required
 *   co_linear_run_tiled         :325-352  per-K-tile input cubes
 *   co_linear_update_weights    :354-364  W/b refresh, bias presence fixed
 *   co_linear_hsig_destroy      :212-217
 * B200 design instead of per-output-tile contexts and chained submits: one context per operator
 * holding FP16 W row-major in HBM (16-byte row pitch, ready for TMA), the FP16 bias, and
 * row-major X/Y staging. A run is: pitched H2D of X, a finiteness scan of X, one persistent
 * tcgen05 GEMM with the fused bias/HardSigmoid epilogue (CO_CHAIN) or GEMM + separate epilogue
 * kernel (CO_SEPARATE), a status check, and a pitched D2H of Y -- all on one CUDA stream.
 */
#include "b2_host.h"

#include <stdlib.h>
#include <string.h>

struct co_linear_hsig {
    int fd;
    int compat;                     /* created through co_* (reference limits) */
    co_linear_plan plan;
    enum co_linear_post post;
    enum co_mode mode;
    enum b2_accumulate acc;
    void *w; size_t ldw;            /* FP16 [n, ldw] */
    void *bias;                     /* FP16 [n] or NULL */
    void *x; size_t ldx;            /* FP16 staging [m, ldx] */
    void *y; size_t ldy;            /* FP16 staging [m, ldy] */
    float *ws; size_t ws_bytes;     /* FP32 workspace, separate mode with FP32 accumulation */
    void *y_stage;                  /* pinned host copy of Y for small outputs (host runs), or NULL */
    size_t bytes;                   /* HBM held, excluding the lazily sized workspace */
};

static int finite_host(const _Float16 *v, size_t n) {
    if (!v) return 0;
    const uint16_t *b = (const uint16_t *)v;
    for (size_t i = 0; i < n; i++)
        if ((b[i] & 0x7c00u) == 0x7c00u) return 0;
    return 1;
}

static int status_rc(uint32_t st, int check_output) {
    if (st & B2_STATUS_TIMEOUT) return ROCKET_E_DEVICE;
    if (st & B2_STATUS_GUARD) return ROCKET_E_DEVICE;
    if (st & B2_STATUS_NONFINITE_INPUT) return ROCKET_E_SHAPE;
    if (check_output && (st & B2_STATUS_NONFINITE_OUTPUT)) return ROCKET_E_DEVICE;
    return 0;
}

void co_linear_hsig_destroy(co_linear_hsig *c) {
    if (!c) return;
    b2h_free(c->fd, c->w, (size_t)c->plan.n * c->ldw * 2);
    b2h_free(c->fd, c->bias, (size_t)c->plan.n * 2);
    b2h_free(c->fd, c->x, (size_t)c->plan.m * c->ldx * 2);
    b2h_free(c->fd, c->y, (size_t)c->plan.m * c->ldy * 2);
    b2h_free(c->fd, c->ws, c->ws_bytes);
    b2d_host_free(c->y_stage);
    free(c);
}
void co_linear_destroy(co_linear *c) { co_linear_hsig_destroy(c); }

/* Host runs whose Y is at most this many bytes copy it into pinned staging right behind the
 * kernels, sync once, check the status and then copy it to the caller's Y on the host: one
 * stream synchronisation fewer than copying into Y after the check. */
#define Y_STAGE_MAX ((size_t)64 << 10)

static int upload_weights(co_linear_hsig *c, const _Float16 *w, const _Float16 *b) {
    b2_dev *d = b2h_dev(c->fd);
    unsigned k = c->plan.k, n = c->plan.n;
    int rc = b2d_copy_2d(d, c->w, c->ldw * 2, w, (size_t)k * 2, (size_t)k * 2, n, B2D_H2D);
    if (!rc && b) rc = b2d_copy_2d(d, c->bias, (size_t)n * 2, b, (size_t)n * 2, (size_t)n * 2, 1, B2D_H2D);
    if (!rc) rc = b2d_sync(d);
    return rc;
}

static int create_impl(int fd, unsigned m, unsigned k, unsigned n, const _Float16 *w,
                       const _Float16 *b, enum co_linear_post post, enum co_mode mode,
                       enum b2_accumulate acc, int compat, co_linear **out) {
    if (!out) return ROCKET_E_SHAPE;
    *out = NULL;
    if (fd < 0 || !b2h_valid_fd(fd) || (mode != CO_CHAIN && mode != CO_SEPARATE) ||
        (acc != B2_ACC_TILE16 && acc != B2_ACC_FP32))
        return ROCKET_E_SHAPE;
    co_linear_plan plan;
    int rc = b2h_plan(&plan, m, k, n, b != NULL, post, compat ? 0 : SIZE_MAX, B2_MAX_DIM, compat);
    if (rc) return rc;
    if (!finite_host(w, (size_t)n * k) || (b && !finite_host(b, n))) return ROCKET_E_SHAPE;
    if (mode == CO_CHAIN && !rocket_batched_submit_supported()) return ROCKET_E_UNSUPPORTED;
    co_linear_hsig *c = calloc(1, sizeof(*c));
    if (!c) return ROCKET_E_NOMEM;
    c->fd = fd;
    c->compat = compat;
    c->plan = plan;
    c->post = post;
    c->mode = mode;
    c->acc = acc;
    c->ldw = c->ldx = b2h_round_up(k, 8);
    c->ldy = b2h_round_up(n, 8);
    if ((rc = b2h_malloc(fd, (size_t)n * c->ldw * 2, &c->w)) ||
        (b && (rc = b2h_malloc(fd, (size_t)n * 2, &c->bias))) ||
        (rc = b2h_malloc(fd, (size_t)m * c->ldx * 2, &c->x)) ||
        (rc = b2h_malloc(fd, (size_t)m * c->ldy * 2, &c->y)) ||
        (rc = upload_weights(c, w, b))) {
        /* members not yet allocated are NULL and free as no-ops; sizes come from the plan */
        co_linear_hsig_destroy(c);
        return rc;
    }
    c->bytes = plan.device_bytes;
    if ((size_t)m * n * 2 <= Y_STAGE_MAX) c->y_stage = b2d_host_alloc((size_t)m * n * 2);   /* NULL: direct copy */
    *out = c;
    return 0;
}

int co_linear_create(int fd, unsigned m, unsigned k, unsigned n, const _Float16 *weights,
                     const _Float16 *bias, enum co_linear_post post, enum co_mode mode,
                     co_linear **out) {
    return create_impl(fd, m, k, n, weights, bias, post, mode, B2_ACC_TILE16, 1, out);
}

int co_linear_hsig_create(int fd, unsigned m, unsigned k, unsigned n, const _Float16 *w,
                          const _Float16 *b, enum co_mode mode, co_linear_hsig **out) {
    if (!b) {
        if (out) *out = NULL;
        return ROCKET_E_SHAPE;
    }
    return co_linear_create(fd, m, k, n, w, b, CO_LINEAR_HSIG, mode, out);
}

int b2_linear_create(int fd, unsigned m, unsigned k, unsigned n, const _Float16 *weights,
                     const _Float16 *bias, enum co_linear_post post, enum co_mode mode,
                     enum b2_accumulate acc, b2_linear **out) {
    return create_impl(fd, m, k, n, weights, bias, post, mode, acc, 0, out);
}

int b2_linear_set_accumulate(b2_linear *c, enum b2_accumulate acc) {
    if (!c || (acc != B2_ACC_TILE16 && acc != B2_ACC_FP32)) return ROCKET_E_SHAPE;
    c->acc = acc;
    return 0;
}

/* FP32 workspace for the separate (unfused) epilogue under FP32 accumulation. */
static size_t ws_ld(const co_linear_hsig *c) { return b2h_round_up(c->plan.n, 4); }

static int ensure_ws(co_linear_hsig *c, unsigned m) {
    size_t need = (size_t)m * ws_ld(c) * 4;
    if (c->ws_bytes >= need) return 0;
    b2h_free(c->fd, c->ws, c->ws_bytes);
    c->ws = NULL;
    c->ws_bytes = 0;
    void *p = NULL;
    int rc = b2h_malloc(c->fd, need, &p);
    if (rc) return rc;
    c->ws = p;
    c->ws_bytes = need;
    return 0;
}

static int launch_linear(co_linear_hsig *c, unsigned m, const void *x, size_t ldx, void *y,
                         size_t ldy, unsigned *launches) {
    *launches = 0;
    b2k_linear a = {.m = m, .n = c->plan.n, .k = c->plan.k, .x = x, .ldx = ldx, .w = c->w,
                    .ldw = c->ldw, .bias = c->bias, .y = y, .ldy = ldy,
                    .post = c->post == CO_LINEAR_HSIG, .acc = (int)c->acc,
                    .fused = c->mode == CO_CHAIN, .raw_only = 0};
    if (!a.fused && c->acc == B2_ACC_FP32) {
        int rc = ensure_ws(c, m);
        if (rc) return rc;
        a.partial = c->ws;
        a.ldp = ws_ld(c);
    }
    if (b2h_fault(B2_FAULT_LAUNCH)) return ROCKET_E_DEVICE;
    return b2d_linear(b2h_dev(c->fd), &a, launches);
}

static void count_run(const co_linear_hsig *c, unsigned launches) {
    b2h_count_run(c->mode == CO_CHAIN ? c->plan.chain_submits : c->plan.tasks, c->plan.tasks,
                  launches);
}

/* Row bands of a host-buffer run. X of 8 MiB or more and at least 1024 rows (fused form) is copied
 * in up to B2D_SIDE_EVENTS bands of at least 512 rows on the side stream, and each band's scan and
 * GEMM start once its rows have landed, so only the last band's kernels follow the copy (4096^3 from
 * pinned buffers: 1.35-1.37 -> 1.29-1.31 ms per call; at 4 MiB of X the bands measured 1 % slower).
 * Every output element is computed from the same operands in the same order either way; Y still
 * leaves the device only after the status check. */
static unsigned host_bands(const co_linear_hsig *c) {
    const unsigned m = c->plan.m;
    if (c->mode != CO_CHAIN || m < 1024 || (size_t)m * c->plan.k * 2 < ((size_t)8 << 20)) return 1;
    return m / 512 < B2D_SIDE_EVENTS ? m / 512 : B2D_SIDE_EVENTS;
}

int co_linear_hsig_run(co_linear_hsig *c, const _Float16 *x, _Float16 *y) {
    if (!c || !y || !x) return ROCKET_E_SHAPE;
    b2_dev *d = b2h_dev(c->fd);
    if (!d) return ROCKET_E_SHAPE;
    unsigned m = c->plan.m, k = c->plan.k, n = c->plan.n, launches = 0, l = 0;
    int rc = b2d_sync(d);
    if (rc) return rc;
    uint32_t prior = b2d_status(d, 1);
    const unsigned bands = host_bands(c);
    if (bands == 1) {
        rc = b2d_copy_2d(d, c->x, c->ldx * 2, x, (size_t)k * 2, (size_t)k * 2, m, B2D_H2D);
        if (!rc) {
            rc = b2d_scan_nonfinite(d, c->x, m, k, c->ldx, B2_STATUS_NONFINITE_INPUT);
            launches += !rc;
        }
        if (!rc) {
            rc = launch_linear(c, m, c->x, c->ldx, c->y, c->ldy, &l);
            launches += l;
        }
    } else {
        /* band i: rows [m * i / bands, m * (i + 1) / bands) rounded down to multiples of 128 */
        unsigned r[B2D_SIDE_EVENTS + 1];
        for (unsigned i = 0; i <= bands; i++) r[i] = i == bands ? m : (unsigned)((size_t)m * i / bands) & ~127u;
        unsigned issued = 0;
        for (unsigned i = 0; !rc && i < bands; i++) {
            rc = b2d_copy_side(d, (_Float16 *)c->x + (size_t)r[i] * c->ldx, c->ldx * 2, x + (size_t)r[i] * k, (size_t)k * 2,
                               (size_t)k * 2, r[i + 1] - r[i], B2D_H2D, i);
            if (!rc) issued = i + 1;
        }
        /* the handle's stream waits for every band that was issued, also after an error, so that the
         * sync below covers the copies still reading the caller's X */
        for (unsigned i = 0; i < issued; i++) {
            const _Float16 *xb = (const _Float16 *)c->x + (size_t)r[i] * c->ldx;
            const int wrc = b2d_wait_side(d, i);
            if (!rc) rc = wrc;
            if (!rc) {
                rc = b2d_scan_nonfinite(d, xb, r[i + 1] - r[i], k, c->ldx, B2_STATUS_NONFINITE_INPUT);
                launches += !rc;
            }
            if (!rc) {
                rc = launch_linear(c, r[i + 1] - r[i], xb, c->ldx, (_Float16 *)c->y + (size_t)r[i] * c->ldy, c->ldy, &l);
                launches += l;
            }
        }
    }
    if (!rc && c->y_stage) rc = b2d_copy_2d(d, c->y_stage, (size_t)n * 2, c->y, c->ldy * 2, (size_t)n * 2, m, B2D_D2H);
    int sync_rc = b2d_sync(d);
    if (!rc) rc = sync_rc;
    uint32_t st = b2d_status(d, 1);
    b2d_status_merge(d, prior);
    if (!rc && b2h_fault(B2_FAULT_NAN_OUTPUT)) st |= B2_STATUS_NONFINITE_OUTPUT;
    if (!rc) rc = status_rc(st, 1);
    if (!rc && c->y_stage) {
        memcpy(y, c->y_stage, (size_t)m * n * 2);
    } else if (!rc) {
        rc = b2d_copy_2d(d, y, (size_t)n * 2, c->y, c->ldy * 2, (size_t)n * 2, m, B2D_D2H);
        if (!rc) rc = b2d_sync(d);
    }
    if (launches) count_run(c, launches);
    return rc;
}

int co_linear_run(co_linear *c, const _Float16 *x, _Float16 *y) { return co_linear_hsig_run(c, x, y); }

/* ------------------------------------------------------------------------------ cube entries */
static void *view_ptr(const co_view *v) { return (char *)v->buffer->bo.ptr + v->offset; }

static int compatible(const co_view *v, const co_tensor *want, int fd) {
    co_view checked;
    const co_tensor *a = &v->tensor;
    return v->buffer && !co_view_init(&checked, v->buffer, v->offset, a) && v->buffer->fd == fd &&
           a->type == want->type && a->layout == want->layout && a->rows == want->rows &&
           a->cols == want->cols && a->physical_rows == want->physical_rows &&
           a->physical_cols == want->physical_cols && a->atom == want->atom &&
           a->bytes == want->bytes;
}

/* Aliasing rule of the cube entries: no output view may share a byte with an input view or another
 * output view (inputs may share bytes with each other); address ranges are compared, so separate
 * co_buffer wrappers of one allocation are caught too. The ranges are sorted by start and swept
 * once, keeping the furthest end of every range and of the output ranges seen so far: a range
 * overlaps an earlier one exactly when it starts before that earlier range's end. */
typedef struct {
    uintptr_t start, end;
    int output;
} view_range;

static int by_start(const void *a, const void *b) {
    uintptr_t x = ((const view_range *)a)->start, y = ((const view_range *)b)->start;
    return x < y ? -1 : x > y;
}

static int outputs_alias(const co_view *x, unsigned nx, const co_view *y, unsigned ny, int *nomem) {
    view_range *r = malloc(sizeof(*r) * (nx + ny));
    *nomem = !r;
    if (!r) return 0;
    for (unsigned i = 0; i < nx + ny; i++) {
        const co_view *v = i < nx ? &x[i] : &y[i - nx];
        r[i].start = (uintptr_t)view_ptr(v);
        r[i].end = r[i].start + v->tensor.bytes;
        r[i].output = i >= nx;
    }
    qsort(r, nx + ny, sizeof(*r), by_start);
    uintptr_t end_all = 0, end_out = 0;
    int alias = 0;
    for (unsigned i = 0; i < nx + ny && !alias; i++) {
        alias = r[i].start < (r[i].output ? end_all : end_out);
        if (r[i].end > end_all) end_all = r[i].end;
        if (r[i].output && r[i].end > end_out) end_out = r[i].end;
    }
    free(r);
    return alias;
}

static unsigned tile_extent(unsigned total, unsigned i) {
    unsigned left = total - i * 256u;
    return left > 256u ? 256u : left;
}

static b2k_cube_tile cube_tile(const co_view *v, unsigned row0, unsigned col0) {
    b2k_cube_tile t = {view_ptr(v), v->tensor.rows, v->tensor.cols, v->tensor.physical_rows,
                       v->tensor.physical_cols, row0, col0};
    return t;
}

static int gather(b2_dev *d, const b2k_cube_tile *t, unsigned count, void *dst, size_t ld,
                  unsigned *launches) {
    for (unsigned i = 0; i < count; i += B2K_MAX_CUBE_TILES) {
        unsigned c = count - i < B2K_MAX_CUBE_TILES ? count - i : B2K_MAX_CUBE_TILES;
        int rc = b2d_cube_to_rowmajor(d, t + i, c, dst, ld);
        if (rc) return rc;
        ++*launches;
    }
    return 0;
}

static int scatter(b2_dev *d, const void *src, size_t ld, const b2k_cube_tile *t, unsigned count,
                   unsigned *launches) {
    for (unsigned i = 0; i < count; i += B2K_MAX_CUBE_TILES) {
        unsigned c = count - i < B2K_MAX_CUBE_TILES ? count - i : B2K_MAX_CUBE_TILES;
        int rc = b2d_rowmajor_to_cube(d, src, ld, t + i, c);
        if (rc) return rc;
        ++*launches;
    }
    return 0;
}

/* Guard check of every distinct caller buffer, batched. */
static int guard_views(b2_dev *d, const co_view *a, unsigned na, const co_view *b, unsigned nb,
                       unsigned *launches) {
    void *bases[B2K_MAX_CUBE_TILES];
    size_t payloads[B2K_MAX_CUBE_TILES];
    unsigned cnt = 0;
    for (unsigned i = 0; i < na + nb; i++) {
        const co_buffer *buf = i < na ? a[i].buffer : b[i - na].buffer;
        int seen = 0;
        for (unsigned j = 0; j < cnt && !seen; j++) seen = bases[j] == buf->bo.ptr;
        if (seen) continue;
        bases[cnt] = buf->bo.ptr;
        payloads[cnt++] = buf->payload;
        if (cnt == B2K_MAX_CUBE_TILES) {
            int rc = b2d_guard_check(d, bases, payloads, cnt, CO_SLACK, CO_GUARD);
            if (rc) return rc;
            ++*launches;
            cnt = 0;
        }
    }
    if (cnt) {
        int rc = b2d_guard_check(d, bases, payloads, cnt, CO_SLACK, CO_GUARD);
        if (rc) return rc;
        ++*launches;
    }
    return 0;
}

/* Shared tail of the cube entries: the GEMM straight from the input cubes into the output cubes
 * (b2d_linear_cube) where the operator and the views allow it, else gather -> GEMM -> scatter; then
 * the guard check and the status. in[] holds kviews views per 256-row band, each kview_k columns. */
static int run_cube_tiles(co_linear_hsig *c, const b2k_cube_tile *in, unsigned nin, unsigned kviews,
                          unsigned kview_k, const b2k_cube_tile *out, unsigned nout, const co_view *xv,
                          unsigned nx, const co_view *yv, unsigned ny) {
    b2_dev *d = b2h_dev(c->fd);
    unsigned launches = 0, l = 0;
    int rc = b2d_sync(d);
    if (rc) return rc;
    uint32_t prior = b2d_status(d, 1);
    /* direct: the fused arm of a GEMM-sized operator, every input view a whole number of 8-channel
     * atoms (a partial atom's unused channels would be read as data) */
    int direct = c->mode == CO_CHAIN && c->plan.m > B2D_GEMV_MAX_M && nin <= B2D_CUBE_MAX_VIEWS &&
                 nout <= B2D_CUBE_MAX_VIEWS;
    for (unsigned i = 0; direct && i < nin; i++) direct = in[i].cols % 8 == 0;
    int fallback = !direct;
    if (direct) {
        if (b2h_fault(B2_FAULT_LAUNCH)) {
            rc = ROCKET_E_DEVICE;
        } else {
            b2k_linear a = {.m = c->plan.m, .n = c->plan.n, .k = c->plan.k, .w = c->w, .ldw = c->ldw,
                            .bias = c->bias, .post = c->post == CO_LINEAR_HSIG, .acc = (int)c->acc,
                            .fused = 1};
            b2k_cube_io io = {in, nin, kviews, kview_k, out, nout, c->plan.ntiles};
            rc = b2d_linear_cube(d, &a, &io, &l);
            launches += l;
            fallback = rc == ROCKET_E_UNSUPPORTED;
            if (fallback) rc = 0;
        }
    }
    if (fallback) {
        rc = gather(d, in, nin, c->x, c->ldx, &launches);
        if (!rc) {
            rc = launch_linear(c, c->plan.m, c->x, c->ldx, c->y, c->ldy, &l);
            launches += l;
        }
        if (!rc) rc = scatter(d, c->y, c->ldy, out, nout, &launches);
    }
    if (!rc) rc = guard_views(d, xv, nx, yv, ny, &launches);
    int sync_rc = b2d_sync(d);
    if (!rc) rc = sync_rc;
    uint32_t st = b2d_status(d, 1);
    b2d_status_merge(d, prior);
    if (!rc) rc = status_rc(st, 0);   /* cube entries do not read or score the tensor payload */
    if (launches) count_run(c, launches);
    return rc;
}

int co_linear_hsig_run_tiles(co_linear_hsig *c, const co_view *x, unsigned nx, const co_view *y,
                             unsigned ny) {
    if (!c || !x || !y || nx != c->plan.mtiles || ny != c->plan.output_tiles) return ROCKET_E_SHAPE;
    const unsigned k = c->plan.k, nt = c->plan.ntiles;
    for (unsigned mi = 0; mi < nx; mi++) {
        co_tensor want;
        if (co_tensor_input(&want, tile_extent(c->plan.m, mi), k) || !compatible(&x[mi], &want, c->fd))
            return ROCKET_E_SHAPE;
    }
    for (unsigned i = 0; i < ny; i++) {
        co_tensor want;
        if (co_tensor_matrix(&want, tile_extent(c->plan.m, i / nt), tile_extent(c->plan.n, i % nt), CO_F16) ||
            !compatible(&y[i], &want, c->fd))
            return ROCKET_E_SHAPE;
    }
    int nomem = 0;
    if (outputs_alias(x, nx, y, ny, &nomem)) return ROCKET_E_SHAPE;
    if (nomem) return ROCKET_E_NOMEM;
    b2k_cube_tile *in = malloc(sizeof(*in) * nx), *out = malloc(sizeof(*out) * ny);
    if (!in || !out) { free(in); free(out); return ROCKET_E_NOMEM; }
    for (unsigned mi = 0; mi < nx; mi++) in[mi] = cube_tile(&x[mi], mi * 256, 0);
    for (unsigned i = 0; i < ny; i++) out[i] = cube_tile(&y[i], (i / nt) * 256, (i % nt) * 256);
    int rc = run_cube_tiles(c, in, nx, 1, b2h_round_up(k, 64), out, ny, x, nx, y, ny);
    free(in);
    free(out);
    return rc;
}

int co_linear_hsig_run_cube(co_linear_hsig *c, co_view x, co_view y) {
    if (!c) return ROCKET_E_SHAPE;
    if (c->plan.output_tiles != 1) return ROCKET_E_UNSUPPORTED;
    return co_linear_hsig_run_tiles(c, &x, 1, &y, 1);
}

int co_linear_run_tiled(co_linear *c, const co_view *x, unsigned nx, const co_view *y, unsigned ny) {
    if (!c || !x || !y || nx != c->plan.mtiles * c->plan.ktiles || ny != c->plan.output_tiles)
        return ROCKET_E_SHAPE;
    const unsigned kt = c->plan.ktiles, nt = c->plan.ntiles;
    for (unsigned i = 0; i < nx; i++) {
        co_tensor want;
        if (co_tensor_matrix(&want, tile_extent(c->plan.m, i / kt), co_k_tile_length(c->plan.k, i % kt), CO_F16) ||
            !compatible(&x[i], &want, c->fd))
            return ROCKET_E_SHAPE;
    }
    for (unsigned i = 0; i < ny; i++) {
        co_tensor want;
        if (co_tensor_matrix(&want, tile_extent(c->plan.m, i / nt), tile_extent(c->plan.n, i % nt), CO_F16) ||
            !compatible(&y[i], &want, c->fd))
            return ROCKET_E_SHAPE;
    }
    int nomem = 0;
    if (outputs_alias(x, nx, y, ny, &nomem)) return ROCKET_E_SHAPE;
    if (nomem) return ROCKET_E_NOMEM;
    b2k_cube_tile *in = malloc(sizeof(*in) * nx), *out = malloc(sizeof(*out) * ny);
    if (!in || !out) { free(in); free(out); return ROCKET_E_NOMEM; }
    for (unsigned i = 0; i < nx; i++) in[i] = cube_tile(&x[i], (i / kt) * 256, (i % kt) * CO_K_TILE);
    for (unsigned i = 0; i < ny; i++) out[i] = cube_tile(&y[i], (i / nt) * 256, (i % nt) * 256);
    int rc = run_cube_tiles(c, in, nx, kt, CO_K_TILE, out, ny, x, nx, y, ny);
    free(in);
    free(out);
    return rc;
}

int co_linear_update_weights(co_linear *c, const _Float16 *weights, const _Float16 *bias) {
    if (!c || !finite_host(weights, (size_t)c->plan.n * c->plan.k) ||
        (c->plan.has_bias ? !finite_host(bias, c->plan.n) : bias != NULL))
        return ROCKET_E_SHAPE;
    b2_dev *d = b2h_dev(c->fd);
    int rc = b2d_sync(d);
    if (!rc) rc = upload_weights(c, weights, bias);
    return rc;
}

/* ------------------------------------------------------------------------------ device entries */
static int device_args_ok(const co_linear_hsig *c, unsigned m, const void *x, size_t ldx,
                          const void *y, size_t ldy, int y_is_f32) {
    return c && x && y && m >= 1 && m <= B2_MAX_DIM && b2h_dev(c->fd) &&
           ldx >= c->plan.k && ldx % 8 == 0 && ldy >= c->plan.n && ldy % (y_is_f32 ? 4 : 8) == 0 &&
           ((uintptr_t)x & 15) == 0 && ((uintptr_t)y & 15) == 0;
}

int b2_linear_run_device(b2_linear *c, unsigned m, const void *x, size_t ldx, void *y, size_t ldy) {
    if (!device_args_ok(c, m, x, ldx, y, ldy, 0)) return ROCKET_E_SHAPE;
    unsigned launches = 0;
    int rc = launch_linear(c, m, x, ldx, y, ldy, &launches);
    if (launches) count_run(c, launches);
    return rc;
}

/* Grouped small-M run: every member is finished in its launch (fused form), which for the
 * separate (CO_SEPARATE) arm is the same arithmetic as its epilogue kernel. */
int b2_linear_group_run_device(b2_linear *const *ops, unsigned count, unsigned m,
                               const void *const *x, const size_t *ldx, void *const *y,
                               const size_t *ldy) {
    if (!ops || !x || !ldx || !y || !ldy || count < 1 || count > B2_GROUP_MAX) return ROCKET_E_SHAPE;
    b2k_linear a[B2_GROUP_MAX];
    for (unsigned i = 0; i < count; ++i) {
        const co_linear_hsig *c = ops[i];
        if (!device_args_ok(c, m, x[i], ldx[i], y[i], ldy[i], 0) || c->fd != ops[0]->fd)
            return ROCKET_E_SHAPE;
        a[i] = (b2k_linear){.m = m, .n = c->plan.n, .k = c->plan.k, .x = x[i], .ldx = ldx[i],
                            .w = c->w, .ldw = c->ldw, .bias = c->bias, .y = y[i], .ldy = ldy[i],
                            .post = c->post == CO_LINEAR_HSIG, .acc = (int)c->acc, .fused = 1,
                            .raw_only = 0};
    }
    if (b2h_fault(B2_FAULT_LAUNCH)) return ROCKET_E_DEVICE;
    unsigned launches = 0;
    int rc = b2d_linear_group(b2h_dev(ops[0]->fd), a, count, &launches);
    for (unsigned i = 0; i < count; ++i) {
        const co_linear_hsig *c = ops[i];
        b2h_count_run(c->mode == CO_CHAIN ? c->plan.chain_submits : c->plan.tasks, c->plan.tasks,
                      i == 0 ? launches : 0);
    }
    return rc;
}

/* Allocation-free unfused FP32 arm: the FP32 accumulator goes to the library's static device
 * scratch (b2d_noalloc_scratch) instead of a cudaMalloc'ed workspace. */
int b2_linear_run_device_noalloc(b2_linear *c, unsigned m, const void *x, size_t ldx, void *y,
                                 size_t ldy) {
    if (!device_args_ok(c, m, x, ldx, y, ldy, 0)) return ROCKET_E_SHAPE;
    if (c->acc != B2_ACC_FP32) return ROCKET_E_UNSUPPORTED;
    const size_t ldp = b2h_round_up(c->plan.n, 4);
    if ((size_t)m * ldp * 4 > B2_NOALLOC_SCRATCH_BYTES) return ROCKET_E_TILING;
    float *scratch = NULL;
    size_t scratch_bytes = 0;
    int rc = b2d_noalloc_scratch(b2h_dev(c->fd), &scratch, &scratch_bytes);
    if (rc) return rc;
    if ((size_t)m * ldp * 4 > scratch_bytes) return ROCKET_E_TILING;
    if (b2h_fault(B2_FAULT_LAUNCH)) return ROCKET_E_DEVICE;
    b2k_linear a = {.m = m, .n = c->plan.n, .k = c->plan.k, .x = x, .ldx = ldx, .w = c->w,
                    .ldw = c->ldw, .bias = c->bias, .y = y, .ldy = ldy, .partial = scratch,
                    .ldp = ldp, .post = c->post == CO_LINEAR_HSIG, .acc = B2_ACC_FP32, .fused = 0,
                    .raw_only = 0};
    unsigned launches = 0;
    rc = b2d_linear(b2h_dev(c->fd), &a, &launches);
    if (launches) count_run(c, launches);
    return rc;
}

int b2_linear_partial_device(b2_linear *c, unsigned m, const void *x, size_t ldx, float *partial,
                             size_t ldp) {
    if (!device_args_ok(c, m, x, ldx, partial, ldp, 1)) return ROCKET_E_SHAPE;
    if (b2h_fault(B2_FAULT_LAUNCH)) return ROCKET_E_DEVICE;
    b2k_linear a = {.m = m, .n = c->plan.n, .k = c->plan.k, .x = x, .ldx = ldx, .w = c->w,
                    .ldw = c->ldw, .bias = NULL, .partial = partial, .ldp = ldp, .post = 0,
                    .acc = B2_ACC_FP32, .fused = 0, .raw_only = 1};
    unsigned launches = 0;
    int rc = b2d_linear(b2h_dev(c->fd), &a, &launches);
    b2h_count_run(0, 0, launches);
    return rc;
}

int b2_linear_epilogue_device(b2_linear *c, unsigned m, const float *partial, size_t ldp, void *y,
                              size_t ldy) {
    if (!c || !partial || !y || m < 1 || m > B2_MAX_DIM || !b2h_dev(c->fd) || ldp < c->plan.n ||
        ldp % 4 || ldy < c->plan.n || ldy % 8 || ((uintptr_t)partial & 15) || ((uintptr_t)y & 15))
        return ROCKET_E_SHAPE;
    if (b2h_fault(B2_FAULT_LAUNCH)) return ROCKET_E_DEVICE;
    int rc = b2d_epilogue(b2h_dev(c->fd), m, c->plan.n, partial, ldp, c->bias,
                          c->post == CO_LINEAR_HSIG, B2_ACC_FP32, y, ldy);
    b2h_count_run(0, 0, rc ? 0 : 1);
    return rc;
}

int b2h_linear_fd(const b2_linear *c) { return c ? c->fd : -1; }

int b2h_linear_desc(const b2_linear *c, unsigned m, const void *x, size_t ldx, b2k_linear *out) {
    if (!c || !out || !x || m < 1 || m > B2_MAX_DIM || ldx < c->plan.k || ldx % 8 || ((uintptr_t)x & 15))
        return ROCKET_E_SHAPE;
    *out = (b2k_linear){.m = m, .n = c->plan.n, .k = c->plan.k, .x = x, .ldx = ldx, .w = c->w,
                        .ldw = c->ldw, .bias = c->bias, .post = c->post == CO_LINEAR_HSIG,
                        .acc = B2_ACC_FP32, .fused = 0, .raw_only = 1};
    return 0;
}

int b2_linear_get_info(const b2_linear *c, b2_linear_info *info) {
    if (!c || !info) return ROCKET_E_SHAPE;
    b2k_linear a = {.m = c->plan.m, .n = c->plan.n, .k = c->plan.k, .x = c->x, .ldx = c->ldx,
                    .w = c->w, .ldw = c->ldw, .bias = c->bias, .y = c->y, .ldy = c->ldy,
                    .post = c->post == CO_LINEAR_HSIG, .acc = (int)c->acc,
                    .fused = c->mode == CO_CHAIN};
    b2k_config cfg;
    int rc = b2d_linear_config(b2h_dev(c->fd), &a, &cfg);
    if (rc) return rc;
    *info = (b2_linear_info){c->plan.m, c->plan.k, c->plan.n, cfg.kernel, cfg.tile_m, cfg.tile_n,
                             cfg.tile_k, cfg.stages, cfg.grid,
                             host_bands(c) * (1u + (c->mode == CO_CHAIN ? 1u : 2u)), c->acc,
                             c->bytes + c->ws_bytes};
    return 0;
}
