/* mock_device.c -- CPU stand-in of the host/device seam (b2_device.h) for host C tests.
 *
 * TEST INFRASTRUCTURE ONLY: linked into tests/c/host_test, never into the shipped library (which
 * has no CPU compute path). It plays the role the reference's mock NPU plays for its host tests
 * (research/custom-ops/tests/c/multitile_host_test.c:14-58): "device" memory is host memory and
 * every operation completes immediately. Linear results come from the oracle's C restatement
 * (oracle/linear_oracle.c): TILE16_EXACT (the reference's arithmetic, bit-identical to its file
 * gate) for tile-16 operators and FP32ACC for FP32 operators, so a host test can check the host
 * layer end to end (staging, descriptors, publish-on-success, error paths, fault seam) against the
 * same oracle bit for bit.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "b2_device.h"
#include "rocket_b200.h"

int oracle_linear(int mode, unsigned m, unsigned k, unsigned n, const uint16_t *x, const uint16_t *w,
                  const uint16_t *bias, int post, uint16_t *y16, double *act, double *raw, int threads);
double oracle_f16_to_double(uint16_t h);
uint16_t oracle_f16_from_double(double d);
uint16_t oracle_ew16(int op, uint16_t a, uint16_t b);
uint16_t oracle_act16(int act, uint16_t a);
unsigned oracle_rmsnorm(unsigned rows, unsigned cols, const uint16_t *x, const uint16_t *gamma, float eps,
                        uint16_t *y);

enum { ORACLE_TILE16_EXACT = 0, ORACLE_FP32ACC = 5 };

struct b2_dev {
    int ordinal;
    void *stream;
    uint32_t status;
};

static int mock_devices(void) {
    const char *e = getenv("B2_MOCK_DEVICES");
    return e ? atoi(e) : 1;
}

int b2d_device_count(void) { return mock_devices(); }

int b2d_open(int ordinal, b2_dev **out) {
    *out = NULL;
    if (ordinal < 0 || ordinal >= mock_devices()) return ROCKET_E_DEVICE;
    b2_dev *d = calloc(1, sizeof(*d));
    if (!d) return ROCKET_E_NOMEM;
    d->ordinal = ordinal;
    *out = d;
    return 0;
}
void b2d_close(b2_dev *d) { free(d); }
int b2d_set_stream(b2_dev *d, void *stream) {
    if (!d) return ROCKET_E_SHAPE;
    d->stream = stream;
    return 0;
}
void *b2d_stream(b2_dev *d) { return d ? d->stream : NULL; }
int b2d_sm_count(b2_dev *d) { return d ? 148 : 0; }
int b2d_ordinal(b2_dev *d) { return d ? d->ordinal : -1; }

int b2d_malloc(b2_dev *d, size_t bytes, void **out) {
    (void)d;
    *out = calloc(1, bytes ? bytes : 1);
    return *out ? 0 : ROCKET_E_NOMEM;
}
void b2d_free(b2_dev *d, void *ptr) {
    (void)d;
    free(ptr);
}
void *b2d_host_alloc(size_t bytes) { return malloc(bytes); }
void b2d_host_free(void *ptr) { free(ptr); }

int b2d_copy_2d(b2_dev *d, void *dst, size_t dpitch, const void *src, size_t spitch, size_t width, size_t rows,
                int kind) {
    (void)d;
    (void)kind;
    if ((!dst || !src) && rows && width) return ROCKET_E_SHAPE;
    for (size_t r = 0; r < rows; r++) memcpy((char *)dst + r * dpitch, (const char *)src + r * spitch, width);
    return 0;
}
int b2d_copy_side(b2_dev *d, void *dst, size_t dpitch, const void *src, size_t spitch, size_t width, size_t rows,
                  int kind, unsigned ev) {
    if (ev >= B2D_SIDE_EVENTS) return ROCKET_E_SHAPE;
    return b2d_copy_2d(d, dst, dpitch, src, spitch, width, rows, kind);
}
int b2d_wait_side(b2_dev *d, unsigned ev) { return d && ev < B2D_SIDE_EVENTS ? 0 : ROCKET_E_SHAPE; }
int b2d_memset(b2_dev *d, void *ptr, int value, size_t bytes) {
    (void)d;
    memset(ptr, value, bytes);
    return 0;
}
int b2d_sync(b2_dev *d) { return d ? 0 : ROCKET_E_DEVICE; }
uint32_t b2d_status(b2_dev *d, int clear) {
    uint32_t s = d->status;
    if (clear) d->status = 0;
    return s;
}
void b2d_status_merge(b2_dev *d, uint32_t bits) {
    if (d) d->status |= bits;
}

/* ------------------------------------------------------------------------------ Linear */
static int f16_nonfinite(uint16_t h) { return (h & 0x7c00u) == 0x7c00u; }

/* Pitched FP16 [rows, ld] -> contiguous [rows, cols]. */
static uint16_t *pack(const void *p, unsigned rows, unsigned cols, size_t ld) {
    uint16_t *out = malloc((size_t)rows * cols * 2);
    if (!out) return NULL;
    for (unsigned r = 0; r < rows; r++) memcpy(out + (size_t)r * cols, (const uint16_t *)p + (size_t)r * ld, (size_t)cols * 2);
    return out;
}

static float finish32(float acc, const uint16_t *bias, unsigned col, int post) {
    float a = acc;
    if (bias) a += (float)oracle_f16_to_double(bias[col]);
    if (post) {
        float t = a / 6.0f + 0.5f;
        a = t < 0.0f ? 0.0f : (t > 1.0f ? 1.0f : t);
    }
    return a;
}

static int linear_plain(b2_dev *d, const b2k_linear *a, unsigned *launches);

/* Gated pair: the folded FP16 sums of the packed gate|up weight, each finished with its half's
 * bias, combined as fp16(fp16(g * fp16(gate(g))) * u) -- the arithmetic of the fused epilogue. */
static int linear_gated(b2_dev *d, const b2k_linear *a, unsigned *launches) {
    const unsigned h = a->gate_n, h32 = (h + 31) / 32 * 32;
    if ((a->gate != 1 && a->gate != 2) || a->acc || a->post || a->res || a->raw_only || !h || a->n != 2 * h32 ||
        !a->y || a->ldy < h)
        return ROCKET_E_SHAPE;
    uint16_t *sums = malloc((size_t)a->m * a->n * 2);
    if (!sums) return ROCKET_E_NOMEM;
    b2k_linear raw = *a;
    raw.gate = 0;
    raw.bias = NULL;
    raw.fused = 1;
    raw.y = sums;
    raw.ldy = a->n;
    int rc = linear_plain(d, &raw, launches);
    const uint16_t *bg = a->bias, *bu = a->bias2;
    for (unsigned r = 0; !rc && r < a->m; r++)
        for (unsigned j = 0; j < h; j++) {
            uint16_t g = sums[(size_t)r * a->n + 64 * (j / 32) + j % 32];
            uint16_t u = sums[(size_t)r * a->n + 64 * (j / 32) + 32 + j % 32];
            if (bg) g = oracle_ew16(0, g, bg[j]);
            if (bu) u = oracle_ew16(0, u, bu[j]);
            const uint16_t o = oracle_ew16(1, oracle_act16(a->gate, g), u);
            if (f16_nonfinite(o)) d->status |= B2D_ST_NONFINITE_OUTPUT;
            ((uint16_t *)a->y)[(size_t)r * a->ldy + j] = o;
        }
    free(sums);
    if (!rc) *launches = (a->fused && a->m > B2D_GEMV_MAX_M) ? 1 : 2;
    return rc;
}

int b2d_linear(b2_dev *d, const b2k_linear *a, unsigned *launches) {
    *launches = 0;
    if (!d || !a) return ROCKET_E_SHAPE;
    if (a->gate) return linear_gated(d, a, launches);
    int rc = linear_plain(d, a, launches);
    if (!rc && a->res) {   /* y = fp16(res + y) */
        for (unsigned r = 0; r < a->m; r++)
            for (unsigned c = 0; c < a->n; c++) {
                uint16_t *y = (uint16_t *)a->y + (size_t)r * a->ldy + c;
                *y = oracle_ew16(0, *y, ((const uint16_t *)a->res)[(size_t)r * a->ldr + c]);
                if (f16_nonfinite(*y)) d->status |= B2D_ST_NONFINITE_OUTPUT;
            }
        if (!(a->fused && a->m > B2D_GEMV_MAX_M)) *launches += 1;
    }
    return rc;
}

static int linear_plain(b2_dev *d, const b2k_linear *a, unsigned *launches) {
    *launches = 0;
    if (!d || !a || !a->m || !a->n || !a->k || !a->x || !a->w) return ROCKET_E_SHAPE;
    uint16_t *x = pack(a->x, a->m, a->k, a->ldx), *w = pack(a->w, a->n, a->k, a->ldw);
    uint16_t *y = malloc((size_t)a->m * a->n * 2);
    double *raw = malloc((size_t)a->m * a->n * sizeof(double));
    int rc = (x && w && y && raw) ? 0 : ROCKET_E_NOMEM;
    const int mode = (a->acc == 0 && !a->raw_only) ? ORACLE_TILE16_EXACT : ORACLE_FP32ACC;
    if (!rc && oracle_linear(mode, a->m, a->k, a->n, x, w, a->raw_only ? NULL : (const uint16_t *)a->bias,
                             a->raw_only ? 0 : a->post, y, NULL, raw, 1))
        rc = ROCKET_E_SHAPE;
    if (!rc) {
        if (a->raw_only) {
            for (unsigned r = 0; r < a->m; r++)
                for (unsigned c = 0; c < a->n; c++) a->partial[(size_t)r * a->ldp + c] = (float)raw[(size_t)r * a->n + c];
        } else {
            for (unsigned r = 0; r < a->m; r++)
                for (unsigned c = 0; c < a->n; c++) {
                    const uint16_t h = y[(size_t)r * a->n + c];
                    if (f16_nonfinite(h)) d->status |= B2D_ST_NONFINITE_OUTPUT;
                    ((uint16_t *)a->y)[(size_t)r * a->ldy + c] = h;
                }
            /* the unfused FP32 arm also leaves its raw accumulator in the workspace */
            if (!a->fused && a->acc != 0 && a->partial)
                for (unsigned r = 0; r < a->m; r++)
                    for (unsigned c = 0; c < a->n; c++)
                        a->partial[(size_t)r * a->ldp + c] = (float)raw[(size_t)r * a->n + c];
        }
        *launches = (a->fused || a->raw_only) ? 1 : 2;
    }
    free(x);
    free(w);
    free(y);
    free(raw);
    return rc;
}

int b2d_linear_config(b2_dev *d, const b2k_linear *a, b2k_config *cfg) {
    if (!d || !a || !cfg) return ROCKET_E_SHAPE;
    memset(cfg, 0, sizeof(*cfg));
    cfg->kernel = a->m <= B2D_GEMV_MAX_M ? 1 : 0;
    cfg->tile_m = cfg->kernel ? a->m : 256;
    cfg->tile_n = cfg->kernel ? 8 : 256;
    cfg->tile_k = cfg->kernel ? 256 : 64;
    cfg->grid = 148;
    return 0;
}

int b2d_linear_group(b2_dev *d, const b2k_linear *ops, unsigned count, unsigned *launches) {
    *launches = 0;
    if (!d || !ops || !count || count > B2D_GROUP_MAX) return ROCKET_E_SHAPE;
    for (unsigned i = 0; i < count; i++) {
        unsigned l = 0;
        int rc = b2d_linear(d, &ops[i], &l);
        if (rc) return rc;
    }
    *launches = 1;
    return 0;
}

int b2d_epilogue(b2_dev *d, unsigned m, unsigned n, const float *partial, size_t ldp, const void *bias, int post,
                 int acc, void *y, size_t ldy) {
    if (!d || !m || !n || !partial || !y || ldp < n || ldy < n || acc != 1) return ROCKET_E_SHAPE;
    for (unsigned r = 0; r < m; r++)
        for (unsigned c = 0; c < n; c++) {
            const uint16_t h = oracle_f16_from_double(finish32(partial[(size_t)r * ldp + c], bias, c, post));
            if (f16_nonfinite(h)) d->status |= B2D_ST_NONFINITE_OUTPUT;
            ((uint16_t *)y)[(size_t)r * ldy + c] = h;
        }
    return 0;
}

int b2d_scan_nonfinite(b2_dev *d, const void *p, size_t rows, size_t cols, size_t ld, uint32_t bit) {
    if (!d || !p || ld % 8) return ROCKET_E_SHAPE;
    for (size_t r = 0; r < rows; r++)
        for (size_t c = 0; c < cols; c++)
            if (f16_nonfinite(((const uint16_t *)p)[r * ld + c])) d->status |= bit;
    return 0;
}

/* C2=8 cubes: atom (group g, row r) = 8 channels at ptr[(g * physical_rows + r) * 8]. */
int b2d_cube_to_rowmajor(b2_dev *d, const b2k_cube_tile *tiles, unsigned count, void *dst, size_t ld) {
    if (!d || !dst || ld % 8 || count > B2K_MAX_CUBE_TILES) return ROCKET_E_SHAPE;
    for (unsigned t = 0; t < count; t++) {
        const b2k_cube_tile *c = &tiles[t];
        if (!c->ptr || c->physical_cols % 8 || c->rows > c->physical_rows || c->cols > c->physical_cols) return ROCKET_E_SHAPE;
        for (unsigned g = 0; g < (c->cols + 7) / 8; g++)
            for (unsigned r = 0; r < c->rows; r++)
                memcpy((uint16_t *)dst + (size_t)(c->row0 + r) * ld + c->col0 + 8 * g,
                       (const uint16_t *)c->ptr + ((size_t)g * c->physical_rows + r) * 8, 16);
    }
    return 0;
}

int b2d_rowmajor_to_cube(b2_dev *d, const void *src, size_t ld, const b2k_cube_tile *tiles, unsigned count) {
    if (!d || !src || ld % 8 || count > B2K_MAX_CUBE_TILES) return ROCKET_E_SHAPE;
    for (unsigned t = 0; t < count; t++) {
        const b2k_cube_tile *c = &tiles[t];
        if (!c->ptr || c->physical_cols % 8 || c->rows > c->physical_rows || c->cols > c->physical_cols) return ROCKET_E_SHAPE;
        for (unsigned g = 0; g < c->physical_cols / 8; g++)
            for (unsigned r = 0; r < c->physical_rows; r++) {
                uint16_t v[8] = {0};
                if (r < c->rows && 8 * g < c->cols) {
                    memcpy(v, (const uint16_t *)src + (size_t)(c->row0 + r) * ld + c->col0 + 8 * g, 16);
                    for (unsigned e = c->cols - 8 * g; e < 8; e++) v[e] = 0;
                }
                memcpy((uint16_t *)c->ptr + ((size_t)g * c->physical_rows + r) * 8, v, 16);
            }
    }
    return 0;
}

static float noalloc_scratch[B2D_NOALLOC_SCRATCH_BYTES / sizeof(float)];
/* The direct cube GEMM: the same gather -> fused Linear -> scatter on the CPU, with the device's
 * eligibility rules, so the host layer's choice between the two forms is tested without a GPU. */
int b2d_linear_cube(b2_dev *d, const b2k_linear *a, const b2k_cube_io *io, unsigned *launches) {
    *launches = 0;
    if (!d || !a || !io || !io->in || !io->out) return ROCKET_E_SHAPE;
    if (a->m <= B2D_GEMV_MAX_M || !a->fused || a->raw_only || a->res || a->gate || !io->kviews || !io->ntiles ||
        io->nin > B2D_CUBE_MAX_VIEWS || io->nout > B2D_CUBE_MAX_VIEWS || io->nin % io->kviews ||
        io->nout % io->ntiles || io->kview_k % 64)
        return ROCKET_E_UNSUPPORTED;
    for (unsigned i = 0; i < io->nin; i++)
        if (io->in[i].cols % 8) return ROCKET_E_UNSUPPORTED;
    const size_t ldx = (a->k + 7) / 8 * 8, ldy = (a->n + 7) / 8 * 8;
    uint16_t *x = calloc((size_t)a->m * ldx, 2), *y = calloc((size_t)a->m * ldy, 2);
    int rc = x && y ? 0 : ROCKET_E_NOMEM;
    for (unsigned i = 0; !rc && i < io->nin; i += B2K_MAX_CUBE_TILES) {
        unsigned n = io->nin - i < B2K_MAX_CUBE_TILES ? io->nin - i : B2K_MAX_CUBE_TILES;
        rc = b2d_cube_to_rowmajor(d, io->in + i, n, x, ldx);
    }
    b2k_linear f = *a;
    f.x = x;
    f.ldx = ldx;
    f.y = y;
    f.ldy = ldy;
    unsigned l = 0;
    if (!rc) rc = b2d_linear(d, &f, &l);
    for (unsigned i = 0; !rc && i < io->nout; i += B2K_MAX_CUBE_TILES) {
        unsigned n = io->nout - i < B2K_MAX_CUBE_TILES ? io->nout - i : B2K_MAX_CUBE_TILES;
        rc = b2d_rowmajor_to_cube(d, y, ldy, io->out + i, n);
    }
    free(x);
    free(y);
    if (!rc) *launches = 1;
    return rc;
}

int b2d_noalloc_scratch(b2_dev *d, float **ptr, size_t *bytes) {
    if (!d) return ROCKET_E_DEVICE;
    *ptr = noalloc_scratch;
    *bytes = B2D_NOALLOC_SCRATCH_BYTES;
    return 0;
}

int b2d_guard_init(b2_dev *d, void *base, size_t payload, size_t slack, size_t guard) {
    if (!d || !base) return ROCKET_E_SHAPE;
    memset((char *)base + payload + slack, 0xa5, guard);
    return 0;
}

int b2d_guard_check(b2_dev *d, void *const *bases, const size_t *payloads, unsigned count, size_t slack,
                    size_t guard) {
    if (!d || count > B2K_MAX_CUBE_TILES) return ROCKET_E_SHAPE;
    for (unsigned i = 0; i < count; i++) {
        const unsigned char *p = (const unsigned char *)bases[i] + payloads[i];
        for (size_t j = 0; j < slack + guard; j++)
            if (p[j] != (j < slack ? 0x00 : 0xa5)) d->status |= B2D_ST_GUARD;
    }
    return 0;
}

/* No peer memory in a single host process. */
int b2d_ipc_export(b2_dev *d, const void *ptr, unsigned char out[B2D_IPC_HANDLE_BYTES]) {
    (void)d;
    (void)ptr;
    (void)out;
    return ROCKET_E_UNSUPPORTED;
}
int b2d_ipc_open(b2_dev *d, const unsigned char in[B2D_IPC_HANDLE_BYTES], void **ptr) {
    (void)d;
    (void)in;
    *ptr = NULL;
    return ROCKET_E_UNSUPPORTED;
}
int b2d_ipc_close(b2_dev *d, void *ptr) {
    (void)d;
    (void)ptr;
    return ROCKET_E_UNSUPPORTED;
}

/* One-rank round: the FP32 partial, then the epilogue of the owned rows. */
/* Timing events: the mock completes everything at once, so every interval is 0. */
struct b2_timer {
    int marked[B2D_TIMER_MARKS];
};
int b2d_timer_create(b2_dev *d, b2_timer **out) {
    *out = d ? calloc(1, sizeof(b2_timer)) : NULL;
    return *out ? 0 : (d ? ROCKET_E_NOMEM : ROCKET_E_DEVICE);
}
void b2d_timer_destroy(b2_timer *t) { free(t); }
int b2d_timer_mark(b2_dev *d, b2_timer *t, unsigned mark) {
    if (!d || !t || mark >= B2D_TIMER_MARKS) return ROCKET_E_SHAPE;
    t->marked[mark] = 1;
    return 0;
}
int b2d_timer_ms(b2_timer *t, unsigned from, unsigned to, float *ms) {
    if (!t || !ms || from >= B2D_TIMER_MARKS || to >= B2D_TIMER_MARKS || !t->marked[from] || !t->marked[to])
        return ROCKET_E_SHAPE;
    *ms = 0.0f;
    return 0;
}

int b2d_ksplit_round(b2_dev *d, const b2k_linear *a, const b2k_ksplit *ks, unsigned *launches) {
    *launches = 0;
    if (!d || !a || !ks || ks->world != 1 || ks->rank != 0 || ks->rows_per_rank % 32) return ROCKET_E_SHAPE;
    const size_t ldp = ks->ldp;
    float *part = malloc((size_t)a->m * ldp * sizeof(float));
    if (!part) return ROCKET_E_NOMEM;
    b2k_linear raw = *a;
    raw.partial = part;
    raw.ldp = ldp;
    raw.raw_only = 1;
    unsigned l = 0;
    int rc = b2d_linear(d, &raw, &l);
    if (!rc && ks->own_rows) rc = b2d_epilogue(d, ks->own_rows, a->n, part, ldp, ks->bias, ks->post, 1, ks->y_own, ks->ldy);
    free(part);
    if (!rc) *launches = 3;
    for (unsigned i = 0; !rc && ks->timer && i < 4; ++i) rc = b2d_timer_mark(d, ks->timer, i);
    return rc;
}

/* ---------------------------------------------------------------------- graph node kernels */
int b2d_elementwise(b2_dev *d, int op, unsigned rows, unsigned cols, const void *a, size_t lda, const void *b,
                    size_t ldb, void *y, size_t ldy) {
    const int bin = op == B2D_EW_ADD || op == B2D_EW_MUL;
    if (!d || op < B2D_EW_ADD || op > B2D_EW_HSIG || !a || !y || lda < cols || ldy < cols || (bin && (!b || ldb < cols)))
        return ROCKET_E_SHAPE;
    for (unsigned r = 0; r < rows; r++)
        for (unsigned c = 0; c < cols; c++) {
            const uint16_t av = ((const uint16_t *)a)[(size_t)r * lda + c];
            const uint16_t bv = bin ? ((const uint16_t *)b)[(size_t)r * ldb + c] : 0;
            const uint16_t o = oracle_ew16(op, av, bv);
            if (f16_nonfinite(o)) d->status |= B2D_ST_NONFINITE_OUTPUT;
            ((uint16_t *)y)[(size_t)r * ldy + c] = o;
        }
    return 0;
}

int b2d_rmsnorm(b2_dev *d, unsigned rows, unsigned cols, const void *x, size_t ldx, const void *gamma, float eps,
                void *y, size_t ldy) {
    if (!d || !x || !y || !gamma || !(eps > 0.0f) || ldx < cols || ldy < cols) return ROCKET_E_SHAPE;
    uint16_t *in = pack(x, rows, cols, ldx), *out = malloc((size_t)rows * cols * 2 + 2);
    if (!in || !out) {
        free(in);
        free(out);
        return ROCKET_E_NOMEM;
    }
    memset(out, 0, (size_t)rows * cols * 2);
    if (oracle_rmsnorm(rows, cols, in, gamma, eps, out)) d->status |= B2D_ST_NONFINITE_INPUT;
    for (unsigned r = 0; r < rows; r++) memcpy((uint16_t *)y + (size_t)r * ldy, out + (size_t)r * cols, (size_t)cols * 2);
    free(in);
    free(out);
    return 0;
}

/* ---------------------------------------------------------------------- CUDA graphs
 * Every mock operation completes at once, so there is nothing to record: capture is reported
 * unavailable and the host issues the launches directly. */
int b2d_capture_begin(b2_dev *d) { return d ? ROCKET_E_UNSUPPORTED : ROCKET_E_DEVICE; }
int b2d_capture_end(b2_dev *d, b2_exec **out, unsigned *kernels) {
    *out = NULL;
    if (kernels) *kernels = 0;
    return ROCKET_E_DEVICE;
}
int b2d_exec_launch(b2_dev *d, b2_exec *x) { return ROCKET_E_SHAPE; }
void b2d_exec_destroy(b2_exec *x) { (void)x; }

/* ---------------------------------------------------------------------- plan (RKPlan) tiles
 * The oracle's restatement (oracle/rkplan_oracle.c) on host memory. mock_rk_inject plays the
 * reference mock's injection knobs (research/custom-ops/tests/mock/npu_mock.c: rk_mock_inject_nan,
 * the guard corruption): 1 writes NaN into element 0 of every task output, 2 overwrites the first
 * slack byte behind every task output's tile. */
typedef struct {
    uint16_t *p;
    unsigned layout, rows, cols, prows, pcols;
} rk_oracle_tile;
int rk_oracle_task(int op, const rk_oracle_tile *x, const rk_oracle_tile *w, const rk_oracle_tile *aux,
                   rk_oracle_tile *y);
void rk_oracle_pack(rk_oracle_tile *dst, unsigned r0, unsigned c0, unsigned rows, unsigned cols, int clear, int mode,
                    int transpose, const uint16_t *src, size_t ld);
void rk_oracle_unpack(const rk_oracle_tile *src, uint16_t *dst, size_t ld);

int mock_rk_inject = 0;
unsigned mock_rk_tasks = 0;   /* tasks run since start */

static rk_oracle_tile mock_tile(const b2k_rk_tile *t) {
    rk_oracle_tile o = {(uint16_t *)t->ptr, t->layout, t->rows, t->cols, t->physical_rows, t->physical_cols};
    return o;
}

int b2d_rk_pack(b2_dev *d, const b2k_rk_pack *items, unsigned count) {
    if (!d || (count && !items)) return ROCKET_E_SHAPE;
    for (unsigned i = 0; i < count; i++) {
        rk_oracle_tile t = mock_tile(&items[i].dst);
        rk_oracle_pack(&t, items[i].r0, items[i].c0, items[i].rows, items[i].cols, (int)items[i].clear,
                       (int)items[i].mode, (int)items[i].transpose, (const uint16_t *)items[i].src, items[i].ld);
    }
    return 0;
}

int b2d_rk_task(b2_dev *d, const b2k_rk_task *t) {
    if (!d || !t) return ROCKET_E_SHAPE;
    rk_oracle_tile x = mock_tile(&t->x), w = mock_tile(&t->w), aux = mock_tile(&t->aux), y = mock_tile(&t->y);
    if (rk_oracle_task((int)t->op, &x, &w, &aux, &y)) return ROCKET_E_SHAPE;
    mock_rk_tasks++;
    if (mock_rk_inject == 1) y.p[0] = 0x7e00;
    if (mock_rk_inject == 2) ((unsigned char *)y.p)[(size_t)y.prows * y.pcols * 2] ^= 0x5a;
    return 0;
}

/* The chain as its separate tasks into host temporaries: only y is written (the intermediate
 * views are left as they were, as on the device). */
int b2d_rk_chain(b2_dev *d, const b2k_rk_chain *t) {
    if (!d || !t || !t->n || t->n > B2K_RK_CHAIN_MAX || (t->n < 2 && !t->lut)) return ROCKET_E_SHAPE;
    const size_t elems = (size_t)t->y.physical_rows * t->y.physical_cols;
    uint16_t *tmp[2] = {calloc(elems, 2), calloc(elems, 2)};
    int rc = tmp[0] && tmp[1] ? 0 : ROCKET_E_NOMEM;
    rk_oracle_tile y = mock_tile(&t->y), prev = y;
    for (unsigned i = 0; !rc && i <= t->n; i++) {
        if (i == t->n && !t->lut) break;
        const int last = t->lut ? i == t->n : i == t->n - 1;
        rk_oracle_tile out = y;
        if (!last) out.p = tmp[i & 1];
        if (i == t->n) {
            rc = rk_oracle_task((int)t->lut, &prev, &prev, &prev, &out);
        } else {
            rk_oracle_tile x = mock_tile(&t->x[i]), w = mock_tile(&t->w[i]);
            rc = rk_oracle_task(i ? 2 : 1, &x, &w, &prev, &out);
        }
        prev = out;
        mock_rk_tasks++;
    }
    free(tmp[0]);
    free(tmp[1]);
    if (rc) return ROCKET_E_SHAPE;
    if (mock_rk_inject == 1) y.p[0] = 0x7e00;
    if (mock_rk_inject == 2) ((unsigned char *)y.p)[(size_t)y.prows * y.pcols * 2] ^= 0x5a;
    return 0;
}

int b2d_rk_unpack(b2_dev *d, const b2k_rk_unpack *items, unsigned count) {
    if (!d || (count && !items)) return ROCKET_E_SHAPE;
    for (unsigned i = 0; i < count; i++) {
        rk_oracle_tile s = mock_tile(&items[i].src);
        rk_oracle_unpack(&s, (uint16_t *)items[i].dst, items[i].ld);
    }
    return 0;
}
