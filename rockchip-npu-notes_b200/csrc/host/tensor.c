/* tensor.c -- tensor descriptors, device buffers, views and host<->device transfers.
 *
 * Descriptor rules and layouts follow research/custom-ops/src/custom_ops.c (reference project):
 *   co_tensor_matrix/input/weight/spatial/linear   :18-33, :62-79
 *   co_k_tiles/_length/_offset, co_tensor_input_slice :34-61
 *   co_index (CUBE, WEIGHT, LINEAR addressing)      :80-85
 *   co_buffer_alloc/free (slack + guard)            :86-101
 *   co_view_init validation                         :102-117
 *   co_upload_f16 / co_download                     :127-188
 *   co_sentinel / co_guard_check                    :189-221
 *   co_copy, co_bias_upload, co_identity_upload, co_ones_upload :222-262
 * The layouts have to be identical for the cube entries to be a drop-in, so the descriptor
 * arithmetic is the same; the transfers are CUDA copies into HBM instead of CPU writes through
 * a DRM mapping, and the reference's 32-bit DMA-window checks do not apply.
 */
#include "b2_host.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

static unsigned round_up_u(unsigned x, unsigned a) { return (x + a - 1) / a * a; }
static unsigned width_of(enum co_type t) { return t == CO_F16 ? 2u : 4u; }

int co_tensor_matrix(co_tensor *t, unsigned m, unsigned n, enum co_type type) {
    if (!t || !m || !n || m > 256 || n > 256 || (type != CO_F16 && type != CO_F32))
        return ROCKET_E_SHAPE;
    *t = (co_tensor){.type = type, .layout = CO_CUBE, .rows = m, .cols = n,
                     .physical_rows = round_up_u(m < 12 ? 12 : m, 4),
                     .physical_cols = round_up_u(n, 32), .atom = type == CO_F16 ? 8u : 4u};
    t->bytes = (size_t)t->physical_rows * t->physical_cols * width_of(type);
    return 0;
}

int co_tensor_input(co_tensor *t, unsigned m, unsigned k) {
    if (!t || !m || m > 256 || !k || k > CO_MAX_K) return ROCKET_E_SHAPE;
    *t = (co_tensor){.type = CO_F16, .layout = CO_CUBE, .rows = m, .cols = k,
                     .physical_rows = round_up_u(m < 12 ? 12 : m, 4),
                     .physical_cols = round_up_u(k, 32), .atom = 8};
    t->bytes = (size_t)t->physical_rows * t->physical_cols * 2;
    return 0;
}

unsigned co_k_tiles(unsigned k) { return k ? (k + CO_K_TILE - 1u) / CO_K_TILE : 0; }

unsigned co_k_tile_length(unsigned k, unsigned index) {
    unsigned k0 = index * CO_K_TILE;
    if (k0 >= k) return 0;
    return k - k0 > CO_K_TILE ? CO_K_TILE : k - k0;
}

size_t co_k_tile_offset(const co_tensor *full, unsigned k0) {
    if (!full || full->layout != CO_CUBE) return 0;
    return (size_t)k0 * full->physical_rows * 2;
}

int co_tensor_input_slice(co_tensor *slice, const co_tensor *full, unsigned k0, unsigned kt,
                          size_t *offset) {
    if (!slice || !full || full->layout != CO_CUBE || full->type != CO_F16 || full->atom != 8 ||
        !full->rows || !full->cols || full->physical_rows < 12 || full->physical_rows % 4 ||
        full->physical_cols % 32 || k0 % CO_K_TILE || !kt || kt > CO_K_TILE ||
        k0 >= full->cols || k0 + kt > full->cols || k0 + round_up_u(kt, 32) > full->physical_cols)
        return ROCKET_E_SHAPE;
    unsigned pc = round_up_u(kt, 32);
    co_tensor s = {.type = CO_F16, .layout = CO_CUBE, .rows = full->rows, .cols = kt,
                   .physical_rows = full->physical_rows, .physical_cols = pc, .atom = 8,
                   .bytes = (size_t)full->physical_rows * pc * 2};
    if (s.bytes > full->bytes) return ROCKET_E_SHAPE;
    *slice = s;
    if (offset) *offset = co_k_tile_offset(full, k0);
    return 0;
}

int co_tensor_weight(co_tensor *t, unsigned n, unsigned k) {
    if (!t || !n || !k || n > 256 || k > 256) return ROCKET_E_SHAPE;
    *t = (co_tensor){.type = CO_F16, .layout = CO_WEIGHT, .rows = n, .cols = k,
                     .physical_rows = round_up_u(n, 32), .physical_cols = round_up_u(k, 32),
                     .atom = 32};
    t->bytes = (size_t)t->physical_rows * t->physical_cols * 2;
    return 0;
}

int co_tensor_spatial(co_tensor *t, unsigned c, unsigned h, unsigned w) {
    if (!t || !c || c > 256 || !h || !w || h > 63 || w > 63 || h * w > 256) return ROCKET_E_SHAPE;
    *t = (co_tensor){.type = CO_F16, .layout = CO_CUBE, .rows = h * w, .cols = c,
                     .physical_rows = h * w, .physical_cols = round_up_u(c, 32), .atom = 8};
    t->bytes = (size_t)t->physical_rows * t->physical_cols * 2;
    return 0;
}

int co_tensor_linear(co_tensor *t, unsigned n) {
    if (!t || !n || n > 65520) return ROCKET_E_SHAPE;
    *t = (co_tensor){.type = CO_F16, .layout = CO_LINEAR, .rows = 1, .cols = n,
                     .physical_rows = 1, .physical_cols = n, .atom = 1, .bytes = (size_t)n * 2};
    return 0;
}

size_t co_index(const co_tensor *t, unsigned r, unsigned c) {
    if (t->layout == CO_LINEAR) return (size_t)r * t->physical_cols + c;
    if (t->layout == CO_WEIGHT)  /* (N/16, K/32, 16, 32) */
        return (((size_t)(r / 16) * (t->physical_cols / 32) + c / 32) * 16 + r % 16) * 32 + c % 32;
    /* CUBE: [physical_cols/atom][physical_rows][atom] */
    return ((size_t)(c / t->atom) * t->physical_rows + r) * t->atom + c % t->atom;
}

/* ------------------------------------------------------------------------------ buffers */
int co_buffer_alloc(int fd, size_t payload, co_buffer *b) {
    if (!b || !payload || payload > SIZE_MAX - CO_SLACK - CO_GUARD) return ROCKET_E_SHAPE;
    memset(b, 0, sizeof(*b));
    b2_dev *d = b2h_dev(fd);
    if (!d) return ROCKET_E_SHAPE;
    b->fd = fd;
    b->payload = payload;
    int rc = rocket_bo_alloc32(fd, payload + CO_SLACK + CO_GUARD, &b->bo);   /* zero-filled */
    if (rc) { memset(b, 0, sizeof(*b)); return rc; }
    rc = b2d_guard_init(d, b->bo.ptr, payload, CO_SLACK, CO_GUARD);
    if (!rc) rc = b2d_sync(d);
    if (rc) co_buffer_free(b);
    return rc;
}

void co_buffer_free(co_buffer *b) {
    if (b && b->bo.handle) rocket_bo_free(b->fd, &b->bo);
    if (b) memset(b, 0, sizeof(*b));
}

int co_view_init(co_view *v, co_buffer *b, size_t offset, const co_tensor *t) {
    if (!v || !b || !t || !b->bo.handle || !t->bytes ||
        (t->type != CO_F16 && t->type != CO_F32) ||
        (t->layout != CO_CUBE && t->layout != CO_WEIGHT && t->layout != CO_LINEAR) ||
        !t->rows || !t->cols || t->rows > t->physical_rows || t->cols > t->physical_cols ||
        t->physical_rows > 256 ||
        t->physical_cols > (t->layout == CO_LINEAR ? 65520u : (t->layout == CO_WEIGHT ? 256u : CO_MAX_K)) ||
        t->atom != (t->layout == CO_LINEAR ? 1u : (t->layout == CO_WEIGHT ? 32u : (t->type == CO_F16 ? 8u : 4u))) ||
        t->physical_cols % t->atom ||
        (t->layout == CO_WEIGHT && (t->type != CO_F16 || t->physical_rows % 16)) ||
        t->bytes != (size_t)t->physical_rows * t->physical_cols * width_of(t->type) ||
        (offset & 15) || offset > b->payload || t->bytes > b->payload - offset)
        return ROCKET_E_SHAPE;
    *v = (co_view){b, offset, *t};
    return 0;
}

static int valid_view(const co_view *v) {
    co_view check;
    return v && !co_view_init(&check, v->buffer, v->offset, &v->tensor) && b2h_dev(v->buffer->fd);
}

static void *view_ptr(const co_view *v) { return (char *)v->buffer->bo.ptr + v->offset; }

/* ------------------------------------------------------------------------------ transfers */
int co_upload_f16(co_view *v, const _Float16 *src) {
    if (!src || !v || v->tensor.type != CO_F16 || !valid_view(v)) return ROCKET_E_SHAPE;
    const co_tensor *t = &v->tensor;
    uint16_t *img = calloc(t->bytes / 2, 2);               /* padding stays zero */
    if (!img) return ROCKET_E_NOMEM;
    const uint16_t *s = (const uint16_t *)src;
    for (unsigned r = 0; r < t->rows; r++)
        for (unsigned c = 0; c < t->cols; c++) img[co_index(t, r, c)] = s[(size_t)r * t->cols + c];
    b2_dev *d = b2h_dev(v->buffer->fd);
    int rc = b2d_copy_2d(d, view_ptr(v), t->bytes, img, t->bytes, t->bytes, 1, B2D_H2D);
    if (!rc) rc = b2d_sync(d);
    free(img);
    return rc;
}

int co_download(co_view *v, void *dst) {
    if (!dst || !v || !valid_view(v)) return ROCKET_E_SHAPE;
    const co_tensor *t = &v->tensor;
    unsigned char *img = malloc(t->bytes);
    if (!img) return ROCKET_E_NOMEM;
    b2_dev *d = b2h_dev(v->buffer->fd);
    int rc = b2d_copy_2d(d, img, t->bytes, view_ptr(v), t->bytes, t->bytes, 1, B2D_D2H);
    if (!rc) rc = b2d_sync(d);
    if (!rc) {
        unsigned w = width_of(t->type);
        for (unsigned r = 0; r < t->rows; r++)
            for (unsigned c = 0; c < t->cols; c++)
                memcpy((char *)dst + ((size_t)r * t->cols + c) * w, img + co_index(t, r, c) * w, w);
    }
    free(img);
    return rc;
}

int co_sentinel(co_buffer *b) {
    if (!b || !b->bo.handle) return ROCKET_E_SHAPE;
    b2_dev *d = b2h_dev(b->fd);
    if (!d) return ROCKET_E_SHAPE;
    int rc = b2d_memset(d, b->bo.ptr, 0xff, b->payload);           /* NaN in f16 and f32 */
    if (!rc) rc = b2d_memset(d, (char *)b->bo.ptr + b->payload + CO_SLACK, 0xa5, CO_GUARD);
    if (!rc) rc = b2d_sync(d);
    return rc;
}

int co_guard_check(co_buffer *b) {
    if (!b || !b->bo.handle) return ROCKET_E_SHAPE;
    b2_dev *d = b2h_dev(b->fd);
    if (!d) return ROCKET_E_SHAPE;
    int rc = b2d_sync(d);
    if (rc) return rc;
    uint32_t before = b2d_status(d, 1);       /* bits of earlier asynchronous work */
    void *base = b->bo.ptr;
    size_t payload = b->payload;
    rc = b2d_guard_check(d, &base, &payload, 1, CO_SLACK, CO_GUARD);
    if (!rc) rc = b2d_sync(d);
    uint32_t got = b2d_status(d, 1);
    b2d_status_merge(d, before);
    if (!rc && (got & B2_STATUS_GUARD)) rc = ROCKET_E_DEVICE;
    return rc;
}

static int same_desc(const co_tensor *x, const co_tensor *y) {
    return x->type == y->type && x->layout == y->layout && x->rows == y->rows &&
           x->cols == y->cols && x->physical_rows == y->physical_rows &&
           x->physical_cols == y->physical_cols && x->atom == y->atom && x->bytes == y->bytes;
}

static int views_overlap(const co_view *a, const co_view *b) {
    uintptr_t pa = (uintptr_t)view_ptr(a), pb = (uintptr_t)view_ptr(b);
    return pa < pb + b->tensor.bytes && pb < pa + a->tensor.bytes;
}

int co_copy(co_view *dst, co_view *src) {
    if (!dst || !src || !valid_view(dst) || !valid_view(src) ||
        !same_desc(&dst->tensor, &src->tensor) || views_overlap(dst, src) ||
        dst->buffer->fd != src->buffer->fd)
        return ROCKET_E_SHAPE;
    b2_dev *d = b2h_dev(dst->buffer->fd);
    int rc = b2d_copy_2d(d, view_ptr(dst), dst->tensor.bytes, view_ptr(src), src->tensor.bytes,
                         src->tensor.bytes, 1, B2D_D2D);
    if (!rc) rc = b2d_sync(d);
    return rc;
}

int co_bias_upload(co_view *v, const _Float16 *bias) {
    if (!v || !bias || v->tensor.type != CO_F16 || v->tensor.layout != CO_CUBE) return ROCKET_E_SHAPE;
    _Float16 *a = malloc((size_t)v->tensor.rows * v->tensor.cols * 2);
    if (!a) return ROCKET_E_NOMEM;
    for (unsigned r = 0; r < v->tensor.rows; r++)
        memcpy(a + (size_t)r * v->tensor.cols, bias, (size_t)v->tensor.cols * 2);
    int rc = co_upload_f16(v, a);
    free(a);
    return rc;
}

int co_identity_upload(co_view *v) {
    if (!v || v->tensor.layout != CO_WEIGHT || v->tensor.rows != v->tensor.cols) return ROCKET_E_SHAPE;
    unsigned n = v->tensor.rows;
    _Float16 *a = calloc((size_t)n * n, 2);
    if (!a) return ROCKET_E_NOMEM;
    for (unsigned i = 0; i < n; i++) a[(size_t)i * n + i] = (_Float16)1.0f;
    int rc = co_upload_f16(v, a);
    free(a);
    return rc;
}

int co_ones_upload(co_view *v, unsigned k, int mean) {
    if (!v || !k || v->tensor.layout != CO_WEIGHT || v->tensor.rows != 16 || k != v->tensor.cols)
        return ROCKET_E_SHAPE;
    _Float16 *a = calloc((size_t)16 * k, 2);
    if (!a) return ROCKET_E_NOMEM;
    for (unsigned i = 0; i < k; i++) a[i] = (_Float16)(mean ? 1.0 / (double)k : 1.0);
    int rc = co_upload_f16(v, a);
    free(a);
    return rc;
}
