/* rkplan_oracle.c -- CPU restatement of the plan runtime's tile arithmetic (RKPlan ABI).
 *
 * TEST INFRASTRUCTURE ONLY: the checker of the plan tests and the arithmetic behind the CPU
 * stand-in of the device seam (tests/c/mock_device.c). The product library never links it.
 *
 * What it restates (paths relative to the reference project root, CO = research/custom-ops):
 *   CO/src/custom_ops.c:80-85 (co_index)   physical element of logical (r, c) per layout:
 *                                          CUBE ((c/8)*prows + r)*8 + c%8, WEIGHT
 *                                          (((r/16)*(pcols/32) + c/32)*16 + r%16)*32 + c%32,
 *                                          LINEAR r*pcols + c.
 *   CO/src/rk_plan_runtime.c:244-339       upload packing (pack_upload_into): the destination view
 *                                          is zeroed, then logical (r, c) receives
 *                                          src[(row_off + (T ? c : r)) * stride + col_off + (T ? r : c)],
 *                                          src[0] (scalar broadcast) or src[col_off + c] (channel).
 *   CO/tests/mock/npu_mock.c:392-537       the host model of the NPU programs the plan emits
 *                                          (rk_plan_emit.c:5-68): over the output's physical extent,
 *                                          MM / MM_ACC value = sum over q < x.physical_cols of
 *                                          double(x[r][q]) * double(w[c][q]) in q order (+ prior);
 *                                          EW pass = the same sum against the identity operand, then
 *                                          pass + b, pass * b, fmax(pass, b) or fmax(pass + b, 0);
 *                                          LUT sigmoid 1/(1+exp(-v)), hardsigmoid
 *                                          fmin(1, fmax(0, v/6 + 0.5)), GELU gate
 *                                          0.5*(1 + erf(v/sqrt 2)), rsqrt 1/sqrt(fmax(0.125, v));
 *                                          each result rounded once to FP16.
 *   CO/src/rk_plan_runtime.c:2036-2098     download: the view's logical rows x cols, row-major
 *                                          (co_download), published at the tile's offsets.
 * Pinned against the reference's own plan test (CO/tests/c/rk_plan_host_test.c:64-377): its
 * multi-tile MM expects, bit for bit, the double sum of the FP16 products rounded once
 * (rk_plan_host_test.c:232-238); tests/c/rk_plan_test.c checks the same case through this file.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

double oracle_f16_to_double(uint16_t h);
uint16_t oracle_f16_from_double(double d);

enum { RO_CUBE = 1, RO_WEIGHT = 2, RO_LINEAR = 3 };
enum {
    RO_MM = 1, RO_MM_ACC = 2, RO_EW_ADD = 3, RO_EW_MUL = 4, RO_LUT_SIGMOID = 5,
    RO_LUT_HARDSIGMOID = 6, RO_LUT_GELU_GATE = 7, RO_EW_MAX = 8, RO_EW_ADD_RELU = 9,
    RO_LUT_RSQRT = 10
};

/* One tile: FP16 words at p in `layout` with the given physical extent. */
typedef struct {
    uint16_t *p;
    unsigned layout, rows, cols, prows, pcols;
} rk_oracle_tile;

size_t rk_oracle_index(const rk_oracle_tile *t, unsigned r, unsigned c) {
    if (t->layout == RO_LINEAR) return (size_t)r * t->pcols + c;
    if (t->layout == RO_WEIGHT)
        return (((size_t)(r / 16) * (t->pcols / 32) + c / 32) * 16 + r % 16) * 32 + c % 32;
    return ((size_t)(c / 8) * t->prows + r) * 8 + c % 8;
}

static double lut(int op, double v) {
    switch (op) {
    case RO_LUT_SIGMOID: return 1.0 / (1.0 + exp(-v));
    case RO_LUT_HARDSIGMOID: return fmin(1.0, fmax(0.0, v / 6.0 + 0.5));
    case RO_LUT_GELU_GATE: return 0.5 * (1.0 + erf(v / sqrt(2.0)));
    default: return 1.0 / sqrt(fmax(0.125, v));
    }
}

/* The device task `op` (rk_template_id values). Returns -1 for an unknown op. */
int rk_oracle_task(int op, const rk_oracle_tile *x, const rk_oracle_tile *w, const rk_oracle_tile *aux,
                   rk_oracle_tile *y) {
    if (op == RO_LUT_SIGMOID || op == RO_LUT_HARDSIGMOID || op == RO_LUT_GELU_GATE || op == RO_LUT_RSQRT) {
        for (unsigned r = 0; r < y->prows; r++)
            for (unsigned c = 0; c < y->pcols; c++)
                y->p[rk_oracle_index(y, r, c)] =
                    oracle_f16_from_double(lut(op, oracle_f16_to_double(x->p[rk_oracle_index(x, r, c)])));
        return 0;
    }
    if (op < RO_MM || op > RO_EW_ADD_RELU) return -1;
    for (unsigned r = 0; r < y->prows; r++)
        for (unsigned c = 0; c < y->pcols; c++) {
            double s = 0;
            for (unsigned q = 0; q < x->pcols; q++)
                s += oracle_f16_to_double(x->p[rk_oracle_index(x, r, q)]) *
                     oracle_f16_to_double(w->p[rk_oracle_index(w, c, q)]);
            double b = op == RO_MM ? 0.0 : oracle_f16_to_double(aux->p[rk_oracle_index(aux, r, c)]);
            double v;
            switch (op) {
            case RO_MM: v = s; break;
            case RO_MM_ACC: case RO_EW_ADD: v = s + b; break;
            case RO_EW_MUL: v = s * b; break;
            case RO_EW_MAX: v = fmax(s, b); break;
            default: v = fmax(s + b, 0.0); break;
            }
            y->p[rk_oracle_index(y, r, c)] = oracle_f16_from_double(v);
        }
    return 0;
}

/* Upload packing into the rectangle [r0, r0+rows) x [c0, c0+cols); mode 0 matrix (src with pitch
 * ld, transposed reads when `transpose`), 1 scalar, 2 channel; `clear` zeroes the rest first. */
void rk_oracle_pack(rk_oracle_tile *dst, unsigned r0, unsigned c0, unsigned rows, unsigned cols, int clear,
                    int mode, int transpose, const uint16_t *src, size_t ld) {
    if (clear) memset(dst->p, 0, (size_t)dst->prows * dst->pcols * 2);
    for (unsigned i = 0; i < rows; i++)
        for (unsigned j = 0; j < cols; j++) {
            uint16_t v = mode == 1 ? src[0]
                       : mode == 2 ? src[j]
                                   : src[(size_t)(transpose ? j : i) * ld + (transpose ? i : j)];
            dst->p[rk_oracle_index(dst, r0 + i, c0 + j)] = v;
        }
}

/* Download: the logical rows x cols of src into row-major dst (pitch ld). */
void rk_oracle_unpack(const rk_oracle_tile *src, uint16_t *dst, size_t ld) {
    for (unsigned r = 0; r < src->rows; r++)
        for (unsigned c = 0; c < src->cols; c++) dst[(size_t)r * ld + c] = src->p[rk_oracle_index(src, r, c)];
}
