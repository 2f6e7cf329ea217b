/* graph_oracle.c -- CPU restatement of the reference's graph node arithmetic (non-Linear nodes).
 *
 * TEST INFRASTRUCTURE ONLY: the checker of the graph tests (and of the CPU stand-in of the device
 * seam used by the host C tests). The product library never links it and never falls back to it.
 *
 * What it restates (paths relative to the reference project root, CO = research/custom-ops):
 *   CO/src/custom_ops.c:357-369        the functions the LUT activations sample: HardSigmoid
 *                                      clamp(v/6 + 0.5, 0, 1), sigmoid 1/(1+exp(-v)), GELU gate
 *                                      0.5*(1+erf(v/sqrt 2)); each is evaluated exactly (double,
 *                                      libm) and rounded once to FP16 instead of being read from a
 *                                      513-entry Q0.15 table with hardware interpolation.
 *   CO/src/co_graph.c:293-313          node semantics: ADD/MUL = fp16(a op b) (co_emit_ew),
 *                                      HSIG = fp16(hsig(a)), SILU/GELU = fp16(a * fp16(gate(a)))
 *                                      (LUT into a gate buffer, then an EW multiply).
 *   CO/tools/python/graph_gate.py:22-41  the reference's own FFN oracle: the same node arithmetic
 *                                      (gated = f16(f16(a*f16(1/(1+exp(-a))))*b), residual
 *                                      f16(x + down)); its RMSNorm divides differently, see below.
 *   CO/src/co_row_ops.c:150-224        RMSNorm as run by the reference: per 256-column tile the
 *                                      FP32 statistic of the FP16 squares fp16(x*x) (here the
 *                                      exact sum rounded once to FP32, which is what
 *                                      graph_gate.py's math.fsum + float32 pack computes), a tile
 *                                      statistic >= 65504 or non-finite rejects the row
 *                                      (ROCKET_E_SHAPE); the statistics are summed in double;
 *                                      coefficient fp16((double)gamma / sqrt(sum/cols + eps)) with
 *                                      eps the node's float, non-finite -> rejected; y = fp16(x*c).
 *                                      graph_gate.py instead forms fp16(gamma * (1/sqrt(total/d +
 *                                      1e-5))): the two agree to within one FP16 rounding of the
 *                                      coefficient, inside the gate's 0.003 tolerance.
 * The FP16 rounding of a double is oracle_f16_from_double (linear_oracle.c): round to nearest even,
 * directly from the double, as Python's struct 'e' format and C's (_Float16) cast do.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

double oracle_f16_to_double(uint16_t h);
uint16_t oracle_f16_from_double(double d);

enum { OG_ADD = 0, OG_MUL = 1, OG_SILU = 2, OG_GELU = 3, OG_HSIG = 4 };
enum { OG_GATE_SIGMOID = 1, OG_GATE_GELU = 2 };

static double f16v(uint16_t h) { return oracle_f16_to_double(h); }

/* FP16 bits of the activation gate of FP16 input a. */
uint16_t oracle_gate16(int act, uint16_t a) {
    const double v = f16v(a);
    const double g = act == OG_GATE_GELU ? 0.5 * (1.0 + erf(v / sqrt(2.0))) : 1.0 / (1.0 + exp(-v));
    return oracle_f16_from_double(g);
}

/* SiLU / GELU node value: fp16(a * fp16(gate(a))). */
uint16_t oracle_act16(int act, uint16_t a) {
    return oracle_f16_from_double(f16v(a) * f16v(oracle_gate16(act, a)));
}

static double hsig(double v) {
    const double t = v / 6.0 + 0.5;
    return t < 0.0 ? 0.0 : (t > 1.0 ? 1.0 : t);
}

/* One elementwise node value (OG_*); b is read only by ADD and MUL. */
uint16_t oracle_ew16(int op, uint16_t a, uint16_t b) {
    switch (op) {
        case OG_ADD: return oracle_f16_from_double(f16v(a) + f16v(b));
        case OG_MUL: return oracle_f16_from_double(f16v(a) * f16v(b));
        case OG_SILU: return oracle_act16(OG_GATE_SIGMOID, a);
        case OG_GELU: return oracle_act16(OG_GATE_GELU, a);
        default: return oracle_f16_from_double(hsig(f16v(a)));
    }
}

/* Elementwise node over n values. */
void oracle_ew(int op, const uint16_t *a, const uint16_t *b, uint16_t *y, size_t n) {
    for (size_t i = 0; i < n; i++) y[i] = oracle_ew16(op, a[i], b ? b[i] : 0);
}

/* Exact sum of FP16 squares (each a multiple of 2^-24 below 2^16) rounded once to FP32; returns
 * infinity when a square overflows FP16. */
static float tile_statistic(const uint16_t *x, unsigned len) {
    int64_t q = 0;
    for (unsigned i = 0; i < len; i++) {
        const double v = f16v(x[i]);
        const uint16_t s = oracle_f16_from_double(v * v);
        if ((s & 0x7c00u) == 0x7c00u) return INFINITY;
        q += (int64_t)ldexp(f16v(s), 24);
    }
    return (float)ldexp((double)q, -24);   /* q < 2^48: exact in double, one rounding to float */
}

/* RMSNorm of rows x cols (contiguous). Returns the number of rejected rows; a rejected row of y
 * is left untouched. */
unsigned oracle_rmsnorm(unsigned rows, unsigned cols, const uint16_t *x, const uint16_t *gamma, float eps,
                        uint16_t *y) {
    unsigned rejected = 0;
    for (unsigned r = 0; r < rows; r++) {
        const uint16_t *xr = x + (size_t)r * cols;
        double sum = 0.0;
        int bad = 0;
        for (unsigned c0 = 0; c0 < cols; c0 += 256) {
            const float st = tile_statistic(xr + c0, cols - c0 < 256 ? cols - c0 : 256);
            if (!(st < 65504.0f)) bad = 1;
            sum += st;
        }
        const double scale = sqrt(sum / cols + (double)eps);
        for (unsigned c = 0; c < cols && !bad; c++) {
            const uint16_t k = oracle_f16_from_double(f16v(gamma[c]) / scale);
            if ((k & 0x7c00u) == 0x7c00u) bad = 1;
        }
        if (bad) {
            rejected++;
            continue;
        }
        for (unsigned c = 0; c < cols; c++) {
            const uint16_t k = oracle_f16_from_double(f16v(gamma[c]) / scale);
            y[(size_t)r * cols + c] = oracle_f16_from_double(f16v(xr[c]) * f16v(k));
        }
    }
    return rejected;
}
