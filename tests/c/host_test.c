/* host_test.c -- the host C layer of the library against a CPU stand-in of the device seam.
 *
 * TEST INFRASTRUCTURE ONLY. Built from the library's own host sources (the C files of csrc/host), the mock
 * seam (tests/c/mock_device.c) and the oracle (oracle/linear_oracle.c), like the reference's host
 * tests built against its mock NPU (research/custom-ops/tests/c/multitile_host_test.c,
 * research/custom-ops/tests/mock/mock_npu.h:20-44 for the fail-Nth seam). Checks, on CPU:
 *   - co_linear_hsig_create/run publish Y equal to the reference arithmetic (oracle TILE16_EXACT),
 *     CO_CHAIN and CO_SEPARATE give identical bytes, ragged shapes, no bias;
 *   - FP32 operators (b2_linear_create) equal the oracle's FP32ACC model;
 *   - non-finite X or W -> ROCKET_E_SHAPE and Y untouched;
 *   - fail-Nth allocation -> ROCKET_E_NOMEM with no device bytes leaked; a refused launch or a
 *     reported non-finite output -> ROCKET_E_DEVICE with Y untouched;
 *   - co_linear_update_weights, the cube entry with the caller buffer's guard checked (a damaged
 *     slack byte -> ROCKET_E_DEVICE), the grouped device entry, a one-rank fused K-split round.
 * Prints "host_test: N checks, 0 failures" and exits 0 when everything holds.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "b2_host.h"
#include "custom_ops.h"

int oracle_linear(int mode, unsigned m, unsigned k, unsigned n, const uint16_t *x, const uint16_t *w,
                  const uint16_t *bias, int post, uint16_t *y16, double *act, double *raw, int threads);
uint16_t oracle_f16_from_double(double d);
enum { TILE16_EXACT = 0, FP32ACC = 5 };

static int checks, failures;
#define CHECK(cond, what)                                                           \
    do {                                                                            \
        ++checks;                                                                   \
        if (!(cond)) {                                                              \
            ++failures;                                                             \
            printf("FAIL %s:%d %s\n", __FILE__, __LINE__, what);                    \
        }                                                                           \
    } while (0)

static uint32_t rng = 12345u;
static double urand(void) {
    rng ^= rng << 13;
    rng ^= rng >> 17;
    rng ^= rng << 5;
    return (rng >> 8) / 16777216.0;
}
static void fill(uint16_t *v, size_t n, double scale) {
    for (size_t i = 0; i < n; i++) v[i] = oracle_f16_from_double((urand() * 2.0 - 1.0) * scale);
}
static uint16_t *alloc16(size_t n) { return calloc(n ? n : 1, 2); }

static void test_hsig_against_reference(int fd) {
    const unsigned m = 64, k = 512, n = 256;
    uint16_t *x = alloc16((size_t)m * k), *w = alloc16((size_t)n * k), *b = alloc16(n);
    uint16_t *ref = alloc16((size_t)m * n), *y1 = alloc16((size_t)m * n), *y2 = alloc16((size_t)m * n);
    fill(x, (size_t)m * k, 1.0);
    fill(w, (size_t)n * k, 1.0 / sqrt((double)k));
    fill(b, n, 0.1);
    CHECK(oracle_linear(TILE16_EXACT, m, k, n, x, w, b, 1, ref, NULL, NULL, 1) == 0, "oracle");
    co_linear_hsig *chain = NULL, *sep = NULL;
    CHECK(co_linear_hsig_create(fd, m, k, n, (const _Float16 *)w, (const _Float16 *)b, CO_CHAIN, &chain) == 0,
          "create chain");
    CHECK(co_linear_hsig_create(fd, m, k, n, (const _Float16 *)w, (const _Float16 *)b, CO_SEPARATE, &sep) == 0,
          "create separate");
    CHECK(co_linear_hsig_run(chain, (const _Float16 *)x, (_Float16 *)y1) == 0, "run chain");
    CHECK(co_linear_hsig_run(sep, (const _Float16 *)x, (_Float16 *)y2) == 0, "run separate");
    CHECK(memcmp(y1, ref, (size_t)m * n * 2) == 0, "chain equals the reference arithmetic");
    CHECK(memcmp(y2, y1, (size_t)m * n * 2) == 0, "separate equals chain");

    /* non-finite input: ROCKET_E_SHAPE, Y untouched */
    memset(y1, 0x5a, (size_t)m * n * 2);
    uint16_t keep = x[7];
    x[7] = 0x7c00u;
    CHECK(co_linear_hsig_run(chain, (const _Float16 *)x, (_Float16 *)y1) == ROCKET_E_SHAPE, "inf input refused");
    CHECK(y1[0] == 0x5a5au && y1[(size_t)m * n - 1] == 0x5a5au, "Y untouched after refused input");
    x[7] = keep;

    /* refused launch and reported non-finite output: ROCKET_E_DEVICE, Y untouched */
    b2_fault_inject(B2_FAULT_LAUNCH, 1);
    CHECK(co_linear_hsig_run(chain, (const _Float16 *)x, (_Float16 *)y1) == ROCKET_E_DEVICE, "launch fault");
    CHECK(y1[0] == 0x5a5au, "Y untouched after launch fault");
    b2_fault_inject(B2_FAULT_NAN_OUTPUT, 1);
    CHECK(co_linear_hsig_run(chain, (const _Float16 *)x, (_Float16 *)y1) == ROCKET_E_DEVICE, "nan-output fault");
    CHECK(y1[0] == 0x5a5au, "Y untouched after nan-output fault");
    CHECK(co_linear_hsig_run(chain, (const _Float16 *)x, (_Float16 *)y1) == 0, "runs again after faults");
    CHECK(memcmp(y1, ref, (size_t)m * n * 2) == 0, "same result after faults");

    /* weight refresh */
    fill(w, (size_t)n * k, 1.0 / sqrt((double)k));
    CHECK(oracle_linear(TILE16_EXACT, m, k, n, x, w, b, 1, ref, NULL, NULL, 1) == 0, "oracle 2");
    CHECK(co_linear_update_weights(chain, (const _Float16 *)w, (const _Float16 *)b) == 0, "update weights");
    CHECK(co_linear_hsig_run(chain, (const _Float16 *)x, (_Float16 *)y1) == 0, "run after update");
    CHECK(memcmp(y1, ref, (size_t)m * n * 2) == 0, "updated weights used");
    CHECK(co_linear_update_weights(chain, (const _Float16 *)w, NULL) == ROCKET_E_SHAPE, "bias presence is fixed");
    co_linear_hsig_destroy(chain);
    co_linear_hsig_destroy(sep);
    free(x); free(w); free(b); free(ref); free(y1); free(y2);
}

static void test_ragged_and_fp32(int fd) {
    const unsigned m = 17, k = 1000, n = 300;
    uint16_t *x = alloc16((size_t)m * k), *w = alloc16((size_t)n * k);
    uint16_t *ref = alloc16((size_t)m * n), *y = alloc16((size_t)m * n);
    fill(x, (size_t)m * k, 1.0);
    fill(w, (size_t)n * k, 1.0 / sqrt((double)k));
    co_linear *op = NULL;
    CHECK(co_linear_create(fd, m, k, n, (const _Float16 *)w, NULL, CO_LINEAR_NONE, CO_CHAIN, &op) == 0, "create ragged");
    CHECK(oracle_linear(TILE16_EXACT, m, k, n, x, w, NULL, 0, ref, NULL, NULL, 1) == 0, "oracle ragged");
    CHECK(co_linear_run(op, (const _Float16 *)x, (_Float16 *)y) == 0, "run ragged");
    CHECK(memcmp(y, ref, (size_t)m * n * 2) == 0, "ragged, no bias, equals the reference arithmetic");
    co_linear_destroy(op);

    b2_linear *op32 = NULL;
    CHECK(b2_linear_create(fd, m, k, n, (const _Float16 *)w, NULL, CO_LINEAR_NONE, CO_SEPARATE, B2_ACC_FP32, &op32) == 0,
          "create fp32");
    CHECK(oracle_linear(FP32ACC, m, k, n, x, w, NULL, 0, ref, NULL, NULL, 1) == 0, "oracle fp32");
    CHECK(co_linear_run(op32, (const _Float16 *)x, (_Float16 *)y) == 0, "run fp32");
    CHECK(memcmp(y, ref, (size_t)m * n * 2) == 0, "fp32 operator equals the FP32ACC model");

    /* device entries on mock "device" memory: grouped run equals the single runs */
    uint16_t *ya = alloc16((size_t)m * 304), *yb = alloc16((size_t)m * 304);
    uint16_t *xp = alloc16((size_t)m * 1000);
    memcpy(xp, x, (size_t)m * k * 2);
    CHECK(b2_linear_run_device(op32, m, xp, 1000, ya, 304) == 0, "run_device");
    b2_linear *ops[2] = {op32, op32};
    const void *xs[2] = {xp, xp};
    void *ys[2] = {yb, yb};
    size_t ldx[2] = {1000, 1000}, ldy[2] = {304, 304};
    CHECK(b2_linear_group_run_device(ops, 2, m, xs, ldx, ys, ldy) == 0, "group run");
    CHECK(memcmp(ya, yb, (size_t)m * 304 * 2) == 0, "group equals single run");
    CHECK(b2_linear_group_run_device(ops, 0, m, xs, ldx, ys, ldy) == ROCKET_E_SHAPE, "empty group refused");

    /* one-rank fused K-split round */
    b2_linear *opk = NULL;
    CHECK(b2_linear_create(fd, 1, k, n, (const _Float16 *)w, NULL, CO_LINEAR_NONE, CO_SEPARATE, B2_ACC_FP32, &opk) == 0,
          "create k-split operator");
    b2_ksplit *ks = NULL;
    CHECK(b2_ksplit_create(opk, 1, 0, 64, &ks) == 0, "k-split create");
    memset(yb, 0, (size_t)m * 304 * 2);
    CHECK(b2_ksplit_run(ks, m, xp, 1000, yb, 304) == 0, "k-split round");
    int same = 1;
    for (unsigned r = 0; r < m; r++) same &= memcmp(yb + (size_t)r * 304, ref + (size_t)r * n, (size_t)n * 2) == 0;
    CHECK(same, "k-split round equals the FP32ACC model");
    CHECK(b2_ksplit_run(ks, 8, xp, 1000, yb, 304) == ROCKET_E_UNSUPPORTED, "k-split needs m > 8");
    /* phase timing: refused before it is enabled, three intervals after a timed round, off again */
    float phase[3] = {-1.0f, -1.0f, -1.0f};
    CHECK(b2_ksplit_phase_ms(ks, phase) == ROCKET_E_SHAPE, "phase times need timing enabled");
    CHECK(b2_ksplit_set_timing(ks, 1) == 0 && b2_ksplit_set_timing(ks, 1) == 0, "timing enabled (idempotent)");
    CHECK(b2_ksplit_phase_ms(ks, phase) == ROCKET_E_SHAPE, "no phase times before a timed round");
    CHECK(b2_ksplit_run(ks, m, xp, 1000, yb, 304) == 0, "timed k-split round");
    CHECK(b2_ksplit_phase_ms(ks, phase) == 0 && phase[0] >= 0.0f && phase[1] >= 0.0f && phase[2] >= 0.0f,
          "phase times of the timed round");
    CHECK(b2_ksplit_set_timing(ks, 0) == 0 && b2_ksplit_phase_ms(ks, phase) == ROCKET_E_SHAPE, "timing disabled");
    CHECK(b2_ksplit_set_timing(ks, 1) == 0, "timing left on for destroy");
    b2_ksplit_destroy(ks);
    co_linear_destroy(opk);
    co_linear_destroy(op32);
    free(ya); free(yb); free(xp);
    free(x); free(w); free(ref); free(y);
}

/* Large host-buffer runs copy X in row bands on a side stream (2 bands at 1100 rows, 8 at 4096; X of
 * 8 MiB or more):
 * the result equals the reference arithmetic and the unbanded CO_SEPARATE run, and a non-finite
 * element in the first or the last band is refused with Y untouched. */
static void test_banded_host_run(int fd) {
    static const unsigned shapes[2][3] = {{1100, 4096, 16}, {4096, 1024, 8}};
    for (int s = 0; s < 2; s++) {
        const unsigned m = shapes[s][0], k = shapes[s][1], n = shapes[s][2];
        uint16_t *x = alloc16((size_t)m * k), *w = alloc16((size_t)n * k), *b = alloc16(n);
        uint16_t *ref = alloc16((size_t)m * n), *y1 = alloc16((size_t)m * n), *y2 = alloc16((size_t)m * n);
        fill(x, (size_t)m * k, 1.0);
        fill(w, (size_t)n * k, 1.0 / sqrt((double)k));
        fill(b, n, 0.1);
        CHECK(oracle_linear(TILE16_EXACT, m, k, n, x, w, b, 1, ref, NULL, NULL, 4) == 0, "oracle banded");
        co_linear_hsig *chain = NULL, *sep = NULL;
        CHECK(co_linear_hsig_create(fd, m, k, n, (const _Float16 *)w, (const _Float16 *)b, CO_CHAIN, &chain) == 0,
              "create banded chain");
        CHECK(co_linear_hsig_create(fd, m, k, n, (const _Float16 *)w, (const _Float16 *)b, CO_SEPARATE, &sep) == 0,
              "create unbanded separate");
        CHECK(co_linear_hsig_run(chain, (const _Float16 *)x, (_Float16 *)y1) == 0, "banded run");
        CHECK(co_linear_hsig_run(sep, (const _Float16 *)x, (_Float16 *)y2) == 0, "unbanded run");
        CHECK(memcmp(y1, ref, (size_t)m * n * 2) == 0, "banded run equals the reference arithmetic");
        CHECK(memcmp(y2, y1, (size_t)m * n * 2) == 0, "banded equals unbanded");
        const size_t bad[2] = {3, (size_t)(m - 1) * k + k / 2};   /* first band, last band */
        for (int i = 0; i < 2; i++) {
            memset(y1, 0x5a, (size_t)m * n * 2);
            const uint16_t keep = x[bad[i]];
            x[bad[i]] = 0x7e00u;   /* NaN */
            CHECK(co_linear_hsig_run(chain, (const _Float16 *)x, (_Float16 *)y1) == ROCKET_E_SHAPE,
                  "NaN in a band refused");
            CHECK(y1[0] == 0x5a5au && y1[(size_t)m * n - 1] == 0x5a5au, "Y untouched after a refused band");
            x[bad[i]] = keep;
        }
        CHECK(co_linear_hsig_run(chain, (const _Float16 *)x, (_Float16 *)y1) == 0 &&
                  memcmp(y1, ref, (size_t)m * n * 2) == 0,
              "banded run again after refusals");
        co_linear_hsig_destroy(chain);
        co_linear_hsig_destroy(sep);
        free(x); free(w); free(b); free(ref); free(y1); free(y2);
    }
}

static void test_create_failures(int fd) {
    const unsigned m = 32, k = 64, n = 64;
    uint16_t *w = alloc16((size_t)n * k), *b = alloc16(n);
    fill(w, (size_t)n * k, 0.1);
    co_linear_hsig *op = NULL;
    const size_t live = b2h_live_bytes();
    for (unsigned nth = 1; nth <= 4; nth++) {
        b2_fault_inject(B2_FAULT_ALLOC, nth);
        CHECK(co_linear_hsig_create(fd, m, k, n, (const _Float16 *)w, (const _Float16 *)b, CO_CHAIN, &op) ==
                  ROCKET_E_NOMEM && op == NULL,
              "fail-Nth allocation -> NOMEM");
        CHECK(b2h_live_bytes() == live, "no device bytes leaked");
    }
    b2_fault_inject(B2_FAULT_NONE, 1);
    w[3] = 0x7e00u;   /* NaN weight */
    CHECK(co_linear_hsig_create(fd, m, k, n, (const _Float16 *)w, (const _Float16 *)b, CO_CHAIN, &op) == ROCKET_E_SHAPE,
          "non-finite W refused");
    CHECK(co_linear_hsig_create(fd, m, k, n, (const _Float16 *)w, NULL, CO_CHAIN, &op) == ROCKET_E_SHAPE,
          "hsig without bias refused");
    CHECK(co_linear_hsig_create(fd, 4097, k, n, (const _Float16 *)w, (const _Float16 *)b, CO_CHAIN, &op) ==
              ROCKET_E_SHAPE,
          "reference M limit");
    free(w);
    free(b);
}

static void test_cube_entry_and_guard(int fd) {
    const unsigned m = 40, k = 96, n = 72;
    uint16_t *x = alloc16((size_t)m * k), *w = alloc16((size_t)n * k), *b = alloc16(n);
    uint16_t *ref = alloc16((size_t)m * n), *y = alloc16((size_t)m * n);
    fill(x, (size_t)m * k, 1.0);
    fill(w, (size_t)n * k, 0.1);
    fill(b, n, 0.1);
    CHECK(oracle_linear(TILE16_EXACT, m, k, n, x, w, b, 1, ref, NULL, NULL, 1) == 0, "oracle cube");
    co_linear_hsig *op = NULL;
    CHECK(co_linear_hsig_create(fd, m, k, n, (const _Float16 *)w, (const _Float16 *)b, CO_CHAIN, &op) == 0, "create");
    co_tensor tx, ty;
    CHECK(co_tensor_input(&tx, m, k) == 0 && co_tensor_matrix(&ty, m, n, CO_F16) == 0, "descriptors");
    co_buffer bx, by;
    CHECK(co_buffer_alloc(fd, tx.bytes, &bx) == 0 && co_buffer_alloc(fd, ty.bytes + 16, &by) == 0, "buffers");
    co_view vx, vy;
    CHECK(co_view_init(&vx, &bx, 0, &tx) == 0 && co_view_init(&vy, &by, 16, &ty) == 0, "views");
    CHECK(co_upload_f16(&vx, (const _Float16 *)x) == 0, "upload");
    CHECK(co_linear_hsig_run_cube(op, vx, vy) == 0, "run cube");
    CHECK(co_download(&vy, y) == 0, "download");
    CHECK(memcmp(y, ref, (size_t)m * n * 2) == 0, "cube entry equals the reference arithmetic");
    CHECK(co_guard_check(&by) == 0, "guard intact");
    /* a refused launch on the direct cube path: ROCKET_E_DEVICE, then the next run succeeds */
    b2_fault_inject(B2_FAULT_LAUNCH, 1);
    CHECK(co_linear_hsig_run_cube(op, vx, vy) == ROCKET_E_DEVICE, "cube launch fault");
    CHECK(co_linear_hsig_run_cube(op, vx, vy) == 0, "cube runs again after the fault");
    /* K = 100 leaves a partial 8-channel atom: the gather -> GEMM -> scatter form, same arithmetic */
    {
        const unsigned k2 = 100;
        uint16_t *x2 = alloc16((size_t)m * k2), *w2 = alloc16((size_t)n * k2), *ref2 = alloc16((size_t)m * n);
        fill(x2, (size_t)m * k2, 1.0);
        fill(w2, (size_t)n * k2, 0.1);
        CHECK(oracle_linear(TILE16_EXACT, m, k2, n, x2, w2, b, 1, ref2, NULL, NULL, 1) == 0, "oracle cube k=100");
        co_linear_hsig *op2 = NULL;
        CHECK(co_linear_hsig_create(fd, m, k2, n, (const _Float16 *)w2, (const _Float16 *)b, CO_CHAIN, &op2) == 0,
              "create k=100");
        co_tensor tx2;
        co_buffer bx2;
        co_view vx2;
        CHECK(co_tensor_input(&tx2, m, k2) == 0 && co_buffer_alloc(fd, tx2.bytes, &bx2) == 0 &&
                  co_view_init(&vx2, &bx2, 0, &tx2) == 0 && co_upload_f16(&vx2, (const _Float16 *)x2) == 0,
              "k=100 input view");
        CHECK(co_linear_hsig_run_cube(op2, vx2, vy) == 0, "run cube k=100");
        CHECK(co_download(&vy, y) == 0 && memcmp(y, ref2, (size_t)m * n * 2) == 0,
              "ragged-K cube entry equals the reference arithmetic");
        co_buffer_free(&bx2);
        co_linear_hsig_destroy(op2);
        free(x2); free(w2); free(ref2);
    }
    /* aliasing: an output sharing bytes with the input is refused before any launch; inputs may
     * share bytes with each other (run_tiled: two K-tile views of one matrix buffer) */
    {
        co_view bad = vy;
        bad.buffer = &bx;
        bad.offset = 0;
        co_tensor tyy;
        CHECK(co_tensor_matrix(&tyy, m, n, CO_F16) == 0, "alias descriptor");
        bad.tensor = tyy;
        CHECK(bx.payload >= tyy.bytes, "alias view fits");
        CHECK(co_linear_hsig_run_cube(op, vx, bad) == ROCKET_E_SHAPE, "output over the input refused");
    }
    /* a byte of the output buffer's slack is damaged: the run reports it */
    ((unsigned char *)by.bo.ptr)[by.payload + 5] = 1;
    CHECK(co_linear_hsig_run_cube(op, vx, vy) == ROCKET_E_DEVICE, "damaged slack -> DEVICE");
    CHECK(co_guard_check(&by) == ROCKET_E_DEVICE, "co_guard_check sees it");
    co_buffer_free(&bx);
    co_buffer_free(&by);
    co_linear_hsig_destroy(op);
    free(x); free(w); free(b); free(ref); free(y);
}

int main(void) {
    int fd = rocket_open();
    CHECK(fd >= 0, "rocket_open on the mock device");
    if (fd < 0) return 1;
    test_hsig_against_reference(fd);
    test_ragged_and_fp32(fd);
    test_banded_host_run(fd);
    test_create_failures(fd);
    test_cube_entry_and_guard(fd);
    rocket_close(fd);
    CHECK(b2h_live_bytes() == 0, "every device byte freed");
    printf("host_test: %d checks, %d failures\n", checks, failures);
    return failures ? 1 : 0;
}
