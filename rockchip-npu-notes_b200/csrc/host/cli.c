/* cli.c -- `linear_hardsigmoid`, the file-to-file operator CLI.
 *
 * Same contract as research/custom-ops/tools/c/operator_cli.c (reference project), which the
 * reference's file gate (tools/python/cli_gate.py) drives:
 *   usage      linear_hardsigmoid M K N X.bin W.bin b.bin Y.bin [chain|separate] [repeat]
 *   files      row-major little-endian IEEE FP16 X[M,K], W[N,K], b[N] -> Y[M,N], no header;
 *              each input must hold exactly its element count and only finite values
 *   limits     M, N in 1..4096, K in 1..CO_MAX_K, repeat in 1..1000; output path distinct from
 *              every input path
 *   exit       0 success, 1 error, 77 no device
 *   output     written through a temporary file and rename, only after every run succeeded;
 *              repeated runs must be byte-identical
 *   stdout     "OPERATOR HardSigmoid(XW^T+b) m= k= n= mode= repeat= submits=S tasks=T PASS"
 *              with the plan-derived counters the gate checks, followed by " launches=L", the
 *              CUDA kernels actually launched.
 * W and b are freed right after creation to show the operator copied them.
 */
#define _GNU_SOURCE
#include "b2_linear.h"

#include <errno.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

static void usage(const char *name) {
    printf("usage: %s M K N X.bin W.bin b.bin Y.bin [chain|separate] [repeat]\n", name);
    printf("row-major little-endian IEEE FP16: X[M,K], W[N,K], b[N], Y[M,N]\n");
    printf("M/N: 1..4096; K: 1..%u; repeat: 1..1000; default: chain, 1 run; CUDA device $B2_DEVICE "
           "(default 0); no CPU fallback\n",
           (unsigned)CO_MAX_K);
}

static int parse_dim(const char *s, unsigned max, unsigned *out) {
    if (!s || !*s || *s == '-' || *s == '+') return -1;
    errno = 0;
    char *end = NULL;
    unsigned long v = strtoul(s, &end, 10);
    if (errno || *end || !v || v > max) return -1;
    *out = (unsigned)v;
    return 0;
}

static int read_f16(const char *path, uint16_t *v, size_t n) {
    FILE *f = fopen(path, "rb");
    if (!f) {
        perror(path);
        return -1;
    }
    int ok = fread(v, 2, n, f) == n;
    if (ok) ok = fgetc(f) == EOF && !ferror(f);
    if (fclose(f)) ok = 0;
    if (!ok) {
        fprintf(stderr, "%s: expected exactly %zu FP16 elements\n", path, n);
        return -1;
    }
    for (size_t i = 0; i < n; i++)
        if ((v[i] & 0x7c00u) == 0x7c00u) {
            fprintf(stderr, "%s: nonfinite input at %zu\n", path, i);
            return -1;
        }
    return 0;
}

static int write_f16(const char *path, const uint16_t *v, size_t n) {
    size_t len = strlen(path) + 32;
    char *tmp = malloc(len);
    if (!tmp) return -1;
    snprintf(tmp, len, "%s.tmp.XXXXXX", path);
    int fd = mkstemp(tmp);
    if (fd < 0) {
        perror(path);
        free(tmp);
        return -1;
    }
    FILE *f = fdopen(fd, "wb");
    if (!f) {
        close(fd);
        unlink(tmp);
        free(tmp);
        return -1;
    }
    int ok = fwrite(v, 2, n, f) == n;
    if (fclose(f)) ok = 0;
    if (ok && rename(tmp, path)) {
        perror(path);
        ok = 0;
    }
    if (!ok) unlink(tmp);
    free(tmp);
    return ok ? 0 : -1;
}

int main(int argc, char **argv) {
    if (argc == 2 && !strcmp(argv[1], "--help")) {
        usage(argv[0]);
        return 0;
    }
    if (argc < 8 || argc > 10) {
        usage(argv[0]);
        return 1;
    }
    uint16_t probe = 1;
    if (*(unsigned char *)&probe != 1 || sizeof(_Float16) != 2) {
        fprintf(stderr, "requires a little-endian FP16 host\n");
        return 1;
    }
    unsigned m, k, n, repeats = 1;
    if (parse_dim(argv[1], CO_MAX_M, &m) || parse_dim(argv[2], CO_MAX_K, &k) ||
        parse_dim(argv[3], CO_MAX_N, &n) || (argc == 10 && parse_dim(argv[9], 1000, &repeats))) {
        usage(argv[0]);
        return 1;
    }
    enum co_mode mode = CO_CHAIN;
    if (argc >= 9) {
        if (!strcmp(argv[8], "separate")) mode = CO_SEPARATE;
        else if (strcmp(argv[8], "chain")) {
            usage(argv[0]);
            return 1;
        }
    }
    for (int i = 4; i < 7; i++)
        if (!strcmp(argv[i], argv[7])) {
            fprintf(stderr, "output must differ from input paths\n");
            return 1;
        }
    uint16_t *x = malloc((size_t)m * k * 2), *w = malloc((size_t)n * k * 2), *b = malloc((size_t)n * 2),
             *y = malloc((size_t)m * n * 2), *first = malloc((size_t)m * n * 2);
    int rc = 1, fd = -1;
    co_linear_hsig *op = NULL;
    if (!x || !w || !b || !y || !first) goto done;
    if (read_f16(argv[4], x, (size_t)m * k) || read_f16(argv[5], w, (size_t)n * k) || read_f16(argv[6], b, n))
        goto done;
    fd = rocket_open();
    if (fd < 0) {
        fprintf(stderr, "no CUDA device: %d\n", fd);
        rc = 77;
        goto done;
    }
    int status = co_linear_hsig_create(fd, m, k, n, (const _Float16 *)w, (const _Float16 *)b, mode, &op);
    if (status) {
        fprintf(stderr, "operator create: %d\n", status);
        goto done;
    }
    free(w);
    w = NULL;
    free(b);
    b = NULL;
    rocket_submit_counters_reset();
    for (unsigned i = 0; i < repeats; i++) {
        status = co_linear_hsig_run(op, (const _Float16 *)x, (_Float16 *)y);
        if (status) {
            fprintf(stderr, "operator run %u: %d\n", i, status);
            goto done;
        }
        if (!i) memcpy(first, y, (size_t)m * n * 2);
        else if (memcmp(first, y, (size_t)m * n * 2)) {
            fprintf(stderr, "repeated output differs\n");
            goto done;
        }
    }
    if (write_f16(argv[7], y, (size_t)m * n)) goto done;
    printf("OPERATOR HardSigmoid(XW^T+b) m=%u k=%u n=%u mode=%s repeat=%u submits=%llu tasks=%llu PASS "
           "launches=%llu\n",
           m, k, n, mode == CO_CHAIN ? "chain" : "separate", repeats,
           (unsigned long long)rocket_submit_ioctl_count(), (unsigned long long)rocket_submit_task_count(),
           (unsigned long long)rocket_launch_count());
    rc = 0;
done:
    co_linear_hsig_destroy(op);
    if (fd >= 0) rocket_close(fd);
    free(x);
    free(w);
    free(b);
    free(y);
    free(first);
    return rc;
}
