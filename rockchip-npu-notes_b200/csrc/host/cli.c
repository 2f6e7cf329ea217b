/* cli.c -- `linear_hardsigmoid`: file-to-file HardSigmoid(X·Wᵀ + b) on one B200.
 *
 * The behaviour is the reference's operator CLI contract, the one its file gate checks
 * (research/custom-ops/tools/python/cli_gate.py:55-114, driving
 * research/custom-ops/tools/c/operator_cli.c):
 *   arguments  M K N X.bin W.bin b.bin Y.bin [chain|separate] [repeat]
 *              M, N in 1..4096, K in 1..CO_MAX_K, repeat in 1..1000 (default chain, 1 run);
 *              the output path must differ from every input path
 *   files      headerless row-major little-endian IEEE FP16: X[M,K], W[N,K], b[N] -> Y[M,N];
 *              an input must hold exactly its element count, all finite
 *   exit       0 success, 1 any error, 77 when no CUDA device can be opened (inputs are
 *              validated first, so a bad input is 1 even without a device)
 *   output     published only after every run succeeded and every run gave the same bytes,
 *              by renaming a fully written sibling file over Y (an existing Y is never touched
 *              on failure)
 *   stdout     "OPERATOR HardSigmoid(XW^T+b) m= k= n= mode= repeat= submits=S tasks=T PASS",
 *              S and T being the plan-derived counters the gate checks, then " launches=L", the
 *              CUDA kernels actually launched (after PASS, so the gate's pattern still matches).
 *
 * How this program does it: argv is parsed into a `job` through a table of the positional
 * dimensions; each input is mapped read-only after fstat has shown its exact size; finiteness is
 * checked four halves per 64-bit word; W and b are unmapped as soon as the operator has been
 * created (any later use of them by the library would fault, so the operator must own copies);
 * runs alternate between two output buffers and each is compared with the run before it.
 */
#define _GNU_SOURCE
#include "b2_linear.h"

#include <errno.h>
#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#if !defined(__BYTE_ORDER__) || __BYTE_ORDER__ != __ORDER_LITTLE_ENDIAN__
#error "the FP16 file format is little-endian; this host is not"
#endif
_Static_assert(sizeof(_Float16) == 2, "IEEE binary16 _Float16 required");

enum { EXIT_PASS = 0, EXIT_FAIL = 1, EXIT_NO_DEVICE = 77 };
enum { MAX_REPEAT = 1000 };

typedef struct {
    unsigned m, k, n, repeat;
    enum co_mode mode;
    const char *in_path[3]; /* X, W, b */
    const char *out_path;
} job;

/* A read-only mapping of one input file holding exactly `count` FP16 values. */
typedef struct {
    const uint16_t *data;
    size_t count;
} fp16_file;

static void print_usage(FILE *to, const char *prog) {
    fprintf(to,
            "usage: %s M K N X.bin W.bin b.bin Y.bin [chain|separate] [repeat]\n"
            "  computes Y = HardSigmoid(X W^T + b) on a CUDA device ($B2_DEVICE, default 0)\n"
            "  files: headerless row-major little-endian FP16, X[M,K] W[N,K] b[N] Y[M,N]\n"
            "  limits: M,N <= 4096, K <= %u, repeat <= %d; defaults: chain, repeat 1\n",
            prog, (unsigned)CO_MAX_K, MAX_REPEAT);
}

/* Decimal integer in [1, max], nothing but digits. */
static int parse_count(const char *text, unsigned max, unsigned *value) {
    unsigned long long v = 0;
    if (!text[0]) return -1;
    for (const char *p = text; *p; p++) {
        if (*p < '0' || *p > '9') return -1;
        v = v * 10 + (unsigned)(*p - '0');
        if (v > max) return -1;
    }
    if (v == 0) return -1;
    *value = (unsigned)v;
    return 0;
}

/* Returns 0 and fills *j, or -1 when argv does not describe a valid job. */
static int parse_job(int argc, char **argv, job *j) {
    if (argc < 8 || argc > 10) return -1;
    const struct {
        unsigned max;
        unsigned *field;
    } dims[3] = {{CO_MAX_M, &j->m}, {CO_MAX_K, &j->k}, {CO_MAX_N, &j->n}};
    for (int i = 0; i < 3; i++)
        if (parse_count(argv[1 + i], dims[i].max, dims[i].field)) return -1;
    for (int i = 0; i < 3; i++) j->in_path[i] = argv[4 + i];
    j->out_path = argv[7];
    j->mode = CO_CHAIN;
    j->repeat = 1;
    if (argc > 8) {
        if (strcmp(argv[8], "chain") == 0) j->mode = CO_CHAIN;
        else if (strcmp(argv[8], "separate") == 0) j->mode = CO_SEPARATE;
        else return -1;
    }
    if (argc > 9 && parse_count(argv[9], MAX_REPEAT, &j->repeat)) return -1;
    return 0;
}

/* Index of the first half whose exponent field is all ones (Inf or NaN), or `count` if none.
 * Four halves are tested per 64-bit word: a lane of `e ^ EXP` is zero exactly when that half is
 * not finite, and the classic zero-lane test finds such a lane without a per-half branch. */
static size_t first_nonfinite(const uint16_t *v, size_t count) {
    const uint64_t EXP = 0x7c007c007c007c00ull, ONE = 0x0001000100010001ull, TOP = 0x8000800080008000ull;
    size_t i = 0;
    for (; i + 4 <= count; i += 4) {
        uint64_t w;
        memcpy(&w, v + i, 8);
        uint64_t t = (w & EXP) ^ EXP; /* bit 15 of every lane is clear */
        if ((t - ONE) & ~t & TOP) break;
    }
    for (; i < count; i++)
        if ((v[i] & 0x7c00u) == 0x7c00u) return i;
    return count;
}

static void unmap(fp16_file *f) {
    if (f->data) munmap((void *)f->data, f->count * 2);
    f->data = NULL;
}

static int map_input(const char *path, size_t count, fp16_file *f) {
    f->data = NULL;
    f->count = count;
    int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) {
        fprintf(stderr, "%s: cannot open: %s\n", path, strerror(errno));
        return -1;
    }
    struct stat st;
    int rc = fstat(fd, &st);
    if (rc || !S_ISREG(st.st_mode) || (unsigned long long)st.st_size != (unsigned long long)count * 2) {
        fprintf(stderr, "%s: must hold exactly %zu FP16 values (%zu bytes)\n", path, count, count * 2);
        close(fd);
        return -1;
    }
    void *p = mmap(NULL, count * 2, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (p == MAP_FAILED) {
        fprintf(stderr, "%s: cannot map: %s\n", path, strerror(errno));
        return -1;
    }
    f->data = p;
    size_t bad = first_nonfinite(f->data, count);
    if (bad != count) {
        fprintf(stderr, "%s: value %zu is not finite\n", path, bad);
        unmap(f);
        return -1;
    }
    return 0;
}

/* Writes `bytes` to a new sibling of `path` and renames it over `path`. */
static int publish(const char *path, const void *data, size_t bytes) {
    size_t cap = strlen(path) + 48;
    char *tmp = malloc(cap);
    if (!tmp) return -1;
    int fd = -1;
    for (unsigned attempt = 0; attempt < 64 && fd < 0; attempt++) {
        snprintf(tmp, cap, "%s.partial-%ld-%u", path, (long)getpid(), attempt);
        fd = open(tmp, O_WRONLY | O_CREAT | O_EXCL | O_CLOEXEC, 0666);
        if (fd < 0 && errno != EEXIST) break;
    }
    if (fd < 0) {
        fprintf(stderr, "%s: cannot create the output: %s\n", path, strerror(errno));
        free(tmp);
        return -1;
    }
    const char *p = data;
    size_t left = bytes;
    int ok = 1;
    while (ok && left) {
        ssize_t got = write(fd, p, left);
        if (got < 0 && errno == EINTR) continue;
        if (got <= 0) ok = 0;
        else {
            p += got;
            left -= (size_t)got;
        }
    }
    if (close(fd)) ok = 0;
    if (ok && rename(tmp, path)) ok = 0;
    if (!ok) {
        fprintf(stderr, "%s: cannot write the output: %s\n", path, strerror(errno));
        unlink(tmp);
    }
    free(tmp);
    return ok ? 0 : -1;
}

/* Creates the operator on device `fd`, drops W and b, runs it j->repeat times and leaves the
 * last output in *result (one of the two buffers in y). Returns EXIT_PASS or EXIT_FAIL. */
static int execute(const job *j, int fd, fp16_file *in, uint16_t *y[2], uint16_t **result) {
    co_linear_hsig *op = NULL;
    int rc = co_linear_hsig_create(fd, j->m, j->k, j->n, (const _Float16 *)in[1].data,
                                   (const _Float16 *)in[2].data, j->mode, &op);
    unmap(&in[1]);
    unmap(&in[2]);
    if (rc) {
        fprintf(stderr, "creating the operator failed: status %d\n", rc);
        return EXIT_FAIL;
    }
    size_t out_bytes = (size_t)j->m * j->n * 2;
    int verdict = EXIT_PASS;
    rocket_submit_counters_reset();
    for (unsigned r = 0; r < j->repeat && verdict == EXIT_PASS; r++) {
        uint16_t *cur = y[r & 1];
        rc = co_linear_hsig_run(op, (const _Float16 *)in[0].data, (_Float16 *)cur);
        if (rc) {
            fprintf(stderr, "run %u of %u failed: status %d\n", r + 1, j->repeat, rc);
            verdict = EXIT_FAIL;
        } else if (r && memcmp(cur, y[(r - 1) & 1], out_bytes)) {
            fprintf(stderr, "run %u gave different bytes from run %u\n", r + 1, r);
            verdict = EXIT_FAIL;
        }
        *result = cur;
    }
    co_linear_hsig_destroy(op);
    return verdict;
}

int main(int argc, char **argv) {
    if (argc == 2 && strcmp(argv[1], "--help") == 0) {
        print_usage(stdout, argv[0]);
        return EXIT_PASS;
    }
    job j;
    if (parse_job(argc, argv, &j)) {
        print_usage(stderr, argv[0]);
        return EXIT_FAIL;
    }
    for (int i = 0; i < 3; i++)
        if (strcmp(j.in_path[i], j.out_path) == 0) {
            fprintf(stderr, "%s: the output may not overwrite an input\n", j.out_path);
            return EXIT_FAIL;
        }

    const size_t counts[3] = {(size_t)j.m * j.k, (size_t)j.n * j.k, j.n};
    fp16_file in[3] = {{0}};
    int status = EXIT_PASS;
    for (int i = 0; i < 3 && status == EXIT_PASS; i++)
        if (map_input(j.in_path[i], counts[i], &in[i])) status = EXIT_FAIL;

    uint16_t *y[2] = {NULL, NULL}, *result = NULL;
    int fd = -1;
    if (status == EXIT_PASS) {
        y[0] = malloc((size_t)j.m * j.n * 2);
        y[1] = malloc((size_t)j.m * j.n * 2);
        if (!y[0] || !y[1]) {
            fprintf(stderr, "out of host memory\n");
            status = EXIT_FAIL;
        }
    }
    if (status == EXIT_PASS) {
        fd = rocket_open();
        if (fd < 0) {
            fprintf(stderr, "no usable CUDA device (status %d)\n", fd);
            status = EXIT_NO_DEVICE;
        }
    }
    if (status == EXIT_PASS) status = execute(&j, fd, in, y, &result);
    if (status == EXIT_PASS && publish(j.out_path, result, (size_t)j.m * j.n * 2)) status = EXIT_FAIL;
    if (status == EXIT_PASS)
        printf("OPERATOR HardSigmoid(XW^T+b) m=%u k=%u n=%u mode=%s repeat=%u submits=%llu tasks=%llu PASS "
               "launches=%llu\n",
               j.m, j.k, j.n, j.mode == CO_CHAIN ? "chain" : "separate", j.repeat,
               (unsigned long long)rocket_submit_ioctl_count(), (unsigned long long)rocket_submit_task_count(),
               (unsigned long long)rocket_launch_count());

    if (fd >= 0) rocket_close(fd);
    for (int i = 0; i < 3; i++) unmap(&in[i]);
    free(y[0]);
    free(y[1]);
    return status;
}
