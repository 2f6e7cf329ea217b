/* ksplit.c -- fused K-split across GPUs, host side (one process per GPU).
 *
 * The reference has one NPU and accumulates K slices through FP16 ping-pong partials inside one
 * operator (research/custom-ops/src/custom_ops.c:297-330); its multi-core scheduler only picks a
 * core per submit (research/custom-ops/src/co_schedule.c). Here each rank's operator holds
 * W[:, k0:k1] (b2_shard_range), and a round adds the ranks' FP32 partials in the owner's memory:
 * see ksplit.cu for the device protocol. This file owns the per-rank buffer (allocated zeroed,
 * exported with CUDA IPC), checks that every rank declared the same layout before any peer
 * mapping is used, and drives the rounds.
 */
#include "b2_host.h"

#include <stdlib.h>
#include <string.h>

/* Exchange blob layout: [IPC handle 64][magic, world, rank, rows_per_rank u32][ldp u64][bytes u64]. */
#define BLOB_MAGIC 0x6b73706cu

struct b2_ksplit {
    b2_linear *op;
    unsigned world, rank, m_max, rows_per_rank;
    size_t ldp;
    void *buf;
    size_t bytes;
    void *peer[B2_KSPLIT_MAX_WORLD];
    int connected;
    b2_timer *timer;   /* phase marks of each round while timing is enabled */
};

static size_t ksplit_bytes(unsigned world, unsigned rpr, size_t ldp) {
    return 512 + 2 * (size_t)world * rpr * ldp * 4;
}

int b2_ksplit_create(b2_linear *op, unsigned world, unsigned rank, unsigned m_max, b2_ksplit **out) {
    if (!out) return ROCKET_E_SHAPE;
    *out = NULL;
    b2_linear_info info;
    if (!op || b2_linear_get_info(op, &info) || world < 1 || world > B2_KSPLIT_MAX_WORLD || rank >= world ||
        m_max < 1 || m_max > B2_MAX_DIM)
        return ROCKET_E_SHAPE;
    if (info.acc != B2_ACC_FP32) return ROCKET_E_UNSUPPORTED;   /* the FP16 fold is sequential in K */
    b2_ksplit *k = calloc(1, sizeof(*k));
    if (!k) return ROCKET_E_NOMEM;
    k->op = op;
    k->world = world;
    k->rank = rank;
    k->m_max = m_max;
    k->rows_per_rank = (unsigned)b2h_round_up((m_max + world - 1) / world, 32);   /* whole 32-row panels */
    k->ldp = b2h_round_up(info.n, 4);
    k->bytes = ksplit_bytes(world, k->rows_per_rank, k->ldp);
    int rc = b2h_malloc(b2h_linear_fd(op), k->bytes, &k->buf);   /* zero-filled: flags and seq start at 0 */
    if (rc) {
        free(k);
        return rc;
    }
    k->peer[rank] = k->buf;
    if (world == 1) k->connected = 1;
    *out = k;
    return 0;
}

int b2_ksplit_export(const b2_ksplit *k, unsigned char blob[B2_KSPLIT_BLOB_BYTES]) {
    if (!k || !blob) return ROCKET_E_SHAPE;
    memset(blob, 0, B2_KSPLIT_BLOB_BYTES);
    int rc = b2d_ipc_export(b2h_dev(b2h_linear_fd(k->op)), k->buf, blob);
    if (rc) return rc;
    const uint32_t head[4] = {BLOB_MAGIC, k->world, k->rank, k->rows_per_rank};
    const uint64_t tail[2] = {k->ldp, k->bytes};
    memcpy(blob + 64, head, sizeof(head));
    memcpy(blob + 80, tail, sizeof(tail));
    return 0;
}

static void close_peers(b2_ksplit *k) {
    b2_dev *d = b2h_dev(b2h_linear_fd(k->op));
    for (unsigned q = 0; q < k->world; ++q) {
        if (q != k->rank && k->peer[q]) b2d_ipc_close(d, k->peer[q]);
        if (q != k->rank) k->peer[q] = NULL;
    }
    k->connected = k->world == 1;
}

int b2_ksplit_connect(b2_ksplit *k, const unsigned char *blobs) {
    if (!k || !blobs) return ROCKET_E_SHAPE;
    if (k->world == 1) return 0;
    /* every rank must have declared this rank's layout: a peer that sized its buffer differently
     * would be written past its end */
    for (unsigned q = 0; q < k->world; ++q) {
        uint32_t head[4];
        uint64_t tail[2];
        memcpy(head, blobs + (size_t)q * B2_KSPLIT_BLOB_BYTES + 64, sizeof(head));
        memcpy(tail, blobs + (size_t)q * B2_KSPLIT_BLOB_BYTES + 80, sizeof(tail));
        if (head[0] != BLOB_MAGIC || head[1] != k->world || head[2] != q || head[3] != k->rows_per_rank ||
            tail[0] != k->ldp || tail[1] != k->bytes)
            return ROCKET_E_SHAPE;
    }
    close_peers(k);
    b2_dev *d = b2h_dev(b2h_linear_fd(k->op));
    for (unsigned q = 0; q < k->world; ++q) {
        if (q == k->rank) continue;
        int rc = b2d_ipc_open(d, blobs + (size_t)q * B2_KSPLIT_BLOB_BYTES, &k->peer[q]);
        if (rc) {
            close_peers(k);
            return rc;
        }
    }
    k->connected = 1;
    return 0;
}

int b2_ksplit_rows(const b2_ksplit *k, unsigned m, unsigned *row0, unsigned *rows) {
    if (!k || !row0 || !rows || m < 1 || m > k->m_max) return ROCKET_E_SHAPE;
    unsigned lo = k->rank * k->rows_per_rank, hi = lo + k->rows_per_rank;
    if (lo > m) lo = m;
    if (hi > m) hi = m;
    *row0 = lo;
    *rows = hi - lo;
    return 0;
}

int b2_ksplit_run(b2_ksplit *k, unsigned m, const void *x, size_t ldx, void *y, size_t ldy) {
    unsigned row0 = 0, rows = 0;
    if (!k || !k->connected || b2_ksplit_rows(k, m, &row0, &rows)) return ROCKET_E_SHAPE;
    if (m <= B2D_GEMV_MAX_M) return ROCKET_E_UNSUPPORTED;   /* the routed output is a GEMM epilogue */
    b2k_linear a;
    b2k_ksplit ks;
    if (b2h_linear_desc(k->op, m, x, ldx, &a)) return ROCKET_E_SHAPE;
    if (rows && (!y || ldy < a.n || ldy % 8 || ((uintptr_t)y & 15))) return ROCKET_E_SHAPE;
    memset(&ks, 0, sizeof(ks));
    ks.world = k->world;
    ks.rank = k->rank;
    ks.rows_per_rank = k->rows_per_rank;
    ks.own_rows = rows;
    ks.ldp = k->ldp;
    for (unsigned q = 0; q < k->world; ++q) ks.bufs[q] = k->peer[q];
    ks.bias = a.bias;
    ks.post = a.post;
    ks.y_own = rows ? (char *)y + (size_t)row0 * ldy * 2 : NULL;
    ks.ldy = ldy;
    ks.timer = k->timer;
    if (b2h_fault(B2_FAULT_LAUNCH)) return ROCKET_E_DEVICE;
    unsigned launches = 0;
    int rc = b2d_ksplit_round(b2h_dev(b2h_linear_fd(k->op)), &a, &ks, &launches);
    b2h_count_run(0, 0, launches);
    return rc;
}

int b2_ksplit_set_timing(b2_ksplit *k, int enable) {
    if (!k) return ROCKET_E_SHAPE;
    if (!enable) {
        b2d_timer_destroy(k->timer);
        k->timer = NULL;
        return 0;
    }
    if (k->timer) return 0;
    return b2d_timer_create(b2h_dev(b2h_linear_fd(k->op)), &k->timer);
}

int b2_ksplit_phase_ms(b2_ksplit *k, float ms[3]) {
    if (!k || !ms || !k->timer) return ROCKET_E_SHAPE;
    for (unsigned i = 0; i < 3; ++i) {
        int rc = b2d_timer_ms(k->timer, i, i + 1, &ms[i]);
        if (rc) return rc;
    }
    return 0;
}

void b2_ksplit_destroy(b2_ksplit *k) {
    if (!k) return;
    int fd = b2h_linear_fd(k->op);
    b2d_sync(b2h_dev(fd));
    b2d_timer_destroy(k->timer);
    close_peers(k);
    b2h_free(fd, k->buf, k->bytes);
    free(k);
}
