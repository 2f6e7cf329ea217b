/* rocket.c -- device handles, buffer objects, counters and the fault-injection seam.
 *
 * Replaces the provider calls the reference's Linear path makes into rknpu-submit
 * (rocket_open/close, rocket_bo_alloc32/free, rocket_batched_submit_supported and the submit
 * counters; uses at research/custom-ops/src/custom_ops.c:86-101 and
 * research/custom-ops/tools/c/operator_cli.c:75-91). A handle names one CUDA device and one
 * stream; the table is process-global and, like the reference's contexts, not thread-safe.
 */
#include "b2_host.h"

#include <stdlib.h>
#include <string.h>

static b2_dev *fds[B2_MAX_FDS];
static unsigned long long n_submits, n_tasks, n_launches;
static size_t live_bytes;
static uint32_t next_handle = 1;

static enum b2_fault fault_kind;
static unsigned fault_countdown;

b2_dev *b2h_dev(int fd) { return (fd >= 0 && fd < B2_MAX_FDS) ? fds[fd] : NULL; }
int b2h_valid_fd(int fd) { return b2h_dev(fd) != NULL; }

int b2_device_count(void) { return b2d_device_count(); }

int b2_open_device(int ordinal) {
    int slot = -1;
    for (int i = 0; i < B2_MAX_FDS; i++) if (!fds[i]) { slot = i; break; }
    if (slot < 0) return ROCKET_E_NOMEM;
    b2_dev *d = NULL;
    int rc = b2d_open(ordinal, &d);
    if (rc) return rc;
    fds[slot] = d;
    return slot;
}

int rocket_open(void) {
    const char *env = getenv("B2_DEVICE");
    int ordinal = env && *env ? atoi(env) : 0;
    if (ordinal < 0 || ordinal >= b2d_device_count()) return ROCKET_E_DEVICE;
    return b2_open_device(ordinal);
}

void rocket_close(int fd) {
    b2_dev *d = b2h_dev(fd);
    if (!d) return;
    b2d_close(d);
    fds[fd] = NULL;
}

int rocket_batched_submit_supported(void) { return 1; }

int b2_set_stream(int fd, void *stream) {
    b2_dev *d = b2h_dev(fd);
    return d ? b2d_set_stream(d, stream) : ROCKET_E_SHAPE;
}
void *b2_get_stream(int fd) {
    b2_dev *d = b2h_dev(fd);
    return d ? b2d_stream(d) : NULL;
}
int b2_sync(int fd) {
    b2_dev *d = b2h_dev(fd);
    return d ? b2d_sync(d) : ROCKET_E_SHAPE;
}
unsigned b2_status(int fd, int clear) {
    b2_dev *d = b2h_dev(fd);
    return d ? b2d_status(d, clear) : 0u;
}
int b2_sm_count(int fd) {
    b2_dev *d = b2h_dev(fd);
    return d ? b2d_sm_count(d) : 0;
}
void *b2_host_alloc(size_t bytes) { return b2d_host_alloc(bytes); }
void b2_host_free(void *p) { b2d_host_free(p); }

/* ------------------------------------------------------------------------------ counters */
void rocket_submit_counters_reset(void) { n_submits = n_tasks = n_launches = 0; }
uint64_t rocket_submit_ioctl_count(void) { return n_submits; }
uint64_t rocket_submit_task_count(void) { return n_tasks; }
uint64_t rocket_launch_count(void) { return n_launches; }
void b2h_count_run(unsigned long long submits, unsigned long long tasks, unsigned launches) {
    n_submits += submits;
    n_tasks += tasks;
    n_launches += launches;
}

/* ------------------------------------------------------------------------------ faults */
void b2_fault_inject(enum b2_fault kind, unsigned nth) {
    if (kind == B2_FAULT_NONE || nth == 0) { fault_kind = B2_FAULT_NONE; fault_countdown = 0; return; }
    fault_kind = kind;
    fault_countdown = nth;
}

int b2h_fault(enum b2_fault kind) {
    if (fault_kind != kind || !fault_countdown) return 0;
    if (--fault_countdown) return 0;
    fault_kind = B2_FAULT_NONE;
    return 1;
}

/* ------------------------------------------------------------------------------ memory */
int b2h_malloc(int fd, size_t bytes, void **out) {
    *out = NULL;
    b2_dev *d = b2h_dev(fd);
    if (!d || !bytes) return ROCKET_E_SHAPE;
    if (b2h_fault(B2_FAULT_ALLOC)) return ROCKET_E_NOMEM;
    int rc = b2d_malloc(d, bytes, out);
    if (!rc) live_bytes += bytes;
    return rc;
}

void b2h_free(int fd, void *ptr, size_t bytes) {
    if (!ptr) return;
    b2_dev *d = b2h_dev(fd);
    if (d) b2d_free(d, ptr);
    live_bytes -= bytes;
}

size_t b2h_live_bytes(void) { return live_bytes; }

int rocket_bo_alloc32(int fd, size_t size, rocket_bo *bo) {
    if (!bo) return ROCKET_E_SHAPE;
    memset(bo, 0, sizeof(*bo));
    void *p = NULL;
    int rc = b2h_malloc(fd, size, &p);
    if (rc) return rc;
    bo->handle = next_handle++;
    if (!next_handle) next_handle = 1;
    bo->size = size;
    bo->ptr = p;
    bo->dma_address = (uint64_t)(uintptr_t)p;
    return 0;
}

void rocket_bo_free(int fd, rocket_bo *bo) {
    if (!bo || !bo->handle) return;
    b2h_free(fd, bo->ptr, bo->size);
    memset(bo, 0, sizeof(*bo));
}
