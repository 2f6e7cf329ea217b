/* rocket_b200.h -- device handle, buffer object and counters for the B200 Linear path.
 *
 * Replaces the subset of the reference's provider header `rocket_npu.h` (rknpu-submit @
 * 6b144b19bb67, not vendored in the reference; included by research/custom-ops/include/
 * custom_ops.h:4) that the Linear operator, its tensor helpers and its file CLI use:
 *   status codes      ROCKET_E_* (values mirrored in research/multidevice-scheduling/backends/
 *                     rk3588.py:76-81)
 *   device handle     rocket_open / rocket_close (operator_cli.c:75-76, :94)
 *   buffer object     rocket_bo {handle, size, ptr, dma_address} (custom_ops.c:86-101)
 *   submit counters   rocket_submit_counters_reset / _ioctl_count / _task_count
 *                     (operator_cli.c:81-91)
 *   chain capability  rocket_batched_submit_supported (linear_hardsigmoid.c:131,229)
 *
 * B200 meaning:
 *   - An `fd` is a small non-negative handle naming one CUDA device plus one CUDA stream. It is
 *     not a file descriptor. rocket_open() opens the device named by $B2_DEVICE (default 0).
 *   - rocket_bo.ptr is a DEVICE pointer (HBM); the CPU cannot dereference it. dma_address holds
 *     the same device virtual address as an integer.
 *   - The submit/task counters keep the reference's accounting, derived from the operator plan
 *     (CO_CHAIN: one "submit" per output tile per run; CO_SEPARATE: one per task), so the
 *     reference's file gate can check them. rocket_launch_count() is the number of CUDA kernels
 *     actually launched.
 */
#ifndef ROCKET_B200_H
#define ROCKET_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum rocket_status {
    ROCKET_OK = 0,
    ROCKET_E_SHAPE = -1,        /* bad dims, bad view, non-finite input, alias */
    ROCKET_E_TILING = -2,       /* over the device budget or too many programs per tile */
    ROCKET_E_NOMEM = -3,        /* host or device allocation failed */
    ROCKET_E_DEVICE = -4,       /* CUDA error, kernel timeout, guard corruption, non-finite output */
    ROCKET_E_UNSUPPORTED = -5,  /* entry not supported for this shape / capability */
};

typedef struct {
    uint32_t handle;        /* nonzero while allocated */
    size_t size;            /* bytes allocated on the device */
    void *ptr;              /* device pointer */
    uint64_t dma_address;   /* device virtual address of ptr */
} rocket_bo;

/* Opens the CUDA device $B2_DEVICE (default 0). Returns a handle >= 0, or ROCKET_E_DEVICE when
 * no CUDA device is usable (the CLI maps this to exit status 77, "no device"). */
int rocket_open(void);
void rocket_close(int fd);
/* Always 1: a CUDA stream orders every launch of an op, so the chained mode is available. */
int rocket_batched_submit_supported(void);
/* Device allocation of `size` bytes (zero-filled). */
int rocket_bo_alloc32(int fd, size_t size, rocket_bo *bo);
void rocket_bo_free(int fd, rocket_bo *bo);

void rocket_submit_counters_reset(void);
uint64_t rocket_submit_ioctl_count(void);
uint64_t rocket_submit_task_count(void);
uint64_t rocket_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif
