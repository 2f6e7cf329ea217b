/* b2_host.h -- internal declarations shared by the host C files. */
#ifndef B2_HOST_H
#define B2_HOST_H
#include "b2_linear.h"
#include "../b2_device.h"

#define B2_MAX_FDS 64

/* Device handle table (rocket.c). */
b2_dev *b2h_dev(int fd);
int b2h_valid_fd(int fd);

/* Counters (rocket.c). */
void b2h_count_run(unsigned long long submits, unsigned long long tasks, unsigned launches);

/* Fault-injection seam (rocket.c): returns 1 when the armed fault of `kind` fires now. */
int b2h_fault(enum b2_fault kind);

/* Allocation wrappers that honour the fault seam and track live device bytes. */
int b2h_malloc(int fd, size_t bytes, void **out);
void b2h_free(int fd, void *ptr, size_t bytes);
size_t b2h_live_bytes(void);

static inline size_t b2h_round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

/* Planner (plan.c). compat=1 applies the reference limits (4096, CO_MAX_PROGRAMS). */
int b2h_plan(co_linear_plan *out, unsigned m, unsigned k, unsigned n, int has_bias,
             enum co_linear_post post, size_t budget, unsigned max_dim, int compat);
size_t b2h_context_bytes(unsigned m, unsigned k, unsigned n, int has_bias);

/* Operator accessors for other host files (linear.c). */
int b2h_linear_fd(const b2_linear *op);
/* Raw-FP32-partial launch descriptor of `op` for device X [m, ldx] (no bias, no activation in
 * the GEMM; bias/post copied into the descriptor for a later epilogue). 0 or ROCKET_E_SHAPE. */
int b2h_linear_desc(const b2_linear *op, unsigned m, const void *x, size_t ldx, b2k_linear *out);

#endif
