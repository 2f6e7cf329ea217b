// plan_kernels.h -- launchers of the plan (RKPlan) tile kernels (plan_kernels.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#include "b2_device.h"

namespace b2 {
namespace rkplan {

// Kernel-parameter tables (by value: no per-launch table copy).
struct PackTable {
    b2k_rk_pack item[B2K_RK_MAX_PACK];
    unsigned count;
};
struct UnpackTable {
    b2k_rk_unpack item[B2K_RK_MAX_UNPACK];
    unsigned count;
};

// The contraction kernels' shared-memory opt-in (over 48 KB) on the current device: done when a device
// handle opens, outside any stream capture.
cudaError_t prepare();
cudaError_t pack(const PackTable &t, size_t max_vectors, cudaStream_t s, int sm_count);
cudaError_t task(const b2k_rk_task &t, cudaStream_t s, int sm_count);
cudaError_t chain(const b2k_rk_chain &t, cudaStream_t s);
cudaError_t unpack(const UnpackTable &t, size_t max_elements, cudaStream_t s, int sm_count);

}  // namespace rkplan
}  // namespace b2
