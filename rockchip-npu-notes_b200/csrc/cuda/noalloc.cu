// noalloc.cu -- fixed device scratch for b2_linear_run_device_noalloc.
//
// The unfused FP32 arm of the operator (GEMM writes raw FP32 accumulators, a second kernel adds
// the bias, applies the activation and writes FP16 Y) needs an M x N FP32 workspace. The regular
// entries allocate it on first use with cudaMalloc. For callers that must not allocate device
// memory while they run, this file reserves the workspace once, statically, as a file-scope
// __device__ array: every GPU that loads the library holds B2D_NOALLOC_SCRATCH_BYTES of it until
// the process exits, and every call on a device shares it.
//
// Host code cannot use the array's name as a device address (it is only a host-side stand-in),
// so the address is looked up with cudaGetSymbolAddress, once per device, with that device
// current, on the first call that needs it; the result is cached per device ordinal. The lookup
// makes the handle's device current only for its duration: the calling thread's current device
// is saved first and restored afterwards, so the call leaves it as it found it. Two threads that
// make their first call at the same time both look the address up and store the same value; the
// cache entries are read and written atomically.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../b2_device.h"
#include "rocket_b200.h"

static __device__ __align__(256) float g_noalloc_scratch[B2D_NOALLOC_SCRATCH_BYTES / sizeof(float)];

namespace {
constexpr int MAX_DEVICES = 64;
float *scratch_addr[MAX_DEVICES];   // device address of g_noalloc_scratch, per device ordinal

int lookup_scratch(int ordinal, float **out) {
    int previous = -1;
    if (cudaGetDevice(&previous) != cudaSuccess) {
        cudaGetLastError();
        return ROCKET_E_DEVICE;
    }
    int rc = 0;
    void *p = nullptr;
    if (cudaSetDevice(ordinal) != cudaSuccess || cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess ||
        !p) {
        cudaGetLastError();
        rc = ROCKET_E_DEVICE;
    }
    if (previous != ordinal && cudaSetDevice(previous) != cudaSuccess) {
        cudaGetLastError();
        rc = ROCKET_E_DEVICE;
    }
    if (!rc) *out = static_cast<float *>(p);
    return rc;
}
}  // namespace

extern "C" int b2d_noalloc_scratch(b2_dev *d, float **ptr, size_t *bytes) {
    *ptr = nullptr;
    *bytes = 0;
    const int ordinal = b2d_ordinal(d);
    if (ordinal < 0 || ordinal >= MAX_DEVICES) return ROCKET_E_DEVICE;
    float *addr = __atomic_load_n(&scratch_addr[ordinal], __ATOMIC_ACQUIRE);
    if (!addr) {
        const int rc = lookup_scratch(ordinal, &addr);
        if (rc) return rc;
        __atomic_store_n(&scratch_addr[ordinal], addr, __ATOMIC_RELEASE);
    }
    *ptr = addr;
    *bytes = B2D_NOALLOC_SCRATCH_BYTES;
    return 0;
}
