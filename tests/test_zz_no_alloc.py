"""The allocation-free entry point, b2_linear_run_device_noalloc (GPU).

Who needs it: code that may not allocate GPU memory while it runs -- a serving loop whose device
memory is planned before the first request, where a cudaMalloc/cudaFree mid-request would
synchronise the device or fail under memory pressure. The unfused FP32 arm of the operator
normally allocates its FP32 workspace on first use; this entry runs the same arm on a fixed
scratch array that the library keeps in static device memory instead.

The test calls it through the C-ABI (device buffers come from the library's own co_buffer_alloc,
which is the caller's allocation, made before the call) and checks, on two calls in a row, that it
produces what the existing b2_linear_run_device entry produces for the same operator, within the
operator tolerance |y - ref| <= 2e-3 + 2e-3*|ref|. It runs last (file name) so that a failure here
leaves every other test already run, and it opens its own device handle so it passes alone too.
"""
import ctypes

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def _linear_view(b2, fd, elements):
    buf = b2.Buffer(fd, elements * 2)
    t = b2.CoTensor()
    b2.check("co_tensor_linear", b2.lib().co_tensor_linear(ctypes.byref(t), elements))
    return buf, buf.view(t)


# m > 8 runs the tcgen05 GEMM; m <= 8 runs the weight-streaming small-M kernel (whole-row units
# up to k = 2048, 16-row x 512-K slices with tile-sum buffers beyond), both writing raw FP32 sums
# into the static scratch before the epilogue kernel.
@pytest.mark.parametrize("m,k,n", [(64, 512, 256), (33, 200, 70), (1, 512, 256), (8, 200, 70), (4, 4096, 512)])
def test_noalloc_matches_existing_entry_on_two_calls(b2, m, k, n):
    L = b2.lib()
    fd = b2.open_device(0)
    try:
        rng = np.random.default_rng(m * 1000 + n)
        x = rng.uniform(-1, 1, (m, k)).astype(np.float16)
        w = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), (n, k)).astype(np.float16)
        b = rng.uniform(-0.1, 0.1, n).astype(np.float16)
        ldx = -(-k // 8) * 8
        ldy = -(-n // 8) * 8
        xpad = np.zeros((m, ldx), np.float16)
        xpad[:, :k] = x
        xbuf, xview = _linear_view(b2, fd, m * ldx)
        b2.upload(xview, xpad.reshape(1, -1))
        outs = [_linear_view(b2, fd, m * ldy) for _ in range(3)]
        op = b2.Linear(fd, 1, k, n, w, b, post=b2.CO_LINEAR_HSIG, mode=b2.CO_CHAIN, acc=b2.ACC_FP32,
                       compat=False)
        # existing entry (fused FP32 kernel) as the reference
        b2.check("b2_linear_run_device", L.b2_linear_run_device(op.h, m, xbuf.ptr, ldx, outs[0][0].ptr, ldy))
        # the allocation-free entry, twice in a row into distinct outputs
        for i in (1, 2):
            rc = L.b2_linear_run_device_noalloc(op.h, m, xbuf.ptr, ldx, outs[i][0].ptr, ldy)
            assert rc == 0, rc
        b2.sync(fd)
        assert b2.status(fd) == 0
        ys = [b2.download(v).reshape(m, ldy)[:, :n] for _, v in outs]
        ref = ys[0].astype(np.float64)
        for y in ys[1:]:
            ok, worst = oracle.tolerance_ok(y, ref)
            assert ok, f"no-alloc entry vs existing entry: worst err/tol {worst:.3f}"
        # and both agree with the FP64 oracle
        ok, worst = oracle.tolerance_ok(ys[2], oracle.linear("fp64", x, w, b, post=1, want=("act",))["act"])
        assert ok, worst
        op.destroy()
        for buf, _ in outs + [(xbuf, None)]:
            buf.free()
    finally:
        b2.close(fd)


def test_noalloc_rejects_oversized_and_tile16(b2):
    L = b2.lib()
    fd = b2.open_device(0)
    try:
        k, n = 64, 4096
        w = np.zeros((n, k), np.float16)
        op = b2.Linear(fd, 1, k, n, w, None, post=b2.CO_LINEAR_NONE, acc=b2.ACC_FP32, compat=False)
        xbuf, _ = _linear_view(b2, fd, 8 * k)
        ybuf, _ = _linear_view(b2, fd, 8 * n)
        limit_rows = (8 << 20) // (n * 4)            # 512 rows of 4096 FP32 fit the 8 MiB scratch
        assert L.b2_linear_run_device_noalloc(op.h, limit_rows + 1, xbuf.ptr, k, ybuf.ptr, n) == b2.E_TILING
        op.set_accumulate(b2.ACC_TILE16)
        assert L.b2_linear_run_device_noalloc(op.h, 8, xbuf.ptr, k, ybuf.ptr, n) == b2.E_UNSUPPORTED
        op.destroy()
        xbuf.free()
        ybuf.free()
    finally:
        b2.close(fd)
