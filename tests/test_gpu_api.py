"""Operator entry points beyond the host run (GPU).

Restates the device-collection checks of research/custom-ops/tests/c/multitile_host_test.c:89-128
(run_tiles equals host assembly; a bad view or an alias is refused before any launch; multi-tile
run_cube is UNSUPPORTED), the K-tile input form of co_linear_run_tiled
(research/custom-ops/src/linear_hardsigmoid.c:325-352), weight refresh (:354-364), the guard
contract of co_buffer_alloc/co_guard_check (research/custom-ops/src/custom_ops.c:86-97,212-221),
and the extended device-pointer entries of include/b2_linear.h.
"""
import ctypes

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def uniform_case(m, n, k, seed):
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1, 1, (m, k)).astype(np.float16)
    w = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), (n, k)).astype(np.float16)
    b = rng.uniform(-0.1, 0.1, n).astype(np.float16)
    return x, w, b


def cuda_runtime():
    """cuda-python's runtime bindings (raw device copies for the padding checks), or None."""
    try:
        from cuda.bindings import runtime
        return runtime
    except Exception:
        return None


def tile_extent(total, i):
    return min(256, total - 256 * i)


def make_input_tiles(b2, fd, x, k_split=False):
    """co_tensor_input(rows, K) cubes per M tile, or co_tensor_matrix(rows, kt) per (M, K) tile."""
    m, k = x.shape
    bufs, views = [], []
    for mi in range((m + 255) // 256):
        rows = tile_extent(m, mi)
        xr = x[mi * 256: mi * 256 + rows]
        pieces = [(0, k)] if not k_split else [(k0, min(256, k - k0)) for k0 in range(0, k, 256)]
        for k0, kt in pieces:
            t = b2.tensor_input(rows, kt) if not k_split else b2.tensor_matrix(rows, kt)
            buf = b2.Buffer(fd, t.bytes)
            v = buf.view(t)
            b2.upload(v, np.ascontiguousarray(xr[:, k0:k0 + kt]))
            bufs.append(buf)
            views.append(v)
    return bufs, views


def make_output_tiles(b2, fd, m, n):
    bufs, views, info = [], [], []
    for mi in range((m + 255) // 256):
        for ni in range((n + 255) // 256):
            t = b2.tensor_matrix(tile_extent(m, mi), tile_extent(n, ni))
            buf = b2.Buffer(fd, t.bytes + 16)
            bufs.append(buf)
            views.append(buf.view(t, 16))          # 16-byte offset view, as the reference test does
            info.append((mi * 256, ni * 256, t.rows, t.cols))
    return bufs, views, info


def assemble(b2, views, info, m, n):
    y = np.zeros((m, n), np.float16)
    for v, (m0, n0, rows, cols) in zip(views, info):
        y[m0:m0 + rows, n0:n0 + cols] = b2.download(v)
    return y


# K a multiple of 8 with M > 8 in CO_CHAIN: the GEMM reads the input cubes and writes the output
# cubes directly (3-D tensor maps, no gather/scatter); other shapes and CO_SEPARATE gather and
# scatter. Both forms must give the host entry's bytes.
@pytest.mark.parametrize("m,k,n", [(13, 37, 45), (257, 257, 257), (513, 33, 289), (40, 96, 72), (257, 264, 257),
                                   (513, 512, 289), (100, 256, 300)])
def test_run_tiles_matches_host_run_and_refuses_bad_views(b2, gpu_fd, m, k, n):
    x, w, b = uniform_case(m, n, k, m + k + n)
    for mode in (b2.CO_SEPARATE, b2.CO_CHAIN):
        op = b2.Linear(gpu_fd, m, k, n, w, b, post=b2.CO_LINEAR_HSIG, mode=mode)
        host = op.run(x)
        xb, xv = make_input_tiles(b2, gpu_fd, x)
        yb, yv, info = make_output_tiles(b2, gpu_fd, m, n)
        before = b2.counters()["launches"]
        bad = list(yv)
        t = b2.CoTensor.from_buffer_copy(bad[-1].tensor)
        t.cols += 1
        tampered = b2.CoView(bad[-1].buffer, bad[-1].offset, t)
        bad[-1] = tampered
        assert op.run_tiles(xv, bad) == b2.E_SHAPE
        assert b2.counters()["launches"] == before          # refused before any launch
        assert op.run_tiles(xv, yv) == 0
        y = assemble(b2, yv, info, m, n)
        assert np.array_equal(y.view(np.uint16), host.view(np.uint16))
        if len(yv) > 1:
            assert op.run_cube(xv[0], yv[0]) == b2.E_UNSUPPORTED
            alias = list(yv)
            alias[1] = b2.CoView(yv[0].buffer, yv[0].offset, yv[1].tensor)
            before = b2.counters()["launches"]
            assert op.run_tiles(xv, alias) == b2.E_SHAPE
            assert b2.counters()["launches"] == before
        else:
            yb2, yv2, _ = make_output_tiles(b2, gpu_fd, m, n)
            assert op.run_cube(xv[0], yv2[0]) == 0
            assert np.array_equal(b2.download(yv2[0]).view(np.uint16), host.view(np.uint16))
        # an output overlapping an input is refused
        ovl = list(yv)
        ovl[0] = b2.CoView(xv[0].buffer, xv[0].offset, yv[0].tensor)
        assert op.run_tiles(xv, ovl) == b2.E_SHAPE
        ref = oracle.linear("tile16", x, w, b, post=1)["y16"]
        assert oracle.tolerance_ok(y, ref)[0]
        op.destroy()


@pytest.mark.parametrize("m,k,n", [(29, 513, 45), (300, 1000, 300), (129, 768, 513), (1024, 1024, 1024)])
def test_run_tiled_k_tile_inputs(b2, gpu_fd, m, k, n):
    x, w, b = uniform_case(m, n, k, 11)
    op = b2.Linear(gpu_fd, m, k, n, w, b, post=b2.CO_LINEAR_NONE)
    host = op.run(x)
    xb, xv = make_input_tiles(b2, gpu_fd, x, k_split=True)
    yb, yv, info = make_output_tiles(b2, gpu_fd, m, n)
    assert op.run_tiled(xv[:-1], yv) == b2.E_SHAPE               # wrong input count
    assert op.run_tiled(xv, yv) == 0
    y = assemble(b2, yv, info, m, n)
    assert np.array_equal(y.view(np.uint16), host.view(np.uint16))
    # again with the same views (the direct form reuses its tensor maps), after filling every byte of
    # the output cubes, padding included, with 0x47: the results and the zero padding come back
    rt = cuda_runtime()
    if rt is not None:
        b2.sync(gpu_fd)
        for v in yv:
            assert rt.cudaMemset(v.buffer.contents.bo.ptr + v.offset, 0x47, v.tensor.bytes)[0] == 0
        assert rt.cudaDeviceSynchronize()[0] == 0
    assert op.run_tiled(xv, yv) == 0
    assert np.array_equal(assemble(b2, yv, info, m, n).view(np.uint16), host.view(np.uint16))
    if rt is not None:
        for v in yv:
            t = v.tensor
            raw = np.empty(t.bytes // 2, np.uint16)
            assert rt.cudaMemcpy(raw.ctypes.data, v.buffer.contents.bo.ptr + v.offset, t.bytes, 2)[0] == 0
            cube = raw.reshape(t.physical_cols // 8, t.physical_rows, 8)          # [atom][row][channel]
            rowmajor = cube.transpose(1, 0, 2).reshape(t.physical_rows, t.physical_cols)
            assert not rowmajor[t.rows:, :].any() and not rowmajor[:, t.cols:].any(), "cube padding not zeroed"
    op.destroy()


def test_guard_corruption_is_detected(b2, gpu_fd):
    """A device write into a buffer's slack is reported by co_guard_check and by run_tiles."""
    m, k, n = 13, 37, 45
    x, w, b = uniform_case(m, n, k, 2)
    op = b2.Linear(gpu_fd, m, k, n, w, b, post=b2.CO_LINEAR_HSIG)
    xb, xv = make_input_tiles(b2, gpu_fd, x)
    yb, yv, info = make_output_tiles(b2, gpu_fd, m, n)
    assert op.run_tiles(xv, yv) == 0
    assert xb[0].guard_check() == 0
    # a tiny M=1 operator writes 8 FP16 values at payload + 0: inside the slack of the x buffer
    small = b2.Linear(gpu_fd, 1, 8, 8, np.ones((8, 8), np.float16), None, post=b2.CO_LINEAR_NONE,
                      acc=b2.ACC_FP32, compat=False)
    payload = xb[0].buf.payload
    assert payload % 16 == 0
    src = b2.Buffer(gpu_fd, 16)
    lin = b2.CoTensor()
    b2.check("co_tensor_linear", b2.lib().co_tensor_linear(ctypes.byref(lin), 8))
    b2.upload(src.view(lin), np.ones((1, 8), np.float16))
    small.run_device(1, src.ptr, 8, xb[0].ptr + payload, 8)
    b2.sync(gpu_fd)
    assert xb[0].guard_check() == b2.E_DEVICE
    assert op.run_tiles(xv, yv) == b2.E_DEVICE
    small.destroy()
    op.destroy()


def test_device_entries_partial_and_epilogue(b2, gpu_fd):
    torch = pytest.importorskip("torch")
    m, k, n = 300, 520, 700
    x, w, b = uniform_case(m, n, k, 21)
    op = b2.Linear(gpu_fd, m, k, n, w, b, post=b2.CO_LINEAR_HSIG, acc=b2.ACC_FP32, compat=False)
    host = op.run(x)
    ldx, ldy, ldp = k + 8, n + 20, n + 4
    xd = torch.zeros((m, ldx), dtype=torch.float16, device="cuda")
    xd[:, :k] = torch.from_numpy(x).cuda()
    yd = torch.full((m, ldy), 7.0, dtype=torch.float16, device="cuda")
    pd = torch.zeros((m, ldp), dtype=torch.float32, device="cuda")
    y2 = torch.zeros((m, ldy), dtype=torch.float16, device="cuda")
    torch.cuda.synchronize()
    op.run_device(m, xd.data_ptr(), ldx, yd.data_ptr(), ldy)
    op.partial_device(m, xd.data_ptr(), ldx, pd.data_ptr(), ldp)
    op.epilogue_device(m, pd.data_ptr(), ldp, y2.data_ptr(), ldy)
    b2.sync(gpu_fd)
    assert b2.status(gpu_fd) == 0
    yd_h = yd.cpu().numpy()
    assert np.array_equal(yd_h[:, :n].view(np.uint16), host.view(np.uint16))
    assert np.all(yd_h[:, n:] == 7.0)                            # padding columns untouched
    assert np.array_equal(y2.cpu().numpy()[:, :n].view(np.uint16), host.view(np.uint16))
    raw = oracle.linear("fp64", x, w, None, post=0, want=("raw",))["raw"]
    assert np.allclose(pd.cpu().numpy()[:, :n], raw, rtol=1e-4, atol=1e-4)
    # misaligned pitch and pointer are refused
    L = b2.lib()
    assert L.b2_linear_run_device(op.h, m, xd.data_ptr(), k + 1, yd.data_ptr(), ldy) == b2.E_SHAPE
    assert L.b2_linear_run_device(op.h, m, xd.data_ptr() + 2, ldx, yd.data_ptr(), ldy) == b2.E_SHAPE
    op.destroy()


@pytest.mark.parametrize("m,k,n,acc", [(1100, 4096, 300, "tile16"), (4096, 1024, 520, "fp32")])
def test_banded_host_run(b2, gpu_fd, m, k, n, acc):
    """Host runs with 8 MiB or more of X and at least 1024 rows copy X in row bands on a side stream
    and start each band's scan and GEMM as its rows land: the bytes equal the device entry's on the
    same input (one launch over all rows), also on a caller's stream, and a NaN in the last band is
    refused with Y untouched."""
    torch = pytest.importorskip("torch")
    x, w, b = uniform_case(m, n, k, 31)
    op = b2.Linear(gpu_fd, m, k, n, w, b, post=b2.CO_LINEAR_HSIG,
                   acc=b2.ACC_TILE16 if acc == "tile16" else b2.ACC_FP32, compat=acc == "tile16")
    before = b2.counters()["launches"]
    host = op.run(x)
    assert b2.counters()["launches"] - before == op.info().launches_per_run == 2 * (m // 512 if m // 512 < 8 else 8)
    xd = torch.from_numpy(x).cuda()
    ldy = (n + 7) // 8 * 8
    yd = torch.zeros((m, ldy), dtype=torch.float16, device="cuda")
    torch.cuda.synchronize()
    op.run_device(m, xd.data_ptr(), k, yd.data_ptr(), ldy)
    b2.sync(gpu_fd)
    assert b2.status(gpu_fd) == 0
    assert np.array_equal(host.view(np.uint16), yd.cpu().numpy()[:, :n].view(np.uint16))
    s = torch.cuda.Stream()
    b2.set_stream(gpu_fd, s.cuda_stream)
    try:
        again = op.run(x)
    finally:
        b2.set_stream(gpu_fd, 0)
    assert np.array_equal(again.view(np.uint16), host.view(np.uint16))
    xbad = x.copy()
    xbad[m - 1, k // 2] = np.nan
    y = np.full((m, n), 3.0, np.float16)
    assert op.run_rc(xbad, y) == b2.E_SHAPE
    assert np.all(y == 3.0)
    op.destroy()


def test_caller_stream(b2, gpu_fd):
    torch = pytest.importorskip("torch")
    m, k, n = 256, 256, 256
    x, w, b = uniform_case(m, n, k, 4)
    op = b2.Linear(gpu_fd, m, k, n, w, b, acc=b2.ACC_FP32)
    host = op.run(x)
    s = torch.cuda.Stream()
    xd = torch.from_numpy(x).cuda()
    yd = torch.zeros((m, n), dtype=torch.float16, device="cuda")
    torch.cuda.synchronize()
    b2.set_stream(gpu_fd, s.cuda_stream)
    try:
        op.run_device(m, xd.data_ptr(), k, yd.data_ptr(), n)
        s.synchronize()
    finally:
        b2.set_stream(gpu_fd, 0)
    assert np.array_equal(yd.cpu().numpy().view(np.uint16), host.view(np.uint16))
    op.destroy()


def test_update_weights(b2, gpu_fd):
    m, k, n = 40, 300, 70
    x, w, b = uniform_case(m, n, k, 8)
    _, w2, b2v = uniform_case(m, n, k, 9)
    op = b2.Linear(gpu_fd, m, k, n, w, b, post=b2.CO_LINEAR_HSIG)
    assert op.update_weights(w2, b2v) == 0
    y = op.run(x)
    assert oracle.tolerance_ok(y, oracle.linear("tile16", x, w2, b2v, post=1)["y16"])[0]
    assert op.update_weights(w2, None) == b2.E_SHAPE              # bias presence cannot change
    wbad = w2.copy()
    wbad[3, 4] = np.nan
    assert op.update_weights(wbad, b2v) == b2.E_SHAPE             # rejected before mutation
    assert np.array_equal(op.run(x).view(np.uint16), y.view(np.uint16))
    op.destroy()


def test_oom_and_alloc_fault_on_create_leak_nothing(b2, gpu_fd):
    w = np.ones((1, 1), np.float16)
    b = np.zeros(1, np.float16)
    h = ctypes.c_void_p(1)
    b2.fault_inject(b2.FAULT_ALLOC, 3)
    rc = b2.lib().co_linear_hsig_create(gpu_fd, 1, 1, 1, w.ctypes.data_as(ctypes.c_void_p),
                                         b.ctypes.data_as(ctypes.c_void_p), b2.CO_CHAIN, ctypes.byref(h))
    assert rc == b2.E_NOMEM and not h.value
    b2.fault_inject(b2.FAULT_NONE, 0)
    # staging for M = 2^20 rows of K = 2^17 would need 256 GiB: NOMEM, and W is freed again
    k = 1 << 17
    wbig = np.ones((8, k), np.float16)
    rc = b2.lib().b2_linear_create(gpu_fd, 1 << 20, k, 8, wbig.ctypes.data_as(ctypes.c_void_p), None,
                                   0, b2.CO_CHAIN, b2.ACC_FP32, ctypes.byref(h))
    assert rc == b2.E_NOMEM and not h.value
    # the device is still usable
    op = b2.Linear(gpu_fd, 4, 8, 8, np.ones((8, 8), np.float16), None, post=b2.CO_LINEAR_NONE)
    assert np.all(op.run(np.ones((4, 8), np.float16)) == 8.0)
    op.destroy()
