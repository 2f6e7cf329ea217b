"""C-ABI library: loads, exports every declared symbol, host-only functions behave (CPU only).

Restates the structural host checks of the reference:
  research/custom-ops/tests/c/multitile_host_test.c:137-156  plan invariants over a 9x9 dim grid
  research/custom-ops/tests/c/ktiling_host_test.c:25-69,224-254  K-slice descriptors and limits
  research/custom-ops/tools/c/ktiling_probe.c:898-911           task accounting (18 / 33 tasks)
"""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in ("rocket_b200.h", "custom_ops.h", "b2_linear.h", "co_graph.h", "rk_plan.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b((?:co|rocket|b2|rk)_[a-z0-9_]+)\s*\(", src):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol(b2):
    L = b2.lib()
    names = declared_functions()
    assert len(names) > 50
    missing = [n for n in sorted(names) if not hasattr(L, n)]
    assert not missing, missing
    assert names == set(b2.SIGNATURES), set(b2.SIGNATURES) ^ names


def test_library_exports_nothing_else(b2):
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", b2.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    assert exported == declared_functions()


def test_no_device_is_reported_not_faked(b2):
    if b2.device_count() > 0:
        pytest.skip("a CUDA device is present")
    assert b2.lib().rocket_open() == b2.E_DEVICE
    assert b2.lib().b2_open_device(0) == b2.E_DEVICE


def test_plan_invariants_over_dim_grid(b2):
    dims = [1, 12, 255, 256, 257, 511, 512, 513, 4096]
    for m in dims:
        for n in dims:
            p = b2.plan(m, 513, n)
            area = 0
            tasks = 0
            for i in range(p.output_tiles):
                t = b2.plan_tile(p, i)
                assert 0 < t.rows <= 256 and 0 < t.cols <= 256
                assert t.m0 == i // p.ntiles * 256 and t.n0 == i % p.ntiles * 256
                assert t.m0 + t.rows <= p.m and t.n0 + t.cols <= p.n
                area += t.rows * t.cols
                tasks += t.programs
            assert area == m * n and tasks == p.tasks
            assert p.chain_submits == p.output_tiles
            assert p.row_classes == (2 if p.mtiles > 1 and m % 256 else 1)
            # budget exact to the byte
            q = b2.CoLinearPlan()
            L = b2.lib()
            assert L.co_linear_plan_init(ctypes.byref(q), m, 513, n, p.device_bytes) == 0
            assert L.co_linear_plan_init(ctypes.byref(q), m, 513, n, p.device_bytes - 1) == b2.E_TILING


def test_plan_tasks_match_oracle_accounting(b2, oracle_mod):
    for (m, k, n) in [(64, 4096, 64), (256, 1024, 256), (256, 4096, 256), (29, 37, 45), (513, 33, 289),
                      (4096, 4096, 4096), (1, 1, 1), (4095, 4097 - 1, 17)]:
        p = b2.plan(m, k, n)
        tiles, tasks = oracle_mod.plan_tasks(m, k, n)
        assert (p.output_tiles, p.tasks) == (tiles, tasks)
        p0 = b2.plan(m, k, n, has_bias=False, post=b2.CO_LINEAR_NONE)
        assert p0.tasks == oracle_mod.plan_tasks(m, k, n, has_bias=False, hsig=False)[1]
    # ktiling_probe.c:905-908: 64/64/4096 fused = 18 tasks; one LUT chunk at 64x64, two at 256x256
    assert b2.plan(64, 4096, 64).tasks == 18
    assert b2.plan(256, 4096, 256).tasks == 16 + 1 + 2


def test_plan_rejects_shapes(b2):
    L = b2.lib()
    p = b2.CoLinearPlan()
    for (m, k, n) in [(0, 1, 1), (4097, 1, 1), (1, 4097, 1), (1, 1, 4097)]:
        assert L.co_linear_plan_init(ctypes.byref(p), m, k, n, 0) == b2.E_SHAPE
    assert L.co_linear_plan_init_ex(ctypes.byref(p), 1, 1, 1, 2, 1, 0) == b2.E_SHAPE
    assert L.co_linear_plan_init_ex(ctypes.byref(p), 1, 1, 1, 1, 7, 0) == b2.E_SHAPE
    t = b2.CoLinearTileInfo()
    q = b2.plan(300, 10, 300)
    assert L.co_linear_plan_tile(ctypes.byref(q), q.output_tiles, ctypes.byref(t)) == b2.E_SHAPE
    q.ntiles += 1
    assert L.co_linear_plan_tile(ctypes.byref(q), 0, ctypes.byref(t)) == b2.E_SHAPE


def test_device_bytes_is_hbm_of_the_context(b2):
    for (m, k, n, bias) in [(64, 512, 256, True), (4096, 4096, 4096, True), (17, 1, 1000, False)]:
        p = b2.plan(m, k, n, has_bias=bias)
        k8, n8 = -(-k // 8) * 8, -(-n // 8) * 8
        assert p.device_bytes == n * k8 * 2 + (n * 2 if bias else 0) + m * k8 * 2 + m * n8 * 2


def test_descriptors_and_k_slices(b2):
    L = b2.lib()
    t = b2.CoTensor()
    assert L.co_tensor_input(ctypes.byref(t), 13, 4096) == 0
    assert (t.physical_rows, t.physical_cols) == (16, 4096)
    assert L.co_tensor_input(ctypes.byref(t), 12, 4097) != 0
    assert L.co_tensor_input(ctypes.byref(t), 257, 256) != 0
    assert L.co_tensor_input(ctypes.byref(t), 0, 256) != 0
    assert L.co_tensor_matrix(ctypes.byref(t), 12, 257, b2.CO_F16) != 0
    assert L.co_tensor_weight(ctypes.byref(t), 64, 257) != 0
    for (m, k) in [(13, 257), (1, 513), (16, 576), (29, 769), (13, 1024), (16, 1536), (29, 2049), (1, 4096),
                   (16, 255), (16, 256), (16, 512)]:
        full = b2.tensor_input(m, k)
        expect_off, total = 0, 0
        for i in range(L.co_k_tiles(k)):
            k0, kt = i * 256, L.co_k_tile_length(k, i)
            assert 1 <= kt <= 256
            s = b2.CoTensor()
            off = ctypes.c_size_t()
            assert L.co_tensor_input_slice(ctypes.byref(s), ctypes.byref(full), k0, kt, ctypes.byref(off)) == 0
            assert off.value == expect_off == k0 * full.physical_rows * 2
            for r in range(m):
                for c in range(0, kt, 7):
                    assert L.co_index(ctypes.byref(full), r, k0 + c) == off.value // 2 + L.co_index(ctypes.byref(s), r, c)
            expect_off = off.value + s.bytes
            total += kt
        assert total == k and expect_off == full.bytes
    full = b2.tensor_input(16, 512)
    s = b2.CoTensor()
    off = ctypes.c_size_t()
    for (k0, kt, ok) in [(0, 257, False), (1, 256, False), (0, 512, False), (0, 0, False), (512, 1, False),
                         (256, 256, True), (0, 256, True)]:
        rc = L.co_tensor_input_slice(ctypes.byref(s), ctypes.byref(full), k0, kt, ctypes.byref(off))
        assert (rc == 0) == ok, (k0, kt)


def test_cube_index_layout(b2):
    """CUBE [pc/8][pr][8] and WEIGHT (N/16, K/32, 16, 32) addressing (custom_ops.c:80-85)."""
    L = b2.lib()
    t = b2.tensor_matrix(29, 45)
    assert (t.physical_rows, t.physical_cols, t.bytes) == (32, 64, 32 * 64 * 2)
    seen = set()
    for r in range(t.physical_rows):
        for c in range(t.physical_cols):
            i = L.co_index(ctypes.byref(t), r, c)
            assert i == ((c // 8) * 32 + r) * 8 + c % 8
            seen.add(i)
    assert seen == set(range(32 * 64))
    w = b2.CoTensor()
    assert L.co_tensor_weight(ctypes.byref(w), 40, 70) == 0
    assert L.co_index(ctypes.byref(w), 17, 33) == (((17 // 16) * (w.physical_cols // 32) + 33 // 32) * 16 + 1) * 32 + 1


def test_views_reject_bad_offsets_without_device(b2):
    """co_view_init rules on a hand-made buffer record (no device memory is touched)."""
    L = b2.lib()
    buf = b2.CoBuffer()
    buf.bo.handle = 7
    buf.bo.ptr = 0x10000
    buf.payload = 4096
    t = b2.tensor_matrix(16, 32)
    v = b2.CoView()
    assert L.co_view_init(ctypes.byref(v), ctypes.byref(buf), 0, ctypes.byref(t)) == 0
    assert L.co_view_init(ctypes.byref(v), ctypes.byref(buf), 8, ctypes.byref(t)) == b2.E_SHAPE
    assert L.co_view_init(ctypes.byref(v), ctypes.byref(buf), 4096 - t.bytes + 16, ctypes.byref(t)) == b2.E_SHAPE
    bad = b2.tensor_matrix(16, 32)
    bad.bytes += 2
    assert L.co_view_init(ctypes.byref(v), ctypes.byref(buf), 0, ctypes.byref(bad)) == b2.E_SHAPE
    buf.bo.handle = 0
    assert L.co_view_init(ctypes.byref(v), ctypes.byref(buf), 0, ctypes.byref(t)) == b2.E_SHAPE


def test_create_without_device_is_refused(b2):
    if b2.device_count() > 0:
        pytest.skip("a CUDA device is present")
    w = np.zeros((4, 4), np.float16)
    h = ctypes.c_void_p(1)
    rc = b2.lib().co_linear_create(0, 4, 4, 4, w.ctypes.data_as(ctypes.c_void_p), None, 1, 1, ctypes.byref(h))
    assert rc == b2.E_SHAPE and not h.value
