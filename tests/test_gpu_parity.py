"""GPU parity of the Linear / HardSigmoid path against the oracle, through the C-ABI library.

Tolerance (north star): element-wise |y - ref| <= 2e-3 + 2e-3*|ref| on FP16 outputs.
  tile-16 mode (the reference's per-256-K FP16 running sum) is checked against the oracle's
  TILE16_EXACT mode, which is bit-identical to the reference's own file-gate oracle
  (research/custom-ops/tools/python/cli_gate.py:38-49);
  FP32 mode is checked against the FP64 oracle.
Exact (bitwise) equality is required where the arithmetic is exact: dyadic impulse and
cancellation cases (research/custom-ops/tools/c/ktiling_probe.c:951-985) and CO_CHAIN vs
CO_SEPARATE outputs (cli_gate.py:90-93).
"""
import json
import os

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def uniform_case(m, n, k, seed):
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1, 1, (m, k)).astype(np.float16)
    w = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), (n, k)).astype(np.float16)
    b = rng.uniform(-0.1, 0.1, n).astype(np.float16)
    return x, w, b


def assert_tol(got, ref, what):
    ok, worst = oracle.tolerance_ok(got, ref)
    assert ok, f"{what}: worst |err|/tol = {worst:.3f}"
    return worst


def test_config1_hardsigmoid_tile16_and_fp32(b2, gpu_fd):
    m, n, k = 64, 256, 512
    x, w, b = uniform_case(m, n, k, 0)
    ref16 = oracle.linear("tile16", x, w, b, post=1)["y16"]
    ref64 = oracle.linear("fp64", x, w, b, post=1, want=("act",))["act"]
    outs = {}
    for mode in (b2.CO_CHAIN, b2.CO_SEPARATE):
        for acc in (b2.ACC_TILE16, b2.ACC_FP32):
            op = b2.Linear(gpu_fd, m, k, n, w, b, post=b2.CO_LINEAR_HSIG, mode=mode, acc=acc)
            y = op.run(x)
            y2 = op.run(x)
            op.destroy()
            assert np.array_equal(y.view(np.uint16), y2.view(np.uint16)), "repeated runs differ"
            outs[(mode, acc)] = y
            assert_tol(y, ref64, f"mode={mode} acc={acc} vs fp64")
            if acc == b2.ACC_TILE16:
                assert_tol(y, ref16, f"mode={mode} vs tile16")
                # the FP16 fold tracks the oracle almost bit for bit
                assert np.mean(y.view(np.uint16) == ref16.view(np.uint16)) > 0.99
    for acc in (b2.ACC_TILE16, b2.ACC_FP32):
        assert np.array_equal(outs[(b2.CO_CHAIN, acc)].view(np.uint16), outs[(b2.CO_SEPARATE, acc)].view(np.uint16))


def test_file_gate_shapes_match_reference_oracle(b2, gpu_fd):
    """cli_gate.SHAPES with its LCG inputs, against the reference oracle's stored outputs."""
    z = np.load(os.path.join(GOLDEN, "cli_gate_shapes.npz"))
    meta = json.loads(bytes(z["meta"]).decode())
    for case in meta:
        m, k, n = case["m"], case["k"], case["n"]
        x = oracle.lcg_fill(m * k, 303, 1.7).reshape(m, k)
        w = oracle.lcg_fill(n * k, 911, 0.21).reshape(n, k)
        b = oracle.lcg_fill(n, 409, 4.7)
        want = z[f"y_{m}_{k}_{n}"].view(np.float16).reshape(m, n)
        for mode in (b2.CO_SEPARATE, b2.CO_CHAIN):
            op = b2.Linear(gpu_fd, m, k, n, w, b, post=b2.CO_LINEAR_HSIG, mode=mode)
            y = op.run(x)
            op.destroy()
            err = np.max(np.abs(y.astype(np.float64) - want.astype(np.float64)))
            assert err <= 0.002, f"{m}x{k}x{n} mode={mode}: max abs {err}"   # cli_gate.py:77
            assert_tol(y, want, f"{m}x{k}x{n}")


def test_ktiling_impulses_and_cancellation_are_exact(b2, gpu_fd):
    z = np.load(os.path.join(GOLDEN, "ktiling_cases.npz"))
    index = json.loads(bytes(z["index"]).decode())
    checked = 0
    for i, case in enumerate(index):
        if not (case["name"].startswith("chan") or case["name"].startswith("cancel")):
            continue
        m, n, k = case["m"], case["n"], case["k"]
        x = z[f"c{i}_x"].view(np.float16).reshape(m, k)
        w = z[f"c{i}_w"].view(np.float16).reshape(n, k)
        want = z[f"c{i}_raw16"].reshape(m, n).astype(np.float16)
        for acc in (b2.ACC_TILE16, b2.ACC_FP32):
            op = b2.Linear(gpu_fd, m, k, n, w, None, post=b2.CO_LINEAR_NONE, acc=acc)
            y = op.run(x)
            op.destroy()
            assert np.array_equal(y.view(np.uint16), want.view(np.uint16)), (case["name"], acc)
        checked += 1
    assert checked == 13


def test_ktiling_contract_cases(b2, gpu_fd):
    """Contract shapes across K tile edges (255..4096): act16/act64 of the reference's gate."""
    z = np.load(os.path.join(GOLDEN, "ktiling_cases.npz"))
    index = json.loads(bytes(z["index"]).decode())
    for i, case in enumerate(index):
        if case["name"] not in ("contract", "prefix"):
            continue
        m, n, k = case["m"], case["n"], case["k"]
        x = z[f"c{i}_x"].view(np.float16).reshape(m, k)
        w = z[f"c{i}_w"].view(np.float16).reshape(n, k)
        b = z[f"c{i}_b"].view(np.float16) if case["bias"] else None
        post = b2.CO_LINEAR_HSIG if case["bias"] else b2.CO_LINEAR_NONE
        op = b2.Linear(gpu_fd, m, k, n, w, b, post=post)
        y = op.run(x)
        op.destroy()
        assert_tol(y, z[f"c{i}_act16"].reshape(m, n), f"{case['name']} {m}x{n}x{k} vs act16")
        assert_tol(y, z[f"c{i}_act64"].reshape(m, n), f"{case['name']} {m}x{n}x{k} vs act64")


def test_small_m_gemv_path(b2, gpu_fd):
    """M <= 8 uses the weight-streaming kernel; both modes, ragged K and N."""
    for (m, k, n) in [(1, 576, 576), (1, 576, 192), (1, 1536, 576), (3, 1000, 17), (8, 4096, 300), (1, 1, 1),
                      (5, 17, 4096)]:
        x, w, b = uniform_case(m, n, k, m * 1000 + k + n)
        op = b2.Linear(gpu_fd, m, k, n, w, b, post=b2.CO_LINEAR_NONE)
        assert op.info().kernel == 1
        y = op.run(x)
        op.set_accumulate(b2.ACC_FP32)
        y32 = op.run(x)
        op.destroy()
        assert_tol(y, oracle.linear("tile16", x, w, b, post=0)["y16"], f"gemv tile16 {m}x{k}x{n}")
        assert_tol(y32, oracle.linear("fp64", x, w, b, post=0, want=("act",))["act"], f"gemv fp32 {m}x{k}x{n}")


def test_ragged_shapes_gemm_path(b2, gpu_fd):
    for (m, k, n) in [(9, 1, 1), (17, 17, 17), (128, 64, 256), (129, 65, 257), (300, 1000, 17), (1000, 17, 1000),
                      (257, 257, 257), (513, 33, 289)]:
        x, w, b = uniform_case(m, n, k, m + 7 * k + 13 * n)
        for post in (b2.CO_LINEAR_NONE, b2.CO_LINEAR_HSIG):
            op = b2.Linear(gpu_fd, m, k, n, w, b, post=post)
            assert op.info().kernel == 0
            y = op.run(x)
            op.set_accumulate(b2.ACC_FP32)
            y32 = op.run(x)
            op.destroy()
            assert_tol(y, oracle.linear("tile16", x, w, b, post=post)["y16"], f"tile16 {m}x{k}x{n} post={post}")
            assert_tol(y32, oracle.linear("fp64", x, w, b, post=post, want=("act",))["act"],
                       f"fp32 {m}x{k}x{n} post={post}")


def test_failure_paths_leave_output_untouched(b2, gpu_fd):
    m, n, k = 40, 300, 70
    x, w, b = uniform_case(m, n, k, 5)
    op = b2.Linear(gpu_fd, m, k, n, w, b)
    y = np.full((m, n), np.float16(0.25))
    marker = y.copy()
    # injected launch failure
    b2.fault_inject(b2.FAULT_LAUNCH, 1)
    assert op.run_rc(x, y) == b2.E_DEVICE
    assert np.array_equal(y.view(np.uint16), marker.view(np.uint16))
    # injected non-finite output
    b2.fault_inject(b2.FAULT_NAN_OUTPUT, 1)
    assert op.run_rc(x, y) == b2.E_DEVICE
    assert np.array_equal(y.view(np.uint16), marker.view(np.uint16))
    # non-finite input is a shape error, detected on the device before publishing
    xbad = x.copy()
    xbad[7, 11] = np.inf
    assert op.run_rc(xbad, y) == b2.E_SHAPE
    xbad[7, 11] = np.nan
    assert op.run_rc(xbad, y) == b2.E_SHAPE
    assert np.array_equal(y.view(np.uint16), marker.view(np.uint16))
    # the context is still usable afterwards
    assert op.run_rc(x, y) == 0
    assert_tol(y, oracle.linear("tile16", x, w, b, post=1)["y16"], "after failures")
    op.destroy()


def test_overflow_output_is_device_error(b2, gpu_fd):
    m, n, k = 16, 16, 300
    x = np.full((m, k), 200.0, np.float16)
    w = np.full((n, k), 200.0, np.float16)
    op = b2.Linear(gpu_fd, m, k, n, w, None, post=b2.CO_LINEAR_NONE)
    y = np.zeros((m, n), np.float16)
    assert op.run_rc(x, y) == b2.E_DEVICE
    assert not y.any()
    op.destroy()
    # HardSigmoid saturates an infinite pre-activation to 1 (finite output, no error)
    op = b2.Linear(gpu_fd, m, k, n, w, np.zeros(n, np.float16), post=b2.CO_LINEAR_HSIG)
    assert np.all(op.run(x) == 1.0)
    op.destroy()


def test_hardsigmoid_every_fp16_preactivation_is_bitexact(b2, gpu_fd):
    """One-hot X makes acc[m, n] = W[n, m] exactly, so the 65536 entries of W sweep every FP16
    pre-activation (non-finite patterns replaced by 0) through bias + HardSigmoid + FP16 rounding.
    Both accumulation modes must equal the oracle bit for bit."""
    m = n = k = 256
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    bits[(bits & 0x7C00) == 0x7C00] = 0
    w = bits.view(np.float16).reshape(n, k)
    x = np.eye(m, k, dtype=np.float16)
    b = np.zeros(n, np.float16)
    want = oracle.linear("tile16", x, w, b, post=1)["y16"].view(np.uint16)
    for acc in (b2.ACC_TILE16, b2.ACC_FP32):
        op = b2.Linear(gpu_fd, m, k, n, w, b, post=b2.CO_LINEAR_HSIG, acc=acc)
        y = op.run(x)
        op.destroy()
        assert np.array_equal(y.view(np.uint16), want), f"acc={acc}: {np.count_nonzero(y.view(np.uint16) != want)} differ"
