"""Shape sweep and large shapes against the oracle (GPU).

* The 125-combination plain Linear sweep M, N, K in {1, 17, 128, 1000, 4096} with
  X ~ U(-1,1), W ~ U(-1/sqrt(K), 1/sqrt(K)), b ~ U(-0.1, 0.1), seeds 0..124 in (M, N, K)
  lexicographic order, through the drop-in co_linear_* API (per-256-K FP16 accumulation) and with
  FP32 accumulation. Rows are independent, so M > 64 is checked on a row sample (first, last and
  evenly spaced rows) to keep the oracle within seconds.
* The square 4096^3 case (X ~ N(0,1), W ~ N(0,1/K), b = 0) and the K-split 2048x2048x16384 case
  (K > 4096 goes through the extended b2_linear API).
Tolerance: |y - ref| <= 2e-3 + 2e-3*|ref| element-wise (tile-16 vs the tile-16 oracle, FP32 vs
the FP64 oracle).
"""
import itertools

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
DIMS = (1, 17, 128, 1000, 4096)


def sample_rows(m, cap=48):
    if m <= cap:
        return np.arange(m)
    return np.unique(np.concatenate([[0, m - 1], np.linspace(0, m - 1, cap - 2).astype(int)]))


def check(y, x, w, b, rows, mode, what):
    xr = x[rows]
    if mode == "fp64":
        ref = oracle.linear("fp64", xr, w, b, post=0, want=("act",))["act"]
    else:
        big = len(rows) * w.shape[0] * w.shape[1] > 40_000_000
        ref = oracle.linear("tile16_fast" if big else "tile16", xr, w, b, post=0)["y16"]
    ok, worst = oracle.tolerance_ok(y[rows], ref)
    assert ok, f"{what}: worst |err|/tol {worst:.3f}"
    return worst


def test_sweep_125_combinations(b2, gpu_fd):
    worst = 0.0
    for seed, (m, n, k) in enumerate(itertools.product(DIMS, DIMS, DIMS)):
        rng = np.random.default_rng(seed)
        x = rng.uniform(-1, 1, (m, k)).astype(np.float16)
        w = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), (n, k)).astype(np.float16)
        b = rng.uniform(-0.1, 0.1, n).astype(np.float16)
        rows = sample_rows(m)
        op = b2.Linear(gpu_fd, m, k, n, w, b, post=b2.CO_LINEAR_NONE, mode=b2.CO_CHAIN)
        y16 = op.run(x)
        op.set_accumulate(b2.ACC_FP32)
        y32 = op.run(x)
        op.destroy()
        worst = max(worst, check(y16, x, w, b, rows, "tile16", f"{m}x{n}x{k} tile16"))
        worst = max(worst, check(y32, x, w, b, rows, "fp64", f"{m}x{n}x{k} fp32"))
    assert worst <= 1.0


@pytest.mark.parametrize("m,n,k", [(4096, 4096, 4096), (2048, 2048, 16384)])
def test_large_square_and_split_k_shapes(b2, gpu_fd, m, n, k):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((m, k)).astype(np.float16)
    w = (rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float16)
    b = np.zeros(n, np.float16)
    rows = sample_rows(m, 24)
    op = b2.Linear(gpu_fd, m, k, n, w, b, post=b2.CO_LINEAR_NONE, acc=b2.ACC_FP32, compat=False)
    y = op.run(x)
    check(y, x, w, b, rows, "fp64", f"{m}x{n}x{k} fp32")
    op.set_accumulate(b2.ACC_TILE16)
    y16 = op.run(x)
    op.destroy()
    check(y16, x, w, b, rows, "tile16", f"{m}x{n}x{k} tile16")
