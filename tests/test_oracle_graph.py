"""The graph oracle (oracle/graph_oracle.c) pinned to the reference's own graph oracle (CPU only).

* The activation gates over every finite FP16 input against the functions the reference's LUTs
  sample (research/custom-ops/src/custom_ops.c:357-369) evaluated with Python's math module, as the
  reference's graph gate does (research/custom-ops/tools/python/graph_gate.py:39).
* ``oracle.ffn`` against ``tests/golden/graph_gate_ffn.npz``, the outputs of the reference's
  ``graph_gate.oracle`` on its own shapes and inputs (made by tests/golden/make_graph_golden.py):
  bit for bit without RMSNorm; with RMSNorm within the gate's 0.003 (graph_gate.py:94), since the
  reference's operator (co_row_ops.c:207) divides gamma by the root where the gate multiplies by
  its reciprocal.
"""
import hashlib
import math
import os
import struct

import numpy as np
import pytest

import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "graph_gate_ffn.npz")


def f16(v):
    return struct.unpack("<e", struct.pack("<e", v))[0]


def finite_f16():
    bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    return bits[(bits & 0x7C00) != 0x7C00].view(np.float16)


def sigmoid(a):
    try:
        return 1 / (1 + math.exp(-a))
    except OverflowError:        # exp(-a) beyond double for a < -709: the limit is 0
        return 0.0


def test_gates_over_every_finite_fp16():
    a = finite_f16()
    silu = oracle.ew(oracle.EW_SILU, a)
    gelu = oracle.ew(oracle.EW_GELU, a)
    hsig = oracle.ew(oracle.EW_HSIG, a)
    for i, v in enumerate(a.astype(np.float64)):
        s = f16(sigmoid(v))
        assert float(silu[i]) == f16(v * s) or (math.isnan(f16(v * s)) and np.isnan(silu[i])), v
        g = f16(0.5 * (1 + math.erf(v / math.sqrt(2.0))))
        assert float(gelu[i]) == f16(v * g), v
        assert float(hsig[i]) == f16(min(1, max(0, v / 6 + 0.5))), v


def test_elementwise_is_one_rounding():
    rng = np.random.default_rng(5)
    a = (rng.standard_normal(4096) * 300).astype(np.float16)
    b = (rng.standard_normal(4096) * 0.01).astype(np.float16)
    add, mul = oracle.ew(oracle.EW_ADD, a, b), oracle.ew(oracle.EW_MUL, a, b)
    for x, y, s, p in zip(a.astype(float), b.astype(float), add, mul):
        assert float(s) == f16(x + y) and float(p) == f16(x * y)


def _inputs(z, m, d, h):
    key = f"{m}_{d}_{h}"
    arrays = dict(x=oracle.lcg_fill(m * d, 123, 0.7), wg=oracle.lcg_fill(h * d, 451, 0.06),
                  wu=oracle.lcg_fill(h * d, 911, 0.07), wd=oracle.lcg_fill(d * h, 771, 0.05),
                  bias=oracle.lcg_fill(h, 153, 0.2))
    arrays["gamma"] = (1 + oracle.lcg_fill(d, 229, 0.3).astype(np.float64)).astype(np.float16)
    for name, v in arrays.items():
        assert hashlib.sha256(v.tobytes()).hexdigest() == str(z[f"sha_{name}_{key}"]), name
    return arrays


@pytest.mark.parametrize("case", range(4))
def test_ffn_matches_the_reference_graph_gate(case):
    z = np.load(GOLDEN)
    m, d, h = (int(v) for v in z["shapes"][case])
    a = _inputs(z, m, d, h)
    x, wg, wu, wd = a["x"].reshape(m, d), a["wg"].reshape(h, d), a["wu"].reshape(h, d), a["wd"].reshape(d, h)
    for use_bias in (0, 1):
        for norm in (0, 1):
            key = f"y_{m}_{d}_{h}_b{use_bias}_n{norm}"
            if key not in z.files:
                continue
            ref = z[key].reshape(m, d)
            got = oracle.ffn(x, wg, wu, wd, a["bias"] if use_bias else None, None, a["gamma"] if norm else None)
            if norm:
                err = np.abs(got.astype(np.float64) - ref.astype(np.float64)).max()
                assert err <= 0.003, (key, err)
            else:
                assert np.array_equal(got.view(np.uint16), ref.view(np.uint16)), key


def test_rmsnorm_rejections():
    x = np.zeros((3, 300), np.float16)
    g = np.ones(300, np.float16)
    x[1, 7] = 256.0                      # fp16(256^2) overflows: the row is rejected
    x[2, :256] = 16.0                    # 256 * 256 = 65536 >= 65504 in one tile: rejected
    y, bad = oracle.rmsnorm(x, g)
    assert bad == 2
    x[2, :256] = 15.0                    # 57600: accepted
    y, bad = oracle.rmsnorm(x[[0, 2]], g)
    assert bad == 0
    y, bad = oracle.rmsnorm(np.full((1, 8), 0.001, np.float16), np.full(8, 60000, np.float16))
    assert bad == 1                      # coefficient 60000 / sqrt(1e-6 + 1e-5) overflows FP16
