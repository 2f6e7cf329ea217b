"""CPU oracle for the FP16 Linear / HardSigmoid path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
import this package.  It is the checker, never the thing measured or shipped: the product
library (``rockchip-npu-notes_b200``) neither links nor calls it.

Contents
--------
* ``linear(...)``          ctypes front-end of ``linear_oracle.c`` (all modes, multi-threaded).
* ``linear_py(...)``       pure-Python restatement of the reference's file-gate oracle
                           (``research/custom-ops/tools/python/cli_gate.py:38-49``) for tiny cases.
* ``lcg_fill``             the file-gate input generator (``cli_gate.py:25-31``).
* ``XorShift``             the K-tiling probe generator and its ``dyadic`` / ``random_small``
                           draws (``research/custom-ops/tools/c/ktiling_probe.c:55-81``).
* ``plan_tasks``           the task/submit accounting the file gate checks (``cli_gate.py:79-86``).
* ``ew`` / ``rmsnorm`` / ``ffn``  ctypes front-end of ``graph_oracle.c``: the graph's elementwise
                           nodes, RMSNorm (``research/custom-ops/src/co_row_ops.c:150-224``) and the
                           SwiGLU FFN of the reference's graph gate (``tools/python/graph_gate.py``).

Parity pins: ``tests/golden/`` holds outputs produced by importing the reference's own Python
oracles; ``tests/test_oracle_golden.py`` checks this package against them bit for bit.
"""
import ctypes
import math
import os
import struct

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "build", "liblinear_oracle.so")

TILE16_EXACT = 0
TILE16_SEQ = 1
TILE16_FAST = 2
UNFUSED_SEQ = 3
FP64 = 4
FP32ACC = 5

MODES = {
    "tile16": TILE16_EXACT,
    "tile16_seq": TILE16_SEQ,
    "tile16_fast": TILE16_FAST,
    "unfused_seq": UNFUSED_SEQ,
    "fp64": FP64,
    "fp32acc": FP32ACC,
}

K_TILE = 256

_lib = None


def build():
    """Compile the C oracle in place (``oracle/build/liblinear_oracle.so``)."""
    import subprocess
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        u16p = ctypes.POINTER(ctypes.c_uint16)
        dp = ctypes.POINTER(ctypes.c_double)
        L.oracle_linear.argtypes = [ctypes.c_int, ctypes.c_uint, ctypes.c_uint, ctypes.c_uint,
                                    u16p, u16p, u16p, ctypes.c_int, u16p, dp, dp, ctypes.c_int]
        L.oracle_linear.restype = ctypes.c_int
        L.oracle_linear_pre.argtypes = [ctypes.c_int, ctypes.c_uint, ctypes.c_uint, ctypes.c_uint,
                                        u16p, u16p, dp, u16p, ctypes.c_int, u16p, dp, dp, ctypes.c_int]
        L.oracle_linear_pre.restype = ctypes.c_int
        L.oracle_f16_encode.argtypes = [dp, u16p, ctypes.c_size_t]
        L.oracle_f16_decode.argtypes = [u16p, dp, ctypes.c_size_t]
        L.oracle_ew.argtypes = [ctypes.c_int, u16p, u16p, u16p, ctypes.c_size_t]
        L.oracle_ew.restype = None
        L.oracle_rmsnorm.argtypes = [ctypes.c_uint, ctypes.c_uint, u16p, u16p, ctypes.c_float, u16p]
        L.oracle_rmsnorm.restype = ctypes.c_uint
        L.oracle_gate16.argtypes = [ctypes.c_int, ctypes.c_uint16]
        L.oracle_gate16.restype = ctypes.c_uint16
        _lib = L
    return _lib


def _u16(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        a = a.view(np.uint16)
    assert a.dtype == np.uint16
    return a


def _ptr(a, ct):
    return a.ctypes.data_as(ctypes.POINTER(ct)) if a is not None else None


class Widened:
    """W converted to float64 once, for repeated oracle calls against the same weights."""

    def __init__(self, w):
        self.w = _u16(w)
        self.wd = self.w.view(np.float16).astype(np.float64)


def linear(mode, x, w, bias=None, post=1, threads=None, want=("y16",)):
    """Run the C oracle.

    ``x`` [m,k], ``w`` [n,k] (or a ``Widened``), ``bias`` [n] or None: float16 arrays (or their
    uint16 bits).  ``post`` 1 = HardSigmoid, 0 = none.  ``want`` selects the outputs among
    ``y16`` (float16 [m,n]), ``act`` (float64 value before the final FP16 rounding) and ``raw``
    (float64 pre-bias accumulator).  Returns a dict.
    """
    if isinstance(mode, str):
        mode = MODES[mode]
    wd = None
    if isinstance(w, Widened):
        wd = w.wd
        w = w.w
    x = _u16(x)
    w = _u16(w)
    m, k = x.shape
    n, k2 = w.shape
    assert k == k2
    b = _u16(bias) if bias is not None else None
    if b is not None:
        assert b.shape == (n,)
    y16 = np.empty((m, n), np.uint16) if "y16" in want else None
    act = np.empty((m, n), np.float64) if "act" in want else None
    raw = np.empty((m, n), np.float64) if "raw" in want else None
    if threads is None:
        threads = os.cpu_count() or 1
    rc = lib().oracle_linear_pre(mode, m, k, n, _ptr(x, ctypes.c_uint16), _ptr(w, ctypes.c_uint16),
                                 _ptr(wd, ctypes.c_double), _ptr(b, ctypes.c_uint16), int(post),
                                 _ptr(y16, ctypes.c_uint16), _ptr(act, ctypes.c_double),
                                 _ptr(raw, ctypes.c_double), int(threads))
    if rc:
        raise RuntimeError(f"oracle_linear failed: {rc}")
    out = {}
    if y16 is not None:
        out["y16"] = y16.view(np.float16)
    if act is not None:
        out["act"] = act
    if raw is not None:
        out["raw"] = raw
    return out


def f16_encode(values):
    """Round float64 values to FP16 with the oracle's own RNE conversion (uint16 bits)."""
    v = np.ascontiguousarray(values, dtype=np.float64).ravel()
    out = np.empty(v.shape, np.uint16)
    lib().oracle_f16_encode(_ptr(v, ctypes.c_double), _ptr(out, ctypes.c_uint16), v.size)
    return out


# ----------------------------------------------------------------------- pure-Python restatement

def _f16(value):
    return struct.unpack("<e", struct.pack("<e", value))[0]


def linear_py(m, k, n, x, w, bias, post=1):
    """Pure-Python form of the file-gate oracle (tiny cases only).

    Follows research/custom-ops/tools/python/cli_gate.py:38-49: per 256-wide K tile an exactly
    rounded partial sum, ``dot = f16(dot + partial)``, ``affine = f16(dot + b)``,
    ``y = f16(clamp(affine / 6 + 0.5, 0, 1))``; ``bias=None`` skips the bias step and
    ``post=0`` skips the activation (research/custom-ops/src/linear_hardsigmoid.c:51-82).
    Inputs are flat lists of Python floats holding FP16 values.
    """
    out = []
    for row in range(m):
        for col in range(n):
            dot = 0.0
            for k0 in range(0, k, K_TILE):
                partial = math.fsum(x[row * k + q] * w[col * k + q]
                                    for q in range(k0, min(k0 + K_TILE, k)))
                dot = _f16(dot + partial)
            affine = _f16(dot + bias[col]) if bias is not None else dot
            if post:
                affine = _f16(min(1.0, max(0.0, affine / 6.0 + 0.5)))
            out.append(affine)
    return out


# ----------------------------------------------------------------------- graph nodes
# graph_oracle.c: elementwise node kinds (co_graph.c:293-313) and RMSNorm (co_row_ops.c:150-224)
EW_ADD, EW_MUL, EW_SILU, EW_GELU, EW_HSIG = 0, 1, 2, 3, 4
GATE_SIGMOID, GATE_GELU = 1, 2


def ew(op, a, b=None):
    """One elementwise graph node over float16 arrays of one shape (b only for ADD/MUL)."""
    a = _u16(a)
    bb = _u16(b) if b is not None else None
    y = np.empty(a.shape, np.uint16)
    lib().oracle_ew(op, _ptr(a, ctypes.c_uint16), _ptr(bb, ctypes.c_uint16), _ptr(y, ctypes.c_uint16), a.size)
    return y.view(np.float16)


def rmsnorm(x, gamma, eps=1e-5):
    """(y float16 [rows, cols], number of rejected rows) of the RMSNorm node; rejected rows are 0."""
    x = _u16(x)
    g = _u16(gamma)
    rows, cols = x.shape
    y = np.zeros((rows, cols), np.uint16)
    bad = lib().oracle_rmsnorm(rows, cols, _ptr(x, ctypes.c_uint16), _ptr(g, ctypes.c_uint16), float(eps),
                               _ptr(y, ctypes.c_uint16))
    return y.view(np.float16), int(bad)


def ffn(x, wg, wu, wd, bias=None, bias_up=None, gamma=None, eps=1e-5, act=EW_SILU):
    """The graph FFN Y = X + Linear(act(Linear(Z, Wg, bias)) * Linear(Z, Wu, bias_up), Wd), Z = X or
    RMSNorm(X): every node with the reference's arithmetic (Linear: TILE16_EXACT, the file gate's
    per-256-K FP16 fold), bit-identical to research/custom-ops/tools/python/graph_gate.py:30-41
    except for the RMSNorm coefficient (graph_oracle.c)."""
    z = x
    if gamma is not None:
        z, bad = rmsnorm(x, gamma, eps)
        if bad:
            raise ValueError("RMSNorm rejected a row")
    g = linear(TILE16_EXACT, z, wg, bias, post=0)["y16"]
    u = linear(TILE16_EXACT, z, wu, bias_up, post=0)["y16"]
    hidden = ew(EW_MUL, ew(act, g), u)
    down = linear(TILE16_EXACT, hidden, wd, None, post=0)["y16"]
    return ew(EW_ADD, down, x)


# ----------------------------------------------------------------------- input generators

def lcg_fill(count, seed, scale):
    """File-gate generator (cli_gate.py:25-31): 32-bit LCG, 16 bits -> [-1,1) * scale -> FP16."""
    out = np.empty(count, np.float64)
    s = seed & 0xFFFFFFFF
    for i in range(count):
        s = (1664525 * s + 1013904223) & 0xFFFFFFFF
        out[i] = (((s >> 8) & 0xFFFF) / 65535 * 2 - 1) * scale
    return out.astype(np.float16)


class XorShift:
    """K-tiling probe generator (ktiling_probe.c:55-81): xorshift32 with two FP16 draws."""

    DYADIC = (0.0, 0.0625, -0.0625, 0.03125, -0.03125, 0.015625, -0.015625, 0.0078125)

    def __init__(self, state):
        self.state = state & 0xFFFFFFFF

    def next(self):
        x = self.state
        x ^= (x << 13) & 0xFFFFFFFF
        x ^= x >> 17
        x ^= (x << 5) & 0xFFFFFFFF
        self.state = x
        return x

    def dyadic(self):
        return self.DYADIC[self.next() % len(self.DYADIC)]

    def random_small(self):
        return ((self.next() % 10001) - 5000.0) / 100000.0

    def fill(self, count, pattern):
        vals = [self.random_small() if pattern else self.dyadic() for _ in range(count)]
        return np.asarray(vals, np.float64).astype(np.float16)


# ----------------------------------------------------------------------- plan accounting

def plan_tasks(m, k, n, has_bias=True, hsig=True):
    """Reference task accounting (research/custom-ops/src/linear_plan.c:17-41, cli_gate.py:79-86).

    Returns (output_tiles, tasks): per output tile ``ceil(K/256) + has_bias + lut_chunks``, where
    lut_chunks = ceil(physical_rows * physical_cols / 32768) for the HardSigmoid post-op.
    """
    tasks = 0
    for m0 in range(0, m, 256):
        rows = ((max(min(256, m - m0), 12) + 3) // 4) * 4
        for n0 in range(0, n, 256):
            cols = ((min(256, n - n0) + 31) // 32) * 32
            tasks += (k + 255) // 256 + int(has_bias) + (((rows * cols + 32767) // 32768) if hsig else 0)
    output_tiles = ((m + 255) // 256) * ((n + 255) // 256)
    return output_tiles, tasks


def tolerance_ok(got, ref, atol=2e-3, rtol=2e-3):
    """Element-wise ``|got - ref| <= atol + rtol*|ref|`` (the operator's stated tolerance)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref)
    bound = atol + rtol * np.abs(ref)
    return bool(np.all(np.isfinite(got)) and np.all(err <= bound)), float(np.max(err / bound)) if err.size else 0.0
