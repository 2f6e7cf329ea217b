#!/usr/bin/env python3
"""Generate the golden fixture that pins the graph tests to the reference's own FFN graph oracle.

Run once, on a machine that has the reference checkout (it is NOT needed at test time):

    python tests/golden/make_graph_golden.py <reference checkout>

It imports research/custom-ops/tools/python/graph_gate.py (standard library only, unmodified;
it imports cli_gate.py from the same directory) and, for every ``SHAPES`` case (m, d, h), with
and without the gate bias and with and without the RMSNorm prologue (the RMSNorm form only for the
shapes below 10^7 multiply-adds per Linear, to keep the file small), stores the output of
``graph_gate.oracle`` -- Y = X + Linear(SiLU(Linear(Z, Wg, b)) * Linear(Z, Wu), Wd) with Z = X or
RMSNorm(X) -- on the gate's own inputs (``fill`` with seeds 123/451/911/771/153/229), plus SHA-256
digests of those inputs, which pin the restated generator ``oracle.lcg_fill`` the tests use to
rebuild them. Output: ``graph_gate_ffn.npz`` next to this script.
"""
import hashlib
import importlib.util
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def sha(values):
    return hashlib.sha256(np.asarray(values, np.float64).astype(np.float16).tobytes()).hexdigest()


def inputs(gate, m, d, h):
    """The gate's own inputs for one shape (graph_gate.py:67-73)."""
    x = gate.fill(m * d, 123, 0.7)
    wg = gate.fill(h * d, 451, 0.06)
    wu = gate.fill(h * d, 911, 0.07)
    wd = gate.fill(d * h, 771, 0.05)
    bias = gate.fill(h, 153, 0.2)
    gamma = [gate.f16(1 + v) for v in gate.fill(d, 229, 0.3)]
    return x, wg, wu, wd, bias, gamma


def main(ref_root):
    tools = os.path.join(ref_root, "research", "custom-ops", "tools", "python")
    sys.path.insert(0, tools)
    gate = load(os.path.join(tools, "graph_gate.py"), "ref_graph_gate")
    out = {"shapes": np.array(gate.SHAPES, np.int64)}
    for (m, d, h) in gate.SHAPES:
        x, wg, wu, wd, bias, gamma = inputs(gate, m, d, h)
        key = f"{m}_{d}_{h}"
        for name, v in (("x", x), ("wg", wg), ("wu", wu), ("wd", wd), ("bias", bias), ("gamma", gamma)):
            out[f"sha_{name}_{key}"] = np.array(sha(v))
        for use_bias in (False, True):
            for norm in (False, True):
                if norm and m * d * h > 10 ** 7:   # keeps the fixture small; the plain case covers the shape
                    continue
                t0 = time.time()
                y = gate.oracle(m, d, h, x, wg, wu, wd, bias if use_bias else None, gamma if norm else None)
                out[f"y_{key}_b{int(use_bias)}_n{int(norm)}"] = np.asarray(y, np.float64).astype(np.float16)
                print(f"{key} bias={use_bias} rmsnorm={norm}: {time.time() - t0:.1f} s", flush=True)
    np.savez_compressed(os.path.join(HERE, "graph_gate_ffn.npz"), **out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: {sys.argv[0]} REFERENCE_CHECKOUT  (the Ecazy/rockchip-npu-notes root)")
    main(sys.argv[1])
