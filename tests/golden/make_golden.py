#!/usr/bin/env python3
"""Generate the golden fixtures that pin the CPU oracle to the reference's own oracles.

Run once, on a machine that has the reference checkout (it is NOT needed at test time):

    python tests/golden/make_golden.py <reference checkout>

It imports two standard-library-only scripts of the reference, unmodified:

* research/custom-ops/tools/python/cli_gate.py    -- ``fill`` (LCG inputs), ``SHAPES`` and
  ``oracle`` (per-256-K-tile exactly rounded partials, FP16 running sum, bias, HardSigmoid);
* research/custom-ops/tools/python/ktiling_gate.py -- ``reference`` (FP64 and tile-FP16 raw and
  activated references, fused and unfused) and ``expected_tasks``/``lut_chunks``.

and writes, next to this script:

* ``cli_gate_shapes.npz``  every ``SHAPES`` case: the oracle's FP16 output plus SHA-256 digests
  of the generated X/W/b bytes (which pin ``oracle.lcg_fill``);
* ``ktiling_cases.npz``    K-boundary, impulse, cancellation, prefix and unfused cases:
  inputs and the four reference arrays raw64/raw16/act64/act16;
* ``ktiling_tasks.json``   task accounting from ``ktiling_gate.expected_tasks``.
"""
import hashlib
import importlib.util
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
import oracle  # noqa: E402  (restated generators, for the ktiling inputs)


def load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def sha(values):
    return hashlib.sha256(np.asarray(values, np.float64).astype(np.float16).tobytes()).hexdigest()


def main(ref_root):
    tools = os.path.join(ref_root, "research", "custom-ops", "tools", "python")
    cli_gate = load(os.path.join(tools, "cli_gate.py"), "ref_cli_gate")
    kgate = load(os.path.join(tools, "ktiling_gate.py"), "ref_ktiling_gate")

    # ---------------------------------------------------------------- file-gate shapes
    out = {}
    meta = []
    for (m, k, n) in cli_gate.SHAPES:
        t0 = time.time()
        x, w, b = cli_gate.fill(m * k, 303, 1.7), cli_gate.fill(n * k, 911, 0.21), cli_gate.fill(n, 409, 4.7)
        y = cli_gate.oracle(m, k, n, x, w, b)
        key = f"{m}_{k}_{n}"
        out["y_" + key] = np.asarray(y, np.float64).astype(np.float16).view(np.uint16)
        meta.append({"m": m, "k": k, "n": n, "x_sha256": sha(x), "w_sha256": sha(w), "b_sha256": sha(b)})
        print(f"cli_gate {key}: {time.time() - t0:.1f}s", flush=True)
    out["meta"] = np.frombuffer(json.dumps(meta).encode(), np.uint8)
    np.savez_compressed(os.path.join(HERE, "cli_gate_shapes.npz"), **out)

    # ---------------------------------------------------------------- K-tiling cases
    cases = []
    contract = [(1, 1, 255, 0), (16, 32, 256, 0), (29, 45, 257, 1), (64, 64, 511, 0),
                (1, 1, 512, 1), (16, 32, 513, 0), (29, 45, 769, 1), (64, 64, 1024, 0),
                (16, 32, 2049, 1), (29, 45, 4096, 0)]
    for i, (m, n, k, pattern) in enumerate(contract):
        rng = oracle.XorShift(0x9E3779B9 * (i + 1) + 131 + 7)
        x = rng.fill(m * k, pattern)
        w = rng.fill(n * k, pattern)
        b = rng.fill(n, 1)
        cases.append(("contract", m, n, k, x, w, b, False))
    # single nonzero channel straddling K-tile edges (ktiling_probe.c:951-976)
    for (m, n, k, kk) in [(16, 32, 255, 254), (16, 32, 256, 255), (16, 32, 257, 256),
                          (16, 32, 513, 257), (29, 45, 511, 255), (29, 45, 512, 256),
                          (29, 45, 513, 512), (29, 45, 1024, 511), (32, 16, 769, 768),
                          (32, 16, 1024, 1023), (32, 16, 2049, 2048), (64, 64, 4096, 4095)]:
        x = np.zeros((m, k), np.float16)
        w = np.zeros((n, k), np.float16)
        x[:, kk] = 1.0
        w[:, kk] = np.where(np.arange(n) & 1, -0.0625, 0.0625)
        cases.append((f"chan-k{kk}", m, n, k, x.ravel(), w.ravel(), None, False))
    # signed cancellation across two K tiles (ktiling_probe.c:977-985)
    m, n, k = 16, 16, 513
    x = np.zeros((m, k), np.float16)
    w = np.zeros((n, k), np.float16)
    x[:, 17] = 1.0
    x[:, 300] = 1.0
    w[:, 17] = 0.0625
    w[:, 300] = -0.0625
    cases.append(("cancel-k513", m, n, k, x.ravel(), w.ravel(), None, False))
    # raw accumulators over several K tiles (ktiling_probe.c:987-997)
    for i, k in enumerate((257, 769, 1024)):
        rng = oracle.XorShift(0x27D4EB2F * (i + 1) + 1)
        x = rng.fill(16 * k, i & 1)
        w = rng.fill(32 * k, i & 1)
        cases.append(("prefix", 16, 32, k, x, w, None, False))
    # unfused graph arm: every tile sum narrowed before the fold (ktiling_gate.py:108)
    rng = oracle.XorShift(0xB5297A4D * 3 + 17)
    x = rng.fill(64 * 1024, 1)
    w = rng.fill(64 * 1024, 1)
    b = rng.fill(64, 1)
    cases.append(("perf-unfused", 64, 64, 1024, x, w, b, True))

    # M=N=256, K=4096 (two LUT chunks in the reference); inputs are regenerated from the seed at
    # test time and only the first 16 output rows are stored (rows are independent).
    rng = oracle.XorShift(0x9E3779B9 * 11 + 131 + 7)
    x = rng.fill(256 * 4096, 1)
    w = rng.fill(256 * 4096, 1)
    b = rng.fill(256, 1)
    cases.append(("contract-regen", 16, 256, 4096, x[:16 * 4096], w, b, False))

    arrays = {}
    index = []
    for ci, (name, m, n, k, x, w, b, unfused) in enumerate(cases):
        t0 = time.time()
        xl = [float(v) for v in np.asarray(x, np.float16)]
        wl = [float(v) for v in np.asarray(w, np.float16)]
        bl = None if b is None else [float(v) for v in np.asarray(b, np.float16)]
        raw64, raw16, act64, act16 = kgate.reference(m, n, k, xl, wl, bl, unfused=unfused)
        p = f"c{ci}_"
        regen = name.endswith("-regen")
        if not regen:
            arrays[p + "x"] = np.asarray(x, np.float16).view(np.uint16)
            arrays[p + "w"] = np.asarray(w, np.float16).view(np.uint16)
            if b is not None:
                arrays[p + "b"] = np.asarray(b, np.float16).view(np.uint16)
        for label, arr in (("raw64", raw64), ("raw16", raw16), ("act64", act64), ("act16", act16)):
            arrays[p + label] = np.asarray(arr, np.float64)
        kind = "raw" if b is None else ("perf-unfused" if unfused else "contract")
        index.append({"name": name, "m": m, "n": n, "k": k, "bias": b is not None, "regen": regen,
                      "inputs_sha256": hashlib.sha256(np.asarray(x, np.float16).tobytes() +
                                                      np.asarray(w, np.float16).tobytes()).hexdigest(),
                      "unfused": unfused, "expected_tasks": kgate.expected_tasks(m, n, k, kind),
                      "lut_chunks": kgate.lut_chunks(m, n)})
        print(f"ktiling {name} {m}x{n}x{k}: {time.time() - t0:.1f}s", flush=True)
    arrays["index"] = np.frombuffer(json.dumps(index).encode(), np.uint8)
    np.savez_compressed(os.path.join(HERE, "ktiling_cases.npz"), **arrays)

    tasks = {f"{m}_{n}_{k}": {"fused": kgate.expected_tasks(m, n, k, "perf"),
                              "unfused": kgate.expected_tasks(m, n, k, "perf-unfused"),
                              "raw": kgate.expected_tasks(m, n, k, "raw")}
             for (m, n, k) in [(64, 64, 4096), (256, 256, 1024), (256, 256, 4096), (1, 1, 1)]}
    with open(os.path.join(HERE, "ktiling_tasks.json"), "w") as f:
        json.dump(tasks, f, indent=1, sort_keys=True)
        f.write("\n")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: {sys.argv[0]} REFERENCE_CHECKOUT  (the Ecazy/rockchip-npu-notes root)")
    main(sys.argv[1])
