"""Pin the CPU oracle to the reference's own oracles (CPU only).

The fixtures under tests/golden/ were produced by importing the reference's unmodified
``cli_gate.py`` and ``ktiling_gate.py`` (research/custom-ops/tools/python/); the generating script
is tests/golden/make_golden.py.  Everything here must match bit for bit: FP16 outputs as bits,
double-valued references with ``==``.
"""
import hashlib
import json
import os

import numpy as np
import pytest

import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _sha(a):
    return hashlib.sha256(np.asarray(a, np.float16).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def cli_fixture():
    z = np.load(os.path.join(GOLDEN, "cli_gate_shapes.npz"))
    return z, json.loads(bytes(z["meta"]).decode())


@pytest.fixture(scope="module")
def ktiling_fixture():
    z = np.load(os.path.join(GOLDEN, "ktiling_cases.npz"))
    return z, json.loads(bytes(z["index"]).decode())


def test_lcg_fill_matches_reference_generator(cli_fixture):
    """oracle.lcg_fill reproduces cli_gate.fill (cli_gate.py:25-31) byte for byte."""
    _, meta = cli_fixture
    for case in meta:
        m, k, n = case["m"], case["k"], case["n"]
        assert _sha(oracle.lcg_fill(m * k, 303, 1.7)) == case["x_sha256"]
        assert _sha(oracle.lcg_fill(n * k, 911, 0.21)) == case["w_sha256"]
        assert _sha(oracle.lcg_fill(n, 409, 4.7)) == case["b_sha256"]


def test_tile16_exact_is_bitwise_cli_gate_oracle(cli_fixture):
    """The C oracle's TILE16_EXACT mode equals cli_gate.oracle on every SHAPES case."""
    z, meta = cli_fixture
    for case in meta:
        m, k, n = case["m"], case["k"], case["n"]
        x = oracle.lcg_fill(m * k, 303, 1.7).reshape(m, k)
        w = oracle.lcg_fill(n * k, 911, 0.21).reshape(n, k)
        b = oracle.lcg_fill(n, 409, 4.7)
        got = oracle.linear("tile16", x, w, b, post=1)["y16"].view(np.uint16).ravel()
        want = z[f"y_{m}_{k}_{n}"]
        assert np.array_equal(got, want), f"{m}x{k}x{n}: {np.count_nonzero(got != want)} differ"


def test_python_restatement_matches_cli_gate_small(cli_fixture):
    """oracle.linear_py (pure Python) equals the reference on the small SHAPES cases."""
    z, meta = cli_fixture
    for case in meta:
        m, k, n = case["m"], case["k"], case["n"]
        if m * k * n > 200_000:
            continue
        x = [float(v) for v in oracle.lcg_fill(m * k, 303, 1.7)]
        w = [float(v) for v in oracle.lcg_fill(n * k, 911, 0.21)]
        b = [float(v) for v in oracle.lcg_fill(n, 409, 4.7)]
        got = np.asarray(oracle.linear_py(m, k, n, x, w, b), np.float64).astype(np.float16)
        assert np.array_equal(got.view(np.uint16), z[f"y_{m}_{k}_{n}"])


def _case_inputs(z, i, case):
    if case["regen"]:
        rng = oracle.XorShift(0x9E3779B9 * 11 + 131 + 7)
        x = rng.fill(256 * 4096, 1)[: case["m"] * case["k"]]
        w = rng.fill(256 * 4096, 1)
        b = rng.fill(256, 1)
        digest = hashlib.sha256(x.tobytes() + w.tobytes()).hexdigest()
        assert digest == case["inputs_sha256"]
        return x, w, b
    x = z[f"c{i}_x"].view(np.float16)
    w = z[f"c{i}_w"].view(np.float16)
    b = z[f"c{i}_b"].view(np.float16) if case["bias"] else None
    return x, w, b


def test_ktiling_references_bitwise(ktiling_fixture):
    """raw16/act16 (tile-FP16, sequential double tiles), raw64/act64 (FP64), fused and unfused."""
    z, index = ktiling_fixture
    for i, case in enumerate(index):
        m, n, k = case["m"], case["n"], case["k"]
        x, w, b = _case_inputs(z, i, case)
        x = x.reshape(m, k)
        w = w.reshape(n, k)
        post = 1 if case["bias"] else 0
        mode16 = "unfused_seq" if case["unfused"] else "tile16_seq"
        r16 = oracle.linear(mode16, x, w, b, post=post, want=("act", "raw"))
        r64 = oracle.linear("fp64", x, w, b, post=post, want=("act", "raw"))
        for label, got in (("raw16", r16["raw"]), ("act16", r16["act"]),
                           ("raw64", r64["raw"]), ("act64", r64["act"])):
            want = z[f"c{i}_{label}"].reshape(m, n)
            assert np.array_equal(got, want), f"{case['name']} {m}x{n}x{k} {label}"


def test_exact_and_sequential_tile_sums_agree_on_dyadic_kats(ktiling_fixture):
    """Impulse / cancellation cases are exact: every tile16 flavour gives identical bits."""
    z, index = ktiling_fixture
    for i, case in enumerate(index):
        if not (case["name"].startswith("chan") or case["name"].startswith("cancel")):
            continue
        m, n, k = case["m"], case["n"], case["k"]
        x, w, b = _case_inputs(z, i, case)
        x = x.reshape(m, k)
        w = w.reshape(n, k)
        outs = [oracle.linear(mode, x, w, None, post=0)["y16"].view(np.uint16)
                for mode in ("tile16", "tile16_seq", "tile16_fast", "fp32acc")]
        for o in outs[1:]:
            assert np.array_equal(o, outs[0]), case["name"]
        want = z[f"c{i}_raw16"].reshape(m, n).astype(np.float16).view(np.uint16)
        assert np.array_equal(outs[0], want)


def test_task_accounting_matches_reference():
    with open(os.path.join(GOLDEN, "ktiling_tasks.json")) as f:
        tasks = json.load(f)
    for key, v in tasks.items():
        m, n, k = map(int, key.split("_"))
        tiles, fused = oracle.plan_tasks(m, k, n, has_bias=True, hsig=True)
        assert tiles == 1 or m > 256 or n > 256
        assert fused == v["fused"], key
        _, raw = oracle.plan_tasks(m, k, n, has_bias=False, hsig=False)
        assert raw == v["raw"], key


def test_f16_rounding_matches_numpy():
    """The oracle's double->FP16 RNE conversion equals numpy's on random and edge values."""
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(200_000) * np.exp2(rng.integers(-30, 17, 200_000)),
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, -65520.0, 1e9, 2.0 ** -24, 2.0 ** -25,
                  2.0 ** -25 * 1.0000001, 3 * 2.0 ** -26, 2.0 ** -14, 2.0 ** -14 - 2.0 ** -25,
                  np.inf, -np.inf]),
        # exact ties between adjacent FP16 values
        (np.arange(1024, 2048, dtype=np.float64) + 0.5) * 2.0 ** -10,
    ])
    with np.errstate(over="ignore"):
        want = vals.astype(np.float16).view(np.uint16)
    got = oracle.f16_encode(vals)
    assert np.array_equal(got, want)


def test_fp32acc_and_fast_within_tolerance_of_exact():
    rng = np.random.default_rng(1)
    m, k, n = 33, 1000, 47
    x = rng.uniform(-1, 1, (m, k)).astype(np.float16)
    w = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), (n, k)).astype(np.float16)
    b = rng.uniform(-0.1, 0.1, n).astype(np.float16)
    ref = oracle.linear("tile16", x, w, b, post=0)["y16"]
    for mode in ("tile16_fast", "tile16_seq", "fp32acc"):
        ok, worst = oracle.tolerance_ok(oracle.linear(mode, x, w, b, post=0)["y16"], ref)
        assert ok, (mode, worst)
    fast = oracle.linear("tile16_fast", x, w, b, post=0)["y16"]
    assert np.array_equal(fast.view(np.uint16), ref.view(np.uint16))
