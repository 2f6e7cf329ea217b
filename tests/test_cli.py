"""The linear_hardsigmoid file CLI against the reference's file-gate contract.

research/custom-ops/tools/python/cli_gate.py drives research/custom-ops/tools/c/operator_cli.c:
  * SHAPES with LCG inputs, both modes, repeat 3: output within 0.002 of the oracle, chain and
    separate outputs byte-identical, and "repeat=3 submits=S tasks=T PASS" with S = output_tiles*3
    (chain) or tasks*3 (separate) and T = tasks*3 (cli_gate.py:55-96);
  * invalid sizes / non-finite input / bad dims exit 1 and leave an existing output file
    untouched (cli_gate.py:98-114);
  * no device exits 77 (operator_cli.c:75-76).
The negative cases fail before any device is opened, so they run on a CPU-only host as well.
"""
import json
import math
import os
import re
import shutil
import struct
import subprocess

import numpy as np
import pytest

import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run(cli, args, timeout=120):
    return subprocess.run([cli] + [str(a) for a in args], capture_output=True, text=True, timeout=timeout)


def write_half(path, values):
    path.write_bytes(np.asarray(values, np.float16).tobytes())


def test_help_and_usage(b2):
    r = run(b2.CLI_PATH, ["--help"])
    assert r.returncode == 0 and "usage:" in r.stdout
    assert run(b2.CLI_PATH, []).returncode == 1
    assert run(b2.CLI_PATH, [1, 1, 1, "a", "b", "c", "d", "sideways"]).returncode == 1


def test_invalid_inputs_preserve_existing_output(b2, tmp_path):
    xfile, wfile, bfile, out = (tmp_path / n for n in ("x.bin", "w.bin", "b.bin", "y.bin"))
    write_half(wfile, [1])
    write_half(bfile, [0])
    marker = b"existing-output-preserved"
    cases = [(b"", "1"), (struct.pack("<ee", 1, 2), "1"), (struct.pack("<e", math.nan), "1"),
             (struct.pack("<e", 1), "0"), (struct.pack("<e", 1), "4097")]
    for data, m in cases:
        xfile.write_bytes(data)
        out.write_bytes(marker)
        r = run(b2.CLI_PATH, [m, 1, 1, xfile, wfile, bfile, out])
        assert r.returncode == 1, (m, data, r.stderr)
        assert out.read_bytes() == marker
    # output path equal to an input path is refused
    xfile.write_bytes(struct.pack("<e", 1))
    assert run(b2.CLI_PATH, [1, 1, 1, xfile, wfile, bfile, wfile]).returncode == 1


def test_no_device_exits_77(b2, tmp_path):
    if b2.device_count() > 0:
        pytest.skip("a CUDA device is present")
    xfile, wfile, bfile, out = (tmp_path / n for n in ("x.bin", "w.bin", "b.bin", "y.bin"))
    for f in (xfile, wfile):
        write_half(f, [1])
    write_half(bfile, [0])
    out.write_bytes(b"keep")
    r = run(b2.CLI_PATH, [1, 1, 1, xfile, wfile, bfile, out])
    assert r.returncode == 77 and out.read_bytes() == b"keep"


def _mock_cli(tmp_path):
    """The CLI linked against the library's host sources and the CPU stand-in of the device seam
    (tests/c/mock_device.c, results from the oracle's exact tile-16 arithmetic)."""
    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("gcc not available")
    host = os.path.join(ROOT, "rockchip-npu-notes_b200", "csrc", "host")
    sources = [os.path.join(host, f) for f in ("cli.c", "rocket.c", "tensor.c", "plan.c", "linear.c", "ksplit.c",
                                                "graph.c")]
    sources += [os.path.join(ROOT, "tests", "c", "mock_device.c"), os.path.join(ROOT, "oracle", "linear_oracle.c"),
                os.path.join(ROOT, "oracle", "graph_oracle.c"), os.path.join(ROOT, "oracle", "rkplan_oracle.c")]
    exe = tmp_path / "linear_hardsigmoid_mock"
    inc = ["-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "rockchip-npu-notes_b200", "csrc"), "-I", host]
    strict = subprocess.run([cc, "-std=gnu11", "-O2", "-Wall", "-Wextra", "-Wno-unused-parameter", "-Werror",
                             "-fsyntax-only", *inc, sources[0]], capture_output=True, text=True)
    assert strict.returncode == 0, strict.stderr
    build = subprocess.run([cc, "-std=gnu11", "-O1", *inc, *sources, "-lpthread", "-lm", "-o", str(exe)],
                           capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    return str(exe)


def _file_gate(cli, tmp_path, env=None):
    """research/custom-ops/tools/python/cli_gate.py:55-96 against `cli`: every SHAPES case in both
    modes with repeat 3 -- output within 0.002 of the reference oracle's stored result, chain and
    separate byte-identical, the plan-derived counters in the PASS line, launches= after PASS."""
    z = np.load(os.path.join(GOLDEN, "cli_gate_shapes.npz"))
    meta = json.loads(bytes(z["meta"]).decode())
    for case in meta:
        m, k, n = case["m"], case["k"], case["n"]
        x, w, b = oracle.lcg_fill(m * k, 303, 1.7), oracle.lcg_fill(n * k, 911, 0.21), oracle.lcg_fill(n, 409, 4.7)
        files = [tmp_path / f"{m}-{k}-{n}-{s}.bin" for s in ("x", "w", "b")]
        for f, v in zip(files, (x, w, b)):
            write_half(f, v)
        want = z[f"y_{m}_{k}_{n}"].view(np.float16)
        tiles, tasks = oracle.plan_tasks(m, k, n)
        outputs = {}
        for mode in ("separate", "chain"):
            out = tmp_path / f"{m}-{k}-{n}-{mode}-y.bin"
            r = subprocess.run([cli, *map(str, (m, k, n, *files, out, mode, 3))], capture_output=True, text=True,
                               timeout=300, env=env)
            assert r.returncode == 0, r.stderr
            got = np.frombuffer(out.read_bytes(), np.float16)
            assert got.size == m * n
            assert np.all(np.isfinite(got)) and np.max(np.abs(got.astype(np.float64) - want)) <= 0.002
            subs = tiles * 3 if mode == "chain" else tasks * 3
            mt = re.search(r"repeat=3 submits=(\d+) tasks=(\d+) PASS", r.stdout)
            assert mt and (int(mt[1]), int(mt[2])) == (subs, tasks * 3), r.stdout
            assert re.search(r"PASS launches=\d+", r.stdout)
            outputs[mode] = out.read_bytes()
        assert outputs["chain"] == outputs["separate"]
        assert not [p for p in os.listdir(tmp_path) if ".partial-" in p], "temporary output left behind"


def test_file_gate_on_mock_device(tmp_path):
    """The CLI's own logic (parsing, input mapping, repeat comparison, publish by rename, PASS
    line) end to end on a CPU-only host, against the reference gate's stored outputs."""
    cli = _mock_cli(tmp_path)
    env = dict(os.environ, B2_MOCK_DEVICES="1")
    env.pop("B2_DEVICE", None)
    _file_gate(cli, tmp_path, env)
    # the negative cases of the gate against the same binary (no device is reached)
    xfile, wfile, bfile, out = (tmp_path / n for n in ("nx.bin", "nw.bin", "nb.bin", "ny.bin"))
    write_half(wfile, [1])
    write_half(bfile, [0])
    for data, m in [(b"", "1"), (struct.pack("<ee", 1, 2), "1"), (struct.pack("<e", math.inf), "1"),
                    (struct.pack("<e", 1), "0"), (struct.pack("<e", 1), "4097"), (struct.pack("<e", 1), "01x")]:
        xfile.write_bytes(data)
        out.write_bytes(b"keep")
        r = subprocess.run([cli, m, "1", "1", str(xfile), str(wfile), str(bfile), str(out)], capture_output=True,
                           text=True, env=env, timeout=60)
        assert r.returncode == 1 and out.read_bytes() == b"keep", (m, data)
    # a directory where an input file belongs, and repeat out of range
    r = subprocess.run([cli, "1", "1", "1", str(tmp_path), str(wfile), str(bfile), str(out)], capture_output=True,
                       text=True, env=env, timeout=60)
    assert r.returncode == 1
    xfile.write_bytes(struct.pack("<e", 1))
    for rep in ("0", "1001", "-3"):
        r = subprocess.run([cli, "1", "1", "1", str(xfile), str(wfile), str(bfile), str(out), "chain", rep],
                           capture_output=True, text=True, env=env, timeout=60)
        assert r.returncode == 1 and out.read_bytes() == b"keep"
    # no device behind the seam: exit 77 after the inputs were found valid
    r = subprocess.run([cli, "1", "1", "1", str(xfile), str(wfile), str(bfile), str(out)], capture_output=True,
                       text=True, env=dict(env, B2_MOCK_DEVICES="0"), timeout=60)
    assert r.returncode == 77 and out.read_bytes() == b"keep"


def test_nonfinite_scan_positions(tmp_path):
    """The word-wise finiteness scan reports a NaN or Inf wherever it sits in a 4-half word and in
    the tail (inputs of 1..9 halves, every position)."""
    cli = _mock_cli(tmp_path)
    env = dict(os.environ, B2_MOCK_DEVICES="1")
    wfile, bfile, xfile, out = (tmp_path / n for n in ("w.bin", "b.bin", "x.bin", "y.bin"))
    write_half(bfile, [0])
    for k in range(1, 10):
        write_half(wfile, np.full(k, 0.5))
        for pos in range(k):
            for bad in (math.nan, math.inf, -math.inf):
                v = np.full(k, 1.0)
                v[pos] = bad
                write_half(xfile, v)
                r = subprocess.run([cli, "1", str(k), "1", str(xfile), str(wfile), str(bfile), str(out)],
                                   capture_output=True, text=True, env=env, timeout=60)
                assert r.returncode == 1 and f"value {pos} is not finite" in r.stderr, (k, pos, r.stderr)
        write_half(xfile, np.full(k, 65504.0 if k % 2 else -65504.0))
        r = subprocess.run([cli, "1", str(k), "1", str(xfile), str(wfile), str(bfile), str(out)],
                           capture_output=True, text=True, env=env, timeout=60)
        assert "not finite" not in r.stderr, (k, r.stderr)


@pytest.mark.gpu
def test_file_gate_on_gpu(b2, tmp_path):
    _file_gate(b2.CLI_PATH, tmp_path)
