"""The host C layer against a CPU stand-in of the device seam (no GPU).

Compiles the library's host sources (rockchip-npu-notes_b200/csrc/host) with tests/c/mock_device.c
(the seam on the CPU, results from the oracle's C restatement) and tests/c/host_test.c, the way
the reference builds its host tests against a mock NPU
(research/custom-ops/tests/c/multitile_host_test.c), and runs the binary: publish-on-success,
error codes, the fail-Nth fault seam without leaks, cube entries with guard checks, weight
refresh, the grouped device entry and a one-rank fused K-split round, all bit-exact against the
oracle; and the graph compiler (tests/c/graph_host_test.c).
"""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST = os.path.join(ROOT, "rockchip-npu-notes_b200", "csrc", "host")


def _build_and_run(tmp_path, test_source, banner):
    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("gcc not available")
    sources = [os.path.join(HOST, f) for f in ("rocket.c", "tensor.c", "plan.c", "linear.c", "ksplit.c", "graph.c")]
    sources += [os.path.join(ROOT, "tests", "c", "mock_device.c"), os.path.join(ROOT, "tests", "c", test_source),
                os.path.join(ROOT, "oracle", "linear_oracle.c"), os.path.join(ROOT, "oracle", "graph_oracle.c"),
                os.path.join(ROOT, "oracle", "rkplan_oracle.c")]
    exe = tmp_path / test_source.replace(".c", "")
    cmd = [cc, "-std=gnu11", "-O1", "-Wall", "-Werror=implicit-function-declaration",
           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "rockchip-npu-notes_b200", "csrc"),
           "-I", HOST, *sources, "-lpthread", "-lm", "-o", str(exe)]
    build = subprocess.run(cmd, capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    env = dict(os.environ, B2_MOCK_DEVICES="1")
    env.pop("B2_DEVICE", None)
    run = subprocess.run([str(exe)], capture_output=True, text=True, env=env, timeout=300)
    assert run.returncode == 0, run.stdout + run.stderr
    assert banner in run.stdout and " 0 failures" in run.stdout, run.stdout


def test_host_layer_with_mock_device(tmp_path):
    _build_and_run(tmp_path, "host_test.c", "host_test:")


def test_graph_compiler_with_mock_device(tmp_path):
    """co_graph_* (csrc/host/graph.c) the way the reference's graph_host_test.c checks its graph
    compiler: plan, slot reuse, bindings, publish-on-success, fail-Nth without leaks, RMSNorm
    rejections, multiple outputs, CO_CHAIN fusion -- every result bit-exact against the oracle."""
    _build_and_run(tmp_path, "graph_host_test.c", "graph_host_test:")
