"""The plan/workspace ABI (include/rk_plan.h) through tests/c/rk_plan_test.c.

The reference tests its RKPlan runtime from C against a mock NPU
(research/custom-ops/tests/c/rk_plan_host_test.c); the same C test runs here twice:
  * CPU: linked with the library's host sources and the CPU stand-in of the device seam
    (tests/c/mock_device.c, results from oracle/rkplan_oracle.c), with the mock's NaN and guard
    injections and the allocation-leak checks;
  * B200: linked with the built library, every expected value computed in the test from the
    templates' definitions and compared bit for bit.
"""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST = os.path.join(ROOT, "rockchip-npu-notes_b200", "csrc", "host")
INC = ["-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "rockchip-npu-notes_b200", "csrc"), "-I", HOST]


def _gcc():
    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("gcc not available")
    return cc


def _run(exe, env):
    run = subprocess.run([exe], capture_output=True, text=True, env=env, timeout=600)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "rk_plan_test:" in run.stdout and " 0 failures" in run.stdout, run.stdout + run.stderr
    return run.stdout


def test_rk_plan_on_mock_device(tmp_path):
    cc = _gcc()
    sources = [os.path.join(HOST, f) for f in ("rocket.c", "tensor.c", "plan.c", "linear.c", "ksplit.c", "graph.c",
                                               "rkplan.c")]
    sources += [os.path.join(ROOT, "tests", "c", f) for f in ("mock_device.c", "rk_plan_test.c")]
    sources += [os.path.join(ROOT, "oracle", f) for f in ("linear_oracle.c", "graph_oracle.c", "rkplan_oracle.c")]
    exe = str(tmp_path / "rk_plan_test")
    build = subprocess.run([cc, "-std=gnu11", "-O1", "-Wall", "-Werror=implicit-function-declaration", "-DRK_TEST_MOCK",
                            *INC, *sources, "-lpthread", "-lm", "-o", exe], capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    env = dict(os.environ, B2_MOCK_DEVICES="1")
    env.pop("B2_DEVICE", None)
    _run(exe, env)


def test_rk_plan_without_device_is_refused(tmp_path):
    """No device behind the seam: verification still works, workspaces are refused."""
    cc = _gcc()
    sources = [os.path.join(HOST, f) for f in ("rocket.c", "tensor.c", "plan.c", "linear.c", "ksplit.c", "graph.c",
                                               "rkplan.c")]
    sources += [os.path.join(ROOT, "tests", "c", f) for f in ("mock_device.c", "rk_plan_test.c")]
    sources += [os.path.join(ROOT, "oracle", f) for f in ("linear_oracle.c", "graph_oracle.c", "rkplan_oracle.c")]
    exe = str(tmp_path / "rk_plan_test")
    build = subprocess.run([cc, "-std=gnu11", "-O1", "-DRK_TEST_MOCK", *INC, *sources, "-lpthread", "-lm", "-o", exe],
                           capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    run = subprocess.run([exe], capture_output=True, text=True, env=dict(os.environ, B2_MOCK_DEVICES="0"), timeout=120)
    assert run.returncode == 77 and " 0 failures" in run.stdout, run.stdout + run.stderr


@pytest.mark.gpu
def test_rk_plan_on_gpu(b2, tmp_path):
    cc = _gcc()
    libdir = os.path.dirname(b2.LIB_PATH)
    exe = str(tmp_path / "rk_plan_test")
    build = subprocess.run([cc, "-std=gnu11", "-O1", "-Wall", *INC, os.path.join(ROOT, "tests", "c", "rk_plan_test.c"),
                            "-L", libdir, "-lcustom_ops_b200", f"-Wl,-rpath,{libdir}", "-lm", "-o", exe],
                           capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    print(_run(exe, dict(os.environ)))
