"""Plans written by the reference's own planner, run through this library's plan/workspace ABI.

tests/golden/rk_plans.json holds the C descriptors that the reference tooling's compile pipeline and
ffi builder produce for six modules in both submit modes (tests/golden/make_rk_plan_golden.py):
a 300^3 matmul (two K tiles, 2x2 output tiles), Linear + HardSigmoid 64x512x256, the two-GEMM
projection with SiLU and residual, the SwiGLU FFN, a SiLU activation and a two-output branch.
Each test rebuilds the structs from that JSON (ctypes mirrors of include/rk_plan.h) and
  * checks the struct sizes the reference's ctypes recorded against this header's (C sizeof);
  * on the CPU seam (host sources + tests/c/mock_device.c as a shared library): every plan is
    accepted by rk_plan_create and its run matches the reference tooling's own numpy models of
    these modules (research/tilelang-rknpu/tests/test_dataflow_multitile.py:26-50: 256-wide FP16
    K chains, SiLU as fp16(z * fp16(sigmoid z)), FP16 residual) within the 8e-3 those tests use;
  * on a B200: the same runs give the same bytes as the CPU seam.
"""
import ctypes
import importlib
import json
import os
import shutil
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST = os.path.join(ROOT, "rockchip-npu-notes_b200", "csrc", "host")
INC = ["-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "rockchip-npu-notes_b200", "csrc"), "-I", HOST]
PLANS = json.load(open(os.path.join(ROOT, "tests", "golden", "rk_plans.json")))

rk = importlib.import_module("rockchip-npu-notes_b200.rkplan")


def f16(x):
    return np.asarray(x, dtype=np.float16)


def kchain(x, w_nk):
    """256-wide K tiles, each tile sum added to the FP16 running result and rounded to FP16."""
    a, b = x.astype(np.float64), w_nk.T.astype(np.float64)
    acc = f16(a[:, :256] @ b[:256, :])
    for k0 in range(256, a.shape[1], 256):
        acc = f16(acc.astype(np.float64) + a[:, k0:k0 + 256] @ b[k0:k0 + 256, :])
    return acc


def silu16(z):
    sig = f16(1.0 / (1.0 + np.exp(-z.astype(np.float32))))
    return f16(z.astype(np.float32) * sig.astype(np.float32))


def case_data(name, entry):
    """Seeded inputs and constants of a case, and the expected outputs by binding name."""
    rng = np.random.default_rng(7)
    shapes = {b["name"]: tuple(b["shape"]) for b in entry["bindings"]}
    data = {}
    for b in entry["bindings"]:
        if b["role"] == "output":
            continue
        if b["name"].startswith("__identity_"):
            data[b["name"]] = f16(np.eye(b["shape"][0]))
        elif b["role"] == "constant":
            data[b["name"]] = f16(rng.normal(0, 0.1, b["shape"]))
        else:
            data[b["name"]] = f16(rng.normal(0, 2.0 if name.startswith("activation") else 0.2, b["shape"]))
    base = name.split("/")[0]
    if base == "matmul_300":
        want = {"Y": kchain(data["A"], data["B"].T)}
    elif base.startswith("linear_hardsigmoid"):
        z = kchain(data["A"], data["B"]).astype(np.float64)
        want = {"A1": f16(np.clip(z / 6.0 + 0.5, 0.0, 1.0))}
    elif base == "projection_300":
        p = kchain(silu16(kchain(data["X"], data["W1"])), data["W2"])
        want = {"Y": f16(p.astype(np.float32) + data["X"].astype(np.float32))}
    elif base == "swiglu_300":
        x = data["X"]
        act = f16(silu16(kchain(x, data["Wg"])).astype(np.float32) * kchain(x, data["Wu"]).astype(np.float32))
        want = {"Y": f16(kchain(act, data["Wd"]).astype(np.float32) + x.astype(np.float32))}
    elif base.startswith("activation_silu"):
        want = {"Y": silu16(data["X"])}
    else:
        want = {"Y1": kchain(data["X"], data["W1"]), "Y2": kchain(data["X"], data["W2"])}
    for k, v in want.items():
        assert v.shape == shapes[k]
    return data, want


def run_case(L, fd, name, entry):
    """rk_plan_create + workspace + one run on library L; returns (outputs, expected) by binding name."""
    data, want = case_data(name, entry)
    ids = {b["name"]: b["id"] for b in entry["bindings"]}
    roles = {b["name"]: b["role"] for b in entry["bindings"]}
    outs = {b["name"]: np.zeros(b["shape"], np.float16) for b in entry["bindings"] if b["role"] == "output"}
    plan = rk.Plan(L, entry)
    ws = None
    try:
        ws = rk.Workspace(L, fd, plan, {ids[n]: a for n, a in data.items() if roles[n] == "constant"})
        prepared = ws.prepare({ids[n]: a for n, a in data.items() if roles[n] == "input"},
                              {ids[n]: a for n, a in outs.items()})
        report = ws.run(prepared)
        assert report.download_calls == len(entry["publish"])
        assert report.task_count == sum(len(s["task_ids"]) for s in entry["submits"])
    finally:
        if ws is not None:
            ws.destroy()
        plan.destroy()
    return outs, want


def mock_library(tmp_path):
    """The library's host sources over the CPU seam, as a shared library (symbols bound locally)."""
    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("gcc not available")
    sources = [os.path.join(HOST, f) for f in ("rocket.c", "tensor.c", "plan.c", "linear.c", "ksplit.c", "graph.c",
                                               "rkplan.c")]
    sources += [os.path.join(ROOT, "tests", "c", "mock_device.c")]
    sources += [os.path.join(ROOT, "oracle", f) for f in ("linear_oracle.c", "graph_oracle.c", "rkplan_oracle.c")]
    so = str(tmp_path / "librk_mock.so")
    build = subprocess.run([cc, "-std=gnu11", "-O2", "-fPIC", "-shared", "-Wl,-Bsymbolic", *INC, *sources,
                            "-lpthread", "-lm", "-o", so], capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    os.environ.setdefault("B2_MOCK_DEVICES", "1")
    return rk.declare(ctypes.CDLL(so))


def test_struct_sizes_match_the_reference_ctypes(tmp_path):
    """Every struct_size the reference's ctypes wrote equals sizeof of this header's struct."""
    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("gcc not available")
    src = tmp_path / "sizes.c"
    names = ["rk_plan_desc", "rk_value_desc", "rk_buffer_desc", "rk_view_desc", "rk_tensor_desc", "rk_action_desc",
             "rk_submit_desc", "rk_publish_desc"]
    src.write_text('#include <stdio.h>\n#include "rk_plan.h"\nint main(void){' +
                   "".join(f'printf("%zu\\n", sizeof({n}));' for n in names) + "return 0;}\n")
    exe = tmp_path / "sizes"
    subprocess.run([cc, "-std=gnu11", *INC, str(src), "-o", str(exe)], check=True)
    sizes = dict(zip(names, map(int, subprocess.run([str(exe)], capture_output=True, text=True).stdout.split())))
    e = PLANS["swiglu_300/chain"]
    got = {"rk_plan_desc": e["struct_size"], "rk_value_desc": e["values"][0]["struct_size"],
           "rk_buffer_desc": e["buffers"][0]["struct_size"], "rk_view_desc": e["views"][0]["struct_size"],
           "rk_tensor_desc": e["views"][0]["tensor"]["struct_size"], "rk_action_desc": e["actions"][0]["struct_size"],
           "rk_submit_desc": e["submits"][0]["struct_size"], "rk_publish_desc": e["publish"][0]["struct_size"]}
    assert got == sizes
    assert {n: ctypes.sizeof(rk.MIRRORS[n]) for n in names} == sizes


@pytest.mark.parametrize("name", sorted(PLANS))
def test_reference_plans_on_cpu_seam(tmp_path, name):
    L = mock_library(tmp_path)
    fd = L.rocket_open()
    assert fd >= 0
    try:
        outs, want = run_case(L, fd, name, PLANS[name])
    finally:
        L.rocket_close(fd)
    for k, v in want.items():
        np.testing.assert_allclose(outs[k].astype(np.float64), v.astype(np.float64), atol=8e-3, rtol=8e-3)


@pytest.mark.gpu
def test_reference_plans_on_gpu_match_cpu_seam(b2, tmp_path):
    M = mock_library(tmp_path)
    G = rk.declare(ctypes.CDLL(b2.LIB_PATH))
    mfd, gfd = M.rocket_open(), G.rocket_open()
    assert mfd >= 0 and gfd >= 0
    try:
        for name in sorted(PLANS):
            cpu, want = run_case(M, mfd, name, PLANS[name])
            gpu, _ = run_case(G, gfd, name, PLANS[name])
            for k in cpu:
                assert np.array_equal(cpu[k].view(np.uint16), gpu[k].view(np.uint16)), (name, k)
                np.testing.assert_allclose(gpu[k].astype(np.float64), want[k].astype(np.float64), atol=8e-3,
                                           rtol=8e-3)
    finally:
        M.rocket_close(mfd)
        G.rocket_close(gfd)
