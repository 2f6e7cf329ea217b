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

u32, u64, i32 = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int32
_PU32 = ctypes.POINTER(u32)


class Tensor(ctypes.Structure):
    _fields_ = [("abi_version", u32), ("struct_size", u32), ("dtype", u32), ("layout", u32), ("rows", u32),
                ("cols", u32), ("physical_rows", u32), ("physical_cols", u32), ("atom", u32), ("reserved", u32),
                ("bytes", u64)]


class Value(ctypes.Structure):
    _fields_ = [("abi_version", u32), ("struct_size", u32), ("id", u32), ("role", u32), ("dtype", u32), ("rank", u32),
                ("shape", u32 * 2), ("nbytes", u64), ("name", ctypes.c_char_p), ("name_len", u32),
                ("reserved", u32)]


class Buffer(ctypes.Structure):
    _fields_ = [(n, u32) for n in ("abi_version", "struct_size", "id", "role", "slot_id", "alignment", "layout_id",
                                   "padding_state", "lifetime_first", "lifetime_last")] + [("offset", u64),
                                                                                            ("capacity", u64)]


class View(ctypes.Structure):
    _fields_ = [("abi_version", u32), ("struct_size", u32), ("id", u32), ("buffer_id", u32), ("offset_bytes", u64),
                ("valid_region", u32 * 4), ("tensor", Tensor)]


class Action(ctypes.Structure):
    _fields_ = [(n, u32) for n in ("abi_version", "struct_size", "id", "kind", "template_id", "ninputs", "noutputs",
                                   "ndeps", "source_binding", "source_row_offset", "source_col_offset",
                                   "source_row_stride", "source_k0", "source_k_index", "source_k_count", "flags",
                                   "act_kind")] + [("inputs", _PU32), ("outputs", _PU32), ("deps", _PU32),
                                                   ("origin", ctypes.c_char * 64)]


class Submit(ctypes.Structure):
    _fields_ = [(n, u32) for n in ("abi_version", "struct_size", "id", "mode", "core_policy", "ntask_ids",
                                   "ndeps")] + [("task_ids", _PU32), ("deps", _PU32)]


class Publish(ctypes.Structure):
    _fields_ = [(n, u32) for n in ("abi_version", "struct_size", "binding_id", "view_id", "dst_row_offset",
                                   "dst_col_offset", "rows", "cols")]


class PlanDesc(ctypes.Structure):
    _fields_ = [("abi_version", u32), ("struct_size", u32), ("schema_version", u32), ("flags", u32),
                ("profile_hash", u64), ("source_hash", u64),
                ("values", ctypes.POINTER(Value)), ("nvalues", u32), ("reserved0", u32),
                ("buffers", ctypes.POINTER(Buffer)), ("nbuffers", u32), ("reserved1", u32),
                ("views", ctypes.POINTER(View)), ("nviews", u32), ("reserved2", u32),
                ("actions", ctypes.POINTER(Action)), ("nactions", u32), ("reserved3", u32),
                ("submits", ctypes.POINTER(Submit)), ("nsubmits", u32), ("reserved4", u32),
                ("publish", ctypes.POINTER(Publish)), ("npublish", u32), ("reserved5", u32),
                ("device_budget_bytes", u64), ("host_budget_bytes", u64), ("claimed_device_bytes", u64),
                ("claimed_host_bytes", u64), ("runtime_abi_version", u32), ("reserved6", u32)]


class Binding(ctypes.Structure):
    _fields_ = [("abi_version", u32), ("struct_size", u32), ("id", u32), ("dtype", u32), ("rank", u32),
                ("shape", u32 * 2), ("data", ctypes.c_void_p), ("nbytes", u64)]


class Diag(ctypes.Structure):
    _fields_ = [("abi_version", u32), ("struct_size", u32), ("code", i32), ("native_status", i32),
                ("action_id", u32), ("has_action", u32), ("stage", ctypes.c_char * 32),
                ("message", ctypes.c_char * 512), ("source", ctypes.c_char * 128), ("profile", ctypes.c_char * 64)]


class RunReport(ctypes.Structure):
    _fields_ = [(n, u32) for n in ("abi_version", "struct_size", "task_count", "submit_count", "fail_action_id",
                                   "numeric_mode")] + [(n, u64) for n in ("upload_calls", "upload_bytes",
                                                                          "download_calls", "download_bytes")] + \
               [(n, ctypes.c_double) for n in ("pack_us", "emit_us", "submit_wait_us", "output_sync_us")]


def _fill(struct, row, skip=()):
    for name, ctype in struct._fields_:
        if name in skip or name not in row:
            continue
        v = row[name]
        if isinstance(v, list):
            arr = getattr(struct, name)
            for i, x in enumerate(v):
                arr[i] = x
        elif isinstance(v, dict):
            _fill(getattr(struct, name), v)
        elif isinstance(v, str):
            setattr(struct, name, v.encode())
        else:
            setattr(struct, name, v)


def build_desc(entry):
    """The plan descriptor of one JSON entry; returns (desc, keepalive)."""
    keep = []

    def arr(ctype, rows, skip=(), extra=None):
        a = (ctype * max(len(rows), 1))()
        for i, row in enumerate(rows):
            _fill(a[i], row, skip)
            if extra:
                extra(a[i], row)
        keep.append(a)
        return a

    def ids(values):
        a = (u32 * max(len(values), 1))(*values)
        keep.append(a)
        return ctypes.cast(a, _PU32) if values else None

    def value_extra(v, row):
        name = ctypes.create_string_buffer(row["name"].encode())
        keep.append(name)
        v.name = ctypes.cast(name, ctypes.c_char_p)

    def action_extra(a, row):
        a.inputs, a.outputs, a.deps = ids(row["inputs"]), ids(row["outputs"]), ids(row["deps"])

    def submit_extra(s, row):
        s.task_ids, s.deps = ids(row["task_ids"]), ids(row["deps"])

    d = PlanDesc()
    _fill(d, entry, skip=("values", "buffers", "views", "actions", "submits", "publish"))
    d.values = arr(Value, entry["values"], skip=("name",), extra=value_extra)
    d.buffers = arr(Buffer, entry["buffers"])
    d.views = arr(View, entry["views"])
    d.actions = arr(Action, entry["actions"], skip=("inputs", "outputs", "deps"), extra=action_extra)
    d.submits = arr(Submit, entry["submits"], skip=("task_ids", "deps"), extra=submit_extra)
    d.publish = arr(Publish, entry["publish"])
    return d, keep


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
    rng = np.random.default_rng(abs(hash(name.split("/")[0])) % (2 ** 32) if False else 7)
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
    """rk_plan_create + workspace + one run on library L; returns the outputs by binding name."""
    desc, keep = build_desc(entry)
    diag = Diag()
    plan = ctypes.c_void_p()
    rc = L.rk_plan_create(ctypes.byref(desc), ctypes.byref(plan), ctypes.byref(diag))
    assert rc == 0, (name, rc, diag.message)
    data, want = case_data(name, entry)

    def binding(b, array):
        x = Binding()
        x.abi_version, x.struct_size, x.id, x.dtype = 1, ctypes.sizeof(Binding), b["id"], 0
        x.rank = 2
        x.shape[0], x.shape[1] = b["shape"]
        x.data, x.nbytes = array.ctypes.data, array.nbytes
        return x

    by_role = {r: [b for b in sorted(entry["bindings"], key=lambda b: b["id"]) if b["role"] == r]
               for r in ("input", "constant", "output")}
    outs = {b["name"]: np.zeros(b["shape"], np.float16) for b in by_role["output"]}
    consts = (Binding * max(len(by_role["constant"]), 1))(*[binding(b, data[b["name"]]) for b in by_role["constant"]])
    ins = (Binding * max(len(by_role["input"]), 1))(*[binding(b, data[b["name"]]) for b in by_role["input"]])
    outb = (Binding * len(by_role["output"]))(*[binding(b, outs[b["name"]]) for b in by_role["output"]])
    ws = ctypes.c_void_p()
    try:
        rc = L.rk_workspace_create(fd, plan, consts, len(by_role["constant"]), ctypes.byref(ws), ctypes.byref(diag))
        assert rc == 0, (name, rc, diag.message)
        report = RunReport()
        rc = L.rk_workspace_run(ws, ins, len(by_role["input"]), outb, len(by_role["output"]), ctypes.byref(report),
                                ctypes.byref(diag))
        assert rc == 0, (name, rc, diag.message)
        assert report.download_calls == len(entry["publish"])
        assert report.task_count == sum(len(s["task_ids"]) for s in entry["submits"])
    finally:
        if ws.value:
            assert L.rk_workspace_destroy(ws, ctypes.byref(diag)) == 0
        L.rk_plan_destroy(plan)
    return outs, want


def _declare(L):
    L.rocket_open.restype = ctypes.c_int
    for fn in ("rk_plan_create", "rk_workspace_create", "rk_workspace_run", "rk_workspace_destroy"):
        getattr(L, fn).restype = ctypes.c_int
    L.rk_plan_destroy.argtypes = [ctypes.c_void_p]
    L.rk_workspace_destroy.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    L.rk_workspace_create.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, u32, ctypes.c_void_p,
                                      ctypes.c_void_p]
    L.rk_workspace_run.argtypes = [ctypes.c_void_p, ctypes.c_void_p, u32, ctypes.c_void_p, u32, ctypes.c_void_p,
                                   ctypes.c_void_p]
    return L


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
    return _declare(ctypes.CDLL(so))


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
    mirrors = {"rk_plan_desc": PlanDesc, "rk_value_desc": Value, "rk_buffer_desc": Buffer, "rk_view_desc": View,
               "rk_tensor_desc": Tensor, "rk_action_desc": Action, "rk_submit_desc": Submit,
               "rk_publish_desc": Publish}
    assert {n: ctypes.sizeof(m) for n, m in mirrors.items()} == sizes


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
    G = _declare(ctypes.CDLL(b2.LIB_PATH))
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
