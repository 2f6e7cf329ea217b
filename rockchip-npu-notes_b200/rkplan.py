"""ctypes mirror of the plan/workspace ABI (``include/rk_plan.h``).

The reference's TileLang tooling drives its plan runtime through ctypes
(research/tilelang-rknpu/python/rknpu_backend/runtime/ffi.py); this module is the same kind of
bridge onto this library: the descriptor, binding, report and diagnostic structs field for field
as the header declares them, ``plan_desc_from_fields`` to build a descriptor from plain field
values (the form ``tests/golden/rk_plans.json`` stores the reference planner's descriptors in), and
``Plan`` / ``Workspace`` wrappers that raise on a non-zero status with the library's diagnostic.
"""
import ctypes

import numpy as np

RK_ABI_VERSION = 1
u32, u64, i32 = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int32
_PU32 = ctypes.POINTER(u32)

RK_ROLE_INPUT, RK_ROLE_CONSTANT, RK_ROLE_OUTPUT = 0, 1, 2


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


MIRRORS = {"rk_plan_desc": PlanDesc, "rk_value_desc": Value, "rk_buffer_desc": Buffer, "rk_view_desc": View,
           "rk_tensor_desc": Tensor, "rk_action_desc": Action, "rk_submit_desc": Submit, "rk_publish_desc": Publish,
           "rk_binding": Binding, "rk_diag": Diag, "rk_run_report": RunReport}


class PlanError(RuntimeError):
    def __init__(self, what, rc, diag):
        super().__init__(f"{what}: {rc} [{diag.stage.decode()}] {diag.message.decode()} (action {diag.action_id})")
        self.rc, self.code, self.action_id = rc, diag.code, diag.action_id


def _fill(struct, row, skip=()):
    for name, _ in struct._fields_:
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


def plan_desc_from_fields(entry):
    """An rk_plan_desc from plain field values: the plan-level fields plus "values", "buffers",
    "views", "actions" (with "inputs"/"outputs"/"deps" id lists), "submits" (with "task_ids"/"deps")
    and "publish" lists. Returns (desc, keepalive); keep the second alive while desc is used."""
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


def declare(L):
    """argtypes/restype of the rk_* entries used here, on a loaded library."""
    P = ctypes.c_void_p
    for fn in ("rk_plan_create", "rk_workspace_create", "rk_workspace_run", "rk_workspace_destroy"):
        getattr(L, fn).restype = ctypes.c_int
    L.rk_plan_create.argtypes = [P, P, P]
    L.rk_plan_destroy.argtypes = [P]
    L.rk_plan_destroy.restype = None
    L.rk_workspace_destroy.argtypes = [P, P]
    L.rk_workspace_create.argtypes = [ctypes.c_int, P, P, u32, P, P]
    L.rk_workspace_run.argtypes = [P, P, u32, P, u32, P, P]
    L.rocket_open.restype = ctypes.c_int
    return L


def binding(value_id, array):
    """A rank-2 binding over a C-contiguous FP16 numpy array (keep the array alive)."""
    a = np.ascontiguousarray(array)
    assert a.dtype == np.float16 and a.ndim == 2
    b = Binding()
    b.abi_version, b.struct_size, b.id, b.dtype, b.rank = RK_ABI_VERSION, ctypes.sizeof(Binding), value_id, 0, 2
    b.shape[0], b.shape[1] = a.shape
    b.data, b.nbytes = a.ctypes.data, a.nbytes
    return b


class Plan:
    """A verified plan (rk_plan_create) built from plain descriptor fields."""

    def __init__(self, L, fields):
        self.L = L
        desc, keep = plan_desc_from_fields(fields)
        self.handle = ctypes.c_void_p()
        diag = Diag()
        rc = L.rk_plan_create(ctypes.byref(desc), ctypes.byref(self.handle), ctypes.byref(diag))
        if rc:
            raise PlanError("rk_plan_create", rc, diag)

    def destroy(self):
        if self.handle.value:
            self.L.rk_plan_destroy(self.handle)
            self.handle = ctypes.c_void_p()


class Workspace:
    """rk_workspace_create over `plan` on device handle fd, with {value id: FP16 array} constants."""

    def __init__(self, L, fd, plan, constants):
        self.L = L
        self._const = [np.ascontiguousarray(a) for a in constants.values()]
        arr = (Binding * max(len(constants), 1))(*[binding(i, a) for i, a in zip(constants, self._const)])
        self.handle = ctypes.c_void_p()
        diag = Diag()
        rc = L.rk_workspace_create(fd, plan.handle, arr, len(constants), ctypes.byref(self.handle), ctypes.byref(diag))
        if rc:
            raise PlanError("rk_workspace_create", rc, diag)

    def prepare(self, inputs, outputs):
        """Binding arrays for {value id: array} inputs and outputs, reusable across run() calls."""
        ins = (Binding * max(len(inputs), 1))(*[binding(i, a) for i, a in inputs.items()])
        outs = (Binding * max(len(outputs), 1))(*[binding(i, a) for i, a in outputs.items()])
        return ins, len(inputs), outs, len(outputs)

    def run(self, prepared, report=None):
        ins, nin, outs, nout = prepared
        diag = Diag()
        rep = report if report is not None else RunReport()
        rc = self.L.rk_workspace_run(self.handle, ins, nin, outs, nout, ctypes.byref(rep), ctypes.byref(diag))
        if rc:
            raise PlanError("rk_workspace_run", rc, diag)
        return rep

    def destroy(self):
        if self.handle.value:
            diag = Diag()
            rc = self.L.rk_workspace_destroy(self.handle, ctypes.byref(diag))
            if rc:
                raise PlanError("rk_workspace_destroy", rc, diag)
            self.handle = ctypes.c_void_p()
