"""ctypes front-end of the B200 FP16 Linear / HardSigmoid library.

Python tooling reaches the operator only through ctypes, as the reference's own Python tooling
reaches its C operators (research/multidevice-scheduling/backends/rk3588.py:76-81 and its ctypes
bridge, research/custom-ops in the reference project).  This module mirrors the C API of
``include/custom_ops.h`` (types, ``co_*`` entries, ``ROCKET_E_*`` codes) and ``include/b2_linear.h``
(devices, streams, extended shapes, device-pointer entries), plus numpy conveniences.

The library is ``lib/libcustom_ops_b200.so`` next to this file, built by ``make`` in this
directory (``build()``).  There is no CPU fallback: without the library, or without a CUDA
device, the calls fail with an exception.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libcustom_ops_b200.so")
CLI_PATH = os.path.join(HERE, "lib", "linear_hardsigmoid")

# rocket_status (include/rocket_b200.h)
OK, E_SHAPE, E_TILING, E_NOMEM, E_DEVICE, E_UNSUPPORTED = 0, -1, -2, -3, -4, -5
STATUS_NAMES = {0: "OK", -1: "ROCKET_E_SHAPE", -2: "ROCKET_E_TILING", -3: "ROCKET_E_NOMEM",
                -4: "ROCKET_E_DEVICE", -5: "ROCKET_E_UNSUPPORTED"}
# enums (include/custom_ops.h, include/b2_linear.h)
CO_F16, CO_F32 = 0, 1
CO_CUBE, CO_WEIGHT, CO_LINEAR = 0, 1, 2
CO_SEPARATE, CO_CHAIN = 0, 1
CO_LINEAR_NONE, CO_LINEAR_HSIG = 0, 1
ACC_TILE16, ACC_FP32 = 0, 1
STATUS_TIMEOUT, STATUS_NONFINITE_OUTPUT, STATUS_NONFINITE_INPUT, STATUS_GUARD = 1, 2, 4, 8
FAULT_NONE, FAULT_ALLOC, FAULT_LAUNCH, FAULT_NAN_OUTPUT = 0, 1, 2, 3
CO_MAX_K = CO_MAX_M = CO_MAX_N = 4096
CO_K_TILE = 256
CO_SLACK, CO_GUARD = 32768, 64
B2_MAX_DIM = 1 << 20


class RocketError(RuntimeError):
    """A library call returned a negative rocket_status."""

    def __init__(self, op, code):
        super().__init__(f"{op} failed: {STATUS_NAMES.get(code, code)} ({code})")
        self.op = op
        self.code = code


class CoTensor(ctypes.Structure):
    _fields_ = [("type", ctypes.c_int), ("layout", ctypes.c_int), ("rows", ctypes.c_uint),
                ("cols", ctypes.c_uint), ("physical_rows", ctypes.c_uint),
                ("physical_cols", ctypes.c_uint), ("atom", ctypes.c_uint), ("bytes", ctypes.c_size_t)]


class RocketBo(ctypes.Structure):
    _fields_ = [("handle", ctypes.c_uint32), ("size", ctypes.c_size_t), ("ptr", ctypes.c_void_p),
                ("dma_address", ctypes.c_uint64)]


class CoBuffer(ctypes.Structure):
    _fields_ = [("bo", RocketBo), ("fd", ctypes.c_int), ("payload", ctypes.c_size_t)]


class CoView(ctypes.Structure):
    _fields_ = [("buffer", ctypes.POINTER(CoBuffer)), ("offset", ctypes.c_size_t), ("tensor", CoTensor)]


class CoLinearPlan(ctypes.Structure):
    _fields_ = [("m", ctypes.c_uint), ("k", ctypes.c_uint), ("n", ctypes.c_uint),
                ("mtiles", ctypes.c_uint), ("ktiles", ctypes.c_uint), ("ntiles", ctypes.c_uint),
                ("output_tiles", ctypes.c_uint), ("has_bias", ctypes.c_uint), ("post", ctypes.c_uint),
                ("row_classes", ctypes.c_uint), ("device_bytes", ctypes.c_size_t),
                ("tasks", ctypes.c_ulonglong), ("chain_submits", ctypes.c_ulonglong)]


class CoLinearTileInfo(ctypes.Structure):
    _fields_ = [("m0", ctypes.c_uint), ("n0", ctypes.c_uint), ("rows", ctypes.c_uint),
                ("cols", ctypes.c_uint), ("ktiles", ctypes.c_uint), ("programs", ctypes.c_uint)]


class B2LinearInfo(ctypes.Structure):
    _fields_ = [("m", ctypes.c_uint), ("k", ctypes.c_uint), ("n", ctypes.c_uint),
                ("kernel", ctypes.c_uint), ("tile_m", ctypes.c_uint), ("tile_n", ctypes.c_uint),
                ("tile_k", ctypes.c_uint), ("stages", ctypes.c_uint), ("grid", ctypes.c_uint),
                ("launches_per_run", ctypes.c_uint), ("acc", ctypes.c_int),
                ("device_bytes", ctypes.c_size_t)]


# include/co_graph.h
CO_GRAPH_MAX_NODES = 64
(CO_GRAPH_INPUT, CO_GRAPH_LINEAR, CO_GRAPH_ADD, CO_GRAPH_MUL, CO_GRAPH_SILU, CO_GRAPH_GELU, CO_GRAPH_HSIG,
 CO_GRAPH_RMSNORM, CO_GRAPH_SOFTMAX, CO_GRAPH_ROPE, CO_GRAPH_ATTENTION) = range(11)
CO_GRAPH_ALLOW_NEG_INF = 1
CO_ROPE_INTERLEAVED, CO_ROPE_SPLIT_HALF = 0, 1


class CoGraphNode(ctypes.Structure):
    _fields_ = [("op", ctypes.c_int), ("a", ctypes.c_uint), ("b", ctypes.c_uint), ("rows", ctypes.c_uint),
                ("cols", ctypes.c_uint), ("c", ctypes.c_uint), ("mask_node", ctypes.c_uint),
                ("has_mask", ctypes.c_uint), ("weights", ctypes.c_void_p), ("bias", ctypes.c_void_p),
                ("gamma", ctypes.c_void_p), ("epsilon", ctypes.c_float), ("flags", ctypes.c_uint),
                ("heads", ctypes.c_uint), ("kv_heads", ctypes.c_uint), ("head_dim", ctypes.c_uint),
                ("rotary_dim", ctypes.c_uint), ("theta", ctypes.c_float), ("scale", ctypes.c_float),
                ("rope_style", ctypes.c_int), ("position_base", ctypes.c_uint32), ("causal", ctypes.c_int),
                ("window", ctypes.c_uint)]


class CoGraphDesc(ctypes.Structure):
    _fields_ = [("nodes", ctypes.POINTER(CoGraphNode)), ("count", ctypes.c_uint), ("output", ctypes.c_uint),
                ("device_budget", ctypes.c_size_t)]


class CoGraphTensorPlan(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_uint), ("cols", ctypes.c_uint), ("tiles", ctypes.c_uint),
                ("slot", ctypes.c_uint), ("first", ctypes.c_uint), ("last", ctypes.c_uint),
                ("bytes", ctypes.c_size_t)]


class CoGraphPlan(ctypes.Structure):
    _fields_ = [("steps", ctypes.c_uint), ("inputs", ctypes.c_uint), ("slots", ctypes.c_uint),
                ("order", ctypes.c_uint * 64), ("noutputs", ctypes.c_uint), ("outputs", ctypes.c_uint * 64),
                ("tensors", CoGraphTensorPlan * 64), ("slot_bytes", ctypes.c_size_t * 64)] + \
               [(f, ctypes.c_size_t) for f in ("tensor_bytes", "linear_bytes", "rowop_bytes", "rope_bytes",
                                               "attention_bytes", "workspace_bytes", "device_bytes")] + \
               [("hybrid_nodes", ctypes.c_uint)] + \
               [(f, ctypes.c_ulonglong) for f in ("host_upload_calls", "statistic_download_calls",
                                                  "activation_download_calls")] + \
               [(f, ctypes.c_size_t) for f in ("host_activation_reads", "statistic_downloads",
                                               "activation_downloads", "host_uploads")] + \
               [("identity_mask", ctypes.c_uint), ("gate_bytes", ctypes.c_size_t),
                ("tasks", ctypes.c_ulonglong), ("chain_submits", ctypes.c_ulonglong)]


class CoGraphInput(ctypes.Structure):
    _fields_ = [("node", ctypes.c_uint), ("data", ctypes.c_void_p)]


class CoGraphOutput(ctypes.Structure):
    _fields_ = [("node", ctypes.c_uint), ("data", ctypes.c_void_p)]


class B2GraphInfo(ctypes.Structure):
    _fields_ = [("gated", ctypes.c_uint), ("residual", ctypes.c_uint), ("kernels", ctypes.c_uint),
                ("captured", ctypes.c_uint)]


_P = ctypes.c_void_p
_U = ctypes.c_uint
_I = ctypes.c_int
_Z = ctypes.c_size_t
_T = ctypes.POINTER(CoTensor)
_V = ctypes.POINTER(CoView)
_B = ctypes.POINTER(CoBuffer)
_PLAN = ctypes.POINTER(CoLinearPlan)

# name -> (restype, argtypes)
SIGNATURES = {
    # rocket_b200.h
    "rocket_open": (_I, []),
    "rocket_close": (None, [_I]),
    "rocket_batched_submit_supported": (_I, []),
    "rocket_bo_alloc32": (_I, [_I, _Z, ctypes.POINTER(RocketBo)]),
    "rocket_bo_free": (None, [_I, ctypes.POINTER(RocketBo)]),
    "rocket_submit_counters_reset": (None, []),
    "rocket_submit_ioctl_count": (ctypes.c_uint64, []),
    "rocket_submit_task_count": (ctypes.c_uint64, []),
    "rocket_launch_count": (ctypes.c_uint64, []),
    # custom_ops.h
    "co_tensor_matrix": (_I, [_T, _U, _U, _I]),
    "co_tensor_input": (_I, [_T, _U, _U]),
    "co_tensor_weight": (_I, [_T, _U, _U]),
    "co_k_tiles": (_U, [_U]),
    "co_k_tile_length": (_U, [_U, _U]),
    "co_k_tile_offset": (_Z, [_T, _U]),
    "co_tensor_input_slice": (_I, [_T, _T, _U, _U, ctypes.POINTER(_Z)]),
    "co_tensor_spatial": (_I, [_T, _U, _U, _U]),
    "co_tensor_linear": (_I, [_T, _U]),
    "co_index": (_Z, [_T, _U, _U]),
    "co_buffer_alloc": (_I, [_I, _Z, _B]),
    "co_buffer_free": (None, [_B]),
    "co_view_init": (_I, [_V, _B, _Z, _T]),
    "co_upload_f16": (_I, [_V, _P]),
    "co_download": (_I, [_V, _P]),
    "co_sentinel": (_I, [_B]),
    "co_guard_check": (_I, [_B]),
    "co_copy": (_I, [_V, _V]),
    "co_bias_upload": (_I, [_V, _P]),
    "co_identity_upload": (_I, [_V]),
    "co_ones_upload": (_I, [_V, _U, _I]),
    "co_linear_plan_init": (_I, [_PLAN, _U, _U, _U, _Z]),
    "co_linear_plan_tile": (_I, [_PLAN, _U, ctypes.POINTER(CoLinearTileInfo)]),
    "co_linear_plan_init_ex": (_I, [_PLAN, _U, _U, _U, _I, _I, _Z]),
    "co_linear_create": (_I, [_I, _U, _U, _U, _P, _P, _I, _I, ctypes.POINTER(_P)]),
    "co_linear_run": (_I, [_P, _P, _P]),
    "co_linear_run_tiled": (_I, [_P, _V, _U, _V, _U]),
    "co_linear_update_weights": (_I, [_P, _P, _P]),
    "co_linear_destroy": (None, [_P]),
    "co_linear_hsig_create": (_I, [_I, _U, _U, _U, _P, _P, _I, ctypes.POINTER(_P)]),
    "co_linear_hsig_run": (_I, [_P, _P, _P]),
    "co_linear_hsig_run_cube": (_I, [_P, CoView, CoView]),
    "co_linear_hsig_run_tiles": (_I, [_P, _V, _U, _V, _U]),
    "co_linear_hsig_destroy": (None, [_P]),
    # b2_linear.h
    "b2_device_count": (_I, []),
    "b2_open_device": (_I, [_I]),
    "b2_set_stream": (_I, [_I, _P]),
    "b2_get_stream": (_P, [_I]),
    "b2_sync": (_I, [_I]),
    "b2_status": (_U, [_I, _I]),
    "b2_sm_count": (_I, [_I]),
    "b2_host_alloc": (_P, [_Z]),
    "b2_host_free": (None, [_P]),
    "b2_linear_create": (_I, [_I, _U, _U, _U, _P, _P, _I, _I, _I, ctypes.POINTER(_P)]),
    "b2_linear_set_accumulate": (_I, [_P, _I]),
    "b2_linear_run_device": (_I, [_P, _U, _P, _Z, _P, _Z]),
    "b2_linear_run_device_noalloc": (_I, [_P, _U, _P, _Z, _P, _Z]),
    "b2_linear_partial_device": (_I, [_P, _U, _P, _Z, _P, _Z]),
    "b2_linear_epilogue_device": (_I, [_P, _U, _P, _Z, _P, _Z]),
    "b2_linear_get_info": (_I, [_P, ctypes.POINTER(B2LinearInfo)]),
    "b2_fault_inject": (None, [_I, _U]),
    "b2_shard_range": (_I, [ctypes.c_ulonglong, _U, _U, _U, ctypes.POINTER(ctypes.c_ulonglong),
                            ctypes.POINTER(ctypes.c_ulonglong)]),
    "b2_linear_group_run_device": (_I, [ctypes.POINTER(_P), _U, _U, ctypes.POINTER(_P), ctypes.POINTER(_Z),
                                        ctypes.POINTER(_P), ctypes.POINTER(_Z)]),
    "b2_ksplit_create": (_I, [_P, _U, _U, _U, ctypes.POINTER(_P)]),
    "b2_ksplit_export": (_I, [_P, ctypes.c_char_p]),
    "b2_ksplit_connect": (_I, [_P, ctypes.c_char_p]),
    "b2_ksplit_rows": (_I, [_P, _U, ctypes.POINTER(_U), ctypes.POINTER(_U)]),
    "b2_ksplit_run": (_I, [_P, _U, _P, _Z, _P, _Z]),
    "b2_ksplit_set_timing": (_I, [_P, _I]),
    "b2_ksplit_phase_ms": (_I, [_P, ctypes.POINTER(ctypes.c_float)]),
    "b2_ksplit_destroy": (None, [_P]),
    # co_graph.h
    "co_graph_plan_init": (_I, [ctypes.POINTER(CoGraphDesc), ctypes.POINTER(CoGraphPlan)]),
    "co_graph_plan_many": (_I, [ctypes.POINTER(CoGraphDesc), ctypes.POINTER(_U), _U, ctypes.POINTER(CoGraphPlan)]),
    "co_graph_compile": (_I, [_I, ctypes.POINTER(CoGraphDesc), _I, ctypes.POINTER(_P)]),
    "co_graph_compile_many": (_I, [_I, ctypes.POINTER(CoGraphDesc), ctypes.POINTER(_U), _U, _I, ctypes.POINTER(_P)]),
    "co_graph_destroy": (None, [_P]),
    "co_graph_run": (_I, [_P, ctypes.POINTER(CoGraphInput), _U, _P]),
    "co_graph_run_many": (_I, [_P, ctypes.POINTER(CoGraphInput), _U, ctypes.POINTER(CoGraphOutput), _U]),
    "b2_graph_tensor": (_I, [_P, _U, ctypes.POINTER(_P), ctypes.POINTER(_Z)]),
    "b2_graph_launch": (_I, [_P]),
    "b2_graph_status": (_I, [_P]),
    "b2_graph_get_info": (_I, [_P, ctypes.POINTER(B2GraphInfo)]),
    # rk_plan.h (descriptor and report structs as opaque pointers; tests/c/rk_plan_test.c drives them)
    "rk_abi_version": (_U, []),
    "rk_target_check": (_I, [_P]),
    "rk_target_validate_text": (_I, [ctypes.c_char_p, _Z, ctypes.c_char_p, _P]),
    "rk_plan_create": (_I, [_P, ctypes.POINTER(_P), _P]),
    "rk_plan_destroy": (None, [_P]),
    "rk_workspace_create": (_I, [_I, _P, _P, _U, ctypes.POINTER(_P), _P]),
    "rk_workspace_create_shared": (_I, [_I, _P, _P, _U, _P, _U, ctypes.POINTER(_P), _P]),
    "rk_workspace_run": (_I, [_P, _P, _U, _P, _U, _P, _P]),
    "rk_workspace_run_group": (_I, [_P, _P, _U, _P, _P]),
    "rk_workspace_run_ex": (_I, [_P, _P, _U, _P, _U, _P, _P]),
    "rk_workspace_destroy": (_I, [_P, _P]),
    "rk_workspace_set_persistent_upload": (_I, [_P, _U, _P]),
    "rk_workspace_update_upload_region": (_I, [_P, _U, _P, _U, _U, _U, _U, _U, _U, _P]),
    "rk_workspace_clear_upload_destination": (_I, [_P, _U, _P]),
    "rk_workspace_get_cache_info": (_I, [_P, _P, _P]),
    "rk_workspace_task_cbuf": (_I, [_P, _U, _P, _U, _P, _P]),
    "rk_shared_constant_get_or_create": (_I, [_I, _P, _U, _P, ctypes.c_char_p, ctypes.POINTER(_P), _P, _P]),
    "rk_shared_constant_retain": (None, [_P]),
    "rk_shared_constant_release": (None, [_P]),
    "rk_shared_constant_bytes": (ctypes.c_uint64, [_P]),
    "rk_shared_constant_live": (_U, []),
}
KSPLIT_BLOB_BYTES = 96

_lib = None


def build(jobs=8):
    """Compile the library and the CLI in place (``make`` in this directory)."""
    subprocess.run(["make", "-s", f"-j{jobs}", "-C", HERE], check=True)


def lib():
    """Load the C-ABI library (raises if it has not been built: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run build() / make -C {HERE}")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(op, rc):
    if rc != 0:
        raise RocketError(op, rc)
    return rc


def _f16(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.float16)
    if a.dtype != np.float16:
        a = a.astype(np.float16)
    return a


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# --------------------------------------------------------------------------------- devices
def device_count():
    return lib().b2_device_count()


def open_device(ordinal=0):
    fd = lib().b2_open_device(int(ordinal))
    if fd < 0:
        raise RocketError("b2_open_device", fd)
    return fd


def close(fd):
    lib().rocket_close(int(fd))


def sync(fd):
    check("b2_sync", lib().b2_sync(fd))


def status(fd, clear=True):
    return lib().b2_status(fd, 1 if clear else 0)


def set_stream(fd, stream):
    """``stream``: an integer cudaStream_t handle (e.g. ``torch.cuda.Stream().cuda_stream``)."""
    check("b2_set_stream", lib().b2_set_stream(fd, ctypes.c_void_p(stream) if stream else None))


def sm_count(fd):
    return lib().b2_sm_count(fd)


def fault_inject(kind, nth):
    lib().b2_fault_inject(int(kind), int(nth))


def shard_range(total, parts, index, align=256):
    """[begin, end) of shard `index` of `parts` (b2_shard_range)."""
    b, e = ctypes.c_ulonglong(), ctypes.c_ulonglong()
    check("b2_shard_range", lib().b2_shard_range(total, parts, index, align, ctypes.byref(b), ctypes.byref(e)))
    return b.value, e.value


def group_run_device(ops, m, x_ptrs, ldx, y_ptrs, ldy):
    """b2_linear_group_run_device over Linear objects `ops` (device pointers, per-op pitches)."""
    n = len(ops)
    arr = lambda t, v: (t * n)(*v)
    check("b2_linear_group_run_device",
          lib().b2_linear_group_run_device(arr(_P, [o.h for o in ops]), n, m, arr(_P, x_ptrs), arr(_Z, ldx),
                                           arr(_P, y_ptrs), arr(_Z, ldy)))


def counters():
    L = lib()
    return {"submits": L.rocket_submit_ioctl_count(), "tasks": L.rocket_submit_task_count(),
            "launches": L.rocket_launch_count()}


def reset_counters():
    lib().rocket_submit_counters_reset()


# --------------------------------------------------------------------------------- plans
def plan(m, k, n, has_bias=True, post=CO_LINEAR_HSIG, budget=0):
    p = CoLinearPlan()
    check("co_linear_plan_init_ex", lib().co_linear_plan_init_ex(ctypes.byref(p), m, k, n, int(has_bias),
                                                                 int(post), budget))
    return p


def plan_tile(p, index):
    t = CoLinearTileInfo()
    check("co_linear_plan_tile", lib().co_linear_plan_tile(ctypes.byref(p), index, ctypes.byref(t)))
    return t


def tensor_matrix(rows, cols, dtype=CO_F16):
    t = CoTensor()
    check("co_tensor_matrix", lib().co_tensor_matrix(ctypes.byref(t), rows, cols, dtype))
    return t


def tensor_input(rows, cols):
    t = CoTensor()
    check("co_tensor_input", lib().co_tensor_input(ctypes.byref(t), rows, cols))
    return t


# --------------------------------------------------------------------------------- buffers / views
class Buffer:
    """A device buffer with the reference's slack and guard tail (co_buffer_alloc)."""

    def __init__(self, fd, payload):
        self.buf = CoBuffer()
        check("co_buffer_alloc", lib().co_buffer_alloc(fd, payload, ctypes.byref(self.buf)))

    def view(self, tensor, offset=0):
        v = CoView()
        check("co_view_init", lib().co_view_init(ctypes.byref(v), ctypes.byref(self.buf), offset,
                                                 ctypes.byref(tensor)))
        v._owner = self
        return v

    def guard_check(self):
        return lib().co_guard_check(ctypes.byref(self.buf))

    def sentinel(self):
        check("co_sentinel", lib().co_sentinel(ctypes.byref(self.buf)))

    @property
    def ptr(self):
        return self.buf.bo.ptr

    def free(self):
        if self.buf.bo.handle:
            lib().co_buffer_free(ctypes.byref(self.buf))

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def upload(view, rows_major):
    a = _f16(rows_major)
    check("co_upload_f16", lib().co_upload_f16(ctypes.byref(view), _ptr(a)))


def download(view):
    t = view.tensor
    out = np.empty((t.rows, t.cols), np.float16 if t.type == CO_F16 else np.float32)
    check("co_download", lib().co_download(ctypes.byref(view), _ptr(out)))
    return out


def views_array(views):
    arr = (CoView * len(views))()
    for i, v in enumerate(views):
        arr[i] = v
    return arr


# --------------------------------------------------------------------------------- operator
class Linear:
    """``Y = act(X @ W.T + b)`` on one device handle.

    ``compat=True`` creates through ``co_linear_create`` (reference limits, per-256-K FP16
    accumulation); otherwise ``b2_linear_create`` with ``acc`` (ACC_TILE16 or ACC_FP32).
    """

    def __init__(self, fd, m, k, n, w, bias=None, post=CO_LINEAR_HSIG, mode=CO_CHAIN, acc=ACC_TILE16,
                 compat=True):
        self.fd, self.m, self.k, self.n = fd, m, k, n
        w16 = _f16(w)
        b16 = None if bias is None else _f16(bias)
        h = ctypes.c_void_p()
        if compat:
            rc = lib().co_linear_create(fd, m, k, n, _ptr(w16), _ptr(b16), post, mode, ctypes.byref(h))
            check("co_linear_create", rc)
            if acc != ACC_TILE16:
                check("b2_linear_set_accumulate", lib().b2_linear_set_accumulate(h, acc))
        else:
            rc = lib().b2_linear_create(fd, m, k, n, _ptr(w16), _ptr(b16), post, mode, acc, ctypes.byref(h))
            check("b2_linear_create", rc)
        self.h = h

    def run(self, x, out=None):
        x16 = _f16(x)
        assert x16.size == self.m * self.k
        y = np.empty((self.m, self.n), np.float16) if out is None else out
        check("co_linear_run", lib().co_linear_run(self.h, _ptr(x16), _ptr(y)))
        return y

    def run_rc(self, x, y):
        """Raw return code of co_linear_run (y is left untouched on failure)."""
        return lib().co_linear_run(self.h, _ptr(_f16(x)), _ptr(y))

    def run_device(self, m, x_ptr, ldx, y_ptr, ldy):
        check("b2_linear_run_device", lib().b2_linear_run_device(self.h, m, x_ptr, ldx, y_ptr, ldy))

    def partial_device(self, m, x_ptr, ldx, p_ptr, ldp):
        check("b2_linear_partial_device", lib().b2_linear_partial_device(self.h, m, x_ptr, ldx, p_ptr, ldp))

    def epilogue_device(self, m, p_ptr, ldp, y_ptr, ldy):
        check("b2_linear_epilogue_device", lib().b2_linear_epilogue_device(self.h, m, p_ptr, ldp, y_ptr, ldy))

    def set_accumulate(self, acc):
        check("b2_linear_set_accumulate", lib().b2_linear_set_accumulate(self.h, acc))

    def update_weights(self, w, bias=None):
        w16 = _f16(w)
        b16 = None if bias is None else _f16(bias)
        return lib().co_linear_update_weights(self.h, _ptr(w16), _ptr(b16))

    def run_tiles(self, xviews, yviews):
        xa, ya = views_array(xviews), views_array(yviews)
        return lib().co_linear_hsig_run_tiles(self.h, xa, len(xviews), ya, len(yviews))

    def run_tiled(self, xviews, yviews):
        xa, ya = views_array(xviews), views_array(yviews)
        return lib().co_linear_run_tiled(self.h, xa, len(xviews), ya, len(yviews))

    def run_cube(self, xview, yview):
        return lib().co_linear_hsig_run_cube(self.h, xview, yview)

    def info(self):
        i = B2LinearInfo()
        check("b2_linear_get_info", lib().b2_linear_get_info(self.h, ctypes.byref(i)))
        return i

    def destroy(self):
        if self.h:
            lib().co_linear_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass
