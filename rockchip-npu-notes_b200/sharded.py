"""Multi-GPU layouts of the Linear path: one process per GPU, torch.distributed as plumbing.

The reference runs on one RK3588 and only chooses an NPU core per submit
(research/custom-ops/src/co_schedule.c); on an 8x B200 box a large Linear is split across GPUs:

* column-parallel over N (``ColumnShard``): rank r owns W[n0:n1, :], b[n0:n1] and Y[:, n0:n1],
  X is replicated; no collective touches the data path.
* K-split (``KSplitLinear``): rank r owns X[:, k0:k1] and W[:, k0:k1] and produces the raw FP32
  partial X_r W_r^T (b2_linear_partial_device); the partials are summed with an NCCL all-reduce
  or reduce-scatter over NVLink, then bias and activation (b2_linear_epilogue_device). This is for
  shapes whose N is too small to split.
* Fused K-split (``FusedKSplit``, b2_ksplit_*): the same split, but the GEMM epilogue stores each
  row block of the partial straight into its owner's memory over NVLink while later tiles are
  still multiplying, and the owner adds the world partials with bias and activation.

Shard boundaries come from b2_shard_range (256-aligned, so 256-wide K tiles and output tiles stay
whole).
"""
import importlib

import numpy as np

_b2 = importlib.import_module(__name__.rsplit(".", 1)[0])


def column_shard(n, world, rank):
    """[n0, n1) output columns of `rank`."""
    return _b2.shard_range(n, world, rank, 256)


def k_shard(k, world, rank):
    """[k0, k1) reduction columns of `rank`."""
    return _b2.shard_range(k, world, rank, 256)


class ColumnShard:
    """This rank's column block of a column-parallel Linear.

    ``w`` is the full FP16 [n, k] weight, or a callable ``w(n0, n1)`` returning rows [n0, n1) only
    (so a rank never materialises the other ranks' weights); ``bias`` likewise, or None."""

    def __init__(self, fd, m_host, n, k, w, bias, world, rank, post=_b2.CO_LINEAR_NONE,
                 acc=_b2.ACC_FP32):
        self.n0, self.n1 = column_shard(n, world, rank)
        self.k = k
        self.op = None
        if self.n1 > self.n0:
            rows = w(self.n0, self.n1) if callable(w) else w[self.n0:self.n1]
            b = None if bias is None else (bias(self.n0, self.n1) if callable(bias) else bias[self.n0:self.n1])
            self.op = _b2.Linear(fd, m_host, k, self.n1 - self.n0, np.ascontiguousarray(rows), b, post=post,
                                 mode=_b2.CO_CHAIN, acc=acc, compat=False)

    def run_device(self, m, x_ptr, ldx, y_ptr, ldy):
        """Y[:, n0:n1] of this rank (y_ptr points at this rank's own [m, ldy] block)."""
        if self.op is not None:
            self.op.run_device(m, x_ptr, ldx, y_ptr, ldy)

    def destroy(self):
        if self.op is not None:
            self.op.destroy()


class KSplitLinear:
    """This rank's K slice of a K-split Linear: partial -> NCCL reduction -> epilogue.

    ``torch`` and ``dist`` are passed in so this module does not import torch at load time; with
    world == 1 no collective is issued. The caller runs ``forward`` with torch's current stream set
    to the library handle's stream, so the NCCL call (ordered after the current stream's work, and
    the current stream after it) falls between the two launches.

    ``all_reduce``: every rank receives the summed [m, n] partial and writes the whole Y.
    ``reduce_scatter``: rank r receives the summed rows [r*mp/world, (r+1)*mp/world) of the partial
    (mp = m rounded up to a multiple of world; padding rows are reduced but never written to Y) and
    writes only its rows of Y --
    half the NVLink bytes of the all-reduce, output sharded by rows.
    """

    def __init__(self, fd, m_max, w_full, bias_full, world, rank, torch, dist, post=_b2.CO_LINEAR_NONE):
        n, k = w_full.shape
        self.k0, self.k1 = k_shard(k, world, rank)
        self.n, self.world, self.rank = n, world, rank
        self.torch, self.dist = torch, dist
        kk = max(self.k1 - self.k0, 1)
        w = w_full[:, self.k0:self.k1] if self.k1 > self.k0 else np.zeros((n, 1), np.float16)
        self.op = _b2.Linear(fd, 1, kk, n, np.ascontiguousarray(w), bias_full, post=post, mode=_b2.CO_SEPARATE,
                             acc=_b2.ACC_FP32, compat=False)
        self.ldp = -(-n // 4) * 4
        rows = -(-m_max // world) * world
        self.partial = torch.zeros((rows, self.ldp), dtype=torch.float32, device="cuda")
        self.shard = torch.zeros((rows // world, self.ldp), dtype=torch.float32, device="cuda")
        self.empty = self.k1 <= self.k0

    def _partial(self, m, x_ptr, ldx):
        p = self.partial[:m]
        if self.empty:
            p.zero_()
        else:
            self.op.partial_device(m, x_ptr, ldx, p.data_ptr(), self.ldp)
        return p

    def row_shard(self, m):
        """[r0, r1) rows of Y this rank writes under ``reduce_scatter``."""
        per = -(-m // self.world)
        return min(self.rank * per, m), min((self.rank + 1) * per, m)

    def forward(self, m, x_ptr, ldx, y_ptr, ldy, collective="all_reduce"):
        """x_ptr: this rank's X[:, k0:k1] block [m, ldx]; y_ptr: Y [m, ldy] (FP16, row-major).

        all_reduce writes all m rows of Y; reduce_scatter writes rows row_shard(m) only."""
        p = self._partial(m, x_ptr, ldx)
        if self.world == 1:
            self.op.epilogue_device(m, p.data_ptr(), self.ldp, y_ptr, ldy)
            return
        if collective == "all_reduce":
            self.dist.all_reduce(p, op=self.dist.ReduceOp.SUM)
            self.op.epilogue_device(m, p.data_ptr(), self.ldp, y_ptr, ldy)
            return
        if collective != "reduce_scatter":
            raise ValueError(f"unknown collective {collective!r}")
        per = -(-m // self.world)
        out = self.shard[:per]
        self.dist.reduce_scatter_tensor(out, self.partial[:per * self.world], op=self.dist.ReduceOp.SUM)
        r0, r1 = self.row_shard(m)
        if r1 > r0:
            self.op.epilogue_device(r1 - r0, out.data_ptr(), self.ldp, y_ptr + r0 * ldy * 2, ldy)

    def destroy(self):
        self.op.destroy()


class FusedKSplit:
    """This rank's part of a fused K-split Linear (b2_ksplit_*): owns X[:, k0:k1], W[:, k0:k1] and
    writes rows ``rows(m)`` of Y. ``dist`` may be None when world == 1. The library must run on
    torch's current stream when ``run`` is called (the caller sets it with b2.set_stream)."""

    def __init__(self, fd, m_max, w_full, bias_full, world, rank, torch, dist, post=_b2.CO_LINEAR_NONE):
        import ctypes
        n, k = w_full.shape
        self.k0, self.k1 = k_shard(k, world, rank)
        if self.k1 <= self.k0:
            raise ValueError("every rank needs a non-empty K slice")
        self.op = _b2.Linear(fd, 1, self.k1 - self.k0, n, np.ascontiguousarray(w_full[:, self.k0:self.k1]), bias_full,
                             post=post, mode=_b2.CO_SEPARATE, acc=_b2.ACC_FP32, compat=False)
        L = _b2.lib()
        h = ctypes.c_void_p()
        _b2.check("b2_ksplit_create", L.b2_ksplit_create(self.op.h, world, rank, m_max, ctypes.byref(h)))
        self.h, self.world, self.rank = h, world, rank
        if world > 1:
            blob = ctypes.create_string_buffer(_b2.KSPLIT_BLOB_BYTES)
            _b2.check("b2_ksplit_export", L.b2_ksplit_export(self.h, blob))
            dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
            mine = torch.frombuffer(bytearray(blob.raw), dtype=torch.uint8).to(dev)
            parts = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(parts, mine)
            blobs = b"".join(bytes(t.cpu().numpy()) for t in parts)
            _b2.check("b2_ksplit_connect", L.b2_ksplit_connect(self.h, blobs))

    def rows(self, m):
        import ctypes
        r0, nr = ctypes.c_uint(), ctypes.c_uint()
        _b2.check("b2_ksplit_rows", _b2.lib().b2_ksplit_rows(self.h, m, ctypes.byref(r0), ctypes.byref(nr)))
        return r0.value, r0.value + nr.value

    def run(self, m, x_ptr, ldx, y_ptr, ldy):
        """x_ptr: this rank's X[:, k0:k1] [m, ldx]; y_ptr: Y [m, ldy] (rows(m) written)."""
        _b2.check("b2_ksplit_run", _b2.lib().b2_ksplit_run(self.h, m, x_ptr, ldx, y_ptr, ldy))

    def set_timing(self, enable=True):
        """Record phase events in every round (b2_ksplit_set_timing)."""
        _b2.check("b2_ksplit_set_timing", _b2.lib().b2_ksplit_set_timing(self.h, 1 if enable else 0))

    def phase_ms(self):
        """Device ms of the last round's phases: (GEMM + NVLink stores, signal, wait + reduction)."""
        import ctypes
        ms = (ctypes.c_float * 3)()
        _b2.check("b2_ksplit_phase_ms", _b2.lib().b2_ksplit_phase_ms(self.h, ms))
        return tuple(float(v) for v in ms)

    def destroy(self):
        if self.h:
            _b2.lib().b2_ksplit_destroy(self.h)
            self.h = None
        self.op.destroy()
