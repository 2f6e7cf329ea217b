"""Fused K-split (b2_ksplit_*): GEMM partials routed to their owner, round signal, owner reduction.

On one GPU (world = 1, the round signals itself):
  * the fused round equals b2_linear_partial_device + b2_linear_epilogue_device bit for bit (the
    same GEMM accumulator; a single partial needs no additions), with bias and HardSigmoid;
  * within tolerance of the FP64 oracle on sampled rows;
  * repeated rounds (alternating parity planes) and a CUDA-graph replay of a round give identical
    bits (the round counter lives on the device);
  * argument errors: m <= 8, m > m_max, a tile-16 operator, world > 8, a peer blob declaring a
    different layout.
On two GPUs (skipped with fewer): two spawned ranks, blobs exchanged over gloo, each rank's rows
of Y within tolerance of the FP64 oracle over the full K; and failure detection: one rank never
runs its round (a host-side failure), the other rank's round ends after its one-second wait limit
with B2_STATUS_TIMEOUT instead of hanging, and its context keeps working.
Tolerance: |y - ref| <= 2e-3 + 2e-3*|ref| element-wise.
"""
import ctypes
import os
import socket

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def case(m, n, k, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k)).astype(np.float16)
    w = (rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float16)
    b = rng.uniform(-0.1, 0.1, n).astype(np.float16)
    return x, w, b


def test_world1_round_equals_partial_plus_epilogue(b2, gpu_fd):
    sharded = __import__("importlib").import_module("rockchip-npu-notes_b200.sharded")
    m, n, k = 1000, 1000, 1536
    x, w, b = case(m, n, k, 3)
    fk = sharded.FusedKSplit(gpu_fd, m, w, b, 1, 0, torch, None, post=b2.CO_LINEAR_HSIG)
    assert fk.rows(m) == (0, m)
    xd = torch.from_numpy(x).cuda()
    y = torch.zeros(m, 1000, dtype=torch.float16, device="cuda")
    ref_y = torch.zeros_like(y)
    ldp = -(-n // 4) * 4
    part = torch.zeros(m, ldp, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    fk.run(m, xd.data_ptr(), k, y.data_ptr(), 1000)
    fk.op.partial_device(m, xd.data_ptr(), k, part.data_ptr(), ldp)
    fk.op.epilogue_device(m, part.data_ptr(), ldp, ref_y.data_ptr(), 1000)
    b2.sync(gpu_fd)
    assert b2.status(gpu_fd) == 0
    assert torch.equal(y.view(torch.int16), ref_y.view(torch.int16))
    rows = np.linspace(0, m - 1, 16).astype(int)
    ref = oracle.linear("fp64", x[rows], w, b, post=1, want=("act",))["act"]
    ok, worst = oracle.tolerance_ok(y.cpu().numpy()[rows], ref)
    assert ok, worst
    # more rounds (parity planes alternate) and a captured round: same bits
    for _ in range(3):
        y2 = torch.zeros_like(y)
        fk.run(m, xd.data_ptr(), k, y2.data_ptr(), 1000)
        b2.sync(gpu_fd)
        assert torch.equal(y.view(torch.int16), y2.view(torch.int16))
    s = torch.cuda.Stream()
    b2.set_stream(gpu_fd, s.cuda_stream)
    try:
        y3 = torch.zeros_like(y)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            fk.run(m, xd.data_ptr(), k, y3.data_ptr(), 1000)
        with torch.cuda.stream(s):
            for _ in range(3):
                y3.zero_()
                g.replay()
        s.synchronize()
        assert torch.equal(y.view(torch.int16), y3.view(torch.int16))
        del g
    finally:
        b2.set_stream(gpu_fd, None)
    assert b2.status(gpu_fd) == 0
    fk.destroy()


def test_ksplit_argument_errors(b2, gpu_fd):
    L = b2.lib()
    x, w, b = case(64, 256, 256, 5)
    op = b2.Linear(gpu_fd, 1, 256, 256, w, b, post=b2.CO_LINEAR_NONE, acc=b2.ACC_FP32, compat=False)
    t16 = b2.Linear(gpu_fd, 1, 256, 256, w, b, post=b2.CO_LINEAR_NONE, acc=b2.ACC_TILE16, compat=False)
    h = ctypes.c_void_p()
    assert L.b2_ksplit_create(t16.h, 1, 0, 64, ctypes.byref(h)) == b2.E_UNSUPPORTED
    assert L.b2_ksplit_create(op.h, 9, 0, 64, ctypes.byref(h)) == b2.E_SHAPE
    assert L.b2_ksplit_create(op.h, 2, 2, 64, ctypes.byref(h)) == b2.E_SHAPE
    assert L.b2_ksplit_create(op.h, 1, 0, 64, ctypes.byref(h)) == 0
    xd = torch.from_numpy(x).cuda()
    y = torch.zeros(64, 256, dtype=torch.float16, device="cuda")
    torch.cuda.synchronize()
    assert L.b2_ksplit_run(h, 8, xd.data_ptr(), 256, y.data_ptr(), 256) == b2.E_UNSUPPORTED
    assert L.b2_ksplit_run(h, 65, xd.data_ptr(), 256, y.data_ptr(), 256) == b2.E_SHAPE
    assert L.b2_ksplit_run(h, 64, xd.data_ptr() + 2, 256, y.data_ptr(), 256) == b2.E_SHAPE
    L.b2_ksplit_destroy(h)
    # a two-rank operator on one process: a peer blob that declares another layout is refused
    # before anything is mapped
    h2 = ctypes.c_void_p()
    assert L.b2_ksplit_create(op.h, 2, 0, 64, ctypes.byref(h2)) == 0
    assert L.b2_ksplit_run(h2, 64, xd.data_ptr(), 256, y.data_ptr(), 256) == b2.E_SHAPE   # not connected
    mine = ctypes.create_string_buffer(b2.KSPLIT_BLOB_BYTES)
    assert L.b2_ksplit_export(h2, mine) == 0
    other = bytearray(mine.raw)
    other[72:76] = (1).to_bytes(4, "little")                  # rank 1
    other[76:80] = (33).to_bytes(4, "little")                 # rows_per_rank 33 instead of 32
    assert L.b2_ksplit_connect(h2, bytes(mine.raw) + bytes(other)) == b2.E_SHAPE
    L.b2_ksplit_destroy(h2)
    b2.sync(gpu_fd)
    assert b2.status(gpu_fd) == 0
    t16.destroy()
    op.destroy()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import importlib
    import sys
    sys.path.insert(0, ROOT)
    import torch as t
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        b2 = importlib.import_module("rockchip-npu-notes_b200")
        sharded = importlib.import_module("rockchip-npu-notes_b200.sharded")
        import oracle as orc
        t.cuda.set_device(rank)
        fd = b2.open_device(rank)
        b2.set_stream(fd, t.cuda.current_stream().cuda_stream)
        m, n, k = 2000, 1024, 4096
        x, w, b = case(m, n, k, 11)
        fk = sharded.FusedKSplit(fd, m, w, b, world, rank, t, dist, post=b2.CO_LINEAR_NONE)
        xs = t.from_numpy(np.ascontiguousarray(x[:, fk.k0:fk.k1])).cuda()
        y = t.zeros(m, n, dtype=t.float16, device="cuda")
        t.cuda.synchronize()
        for _ in range(3):
            fk.run(m, xs.data_ptr(), fk.k1 - fk.k0, y.data_ptr(), n)
        t.cuda.synchronize()
        st = b2.status(fd)
        r0, r1 = fk.rows(m)
        rows = np.unique(np.linspace(r0, r1 - 1, 12).astype(int))
        ref = orc.linear("fp64", x[rows], w, b, post=0, want=("act",))["act"]
        ok, worst = orc.tolerance_ok(y.cpu().numpy()[rows], ref)
        dist.barrier()
        fk.destroy()
        b2.close(fd)
        out[rank] = (int(st), bool(ok), float(worst))
    finally:
        dist.destroy_process_group()


def test_two_gpu_fused_ksplit(b2):
    if b2.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(2):
        st, ok, worst = out[r]
        assert st == 0 and ok, (r, st, worst)


def _lonely_rank(rank, world, port, out):
    """Rank 1 never runs a round; rank 0's round must time out and report it."""
    import importlib
    import sys
    import time
    sys.path.insert(0, ROOT)
    import torch as t
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        b2 = importlib.import_module("rockchip-npu-notes_b200")
        sharded = importlib.import_module("rockchip-npu-notes_b200.sharded")
        t.cuda.set_device(rank)
        fd = b2.open_device(rank)
        m, n, k = 256, 512, 1024
        x, w, b = case(m, n, k, 13)
        fk = sharded.FusedKSplit(fd, m, w, b, world, rank, t, dist)
        dist.barrier()
        result = None
        if rank == 0:
            xs = t.from_numpy(np.ascontiguousarray(x[:, fk.k0:fk.k1])).cuda()
            y = t.zeros(m, n, dtype=t.float16, device="cuda")
            t.cuda.synchronize()
            t0 = time.time()
            fk.run(m, xs.data_ptr(), fk.k1 - fk.k0, y.data_ptr(), n)
            b2.sync(fd)
            waited = time.time() - t0
            st = b2.status(fd)
            # the context still works: a plain run afterwards
            op = b2.Linear(fd, 1, k, n, w, b, post=b2.CO_LINEAR_NONE, acc=b2.ACC_FP32, compat=False)
            xf = t.from_numpy(x).cuda()
            y2 = t.zeros(m, n, dtype=t.float16, device="cuda")
            t.cuda.synchronize()
            op.run_device(m, xf.data_ptr(), k, y2.data_ptr(), n)
            b2.sync(fd)
            st2 = b2.status(fd)
            op.destroy()
            result = (int(st), float(waited), int(st2), bool(t.isfinite(y2.float()).all()))
        dist.barrier()                      # rank 1 keeps its buffer until rank 0 is done
        fk.destroy()
        b2.close(fd)
        out[rank] = result
    finally:
        dist.destroy_process_group()


def test_two_gpu_missing_rank_times_out(b2):
    if b2.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_lonely_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    st, waited, st2, finite = out[0]
    assert st & b2.STATUS_TIMEOUT, st
    assert 0.5 < waited < 30, waited
    assert st2 == 0 and finite
