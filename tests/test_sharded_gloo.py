"""Multi-GPU layouts, host side, on CPU: two gloo ranks (no GPU).

Checks the partition (b2_shard_range through the C-ABI) and the data flow of the two layouts of
rockchip-npu-notes_b200/sharded.py with numpy standing in for the GPU kernels:
  * column-parallel: the ranks' column blocks tile [0, N) and all-gathered blocks equal the full
    product;
  * K-split: the ranks' K slices tile [0, K) on 256-column boundaries and the all-reduced FP32
    partials equal the full FP32 product.
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, shapes, out):
    import importlib
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    sharded = importlib.import_module("rockchip-npu-notes_b200.sharded")
    try:
        for (m, n, k) in shapes:
            rng = np.random.default_rng(m + n + k)
            x = rng.standard_normal((m, k)).astype(np.float32)
            w = rng.standard_normal((n, k)).astype(np.float32)
            full = x @ w.T
            # column-parallel
            n0, n1 = sharded.column_shard(n, world, rank)
            sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
            dist.all_gather(sizes, torch.tensor([n1 - n0]))
            widest = max(int(s.item()) for s in sizes)
            block = torch.zeros((m, widest), dtype=torch.float32)  # gloo gathers equal shapes
            block[:, :n1 - n0] = torch.from_numpy(np.ascontiguousarray(full[:, n0:n1]))
            gathered = [torch.zeros((m, widest), dtype=torch.float32) for _ in range(world)]
            dist.all_gather(gathered, block)
            cols = torch.cat([g[:, :int(s.item())] for g, s in zip(gathered, sizes)], dim=1).numpy()
            assert cols.shape == full.shape and np.array_equal(cols, full)
            # K-split
            k0, k1 = sharded.k_shard(k, world, rank)
            assert k0 % 256 == 0 and (k1 == k or k1 % 256 == 0)
            part = torch.from_numpy(np.ascontiguousarray(x[:, k0:k1] @ w[:, k0:k1].T))
            dist.all_reduce(part, op=dist.ReduceOp.SUM)
            assert np.allclose(part.numpy(), full, rtol=1e-4, atol=1e-3)
            spans = [torch.zeros(2, dtype=torch.int64) for _ in range(world)]
            dist.all_gather(spans, torch.tensor([k0, k1]))
            edges = sorted((int(a), int(b)) for a, b in (s.tolist() for s in spans))
            assert edges[0][0] == 0 and edges[-1][1] == k
            assert all(edges[i][1] == edges[i + 1][0] for i in range(world - 1))
        out[rank] = 1
    finally:
        dist.destroy_process_group()


def test_two_rank_layouts_on_gloo():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    out = manager.dict()
    shapes = [(8, 1024, 1000), (5, 300, 513), (4, 17, 256)]
    procs = [ctx.Process(target=_worker, args=(r, world, port, shapes, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(out) == {0: 1, 1: 1}
