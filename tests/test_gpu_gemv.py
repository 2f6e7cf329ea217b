"""Small-M (decode) kernels and the grouped projection launch, through the C-ABI library.

* The streamed tensor-core kernel (K <= 16384; M split into row groups whose x rows fit its 32 KB
  table; whole-row launches whose x rows fit 12 KB run as half-SM CTAs with a 6-slot ring, the
  others with 12 slots) computes each x row independently of the rest of the batch: rows of M=1, 2, 3, 8 runs
  agree bit for bit, both accumulation modes, with and without bias and HardSigmoid, ragged K, NaN
  in the x pitch padding; all within tolerance of the oracle.
* b2_linear_group_run_device: every member's output equals that operator's own
  b2_linear_run_device bit for bit (shared and separate inputs, CO_SEPARATE and tile-16 members,
  a K=4096 member that joins the shared launch at m <= 2 and runs on its own at m = 8), and a
  group whose members all stream is one launch.
  The group replaces the Q/K/V projection step of research/custom-ops/src/co_decoder.c:128-129.
* An LM-head-sized M=1 run (N=49152, K=576) against the oracle (tile-16) and FP64 (FP32 mode).
* Long-K launches at decode sizes (up to K = 16384), against the oracle / FP64, with rows of M = 1
  and M = 4 identical and repeated launches identical.
Tolerance: |y - ref| <= 2e-3 + 2e-3*|ref| element-wise.
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def uniform_case(m, n, k, seed):
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1, 1, (m, k)).astype(np.float16)
    w = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), (n, k)).astype(np.float16)
    b = rng.uniform(-0.1, 0.1, n).astype(np.float16)
    return x, w, b


def r8(v):
    return -(-v // 8) * 8


def dev(a, ld, fill=0.0):
    """FP16 device copy of host rows `a` with row pitch `ld` elements."""
    t = torch.full((a.shape[0], ld), fill, dtype=torch.float16, device="cuda")
    t[:, :a.shape[1]] = torch.from_numpy(a).cuda()
    return t


def bits(t, cols):
    return t[:, :cols].cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("k", [1, 17, 576, 1000, 1536, 2048, 2056, 3000, 4096, 6000, 8192, 8200, 12288])
def test_small_m_rows_are_batch_independent_and_within_tolerance(b2, gpu_fd, k):
    """Rows of M=1, 2, 3, 4 and 8 runs agree bit for bit (each x row's result does not depend on the
    rest of the batch, nor on the unit kind that serves it: above K = 2048, M <= 4 runs long-K
    whole-row (octet) units when the x rows fit 32 KB -- two W rows per unit up to K = 4096, one
    above -- and the other batches 16-row K slices; M=8 at K=4096 is one wide sliced launch with a
    64 KB x table, at K=8192 two launches of 4 rows; above K = 8192, M = 1 runs one-row octet units
    in 24 KB slots and the other batches slices), in both accumulation modes, with and without
    bias and HardSigmoid; all rows within tolerance. N is odd, so a two-row unit ends with one row."""
    n = 301
    x, w, b = uniform_case(8, n, k, 7000 + k)
    ldx, ldy = r8(k), r8(n)
    xd = dev(x, ldx, fill=float("nan"))          # pitch padding must never be read as data
    for acc in (b2.ACC_TILE16, b2.ACC_FP32):
        for post in (b2.CO_LINEAR_NONE, b2.CO_LINEAR_HSIG):
            for bias in (b, None):
                op = b2.Linear(gpu_fd, 1, k, n, w, bias, post=post, mode=b2.CO_CHAIN, acc=acc, compat=False)
                info = op.info()
                # M=1: half-SM ring while the x row fits its 12 KB table (whole-row and long-K octet
                # units alike); K = 8192 (16 KB) runs full-SM CTAs with 12 slots; longer rows 8 wide slots
                assert info.kernel == 1 and info.stages == (6 if k <= 6144 else (12 if k <= 8192 else 8))
                ys = {m: torch.zeros((m, ldy), dtype=torch.float16, device="cuda") for m in (1, 2, 3, 4, 8)}
                torch.cuda.synchronize()
                for m, y in ys.items():
                    op.run_device(m, xd.data_ptr(), ldx, y.data_ptr(), ldy)
                b2.sync(gpu_fd)
                assert b2.status(gpu_fd) == 0
                what = f"k={k} acc={acc} post={post} bias={bias is not None}"
                full = bits(ys[8], n)
                for m in (1, 2, 3, 4):
                    assert np.array_equal(full[:m], bits(ys[m], n)), f"{what} m={m}"
                p = 1 if post == b2.CO_LINEAR_HSIG else 0
                if acc == b2.ACC_TILE16:
                    ref = oracle.linear("tile16", x, w, bias, post=p)["y16"]
                else:
                    ref = oracle.linear("fp64", x, w, bias, post=p, want=("act",))["act"]
                ok, worst = oracle.tolerance_ok(ys[8][:, :n].cpu().numpy(), ref)
                assert ok, f"{what}: worst {worst:.3f}"
                op.destroy()


def _projection_set(b2, fd, m):
    """A decoder-layer-like set: Q/K/V/gate share one input, down and a K=4096 member their own."""
    spec = [  # name, n, k, input, acc, post, bias, mode
        ("q", 576, 576, "h", b2.ACC_TILE16, b2.CO_LINEAR_HSIG, True, b2.CO_CHAIN),
        ("k", 192, 576, "h", b2.ACC_FP32, b2.CO_LINEAR_NONE, False, b2.CO_CHAIN),
        ("v", 192, 576, "h", b2.ACC_FP32, b2.CO_LINEAR_HSIG, True, b2.CO_SEPARATE),
        ("gate", 1536, 576, "h", b2.ACC_TILE16, b2.CO_LINEAR_NONE, True, b2.CO_SEPARATE),
        ("down", 576, 1536, "f", b2.ACC_FP32, b2.CO_LINEAR_NONE, False, b2.CO_CHAIN),
        ("wide", 64, 4096, "g", b2.ACC_FP32, b2.CO_LINEAR_HSIG, True, b2.CO_CHAIN),
    ]
    inputs = {"h": 576, "f": 1536, "g": 4096}
    rng = np.random.default_rng(99)
    host = {key: rng.uniform(-1, 1, (m, kk)).astype(np.float16) for key, kk in inputs.items()}
    xs = {key: dev(a, a.shape[1]) for key, a in host.items()}
    ops, items, refs = [], [], []
    for i, (name, n, k, inp, acc, post, has_bias, mode) in enumerate(spec):
        _, w, b = uniform_case(1, n, k, 500 + i)
        bias = b if has_bias else None
        ops.append(b2.Linear(fd, 1, k, n, w, bias, post=post, mode=mode, acc=acc, compat=False))
        items.append((name, n, k, xs[inp]))
        p = 1 if post == b2.CO_LINEAR_HSIG else 0
        if acc == b2.ACC_TILE16:
            refs.append(oracle.linear("tile16", host[inp], w, bias, post=p)["y16"])
        else:
            refs.append(oracle.linear("fp64", host[inp], w, bias, post=p, want=("act",))["act"])
    return ops, items, xs, refs


@pytest.mark.parametrize("m", [1, 2, 8])
def test_group_equals_individual_runs_bitwise(b2, gpu_fd, m):
    ops, items, xs, refs = _projection_set(b2, gpu_fd, m)
    solo = [torch.zeros((m, r8(n)), dtype=torch.float16, device="cuda") for _, n, _, _ in items]
    grp = [torch.full((m, r8(n)), 3.0, dtype=torch.float16, device="cuda") for _, n, _, _ in items]
    torch.cuda.synchronize()
    for op, (_, n, k, x), y in zip(ops, items, solo):
        op.run_device(m, x.data_ptr(), x.shape[1], y.data_ptr(), r8(n))
    b2.sync(gpu_fd)
    b2.group_run_device(ops, m, [x.data_ptr() for _, _, _, x in items], [x.shape[1] for _, _, _, x in items],
                        [y.data_ptr() for y in grp], [r8(n) for _, n, _, _ in items])
    b2.sync(gpu_fd)
    assert b2.status(gpu_fd) == 0
    for (name, n, _, _), a, g, ref in zip(items, solo, grp, refs):
        assert np.array_equal(bits(a, n), bits(g, n)), name
        # and every member directly against the oracle: tile-16 members against the reference's
        # arithmetic, FP32 members against FP64 (mixed widths, HardSigmoid and CO_SEPARATE members)
        ok, worst = oracle.tolerance_ok(g[:, :n].cpu().numpy(), ref)
        assert ok, f"{name} m={m}: worst err/tol {worst:.3f}"

    # the streamed members share one launch while their distinct x rows fit the 32 KB shared
    # x table (Q/K/V/gate share one input); at m=8 the 1536-wide input needs a second launch
    streamed = [i for i, it in enumerate(items) if it[2] <= 2048]
    distinct = {items[i][3].data_ptr(): items[i][2] for i in streamed}
    expect = 1 if sum(m * r8(k) * 2 for k in distinct.values()) <= 32768 else 2
    before = b2.counters()["launches"]
    b2.group_run_device([ops[i] for i in streamed], m, [items[i][3].data_ptr() for i in streamed],
                        [items[i][3].shape[1] for i in streamed], [grp[i].data_ptr() for i in streamed],
                        [r8(items[i][1]) for i in streamed])
    b2.sync(gpu_fd)
    assert b2.counters()["launches"] - before == expect
    if m <= 2:
        # the K=4096 member streams whole rows (octet units) and joins the shared launch: the
        # 576/1536/4096-wide inputs fit the 32 KB x table together
        before = b2.counters()["launches"]
        b2.group_run_device(ops, m, [x.data_ptr() for _, _, _, x in items], [x.shape[1] for _, _, _, x in items],
                            [y.data_ptr() for y in grp], [r8(n) for _, n, _, _ in items])
        b2.sync(gpu_fd)
        assert b2.counters()["launches"] - before == 1
    for op in ops:
        op.destroy()


def test_group_argument_errors(b2, gpu_fd):
    L = b2.lib()
    x, w, b = uniform_case(1, 64, 64, 3)
    op = b2.Linear(gpu_fd, 1, 64, 64, w, b, post=b2.CO_LINEAR_NONE, compat=False)
    fd2 = b2.open_device(0)
    other = b2.Linear(fd2, 1, 64, 64, w, b, post=b2.CO_LINEAR_NONE, compat=False)
    xd = dev(x, 64)
    yd = torch.zeros((1, 64), dtype=torch.float16, device="cuda")
    torch.cuda.synchronize()
    ptr, ld = xd.data_ptr(), 64
    with pytest.raises(b2.RocketError):
        b2.group_run_device([], 1, [], [], [], [])
    with pytest.raises(b2.RocketError):
        b2.group_run_device([op] * 17, 1, [ptr] * 17, [ld] * 17, [yd.data_ptr()] * 17, [ld] * 17)
    with pytest.raises(b2.RocketError):        # members on two handles
        b2.group_run_device([op, other], 1, [ptr] * 2, [ld] * 2, [yd.data_ptr()] * 2, [ld] * 2)
    with pytest.raises(b2.RocketError):        # misaligned input
        b2.group_run_device([op], 1, [ptr + 2], [ld], [yd.data_ptr()], [ld])
    with pytest.raises(b2.RocketError):        # m = 0
        b2.group_run_device([op], 0, [ptr], [ld], [yd.data_ptr()], [ld])
    b2.sync(gpu_fd)
    assert b2.status(gpu_fd) == 0
    other.destroy()
    op.destroy()
    b2.close(fd2)


def test_lm_head_sized_decode_against_oracle(b2, gpu_fd):
    n, k = 49152, 576
    rng = np.random.default_rng(11)
    x = rng.standard_normal((1, k)).astype(np.float16)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float16)
    xd = dev(x, k)
    for acc in (b2.ACC_TILE16, b2.ACC_FP32):
        op = b2.Linear(gpu_fd, 1, k, n, w, None, post=b2.CO_LINEAR_NONE, acc=acc, compat=False)
        y = torch.zeros((1, n), dtype=torch.float16, device="cuda")
        torch.cuda.synchronize()
        op.run_device(1, xd.data_ptr(), k, y.data_ptr(), n)
        b2.sync(gpu_fd)
        assert b2.status(gpu_fd) == 0
        if acc == b2.ACC_TILE16:
            ref = oracle.linear("tile16", x, w, None, post=0)["y16"]
        else:
            ref = oracle.linear("fp64", x, w, None, post=0, want=("act",))["act"]
        ok, worst = oracle.tolerance_ok(y.cpu().numpy(), ref)
        assert ok, f"acc={acc}: worst {worst:.3f}"
        op.destroy()


@pytest.mark.parametrize("n,k", [(8192, 4096), (16384, 2560), (4100, 11008), (2048, 16384)])
def test_long_k_blocks_against_oracle(b2, gpu_fd, n, k):
    """Long-K streamed launches at decode sizes. K <= 4096: M = 8 streams 16-row K slices (each CTA
    finishes most of its blocks itself and reuses its shared tile-sum buffers -- 16384 x 2560 gives
    about seven blocks per CTA, more than the four buffers -- and completes the blocks at the ends of
    its range across CTAs), while M = 4 (two passes) and M = 1 stream whole rows as octet units; all
    give the same bits for the same x row. Up to K = 12288, M = 1 streams whole rows longer than a
    16 KB slot as octet units in the 8-slot wide configuration (24 KB slots) and M = 4 is sliced,
    again with the same bits; above, every M is sliced. Tile-16 and FP32 results within tolerance
    of the oracle / FP64, repeated launches identical (the block counters return to zero)."""
    rng = np.random.default_rng(n + k)
    ms = (8, 4, 1) if k <= 4096 else ((4, 1) if k <= 12288 else (1,))
    m = ms[0]
    x = rng.uniform(-1, 1, (m, k)).astype(np.float16)
    w = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), (n, k)).astype(np.float16)
    b = rng.uniform(-0.1, 0.1, n).astype(np.float16)
    xd = dev(x, k)
    for acc in (b2.ACC_TILE16, b2.ACC_FP32):
        op = b2.Linear(gpu_fd, 1, k, n, w, b, post=b2.CO_LINEAR_NONE, acc=acc, compat=False)
        info = op.info()
        # M=1: octet (half-SM) / octet in wide slots / sliced
        assert info.kernel == 1 and info.stages == (6 if k <= 4096 else (8 if k <= 12288 else 11))
        ldy = r8(n)
        ys = [torch.zeros((m, ldy), dtype=torch.float16, device="cuda") for _ in range(3)]
        others = {mm: torch.zeros((mm, ldy), dtype=torch.float16, device="cuda") for mm in ms[1:]}
        torch.cuda.synchronize()
        for y in ys:
            op.run_device(m, xd.data_ptr(), k, y.data_ptr(), ldy)
        for mm, y in others.items():
            op.run_device(mm, xd.data_ptr(), k, y.data_ptr(), ldy)
        b2.sync(gpu_fd)
        assert b2.status(gpu_fd) == 0
        assert torch.equal(ys[0].view(torch.int16), ys[1].view(torch.int16))
        assert torch.equal(ys[0].view(torch.int16), ys[2].view(torch.int16))
        for mm, y in others.items():
            assert torch.equal(ys[0][:mm].view(torch.int16), y.view(torch.int16)), f"n={n} k={k} m={mm}"
        if acc == b2.ACC_TILE16:
            ref = oracle.linear("tile16", x, w, b, post=0)["y16"]
        else:
            ref = oracle.linear("fp64", x, w, b, post=0, want=("act",))["act"]
        ok, worst = oracle.tolerance_ok(ys[0][:, :n].cpu().numpy(), ref)
        assert ok, f"n={n} k={k} acc={acc}: worst {worst:.3f}"
        op.destroy()


def test_dependent_chain_under_programmatic_launch(b2, gpu_fd):
    """Back-to-back decode launches may overlap (programmatic dependent launch): a chain whose
    input is the previous launch's output (ping-pong buffers, so each launch also overwrites the
    buffer the launch before it read) gives the same bits with and without a sync after every
    launch, eagerly and as a replayed CUDA graph."""
    k = n = 576
    rng = np.random.default_rng(21)
    ws = [(rng.standard_normal((n, k)) * 0.03).astype(np.float16) for _ in range(3)]
    ops = [b2.Linear(gpu_fd, 1, k, n, w, None, post=b2.CO_LINEAR_HSIG, acc=b2.ACC_FP32, compat=False) for w in ws]
    x0 = torch.from_numpy(rng.standard_normal((1, k)).astype(np.float16)).cuda()
    bufs = [torch.zeros(1, k, dtype=torch.float16, device="cuda") for _ in range(2)]
    steps = 12

    def chain(sync):
        bufs[0].copy_(x0)
        torch.cuda.synchronize()
        for i in range(steps):
            src, dst = bufs[i % 2], bufs[(i + 1) % 2]
            ops[i % 3].run_device(1, src.data_ptr(), k, dst.data_ptr(), n)
            if sync:
                b2.sync(gpu_fd)
        b2.sync(gpu_fd)
        return bufs[steps % 2].clone()

    ref = chain(True)
    got = chain(False)
    assert b2.status(gpu_fd) == 0
    assert torch.equal(ref.view(torch.int16), got.view(torch.int16))
    assert torch.isfinite(ref.float()).all() and ref.float().abs().sum() > 0
    s = torch.cuda.Stream()
    b2.set_stream(gpu_fd, s.cuda_stream)
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(steps):
                src, dst = bufs[i % 2], bufs[(i + 1) % 2]
                ops[i % 3].run_device(1, src.data_ptr(), k, dst.data_ptr(), n)
        for _ in range(2):
            with torch.cuda.stream(s):
                bufs[0].copy_(x0)
                g.replay()
            s.synchronize()
            assert torch.equal(ref.view(torch.int16), bufs[steps % 2].view(torch.int16))
        del g
    finally:
        b2.set_stream(gpu_fd, None)
    for op in ops:
        op.destroy()
