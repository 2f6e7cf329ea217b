"""Static FP16 graph (co_graph_*) on the GPU, through the C-ABI library, against the oracle.

Follows the reference's graph gate (research/custom-ops/tools/python/graph_gate.py:60-124) on its
own shapes and inputs: the SwiGLU FFN Y = X + Linear(SiLU(Linear(Z, Wg, b)) * Linear(Z, Wu), Wd),
Z = X or RMSNorm(X), with and without bias; every output within the gate's 0.003 of the gate's own
oracle (tests/golden/graph_gate_ffn.npz), CO_CHAIN and CO_SEPARATE byte-identical, three repeated
runs byte-identical. Plus, bit for bit against the oracle's C restatement: the SiLU / GELU /
HardSigmoid nodes over every finite FP16 input and the RMSNorm node (exact statistics); the CO_CHAIN
program fused (one gated GEMM, one residual epilogue) and replayed as a CUDA graph; small-M FFNs
through the weight-streaming kernel; larger FFNs against the oracle within the operator tolerance.
"""
import os

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "graph_gate_ffn.npz")


@pytest.fixture(scope="module")
def G():
    import importlib
    return importlib.import_module("rockchip-npu-notes_b200.graph")


def bits(a):
    return np.ascontiguousarray(a).view(np.uint16)


def finite_f16():
    b = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    return b[(b & 0x7C00) != 0x7C00].view(np.float16)


def test_activation_nodes_bitwise_over_every_finite_fp16(b2, G, gpu_fd):
    a = finite_f16().reshape(248, 256)
    nodes = [G.input_node(248, 256), G.unary_node(b2.CO_GRAPH_SILU, 0), G.unary_node(b2.CO_GRAPH_GELU, 0),
             G.unary_node(b2.CO_GRAPH_HSIG, 0)]
    for mode in (b2.CO_SEPARATE, b2.CO_CHAIN):
        g = G.Graph(gpu_fd, nodes, [1, 2, 3], mode)
        out = g.run({0: a})
        for node, op in ((1, oracle.EW_SILU), (2, oracle.EW_GELU), (3, oracle.EW_HSIG)):
            want = oracle.ew(op, a)
            diff = np.flatnonzero(bits(out[node]) != bits(want))
            assert diff.size == 0, (node, a.ravel()[diff[:8]], out[node].ravel()[diff[:8]], want.ravel()[diff[:8]])
        g.destroy()


def test_add_mul_bitwise(b2, G, gpu_fd):
    rng = np.random.default_rng(3)
    a = (rng.standard_normal((77, 301)) * 40).astype(np.float16)
    c = (rng.standard_normal((77, 301)) * 3).astype(np.float16)
    nodes = [G.input_node(77, 301), G.input_node(77, 301), G.binary_node(b2.CO_GRAPH_ADD, 0, 1),
             G.binary_node(b2.CO_GRAPH_MUL, 1, 0)]
    g = G.Graph(gpu_fd, nodes, [2, 3], b2.CO_CHAIN)
    out = g.run({1: c, 0: a})
    assert np.array_equal(bits(out[2]), bits(oracle.ew(oracle.EW_ADD, a, c)))
    assert np.array_equal(bits(out[3]), bits(oracle.ew(oracle.EW_MUL, c, a)))


def _gate_inputs(m, d, h):
    x = oracle.lcg_fill(m * d, 123, 0.7).reshape(m, d)
    wg = oracle.lcg_fill(h * d, 451, 0.06).reshape(h, d)
    wu = oracle.lcg_fill(h * d, 911, 0.07).reshape(h, d)
    wd = oracle.lcg_fill(d * h, 771, 0.05).reshape(d, h)
    bias = oracle.lcg_fill(h, 153, 0.2)
    gamma = (1 + oracle.lcg_fill(d, 229, 0.3).astype(np.float64)).astype(np.float16)
    return x, wg, wu, wd, bias, gamma


@pytest.mark.parametrize("case", range(4))
def test_ffn_on_the_reference_gate_shapes(b2, G, gpu_fd, case):
    z = np.load(GOLDEN)
    m, d, h = (int(v) for v in z["shapes"][case])
    x, wg, wu, wd, bias, gamma = _gate_inputs(m, d, h)
    for use_bias in (0, 1):
        for norm in (0, 1):
            nodes, out = G.swiglu_ffn(m, d, h, wg, wu, wd, bias if use_bias else None, gamma if norm else None)
            results = []
            for mode in (b2.CO_SEPARATE, b2.CO_CHAIN):
                g = G.Graph(gpu_fd, nodes, out, mode)
                runs = [g.run({0: x}) for _ in range(3)]
                assert all(np.array_equal(bits(r), bits(runs[0])) for r in runs), "repeat mismatch"
                if mode == b2.CO_CHAIN:
                    info = g.info()
                    assert info["gated"] == 1 and info["residual"] == 1 and info["captured"] == 1, info
                results.append(runs[0])
                g.destroy()
            assert np.array_equal(bits(results[0]), bits(results[1])), "chain/separate byte mismatch"
            y = results[1].astype(np.float64)
            assert np.isfinite(y).all()
            key = f"y_{m}_{d}_{h}_b{use_bias}_n{norm}"
            if key in z.files:
                err = np.abs(y - z[key].reshape(m, d).astype(np.float64)).max()
                assert err <= 0.003, (key, err)          # the reference gate's own bound
            ref = oracle.ffn(x, wg, wu, wd, bias if use_bias else None, None, gamma if norm else None)
            assert oracle.tolerance_ok(results[1], ref), (m, d, h, use_bias, norm)


def _ffn_case(m, d, h, seed, gelu=False, up_bias=False):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((m, d)) * 0.7).astype(np.float16)
    wg = (rng.standard_normal((h, d)) / np.sqrt(d)).astype(np.float16)
    wu = (rng.standard_normal((h, d)) / np.sqrt(d)).astype(np.float16)
    wd = (rng.standard_normal((d, h)) / np.sqrt(h)).astype(np.float16)
    bias = (rng.standard_normal(h) * 0.2).astype(np.float16)
    bias2 = (rng.standard_normal(h) * 0.2).astype(np.float16) if up_bias else None
    return x, wg, wu, wd, bias, bias2


@pytest.mark.parametrize("m,d,h,gelu,up_bias", [(1, 1024, 2816, 0, 0), (3, 512, 1000, 1, 1), (8, 4096, 4096, 0, 0),
                                                (9, 256, 300, 0, 1), (300, 512, 1000, 1, 0),
                                                (1024, 1024, 2816, 0, 0), (512, 4096, 4096, 0, 1)])
def test_ffn_against_oracle(b2, G, gpu_fd, m, d, h, gelu, up_bias):
    x, wg, wu, wd, bias, bias2 = _ffn_case(m, d, h, m + d + h, gelu, up_bias)
    act = b2.CO_GRAPH_GELU if gelu else b2.CO_GRAPH_SILU
    nodes, out = G.swiglu_ffn(m, d, h, wg, wu, wd, bias, act=act)
    nodes[2]["bias"] = bias2
    outs = []
    for mode in (b2.CO_SEPARATE, b2.CO_CHAIN):
        g = G.Graph(gpu_fd, nodes, out, mode, budget=4 << 30)
        outs.append(g.run({0: x}))
        g.destroy()
    assert np.array_equal(bits(outs[0]), bits(outs[1])), "chain/separate byte mismatch"
    ref = oracle.ffn(x, wg, wu, wd, bias, bias2, act=oracle.EW_GELU if gelu else oracle.EW_SILU)
    assert oracle.tolerance_ok(outs[1], ref), np.abs(outs[1].astype(np.float64) - ref.astype(np.float64)).max()


def test_rmsnorm_node_bitwise_and_rejection(b2, G, gpu_fd):
    rng = np.random.default_rng(11)
    m, n = 257, 4096
    x = (rng.standard_normal((m, n)) * 2).astype(np.float16)
    x[5] = 0
    gamma = (1 + rng.standard_normal(n) * 0.3).astype(np.float16)
    nodes = [G.input_node(m, n), G.rmsnorm_node(0, gamma, 1e-5)]
    g = G.Graph(gpu_fd, nodes, 1, b2.CO_CHAIN)
    y = g.run({0: x})
    want, bad = oracle.rmsnorm(x, gamma, 1e-5)
    assert bad == 0 and np.array_equal(bits(y), bits(want))
    x[9, 100] = 256.0                                   # its FP16 square overflows: ROCKET_E_SHAPE
    rc, outs = g.run_rc({0: x}, {1: np.full((m, n), 7.0, np.float16)})
    assert rc == b2.E_SHAPE and (outs[1] == 7.0).all()
    x[9, 100] = 1.0
    assert np.array_equal(bits(g.run({0: x})), bits(oracle.rmsnorm(x, gamma, 1e-5)[0]))


def _view(ptr, rows, ld):
    class Iface:
        __cuda_array_interface__ = {"shape": (rows, ld), "typestr": "<f2", "data": (ptr, False), "version": 2}
    return torch.as_tensor(Iface(), device="cuda")


def test_device_resident_launch(b2, G, gpu_fd):
    m, d, h = 64, 512, 768
    x, wg, wu, wd, bias, _ = _ffn_case(m, d, h, 7)
    nodes, out = G.swiglu_ffn(m, d, h, wg, wu, wd, bias)
    g = G.Graph(gpu_fd, nodes, out, b2.CO_CHAIN)
    want = g.run({0: x})
    xp, ldx = g.tensor(0)
    yp, ldy = g.tensor(out)
    xin, yout = _view(xp, m, ldx), _view(yp, m, ldy)
    yout.zero_()
    xin[:, :d].copy_(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    for _ in range(3):
        g.launch()
    b2.sync(gpu_fd)
    assert g.status() == 0
    got = yout[:, :d].cpu().numpy()
    assert np.array_equal(bits(got), bits(want))
    assert g.info()["kernels"] == 4       # gated GEMM, residual GEMM, guard check, output scan
