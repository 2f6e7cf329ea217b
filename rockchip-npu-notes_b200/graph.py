"""Static FP16 graph compiler (``include/co_graph.h``) through ctypes.

Mirrors the reference's graph API (research/custom-ops/include/co_graph.h): nodes are
``CoGraphNode`` records built with the helpers below, planned with ``plan()``, compiled into a
``Graph`` on an opened device handle and run with host arrays.  Node kinds built on B200: INPUT,
LINEAR, ADD, MUL, SILU, GELU, HSIG, RMSNORM (SOFTMAX / ROPE / ATTENTION plan as
ROCKET_E_UNSUPPORTED).  There is no CPU fallback.
"""
import ctypes

import numpy as np

from . import (CO_CHAIN, CO_GRAPH_ADD, CO_GRAPH_GELU, CO_GRAPH_HSIG, CO_GRAPH_INPUT, CO_GRAPH_LINEAR,
               CO_GRAPH_MUL, CO_GRAPH_RMSNORM, CO_GRAPH_SILU, B2GraphInfo, CoGraphDesc, CoGraphInput,
               CoGraphNode, CoGraphOutput, CoGraphPlan, RocketError, _f16, check, lib)


def input_node(rows, cols, flags=0):
    return dict(op=CO_GRAPH_INPUT, rows=rows, cols=cols, flags=flags)


def linear_node(a, cols, weights, bias=None):
    return dict(op=CO_GRAPH_LINEAR, a=a, cols=cols, weights=weights, bias=bias)


def binary_node(op, a, b):
    return dict(op=op, a=a, b=b)


def unary_node(op, a):
    return dict(op=op, a=a)


def rmsnorm_node(a, gamma, epsilon=1e-5):
    return dict(op=CO_GRAPH_RMSNORM, a=a, gamma=gamma, epsilon=epsilon)


def swiglu_ffn(rows, d, h, wg, wu, wd, bias=None, gamma=None, epsilon=1e-5, act=CO_GRAPH_SILU):
    """The reference graph CLI's FFN (research/custom-ops/tools/c/graph_cli.c:67-74):
    Y = X + Linear(act(Linear(Z, Wg, b)) * Linear(Z, Wu), Wd), Z = RMSNorm(X) when gamma is
    given, else X.  Returns (nodes, output node id)."""
    z = 7 if gamma is not None else 0
    nodes = [input_node(rows, d),
             linear_node(z, h, wg, bias),
             linear_node(z, h, wu),
             unary_node(act, 1),
             binary_node(CO_GRAPH_MUL, 3, 2),
             linear_node(4, d, wd),
             binary_node(CO_GRAPH_ADD, 5, 0)]
    if gamma is not None:
        nodes.append(rmsnorm_node(0, gamma, epsilon))
    return nodes, 6


class Desc:
    """A ``co_graph_desc`` and the FP16 arrays its nodes point at (kept alive with it)."""

    def __init__(self, nodes, output=0, budget=0):
        self.keep = []
        self.nodes = (CoGraphNode * max(1, len(nodes)))()
        for i, spec in enumerate(nodes):
            n = self.nodes[i]
            for key, value in spec.items():
                if key in ("weights", "bias", "gamma"):
                    if value is None:
                        continue
                    arr = _f16(value)
                    self.keep.append(arr)
                    setattr(n, key, arr.ctypes.data_as(ctypes.c_void_p))
                else:
                    setattr(n, key, value)
        self.desc = CoGraphDesc(self.nodes, len(nodes), output, budget)


def plan(nodes, outputs, budget=0):
    """(rc, CoGraphPlan) of co_graph_plan_many for the node list and output ids."""
    d = Desc(nodes, outputs[0], budget)
    ids = (ctypes.c_uint * len(outputs))(*outputs)
    p = CoGraphPlan()
    rc = lib().co_graph_plan_many(ctypes.byref(d.desc), ids, len(outputs), ctypes.byref(p))
    return rc, p


class Graph:
    """A compiled graph (co_graph_compile_many) bound to device handle ``fd``."""

    def __init__(self, fd, nodes, outputs, mode=CO_CHAIN, budget=0):
        if isinstance(outputs, int):
            outputs = [outputs]
        self.outputs = list(outputs)
        d = Desc(nodes, self.outputs[0], budget)
        ids = (ctypes.c_uint * len(outputs))(*outputs)
        h = ctypes.c_void_p()
        check("co_graph_compile_many", lib().co_graph_compile_many(fd, ctypes.byref(d.desc), ids, len(outputs),
                                                                   mode, ctypes.byref(h)))
        self.h = h
        self.mode = mode
        rc, self.plan = plan(nodes, self.outputs, budget)
        check("co_graph_plan_many", rc)

    def shape(self, node):
        t = self.plan.tensors[node]
        return t.rows, t.cols

    def run_rc(self, inputs, outs=None):
        """co_graph_run_many: inputs {node: array}; returns (rc, {node: float16 array})."""
        keep = [_f16(v) for v in inputs.values()]
        ins = (CoGraphInput * max(1, len(keep)))()
        for i, (node, arr) in enumerate(zip(inputs.keys(), keep)):
            ins[i].node = node
            ins[i].data = arr.ctypes.data_as(ctypes.c_void_p)
        if outs is None:
            outs = {o: np.zeros(self.shape(o), np.float16) for o in self.outputs}
        ob = (CoGraphOutput * max(1, len(outs)))()
        for i, (node, arr) in enumerate(outs.items()):
            ob[i].node = node
            ob[i].data = arr.ctypes.data_as(ctypes.c_void_p)
        rc = lib().co_graph_run_many(self.h, ins, len(keep), ob, len(outs))
        return rc, outs

    def run(self, inputs):
        rc, outs = self.run_rc(inputs)
        check("co_graph_run_many", rc)
        return outs[self.outputs[0]] if len(self.outputs) == 1 else outs

    def tensor(self, node):
        """(device pointer, row pitch in elements) of a planned node's tensor."""
        p, ld = ctypes.c_void_p(), ctypes.c_size_t()
        check("b2_graph_tensor", lib().b2_graph_tensor(self.h, node, ctypes.byref(p), ctypes.byref(ld)))
        return p.value, ld.value

    def launch(self):
        check("b2_graph_launch", lib().b2_graph_launch(self.h))

    def status(self):
        return lib().b2_graph_status(self.h)

    def info(self):
        i = B2GraphInfo()
        check("b2_graph_get_info", lib().b2_graph_get_info(self.h, ctypes.byref(i)))
        return dict(gated=i.gated, residual=i.residual, kernels=i.kernels, captured=i.captured)

    def destroy(self):
        if getattr(self, "h", None):
            lib().co_graph_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


__all__ = ["Desc", "Graph", "RocketError", "binary_node", "input_node", "linear_node", "plan", "rmsnorm_node",
           "swiglu_ffn", "unary_node"]
