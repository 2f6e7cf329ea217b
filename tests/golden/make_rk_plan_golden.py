"""Generates tests/golden/rk_plans.json: plan descriptors produced by the reference's own planner.

Run once, in a checkout that has the reference project:

    python tests/golden/make_rk_plan_golden.py <reference-root>

For each case it builds an RKIR module with the reference tooling's module builders
(research/tilelang-rknpu/python/rknpu_backend: matmul_module, projection_module, swiglu_module,
activation_module, branch_outputs_module), compiles it with its pipeline (compile_rkir, the same
options as its dataflow tests, tests/test_dataflow_multitile.py:80-85) in both submit modes, turns the
plan into the C descriptors with its ffi builder (runtime/ffi.py build_plan_descriptor, exactly what
its LibRKPlan.create_plan hands to rk_plan_create) and records every descriptor field as plain
JSON, plus the plan's constants and bindings. tests/test_rk_plan_golden.py rebuilds the C
structs from that JSON and runs them through this library's rk_plan_create / rk_workspace_run.
"""
import ctypes
import json
import os
import sys


def scalar_fields(s, skip=()):
    out = {}
    for name, ctype in s._fields_:
        if name in skip:
            continue
        v = getattr(s, name)
        if isinstance(v, (int, float)):
            out[name] = v
        elif isinstance(v, bytes):
            out[name] = v.decode()
        elif isinstance(v, ctypes.Array):
            out[name] = list(v)
        elif isinstance(v, ctypes.Structure):
            out[name] = scalar_fields(v)
    return out


def ids(ptr, n):
    return [int(ptr[i]) for i in range(n)] if n else []


def dump(desc):
    d = scalar_fields(desc, skip=("values", "buffers", "views", "actions", "submits", "publish"))
    d["values"] = []
    for i in range(desc.nvalues):
        v = desc.values[i]
        row = scalar_fields(v, skip=("name",))
        row["name"] = ctypes.string_at(v.name, v.name_len).decode()
        d["values"].append(row)
    d["buffers"] = [scalar_fields(desc.buffers[i]) for i in range(desc.nbuffers)]
    d["views"] = [scalar_fields(desc.views[i]) for i in range(desc.nviews)]
    d["actions"] = []
    for i in range(desc.nactions):
        a = desc.actions[i]
        row = scalar_fields(a, skip=("inputs", "outputs", "deps", "origin"))
        row["inputs"] = ids(a.inputs, a.ninputs)
        row["outputs"] = ids(a.outputs, a.noutputs)
        row["deps"] = ids(a.deps, a.ndeps)
        row["origin"] = bytes(a.origin).split(b"\0", 1)[0].decode()
        d["actions"].append(row)
    d["submits"] = []
    for i in range(desc.nsubmits):
        s = desc.submits[i]
        row = scalar_fields(s, skip=("task_ids", "deps"))
        row["task_ids"] = ids(s.task_ids, s.ntask_ids)
        row["deps"] = ids(s.deps, s.ndeps)
        d["submits"].append(row)
    d["publish"] = [scalar_fields(desc.publish[i]) for i in range(desc.npublish)]
    return d


def main():
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    ref = os.path.abspath(sys.argv[1])
    sys.path.insert(0, os.path.join(ref, "research", "tilelang-rknpu", "python"))
    import rknpu_backend as rb
    from rknpu_backend import CompileOptions, compile_rkir, default_profile
    from rknpu_backend.runtime.ffi import build_plan_descriptor

    profile = default_profile()
    cases = {
        "matmul_300": lambda: rb.matmul_module(m=300, k=300, n=300),
        "linear_hardsigmoid_64x512x256": lambda: rb.matmul_module(m=64, k=512, n=256, b_layout="nk",
                                                                  activation="hardsigmoid"),
        "projection_300": lambda: rb.projection_module(m=300, d=300, h=300),
        "swiglu_300": lambda: rb.swiglu_module(m=300, d=300, h=300),
        "activation_silu_40x72": lambda: rb.activation_module(m=40, n=72, activation="silu"),
        "branch_64x512": lambda: rb.branch_outputs_module(m=64, k=512, n1=96, n2=40),
    }
    out = {}
    for name, make in cases.items():
        for mode in ("chain", "separate"):
            try:
                plan = compile_rkir(make(), profile=profile,
                                    options=CompileOptions(numeric_mode="rk_f16_tiled", allow_approx_lut=True,
                                                           submit_mode=mode)).plan
            except Exception as e:        # a builder option this checkout does not support
                print(f"skip {name}/{mode}: {type(e).__name__}: {e}")
                continue
            desc, holder = build_plan_descriptor(plan)
            entry = dump(desc)
            del holder
            entry["constants"] = [{"binding_id": c.binding_id, "name": c.name, "shape": list(c.shape),
                                   "identity": c.name.startswith("__identity_")} for c in plan.constants]
            entry["bindings"] = [{"id": b.id, "name": b.name, "role": b.role, "shape": list(b.shape)}
                                 for b in plan.bindings]
            out[f"{name}/{mode}"] = entry
            print(f"{name}/{mode}: {len(entry['actions'])} actions, {len(entry['submits'])} submits")
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "rk_plans.json")
    with open(path, "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
