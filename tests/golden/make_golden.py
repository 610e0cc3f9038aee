"""Generates tests/golden/*.npz by running the reference itself.

For every case in cases.py: build the graph (GraphBuilder, the reference's
graph ABI), run the reference's optimizer (bafe_optimize) on it, JIT the
optimized graph with the reference's own emitter and `cc`
(bafe_jit_get_or_compile), call the generated kernel on the seeded inputs
(in the optimized graph's input order, as jit.h's contract says), and store
  meta: case, citation, the optimized graph's nodes / inputs / root,
        input specs, row panel;
  in_<name>: the inputs (small cases only; the others are regenerated
        from their seeds by tests/golden/inputs.py);
  out: the reference's output.

Needs oracle/_ref/libbafe.so (make -C oracle ref, from the reference sources)
and runs in this container only -- the GPU host has no reference.
Usage: python tests/golden/make_golden.py [case ...]
"""
from __future__ import annotations

import json
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(ROOT / "bafe-basic-algibra-fusion-engine-_b200"))
sys.path.insert(0, str(ROOT))

from cases import CASES, make_input  # noqa: E402
from bafe_b200.graph import GraphBuilder  # noqa: E402
from oracle import refbafe  # noqa: E402

DT = {"float32": 0, "float64": 1, "int32": 2, "int64": 3, "float16": 4, "bfloat16": 5}
NPDT = {0: np.float32, 1: np.float64, 2: np.int32, 3: np.int64, 4: np.float16, 5: np.uint16}


def run_case(ref: refbafe.Reference, case: dict, cache: dict) -> None:
    t0 = time.time()
    panel = case.get("panel")
    arrays = {}
    for spec in case["inputs"]:
        key = (spec[0], spec[1], spec[2], spec[3], json.dumps(spec[5], sort_keys=True))
        if key not in cache:
            cache.clear() if len(cache) > 4 else None
            cache[key] = make_input(spec)
        a = cache[key]
        if panel and spec[0] in case.get("panel_inputs", ()):
            a = np.ascontiguousarray(a[panel[0]:panel[1]])
        arrays[spec[0]] = a
    if case.get("fuse"):
        opt = fused_graph(ref, case, arrays)
    else:
        g = GraphBuilder()
        ids = [g.add_input(s[0], arrays[s[0]].shape, DT[s[2]], s[4]) for s in case["inputs"]]
        root = case["build"](g, *ids)
        g.set_output(root)
        opt = ref.optimize(g.graph)
    nodes = refbafe.graph_nodes(opt)
    input_ids = [opt.inputs[i] for i in range(opt.n_inputs)]
    oroot = opt.outputs[0]
    fn = ref.compile(opt)
    call = [arrays[nodes[i]["name"]] for i in input_ids]
    rn = nodes[oroot]
    out = np.zeros(tuple(rn["shape"]), NPDT[rn["dtype"]])
    ref.call_kernel(fn, call, out, stack_bytes=refbafe.stack_bytes_for(nodes))
    meta = {
        "name": case["name"], "cite": case["cite"], "nodes": nodes, "input_ids": input_ids, "root": oroot,
        "inputs": [{"name": s[0], "shape": list(s[1]), "dtype": s[2], "fortran": s[3], "layout": s[4],
                    "spec": s[5]} for s in case["inputs"]],
        "fuse": list(case["fuse"]) if case.get("fuse") else None, "fuse_na": case.get("na"),
        "panel": list(panel) if panel else None, "panel_inputs": list(case.get("panel_inputs", ())),
        "reference_graph_hash": ref.hash(opt), "ops": [n["op"] for n in nodes if not n["is_input"]],
    }
    save = {"meta": np.array(json.dumps(meta)), "out": out}
    if case.get("store_inputs", True):
        for k, v in arrays.items():
            save[f"in_{k}"] = v
    np.savez_compressed(HERE / f"{case['name']}.npz", **save)
    print(f"{case['name']:28s} ops={meta['ops']} out={out.shape} {time.time() - t0:.1f}s", flush=True)


def fused_graph(ref: refbafe.Reference, case: dict, arrays: dict):
    """The graph the reference's FusedFunction compiles (__init__.py:844-885):
    f and g each optimized on their own (g traced on an input shaped like
    f's output), concatenated by bafe_fuse_concat, optimized again."""
    specs = case["inputs"]
    na = case["na"]
    ga = GraphBuilder()
    ids_a = [ga.add_input(s[0], arrays[s[0]].shape, DT[s[2]], s[4]) for s in specs[:na]]
    root_a = case["build_a"](ga, *ids_a)
    ga.set_output(root_a)
    gb = GraphBuilder()
    x = gb.add_input("X", ga.shape(root_a), ga.dtype(root_a), 0)
    ids_b = [gb.add_input(s[0], arrays[s[0]].shape, DT[s[2]], s[4]) for s in specs[na:]]
    gb.set_output(case["build_b"](gb, x, *ids_b))
    cat = ref.fuse_concat(ref.optimize(ga.graph), ref.optimize(gb.graph))
    return ref.optimize(cat)


def main() -> None:
    if not refbafe.build():
        raise SystemExit("reference library not built and BAFE_REF_SRC (the reference's bafe/ directory) not set")
    want = set(sys.argv[1:])
    with tempfile.TemporaryDirectory() as d:
        ref = refbafe.Reference(cache_dir=d)
        cache: dict = {}
        for case in CASES:
            if want and case["name"] not in want:
                continue
            run_case(ref, case, cache)


if __name__ == "__main__":
    main()
