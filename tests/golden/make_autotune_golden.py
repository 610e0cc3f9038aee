"""Generates tests/golden/autotune_golden.json by running the reference itself.

The backend restates BAFE's profiling layer (profiling.c: feature vector,
log, JSONL dump, least-squares refit, prediction) so that records and
learned models are interchangeable.  This script pins that restatement to
the reference's own library (oracle/_ref/libbafe.so, built from the
reference sources by `make -C oracle ref`):

  features: bafe_profiling_extract_features of every golden case's graph,
            as traced and as the reference's optimizer returned it (stored
            as float.hex so the comparison is bit for bit);
  refit:    seeded synthetic logs (a planted linear model with noise, the
            reference's own quadratic example, a log with constant and
            all-zero feature columns, a log with non-positive times) fed to
            bafe_profiling_add, then bafe_profiling_refit, the learned model
            and bafe_profiling_predict_log on probe vectors;
  jsonl:    bafe_profiling_dump_jsonl of two fixed records.

Runs in this container only (the GPU host has no reference).
Usage: python tests/golden/make_autotune_golden.py
"""
from __future__ import annotations

import ctypes
import json
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(ROOT / "bafe-basic-algibra-fusion-engine-_b200"))
sys.path.insert(0, str(ROOT))

import cases  # noqa: E402
from cases import CASES, graph_from_nodes, load  # noqa: E402
from bafe_b200 import _binding  # noqa: E402
from bafe_b200.graph import GraphBuilder  # noqa: E402
from oracle import refbafe  # noqa: E402

NF = 8
DT = {"float32": 0, "float64": 1, "int32": 2, "int64": 3, "float16": 4, "bfloat16": 5}


def ref_lib():
    refbafe.build()
    lib = ctypes.CDLL(str(refbafe.REF_LIB))
    G = ctypes.POINTER(_binding.BafeGraph)
    D = ctypes.POINTER(ctypes.c_double)
    lib.bafe_profiling_reset.argtypes = []
    lib.bafe_profiling_extract_features.argtypes = [G, D]
    lib.bafe_profiling_add.argtypes = [ctypes.c_char_p, D, ctypes.c_double, ctypes.c_double, ctypes.c_int]
    lib.bafe_profiling_refit.restype = ctypes.c_int
    lib.bafe_profiling_get_model.restype = ctypes.POINTER(_binding.BafeLearnedCostModel)
    lib.bafe_profiling_predict_log.argtypes = [D]
    lib.bafe_profiling_predict_log.restype = ctypes.c_double
    lib.bafe_profiling_dump_jsonl.argtypes = [ctypes.c_char_p]
    lib.bafe_profiling_dump_jsonl.restype = ctypes.c_int
    return lib


def feats(lib, g) -> list:
    f = (ctypes.c_double * NF)()
    lib.bafe_profiling_extract_features(ctypes.byref(g), f)
    return [float(v).hex() for v in f]


def traced_graph(case) -> GraphBuilder:
    """The case's graph as traced (cases.traced_graph)."""
    return cases.traced_graph(case)


def refit_logs():
    rng = np.random.default_rng(2024)
    logs = {}
    # a planted model with noise over varied features
    X = np.column_stack([rng.integers(1, 5, 60), rng.integers(1, 9, 60), rng.integers(0, 3, 60),
                         rng.integers(0, 2, 60), rng.uniform(5, 40, 60), rng.uniform(5, 30, 60),
                         rng.integers(0, 6, 60), rng.integers(0, 2, 60)]).astype(np.float64)
    w = np.array([0.05, 0.1, 0.3, -0.2, 0.4, 0.25, 0.05, 0.1])
    y = X @ w - 9.0 + rng.normal(0, 0.05, 60)
    logs["planted"] = [(list(map(float, x)), float(np.exp(v))) for x, v in zip(X, y)]
    # the reference's own example: feature 4 = i+1, runtime 0.01 (i+1)^2
    logs["quadratic"] = [([0, 0, 0, 0, float(i + 1), 0, 0, 0], 0.01 * (i + 1) ** 2) for i in range(20)]
    # constant / all-zero columns (singular normal equations)
    logs["singular"] = [([2.0, 3.0, 1.0, 0.0, float(i), float(2 * i), 0.0, 1.0], 0.5 + 0.1 * i) for i in range(12)]
    # non-positive observations are skipped by the fit
    logs["skips"] = [([1.0, 1.0, 0.0, 0.0, float(i), 3.0, 1.0, 0.0], (0.2 * i if i % 3 else 0.0)) for i in range(15)]
    return logs


def main():
    lib = ref_lib()
    out = {"features": {}, "refit": {}, "jsonl": ""}
    for case in CASES:
        meta, _, _ = load(case["name"])
        g_opt = graph_from_nodes(meta["nodes"], meta["input_ids"], meta["root"])
        out["features"][case["name"]] = {"traced": feats(lib, traced_graph(case).graph),
                                         "optimized": feats(lib, g_opt)}
    probes = [[1, 2, 1, 0, 10, 12, 2, 0], [3, 5, 0, 1, 25, 20, 4, 1], [0] * 8]
    for name, log in refit_logs().items():
        lib.bafe_profiling_reset()
        for k, (f, ms) in enumerate(log):
            fa = (ctypes.c_double * NF)(*f)
            lib.bafe_profiling_add(b"h%03d" % k, fa, 1.0, ms, k)
        rc = lib.bafe_profiling_refit()
        m = lib.bafe_profiling_get_model().contents
        preds = [float(lib.bafe_profiling_predict_log((ctypes.c_double * NF)(*p))).hex() for p in probes]
        out["refit"][name] = {
            "records": [[f, float(ms).hex()] for f, ms in log], "rc": rc,
            "weights": [float(m.weights[i]).hex() for i in range(NF)], "bias": float(m.bias).hex(),
            "r_squared": float(m.r_squared).hex(), "n_samples": m.n_samples, "valid": bool(m.valid),
            "probes": probes, "predict_log": preds,
        }
    lib.bafe_profiling_reset()
    f1 = (ctypes.c_double * NF)(*([1.5] * NF))
    f2 = (ctypes.c_double * NF)(*[0.125 * i for i in range(NF)])
    lib.bafe_profiling_add(b"deadbeefdeadbeefdeadbeef", f1, 3.0, 0.5, 0)
    lib.bafe_profiling_add(b"cafef00d", f2, 4.25, 1e-3, 7)
    with tempfile.TemporaryDirectory() as d:
        p = Path(d) / "log.jsonl"
        lib.bafe_profiling_dump_jsonl(str(p).encode())
        out["jsonl"] = p.read_text()
    lib.bafe_profiling_reset()
    (HERE / "autotune_golden.json").write_text(json.dumps(out, indent=0, sort_keys=True) + "\n")
    print(f"wrote {HERE / 'autotune_golden.json'}: {len(out['features'])} graphs, {len(out['refit'])} logs")


if __name__ == "__main__":
    main()
