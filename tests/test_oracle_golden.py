"""Pins the CPU oracle (oracle/bafe_oracle.c) to the reference's own outputs.

Every golden fixture holds the graph the reference's optimizer produced and
the output its generated C kernel computed on seeded inputs
(tests/golden/make_golden.py).  The oracle must reproduce every output bit
for bit -- including the half-precision conversions, sigmoid/tanh (same
libm) and the NaN / -0 / inf edge values.
"""
import numpy as np
import pytest

import cases
from oracle import oracle

SMALL = [c["name"] for c in cases.CASES if not c.get("panel") and c["name"] != "cfg4_chunk"]
PANELS = [c["name"] for c in cases.CASES if c.get("panel")]


def _inputs(meta, stored):
    arrays = {}
    for spec in meta["inputs"]:
        if spec["name"] in stored:
            arrays[spec["name"]] = stored[spec["name"]]
        else:
            t = (spec["name"], tuple(spec["shape"]), spec["dtype"], spec["fortran"], spec["layout"], spec["spec"])
            if meta["panel"] and spec["name"] in meta["panel_inputs"]:
                r0, r1 = meta["panel"]
                a = np.ascontiguousarray(cases.make_input(t, rows=r1)[r0:r1])
            else:
                a = cases.make_input(t)
            arrays[spec["name"]] = a
    return arrays


def _check(name):
    meta, stored, golden = cases.load(name)
    arrays = _inputs(meta, stored)
    nodes = meta["nodes"]
    by_id = {i: arrays[nodes[i]["name"]] for i in meta["input_ids"]}
    got = oracle.evaluate(nodes, by_id, meta["root"])
    want = np.ascontiguousarray(golden).reshape(-1)
    assert got.shape == want.shape
    assert got.view(np.uint8).tobytes() == want.view(np.uint8).tobytes(), (
        f"{name}: oracle differs from the reference on "
        f"{int(np.sum(got.view(np.uint8) != want.view(np.uint8)))} bytes")


@pytest.mark.parametrize("name", SMALL)
def test_oracle_matches_reference(name):
    _check(name)


def test_oracle_matches_reference_cfg4_chunk():
    _check("cfg4_chunk")


@pytest.mark.parametrize("name", PANELS)
def test_oracle_matches_reference_row_panels(name):
    _check(name)


def test_row_panel_equals_full_rows():
    """The property the large goldens rely on: a row panel of the chunked
    matmul is bit-identical to the same rows of the full product."""
    rng = np.random.default_rng(5)
    A = rng.standard_normal((96, 80), dtype=np.float32)
    B = rng.standard_normal((80, 72), dtype=np.float32)
    full = oracle.matmul(A.reshape(-1), B.reshape(-1), 1, 96, 72, 80, False, False, oracle.F32, False, 0, 0)
    full = full.reshape(96, 72)
    for r0, r1 in ((0, 5), (33, 40), (90, 96)):
        panel = oracle.matmul_panel_f32(A, B, 96, 72, 80, False, False, r0, r1)
        assert panel.tobytes() == full[r0:r1].tobytes()


def test_transpose_nd_restatement_for_self_inverse_perms():
    """The emitter's rank-N transpose index is right for self-inverse
    permutations; there it equals the true transpose the oracle uses."""
    x = np.arange(2 * 3 * 4, dtype=np.float32).reshape(2, 3, 4)
    for perm in ((2, 1, 0), (0, 2, 1), (1, 0, 2)):
        out_dims = [x.shape[p] for p in perm]
        got = oracle.transpose_nd_reference(x.reshape(-1), list(x.shape), out_dims, list(perm))
        assert got.tobytes() == np.ascontiguousarray(np.transpose(x, perm)).tobytes()


def test_relu_edge_semantics():
    """relu as emitted: NaN -> +0, -0 -> +0 (codegen.c:338-344)."""
    x = np.array([np.nan, -0.0, 0.0, -1.0, 2.0, np.inf, -np.inf], np.float32)
    y = oracle.unary("relu", x, oracle.F32, oracle.F32)
    assert y.tobytes() == np.array([0, 0, 0, 0, 2, np.inf, 0], np.float32).tobytes()
