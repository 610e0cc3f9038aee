"""Host-side lowering: which kernels a graph becomes, compile of every
generated module (NVRTC, sm_100a) and the JIT-cache contract.  CPU only:
plans are built and compiled without a GPU."""
import numpy as np
import pytest

import bafe_b200 as bafe
import cases
from conftest import gpu_available
from bafe_b200.graph import GraphBuilder


def _kernel(build, *inputs):
    g = GraphBuilder()
    ids = [g.add_input(n, s, dt, lay) for (n, s, dt, lay) in inputs]
    g.set_output(build(g, *ids))
    return bafe.compile_graph(g)


def test_cfg1_is_one_fused_gemm():
    k = _kernel(lambda g, A, B, C: g.add("relu", [g.add("add", [g.add("matmul", [A, B]), C])]),
                ("A", (64, 64), 0, 0), ("B", (64, 64), 0, 0), ("C", (64, 64), 0, 0))
    steps = k.describe().strip().splitlines()
    assert len(steps) == 1
    assert steps[0].startswith("gemm.") and "epi=relu(add(acc,C))" in steps[0] and steps[0].endswith("-> out")


def test_cfg3_epilogue_holds_the_product():
    k = _kernel(lambda g, A, B, C, D: g.add("relu", [g.add("add", [g.add("matmul", [A, B]), g.add("mul", [C, D])])]),
                ("A", (128, 64), 0, 0), ("B", (64, 96), 0, 0), ("C", (128, 96), 0, 0), ("D", (128, 96), 0, 0))
    steps = k.describe().strip().splitlines()
    assert len(steps) == 1 and "epi=relu(add(acc,mul(C,D)))" in steps[0]


def test_cfg4_is_one_streaming_kernel():
    k = _kernel(lambda g, X, Y, Z: g.add("relu", [g.add("add", [g.add("mul", [X, Y]), Z])]),
                ("X", (1 << 12,), 0, 0), ("Y", (1 << 12,), 0, 0), ("Z", (1 << 12,), 0, 0))
    steps = k.describe().strip().splitlines()
    assert steps == ["ew n=4096 float relu(add(mul(X,Y),Z)) -> out"]


def test_bias_epilogue_reads_row_vector():
    k = _kernel(lambda g, A, B, b: g.add("relu", [g.add("add", [g.add("matmul", [A, B]), b])]),
                ("A", (64, 32), 0, 0), ("B", (32, 48), 0, 0), ("b", (48,), 0, 0))
    assert "epi=relu(add(acc,b[j]))" in k.describe()


def test_transpose_materialisation_and_consumer():
    k = _kernel(lambda g, X: g.add("relu", [g.add("transpose", [X], perm=[1, 0])]), ("X", (40, 72), 0, 0))
    steps = k.describe().strip().splitlines()
    assert steps[0].startswith("transpose2d m=72 n=40") and steps[1].startswith("ew n=2880")


def test_shared_matmul_is_materialised():
    """A product read twice is computed once into a temporary."""
    k = _kernel(lambda g, A, B: (lambda m: g.add("add", [g.add("relu", [m]), g.add("neg", [m])]))(g.add("matmul", [A, B])),
                ("A", (32, 32), 0, 0), ("B", (32, 32), 0, 0))
    steps = k.describe().strip().splitlines()
    assert steps[0].startswith("gemm.") and "-> tmp0" in steps[0]
    assert steps[1].startswith("ew ") and steps[1].endswith("-> out")


def test_unsupported_broadcast_is_an_error():
    g = GraphBuilder()
    a = g.add_input("A", (4, 8), 0, 0)
    b = g.add_input("B", (1, 8), 0, 0)
    g.set_output(g.add("add", [a, b]))
    with pytest.raises(RuntimeError, match="unsupported broadcast"):
        bafe.compile_graph(g)
    assert bafe.jit_stats()["compile_failures"] == 1


def test_unknown_op_zero_fills_like_the_emitter():
    g = GraphBuilder()
    a = g.add_input("A", (4, 8), 0, 0)
    b = g.add_input("s", (1,), 0, 0)
    g.set_output(g.add("scale", [a, b]))
    k = bafe.compile_graph(g)
    assert "zero-fill" in k.describe()


def test_jit_cache_contract():
    """Same graph -> memory hit; jit_clear -> disk hit; stats like jit.c."""
    build = lambda g, X: g.add("relu", [X])
    k1 = _kernel(build, ("X", (32, 32), 0, 0))
    k2 = _kernel(build, ("X", (32, 32), 0, 0))
    assert k1.fn_ptr == k2.fn_ptr and k1.plan == k2.plan
    s = bafe.jit_stats()
    assert s["misses"] == 1 and s["hits"] >= 1
    bafe.jit_clear()
    _kernel(build, ("X", (32, 32), 0, 0))
    s = bafe.jit_stats()
    assert s == {"hits": 1, "misses": 1, "compiles": 0, "compile_failures": 0}   # cubin came from disk
    _kernel(build, ("X", (32, 33), 0, 0))
    assert bafe.jit_stats()["misses"] == 2


def test_precision_option_changes_the_plan():
    build = lambda g, A, B: g.add("matmul", [A, B])
    bafe.set_option("gemm_precision", "exact")
    k = _kernel(build, ("A", (256, 256), 0, 0), ("B", (256, 256), 0, 0))
    assert k.describe().startswith("gemm.exact")


def test_stale_function_reports_an_error():
    k = _kernel(lambda g, X: g.add("relu", [X]), ("X", (8,), 0, 0))
    bafe.jit_clear()
    x = np.ones(8, np.float32)
    with pytest.raises(RuntimeError, match="stale kernel function"):
        k(x)


@pytest.mark.skipif(gpu_available(), reason="checks the no-device error path")
def test_no_device_fails_loudly():
    k = _kernel(lambda g, X: g.add("relu", [X]), ("X", (8,), 0, 0))
    with pytest.raises(RuntimeError, match="no CUDA device"):
        k(np.ones(8, np.float32))


@pytest.mark.parametrize("name", [c["name"] for c in cases.CASES])
def test_every_golden_graph_lowers_and_compiles(name):
    """The reference-optimized graph of every golden case lowers and its
    generated module compiles for sm_100a (NVRTC) -- no GPU needed."""
    meta, _, _ = cases.load(name)
    g = cases.graph_from_nodes(meta["nodes"], meta["input_ids"], meta["root"])
    for prec in ("exact", "auto"):
        bafe.set_option("gemm_precision", prec)

        class B:  # minimal builder facade for compile_graph
            graph = g
            output = meta["root"]

            @staticmethod
            def shape(i):
                return tuple(meta["nodes"][i]["shape"])

            @staticmethod
            def dtype(i):
                return meta["nodes"][i]["dtype"]
        k = bafe.compile_graph(B)
        assert k.describe()


def test_tc_convert_option_drops_the_residual_pre_pass():
    g = GraphBuilder()
    a = g.add_input("A", (512, 512), 0, 0)
    b = g.add_input("B", (512, 512), 0, 0)
    g.set_output(g.add("matmul", [a, b]))
    bafe.set_option("gemm_precision", "3xtf32")
    default = bafe.compile_graph(g).describe().strip().splitlines()
    assert [l.split()[0] for l in default][:2] == ["ew", "ew"] and default[2].startswith("gemm.tc.3xtf32")
    assert bafe.get_option("tc_convert") == "auto"
    bafe.set_option("tc_convert", "1")
    try:
        conv = bafe.compile_graph(g).describe().strip().splitlines()
        bafe.set_option("tc_convert", "auto")
        g2 = GraphBuilder()                  # 256^3: auto keeps the pre-pass too
        a2 = g2.add_input("A", (256, 256), 0, 0)
        b2 = g2.add_input("B", (256, 256), 0, 0)
        g2.set_output(g2.add("matmul", [a2, b2]))
        small = bafe.compile_graph(g2).describe().strip().splitlines()
        bafe.set_option("gemm_precision", "auto")
        dflt = bafe.compile_graph(g2).describe().strip().splitlines()
    finally:
        bafe.set_option("tc_convert", "auto")
        bafe.set_option("gemm_precision", "auto")
    assert len(conv) == 1 and conv[0].startswith("gemm.tc.3xtf32")
    assert len(small) == 3 and small[2].startswith("gemm.tc.3xtf32")
    # default precision: an f32 GEMM of 256^3 multiply-adds runs the exact kernel
    assert len(dflt) == 1 and dflt[0].startswith("gemm.exact"), dflt


def _sum_chain(n, tree=False):
    g = GraphBuilder()
    ids = [g.add_input(f"X{i}", (1000,), 0, 0) for i in range(n)]
    if tree:
        while len(ids) > 1:
            ids = [g.add("add", [ids[i], ids[i + 1]]) for i in range(0, len(ids), 2)]
        root = ids[0]
    else:
        root = ids[0]
        for i in ids[1:]:
            root = g.add("add", [root, i])
    g.set_output(root)
    return g


def _operands(step):
    import re
    return len(set(re.findall(r"\b(?:X\d+|C\d+|%\d+)\b", step)))


@pytest.mark.parametrize("n,tree,kernels", [(20, False, 2), (40, False, 3), (32, True, 3), (64, False, 5)])
def test_wide_expressions_are_cut_into_kernels_that_fit(n, tree, kernels):
    """A region reads at most 16 operands: wider elementwise expressions are
    cut at internal nodes (each becomes a buffer, as every node is in the
    emitter), with few kernels."""
    steps = bafe.compile_graph(_sum_chain(n, tree)).describe().strip().splitlines()
    assert len(steps) == kernels, steps
    assert all(s.startswith("ew ") and _operands(s) <= 16 for s in steps), steps


def test_wide_gemm_epilogue_is_unfused():
    """A GEMM epilogue reads at most 8 operands: a wider one leaves the
    product in a buffer and runs as an elementwise region."""
    def build(n):
        g = GraphBuilder()
        r = g.add("matmul", [g.add_input("A", (64, 32), 0, 0), g.add_input("B", (32, 48), 0, 0)])
        for i in range(n):
            r = g.add("add", [r, g.add_input(f"C{i}", (64, 48), 0, 0)])
        g.set_output(g.add("relu", [r]))
        return g
    fused = bafe.compile_graph(build(7)).describe().strip().splitlines()
    assert len(fused) == 1 and "epi=relu(" in fused[0]
    split = bafe.compile_graph(build(10)).describe().strip().splitlines()
    assert len(split) == 2 and "epi=acc -> tmp0" in split[0] and split[1].startswith("ew "), split


def test_input_count_limit():
    """The returned host function takes up to 64 inputs plus out (graphs with
    more than 16 get a function of a wider bank); 65 inputs are refused."""
    k = bafe.compile_graph(_sum_chain(64))
    assert k.n_inputs == 64
    with pytest.raises(RuntimeError, match="more than 64 inputs"):
        bafe.compile_graph(_sum_chain(65))


def test_gemm_beyond_32_bit_tile_coordinates_takes_the_exact_kernel():
    """The tensor-core kernel keeps tile origins and TMA coordinates in 32
    bits: a GEMM with ~2^31 rows (the exact kernel indexes in 64 bits and
    launches in blocks of rows) is planned on the exact kernel."""
    def plan(m):
        g = GraphBuilder()
        g.set_output(g.add("matmul", [g.add_input("A", (m, 64), 0, 0), g.add_input("B", (64, 64), 0, 0)]))
        return bafe.compile_graph(g).describe().strip()
    if gpu_available():
        assert plan(1 << 20).startswith("gemm.tc")
    assert plan((1 << 31) - 100).startswith("gemm.exact")


def test_plan_steps_match_the_description():
    """bafe_cuda_plan_num_steps counts the launch steps describe() lists
    (one line each): the per-step timing events follow it."""
    g = GraphBuilder()
    a = g.add_input("A", (512, 512), 0, 0)
    b = g.add_input("B", (512, 512), 0, 2)
    c = g.add_input("C", (512, 512), 0, 0)
    g.set_output(g.add("relu", [g.add("add", [g.add("matmul", [a, b]), c])]))
    bafe.set_option("gemm_precision", "3xtf32")
    try:
        k = bafe.compile_graph(g)
    finally:
        bafe.set_option("gemm_precision", "auto")
    assert k.num_steps == len(k.describe().strip().splitlines()) == 3
    e = GraphBuilder()
    x = e.add_input("X", (1000,), 0, 0)
    e.set_output(e.add("relu", [x]))
    assert bafe.compile_graph(e).num_steps == 1
