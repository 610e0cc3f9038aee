"""The backend behind the reference's own entry points.

oracle/_ref/libbafe_dropin.so is the reference library compiled from its
unmodified sources with the one-line backend dispatch in front of
bafe_jit_get_or_compile (oracle/dropin_shim.c; `make -C oracle dropin`).
These tests build graphs with the reference's graph API
(bafe_graph_add_input_with_layout / bafe_graph_add / bafe_graph_set_output,
ir.h:56-107), compile them with the reference's bafe_optimize_and_compile
(bafe.c:260-268) or bafe_fuse_compile (fuse.c:109-125), and call the
returned function as scripts/test_smoke.c:34-60 does: host pointers in the
optimized graph's input order, then a zeroed output.

Without BAFE_BACKEND the reference's C99 emitter answers (CPU test); with
BAFE_BACKEND=cuda the same calls return the B200 backend's host function
(GPU tests).  Both must reproduce the reference's golden outputs.
"""
import ctypes
import os
from ctypes import c_char_p, c_int, c_size_t, c_void_p
from pathlib import Path

import numpy as np
import pytest

import cases
from oracle import refgraph

ROOT = Path(__file__).resolve().parent.parent
DROPIN = ROOT / "oracle" / "_ref" / "libbafe_dropin.so"

needs_dropin = pytest.mark.skipif(not DROPIN.exists(), reason="oracle/_ref/libbafe_dropin.so not built "
                                  "(make -C oracle dropin REF_SRC=<reference>/bafe)")


def _lib():
    lib = ctypes.CDLL(str(DROPIN))
    lib.bafe_optimize_and_compile.argtypes = [c_void_p, c_char_p, c_size_t]
    lib.bafe_optimize_and_compile.restype = c_void_p
    lib.bafe_optimize.argtypes = [c_void_p, c_void_p, c_char_p, c_size_t]
    lib.bafe_optimize.restype = c_int
    lib.bafe_fuse_compile.argtypes = [c_void_p, c_void_p, c_char_p, c_size_t]
    lib.bafe_fuse_compile.restype = c_void_p
    lib.bafe_jit_set_cache_dir.argtypes = [c_char_p]
    return lib


class _RefBuilder:
    """The case builders' g.add(op, children[, perm]) over the reference's
    own graph API."""

    def __init__(self, lib):
        self.b = refgraph.Builder(lib)

    def add(self, op, children, perm=None):
        return self.b.add(op, children, perm=perm)


def _case_arrays(name):
    meta, stored, golden = cases.load(name)
    arrays = {}
    for spec in meta["inputs"]:
        if spec["name"] in stored:
            arrays[spec["name"]] = stored[spec["name"]]
        else:
            t = (spec["name"], tuple(spec["shape"]), spec["dtype"], spec["fortran"], spec["layout"], spec["spec"])
            arrays[spec["name"]] = cases.make_input(t)
    return meta, arrays, golden


def _call(fn, meta, arrays, golden):
    """Call a returned kernel the way the reference's callers do."""
    names = [meta["nodes"][i]["name"] for i in meta["input_ids"]]
    ins = [arrays[n] for n in names]
    out = np.zeros(golden.shape, golden.dtype)
    sig = ctypes.CFUNCTYPE(None, *([c_void_p] * (len(ins) + 1)))
    sig(fn)(*[c_void_p(a.ctypes.data) for a in ins], c_void_p(out.ctypes.data))
    return out


def _optimize_and_compile(lib, name):
    c = cases.CASE_BY_NAME[name]
    meta, arrays, golden = _case_arrays(name)
    g = _RefBuilder(lib)
    ids = [g.b.input(s[0], arrays[s[0]].shape, s[2], s[4]) for s in c["inputs"]]
    g.b.output(c["build"](g, *ids))
    err = ctypes.create_string_buffer(512)
    fn = lib.bafe_optimize_and_compile(ctypes.addressof(g.b.graph), err, len(err))
    assert fn, err.value.decode()
    return fn, meta, arrays, golden


def _fuse_compile(lib, name):
    """FusedFunction's graphs (__init__.py:844-885): f and g optimized apart,
    g's first input shaped like f's output; bafe_fuse_compile concatenates,
    optimizes and compiles."""
    c = cases.CASE_BY_NAME[name]
    meta, arrays, golden = _case_arrays(name)
    specs, na = c["inputs"], c["na"]
    ga = _RefBuilder(lib)
    ids_a = [ga.b.input(s[0], arrays[s[0]].shape, s[2], s[4]) for s in specs[:na]]
    root_a = c["build_a"](ga, *ids_a)
    ga.b.output(root_a)
    rn = ga.b.graph.nodes[root_a]
    f_shape = tuple(rn.shape.dims[d] for d in range(rn.shape.rank))
    gb = _RefBuilder(lib)
    x = gb.b.input("X", f_shape, "float32", 0)
    ids_b = [gb.b.input(s[0], arrays[s[0]].shape, s[2], s[4]) for s in specs[na:]]
    gb.b.output(c["build_b"](gb, x, *ids_b))
    err = ctypes.create_string_buffer(512)
    opt = []
    for b in (ga, gb):
        o = refgraph.Graph()
        assert lib.bafe_optimize(ctypes.addressof(b.b.graph), ctypes.addressof(o), err, len(err)) == 0, err.value
        opt.append(o)
    fn = lib.bafe_fuse_compile(ctypes.addressof(opt[0]), ctypes.addressof(opt[1]), err, len(err))
    assert fn, err.value.decode()
    return fn, meta, arrays, golden


@pytest.fixture
def backend(monkeypatch, tmp_path):
    """Selects the dispatch target for one test; the reference's JIT cache
    goes to a scratch directory."""
    lib = _lib()
    lib.bafe_jit_set_cache_dir(str(tmp_path).encode())

    def select(name):
        if name is None:
            monkeypatch.delenv("BAFE_BACKEND", raising=False)
        else:
            monkeypatch.setenv("BAFE_BACKEND", name)
        return lib
    return select


@needs_dropin
def test_dropin_exports_the_reference_api_and_the_dispatch():
    lib = ctypes.CDLL(str(DROPIN))
    for sym in ("bafe_optimize_and_compile", "bafe_optimize_and_compile_with_budget", "bafe_fuse_compile",
                "bafe_jit_get_or_compile", "bafe_jit_get_or_compile_c99", "bafe_graph_init", "bafe_optimize"):
        assert hasattr(lib, sym), sym


@needs_dropin
@pytest.mark.parametrize("name", ["cfg1_seed0", "e2e_matmul_bias", "transpose_64x48"])
def test_reference_route_without_backend_variable(backend, name):
    """BAFE_BACKEND unset: the dispatch keeps the reference's own emitter,
    which reproduces its golden bit for bit (its C compiler runs here)."""
    lib = backend(None)
    fn, meta, arrays, golden = _optimize_and_compile(lib, name)
    out = _call(fn, meta, arrays, golden)
    assert out.tobytes() == np.ascontiguousarray(golden).tobytes()


GPU_EXACT = ["cfg1_seed0", "e2e_matmul_bias", "e2e_relu_matmul_bias", "layout_col_b", "transpose_64x48",
             "ew_special_values", "batched_matmul_relu_3d", "f16_matmul_bias_relu", "bf16_matmul_bias_relu",
             "smoke_c_pattern"]


@needs_dropin
@pytest.mark.gpu
@pytest.mark.parametrize("name", GPU_EXACT)
def test_optimize_and_compile_routes_to_b200(backend, cuda, name):
    """BAFE_BACKEND=cuda: bafe_optimize_and_compile returns the B200
    backend's host function; in `exact` GEMM precision it is bit-exact to
    the reference's golden output."""
    import bafe_b200 as bafe
    lib = backend("cuda")
    bafe.set_option("gemm_precision", "exact")
    try:
        before = bafe.launch_count()
        fn, meta, arrays, golden = _optimize_and_compile(lib, name)
        out = _call(fn, meta, arrays, golden)
        assert bafe.launch_count() > before, "the call launched no kernel of the backend"
    finally:
        bafe.set_option("gemm_precision", "auto")
    assert out.tobytes() == np.ascontiguousarray(golden).tobytes()


@needs_dropin
@pytest.mark.gpu
@pytest.mark.parametrize("name", ["cfg2_row_col", "cfg2_row_row"])
def test_optimize_and_compile_tensor_core_plan(backend, cuda, name):
    """The 256^3 configurations through the reference's entry point on the
    3xTF32 tensor-core plan (forced: at 256^3 the default is the bit-exact
    CUDA-core kernel), within 1e-4*sqrt(K/64)*rms(A)*rms(B)."""
    import bafe_b200 as bafe
    lib = backend("cuda")
    bafe.set_option("gemm_precision", "3xtf32")
    try:
        before = bafe.launch_count()
        fn, meta, arrays, golden = _optimize_and_compile(lib, name)
        out = _call(fn, meta, arrays, golden)
        assert bafe.launch_count() > before
    finally:
        bafe.set_option("gemm_precision", "auto")
    A, B = arrays["A"].astype(np.float64), arrays["B"].astype(np.float64)
    bound = 1e-4 * np.sqrt(A.shape[1] / 64) * np.sqrt(np.mean(A * A)) * np.sqrt(np.mean(B * B))
    err = float(np.abs(out.astype(np.float64) - golden).max())
    print(f"{name} via bafe_optimize_and_compile: max |err| {err:.3e} (bound {bound:.3e})")
    assert err <= bound


@needs_dropin
@pytest.mark.gpu
@pytest.mark.parametrize("name", ["fuse_two_matmuls", "fuse_matmul_then_add_bias"])
def test_fuse_compile_routes_to_b200(backend, cuda, name):
    """bafe_fuse_compile (fuse.c:109-125) with BAFE_BACKEND=cuda: the fused
    graph compiles on the B200 backend and is bit-exact to the reference's
    fused output."""
    import bafe_b200 as bafe
    lib = backend("cuda")
    bafe.set_option("gemm_precision", "exact")
    try:
        fn, meta, arrays, golden = _fuse_compile(lib, name)
        out = _call(fn, meta, arrays, golden)
    finally:
        bafe.set_option("gemm_precision", "auto")
    assert out.tobytes() == np.ascontiguousarray(golden).tobytes()


# ---- the reference's own Python front end -------------------------------
# baseline/_ref holds the reference's Python package, installed unmodified
# (pip install --target baseline/_ref from a copy of the reference).  Its
# binding loads the library named by $BAFE_LIB -- here the drop-in library
# -- and its JittedFunction / FusedFunction compile through
# bafe_jit_get_or_compile (__init__.py:509-522, 844-885) and call the
# result with numpy buffers and an np.zeros output (__init__.py:364-383).

REF_PY = ROOT / "baseline" / "_ref"
needs_ref_py = pytest.mark.skipif(not (REF_PY / "bafe" / "__init__.py").exists() or not DROPIN.exists(),
                                  reason="the reference's Python package is not installed in baseline/_ref")


@pytest.fixture
def ref_bafe(monkeypatch, tmp_path):
    """The reference's `bafe` module bound to the drop-in library; returns
    (module, select), select(name) setting BAFE_BACKEND for the next compile."""
    import importlib
    import sys
    monkeypatch.setenv("BAFE_LIB", str(DROPIN))
    monkeypatch.setenv("BAFE_CACHE_DIR", str(tmp_path))
    if str(REF_PY) not in sys.path:
        sys.path.insert(0, str(REF_PY))
    mod = importlib.import_module("bafe")
    assert Path(mod.__file__).resolve().is_relative_to(REF_PY.resolve()), mod.__file__

    def select(name):
        if name is None:
            monkeypatch.delenv("BAFE_BACKEND", raising=False)
        else:
            monkeypatch.setenv("BAFE_BACKEND", name)
    return mod, select


def _reference_front_end_cases(bafe):
    """(golden name, jitted callable, its arguments) -- the reference's own
    front end: @bafe.jit (test_e2e.py:61) and bafe.fuse (test_fuse.py:54)."""
    @bafe.jit
    def relu_mm_plus_c(A, B, C):
        return bafe.relu(bafe.matmul(A, B) + C)

    @bafe.jit
    def mm(A, B):
        return bafe.matmul(A, B)

    @bafe.jit
    def relu_add(X, bias):
        return bafe.relu(X + bias)

    out = []
    meta, stored, golden = cases.load("e2e_relu_matmul_plus_c")
    out.append(("e2e_relu_matmul_plus_c", relu_mm_plus_c, [stored[n] for n in "ABC"], golden))
    meta, stored, golden = cases.load("fuse_matmul_then_add_bias")
    out.append(("fuse_matmul_then_add_bias", bafe.fuse(mm, relu_add), [stored["A"], stored["B"], stored["bias"]], golden))
    return out


@needs_ref_py
def test_reference_python_front_end_on_its_own_emitter(ref_bafe):
    """BAFE_BACKEND unset: the reference's Python package over the drop-in
    library still runs the C99 emitter and reproduces the goldens."""
    bafe, select = ref_bafe
    select(None)
    for name, fn, args, golden in _reference_front_end_cases(bafe):
        out = fn(*args)
        assert np.asarray(out).tobytes() == np.ascontiguousarray(golden).tobytes(), name


@needs_ref_py
@pytest.mark.gpu
def test_reference_python_front_end_on_b200(ref_bafe, cuda):
    """BAFE_BACKEND=cuda: the reference's @bafe.jit and bafe.fuse compile
    onto this backend and, in `exact` GEMM precision, reproduce the goldens
    bit for bit."""
    import bafe_b200
    bafe, select = ref_bafe
    select("cuda")
    bafe_b200.set_option("gemm_precision", "exact")
    try:
        for name, fn, args, golden in _reference_front_end_cases(bafe):
            before = bafe_b200.launch_count()
            out = fn(*args)
            assert bafe_b200.launch_count() > before, f"{name}: no kernel of the backend ran"
            assert np.asarray(out).tobytes() == np.ascontiguousarray(golden).tobytes(), name
    finally:
        bafe_b200.set_option("gemm_precision", "auto")
