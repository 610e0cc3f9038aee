"""The C ABI: library loads, exports every declared symbol, struct layouts
match BAFE's graph ABI, graph hashes match the reference's.  CPU only."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

import bafe_b200
import cases
from bafe_b200 import _binding
from bafe_b200.graph import GraphBuilder
from conftest import gpu_available
from oracle import refbafe

ROOT = Path(__file__).resolve().parent.parent


def declared_functions():
    text = (ROOT / "include" / "bafe_cuda.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(bafe_cuda_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_binding.library_path())
    names = declared_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/bafe_cuda.h but not exported"
    assert set(names) == set(_binding.EXPORTED_SYMBOLS)


def test_library_exports_only_the_c_abi():
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", _binding.library_path()], capture_output=True,
                         text=True, check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    ours = {s for s in exported if s.startswith("bafe_")}
    assert ours == set(declared_functions())


def test_struct_layouts_match_library():
    lib = _binding.lib
    assert lib.bafe_cuda_abi_size(0) == ctypes.sizeof(_binding.BafeGraph)
    assert lib.bafe_cuda_abi_size(1) == ctypes.sizeof(_binding.BafeNode)
    assert lib.bafe_cuda_abi_size(2) == ctypes.sizeof(_binding.BafeOpAttrs)
    assert lib.bafe_cuda_abi_size(3) == ctypes.sizeof(_binding.BafeShape)


@pytest.mark.skipif(not refbafe.available(), reason="reference library not built here")
@pytest.mark.parametrize("name", ["cfg1_seed0", "cfg3_panel_top", "layout_col_b", "f16_matmul_bias_relu",
                                  "batched_matmul_relu_3d", "transpose_then_relu"])
def test_graph_hash_matches_reference(name):
    """bafe_cuda_jit_hash_graph == the reference's bafe_jit_hash_graph (jit.c:131-154)."""
    meta, _, _ = cases.load(name)
    g = cases.graph_from_nodes(meta["nodes"], meta["input_ids"], meta["root"])
    ref = refbafe.Reference()
    assert bafe_b200.graph_hash(g) == ref.hash(g) == meta["reference_graph_hash"]


@pytest.mark.skipif(not refbafe.available(), reason="reference library not built here")
def test_graph_builder_matches_reference_builder():
    """GraphBuilder builds the struct BAFE's own bafe_graph_add builds (same hash)."""
    ref = refbafe.Reference()
    L = ref.lib
    G = ctypes.POINTER(_binding.BafeGraph)
    L.bafe_graph_init.argtypes = [G]
    L.bafe_graph_add_input_with_layout.argtypes = [G, ctypes.c_char_p, ctypes.POINTER(_binding.BafeShape),
                                                   ctypes.c_int, ctypes.c_int]
    L.bafe_graph_add.argtypes = [G, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int32), ctypes.c_int, ctypes.c_void_p]
    L.bafe_graph_set_output.argtypes = [G, ctypes.c_int32]

    def shp(*d):
        s = _binding.BafeShape()
        s.rank = len(d)
        for i, v in enumerate(d):
            s.dims[i] = v
        return s

    rg = _binding.BafeGraph()
    L.bafe_graph_init(ctypes.byref(rg))
    a = L.bafe_graph_add_input_with_layout(ctypes.byref(rg), b"A", ctypes.byref(shp(64, 32)), 0, 0)
    b = L.bafe_graph_add_input_with_layout(ctypes.byref(rg), b"B", ctypes.byref(shp(32, 48)), 0, 1)
    c = L.bafe_graph_add_input_with_layout(ctypes.byref(rg), b"C", ctypes.byref(shp(48,)), 0, 0)
    mm = L.bafe_graph_add(ctypes.byref(rg), b"matmul", (ctypes.c_int32 * 2)(a, b), 2, None)
    ad = L.bafe_graph_add(ctypes.byref(rg), b"add", (ctypes.c_int32 * 2)(mm, c), 2, None)
    r = L.bafe_graph_add(ctypes.byref(rg), b"relu", (ctypes.c_int32 * 1)(ad), 1, None)
    L.bafe_graph_set_output(ctypes.byref(rg), r)

    g = GraphBuilder()
    a2 = g.add_input("A", (64, 32), 0, 0)
    b2 = g.add_input("B", (32, 48), 0, 1)
    c2 = g.add_input("C", (48,), 0, 0)
    g.set_output(g.add("relu", [g.add("add", [g.add("matmul", [a2, b2]), c2])]))
    assert bafe_b200.graph_hash(g.graph) == ref.hash(rg)


def test_cache_dir_follows_environment(tmp_path):
    import os
    assert bafe_b200.cache_dir() == os.environ["BAFE_CACHE_DIR"]


def test_options_roundtrip():
    for v in ("exact", "tf32", "3xtf32", "auto"):
        bafe_b200.set_option("gemm_precision", v)
        assert bafe_b200.get_option("gemm_precision") == v
    with pytest.raises(ValueError):
        bafe_b200.set_option("gemm_precision", "fp8")
    with pytest.raises(ValueError):
        bafe_b200.set_option("nonsense", "1")


@pytest.mark.parametrize("n", [3, 20, 64])
def test_host_function_reaches_its_plan_without_a_gpu(n):
    """The returned function (17-pointer bank up to 16 inputs, 65-pointer
    bank above) runs the plan of its own slot: on a machine without a GPU the
    call records "no CUDA device" instead of failing silently or crashing."""
    if gpu_available():
        pytest.skip("covered by the GPU parity tests on a machine with a GPU")
    import bafe_b200 as bafe
    import numpy as np
    g = GraphBuilder()
    ids = [g.add_input(f"X{i}", (64,), 0, 0) for i in range(n)]
    root = ids[0]
    for i in ids[1:]:
        root = g.add("add", [root, i])
    g.set_output(root)
    k = bafe.compile_graph(g)
    xs = [np.ones(64, np.float32) for _ in range(n)]
    with pytest.raises(RuntimeError, match="no CUDA device"):
        k(*xs)


@pytest.mark.parametrize("M,N,K", [(1 << 31, 1 << 31, 1 << 31), (1 << 40, 4, 1 << 24), (4, 1 << 62, 2),
                                   (4096, 4096, 4096)])
def test_static_scratch_rejects_oversize_before_touching_the_device(M, N, K):
    """The allocation-free GEMM compares element counts with its fixed
    scratch capacity before forming any byte count, so sizes whose products
    would wrap a 64-bit integer are refused too; nothing reaches the device
    (the pointers here are never dereferenced)."""
    fake = ctypes.c_void_p(256)
    rc = _binding.lib.bafe_cuda_gemm_3xtf32_static_scratch(fake, fake, fake, M, N, K, 0, 0, None)
    assert rc == 15
    assert "static scratch" in _binding.last_error()[1]
