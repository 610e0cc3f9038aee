"""Runs the reference itself -- TEST INFRASTRUCTURE ONLY.

oracle/_ref/libbafe.so is the reference compiled from its own sources by
`make -C oracle ref` (see oracle/Makefile).  This module drives its public C
API through ctypes exactly as the reference's own callers do
(bafe/python/bafe/__init__.py:440-544, scripts/test_smoke.c:31-60):
bafe_optimize -> bafe_jit_get_or_compile (which emits C, runs `cc -O3
-march=native` and dlopens it) -> call the generated kernel with host
pointers.  Graph structs are built with oracle/refgraph.py (the
reference's own graph API on a struct-only mirror of its ABI) or, in the
golden-fixture generator, with the backend's GraphBuilder, whose struct
layout is the same ABI; graph arguments are passed by address, so either
struct works.  This module itself never imports the backend.

The generated kernels keep one stack array per node (codegen.c:188), so
large problems must run on a thread with a big stack: `call_kernel` does.
Used by tests/golden/make_golden.py (golden fixtures) and by bench.py's
reference arm / cpu_baseline leg.  Never by the product.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from ctypes import c_char_p, c_int, c_size_t, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF_LIB = HERE / "_ref" / "libbafe.so"


def available() -> bool:
    return REF_LIB.exists()


def build() -> bool:
    """Build oracle/_ref/libbafe.so from the reference sources named by
    $BAFE_REF_SRC (the reference's bafe/ directory); False when neither the
    library nor the variable is there."""
    if REF_LIB.exists():
        return True
    src = os.environ.get("BAFE_REF_SRC")
    if not src or not Path(src, "src").exists():
        return False
    subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF_SRC={src}"], check=True)
    return REF_LIB.exists()


class Reference:
    def __init__(self, cache_dir: str | None = None):
        from oracle.refgraph import Graph   # struct-only mirror of the graph ABI
        self.BafeGraph = Graph
        if not REF_LIB.exists():
            raise FileNotFoundError(f"{REF_LIB} missing (make -C oracle ref REF_SRC=...)")
        self.lib = ctypes.CDLL(str(REF_LIB))
        G = c_void_p                        # graphs by address: any struct with the ABI's layout
        self.lib.bafe_optimize.argtypes = [G, G, c_char_p, c_size_t]
        self.lib.bafe_optimize.restype = c_int
        self.lib.bafe_jit_get_or_compile.argtypes = [G, c_char_p, c_size_t]
        self.lib.bafe_jit_get_or_compile.restype = c_void_p
        self.lib.bafe_jit_hash_graph.argtypes = [G, c_char_p, c_size_t]
        self.lib.bafe_jit_hash_graph.restype = c_int
        self.lib.bafe_fuse_concat.argtypes = [G, G, G, c_char_p, c_size_t]
        self.lib.bafe_fuse_concat.restype = c_int
        self.lib.bafe_jit_set_cache_dir.argtypes = [c_char_p]
        self.lib.bafe_jit_clear.argtypes = []
        if cache_dir:
            os.makedirs(cache_dir, exist_ok=True)
            self.lib.bafe_jit_set_cache_dir(cache_dir.encode())

    def optimize(self, graph) -> object:
        """bafe_optimize (bafe.c:250-258): the graph the backend receives."""
        out = self.BafeGraph()
        err = ctypes.create_string_buffer(512)
        rc = self.lib.bafe_optimize(ctypes.addressof(graph), ctypes.addressof(out), err, len(err))
        if rc != 0:
            raise RuntimeError(f"bafe_optimize failed ({rc}): {err.value.decode()}")
        return out

    def fuse_concat(self, graph_a, graph_b) -> object:
        """bafe_fuse_concat (fuse.c:12-106): graph_a's output feeds graph_b's
        first input; the inputs are graph_a's then graph_b's inputs[1:]."""
        out = self.BafeGraph()
        err = ctypes.create_string_buffer(256)
        rc = self.lib.bafe_fuse_concat(ctypes.addressof(graph_a), ctypes.addressof(graph_b),
                                       ctypes.addressof(out), err, len(err))
        if rc != 0:
            raise RuntimeError(f"bafe_fuse_concat failed ({rc}): {err.value.decode()}")
        return out

    def compile(self, graph) -> int:
        """bafe_jit_get_or_compile (jit.c:204-328) -> generated-kernel address."""
        err = ctypes.create_string_buffer(2048)
        fn = self.lib.bafe_jit_get_or_compile(ctypes.addressof(graph), err, len(err))
        if not fn:
            raise RuntimeError(f"reference JIT failed: {err.value.decode()}")
        return fn

    def hash(self, graph) -> str:
        buf = ctypes.create_string_buffer(65)
        self.lib.bafe_jit_hash_graph(ctypes.addressof(graph), buf, 65)
        return buf.value.decode()

    @staticmethod
    def call_kernel(fn: int, arrays, out: np.ndarray, stack_bytes: int = 0) -> None:
        """Call the generated kernel with host pointers (__init__.py:369-383).
        Runs on a thread whose stack holds the kernel's per-node arrays."""
        n = len(arrays)
        sig = ctypes.CFUNCTYPE(None, *([c_void_p] * (n + 1)))
        kern = sig(fn)
        ptrs = [c_void_p(a.ctypes.data) for a in arrays] + [c_void_p(out.ctypes.data)]
        if stack_bytes <= 0:
            kern(*ptrs)
            return
        err = []

        def run():
            try:
                kern(*ptrs)
            except BaseException as e:   # pragma: no cover
                err.append(e)

        old = threading.stack_size()
        threading.stack_size(int(stack_bytes))
        try:
            t = threading.Thread(target=run)
            t.start()
            t.join()
        finally:
            threading.stack_size(old)
        if err:
            raise err[0]


def graph_nodes(graph) -> list:
    """Plain-Python node list of a BafeGraph (same keys as GraphBuilder.to_list)."""
    out = []
    for i in range(graph.n_nodes):
        n = graph.nodes[i]
        out.append({
            "id": i, "op": n.op_name.decode(), "children": [n.children[k] for k in range(n.n_children)],
            "shape": [n.shape.dims[d] for d in range(n.shape.rank)], "dtype": n.dtype, "layout": n.layout,
            "name": n.input_name.decode(), "is_input": bool(n.is_input),
            "perm": [n.attrs.perm[k] for k in range(n.attrs.n_perm)],
            "axes": [n.attrs.axes[k] for k in range(n.attrs.n_axes)],
            "tshape": [n.attrs.shape[k] for k in range(n.attrs.n_shape)],
            "keepdims": bool(n.attrs.keepdims), "attr_name": n.attrs.name.decode(),
        })
    return out


def stack_bytes_for(nodes: list, margin: int = 64 << 20) -> int:
    """Stack the generated kernel needs: one array per non-input node
    (codegen.c:184-188) plus converted half inputs."""
    total = margin
    for n in nodes:
        numel = 1
        for d in n["shape"]:
            numel *= d
        if not n["is_input"]:
            total += numel * 8
        elif n["dtype"] in (4, 5):
            total += numel * 4
    return total
