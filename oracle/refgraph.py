"""Graphs for the reference library, built through the reference's own C
API -- TEST AND BASELINE INFRASTRUCTURE ONLY.

A struct-only ctypes mirror of BAFE's POD graph (the layout the reference
binds at bafe/python/bafe/_binding.py:62-112; types.h:55-58, ops.h:239-250,
ir.h:133-155) and a small builder that calls the reference's
bafe_graph_init / bafe_graph_add_input_with_layout / bafe_graph_add /
bafe_graph_set_output (ir.h:56-107), exactly as the reference's C callers
do (scripts/test_smoke.c:31-52).  Nothing here imports the B200 backend, so
a process that builds and runs reference kernels with it loads only the
reference's library (oracle/_ref/libbafe.so).
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, Structure, c_bool, c_char, c_char_p, c_double, c_int, c_int32, c_void_p

MAX_RANK = 8
MAX_ATTR_LEN = 32
MAX_CHILDREN = 4
MAX_NODES = 4096

DTYPE = {"float32": 0, "float64": 1, "int32": 2, "int64": 3, "float16": 4, "bfloat16": 5}
LAYOUT_ROW, LAYOUT_COL, LAYOUT_BLOCKED, LAYOUT_TC = range(4)


class Shape(Structure):
    _fields_ = [("dims", c_int32 * MAX_RANK), ("rank", c_int32)]


class OpAttrs(Structure):
    _fields_ = [
        ("n_axes", c_int32), ("axes", c_int32 * MAX_ATTR_LEN),
        ("n_perm", c_int32), ("perm", c_int32 * MAX_ATTR_LEN),
        ("n_shape", c_int32), ("shape", c_int32 * MAX_ATTR_LEN),
        ("keepdims", c_bool), ("scalar_value", c_double), ("has_scalar", c_bool),
        ("name", c_char * MAX_ATTR_LEN),
    ]


class Node(Structure):
    _fields_ = [
        ("id", c_int32), ("op_name", c_char_p), ("attrs", OpAttrs),
        ("n_children", c_int), ("children", c_int32 * MAX_CHILDREN),
        ("shape", Shape), ("dtype", c_int), ("layout", c_int),
        ("input_name", c_char * MAX_ATTR_LEN), ("is_input", c_bool),
        ("is_constant", c_bool), ("const_value", c_double),
    ]


class Graph(Structure):
    _fields_ = [
        ("nodes", Node * MAX_NODES), ("n_nodes", c_int),
        ("inputs", c_int32 * MAX_NODES), ("n_inputs", c_int),
        ("outputs", c_int32 * MAX_NODES), ("n_outputs", c_int),
    ]


def _shape(dims) -> Shape:
    s = Shape()
    s.rank = len(dims)
    for i, v in enumerate(dims):
        s.dims[i] = int(v)
    return s


class Builder:
    """Builds a bafe_graph with the reference library's own graph API.

    `lib` is the reference's libbafe.so (a ctypes.CDLL).  Node ids are the
    int32 ids bafe_graph_add returns; a negative id is the library's error.
    """

    def __init__(self, lib):
        self.lib = lib
        G = POINTER(Graph)
        lib.bafe_graph_init.argtypes = [G]
        lib.bafe_graph_init.restype = None
        lib.bafe_graph_add_input_with_layout.argtypes = [G, c_char_p, POINTER(Shape), c_int, c_int]
        lib.bafe_graph_add_input_with_layout.restype = c_int32
        lib.bafe_graph_add.argtypes = [G, c_char_p, POINTER(c_int32), c_int, c_void_p]
        lib.bafe_graph_add.restype = c_int32
        lib.bafe_graph_set_output.argtypes = [G, c_int32]
        lib.bafe_graph_set_output.restype = None
        self.graph = Graph()
        lib.bafe_graph_init(ctypes.byref(self.graph))

    def input(self, name: str, shape, dtype: str = "float32", layout: int = LAYOUT_ROW) -> int:
        i = self.lib.bafe_graph_add_input_with_layout(ctypes.byref(self.graph), name.encode(),
                                                      ctypes.byref(_shape(shape)), DTYPE[dtype], layout)
        if i < 0:
            raise RuntimeError(f"bafe_graph_add_input_with_layout({name}) failed")
        return i

    def add(self, op: str, children, perm=None) -> int:
        attrs = None
        if perm is not None:
            a = OpAttrs()
            a.n_perm = len(perm)
            for k, v in enumerate(perm):
                a.perm[k] = v
            attrs = ctypes.byref(a)
        ids = (c_int32 * len(children))(*children)
        i = self.lib.bafe_graph_add(ctypes.byref(self.graph), op.encode(), ids, len(children), attrs)
        if i < 0:
            raise RuntimeError(f"bafe_graph_add({op}) failed")
        return i

    def output(self, node: int) -> None:
        self.lib.bafe_graph_set_output(ctypes.byref(self.graph), node)
