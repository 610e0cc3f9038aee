"""Builds BAFE graph structs (BafeGraph) in Python.

The rules restate the reference's graph construction so that a graph built
here is the struct BAFE itself would build for the same expression:
  * arity and shape inference per op: bafe/src/ops.c:24-149 with the shape
    algebra of bafe/src/types.c:97-143 (broadcast, reduce, transpose);
  * dtype = first child's dtype, layout propagation: bafe/src/ir.c:89-145
    (transpose of a rank-2 tensor with perm (1,0) flips ROW<->COL,
    layout_transform sets it from attrs.name, everything else inherits
    child 0's layout);
  * inputs are appended to graph.inputs in creation order (ir.c:50), which
    is the kernel's parameter order.
"""
from __future__ import annotations

import ctypes
from typing import Iterable, Sequence

from ._binding import (BAFE_MAX_ATTR_LEN, BAFE_MAX_CHILDREN, BAFE_MAX_NODES, BAFE_MAX_RANK, BafeGraph,
                       LAYOUT_BLOCKED, LAYOUT_COL, LAYOUT_ROW, LAYOUT_TC)

# op name -> arity (ops.c:125-149)
ARITY = {
    "input": 0, "constant": 0, "matmul": 2, "add": 2, "mul": 2, "sub": 2, "scale": 2, "bias_add": 2,
    "relu": 1, "sigmoid": 1, "tanh": 1, "neg": 1, "layout_transform": 1, "transpose": 1,
    "reduce_sum": 1, "reduce_max": 1, "reshape": 1, "broadcast_to": 1,
    "fused_matmul_relu": 2, "fused_matmul_bias": 3, "fused_matmul_bias_relu": 3, "fused_bias_relu": 2,
}
# Interned op-name strings: node.op_name points into these for the life of
# the process (BAFE's op_name is a borrowed pointer into its registry).
_OPNAME = {k: k.encode() for k in ARITY}

LAYOUT_NAMES = {"row": LAYOUT_ROW, "col": LAYOUT_COL, "blocked": LAYOUT_BLOCKED, "tc": LAYOUT_TC}


def shape_broadcast(a: Sequence[int], b: Sequence[int]) -> tuple:
    """types.c:97-111; -1 marks an incompatible dimension."""
    n = min(max(len(a), len(b)), BAFE_MAX_RANK)
    out = []
    for i in range(n):
        da = 1 if i < n - len(a) else a[i - (n - len(a))]
        db = 1 if i < n - len(b) else b[i - (n - len(b))]
        if da == 1:
            out.append(db)
        elif db == 1 or db == da:
            out.append(da)
        else:
            out.append(-1)
    return tuple(out)


def shape_reduce(s: Sequence[int], axes: Sequence[int], keepdims: bool) -> tuple:
    """types.c:113-136 (no axes = reduce everything)."""
    mask = [False] * len(s)
    if not axes:
        mask = [True] * len(s)
    for a in axes:
        if a < 0:
            a += len(s)
        if 0 <= a < len(s):
            mask[a] = True
    out = []
    for i, d in enumerate(s):
        if mask[i]:
            if keepdims:
                out.append(1)
        else:
            out.append(d)
    return tuple(out)


def _matmul_shape(a: Sequence[int], b: Sequence[int]) -> tuple:
    """ops.c:24-51."""
    if len(a) < 2 or len(b) < 2:
        return ()
    M, N = a[-2], b[-1]
    if len(a) == 2 and len(b) == 2:
        return (M, N)
    batch = shape_broadcast(a[:-2], b[:-2])
    if len(batch) + 2 > BAFE_MAX_RANK:
        return (M, N)
    return tuple(batch) + (M, N)


def _reshape_shape(s: Sequence[int], target: Sequence[int]) -> tuple:
    """ops.c:85-107 (-1 resolved from the element count)."""
    numel = 1
    for d in s:
        numel *= d
    target = list(target)
    neg = [i for i, d in enumerate(target) if d == -1]
    if len(neg) > 1:
        return ()
    if neg:
        known = 1
        for d in target:
            if d != -1:
                known *= d
        if known == 0 or numel % known:
            return ()
        target[neg[0]] = numel // known
    return tuple(target)


class GraphBuilder:
    """Incrementally builds a BafeGraph, like bafe_graph_add & friends."""

    def __init__(self) -> None:
        self.graph = BafeGraph()
        ctypes.memset(ctypes.byref(self.graph), 0, ctypes.sizeof(BafeGraph))

    # -- queries -----------------------------------------------------------
    @property
    def n_nodes(self) -> int:
        return self.graph.n_nodes

    def shape(self, nid: int) -> tuple:
        s = self.graph.nodes[nid].shape
        return tuple(s.dims[i] for i in range(s.rank))

    def dtype(self, nid: int) -> int:
        return self.graph.nodes[nid].dtype

    def layout(self, nid: int) -> int:
        return self.graph.nodes[nid].layout

    def op(self, nid: int) -> str:
        return self.graph.nodes[nid].op_name.decode()

    def children(self, nid: int) -> list:
        n = self.graph.nodes[nid]
        return [n.children[i] for i in range(n.n_children)]

    # -- construction ------------------------------------------------------
    def _new(self) -> int:
        g = self.graph
        if g.n_nodes >= BAFE_MAX_NODES:
            raise RuntimeError("graph is full")
        nid = g.n_nodes
        g.n_nodes += 1
        ctypes.memset(ctypes.byref(g.nodes[nid]), 0, ctypes.sizeof(g.nodes[nid]))
        g.nodes[nid].id = nid
        return nid

    @staticmethod
    def _set_shape(node, shape: Iterable[int]) -> None:
        shape = tuple(int(d) for d in shape)
        if len(shape) > BAFE_MAX_RANK:
            raise ValueError(f"rank {len(shape)} exceeds {BAFE_MAX_RANK}")
        node.shape.rank = len(shape)
        for i, d in enumerate(shape):
            node.shape.dims[i] = d

    def add_input(self, name: str, shape: Sequence[int], dtype: int = 0, layout: int = LAYOUT_ROW) -> int:
        """ir.c:26-52."""
        nid = self._new()
        n = self.graph.nodes[nid]
        n.op_name = _OPNAME["input"]
        n.is_input = True
        self._set_shape(n, shape)
        n.dtype = int(dtype)
        n.layout = int(layout)
        raw = name.encode()[: BAFE_MAX_ATTR_LEN - 1]
        n.input_name = raw
        n.attrs.name = raw
        self.graph.inputs[self.graph.n_inputs] = nid
        self.graph.n_inputs += 1
        return nid

    def add(self, op: str, children: Sequence[int], *, perm: Sequence[int] = (), axes: Sequence[int] = (),
            keepdims: bool = False, shape: Sequence[int] = (), name: str = "") -> int:
        """ir.c:115-145 with ops.c's shape functions."""
        if op not in ARITY or op in ("input", "constant"):
            raise ValueError(f"unknown op {op!r}")
        if len(children) != ARITY[op]:
            raise ValueError(f"{op} takes {ARITY[op]} children, got {len(children)}")
        for c in children:
            if not 0 <= c < self.graph.n_nodes:
                raise ValueError(f"child {c} out of range")
        shapes = [self.shape(c) for c in children]
        if op == "matmul" or op == "fused_matmul_relu" or op.startswith("fused_matmul_bias"):
            out = _matmul_shape(shapes[0], shapes[1])
        elif op in ("add", "mul", "sub"):
            out = shape_broadcast(shapes[0], shapes[1])
        elif op == "transpose":
            out = tuple(shapes[0][p] for p in perm)
        elif op in ("reduce_sum", "reduce_max"):
            out = shape_reduce(shapes[0], axes, keepdims)
        elif op == "reshape":
            out = _reshape_shape(shapes[0], shape)
        elif op == "broadcast_to":
            out = tuple(shape)
        else:   # scale, bias_add, unary, layout_transform, fused_bias_relu
            out = shapes[0]
        nid = self._new()
        n = self.graph.nodes[nid]
        n.op_name = _OPNAME[op]
        n.n_children = len(children)
        for i, c in enumerate(children):
            n.children[i] = c
        for field, vals in (("axes", axes), ("perm", perm), ("shape", shape)):
            vals = list(vals)[:BAFE_MAX_ATTR_LEN]
            setattr(n.attrs, "n_" + field, len(vals))
            arr = getattr(n.attrs, field)
            for i, v in enumerate(vals):
                arr[i] = int(v)
        n.attrs.keepdims = bool(keepdims)
        if name:
            n.attrs.name = name.encode()[: BAFE_MAX_ATTR_LEN - 1]
        self._set_shape(n, out)
        if children:
            n.dtype = self.graph.nodes[children[0]].dtype
        n.layout = self._infer_layout(op, n, children)
        return nid

    def _infer_layout(self, op: str, n, children: Sequence[int]) -> int:
        """ir.c:89-113."""
        if op == "layout_transform":
            return LAYOUT_NAMES.get(n.attrs.name.decode(), LAYOUT_ROW)
        if op == "transpose" and len(children) == 1:
            x = self.graph.nodes[children[0]]
            if x.shape.rank == 2 and n.attrs.n_perm == 2 and n.attrs.perm[0] == 1 and n.attrs.perm[1] == 0:
                if x.layout == LAYOUT_ROW:
                    return LAYOUT_COL
                if x.layout == LAYOUT_COL:
                    return LAYOUT_ROW
            return x.layout
        if children:
            return self.graph.nodes[children[0]].layout
        return LAYOUT_ROW

    def set_output(self, nid: int) -> None:
        g = self.graph
        g.outputs[g.n_outputs] = nid
        g.n_outputs += 1

    # -- cross-call fusion ------------------------------------------------------
    @classmethod
    def concat(cls, a: "GraphBuilder", b: "GraphBuilder") -> "GraphBuilder":
        """fuse.c:12-104: a's nodes, then b's nodes with children shifted by
        a's node count, except that uses of b's FIRST input read a's output;
        inputs = a's inputs + b's inputs[1:]; output = b's output.  b's first
        input node stays in the node list, unreferenced."""
        ga, gb = a.graph, b.graph
        if ga.n_outputs == 0:
            raise ValueError("graph_a has no outputs")
        if gb.n_inputs == 0:
            raise ValueError("graph_b has no inputs")
        if ga.n_nodes + gb.n_nodes > BAFE_MAX_NODES:
            raise ValueError("fused graph too large")
        out = cls()
        g = out.graph
        off = ga.n_nodes
        a_out = ga.outputs[0]
        b_first = gb.inputs[0]
        b_inputs = {gb.inputs[k] for k in range(gb.n_inputs)}
        for i in range(ga.n_nodes):
            g.nodes[i] = ga.nodes[i]
            g.nodes[i].id = i
        for j in range(gb.n_nodes):
            g.nodes[off + j] = gb.nodes[j]
            d = g.nodes[off + j]
            d.id = off + j
            for c in range(d.n_children):
                ch = d.children[c]
                d.children[c] = a_out if (ch == b_first and ch in b_inputs) else ch + off
        g.n_nodes = ga.n_nodes + gb.n_nodes
        for i in range(ga.n_inputs):
            g.inputs[g.n_inputs] = ga.inputs[i]
            g.n_inputs += 1
        for i in range(1, gb.n_inputs):
            g.inputs[g.n_inputs] = gb.inputs[i] + off
            g.n_inputs += 1
        g.outputs[0] = gb.outputs[0] + off
        g.n_outputs = 1
        return out

    # -- export for the oracle -------------------------------------------------
    def to_list(self) -> list:
        """Plain-Python view of the nodes (for the CPU oracle)."""
        out = []
        for i in range(self.graph.n_nodes):
            n = self.graph.nodes[i]
            out.append({
                "id": i, "op": n.op_name.decode(), "children": self.children(i), "shape": self.shape(i),
                "dtype": n.dtype, "layout": n.layout, "name": n.input_name.decode(), "is_input": bool(n.is_input),
                "perm": [n.attrs.perm[k] for k in range(n.attrs.n_perm)],
                "axes": [n.attrs.axes[k] for k in range(n.attrs.n_axes)],
                "tshape": [n.attrs.shape[k] for k in range(n.attrs.n_shape)],
                "keepdims": bool(n.attrs.keepdims),
            })
        return out

    @property
    def inputs(self) -> list:
        return [self.graph.inputs[i] for i in range(self.graph.n_inputs)]

    @property
    def output(self) -> int:
        return self.graph.outputs[0]
