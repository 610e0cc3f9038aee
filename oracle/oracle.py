"""CPU oracle for the BAFE hot path -- TEST INFRASTRUCTURE ONLY.

Nothing in the product imports this module: only tests/, __graft_entry__.smoke()
and bench.py's cpu_baseline leg do, to check results and time the CPU baseline.

`evaluate(nodes, arrays)` interprets a BAFE graph node by node the way the
reference's C99 emitter compiles it (bafe/src/codegen.c:172-551): one
buffer per node in raw storage order, the per-op loop nests restated in
oracle/bafe_oracle.c (each citing the emitter lines it follows), and the
output converted to the root's dtype.  It accepts the node list of
GraphBuilder.to_list() (or the same dicts loaded from tests/golden).

Parity of this restatement is pinned against the reference's own compiled
kernels: tests/golden/*.npz hold outputs the reference produced
(tests/golden/make_golden.py) and tests/test_oracle_golden.py requires
bit-identical results.

Deliberate departures, where the reference is defective (its output is not
the operation's value) and the backend computes the intended value:
  * rank-N transpose: the emitter's index (codegen.c:371-404) is the inverse
    permutation; the oracle uses the true transpose (identical for
    self-inverse perms, which oracle_transpose_nd covers);
  * broadcast_to: the emitter memcpy's numel(out) elements out of a smaller
    buffer (codegen.c:465); the oracle broadcasts;
  * matmul operand produced by a transpose node: the emitter reads it as
    column-major because of the layout tag (codegen.c:206-213 vs
    ir.c:101-110) although it is stored row-major; the oracle reads the
    stored layout;
  * fused_matmul_* with column-major operands: the emitter ignores the
    layout tags (codegen.c:482,498,513); the oracle honours them.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, c_double, c_float, c_int, c_int32, c_int64, c_uint16, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

F32, F64, I32, I64, F16, BF16 = range(6)
LAYOUT_COL = 1
NP = {F32: np.float32, F64: np.float64, I32: np.int32, I64: np.int64, F16: np.uint16, BF16: np.uint16}
SFX = {F32: "f32", F64: "f64", I32: "i32", I64: "i64"}
OP_CODE = {"add": 0, "sub": 1, "mul": 2, "bias_add": 0, "fused_bias_relu": 0}


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)
    lib = ctypes.CDLL(str(LIB_PATH))
    for s in SFX.values():
        getattr(lib, f"oracle_binary_{s}").argtypes = [c_int, c_int, c_void_p, c_void_p, c_void_p, c_int64, c_int64]
        for u in ("relu", "neg"):
            getattr(lib, f"oracle_{u}_{s}").argtypes = [c_void_p, c_void_p, c_int64]
        getattr(lib, f"oracle_matmul_{s}").argtypes = [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                                      c_int64, c_int, c_int, c_int64, c_int]
        getattr(lib, f"oracle_reduce_{s}").argtypes = [c_void_p, c_void_p, c_int64, c_int64, c_int, c_int]
    for s in ("f32", "f64"):
        for u in ("sigmoid", "tanh"):
            getattr(lib, f"oracle_{u}_{s}").argtypes = [c_void_p, c_void_p, c_int64]
    lib.oracle_transpose2d.argtypes = [c_void_p, c_void_p, c_int64, c_int64, c_int]
    lib.oracle_transpose_nd.argtypes = [c_void_p, c_void_p, c_int, POINTER(c_int32), POINTER(c_int32),
                                        POINTER(c_int32), c_int]
    lib.oracle_matmul_panel_f32.argtypes = [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int, c_int,
                                            c_int64, c_int64]
    for fn in ("oracle_f16_to_f32_n", "oracle_bf16_to_f32_n", "oracle_f32_to_f16_n", "oracle_f32_to_bf16_n"):
        getattr(lib, fn).argtypes = [c_void_p, c_void_p, c_int64]
    return lib


lib = _load()


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"] or a.ndim <= 1
    return a.ctypes.data


def compute_dtype(dt: int) -> int:
    return F32 if dt in (F16, BF16) else dt


def common_type(a: int, b: int) -> int:
    """C's usual arithmetic conversions over the emitter's buffer types."""
    if F64 in (a, b):
        return F64
    if F32 in (a, b):
        return F32
    if I64 in (a, b):
        return I64
    return I32


# --------------------------------------------------------------- kernels --

def half_to_f32(raw: np.ndarray, dt: int) -> np.ndarray:
    """codegen.c:157-169 with the emitter's helpers (codegen.c:91-127)."""
    raw = np.ascontiguousarray(raw.reshape(-1).view(np.uint16))
    out = np.empty(raw.size, np.float32)
    fn = lib.oracle_f16_to_f32_n if dt == F16 else lib.oracle_bf16_to_f32_n
    fn(_p(raw), _p(out), raw.size)
    return out


def f32_to_half(v: np.ndarray, dt: int) -> np.ndarray:
    """codegen.c:542-547."""
    v = np.ascontiguousarray(v.reshape(-1), dtype=np.float32)
    out = np.empty(v.size, np.uint16)
    fn = lib.oracle_f32_to_f16_n if dt == F16 else lib.oracle_f32_to_bf16_n
    fn(_p(v), _p(out), v.size)
    return out


def binary(op: str, a: np.ndarray, b: np.ndarray, mode: int, M: int, N: int, ta: int, tb: int, tout: int) -> np.ndarray:
    """codegen.c:294-326 (mode 0 same shape, 1 b is the row vector, 2 a is)."""
    cm = common_type(ta, tb)
    a = np.ascontiguousarray(a, dtype=NP[cm])
    b = np.ascontiguousarray(b, dtype=NP[cm])
    out = np.empty(M * N, NP[cm])
    getattr(lib, f"oracle_binary_{SFX[cm]}")(OP_CODE[op], mode, _p(a), _p(b), _p(out), M, N)
    return out.astype(NP[tout])


def unary(op: str, x: np.ndarray, tx: int, tout: int) -> np.ndarray:
    """relu/neg codegen.c:338-344,357-359; sigmoid/tanh codegen.c:345-356."""
    x = np.ascontiguousarray(x)
    if op in ("relu",):
        x = x.astype(NP[tout])
        out = np.empty_like(x)
        getattr(lib, f"oracle_relu_{SFX[tout]}")(_p(x), _p(out), x.size)
        return out
    if op == "neg":
        out = np.empty_like(x)
        getattr(lib, f"oracle_neg_{SFX[tx]}")(_p(x), _p(out), x.size)
        return out.astype(NP[tout])
    # sigmoid / tanh: float libm on the float-converted argument
    if tx == F64:
        out = np.empty_like(x)
        getattr(lib, f"oracle_{op}_f64")(_p(x), _p(out), x.size)
    else:
        xf = x.astype(np.float32)
        out = np.empty_like(xf)
        getattr(lib, f"oracle_{op}_f32")(_p(xf), _p(out), xf.size)
    return out.astype(NP[tout])


def matmul(A: np.ndarray, B: np.ndarray, batch: int, M: int, N: int, K: int, a_col: bool, b_col: bool,
           t: int, direct: bool, a_bstride: int, b_bstride: int) -> np.ndarray:
    """codegen.c:191-293 (chunked) and 467-517 (direct)."""
    A = np.ascontiguousarray(A, dtype=NP[t])
    B = np.ascontiguousarray(B, dtype=NP[t])
    out = np.empty(batch * M * N, NP[t])
    fn = getattr(lib, f"oracle_matmul_{SFX[t]}")
    for b in range(batch):
        Ab = np.ascontiguousarray(A[b * a_bstride: b * a_bstride + M * K])
        Bb = np.ascontiguousarray(B[b * b_bstride: b * b_bstride + K * N])
        ob = np.empty(M * N, NP[t])
        fn(_p(Ab), _p(Bb), _p(ob), 1, M, N, K, int(a_col), int(b_col), K if direct else 32, int(direct))
        out[b * M * N:(b + 1) * M * N] = ob
    return out


def matmul_panel_f32(A: np.ndarray, B: np.ndarray, M: int, N: int, K: int, a_col: bool, b_col: bool, r0: int,
                     r1: int) -> np.ndarray:
    """Rows [r0, r1) of the chunked f32 matmul (bit-identical to the full run)."""
    A = np.ascontiguousarray(A, dtype=np.float32).reshape(-1)
    B = np.ascontiguousarray(B, dtype=np.float32).reshape(-1)
    out = np.empty((r1 - r0) * N, np.float32)
    lib.oracle_matmul_panel_f32(_p(A), _p(B), _p(out), M, N, K, int(a_col), int(b_col), r0, r1)
    return out.reshape(r1 - r0, N)


def transpose2d(x: np.ndarray, M: int, N: int) -> np.ndarray:
    """codegen.c:363-369: out (M,N) from x (N,M)."""
    x = np.ascontiguousarray(x)
    out = np.empty(M * N, x.dtype)
    lib.oracle_transpose2d(_p(x), _p(out), M, N, x.itemsize)
    return out


def transpose_nd_reference(x: np.ndarray, in_dims, out_dims, perm) -> np.ndarray:
    """The emitter's own rank-N indexing (codegen.c:371-404); valid for
    self-inverse permutations only."""
    x = np.ascontiguousarray(x)
    R = len(perm)
    arr = lambda v: (c_int32 * R)(*v)
    out = np.empty(int(np.prod(out_dims)), x.dtype)
    lib.oracle_transpose_nd(_p(x), _p(out), R, arr(out_dims), arr(in_dims), arr(perm), x.itemsize)
    return out


def reduce(x: np.ndarray, M: int, N: int, ax: int, is_max: bool, t: int) -> np.ndarray:
    """codegen.c:410-445."""
    x = np.ascontiguousarray(x, dtype=NP[t])
    out = np.empty(N if ax == 0 else M, NP[t])
    getattr(lib, f"oracle_reduce_{SFX[t]}")(_p(x), _p(out), M, N, ax, int(is_max))
    return out


# ------------------------------------------------------------ evaluator --

def _numel(shape) -> int:
    n = 1
    for d in shape:
        n *= d
    return n


def evaluate(nodes: list, arrays: dict, root: int) -> np.ndarray:
    """Interpret the graph.  arrays maps input node id -> numpy array in the
    layout its tag declares (Fortran order for COL_MAJOR inputs).  Returns
    the output as a flat array of the root's stored dtype."""
    vals: dict = {}

    def col_storage(i: int) -> bool:
        n = nodes[i]
        return n["is_input"] and n["layout"] == LAYOUT_COL

    def ev(i: int) -> np.ndarray:
        if i in vals:
            return vals[i]
        n = nodes[i]
        op, ch, dt = n["op"], n["children"], n["dtype"]
        T = compute_dtype(dt)
        shape = tuple(n["shape"])
        if n["is_input"]:
            a = np.asarray(arrays[i])
            fortran = a.ndim >= 2 and a.flags["F_CONTIGUOUS"] and not a.flags["C_CONTIGUOUS"]
            raw = np.ravel(a, order="F" if fortran else "C")
            v = half_to_f32(raw, dt) if dt in (F16, BF16) else np.ascontiguousarray(raw, dtype=NP[dt])
        elif op in ("add", "sub", "mul", "bias_add", "fused_bias_relu"):
            a, b = ev(ch[0]), ev(ch[1])
            sa, sb = tuple(nodes[ch[0]]["shape"]), tuple(nodes[ch[1]]["shape"])
            ta, tb = compute_dtype(nodes[ch[0]]["dtype"]), compute_dtype(nodes[ch[1]]["dtype"])
            if op in ("bias_add", "fused_bias_relu"):
                v = binary(op, a, b, 1, shape[0], shape[1], ta, tb, T)
            elif len(sa) == 2 and len(sb) == 1 and sa[1] == sb[0]:
                v = binary(op, a, b, 1, sa[0], sa[1], ta, tb, T)
            elif len(sa) == 1 and len(sb) == 2 and sa[0] == sb[1]:
                v = binary(op, a, b, 2, sb[0], sb[1], ta, tb, T)
            else:
                assert a.size == b.size == _numel(shape), f"unsupported broadcast {sa} {sb}"
                v = binary(op, a, b, 0, 1, _numel(shape), ta, tb, T)
            if op == "fused_bias_relu":
                v = unary("relu", v, T, T)
        elif op in ("relu", "neg", "sigmoid", "tanh"):
            v = unary(op, ev(ch[0]), compute_dtype(nodes[ch[0]]["dtype"]), T)
        elif op in ("reshape", "layout_transform"):
            v = ev(ch[0]).astype(NP[T])
        elif op in ("matmul", "fused_matmul_relu", "fused_matmul_bias", "fused_matmul_bias_relu"):
            a_n, b_n = nodes[ch[0]], nodes[ch[1]]
            sa, sb = a_n["shape"], b_n["shape"]
            M, N, K = shape[-2], shape[-1], sa[-1]
            batch = _numel(shape[:-2])
            a_items, b_items = _numel(sa[:-2]), _numel(sb[:-2])
            ta, tb = compute_dtype(a_n["dtype"]), compute_dtype(b_n["dtype"])
            assert ta == tb == T, "mixed-dtype matmul is not restated"
            v = matmul(ev(ch[0]), ev(ch[1]), batch, M, N, K, col_storage(ch[0]), col_storage(ch[1]), T,
                       op != "matmul", 0 if a_items == 1 else M * K, 0 if b_items == 1 else K * N)
            if op in ("fused_matmul_bias", "fused_matmul_bias_relu"):
                v = binary("add", v, ev(ch[2]), 1, M, N, T, compute_dtype(nodes[ch[2]]["dtype"]), T)
            if op in ("fused_matmul_relu", "fused_matmul_bias_relu"):
                v = unary("relu", v, T, T)
        elif op == "transpose":
            x = ev(ch[0])
            xs = tuple(nodes[ch[0]]["shape"])
            if len(shape) == 2:
                v = transpose2d(x, shape[0], shape[1])
            else:
                v = np.ascontiguousarray(np.transpose(x.reshape(xs), n["perm"])).reshape(-1)
        elif op == "broadcast_to":
            xs = tuple(nodes[ch[0]]["shape"])
            v = np.ascontiguousarray(np.broadcast_to(ev(ch[0]).reshape(xs), shape)).reshape(-1).astype(NP[T])
        elif op in ("reduce_sum", "reduce_max"):
            x = ev(ch[0])
            xs = tuple(nodes[ch[0]]["shape"])
            if len(n["axes"]) == 1 and len(xs) == 1:
                v = reduce(x, 1, xs[0], 1, op == "reduce_max", T)
            elif len(n["axes"]) == 1 and len(xs) == 2:
                ax = int(np.fmod(n["axes"][0], 2))   # C's % (codegen.c:421)
                v = reduce(x, xs[0], xs[1], 0 if ax == 0 else 1, op == "reduce_max", T)
            else:
                v = np.zeros(_numel(shape), NP[T])
        else:
            v = np.zeros(_numel(shape), NP[T])     # codegen.c:529-533
        vals[i] = v
        return v

    v = ev(root)
    rdt = nodes[root]["dtype"]
    if rdt in (F16, BF16):
        return f32_to_half(v, rdt)
    return np.ascontiguousarray(v, dtype=NP[rdt])
