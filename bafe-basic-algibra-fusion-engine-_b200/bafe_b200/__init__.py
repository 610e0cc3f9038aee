"""bafe_b200 -- B200 execution backend for BAFE, with a front end that
mirrors BAFE's `@bafe.jit` API (bafe/python/bafe/__init__.py).

    import bafe_b200 as bafe

    @bafe.jit
    def f(A, B, C):
        return bafe.relu(bafe.matmul(A, B) + C)

    out = f(A, B, C)        # numpy in, numpy out; runs on the GPU

Tracing, argument-layout detection (Fortran-contiguous -> "col"), the
per-(shape, dtype, layout) cache and the host-pointer call follow the
reference's JittedFunction (__init__.py:310-545).  The graph goes to
libbafe_cuda.so's bafe_cuda_jit_get_or_compile -- the drop-in for BAFE's
bafe_jit_get_or_compile -- without BAFE's optimizer in between: at the
sizes BAFE targets its extractor returns the same unfused chain the trace
builds, and the backend does the fusion.

Lower-level entry points: GraphBuilder (graph.py), compile_graph() ->
Kernel, Kernel.run_device() for device-resident buffers (torch tensors or
raw pointers) on a CUDA stream.
"""
from __future__ import annotations

import ctypes
import functools
from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np

from . import _binding
from ._binding import (BafeGraph, DTYPE_BF16, DTYPE_F16, DTYPE_F32, DTYPE_F64, DTYPE_I32, DTYPE_I64, check,
                       last_error, lib)
from .graph import LAYOUT_NAMES, GraphBuilder

__version__ = "0.1.0"

_NP_TO_BAFE = {
    np.dtype("float32"): DTYPE_F32, np.dtype("float64"): DTYPE_F64, np.dtype("int32"): DTYPE_I32,
    np.dtype("int64"): DTYPE_I64, np.dtype("float16"): DTYPE_F16,
}
_BAFE_TO_NP = {v: k for k, v in _NP_TO_BAFE.items()}
_BAFE_TO_NP[DTYPE_BF16] = np.dtype("uint16")   # bf16 travels as raw 16-bit words


# ---------------------------------------------------------------- backend --

def set_option(key: str, value: str) -> None:
    """Backend option, e.g. set_option("gemm_precision", "exact")."""
    if lib.bafe_cuda_set_option(key.encode(), str(value).encode()) != 0:
        raise ValueError(f"bad option {key}={value}")


def get_option(key: str) -> str:
    buf = ctypes.create_string_buffer(64)
    if lib.bafe_cuda_get_option(key.encode(), buf, len(buf)) != 0:
        raise KeyError(key)
    return buf.value.decode()


def jit_stats() -> dict:
    s = lib.bafe_cuda_jit_get_stats()
    return {"hits": s.hits, "misses": s.misses, "compiles": s.compiles, "compile_failures": s.compile_failures}


def jit_clear() -> None:
    lib.bafe_cuda_jit_clear()


def jit_invalidate_memory_cache() -> None:
    lib.bafe_cuda_jit_invalidate_memory_cache()


def set_cache_dir(path: str) -> None:
    lib.bafe_cuda_jit_set_cache_dir(str(path).encode())


def cache_dir() -> str:
    return lib.bafe_cuda_jit_cache_dir().decode()


def graph_hash(graph: BafeGraph) -> str:
    buf = ctypes.create_string_buffer(65)
    if lib.bafe_cuda_jit_hash_graph(ctypes.byref(graph), buf, 65) != 0:
        raise RuntimeError("hash failed")
    return buf.value.decode()


def launch_count() -> int:
    return int(lib.bafe_cuda_launch_count())


def synchronize() -> None:
    """Wait for the current device; raise if a kernel reported an error
    (e.g. a tensor-core pipeline wait that ran past its deadline)."""
    check(lib.bafe_cuda_synchronize(), "synchronize")


class Kernel:
    """A compiled plan: the host function BAFE's ABI returns, plus device entry."""

    def __init__(self, fn_ptr: int, n_inputs: int, out_shape: tuple, out_dtype: np.dtype, graph: BafeGraph):
        self.fn_ptr = fn_ptr
        self.plan = lib.bafe_cuda_plan_of(ctypes.c_void_p(fn_ptr))
        if self.plan < 0:
            raise RuntimeError("function pointer is not a bafe_cuda plan")
        self.n_inputs = n_inputs
        self.out_shape = out_shape
        self.out_dtype = out_dtype
        self.graph = graph
        self._sig = ctypes.CFUNCTYPE(None, *([ctypes.c_void_p] * (n_inputs + 1)))
        self._call = self._sig(fn_ptr)

    def describe(self) -> str:
        n = lib.bafe_cuda_plan_describe(self.plan, None, 0)
        buf = ctypes.create_string_buffer(n + 1)
        lib.bafe_cuda_plan_describe(self.plan, buf, n + 1)
        return buf.value.decode()

    @property
    def output_bytes(self) -> int:
        return int(lib.bafe_cuda_plan_output_bytes(self.plan))

    def input_bytes(self, i: int) -> int:
        return int(lib.bafe_cuda_plan_input_bytes(self.plan, i))

    def row_split(self):
        """(rows, per-input bytes per row, output bytes per row) when host
        calls stream this plan in row panels (0 bytes: input read whole),
        else None."""
        rows = ctypes.c_int64()
        out_rb = ctypes.c_int64()
        in_rb = (ctypes.c_int64 * max(self.n_inputs, 1))()
        rc = lib.bafe_cuda_plan_row_split(self.plan, ctypes.byref(rows), in_rb, self.n_inputs, ctypes.byref(out_rb))
        if rc < 0:
            raise RuntimeError("unknown plan")
        if rc == 0:
            return None
        return int(rows.value), [int(in_rb[i]) for i in range(self.n_inputs)], int(out_rb.value)

    def call_host_ptrs(self, ptrs: Sequence[int]) -> None:
        """Call the ABI function (host pointers, synchronous) and raise on error."""
        lib.bafe_cuda_clear_error()
        self._call(*[ctypes.c_void_p(p) for p in ptrs])
        code, msg = last_error()
        if code:
            raise RuntimeError(f"bafe_cuda kernel failed (code {code}): {msg}")

    def call_host_resident(self, ptrs: Sequence[int], resident: Sequence[bool], ready=None) -> None:
        """bafe_cuda_run_host_resident: host pointers, except the inputs whose
        `resident` flag is set, which are device buffers read in place;
        `ready` (a torch.cuda.Event or a raw cudaEvent_t) is recorded after
        the work that fills them: the copies start at once, the kernels wait."""
        if len(resident) != self.n_inputs:
            raise TypeError(f"kernel takes {self.n_inputs} inputs, got {len(resident)} resident flags")
        arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
        flags = (ctypes.c_ubyte * self.n_inputs)(*[1 if r else 0 for r in resident])
        ev = getattr(ready, "cuda_event", ready)
        if lib.bafe_cuda_run_host_resident(self.plan, arr, len(ptrs), flags, ctypes.c_void_p(ev) if ev else None):
            code, msg = last_error()
            raise RuntimeError(f"bafe_cuda_run_host_resident failed (code {code}): {msg}")

    def __call__(self, *arrays: np.ndarray, out: Optional[np.ndarray] = None) -> np.ndarray:
        if len(arrays) != self.n_inputs:
            raise TypeError(f"kernel takes {self.n_inputs} inputs, got {len(arrays)}")
        if out is None:
            out = np.zeros(self.out_shape, dtype=self.out_dtype)
        self.call_host_ptrs([a.ctypes.data for a in arrays] + [out.ctypes.data])
        return out

    def run_device(self, ptrs: Sequence[int], stream: int = 0) -> None:
        """Enqueue on device buffers (inputs..., out) on `stream` (cudaStream_t)."""
        arr = (ctypes.c_void_p * len(ptrs))(*[ctypes.c_void_p(int(p)) for p in ptrs])
        check(lib.bafe_cuda_run_device(self.plan, arr, len(ptrs), ctypes.c_void_p(int(stream))), "run_device")

    def run_torch(self, inputs: Sequence, out, stream=None) -> None:
        """run_device on torch CUDA tensors (contiguous in the layout the graph declares)."""
        import torch
        s = stream if stream is not None else torch.cuda.current_stream()
        self.run_device([t.data_ptr() for t in inputs] + [out.data_ptr()], s.cuda_stream)

    @property
    def num_steps(self) -> int:
        """Launch steps of the plan (the lines of describe())."""
        return int(lib.bafe_cuda_plan_num_steps(self.plan))

    def run_torch_timed(self, inputs: Sequence, out, events: Sequence, stream=None) -> None:
        """run_torch with events[2i] / events[2i+1] (torch.cuda.Event with
        timing) recorded before / after step i's launches."""
        import torch
        s = stream if stream is not None else torch.cuda.current_stream()
        ptrs = [t.data_ptr() for t in inputs] + [out.data_ptr()]
        arr = (ctypes.c_void_p * len(ptrs))(*[ctypes.c_void_p(int(p)) for p in ptrs])
        for e in events:
            if not e.cuda_event:          # torch creates the CUDA event at its first record
                e.record(s)
        evs = (ctypes.c_void_p * len(events))(*[ctypes.c_void_p(e.cuda_event) for e in events])
        check(lib.bafe_cuda_run_device_timed(self.plan, arr, len(ptrs), ctypes.c_void_p(int(s.cuda_stream)), evs,
                                             len(events)), "run_device_timed")

    @property
    def k_slice_align(self) -> int:
        """Multiple of K that K-slice bounds must be; 0: the plan cannot run in K slices."""
        return int(lib.bafe_cuda_plan_k_slice_align(self.plan))

    def run_torch_ksliced(self, inputs: Sequence, out, k_bounds: Sequence[int], ready=None, stream=None) -> None:
        """bafe_cuda_run_device_ksliced on torch CUDA tensors: the GEMM over
        K slices [k_bounds[j], k_bounds[j+1]), slice j waiting on ready[j]
        (torch.cuda.Event, raw cudaEvent_t or None)."""
        import torch
        s = stream if stream is not None else torch.cuda.current_stream()
        ptrs = [t.data_ptr() for t in inputs] + [out.data_ptr()]
        arr = (ctypes.c_void_p * len(ptrs))(*[ctypes.c_void_p(int(p)) for p in ptrs])
        n = len(k_bounds) - 1
        kb = (ctypes.c_int64 * len(k_bounds))(*[int(k) for k in k_bounds])
        evs = None
        if ready is not None:
            if len(ready) != n:
                raise TypeError(f"{n} K slices but {len(ready)} events")
            evs = (ctypes.c_void_p * n)(*[ctypes.c_void_p(getattr(e, "cuda_event", e) or 0) for e in ready])
        check(lib.bafe_cuda_run_device_ksliced(self.plan, arr, len(ptrs), ctypes.c_void_p(int(s.cuda_stream)), n, kb,
                                               evs), "run_device_ksliced")


def compile_graph(builder: GraphBuilder) -> Kernel:
    """bafe_cuda_jit_get_or_compile on a built graph."""
    err = ctypes.create_string_buffer(4096)
    fn = lib.bafe_cuda_jit_get_or_compile(ctypes.byref(builder.graph), err, len(err))
    if not fn:
        raise RuntimeError(f"bafe_cuda_jit_get_or_compile failed: {err.value.decode(errors='replace')}")
    out = builder.output
    out_shape = builder.shape(out)
    out_dtype = _BAFE_TO_NP[builder.dtype(out)]
    return Kernel(fn, builder.graph.n_inputs, out_shape, out_dtype, builder.graph)


# ------------------------------------------------------------- tracing --

_TRACE: Optional[GraphBuilder] = None


def _trace() -> GraphBuilder:
    if _TRACE is None:
        raise RuntimeError("no active trace - bafe ops can only be called inside a function decorated with @bafe.jit")
    return _TRACE


class Tensor:
    """Symbolic tensor handle during tracing (bafe/python/bafe/__init__.py:123-177)."""
    __slots__ = ("node_id", "shape", "dtype", "_name")

    def __init__(self, node_id: int, shape: tuple, dtype: int, name: Optional[str] = None):
        self.node_id = node_id
        self.shape = shape
        self.dtype = dtype
        self._name = name

    def __add__(self, other: "Tensor") -> "Tensor":
        return _op("add", self, other)

    def __sub__(self, other: "Tensor") -> "Tensor":
        return _op("sub", self, other)

    def __mul__(self, other: "Tensor") -> "Tensor":
        return _op("mul", self, other)

    def __matmul__(self, other: "Tensor") -> "Tensor":
        if len(self.shape) < 2 or len(other.shape) < 2:
            raise ValueError("matmul requires rank>=2 tensors")
        if self.shape[-1] != other.shape[-2]:
            raise ValueError(f"matmul shape mismatch: {self.shape} @ {other.shape} (K dim must match)")
        return _op("matmul", self, other)

    @property
    def name(self) -> Optional[str]:
        return self._name

    def __repr__(self) -> str:
        return f"Tensor(shape={self.shape}, dtype={_BAFE_TO_NP[self.dtype]})"


def _op(op: str, *xs: Tensor, **attrs) -> Tensor:
    tb = _trace()
    nid = tb.add(op, [x.node_id for x in xs], **attrs)
    return Tensor(nid, tb.shape(nid), tb.dtype(nid))


def input(shape: Tuple[int, ...], dtype="float32", name: str = "x", layout: str = "row") -> Tensor:
    """Declare an input (bafe/python/bafe/__init__.py:196-218)."""
    tb = _trace()
    np_dt = np.dtype(dtype)
    if np_dt not in _NP_TO_BAFE:
        raise ValueError(f"unsupported dtype {dtype}; supported: {list(_NP_TO_BAFE)}")
    if layout not in LAYOUT_NAMES:
        raise ValueError(f"unsupported layout {layout!r}; supported: {list(LAYOUT_NAMES)}")
    nid = tb.add_input(name, tuple(int(s) for s in shape), _NP_TO_BAFE[np_dt], LAYOUT_NAMES[layout])
    return Tensor(nid, tb.shape(nid), _NP_TO_BAFE[np_dt], name=name)


def matmul(a: Tensor, b: Tensor) -> Tensor:
    return a @ b


def add(a: Tensor, b: Tensor) -> Tensor:
    return a + b


def sub(a: Tensor, b: Tensor) -> Tensor:
    return a - b


def mul(a: Tensor, b: Tensor) -> Tensor:
    return a * b


def relu(x: Tensor) -> Tensor:
    return _op("relu", x)


def sigmoid(x: Tensor) -> Tensor:
    return _op("sigmoid", x)


def tanh(x: Tensor) -> Tensor:
    return _op("tanh", x)


def neg(x: Tensor) -> Tensor:
    return _op("neg", x)


def bias_add(x: Tensor, bias: Tensor) -> Tensor:
    return _op("bias_add", x, bias)


def transpose(x: Tensor, perm: Tuple[int, ...]) -> Tensor:
    return _op("transpose", x, perm=list(perm))


def reduce_sum(x: Tensor, axes: Tuple[int, ...], keepdims: bool = False) -> Tensor:
    return _op("reduce_sum", x, axes=list(axes), keepdims=keepdims)


def reduce_max(x: Tensor, axes: Tuple[int, ...], keepdims: bool = False) -> Tensor:
    return _op("reduce_max", x, axes=list(axes), keepdims=keepdims)


def reshape(x: Tensor, shape: Tuple[int, ...]) -> Tensor:
    return _op("reshape", x, shape=list(shape))


def broadcast_to(x: Tensor, shape: Tuple[int, ...]) -> Tensor:
    return _op("broadcast_to", x, shape=list(shape))


def _layout_of(a: np.ndarray) -> str:
    """__init__.py:345-349: Fortran-contiguous rank>=2 arrays are "col"."""
    if a.ndim >= 2 and a.flags["F_CONTIGUOUS"] and not a.flags["C_CONTIGUOUS"]:
        return "col"
    return "row"


class JittedFunction:
    """A traced function compiled by the B200 backend (mirrors __init__.py:310-545).

    With autotune=True each call past the warm-up is timed on the DEVICE
    (CUDA events around the plan's kernels, copies excluded), logged with
    the graph's features and the plan's roofline prediction, and the
    learned model is refitted every refit_threshold records, after which
    the compiled plans are dropped so the next call re-plans
    (__init__.py:386-430 times by wall clock around the host call)."""

    def __init__(self, fn: Callable, autotune: bool = False):
        self._fn = fn
        self._compiled: dict = {}
        self._autotune = bool(autotune)
        self._call_count: dict = {}
        functools.update_wrapper(self, fn)

    def kernel_for(self, *args: np.ndarray) -> Kernel:
        key = tuple((a.shape, str(a.dtype), _layout_of(a)) for a in args)
        if key not in self._compiled:
            self._compiled[key] = self._compile(args)
        return self._compiled[key]

    def __call__(self, *args: np.ndarray) -> np.ndarray:
        if not args:
            raise TypeError("jitted function requires at least one input")
        for a in args:
            if not isinstance(a, np.ndarray):
                raise TypeError(f"expected numpy array, got {type(a)}")
        k = self.kernel_for(*args)
        # Keep each argument's memory layout: a col-major kernel reads the
        # Fortran buffer as is (__init__.py:369-380).
        ptrs = []
        keep = []
        for a in args:
            if not (a.flags["C_CONTIGUOUS"] or a.flags["F_CONTIGUOUS"]):
                a = np.ascontiguousarray(a)
            keep.append(a)
            ptrs.append(a.ctypes.data)
        out = np.zeros(k.out_shape, dtype=k.out_dtype)
        call = ptrs + [out.ctypes.data]
        if not self._autotune:
            k.call_host_ptrs(call)
            return out
        key = tuple((a.shape, str(a.dtype), _layout_of(a)) for a in args)
        cfg = lib.bafe_cuda_autotune_get_config()
        n = self._call_count.get(key, 0) + 1
        self._call_count[key] = n
        if n <= cfg.warmup_calls:
            k.call_host_ptrs(call)
            return out
        iters = cfg.timing_iters if cfg.timing_iters > 0 else 1
        total = 0.0
        for _ in range(iters):
            k.call_host_ptrs(call)
            total += lib.bafe_cuda_plan_last_device_ms(k.plan)
        features = (ctypes.c_double * _binding.BAFE_NUM_FEATURES)()
        lib.bafe_cuda_profiling_extract_features(ctypes.byref(k.graph), features)
        lib.bafe_cuda_profiling_add(graph_hash(k.graph).encode(), features, lib.bafe_cuda_plan_predict_ms(k.plan),
                                    total / iters, k.plan)
        log = lib.bafe_cuda_profiling_get_log().contents
        if cfg.refit_threshold > 0 and log.n > 0 and log.n % cfg.refit_threshold == 0:
            lib.bafe_cuda_profiling_refit()
            self._compiled.clear()
            lib.bafe_cuda_jit_invalidate_memory_cache()
        return out

    def _compile(self, args: Sequence[np.ndarray]) -> Kernel:
        return compile_graph(self._trace_graph(args))

    @property
    def n_args(self) -> int:
        return self._fn.__code__.co_argcount

    def _trace_graph(self, args: Sequence) -> GraphBuilder:
        """Trace the function on arguments of these shapes / dtypes / layouts."""
        global _TRACE
        _TRACE = GraphBuilder()
        try:
            tensors = []
            code = self._fn.__code__
            for i, a in enumerate(args):
                np_dt = np.dtype(a.dtype)
                if np_dt not in _NP_TO_BAFE:
                    raise TypeError(f"unsupported dtype {np_dt}")
                name = code.co_varnames[i] if i < len(code.co_varnames) else f"in{i}"
                tensors.append(input(a.shape, np_dt, name=name, layout=_layout_of(a)))
            result = self._fn(*tensors)
            if not isinstance(result, Tensor):
                raise TypeError(f"jitted function must return a Tensor, got {type(result)}")
            _TRACE.set_output(result.node_id)
            builder = _TRACE
        finally:
            _TRACE = None
        return builder


class FusedFunction(JittedFunction):
    """h = fuse(f, g): h(*f_args, *g_args[1:]) == g(f(*f_args), *g_args[1:]),
    compiled as ONE plan (__init__.py:758-916, fuse.c:12-125).  The graphs
    are concatenated with f's output feeding g's first input, so on the
    device the intermediate is a plan temporary -- or, when it is
    elementwise-consumed, never stored at all (the lowering merges the
    chain into one region or into the GEMM's epilogue) -- and it never
    crosses PCIe.  Chains: fuse(fuse(f, g), h)."""

    def __init__(self, func_a, func_b):
        self._func_a = func_a
        self._func_b = func_b
        self._compiled = {}
        self._autotune = False
        self._call_count = {}
        self._fn = func_a._fn
        # name / doc of f only: copying f's __dict__ (update_wrapper's default)
        # would overwrite _func_a / _func_b when f is itself fused, which is
        # what breaks 3-way chains in the reference (its test_fuse.py xfails
        # fuse(fuse(f, g), h))
        functools.update_wrapper(self, func_a._fn, updated=())

    @property
    def n_args(self) -> int:
        return self._func_a.n_args + self._func_b.n_args - 1

    def _trace_graph(self, args: Sequence) -> GraphBuilder:
        na = self._func_a.n_args
        if len(args) != self.n_args:
            raise TypeError(f"fused function expects {self.n_args} args ({na} for f + "
                            f"{self._func_b.n_args - 1} for g, since g's first input is f's output), got {len(args)}")
        ga = self._func_a._trace_graph(args[:na])
        out = ga.output
        # g is traced on a row-major stand-in of f's output, as the reference
        # does (a zero array, __init__.py:853-855); concat then rewires g's
        # uses of it to f's output node.  Zero strides: nothing is allocated.
        shape = ga.shape(out)
        stand_in = np.lib.stride_tricks.as_strided(np.zeros(1, _BAFE_TO_NP[ga.dtype(out)]), shape=shape,
                                                   strides=(0,) * len(shape))
        gb = self._func_b._trace_graph((stand_in,) + tuple(args[na:]))
        return GraphBuilder.concat(ga, gb)


def fuse(func_a, func_b):
    """bafe.fuse (__init__.py:918-938)."""
    if not isinstance(func_a, JittedFunction) or not isinstance(func_b, JittedFunction):
        raise TypeError("fuse() requires @bafe.jit-decorated or fused functions")
    return FusedFunction(func_a, func_b)


def jit(fn: Callable = None, *, autotune: bool = False, **_ignored):
    """Decorator (bafe.jit).  autotune=True: device-timed profiling loop (see
    JittedFunction).  The reference's search options configure its
    optimizer, which this backend does not run; they are accepted and
    ignored."""
    if fn is not None:
        return JittedFunction(fn, autotune=autotune)
    return lambda f: JittedFunction(f, autotune=autotune)


# ------------------------------------------------ cost model / autotune --
# Same names and return shapes as the reference's Python API
# (__init__.py:646-717), on the backend's device-timed profiling state.

def configure_autotune(refit_threshold: int = 20, invalidation_drift: float = 0.25, warmup_calls: int = 2,
                       timing_iters: int = 5) -> None:
    cfg = lib.bafe_cuda_autotune_config_default()
    cfg.enabled = True
    cfg.refit_threshold = int(refit_threshold)
    cfg.invalidation_drift = float(invalidation_drift)
    cfg.warmup_calls = int(warmup_calls)
    cfg.timing_iters = int(timing_iters)
    lib.bafe_cuda_autotune_configure(ctypes.byref(cfg))


def autotune_stats() -> dict:
    s = lib.bafe_cuda_autotune_get_stats()
    return {"total_calls": s.total_calls, "total_compiles": s.total_compiles, "total_refits": s.total_refits,
            "total_invalidations": s.total_invalidations, "last_refit_r_squared": s.last_refit_r_squared,
            "log_size": s.log_size}


def autotune_refit() -> int:
    return int(lib.bafe_cuda_profiling_refit())


def autotune_model() -> dict:
    m = lib.bafe_cuda_profiling_get_model().contents
    return {"weights": [m.weights[i] for i in range(_binding.BAFE_NUM_FEATURES)], "bias": m.bias,
            "r_squared": m.r_squared, "n_samples": m.n_samples, "valid": bool(m.valid)}


def autotune_dump_log(path: str) -> int:
    return int(lib.bafe_cuda_profiling_dump_jsonl(path.encode("utf-8")))


def autotune_reset() -> None:
    lib.bafe_cuda_profiling_reset()


def extract_features(graph: BafeGraph) -> List[float]:
    f = (ctypes.c_double * _binding.BAFE_NUM_FEATURES)()
    lib.bafe_cuda_profiling_extract_features(ctypes.byref(graph), f)
    return list(f)


def calibrate(device: int = 0, what: int = 3) -> None:
    """Measure the B200 figures of the hardware model (bafe_cuda_calibrate)."""
    check(lib.bafe_cuda_calibrate(int(device), int(what)), "calibrate")


def hardware_model(device: int = -1) -> dict:
    """BAFE's bafe_hardware_model filled with this GPU's figures; key
    'measured' tells whether bafe_cuda_calibrate measured them."""
    h = _binding.BafeHardwareModel()
    rc = lib.bafe_cuda_hardware_model(int(device), ctypes.byref(h))
    d = {name: getattr(h, name) for name, _ in h._fields_}
    d["measured"] = rc == 1
    return d


__all__ = [
    "Tensor", "jit", "input", "matmul", "add", "sub", "mul", "relu", "sigmoid", "tanh", "neg", "bias_add",
    "transpose", "reduce_sum", "reduce_max", "reshape", "broadcast_to", "GraphBuilder", "compile_graph",
    "Kernel", "set_option", "get_option", "jit_stats", "jit_clear", "jit_invalidate_memory_cache",
    "set_cache_dir", "cache_dir", "graph_hash", "launch_count", "last_error", "synchronize",
    "configure_autotune", "autotune_stats", "autotune_refit", "autotune_model", "autotune_dump_log",
    "autotune_reset", "extract_features", "calibrate", "hardware_model", "fuse", "FusedFunction",
]
