"""ctypes binding to libbafe_cuda.so (the C ABI declared in include/bafe_cuda.h).

The graph structs mirror BAFE's POD graph byte for byte: the reference
binds the same layout at bafe/python/bafe/_binding.py:62-112 (types.h:55-58,
ops.h:239-250, ir.h:133-155).  The backend reads these structs by pointer,
so the field order and types are fixed by the reference's ABI.

The library is found at $BAFE_CUDA_LIB, else next to this package
(../lib/libbafe_cuda.so).  There is no fallback: without the CUDA library
the import fails.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import (POINTER, Structure, c_bool, c_char, c_char_p, c_double, c_int, c_int32, c_int64,
                    c_size_t, c_void_p)
from pathlib import Path

BAFE_MAX_RANK = 8
BAFE_MAX_ATTR_LEN = 32
BAFE_MAX_CHILDREN = 4
BAFE_MAX_NODES = 4096

DTYPE_F32, DTYPE_F64, DTYPE_I32, DTYPE_I64, DTYPE_F16, DTYPE_BF16 = range(6)
LAYOUT_ROW, LAYOUT_COL, LAYOUT_BLOCKED, LAYOUT_TC = range(4)


class BafeShape(Structure):
    _fields_ = [("dims", c_int32 * BAFE_MAX_RANK), ("rank", c_int32)]


class BafeOpAttrs(Structure):
    _fields_ = [
        ("n_axes", c_int32), ("axes", c_int32 * BAFE_MAX_ATTR_LEN),
        ("n_perm", c_int32), ("perm", c_int32 * BAFE_MAX_ATTR_LEN),
        ("n_shape", c_int32), ("shape", c_int32 * BAFE_MAX_ATTR_LEN),
        ("keepdims", c_bool), ("scalar_value", c_double), ("has_scalar", c_bool),
        ("name", c_char * BAFE_MAX_ATTR_LEN),
    ]


class BafeNode(Structure):
    _fields_ = [
        ("id", c_int32), ("op_name", c_char_p), ("attrs", BafeOpAttrs),
        ("n_children", c_int), ("children", c_int32 * BAFE_MAX_CHILDREN),
        ("shape", BafeShape), ("dtype", c_int), ("layout", c_int),
        ("input_name", c_char * BAFE_MAX_ATTR_LEN), ("is_input", c_bool),
        ("is_constant", c_bool), ("const_value", c_double),
    ]


class BafeGraph(Structure):
    _fields_ = [
        ("nodes", BafeNode * BAFE_MAX_NODES), ("n_nodes", c_int),
        ("inputs", c_int32 * BAFE_MAX_NODES), ("n_inputs", c_int),
        ("outputs", c_int32 * BAFE_MAX_NODES), ("n_outputs", c_int),
    ]


class BafeJitStats(Structure):
    _fields_ = [("hits", c_int), ("misses", c_int), ("compiles", c_int), ("compile_failures", c_int)]


# cost.h:27-44 and profiling.h:37-75, 137-143 (layouts of the reference).
BAFE_NUM_FEATURES = 8
BAFE_PROFILING_LOG_SIZE = 4096


class BafeHardwareModel(Structure):
    _fields_ = [
        ("peak_gflops", c_double), ("clock_ghz", c_double), ("simd_width", c_int),
        ("l1_cache_size", c_int), ("l2_cache_size", c_int), ("l3_cache_size", c_int),
        ("l1_bandwidth_gbs", c_double), ("l2_bandwidth_gbs", c_double), ("l3_bandwidth_gbs", c_double),
        ("dram_bandwidth_gbs", c_double), ("f32_flop_rate", c_double), ("f64_flop_rate", c_double),
        ("f16_flop_rate", c_double), ("bf16_flop_rate", c_double), ("i32_flop_rate", c_double),
        ("i64_flop_rate", c_double),
    ]


class BafeProfilingRecord(Structure):
    _fields_ = [("graph_hash", c_char * 65), ("features", c_double * BAFE_NUM_FEATURES),
                ("predicted_cost", c_double), ("observed_ms", c_double), ("kernel_id", c_int)]


class BafeProfilingLog(Structure):
    _fields_ = [("records", BafeProfilingRecord * BAFE_PROFILING_LOG_SIZE), ("n", c_int), ("head", c_int),
                ("wrapped", c_bool)]


class BafeLearnedCostModel(Structure):
    _fields_ = [("weights", c_double * BAFE_NUM_FEATURES), ("bias", c_double), ("r_squared", c_double),
                ("n_samples", c_int), ("valid", c_bool)]


class BafeAutotuneStats(Structure):
    _fields_ = [("total_calls", c_int), ("total_compiles", c_int), ("total_refits", c_int),
                ("total_invalidations", c_int), ("last_refit_r_squared", c_double), ("log_size", c_int)]


class BafeAutotuneConfig(Structure):
    _fields_ = [("enabled", c_bool), ("refit_threshold", c_int), ("invalidation_drift", c_double),
                ("warmup_calls", c_int), ("timing_iters", c_int)]


PACKAGE_ROOT = Path(__file__).resolve().parent.parent


def library_path() -> str:
    env = os.environ.get("BAFE_CUDA_LIB")
    if env:
        return env
    return str(PACKAGE_ROOT / "lib" / "libbafe_cuda.so")


def _load() -> ctypes.CDLL:
    path = library_path()
    if not Path(path).exists():
        raise ImportError(
            f"libbafe_cuda.so not found at {path}: build it with "
            f"`make -C {PACKAGE_ROOT}` (or __graft_entry__.build())")
    lib = ctypes.CDLL(path)
    G = POINTER(BafeGraph)
    proto = {
        "bafe_cuda_version": ([], c_int),
        "bafe_cuda_jit_hash_graph": ([G, c_char_p, c_size_t], c_int),
        "bafe_cuda_jit_get_or_compile": ([G, c_char_p, c_size_t], c_void_p),
        "bafe_cuda_jit_set_cache_dir": ([c_char_p], None),
        "bafe_cuda_jit_cache_dir": ([], c_char_p),
        "bafe_cuda_jit_get_stats": ([], BafeJitStats),
        "bafe_cuda_jit_clear": ([], None),
        "bafe_cuda_jit_invalidate_memory_cache": ([], None),
        "bafe_cuda_plan_of": ([c_void_p], c_int),
        "bafe_cuda_plan_num_inputs": ([c_int], c_int),
        "bafe_cuda_plan_describe": ([c_int, c_char_p, c_size_t], c_int),
        "bafe_cuda_plan_output_bytes": ([c_int], c_int64),
        "bafe_cuda_plan_input_bytes": ([c_int, c_int], c_int64),
        "bafe_cuda_plan_row_split": ([c_int, POINTER(c_int64), POINTER(c_int64), c_int, POINTER(c_int64)], c_int),
        "bafe_cuda_run_device": ([c_int, POINTER(c_void_p), c_int, c_void_p], c_int),
        "bafe_cuda_run_device_ksliced": ([c_int, POINTER(c_void_p), c_int, c_void_p, c_int, POINTER(ctypes.c_int64),
                                          POINTER(c_void_p)], c_int),
        "bafe_cuda_plan_k_slice_align": ([c_int], c_int),
        "bafe_cuda_relay_alloc": ([c_int, c_int64, POINTER(ctypes.c_uint64), c_void_p], c_int),
        "bafe_cuda_relay_free": ([ctypes.c_uint64], c_int),
        "bafe_cuda_relay_open": ([c_int, c_void_p, POINTER(ctypes.c_uint64)], c_int),
        "bafe_cuda_relay_close": ([ctypes.c_uint64], c_int),
        "bafe_cuda_signal_wait": ([ctypes.c_uint64, ctypes.c_uint32, c_void_p], c_int),
        "bafe_cuda_signal_write": ([ctypes.c_uint64, ctypes.c_uint32, c_void_p], c_int),
        "bafe_cuda_relay_step": ([ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, POINTER(c_int64),
                                  c_int, ctypes.c_uint32, c_int, c_void_p], c_int),
        "bafe_cuda_plan_num_steps": ([c_int], c_int),
        "bafe_cuda_run_device_timed": ([c_int, POINTER(c_void_p), c_int, c_void_p, POINTER(c_void_p), c_int], c_int),
        "bafe_cuda_run_host": ([c_int, POINTER(c_void_p), c_int], c_int),
        "bafe_cuda_run_host_resident": ([c_int, POINTER(c_void_p), c_int, POINTER(ctypes.c_ubyte), c_void_p], c_int),
        "bafe_cuda_synchronize": ([], c_int),
        "bafe_cuda_last_error": ([c_char_p, c_size_t], c_int),
        "bafe_cuda_clear_error": ([], None),
        "bafe_cuda_set_option": ([c_char_p, c_char_p], c_int),
        "bafe_cuda_get_option": ([c_char_p, c_char_p, c_size_t], c_int),
        "bafe_cuda_launch_count": ([], c_int64),
        "bafe_cuda_abi_size": ([c_int], c_int64),
        "bafe_cuda_gemm_3xtf32_static_scratch": ([c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int,
                                                  c_int, c_void_p], c_int),
        "bafe_cuda_calibrate": ([c_int, c_int], c_int),
        "bafe_cuda_selftest_wait_timeout": ([c_int, POINTER(ctypes.c_uint), POINTER(c_double)], c_int),
        "bafe_cuda_hardware_model": ([c_int, POINTER(BafeHardwareModel)], c_int),
        "bafe_cuda_plan_predict_ms": ([c_int], c_double),
        "bafe_cuda_plan_last_device_ms": ([c_int], c_double),
        "bafe_cuda_time_device": ([c_int, POINTER(c_void_p), c_int, c_void_p, c_int, POINTER(c_double)], c_int),
        "bafe_cuda_profiling_init": ([], None),
        "bafe_cuda_profiling_reset": ([], None),
        "bafe_cuda_profiling_extract_features": ([G, POINTER(c_double)], None),
        "bafe_cuda_profiling_add": ([c_char_p, POINTER(c_double), c_double, c_double, c_int], None),
        "bafe_cuda_profiling_get_log": ([], POINTER(BafeProfilingLog)),
        "bafe_cuda_profiling_dump_jsonl": ([c_char_p], c_int),
        "bafe_cuda_profiling_refit": ([], c_int),
        "bafe_cuda_profiling_get_model": ([], POINTER(BafeLearnedCostModel)),
        "bafe_cuda_profiling_predict_log": ([POINTER(c_double)], c_double),
        "bafe_cuda_profiling_predict_ms": ([POINTER(c_double)], c_double),
        "bafe_cuda_autotune_config_default": ([], BafeAutotuneConfig),
        "bafe_cuda_autotune_configure": ([POINTER(BafeAutotuneConfig)], None),
        "bafe_cuda_autotune_get_config": ([], BafeAutotuneConfig),
        "bafe_cuda_autotune_get_stats": ([], BafeAutotuneStats),
        "bafe_cuda_autotune_dispatch": ([c_void_p, POINTER(c_void_p), c_int, G, c_char_p, c_double], c_double),
    }
    for name, (args, res) in proto.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


lib = _load()

# Every symbol include/bafe_cuda.h declares (checked by the CPU test suite).
EXPORTED_SYMBOLS = (
    "bafe_cuda_jit_hash_graph", "bafe_cuda_jit_get_or_compile", "bafe_cuda_jit_set_cache_dir",
    "bafe_cuda_jit_cache_dir", "bafe_cuda_jit_get_stats", "bafe_cuda_jit_clear",
    "bafe_cuda_jit_invalidate_memory_cache", "bafe_cuda_version", "bafe_cuda_plan_of",
    "bafe_cuda_plan_num_inputs", "bafe_cuda_plan_describe", "bafe_cuda_plan_output_bytes",
    "bafe_cuda_plan_input_bytes", "bafe_cuda_plan_row_split", "bafe_cuda_run_device", "bafe_cuda_run_device_ksliced", "bafe_cuda_plan_k_slice_align",
    "bafe_cuda_relay_alloc", "bafe_cuda_relay_free", "bafe_cuda_relay_open", "bafe_cuda_relay_close",
    "bafe_cuda_signal_wait", "bafe_cuda_signal_write", "bafe_cuda_relay_step", "bafe_cuda_plan_num_steps", "bafe_cuda_run_device_timed", "bafe_cuda_run_host", "bafe_cuda_run_host_resident", "bafe_cuda_synchronize", "bafe_cuda_last_error",
    "bafe_cuda_clear_error", "bafe_cuda_set_option", "bafe_cuda_get_option", "bafe_cuda_launch_count",
    "bafe_cuda_abi_size", "bafe_cuda_gemm_3xtf32_static_scratch",
    "bafe_cuda_calibrate", "bafe_cuda_hardware_model", "bafe_cuda_plan_predict_ms", "bafe_cuda_plan_last_device_ms",
    "bafe_cuda_time_device", "bafe_cuda_profiling_init", "bafe_cuda_profiling_reset",
    "bafe_cuda_profiling_extract_features", "bafe_cuda_profiling_add", "bafe_cuda_profiling_get_log",
    "bafe_cuda_profiling_dump_jsonl", "bafe_cuda_profiling_refit", "bafe_cuda_profiling_get_model",
    "bafe_cuda_profiling_predict_log", "bafe_cuda_profiling_predict_ms", "bafe_cuda_autotune_config_default",
    "bafe_cuda_autotune_configure", "bafe_cuda_autotune_get_config", "bafe_cuda_autotune_get_stats",
    "bafe_cuda_autotune_dispatch", "bafe_cuda_selftest_wait_timeout",
)


def last_error() -> tuple[int, str]:
    buf = ctypes.create_string_buffer(8192)
    code = lib.bafe_cuda_last_error(buf, len(buf))
    return code, buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    """Raise RuntimeError with the library's message when rc is nonzero."""
    if rc != 0:
        code, msg = last_error()
        raise RuntimeError(f"{what} failed (code {rc}): {msg}")
