"""Cost model and profiling layer, on CPU.

The backend's profiling log, feature vector, JSONL dump and least-squares
refit restate BAFE's profiling.c; they are checked bit for bit against the
reference's own library through tests/golden/autotune_golden.json (made by
tests/golden/make_autotune_golden.py), then exercised the way the
reference's tests exercise its own (bafe/tests/test_autotune.py).  The B200
hardware model and the plan roofline are checked without a GPU on their
nominal figures; the device-timed parts are in test_gpu_autotune.py."""
import ctypes
import json
from pathlib import Path

import numpy as np
import pytest

import bafe_b200 as bafe
import cases
from bafe_b200 import _binding
from bafe_b200._binding import BAFE_NUM_FEATURES, lib
from bafe_b200.graph import GraphBuilder

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "autotune_golden.json").read_text())
NF = BAFE_NUM_FEATURES


@pytest.fixture(autouse=True)
def _reset_profiling():
    lib.bafe_cuda_profiling_reset()
    yield
    lib.bafe_cuda_profiling_reset()


def _features(g) -> list:
    f = (ctypes.c_double * NF)()
    lib.bafe_cuda_profiling_extract_features(ctypes.byref(g), f)
    return list(f)


def _traced(case) -> GraphBuilder:
    return cases.traced_graph(case)


# ------------------------------------------------------------ vs reference --

@pytest.mark.parametrize("case", cases.CASES, ids=[c["name"] for c in cases.CASES])
def test_features_equal_the_references(case):
    want = GOLDEN["features"][case["name"]]
    meta, _, _ = cases.load(case["name"])
    g_opt = cases.graph_from_nodes(meta["nodes"], meta["input_ids"], meta["root"])
    assert [v.hex() for v in _features(g_opt)] == want["optimized"]
    assert [v.hex() for v in _features(_traced(case).graph)] == want["traced"]


@pytest.mark.parametrize("name", sorted(GOLDEN["refit"]))
def test_refit_equals_the_references(name):
    ref = GOLDEN["refit"][name]
    for k, (f, ms) in enumerate(ref["records"]):
        lib.bafe_cuda_profiling_add(b"h%03d" % k, (ctypes.c_double * NF)(*f), 1.0, float.fromhex(ms), k)
    assert lib.bafe_cuda_profiling_refit() == ref["rc"]
    m = lib.bafe_cuda_profiling_get_model().contents
    assert m.valid == ref["valid"] and m.n_samples == ref["n_samples"]
    got = [m.weights[i] for i in range(NF)] + [m.bias, m.r_squared]
    want = [float.fromhex(x) for x in ref["weights"]] + [float.fromhex(ref["bias"]), float.fromhex(ref["r_squared"])]
    assert got == want
    for p, lp in zip(ref["probes"], ref["predict_log"]):
        assert lib.bafe_cuda_profiling_predict_log((ctypes.c_double * NF)(*p)) == float.fromhex(lp)


def test_jsonl_dump_equals_the_references(tmp_path):
    lib.bafe_cuda_profiling_add(b"deadbeefdeadbeefdeadbeef", (ctypes.c_double * NF)(*([1.5] * NF)), 3.0, 0.5, 0)
    lib.bafe_cuda_profiling_add(b"cafef00d", (ctypes.c_double * NF)(*[0.125 * i for i in range(NF)]), 4.25, 1e-3, 7)
    p = tmp_path / "log.jsonl"
    assert lib.bafe_cuda_profiling_dump_jsonl(str(p).encode()) == 2
    assert p.read_text() == GOLDEN["jsonl"]


# ------------------------------------- the reference's own checks, mirrored --

def _mm_relu(M=16, N=16, K=16):
    g = GraphBuilder()
    a = g.add_input("A", (M, K), 0, 0)
    b = g.add_input("B", (K, N), 0, 0)
    g.set_output(g.add("relu", [g.add("matmul", [a, b])]))
    return g


def test_feature_vector_of_matmul_relu():
    v = _features(_mm_relu().graph)
    assert v[:4] == [2.0, 2.0, 1.0, 0.0] and v[4] > 0 and v[5] > 0 and v[6:] == [2.0, 0.0]
    w = _features(_mm_relu(64, 64, 64).graph)
    assert abs(v[4] - w[4]) > 0.1 and abs(v[5] - w[5]) > 0.1


def test_log_records_and_ring_buffer():
    lib.bafe_cuda_profiling_add(b"abc123", (ctypes.c_double * NF)(*([1.0] * NF)), 5.0, 1.5, 0)
    log = lib.bafe_cuda_profiling_get_log().contents
    assert log.n == 1 and log.records[0].graph_hash.startswith(b"abc123")
    assert (log.records[0].predicted_cost, log.records[0].observed_ms) == (5.0, 1.5)
    for i in range(_binding.BAFE_PROFILING_LOG_SIZE + 10):
        lib.bafe_cuda_profiling_add(b"h", (ctypes.c_double * NF)(), float(i), 0.1, i)
    log = lib.bafe_cuda_profiling_get_log().contents
    assert log.n == _binding.BAFE_PROFILING_LOG_SIZE and log.wrapped
    assert bafe.autotune_stats()["log_size"] == _binding.BAFE_PROFILING_LOG_SIZE


def test_refit_needs_five_samples_and_learns_a_trend():
    lib.bafe_cuda_profiling_add(b"h", (ctypes.c_double * NF)(*([1.0] * NF)), 1.0, 1.0, 0)
    assert lib.bafe_cuda_profiling_refit() != 0
    lib.bafe_cuda_profiling_reset()
    for i in range(20):
        f = (ctypes.c_double * NF)()
        f[4] = float(i + 1)
        lib.bafe_cuda_profiling_add(b"h", f, 1.0, float(i + 1) * 0.01, 0)
    assert lib.bafe_cuda_profiling_refit() == 0
    m = bafe.autotune_model()
    assert m["valid"] and m["n_samples"] == 20 and m["weights"][4] > 0 and m["r_squared"] > 0.3
    assert lib.bafe_cuda_profiling_predict_ms((ctypes.c_double * NF)(*([1.0] * NF))) > 0


def test_autotune_config_round_trip():
    cfg = lib.bafe_cuda_autotune_config_default()
    assert (cfg.refit_threshold, cfg.invalidation_drift, cfg.warmup_calls, cfg.timing_iters) == (20, 0.25, 2, 5)
    bafe.configure_autotune(refit_threshold=99, invalidation_drift=0.5, warmup_calls=3, timing_iters=7)
    got = lib.bafe_cuda_autotune_get_config()
    assert (got.enabled, got.refit_threshold, got.invalidation_drift, got.warmup_calls, got.timing_iters) == \
        (True, 99, 0.5, 3, 7)
    bafe.configure_autotune()


def test_dispatch_rejects_foreign_function_pointers():
    g = _mm_relu()
    arr = (ctypes.c_void_p * 3)()
    assert lib.bafe_cuda_autotune_dispatch(ctypes.c_void_p(1234), arr, 3, ctypes.byref(g.graph), None, 0.0) == -1.0


# ------------------------------------------------ hardware model, roofline --

def test_nominal_hardware_model_without_a_gpu():
    if __import__("conftest").gpu_available():
        pytest.skip("this checks the figures used before any calibration on a machine without a GPU")
    h = bafe.hardware_model()
    assert not h["measured"]
    assert h["dram_bandwidth_gbs"] == 7700.0 and h["l2_bandwidth_gbs"] > h["dram_bandwidth_gbs"]
    assert h["peak_gflops"] == pytest.approx(1100e3 / 3)          # 3xTF32 at the nominal TF32 rate
    assert h["l3_cache_size"] == h["l2_cache_size"] and h["simd_width"] == 32
    assert h["f32_flop_rate"] == 1.0 and 0 < h["f64_flop_rate"] < 1


def test_plan_roofline_prediction():
    g = GraphBuilder()
    x, y, z = (g.add_input(n, (1 << 26,), 0, 0) for n in "XYZ")
    g.set_output(g.add("relu", [g.add("add", [g.add("mul", [x, y]), z])]))
    ew = bafe.compile_graph(g)
    ms = lib.bafe_cuda_plan_predict_ms(ew.plan)
    h = bafe.hardware_model()
    bytes_ = 16.0 * (1 << 26)
    assert ms == pytest.approx(bytes_ / (h["dram_bandwidth_gbs"] * 1e9) * 1e3, rel=0.05)
    bafe.set_option("gemm_precision", "3xtf32")
    gm = bafe.compile_graph(_mm_relu(4096, 4096, 4096))
    t = lib.bafe_cuda_plan_predict_ms(gm.plan)
    flops = 2.0 * 4096 ** 3
    assert t >= flops / (h["peak_gflops"] * 1e9) * 1e3
    assert lib.bafe_cuda_plan_predict_ms(-5) == -1.0
    assert lib.bafe_cuda_plan_last_device_ms(ew.plan) == -1.0      # never called
