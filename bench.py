#!/usr/bin/env python
"""Benchmark of the BAFE hot path on B200.

Headline workload (one "step" = one call of the plan):
  gemm: relu(matmul(A,B) + C), fp32, M=N=K=16384, A row-major, B tagged
        BLOCKED (row-major storage), C full -- one fused GEMM+epilogue
        kernel.  Metric TFLOP/s (2*M*N*K per call).  Under torchrun the M
        rows are split into contiguous row panels, one per rank; B is
        broadcast once from rank 0 over NCCL (outside the timed region, as
        the runtime keeps B resident; its time is reported separately).
Secondary (same JSON line, keys "gemm_bf16", "ew", "transpose", "configs"):
  gemm_bf16: the same fused GEMM with bf16 A, B, C and output (kind::f16
        tensor cores, f32 accumulation).
  ew:   relu(add(mul(X,Y),Z)) over 2^28 fp32 elements (1 GiB per vector),
        range-split across ranks with no collective.  Metric GB/s
        (16 bytes per element).
  transpose: materialisation of transpose(X), X 16384 x 16384 fp32; ranks
        own output row blocks (input column panels), no collective.
        Metric GB/s (8 bytes per element).
  configs: the reference's other benchmark configurations on rank 0's GPU:
        relu(matmul(A,B)+C) 64^3 and matmul 256^3 (B row- / col-major) in
        microseconds per call (launch-latency bound), relu(add(matmul(A,B),
        mul(C,D))) 4096^3 in TFLOP/s.

value:   device-resident inputs, CUDA events around every step on the
         launching stream, max over ranks; inputs are larger than L2
         (126 MB), so no flush is needed between steps.
e2e:     the same metric through the C-ABI host function (host pointers,
         pinned): every step copies its inputs host->device and the
         result device->host inside the timed region (row-streamed).  For
         the GEMM under torchrun each rank copies its row panels of A and C
         and a 1/N slab of B, and an NCCL all-gather completes B on every
         rank (bafe_cuda_run_host_resident), all inside the timed region.
cpu_baseline: the reference's own generated C kernel (oracle/_ref, built
         from the reference sources) on a bounded row-panel / chunk sample,
         1 core, rank 0 only.  Falls back to the oracle restatement.

--impl reference runs the reference's CPU implementation alone, on every
host core (one process per core, each a row panel / chunk of the same
workload), and prints the same metric.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "bafe-basic-algibra-fusion-engine-_b200"
sys.path.insert(0, str(PKG))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

GEMM_M = GEMM_N = GEMM_K = 16384
EW_N = 1 << 28
TR_N = 16384
STD = 1.0 / math.sqrt(GEMM_K)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--precision", default=os.environ.get("BAFE_GEMM_PRECISION", "auto"))
    p.add_argument("--e2e-steps", type=int, default=3, help="0 skips the host-pointer measurement")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--only", choices=["gemm", "gemm_tf32", "gemm_bf16", "ew", "transpose"], default=None,
                   help="run one workload (profiling); prints its own line")
    p.add_argument("--gemm-size", type=int, default=GEMM_M, help="M=N=K (profiling smaller cases)")
    p.add_argument("--gemm-epilogue", choices=["c", "mul_cd"], default="c",
                   help="c: relu(matmul(A,B)+C) (the headline); mul_cd: relu(add(matmul(A,B), mul(C,D))), "
                        "the 4096^3 configuration's epilogue, for profiling it at any size")
    p.add_argument("--ew-elements", type=int, default=EW_N)
    p.add_argument("--transpose-size", type=int, default=TR_N, help="transpose of an S x S fp32 matrix")
    return p.parse_args()


def peaks():
    """(hbm GB/s, bf16 burst TFLOP/s, bf16 sustained TFLOP/s, source)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        burst = d.get("bf16_tflops", 1590.0)
        return d.get("hbm_gbs", 6650.0), burst, d.get("bf16_tflops_sustained", burst), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# ------------------------------------------------------------- clocks --

class Clocks:
    """nvidia-smi sampler running during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"bafe_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for nm, v in zip(names, f[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        self.path.unlink(missing_ok=True)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons)}


# ------------------------------------------------------------ workloads --

def gemm_config(S: int) -> dict:
    """The headline workload's `config`, identical in both arms."""
    return {"workload": f"relu(matmul(A,B)+C) M=N=K={S} fp32, A row-major, B BLOCKED tag, "
                        f"A, B, C i.i.d. N(0, 1/sqrt(K)) (std 1/{int(round(math.sqrt(S)))})",
            "l2": "inputs larger than L2 (1 GiB each); no flush" if S >= 8192 else "inputs smaller than L2"}


def roofline_basis(c, clocks: dict, div: float):
    """(peak, basis name, burst peak, sustained peak) for a tensor-core
    kernel whose rate is the bf16 peak / div.  A timed region whose median
    SM clock stayed within 5 % of the maximum ran as a burst; one the power
    cap held lower is measured against the sustained (power-capped) peak."""
    burst, sustained = c.bf16_peak / div, c.bf16_sustained / div
    med, mx = clocks.get("sm_mhz"), clocks.get("sm_max_mhz")
    if med and mx and med >= 0.95 * mx:
        return burst, "burst", burst, sustained
    return sustained, "sustained", burst, sustained


def gemm_graph(m_rows: int, size: int = GEMM_N, epilogue: str = "c"):
    import bafe_b200 as bafe
    g = bafe.GraphBuilder()
    a = g.add_input("A", (m_rows, size), 0, 0)
    b = g.add_input("B", (size, size), 0, 2)      # BLOCKED tag, row-major storage
    c = g.add_input("C", (m_rows, size), 0, 0)
    if epilogue == "mul_cd":
        d = g.add_input("D", (m_rows, size), 0, 0)
        g.set_output(g.add("relu", [g.add("add", [g.add("matmul", [a, b]), g.add("mul", [c, d])])]))
    else:
        g.set_output(g.add("relu", [g.add("add", [g.add("matmul", [a, b]), c])]))
    return g


def ew_graph(n: int):
    import bafe_b200 as bafe
    g = bafe.GraphBuilder()
    ids = [g.add_input(nm, (n,), 0, 0) for nm in "XYZ"]
    g.set_output(g.add("relu", [g.add("add", [g.add("mul", [ids[0], ids[1]]), ids[2]])]))
    return g


def transpose_graph(rows: int, cols: int):
    import bafe_b200 as bafe
    g = bafe.GraphBuilder()
    x = g.add_input("X", (rows, cols), 0, 0)
    g.set_output(g.add("transpose", [x], perm=[1, 0]))
    return g


def time_steps(torch, kernel, ins, out, steps, warmup, per_kernel=False):
    """Per-step CUDA-event durations (ms) on the launching stream.  With
    per_kernel, the plan also records events around each of its launch steps
    inside the timed steps (bafe_cuda_run_device_timed), and the mean
    duration of each plan step is returned as a fourth value."""
    s = torch.cuda.current_stream()
    n_k = kernel.num_steps if per_kernel else 0
    kev = [[torch.cuda.Event(enable_timing=True) for _ in range(2 * n_k)] for _ in range(steps)]
    for evs in kev:                       # create the CUDA events outside the timed region
        for e in evs:
            e.record(s)
    for _ in range(warmup):
        kernel.run_torch(ins, out, s)
    torch.cuda.synchronize()
    time.sleep(0.3)   # let the clock sampler (started by the caller) take its first samples
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    launches0 = __import__("bafe_b200").launch_count()
    ev[0].record(s)
    for i in range(steps):
        if n_k:
            kernel.run_torch_timed(ins, out, kev[i], s)
        else:
            kernel.run_torch(ins, out, s)
        ev[i + 1].record(s)
    torch.cuda.synchronize()
    launches = __import__("bafe_b200").launch_count() - launches0
    per = [ev[i].elapsed_time(ev[i + 1]) for i in range(steps)]
    if not per_kernel:
        return per, ev[0].elapsed_time(ev[steps]), launches
    step_ms = [statistics.mean(kev[i][2 * j].elapsed_time(kev[i][2 * j + 1]) for i in range(steps)) for j in range(n_k)]
    return per, ev[0].elapsed_time(ev[steps]), launches, step_ms


def time_bcast_steps(c, kernel, ins, out, bounds, free_sms, steps, warmup):
    """Steps whose B arrives inside the step: rank 0's B is broadcast slab by
    slab (rows [bounds[j], bounds[j+1])) over NCCL on a side stream, and the
    plan runs in K slices, slice j waiting for slab j
    (Kernel.run_torch_ksliced); bounds [0, K] is the broadcast followed by
    the whole GEMM.  Every step's broadcast starts after the previous step's
    work (an event on the launching stream).  -> (max-over-ranks ms of the
    timed region, GEMM launches counted)."""
    import bafe_b200 as bafe
    from bafe_b200.parallel import broadcast_slabs
    torch = c.torch
    cur = torch.cuda.current_stream()
    comm = torch.cuda.Stream()
    bafe.set_option("kslice_free_sms", str(free_sms))

    def step(start):
        start.record(cur)
        comm.wait_event(start)
        evs = broadcast_slabs(ins[1], bounds, c.dist, 0, comm)
        kernel.run_torch_ksliced(ins, out, bounds, ready=evs, stream=cur)

    try:
        for _ in range(warmup):
            step(torch.cuda.Event())
        torch.cuda.synchronize()
        c.barrier()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
        launches0 = bafe.launch_count()
        for i in range(steps):
            step(ev[i])
        ev[steps].record(cur)
        torch.cuda.synchronize()
        launches = bafe.launch_count() - launches0
    finally:
        bafe.set_option("kslice_free_sms", "0")
    c.barrier()
    return c.max(ev[0].elapsed_time(ev[steps])), launches


def time_relay_steps(c, kernel, ins, out, bounds, relay, steps, warmup, timeout_s=30.0):
    """Steps whose B reaches every rank inside the step through the
    copy-engine relay (parallel.CopyEngineRelay): rank 0's B is pushed down
    the chain 0 -> 1 -> ... chunk by chunk by copy engines, and the plan
    runs in K slices, slice j waiting (a stream wait on the flag of slab j's
    last chunk) for slab j only; the GEMM keeps every SM.  Each step's relay
    starts after the previous step on rank 0 and after the next rank
    acknowledged it.  Runs on its own streams; completion is polled with a
    deadline, after which the rank raises its own flags so that no stream
    wait stays pending.  -> (max-over-ranks ms of the timed region or None,
    GEMM launches counted, True when every rank completed)."""
    import bafe_b200 as bafe
    from bafe_b200.parallel import relay_chunks
    torch = c.torch
    comp, copy, watch = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    comp.wait_stream(torch.cuda.current_stream())
    chunk_bounds, last = relay_chunks(bounds, ins[1].shape[1] * ins[1].element_size())
    n = [0]

    def step(start):
        n[0] += 1
        start.record(comp)
        relay.send(n[0], chunk_bounds, copy, start if c.rank == 0 else None)
        evs = relay.ready(n[0], last, watch)
        kernel.run_torch_ksliced(ins, out, bounds, ready=evs, stream=comp)
        relay.finish(n[0], comp)

    def drained(ev):
        t_end = time.perf_counter() + timeout_s
        while not ev.query():
            if time.perf_counter() > t_end:
                return False
            time.sleep(0.0005)
        return True

    def run(k_steps, events):
        try:
            for i in range(k_steps):
                step(events[i])
        except Exception:
            return False
        finally:
            events[k_steps].record(comp)
        return drained(events[k_steps])

    ok = run(warmup, [torch.cuda.Event() for _ in range(warmup + 1)])
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    launches = 0
    if c.sum(0.0 if ok else 1.0) == 0:
        c.barrier()
        launches0 = bafe.launch_count()
        ok = run(steps, ev)
        launches = bafe.launch_count() - launches0
    else:
        ok = False
    if not ok:
        relay.release(n[0])
    comp.synchronize()
    copy.synchronize()
    watch.synchronize()
    all_ok = c.sum(0.0 if ok else 1.0) == 0
    c.barrier()
    return (c.max(ev[0].elapsed_time(ev[steps])) if all_ok else None), launches, all_ok


def bench_relay(c, k, ins, out, S, ms_bcast, flops_total, steps, warmup):
    """The B-inside-the-step variant over the copy-engine relay: K slabs
    sized from the K-sliced GEMM's time with B resident, the NCCL
    broadcast's time (the relay moves B at a similar link rate) and a
    measured slice-boundary cost, with every SM kept by the GEMM."""
    from bafe_b200.parallel import CopyEngineRelay, k_slab_schedule
    torch = c.torch
    relay, Brel, err = CopyEngineRelay.over_ranks(tuple(ins[1].shape), c.dist, c.local)
    if c.sum(0.0 if err is None else 1.0) > 0:
        relay.close(c.dist)
        return {"unavailable": (err or "relay setup failed on another rank")[:300]}
    all_ok, t, bounds, boundary_ms = False, {}, [0, S], 0.0
    try:
        if c.rank == 0:
            Brel.copy_(ins[1])
        torch.cuda.synchronize()
        rins = [ins[0], Brel] + list(ins[2:])
        # the cost of one more slice: two equal slices against one, B resident
        # (interleaved, the fastest of three each: the clock under the power
        # cap moves by more than the difference; floored at the sums' store
        # and reload at HBM speed)
        half = (S // 2) // k.k_slice_align * k.k_slice_align
        for name, b in (("one", [0, S]), ("two", [0, half, S])):
            k.run_torch_ksliced(rins, out, b)
        torch.cuda.synchronize()
        for _ in range(3):
            for name, b in (("one", [0, S]), ("two", [0, half, S])):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                k.run_torch_ksliced(rins, out, b)
                e1.record()
                torch.cuda.synchronize()
                t[name] = min(t.get(name, 1e30), c.max(e0.elapsed_time(e1)))
        boundary_ms = max(t["two"] - t["one"], 2.0 * out.numel() * 4 / (c.hbm_peak * 1e9) * 1e3 + 0.03)
        bounds = k_slab_schedule(S, k.k_slice_align, t["one"], max(ms_bcast, 0.1), boundary_ms, keep=1.0)
        if os.environ.get("BENCH_RELAY_SLABS"):
            bounds = [int(x) for x in os.environ["BENCH_RELAY_SLABS"].split(",")]
        ms_total, n_launch, all_ok = time_relay_steps(c, k, rins, out, bounds, relay, steps, warmup)
    finally:
        torch.cuda.synchronize()
        relay.close(c.dist)
    if not all_ok:
        return {"unavailable": "a relay step did not complete within its deadline on some rank"}
    ms = ms_total / steps
    return {"value": round(flops_total / (ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
            "k_slabs": bounds, "slice_boundary_ms": round(boundary_ms, 4),
            "gemm_k_sliced_ms": round(t["one"], 4), "gpu_launches": int(c.sum(n_launch)),
            "how": ("rank 0's B pushed down the chain of ranks by copy engines inside each timed step "
                    "(CUDA IPC buffers, stream-ordered flag waits, no SM used by the transfer); "
                    f"{len(bounds) - 1} K slabs, GEMM K slice j waits for slab j; max over ranks")}


class _NpPtr:
    """A numpy array seen through time_e2e's data_ptr() (pageable host memory)."""

    def __init__(self, a):
        self.a = np.ascontiguousarray(a)

    def data_ptr(self):
        return self.a.ctypes.data


def time_e2e(torch, kernel, host_ins, host_out, steps):
    """Host-pointer C-ABI calls (H2D + kernels + D2H + sync per call)."""
    ptrs = [t.data_ptr() for t in host_ins] + [host_out.data_ptr()]
    for _ in range(3):            # warm: allocates staging, loads the module, captures a small call's graph
        kernel.call_host_ptrs(ptrs)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        kernel.call_host_ptrs(ptrs)
    return (time.perf_counter() - t0) / steps * 1e3


def time_e2e_shared(torch, kernel, host_ins, host_out, shared, steps):
    """Host-pointer calls whose `shared` inputs each rank assembles on its
    device from its own slab plus an NCCL all-gather (parallel.run_host_shared),
    every copy and collective inside the timed region."""
    from bafe_b200.parallel import run_host_shared
    run_host_shared(kernel, host_ins, host_out, shared)   # warm: buffers, module
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        run_host_shared(kernel, host_ins, host_out, shared)
    return (time.perf_counter() - t0) / steps * 1e3


def reduce_max(torch, dist, x: float, dev) -> float:
    if dist is None:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def reduce_sum(torch, dist, x: float, dev) -> float:
    if dist is None:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def traffic_from_profiles(name: str):
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get(name)
    return None


# ------------------------------------------------------- CPU baselines --
# The reference's own generated C kernels, built and run through its public
# C API (oracle/refgraph.py builds the graphs with the reference's graph
# functions; oracle/refbafe.py optimizes, JITs and calls).  None of these
# import the B200 backend.

def _ref_kernel(build, cache: str | None = None):
    """build(builder) -> root, with inputs named as the caller's arrays.
    Returns (reference, kernel address, input names in call order, stack bytes)."""
    import tempfile
    from oracle import refbafe, refgraph
    ref = refbafe.Reference(cache_dir=cache or tempfile.mkdtemp(prefix="bafe_ref_"))
    b = refgraph.Builder(ref.lib)
    b.output(build(b))
    opt = ref.optimize(b.graph)
    fn = ref.compile(opt)
    nodes = refbafe.graph_nodes(opt)
    names = [nodes[opt.inputs[i]]["name"] for i in range(opt.n_inputs)]
    return ref, fn, names, refbafe.stack_bytes_for(nodes)


def _ref_time(build, arrays: dict, out: np.ndarray, reps: int, cache: str | None = None) -> float:
    """Seconds per call of the reference kernel (one warm call first)."""
    ref, fn, names, stack = _ref_kernel(build, cache)
    call = [arrays[n] for n in names]
    ref.call_kernel(fn, call, out, stack_bytes=stack)
    t0 = time.perf_counter()
    for _ in range(reps):
        ref.call_kernel(fn, call, out, stack_bytes=stack)
    return (time.perf_counter() - t0) / reps


def _build_gemm_relu_add(rows: int, S: int):
    def build(b):
        a = b.input("A", (rows, S))
        bb = b.input("B", (S, S), layout=2)          # BLOCKED tag, row-major storage
        c = b.input("C", (rows, S))
        return b.add("relu", [b.add("add", [b.add("matmul", [a, bb]), c])])
    return build


def cpu_baseline_gemm(A_rows: np.ndarray, B: np.ndarray, C_rows: np.ndarray):
    """The reference's generated kernel on a row panel of the 16384^3
    problem (1 core): 32 rows, one of the emitter's row tiles
    (MATMUL_TILE, codegen.c:23), so B streams once per 32 rows as in the
    full-size run."""
    from oracle import refbafe
    rows = A_rows.shape[0]
    flops = 2.0 * rows * GEMM_N * GEMM_K
    out = np.zeros((rows, GEMM_N), np.float32)
    if refbafe.available():
        dt = _ref_time(_build_gemm_relu_add(rows, GEMM_N), {"A": A_rows, "B": B, "C": C_rows}, out, 1)
        kind = "reference"
    else:
        from oracle import oracle
        t0 = time.perf_counter()
        mm = oracle.matmul_panel_f32(A_rows, B, rows, GEMM_N, GEMM_K, False, False, 0, rows)
        oracle.unary("relu", oracle.binary("add", mm.reshape(-1), C_rows.reshape(-1), 0, 1, mm.size, 0, 0, 0), 0, 0)
        dt = time.perf_counter() - t0
        kind = "port"
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": 1, "kind": kind,
            "sample": f"{rows}-row panel of relu(matmul(A,B)+C) 16384^3 ({flops / 1e9:.1f} GFLOP, {dt:.2f} s)"}


def _build_ew(n: int):
    def build(b):
        x, y, z = (b.input(nm, (n,)) for nm in "XYZ")
        return b.add("relu", [b.add("add", [b.add("mul", [x, y]), z])])
    return build


def cpu_baseline_ew(x: np.ndarray, y: np.ndarray, z: np.ndarray):
    from oracle import refbafe
    n = x.size
    if refbafe.available():
        dt = _ref_time(_build_ew(n), {"X": x, "Y": y, "Z": z}, np.zeros(n, np.float32), 3)
        kind = "reference"
    else:
        from oracle import oracle
        t0 = time.perf_counter()
        m = oracle.binary("mul", x, y, 0, 1, n, 0, 0, 0)
        oracle.unary("relu", oracle.binary("add", m, z, 0, 1, n, 0, 0, 0), 0, 0)
        dt = time.perf_counter() - t0
        kind = "port"
    return {"value": 16.0 * n / dt / 1e9, "unit": "GB/s", "cores": 1, "kind": kind,
            "sample": f"{n} elements of relu(add(mul(X,Y),Z)) ({dt * 1e3:.1f} ms per call)"}


def cpu_baseline_transpose(x: np.ndarray):
    """The reference's generated transpose kernel (codegen.c:360-369) on a
    column panel: X[:, c0:c1] stored contiguously, transposed to rows."""
    from oracle import refbafe
    rows, cols = x.shape
    if refbafe.available():
        def build(b):
            return b.add("transpose", [b.input("X", (rows, cols))], perm=[1, 0])
        dt = _ref_time(build, {"X": x}, np.zeros((cols, rows), np.float32), 3)
        kind = "reference"
    else:
        from oracle import oracle
        t0 = time.perf_counter()
        oracle.transpose2d(x, cols, rows)
        dt = time.perf_counter() - t0
        kind = "port"
    return {"value": 8.0 * x.size / dt / 1e9, "unit": "GB/s", "cores": 1, "kind": kind,
            "sample": f"{rows}x{cols} column panel ({dt * 1e3:.1f} ms per call)"}


# ------------------------------------------------------------ our arm --

class Ctx:
    def __init__(self, args):
        import torch
        self.torch = torch
        self.args = args
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if args.gpus != self.world:
            raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={self.world}")
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        self.dist = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist_mod
            # rank 0's stdout carries exactly one JSON line: NCCL prints its
            # version banner (and warnings) to stdout at NCCL_DEBUG=VERSION or
            # WARN, so its log goes to stderr unless a log file was chosen
            os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
            if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
                os.environ["NCCL_DEBUG"] = "WARN"
            dist_mod.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=self.dev)
            self.dist = dist_mod
        self.hbm_peak, self.bf16_peak, self.bf16_sustained, self.peak_src = peaks()
        self.gen = torch.Generator(device=self.dev).manual_seed(1234 + self.rank)

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def max(self, x):
        return reduce_max(self.torch, self.dist, x, self.dev)

    def sum(self, x):
        return reduce_sum(self.torch, self.dist, x, self.dev)


def bench_gemm(c: Ctx) -> dict:
    import bafe_b200 as bafe
    torch, args = c.torch, c.args
    from bafe_b200.parallel import broadcast_resident, row_panels
    S = args.gemm_size
    std = 1.0 / math.sqrt(S)
    r0, r1 = row_panels(S, c.world)[c.rank]
    rows = r1 - r0
    A = torch.randn(rows, S, device=c.dev, generator=c.gen) * std
    C = torch.randn(rows, S, device=c.dev, generator=c.gen) * std
    B = torch.empty(S, S, device=c.dev)
    if c.rank == 0:
        B.copy_(torch.randn(S, S, device=c.dev, generator=torch.Generator(device=c.dev).manual_seed(99)) * std)
    bcast_ms = 0.0
    if c.dist is not None:
        c.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        broadcast_resident(B, c.dist, src=0)
        e1.record()
        torch.cuda.synchronize()
        bcast_ms = c.max(e0.elapsed_time(e1))
    out = torch.empty(rows, S, device=c.dev)
    epi = args.gemm_epilogue
    ins = [A, B, C]
    if epi == "mul_cd":
        ins.append(torch.randn(rows, S, device=c.dev, generator=c.gen))
    t_compile = time.perf_counter()
    k = bafe.compile_graph(gemm_graph(rows, S, epi))
    t_compile = time.perf_counter() - t_compile
    plan = k.describe().strip()
    c.barrier()
    with Clocks(c.local) as ck:
        per, total_ms, launches, step_ms = time_steps(torch, k, ins, out, args.steps, args.warmup, per_kernel=True)
    c.barrier()
    clocks = ck.summary()
    total_ms = c.max(total_ms)
    launches = int(c.sum(launches))
    ms_step = total_ms / args.steps
    flops_total = 2.0 * S * S * S
    # the dominant kernel: the plan's GEMM step (its launch and split-tail
    # fixup), timed by events around it inside every timed step
    gemm_idx = max(i for i, line in enumerate(plan.splitlines()) if line.startswith("gemm"))
    kern_ms = c.max(step_ms[gemm_idx])
    achieved = 2.0 * rows * S * S / (kern_ms * 1e-3) / 1e12
    tc3 = "3xtf32" in plan
    # tf32 MMAs run at half the bf16 rate; 3xTF32 issues three per product
    peak, basis, peak_burst, peak_sus = roofline_basis(c, clocks, 2.0 * (3.0 if tc3 else 1.0))
    res = {
        "metric": "TFLOP/s (fused GEMM relu(matmul(A,B)+C))",
        "value": round(flops_total / (ms_step * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
        "ms_per_step": round(ms_step, 4),
        "dtype": "fp32 via 3xtf32" if tc3 else ("tf32" if "tc.tf32" in plan else "fp32"),
        "config": gemm_config(S) if epi == "c" else
                  {"workload": f"relu(add(matmul(A,B), mul(C,D))) M=N=K={S} fp32, A, C, D row-major, B BLOCKED tag"},
        "run": {"parallelism": f"M-row panels x{c.world}, B broadcast once (outside the timed region)",
                "plan": plan, "precision_option": args.precision},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 3), "peak": round(peak, 2), "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic_from_profiles(f"gemm_{S}" if epi == "c" else f"gemm_mul_cd_{S}"),
                     "peak_basis": f"{c.peak_src} {basis} bf16 TFLOP/s / 2 (tf32 rate)"
                                   + (" / 3 (three products)" if tc3 else "")
                                   + f"; {basis} because the timed region's median SM clock was "
                                   + f"{clocks.get('sm_mhz')} of {clocks.get('sm_max_mhz')} MHz",
                     "frac_of_burst": round(achieved / peak_burst, 4),
                     "frac_of_sustained": round(achieved / peak_sus, 4),
                     "achieved_over": "CUDA events around the plan's GEMM launch (with its split-tail fixup) "
                                      "inside every timed step; max over ranks",
                     "gemm_kernel_ms": round(kern_ms, 4),
                     "plan_step_ms": [round(x, 4) for x in step_ms]},
        "gpu_launches": launches, "clocks": clocks, "b_broadcast_ms": round(bcast_ms, 3),
        "compile_s": round(t_compile, 2),
    }
    if c.world > 1 and epi == "c":
        # B crosses NVLink inside every step (the same workload when B changes
        # from call to call): broadcast, then the GEMM; and broadcast in K
        # slabs overlapped with the GEMM's K slices
        from bafe_b200.parallel import k_slab_schedule
        variants = {"b_broadcast_in_step": ([0, S], 0)}
        if k.k_slice_align:
            variants["b_broadcast_overlapped"] = (None, int(os.environ.get("BENCH_KSLICE_FREE_SMS", "16")))
        ms_plain = None
        for name, (bounds, free) in variants.items():
            if bounds is None:
                # slabs sized from the two times just measured (the GEMM with B
                # resident, the broadcast = the plain variant's excess): each
                # slab's broadcast hides behind the previous slab's GEMM slice
                sms = torch.cuda.get_device_properties(c.dev).multi_processor_count
                boundary_ms = 2.0 * out.numel() * 4 / (c.hbm_peak * 1e9) * 1e3   # sums stored + reloaded
                bounds = k_slab_schedule(S, k.k_slice_align, ms_step, max(ms_plain - ms_step, 1e-3), boundary_ms,
                                         keep=(sms - free) / sms)
            ms_total, n_launch = time_bcast_steps(c, k, ins, out, bounds, free, args.steps, args.warmup)
            ms = ms_total / args.steps
            if ms_plain is None:
                ms_plain = ms
            res[name] = {"value": round(flops_total / (ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                         "ms_per_step": round(ms, 4), "k_slabs": bounds, "free_sms_while_slabs_arrive": free,
                         "gpu_launches": int(c.sum(n_launch)),
                         "how": "rank 0's B broadcast over NCCL inside each timed step ("
                                + ("one piece, then the GEMM" if len(bounds) == 2 else
                                   f"{len(bounds) - 1} K slabs on a side stream; GEMM K slice j waits for slab j")
                                + "); max over ranks"}
        if k.k_slice_align and os.environ.get("BENCH_RELAY", "1") != "0":
            res["b_relay_copy_engine"] = bench_relay(c, k, ins, out, S, max(ms_plain - ms_step, 0.0),
                                                     flops_total, args.steps, args.warmup)
    if args.e2e_steps > 0 and epi == "c":
        hA, hB, hC = A.cpu().pin_memory(), B.cpu().pin_memory(), C.cpu().pin_memory()
        hO = torch.empty(rows, S).pin_memory()
        c.barrier()
        if c.world > 1:
            # B: each rank copies its 1/N slab from the host, NCCL all-gathers it
            from bafe_b200.parallel import SharedInput
            e2e_ms = c.max(time_e2e_shared(torch, k, [hA, hB, hC], hO, {1: SharedInput(c.dist, c.dev)},
                                           args.e2e_steps))
            h2d = float(4 * (A.numel() + C.numel())) * c.world + float(4 * B.numel())
            path = ("bafe_cuda_run_host_resident (A, C, output: pinned host buffers, row-streamed; "
                    "B: 1/N slab per rank from pinned host memory + NCCL all-gather)")
        else:
            e2e_ms = c.max(time_e2e(torch, k, [hA, hB, hC], hO, args.e2e_steps))
            h2d = float(4 * (A.numel() + B.numel() + C.numel()))
            path = "bafe_cuda_jit_get_or_compile host function, pinned host buffers"
        res["e2e"] = {"value": round(flops_total / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                      "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": float(4 * out.numel()) * c.world,
                      "ms_per_step": round(e2e_ms, 2), "path": path}
        if c.rank == 0 and not args.no_cpu_baseline and S == GEMM_M:
            res["cpu_baseline"] = cpu_baseline_gemm(hA[:32].numpy(), hB.numpy(), hC[:32].numpy())
        del hA, hB, hC, hO
    elif c.rank == 0 and not args.no_cpu_baseline and S == GEMM_M and epi == "c":
        res["cpu_baseline"] = cpu_baseline_gemm(A[:32].cpu().numpy(), B.cpu().numpy(), C[:32].cpu().numpy())
    return res


def bench_gemm_bf16(c: Ctx) -> dict:
    """The same fused GEMM with bf16 A, B, C and output (kind::f16 tensor
    cores, f32 accumulation): device-resident, row panels per rank."""
    import bafe_b200 as bafe
    torch, args = c.torch, c.args
    from bafe_b200.parallel import broadcast_resident, row_panels
    S = args.gemm_size
    r0, r1 = row_panels(S, c.world)[c.rank]
    rows = r1 - r0
    std = 1.0 / math.sqrt(S)
    A = (torch.randn(rows, S, device=c.dev, generator=c.gen) * std).to(torch.bfloat16).view(torch.int16)
    C = (torch.randn(rows, S, device=c.dev, generator=c.gen) * std).to(torch.bfloat16).view(torch.int16)
    B = (torch.randn(S, S, device=c.dev, generator=c.gen) * std).to(torch.bfloat16).view(torch.int16)
    if c.dist is not None:
        broadcast_resident(B, c.dist, src=0)
    out = torch.empty(rows, S, dtype=torch.int16, device=c.dev)
    g = bafe.GraphBuilder()
    a = g.add_input("A", (rows, S), 5, 0)
    b = g.add_input("B", (S, S), 5, 2)
    cc = g.add_input("C", (rows, S), 5, 0)
    g.set_output(g.add("relu", [g.add("add", [g.add("matmul", [a, b]), cc])]))
    k = bafe.compile_graph(g)
    c.barrier()
    with Clocks(c.local) as ck:
        per, total, launches = time_steps(torch, k, [A, B, C], out, args.steps, args.warmup)
    c.barrier()
    total = c.max(total)
    ms = total / args.steps
    achieved = 2.0 * rows * S * S / (statistics.mean(per) * 1e-3) / 1e12
    clocks = ck.summary()
    peak, basis, burst, sus = roofline_basis(c, clocks, 1.0)
    return {
        "metric": "TFLOP/s (fused GEMM relu(matmul(A,B)+C), bf16 operands and output)",
        "value": round(2.0 * S ** 3 / (ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
        "dtype": "bf16 (f32 accumulate)",
        "config": {"workload": f"relu(matmul(A,B)+C) M=N=K={S} bf16, A row-major, B BLOCKED tag",
                   "l2": "inputs larger than L2; no flush" if S >= 8192 else "inputs smaller than L2"},
        "run": {"parallelism": f"M-row panels x{c.world}, B broadcast once", "plan": k.describe().strip()},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "frac_of_burst": round(achieved / burst, 4),
                     "frac_of_sustained": round(achieved / sus, 4), "traffic": None,
                     "peak_basis": f"{c.peak_src} {basis} bf16 (cuBLAS); {basis} because the timed region's median "
                                   f"SM clock was {clocks.get('sm_mhz')} of {clocks.get('sm_max_mhz')} MHz"},
        "gpu_launches": int(c.sum(launches)), "clocks": clocks,
    }


def bench_gemm_tf32(c: Ctx) -> dict:
    """The headline workload with gemm_precision=tf32 (one kind::tf32 MMA
    per product): throughput against the TF32 peak, and its measured
    relative error against fp64 on rank 0's first rows:
    max |out - fp64| / (|A| |B|) elementwise (the bound the tests state is
    2^-9: two operand truncations to tf32's 10-bit mantissa)."""
    import bafe_b200 as bafe
    torch, args = c.torch, c.args
    from bafe_b200.parallel import broadcast_resident, row_panels
    S = args.gemm_size
    std = 1.0 / math.sqrt(S)
    r0, r1 = row_panels(S, c.world)[c.rank]
    rows = r1 - r0
    A = torch.randn(rows, S, device=c.dev, generator=c.gen) * std
    C = torch.randn(rows, S, device=c.dev, generator=c.gen) * std
    B = torch.randn(S, S, device=c.dev, generator=torch.Generator(device=c.dev).manual_seed(99)) * std
    if c.dist is not None:
        broadcast_resident(B, c.dist, src=0)
    out = torch.empty(rows, S, device=c.dev)
    old = bafe.get_option("gemm_precision")
    bafe.set_option("gemm_precision", "tf32")
    try:
        k = bafe.compile_graph(gemm_graph(rows, S))
    finally:
        bafe.set_option("gemm_precision", old)
    plan = k.describe().strip()
    c.barrier()
    with Clocks(c.local) as ck:
        per, total, launches = time_steps(torch, k, [A, B, C], out, args.steps, args.warmup)
    c.barrier()
    total = c.max(total)
    ms = total / args.steps
    achieved = 2.0 * rows * S * S / (statistics.mean(per) * 1e-3) / 1e12
    clocks = ck.summary()
    peak, basis, burst, sus = roofline_basis(c, clocks, 2.0)
    # accuracy on 16 rows: fp64 product on the device
    Bd = B.double()
    ref = torch.relu(A[:16].double() @ Bd + C[:16].double())
    scale = A[:16].double().abs() @ Bd.abs()
    err = (out[:16].double() - ref).abs()
    rel = float((err / scale).max())
    del Bd, scale
    return {
        "metric": "TFLOP/s (fused GEMM relu(matmul(A,B)+C), 1xTF32)",
        "value": round(2.0 * S ** 3 / (ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
        "dtype": "tf32 (f32 accumulate)",
        "config": gemm_config(S),
        "run": {"parallelism": f"M-row panels x{c.world}, B broadcast once", "plan": plan,
                "precision_option": "tf32"},
        "accuracy": {"max_abs_err_vs_fp64": float(err.max()), "max_rel_err_vs_fp64": rel,
                     "rel_err": "max over 16 rows of |out - fp64| / (|A| |B|)", "rel_tolerance": 2.0 ** -9},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "frac_of_burst": round(achieved / burst, 4),
                     "frac_of_sustained": round(achieved / sus, 4), "traffic": None,
                     "peak_basis": f"{c.peak_src} {basis} bf16 TFLOP/s / 2 (tf32 rate); {basis} because the timed "
                                   f"region's median SM clock was {clocks.get('sm_mhz')} of {clocks.get('sm_max_mhz')} MHz"},
        "gpu_launches": int(c.sum(launches)), "clocks": clocks,
    }


def bench_ew(c: Ctx) -> dict:
    import bafe_b200 as bafe
    torch, args = c.torch, c.args
    from bafe_b200.parallel import element_ranges
    n_total = args.ew_elements
    e0_, e1_ = element_ranges(n_total, c.world)[c.rank]
    n_local = e1_ - e0_
    X, Y, Z = (torch.rand(n_local, device=c.dev, generator=c.gen) * 2 - 1 for _ in range(3))
    O = torch.empty(n_local, device=c.dev)
    k = bafe.compile_graph(ew_graph(n_local))
    steps = max(args.steps, 200)
    c.barrier()
    with Clocks(c.local) as ck:
        per, total, launches = time_steps(torch, k, [X, Y, Z], O, steps, args.warmup)
    c.barrier()
    total = c.max(total)
    ms = total / steps
    achieved = 16.0 * n_local / (statistics.mean(per) * 1e-3) / 1e9
    res = {
        "metric": f"GB/s (relu(add(mul(X,Y),Z)) {n_total} fp32)", "value": round(16.0 * n_total / (ms * 1e-3) / 1e9, 1),
        "unit": "GB/s", "ms_per_step": round(ms, 4), "steps": steps,
        "config": {"workload": f"relu(add(mul(X,Y),Z)) over {n_total} fp32 elements, U(-1,1)",
                   "parallelism": f"contiguous ranges x{c.world}, no collective",
                   "l2": "inputs larger than L2; no flush" if n_local * 4 > (126 << 20) else "inputs smaller than L2",
                   "plan": k.describe().strip()},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": c.hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / c.hbm_peak, 4),
                     "traffic": traffic_from_profiles(f"ew_{n_total}"), "peak_basis": f"{c.peak_src} hbm_gbs"},
        "gpu_launches": int(c.sum(launches)), "clocks": ck.summary(),
    }
    if args.e2e_steps > 0:
        hX, hY, hZ = X.cpu().pin_memory(), Y.cpu().pin_memory(), Z.cpu().pin_memory()
        hO = torch.empty(n_local).pin_memory()
        c.barrier()
        e2e_ms = c.max(time_e2e(torch, k, [hX, hY, hZ], hO, args.e2e_steps))
        res["e2e"] = {"value": round(16.0 * n_total / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                      "h2d_bytes_per_step": 12.0 * n_total, "d2h_bytes_per_step": 4.0 * n_total,
                      "ms_per_step": round(e2e_ms, 2)}
        if c.rank == 0 and not args.no_cpu_baseline:
            m = min(1 << 24, n_local)
            res["cpu_baseline"] = cpu_baseline_ew(hX[:m].numpy(), hY[:m].numpy(), hZ[:m].numpy())
    return res


def bench_transpose(c: Ctx) -> dict:
    """Transpose materialisation of an S x S fp32 matrix.  Rank r owns output
    rows [r0, r1) = input columns r0:r1, held as its own contiguous S x
    (r1 - r0) panel; no collective."""
    import bafe_b200 as bafe
    torch, args = c.torch, c.args
    from bafe_b200.parallel import transpose_blocks
    S = args.transpose_size
    r0, r1 = transpose_blocks(S, c.world)[c.rank]
    cols = r1 - r0
    X = torch.rand(S, cols, device=c.dev, generator=c.gen)
    O = torch.empty(cols, S, device=c.dev)
    k = bafe.compile_graph(transpose_graph(S, cols))
    steps = max(args.steps, 100)
    c.barrier()
    with Clocks(c.local) as ck:
        per, total, launches = time_steps(torch, k, [X], O, steps, args.warmup)
    c.barrier()
    total = c.max(total)
    ms = total / steps
    achieved = 8.0 * S * cols / (statistics.mean(per) * 1e-3) / 1e9
    if not torch.equal(O[:, :64], X[:64, :].t()):
        raise RuntimeError("transpose output check failed")
    res = {
        "metric": f"GB/s (transpose materialisation {S}x{S} fp32)",
        "value": round(8.0 * S * S / (ms * 1e-3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(ms, 4),
        "steps": steps,
        "config": {"workload": f"transpose(X) perm (1,0), X {S}x{S} fp32, materialised row-major",
                   "parallelism": f"output row blocks x{c.world} (input column panels), no collective",
                   "l2": "input and output larger than L2; no flush" if S * cols * 4 > (126 << 20)
                         else "inputs smaller than L2",
                   "plan": k.describe().strip()},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": c.hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / c.hbm_peak, 4),
                     "traffic": traffic_from_profiles(f"transpose_{S}"), "peak_basis": f"{c.peak_src} hbm_gbs"},
        "gpu_launches": int(c.sum(launches)), "clocks": ck.summary(),
    }
    if args.e2e_steps > 0:
        hX = X.cpu().pin_memory()
        hO = torch.empty(cols, S).pin_memory()
        c.barrier()
        e2e_ms = c.max(time_e2e(torch, k, [hX], hO, args.e2e_steps))
        res["e2e"] = {"value": round(8.0 * S * S / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                      "h2d_bytes_per_step": 4.0 * S * S, "d2h_bytes_per_step": 4.0 * S * S,
                      "ms_per_step": round(e2e_ms, 2)}
        if c.rank == 0 and not args.no_cpu_baseline:
            res["cpu_baseline"] = cpu_baseline_transpose(np.ascontiguousarray(hX[:, :min(cols, 256)].numpy()))
    return res


def bench_configs(c: Ctx, cpu: bool = True) -> dict:
    """The other configurations of the reference's benchmark set, on one GPU
    (rank 0; they are too small to shard): relu(matmul(A,B)+C) at 64^3,
    matmul at 256^3 with B row- and column-major (launch-latency bound:
    microseconds per call, no roofline claim), and relu(add(matmul(A,B),
    mul(C,D))) at 4096^3 (tensor-core bound).  Each entry carries the
    reference's generated C kernel timed on the same host (1 core, the same
    inputs; 4096^3 on a 32-row panel, one of the emitter's row tiles,
    scaled to the full problem by its row count)."""
    import bafe_b200 as bafe
    torch = c.torch
    g0 = torch.Generator(device=c.dev).manual_seed(5)
    out = {}

    def run(name, g, ref_build, names, shapes, steps, flops, ref_rows=None):
        import ctypes
        from bafe_b200._binding import lib
        k = bafe.compile_graph(g)
        ins = [torch.randn(*sh, device=c.dev, generator=g0) for sh in shapes]
        o = torch.empty(*k.out_shape, device=c.dev)
        per, total, _ = time_steps(torch, k, ins, o, steps, 5)
        # device time per call with the launches issued back to back from C
        # (bafe_cuda_time_device), free of the Python call overhead that the
        # per-step events above include for microsecond-sized calls
        ptrs = (ctypes.c_void_p * (len(ins) + 1))(*[t.data_ptr() for t in ins + [o]])
        dev_ms = ctypes.c_double()
        lib.bafe_cuda_time_device(k.plan, ptrs, len(ins) + 1, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                                  steps, ctypes.byref(dev_ms))
        hins = [t.cpu().pin_memory() for t in ins]
        hout = torch.empty(*k.out_shape).pin_memory()
        e2e_ms = time_e2e(torch, k, hins, hout, 20)
        # the same call on pageable numpy arrays, as BAFE's Python binding passes them
        nins = [t.numpy().copy() for t in hins]   # a fresh (pageable) numpy allocation
        nout = np.empty(tuple(k.out_shape), np.float32)
        e2e_np_ms = time_e2e(torch, k, [_NpPtr(a) for a in nins], _NpPtr(nout), 20)
        ms = total / steps
        r = {"plan": k.describe().strip(), "device_us_per_call": round(dev_ms.value * 1e3, 2),
             "python_loop_us_per_call": round(ms * 1e3, 2), "e2e_us_per_call": round(e2e_ms * 1e3, 1),
             "e2e_pageable_us_per_call": round(e2e_np_ms * 1e3, 1),
             "tflops_device": round(flops / (dev_ms.value * 1e-3) / 1e12, 3),
             "tflops_e2e": round(flops / (e2e_ms * 1e-3) / 1e12, 4)}
        if "gemm.tc" in r["plan"]:
            achieved = flops / (dev_ms.value * 1e-3) / 1e12
            div = 2.0 * (3.0 if "3xtf32" in r["plan"] else 1.0)
            r["roofline"] = {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(c.bf16_peak / div, 1),
                             "unit": "TFLOP/s", "frac": round(achieved / (c.bf16_peak / div), 4),
                             "peak_basis": f"{c.peak_src} burst bf16 / 2 (tf32 rate)"
                                           + (" / 3 (three products)" if "3xtf32" in r["plan"] else "")
                                           + " (back-to-back calls of a few ms run at the burst clock)"}
        from oracle import refbafe
        if cpu and refbafe.available():
            arrays = dict(zip(names, nins))
            if ref_rows:
                full_rows = shapes[0][0]
                arrays = {n: (np.ascontiguousarray(a[:ref_rows]) if n in ("A", "C", "D") else a)
                          for n, a in arrays.items()}
                ref_out = np.zeros((ref_rows, k.out_shape[1]), np.float32)
                dt = _ref_time(ref_build(ref_rows), arrays, ref_out, 1) * full_rows / ref_rows
                sample = f"{ref_rows}-row panel, scaled by {full_rows // ref_rows} to the full problem"
            else:
                ref_out = np.zeros(tuple(k.out_shape), np.float32)
                reps = max(3, min(50, int(0.5 / max(flops / 2e9, 1e-4))))
                dt = _ref_time(ref_build(None), arrays, ref_out, reps)
                sample = f"the full problem, mean of {reps} calls"
            r["cpu_baseline"] = {"value": round(flops / dt / 1e12, 6), "unit": "TFLOP/s",
                                 "us_per_call": round(dt * 1e6, 1), "cores": 1, "kind": "reference",
                                 "sample": sample}
        out[name] = r

    g = bafe.GraphBuilder()
    a, b, cc = (g.add_input(n, (64, 64), 0, 0) for n in "ABC")
    g.set_output(g.add("relu", [g.add("add", [g.add("matmul", [a, b]), cc])]))

    def ref_cfg1(_rows):
        def build(rb):
            x, y, z = (rb.input(n, (64, 64)) for n in "ABC")
            return rb.add("relu", [rb.add("add", [rb.add("matmul", [x, y]), z])])
        return build
    run("cfg1 relu(matmul(A,B)+C) 64^3", g, ref_cfg1, "ABC", [(64, 64)] * 3, 200, 2.0 * 64 ** 3)
    for col in (0, 1):
        g = bafe.GraphBuilder()
        a = g.add_input("A", (256, 256), 0, 0)
        b = g.add_input("B", (256, 256), 0, col)
        g.set_output(g.add("matmul", [a, b]))

        def ref_cfg2(_rows, col=col):
            def build(rb):
                return rb.add("matmul", [rb.input("A", (256, 256)), rb.input("B", (256, 256), layout=col)])
            return build
        name = f"cfg2 matmul 256^3 B {'col' if col else 'row'}-major"
        run(name, g, ref_cfg2, "AB", [(256, 256)] * 2, 200, 2.0 * 256 ** 3)
        # the one configuration the reference publishes a time for (its README,
        # generated C on unstated hardware): for context beside the same-box baseline
        out[name]["reference_published"] = {"ms_per_call": 6.84 if col else 10.09,
                                            "source": "reference README.md:90-91 (generated C, hardware unstated)"}
    n = 4096
    g = bafe.GraphBuilder()
    a, b, cc, dd = (g.add_input(x, (n, n), 0, 0) for x in "ABCD")
    g.set_output(g.add("relu", [g.add("add", [g.add("matmul", [a, b]), g.add("mul", [cc, dd])])]))

    def ref_cfg3(rows):
        def build(rb):
            x = rb.input("A", (rows, n))
            y = rb.input("B", (n, n))
            z = rb.input("C", (rows, n))
            w = rb.input("D", (rows, n))
            return rb.add("relu", [rb.add("add", [rb.add("matmul", [x, y]), rb.add("mul", [z, w])])])
        return build
    run("cfg3 relu(add(matmul(A,B),mul(C,D))) 4096^3", g, ref_cfg3, "ABCD", [(n, n)] * 4, 20, 2.0 * n ** 3,
        ref_rows=32)
    return out


def run_ours(args):
    import bafe_b200 as bafe
    c = Ctx(args)
    bafe.set_option("gemm_precision", args.precision)
    common = {"n_gpus": c.world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
              "scaling": "strong", "vs_baseline": None, "data": "synthetic, generated on device"}
    if args.only in ("ew", "transpose"):
        fn = bench_ew if args.only == "ew" else bench_transpose
        line = dict(fn(c), **{k: v for k, v in common.items() if k != "steps"})
        line["scaling"] = "strong"
    elif args.only == "gemm_bf16":
        line = dict(common, **bench_gemm_bf16(c))
    elif args.only == "gemm_tf32":
        line = dict(common, **bench_gemm_tf32(c))
    else:
        line = dict(common, **bench_gemm(c))
        if args.only is None:
            line["gemm_tf32"] = bench_gemm_tf32(c)
            line["gemm_bf16"] = bench_gemm_bf16(c)
            line["ew"] = bench_ew(c)
            line["transpose"] = bench_transpose(c)
            if c.rank == 0:
                line["configs"] = bench_configs(c, cpu=not args.no_cpu_baseline)
    if c.rank == 0:
        print(json.dumps(line), flush=True)
    if c.dist is not None:
        c.dist.barrier()
        c.dist.destroy_process_group()


# ------------------------------------------------------ reference arm --

def _ref_worker(job):
    """One host process: the reference's generated kernel on its own 32-row
    panel of the 16384^3 problem, built and run through the reference's
    own C API (this process never loads the B200 backend)."""
    import numpy as np
    from multiprocessing import shared_memory
    sys.path.insert(0, str(ROOT))
    from oracle import refbafe
    shm_name, shape, rows, steps, cache = job
    shm = shared_memory.SharedMemory(name=shm_name)
    try:
        B = np.ndarray(shape, np.float32, buffer=shm.buf)
        rng = np.random.default_rng(os.getpid())
        A = rng.standard_normal((rows, GEMM_K), dtype=np.float32) * np.float32(STD)
        C = rng.standard_normal((rows, GEMM_N), dtype=np.float32) * np.float32(STD)
        out = np.zeros((rows, GEMM_N), np.float32)
        ref, fn, names, stack = _ref_kernel(_build_gemm_relu_add(rows, GEMM_N), cache)
        call = [{"A": A, "B": B, "C": C}[n] for n in names]
        times = []
        for _ in range(steps):
            t0 = time.perf_counter()
            ref.call_kernel(fn, call, out, stack_bytes=stack)
            times.append(time.perf_counter() - t0)
        return times
    finally:
        shm.close()


def run_reference(args):
    """The reference's own CPU implementation of the headline workload on
    every host core: one process per core, each computing a 32-row panel
    (one of the emitter's row tiles, MATMUL_TILE = 32, codegen.c:23) of
    relu(matmul(A,B)+C) at 16384^3 per step with the reference's
    generated, single-threaded kernel (codegen.c:13-14); a step takes as
    long as its slowest process.  Only oracle/_ref/libbafe.so (the
    reference compiled from its own sources) is loaded."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import multiprocessing as mp
    import tempfile
    from multiprocessing import shared_memory
    from oracle import refbafe
    if not refbafe.available():
        refbafe.build()
    if not refbafe.available():
        print(json.dumps({"impl": "reference", "unavailable": "reference library oracle/_ref/libbafe.so not built"}))
        return
    cores = len(os.sched_getaffinity(0))
    procs = max(1, min(cores, 64))
    steps = args.warmup + args.steps
    cache = tempfile.mkdtemp(prefix="bafe_ref_cache_")
    rows = 32
    shm = shared_memory.SharedMemory(create=True, size=4 * GEMM_K * GEMM_N)
    try:
        B = np.ndarray((GEMM_K, GEMM_N), np.float32, buffer=shm.buf)
        B[:] = np.random.default_rng(99).standard_normal((GEMM_K, GEMM_N), dtype=np.float32) * np.float32(STD)
        # build the kernel once here, so the workers find it in the reference's on-disk JIT cache
        _ref_kernel(_build_gemm_relu_add(rows, GEMM_N), cache)
        ctx = mp.get_context("spawn")
        with ctx.Pool(procs) as pool:
            res = pool.map(_ref_worker, [(shm.name, (GEMM_K, GEMM_N), rows, steps, cache)] * procs)
    finally:
        shm.close()
        shm.unlink()
    step_times = [max(r[i] for r in res) for i in range(args.warmup, steps)]
    ms = statistics.mean(step_times) * 1e3
    flops = 2.0 * rows * procs * GEMM_N * GEMM_K
    value = flops / (ms * 1e-3) / 1e12
    sample = (f"{procs} processes x one {rows}-row panel of relu(matmul(A,B)+C) 16384^3 per step "
              f"({flops / 1e9:.0f} GFLOP per step; the reference kernel is single-threaded)")
    line = {
        "metric": "TFLOP/s (fused GEMM relu(matmul(A,B)+C))", "value": value, "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic, generated on the host",
        "config": gemm_config(GEMM_M),
        "run": {"sample": sample, "library": "oracle/_ref/libbafe.so (the reference built from its own sources)"},
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": procs, "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
