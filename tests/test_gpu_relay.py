"""Copy-engine relay of B down a chain of ranks (parallel.CopyEngineRelay,
bafe_cuda_relay_step / bafe_cuda_signal_wait / bafe_cuda_signal_write).

Each step, the root's B (new contents every step) is pushed chunk by chunk
down the chain by copy engines; every rank's K-sliced GEMM waits, slice by
slice, only for its slab's flags.  If a slice ran before its slab landed,
or a sender overwrote a rank's B before that rank's GEMM was done with the
previous step, the rank's output would differ from the same K-sliced run
over a resident copy of that step's B: the comparison is bit for bit.

The one-GPU test emulates three ranks in one process (their own buffers
and streams on cuda:0; the waits are stream waits executed by the GPU's
front end, no kernel spins on another's work).  The two-process test runs
the IPC path on two GPUs and is skipped with fewer.
"""
import os

import pytest

import bafe_b200 as bafe
from bafe_b200.parallel import CopyEngineRelay, relay_chunks

pytestmark = pytest.mark.gpu

M, N, K = 256, 512, 1152          # K = 12 promotion chunks of 96
SLABS = [0, 96, 480, 1152]


def _graph(rows):
    from bafe_b200.graph import GraphBuilder
    g = GraphBuilder()
    a = g.add_input("A", (rows, K), 0, 0)
    b = g.add_input("B", (K, N), 0, 2)
    c = g.add_input("C", (rows, N), 0, 0)
    g.set_output(g.add("relu", [g.add("add", [g.add("matmul", [a, b]), c])]))
    return g


def _compile(rows):
    bafe.set_option("gemm_precision", "3xtf32")
    try:
        k = bafe.compile_graph(_graph(rows))
    finally:
        bafe.set_option("gemm_precision", "auto")
    assert k.k_slice_align == 96, k.describe()
    return k


def _b_of_step(torch, step, device):
    g = torch.Generator(device=device).manual_seed(1000 + step)
    return torch.randn(K, N, device=device, generator=g) / K ** 0.5


def _panel(torch, rank, device):
    g = torch.Generator(device=device).manual_seed(10 + rank)
    return (torch.randn(M, K, device=device, generator=g) / K ** 0.5,
            torch.randn(M, N, device=device, generator=g) / K ** 0.5)


def _step(relay, k, s, chunk_bounds, last, A, B, C, out, comp, copy, watch, new_b, root):
    start = None
    if root:
        torch = __import__("torch")
        with torch.cuda.stream(comp):
            B.copy_(new_b)                         # the root's operand of this step
        start = torch.cuda.Event()
        start.record(comp)
    relay.send(s, chunk_bounds, copy, start)
    evs = relay.ready(s, last, watch)
    k.run_torch_ksliced([A, B, C], out, SLABS, ready=evs, stream=comp)
    relay.finish(s, comp)


def test_relay_three_ranks_one_gpu(cuda):
    torch = cuda
    ranks, steps = 3, 3
    k = _compile(M)
    relays, Bs = CopyEngineRelay.chain((K, N), [0] * ranks)
    try:
        chunk_bounds, last = relay_chunks(SLABS, N * 4, min_bytes=64 << 10)
        panels = [_panel(torch, r, "cuda") for r in range(ranks)]
        outs = [torch.empty(M, N, device="cuda") for _ in range(ranks)]
        comp = [torch.cuda.Stream() for _ in range(ranks)]
        copy = [torch.cuda.Stream() for _ in range(ranks)]
        watch = [torch.cuda.Stream() for _ in range(ranks)]
        new_b = [_b_of_step(torch, s, "cuda") for s in range(1, steps + 1)]
        torch.cuda.synchronize()
        snaps = []
        for s in range(1, steps + 1):
            row = []
            for r in range(ranks):
                A, C = panels[r]
                _step(relays[r], k, s, chunk_bounds, last, A, Bs[r], C, outs[r], comp[r], copy[r], watch[r],
                      new_b[s - 1], r == 0)
                with torch.cuda.stream(comp[r]):
                    row.append(outs[r].clone())
            snaps.append(row)
        torch.cuda.synchronize()
        bafe.synchronize()
        for s in range(1, steps + 1):
            for r in range(ranks):
                A, C = panels[r]
                ref = torch.empty(M, N, device="cuda")
                k.run_torch_ksliced([A, new_b[s - 1], C], ref, SLABS)
                torch.cuda.synchronize()
                assert torch.equal(snaps[s - 1][r], ref), (s, r)
        for r in range(ranks):
            assert torch.equal(Bs[r], new_b[-1]), r
    except BaseException:
        for rl in relays:                 # no stream may stay waiting on a flag nobody raises
            rl.release(steps)
        raise
    finally:
        torch.cuda.synchronize()
        for rl in relays:
            rl.close()


def _two_process_worker(rank, world, port, result_dir):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        k = _compile(M)
        relay, B, err = CopyEngineRelay.over_ranks((K, N), dist, rank)
        assert err is None, err
        chunk_bounds, last = relay_chunks(SLABS, N * 4, min_bytes=64 << 10)
        A, C = _panel(torch, rank, "cuda")
        out = torch.empty(M, N, device="cuda")
        comp, copy, watch = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
        steps = 3
        new_b = [_b_of_step(torch, s, "cuda") for s in range(1, steps + 1)]
        torch.cuda.synchronize()
        snaps = []
        try:
            for s in range(1, steps + 1):
                _step(relay, k, s, chunk_bounds, last, A, B, C, out, comp, copy, watch, new_b[s - 1], rank == 0)
                with torch.cuda.stream(comp):
                    snaps.append(out.clone())
        except BaseException:
            relay.release(steps)
            raise
        torch.cuda.synchronize()
        ok = []
        for s in range(1, steps + 1):
            ref = torch.empty(M, N, device="cuda")
            k.run_torch_ksliced([A, new_b[s - 1], C], ref, SLABS)
            torch.cuda.synchronize()
            ok.append(bool(torch.equal(snaps[s - 1], ref)))
        relay.close(dist)
        with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
            f.write(",".join(str(int(x)) for x in ok))
    finally:
        dist.destroy_process_group()


def test_relay_two_processes_two_gpus(cuda, tmp_path):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_two_process_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(2):
        assert open(tmp_path / f"rank{r}.txt").read() == "1,1,1", r
