"""Multi-rank host logic on CPU (gloo, world_size 2): row-panel sharding of
the fused GEMM, broadcast of the resident B, all-gather of the output, range
split of the elementwise chain, and a rank failure surfacing as an error on
the other rank.  Each rank computes its panel with the CPU oracle (the
product is the GPU kernel; here the sharding plumbing is under test)."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

from bafe_b200.parallel import element_ranges, relay_chunks, row_panels

ROOT = Path(__file__).resolve().parent.parent
PATHS = [str(ROOT / "bafe-basic-algibra-fusion-engine-_b200"), str(ROOT), str(ROOT / "tests" / "golden")]


def test_row_panels_cover_and_align():
    for M, W in [(16384, 8), (16384, 3), (300, 2), (5, 4), (128, 1), (1000, 7)]:
        p = row_panels(M, W)
        assert p[0][0] == 0 and p[-1][1] == M
        assert all(a <= b for a, b in p)
        assert all(p[i][1] == p[i + 1][0] for i in range(W - 1))
        if M >= 128 * W:
            assert all(a % 128 == 0 for a, _ in p)
            sizes = [b - a for a, b in p]
            assert max(sizes) - min(sizes) <= 128


def test_element_ranges_keep_vector_alignment():
    for n, W in [(1 << 28, 8), (1 << 28, 3), (1001, 2)]:
        r = element_ranges(n, W)
        assert r[0][0] == 0 and r[-1][1] == n
        if n >= 4 * W:
            assert all(a % 4 == 0 for a, _ in r)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, mode, q):
    for p in PATHS:
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime
    import torch
    import torch.distributed as dist
    from bafe_b200.graph import GraphBuilder
    from bafe_b200.parallel import broadcast_resident, gather_rows, row_panels
    from oracle import oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
    try:
        M, N, K = 300, 72, 40
        rng = np.random.default_rng(3)
        A = rng.standard_normal((M, K), dtype=np.float32)
        Bfull = rng.standard_normal((K, N), dtype=np.float32)
        C = rng.standard_normal((M, N), dtype=np.float32)
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before the broadcast")
        B = torch.from_numpy(Bfull.copy()) if rank == 0 else torch.zeros(K, N)
        broadcast_resident(B, dist)
        panels = row_panels(M, world)
        r0, r1 = panels[rank]

        def graph(rows):
            g = GraphBuilder()
            a = g.add_input("A", (rows, K), 0, 0)
            b = g.add_input("B", (K, N), 0, 2)
            c = g.add_input("C", (rows, N), 0, 0)
            g.set_output(g.add("relu", [g.add("add", [g.add("matmul", [a, b]), c])]))
            return g

        gp = graph(r1 - r0)
        ids = gp.inputs
        mine = oracle.evaluate(gp.to_list(), {ids[0]: A[r0:r1], ids[1]: B.numpy(), ids[2]: C[r0:r1]}, gp.output)
        full = gather_rows(torch.from_numpy(mine.reshape(r1 - r0, N)), M, dist, panels)
        if rank == 0:
            gf = graph(M)
            want = oracle.evaluate(gf.to_list(), dict(zip(gf.inputs, (A, Bfull, C))), gf.output)
            q.put(("ok", full.numpy().tobytes() == want.tobytes()))
    except Exception as e:   # reported to the parent
        q.put(("error", f"rank {rank}: {type(e).__name__}: {e}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _spawn(mode):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    out = []
    while not q.empty():
        out.append(q.get())
    return out


def test_sharded_gemm_equals_full_problem():
    res = _spawn("ok")
    assert ("ok", True) in res, res


def test_failed_rank_surfaces_as_error_on_the_other_rank():
    """Rank 1 raises before the collective; rank 0's broadcast ends with an
    error (short process-group timeout) instead of hanging."""
    res = _spawn("fail")
    errs = [m for kind, m in res if kind == "error"]
    assert any(m.startswith("rank 1") for m in errs), res
    assert any(m.startswith("rank 0") for m in errs), res


def _bcast_worker(rank, world, port, q):
    for p in PATHS:
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime
    import torch
    import torch.distributed as dist
    from bafe_b200.parallel import broadcast_resident

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
    try:
        want = torch.arange(64, dtype=torch.int16).reshape(8, 8) * 311
        t = want.clone() if rank == 0 else torch.zeros(8, 8, dtype=torch.int16)
        broadcast_resident(t, dist)
        q.put(("ok", bool(torch.equal(t, want))))
    except Exception as e:
        q.put(("error", f"rank {rank}: {type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


def test_broadcast_of_raw_half_buffers():
    """bf16 / f16 operands travel as raw 16-bit words; the broadcast moves
    their bytes (NCCL has no 16-bit integer type)."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_bcast_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    out = []
    while not q.empty():
        out.append(q.get())
    assert out == [("ok", True), ("ok", True)], out


def _shared_worker(rank, world, port, q):
    for p in PATHS:
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime
    import torch
    import torch.distributed as dist
    from bafe_b200.parallel import SharedInput

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
    try:
        sh = SharedInput(dist, device="cpu")
        ok = True
        for shape, dtype in [((37, 53), torch.float32), ((1001,), torch.int16), ((3, 5, 7), torch.float64)]:
            host = (torch.arange(int(np.prod(shape))) * 7 - 11).to(dtype).reshape(shape)
            got = sh.assemble(host)
            ok = ok and got.dtype == host.dtype and got.shape == host.shape and bool(torch.equal(got, host))
        q.put(("ok", ok))
    except Exception as e:
        q.put(("error", f"rank {rank}: {type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_shared_input_assembled_from_slabs(world):
    """Each rank copies its byte slab of the host buffer; the all-gather
    completes it on every rank (odd sizes: the last slab is short)."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_shared_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    out = []
    while not q.empty():
        out.append(q.get())
    assert out == [("ok", True)] * world, out


def test_k_slices_are_chunk_aligned_and_grow():
    from bafe_b200.parallel import k_slices
    for K, align in [(16384, 64), (16384, 1024), (16384, 2048), (4096, 64), (2048, 64), (64, 64), (1000, 64)]:
        b = k_slices(K, align)
        assert b[0] == 0 and b[-1] == K
        assert all(b[i] < b[i + 1] for i in range(len(b) - 1))
        assert all(x % align == 0 for x in b[1:-1])
        sizes = [b[i + 1] - b[i] for i in range(len(b) - 1)]
        # geometric growth up to the last slab, which is never under half of the one before
        assert all(sizes[i + 1] >= sizes[i] for i in range(len(sizes) - 2))
        if len(sizes) > 2:
            assert 2 * sizes[-1] >= sizes[-2]
    assert k_slices(16384, 64) == [0, 1024, 3072, 7168, 16384]


def test_transpose_blocks_cover_the_output_rows():
    """Each rank writes rows [c0, c1) of transpose(X) = columns [c0, c1) of
    X; together the blocks are the whole transpose."""
    from bafe_b200.parallel import transpose_blocks
    rng = np.random.default_rng(2)
    for rows, cols, world in [(300, 1000, 8), (64, 130, 3), (5, 7, 2), (16384 // 64, 16384, 8)]:
        X = rng.standard_normal((rows, cols)).astype(np.float32)
        blocks = transpose_blocks(cols, world)
        assert blocks[0][0] == 0 and blocks[-1][1] == cols
        assert all(blocks[i][1] == blocks[i + 1][0] for i in range(world - 1))
        if cols >= 64 * world:
            assert all(a % 64 == 0 for a, _ in blocks)
        parts = [np.ascontiguousarray(X[:, a:b].T) for a, b in blocks]   # each rank's own output rows
        assert np.concatenate(parts, axis=0).tobytes() == np.ascontiguousarray(X.T).tobytes()


def _slab_worker(rank, world, port, q):
    for p in PATHS:
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime
    import torch
    import torch.distributed as dist
    from bafe_b200.parallel import broadcast_slabs, k_slices

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
    try:
        K, N = 1000, 24
        want = torch.arange(K * N, dtype=torch.float32).reshape(K, N) * 0.5 - 3
        B = want.clone() if rank == 0 else torch.full((K, N), float("nan"))
        bounds = k_slices(K, 64)
        evs = broadcast_slabs(B, bounds, dist, src=0)
        q.put(("ok", bool(torch.equal(B, want)) and len(evs) == len(bounds) - 1 and len(bounds) > 2))
    except Exception as e:
        q.put(("error", f"rank {rank}: {type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_b_broadcast_in_k_slabs(world):
    """B crosses from the root slab by slab (contiguous row ranges); every
    rank ends with the root's B."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_slab_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    out = []
    while not q.empty():
        out.append(q.get())
    assert out == [("ok", True)] * world, out


def test_k_slab_schedule_follows_the_measured_times():
    from bafe_b200.parallel import k_slab_schedule
    K, align = 16384, 64
    for t_gemm, t_bcast, bd in [(18.4, 1.6, 0.16), (9.2, 1.7, 0.08), (4.6, 1.8, 0.04), (4.6, 0.2, 0.04)]:
        b = k_slab_schedule(K, align, t_gemm, t_bcast, bd, keep=132 / 148)
        assert b[0] == 0 and b[-1] == K and len(b) >= 3
        assert all(x % align == 0 for x in b[1:-1]) and all(b[i] < b[i + 1] for i in range(len(b) - 1))
        sizes = [b[i + 1] - b[i] for i in range(len(b) - 1)]
        assert sizes[0] <= K // 8                          # little of B waits for nothing to overlap it
        assert all(sizes[i + 1] > sizes[i] for i in range(len(sizes) - 1))
    # slower broadcast relative to the GEMM: more, more gradual slabs
    assert len(k_slab_schedule(K, align, 4.6, 1.8, 0.04, keep=0.9)) > len(k_slab_schedule(K, align, 18.4, 1.6, 0.16, keep=0.9))
    # a broadcast cheaper than a slice boundary is not worth slicing
    assert k_slab_schedule(K, align, 18.4, 0.05, 0.16, keep=0.9) == [0, K]
    assert k_slab_schedule(100, 64, 1.0, 1.0, 0.01) == [0, 100]


def test_relay_chunks_cover_the_slabs_in_whole_rows():
    slabs, row = [0, 96, 480, 1152], 512 * 4
    bounds, last = relay_chunks(slabs, row, min_bytes=64 << 10)
    assert bounds[0] == 0 and bounds[-1] == 1152 * row
    assert all(b > a for a, b in zip(bounds, bounds[1:]))
    assert all(b % row == 0 for b in bounds)
    assert [bounds[i + 1] // row for i in last] == slabs[1:]      # each slab ends on a chunk bound
    # the 16384^3 operand: a small first slab in a few chunks, later chunks at most 16 MiB
    big, last = relay_chunks([0, 96, 1056, 16384], 16384 * 4)
    assert len(big) - 1 <= 1023 and max(b - a for a, b in zip(big, big[1:])) <= 16 << 20
    assert last[0] >= 2
    with pytest.raises(ValueError):
        relay_chunks([0, 96, 96], row)
