"""K-sliced tensor-core GEMM (bafe_cuda_run_device_ksliced): the multi-GPU
path runs the GEMM over K slabs of B as they arrive.  Every slice continues
the fp32 sums the previous one left in the output, in the same promotion
chunks, and only the last applies the epilogue -- so the result must be
the single launch's bit for bit.

The single launch's last wave may split tail tiles along K (partials added
by a fixup kernel, a different rounding order); BAFE_TC_SPLIT=0 turns that
off for the bit-for-bit comparisons, and the default launch is compared
within the 3xTF32 bound.
"""
import numpy as np
import pytest

import bafe_b200 as bafe
from bafe_b200.graph import GraphBuilder
from bafe_b200.parallel import k_slices

pytestmark = pytest.mark.gpu


def _graph(M, N, K, epi=True):
    g = GraphBuilder()
    a = g.add_input("A", (M, K), 0, 0)
    b = g.add_input("B", (K, N), 0, 2)            # BLOCKED tag, row-major storage
    root = g.add("matmul", [a, b])
    if epi:
        c = g.add_input("C", (M, N), 0, 0)
        root = g.add("relu", [g.add("add", [root, c])])
    g.set_output(root)
    return g


def _compile_3xtf32(g):
    """The 3xTF32 plan (at 512^3 multiply-adds and below `auto` picks the
    exact CUDA-core kernel, which has no K slices)."""
    bafe.set_option("gemm_precision", "3xtf32")
    try:
        return bafe.compile_graph(g)
    finally:
        bafe.set_option("gemm_precision", "auto")


def _operands(torch, M, N, K, seed, epi=True):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    std = 1.0 / K ** 0.5
    ins = [torch.randn(M, K, device="cuda", generator=gen) * std, torch.randn(K, N, device="cuda", generator=gen) * std]
    if epi:
        ins.append(torch.randn(M, N, device="cuda", generator=gen) * std)
    return ins


def _whole(torch, k, ins, M, N, split):
    out = torch.empty(M, N, device="cuda")
    import os
    old = os.environ.get("BAFE_TC_SPLIT")
    os.environ["BAFE_TC_SPLIT"] = "1" if split else "0"
    try:
        k.run_torch(ins, out)
        torch.cuda.synchronize()
        bafe.synchronize()
    finally:
        if old is None:
            del os.environ["BAFE_TC_SPLIT"]
        else:
            os.environ["BAFE_TC_SPLIT"] = old
    return out


@pytest.mark.parametrize("precision,shape,chunks", [
    ("3xtf32", (512, 1024, 4096), [3, 11, 22]),       # interior bounds, in promotion chunks
    ("3xtf32", (768, 512, 2048), [1]),
    ("tf32", (512, 1024, 4096), [1, 3]),
])
def test_k_slices_equal_one_launch(cuda, precision, shape, chunks):
    torch = cuda
    M, N, K = shape
    bafe.set_option("gemm_precision", precision)
    try:
        k = bafe.compile_graph(_graph(M, N, K))
    finally:
        bafe.set_option("gemm_precision", "auto")
    assert "gemm.tc" in k.describe() and ".pair" in k.describe(), k.describe()
    align = k.k_slice_align
    assert align == (96 if precision == "3xtf32" else 1024)   # one promotion chunk
    bounds = [0] + [c * align for c in chunks] + [K]
    ins = _operands(torch, M, N, K, M + K)
    want = _whole(torch, k, ins, M, N, split=False)
    # slabs "arrive" on a side stream: each slice waits for its event
    side = torch.cuda.Stream()
    evs = []
    with torch.cuda.stream(side):
        torch.cuda._sleep(2_000_000)                 # the slabs land well after the call is enqueued
        for _ in range(len(bounds) - 1):
            e = torch.cuda.Event()
            e.record()
            evs.append(e)
    out = torch.full((M, N), float("nan"), device="cuda")
    before = bafe.launch_count()
    k.run_torch_ksliced(ins, out, bounds, ready=evs)
    torch.cuda.synchronize()
    bafe.synchronize()
    n = len(bounds) - 1
    # one GEMM launch per slice; 3xTF32 adds A's residual pass and a B split per slice
    assert bafe.launch_count() - before == (2 * n + 1 if precision == "3xtf32" else n)
    assert torch.equal(out, want)
    # the default launch (split tail) is within the 3xTF32 / tf32 bound of it
    dflt = _whole(torch, k, ins, M, N, split=True)
    ref = torch.relu(ins[0].double() @ ins[1].double() + ins[2].double())
    tol = (1e-4 if precision == "3xtf32" else 4e-2) * (K / 64) ** 0.5 / K
    assert float((dflt.double() - ref).abs().max()) <= tol
    assert float((out.double() - ref).abs().max()) <= tol


def test_k_slices_rank_panel_of_the_headline(cuda):
    """The per-rank problem of the 16384^3 GEMM on 8 GPUs (a 2048-row panel),
    sliced as the broadcast cuts B, with SMs left free for the collective:
    bit-identical to the single launch."""
    torch = cuda
    M, N, K = 2048, 16384, 16384
    k = bafe.compile_graph(_graph(M, N, K))
    assert "gemm.tc.3xtf32.pair" in k.describe(), k.describe()
    ins = _operands(torch, M, N, K, 17)
    want = _whole(torch, k, ins, M, N, split=False)
    bounds = k_slices(K, k.k_slice_align)
    assert len(bounds) > 3
    out = torch.empty(M, N, device="cuda")
    bafe.set_option("kslice_free_sms", "16")
    try:
        k.run_torch_ksliced(ins, out, bounds)
        torch.cuda.synchronize()
        bafe.synchronize()
    finally:
        bafe.set_option("kslice_free_sms", "0")
    assert torch.equal(out, want)


def test_k_slices_without_epilogue(cuda):
    """A plain matmul (no epilogue operands): the last slice stores the sums."""
    torch = cuda
    M, N, K = 256, 512, 1024
    k = _compile_3xtf32(_graph(M, N, K, epi=False))
    ins = _operands(torch, M, N, K, 5, epi=False)
    want = _whole(torch, k, ins, M, N, split=False)
    out = torch.empty(M, N, device="cuda")
    a = k.k_slice_align
    k.run_torch_ksliced(ins, out, [0, 2 * a, 6 * a, 1024])
    torch.cuda.synchronize()
    bafe.synchronize()
    assert torch.equal(out, want)


def test_k_slices_refused_where_they_do_not_apply(cuda):
    torch = cuda
    M, N, K = 256, 512, 1024
    bafe.set_option("gemm_precision", "exact")
    try:
        kx = bafe.compile_graph(_graph(M, N, K))
    finally:
        bafe.set_option("gemm_precision", "auto")
    assert kx.k_slice_align == 0
    ins = _operands(torch, M, N, K, 6)
    out = torch.empty(M, N, device="cuda")
    with pytest.raises(RuntimeError):
        kx.run_torch_ksliced(ins, out, [0, 512, 1024])
    k = _compile_3xtf32(_graph(M, N, K))
    a = k.k_slice_align
    for bad in ([0, a + 4, 1024], [0, 5 * a, 5 * a, 1024], [a, 1024], [0, 5 * a]):
        with pytest.raises(RuntimeError):
            k.run_torch_ksliced(ins, out, bad)
    # the context stays usable
    k.run_torch_ksliced(ins, out, [0, 5 * a, 1024])
    torch.cuda.synchronize()
    bafe.synchronize()
    assert torch.equal(out, _whole(torch, k, ins, M, N, split=False))
