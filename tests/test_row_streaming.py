"""Row-streamed host calls.

A host-pointer call of a row-separable plan copies the row-split inputs,
runs the kernels and copies the output back in row panels on three streams
(host_panels option).  CPU tests check which inputs split (the analysis
runs when the plan is built, without a GPU); GPU tests check that a
streamed call returns exactly what the one-piece call returns, on ragged
panel sizes, row-vector operands, the exact GEMM, the 3xTF32 tensor-core
GEMM and the elementwise chain."""
import numpy as np
import pytest

import bafe_b200 as bafe
from bafe_b200.graph import GraphBuilder

import oracle.oracle as oracle


def _kernel(build, *inputs):
    g = GraphBuilder()
    ids = [g.add_input(n, s, dt, lay) for (n, s, dt, lay) in inputs]
    g.set_output(build(g, *ids))
    return bafe.compile_graph(g), g


def _gemm_relu_add(g, A, B, C):
    return g.add("relu", [g.add("add", [g.add("matmul", [A, B]), C])])


def test_fused_gemm_splits_a_and_c_keeps_b_whole():
    for prec in ("3xtf32", "tf32", "exact"):
        bafe.set_option("gemm_precision", prec)
        k, _ = _kernel(_gemm_relu_add, ("A", (16384, 16384), 0, 0), ("B", (16384, 16384), 0, 2),
                       ("C", (16384, 16384), 0, 0))
        rows, in_rb, out_rb = k.row_split()
        assert rows == 16384 and in_rb == [16384 * 4, 0, 16384 * 4] and out_rb == 16384 * 4, prec


def test_gemm_epilogue_product_and_bias_vector():
    k, _ = _kernel(lambda g, A, B, C, D, b: g.add("relu", [g.add("add", [
        g.add("add", [g.add("matmul", [A, B]), g.add("mul", [C, D])]), b])]),
                   ("A", (4096, 512), 0, 0), ("B", (512, 1024), 0, 0), ("C", (4096, 1024), 0, 0),
                   ("D", (4096, 1024), 0, 0), ("b", (1024,), 0, 0))
    rows, in_rb, out_rb = k.row_split()
    assert rows == 4096 and in_rb == [512 * 4, 0, 1024 * 4, 1024 * 4, 0] and out_rb == 1024 * 4


def test_elementwise_chain_splits_every_operand():
    k, _ = _kernel(lambda g, X, Y, Z: g.add("relu", [g.add("add", [g.add("mul", [X, Y]), Z])]),
                   ("X", (1 << 28,), 0, 0), ("Y", (1 << 28,), 0, 0), ("Z", (1 << 28,), 0, 0))
    assert k.row_split() == (1 << 28, [4, 4, 4], 4)


def test_column_major_a_and_transpose_are_not_streamed():
    bafe.set_option("gemm_precision", "3xtf32")
    k, _ = _kernel(_gemm_relu_add, ("A", (1024, 512), 0, 1), ("B", (512, 256), 0, 0), ("C", (1024, 256), 0, 0))
    assert k.row_split() is None
    k, _ = _kernel(lambda g, X: g.add("relu", [g.add("transpose", [X], perm=[1, 0])]), ("X", (512, 768), 0, 0))
    assert k.row_split() is None


def test_host_panels_option_round_trip():
    assert bafe.get_option("host_panels") == "auto"
    bafe.set_option("host_panels", "5")
    assert bafe.get_option("host_panels") == "5"
    with pytest.raises(Exception):
        bafe.set_option("host_panels", "-2")
    bafe.set_option("host_panels", "auto")


def _both(k, arrays, panels):
    bafe.set_option("host_panels", "0")
    whole = k(*arrays)
    bafe.set_option("host_panels", str(panels))
    split = k(*arrays)
    bafe.set_option("host_panels", "auto")
    return whole, split


@pytest.mark.gpu
def test_streamed_exact_gemm_with_bias_is_bit_identical(cuda):
    bafe.set_option("gemm_precision", "exact")
    M, K, N = 1000, 96, 40       # 1000 rows: panels of 256, 256, 256, 232
    rng = np.random.default_rng(5)
    A = rng.standard_normal((M, K), dtype=np.float32)
    B = rng.standard_normal((K, N), dtype=np.float32)
    b = rng.standard_normal(N, dtype=np.float32)
    k, g = _kernel(lambda g, A_, B_, b_: g.add("relu", [g.add("add", [g.add("matmul", [A_, B_]), b_])]),
                   ("A", (M, K), 0, 0), ("B", (K, N), 0, 0), ("b", (N,), 0, 0))
    whole, split = _both(k, (A, B, b), 4)
    np.testing.assert_array_equal(split, whole)
    want = oracle.evaluate(g.to_list(), dict(zip(g.inputs, (A, B, b))), g.output)
    assert split.tobytes() == want.reshape(M, N).tobytes()


@pytest.mark.gpu
def test_streamed_tensor_core_gemm_matches_one_piece(cuda):
    bafe.set_option("gemm_precision", "3xtf32")
    M, K, N = 2304, 512, 768     # 9 row blocks of 256 over 4 panels
    rng = np.random.default_rng(6)
    A = rng.standard_normal((M, K), dtype=np.float32)
    B = rng.standard_normal((K, N), dtype=np.float32)
    C = rng.standard_normal((M, N), dtype=np.float32)
    k, _ = _kernel(_gemm_relu_add, ("A", (M, K), 0, 0), ("B", (K, N), 0, 0), ("C", (M, N), 0, 0))
    assert "gemm.tc.3xtf32" in k.describe()
    whole, split = _both(k, (A, B, C), 4)
    bound = 1e-4 * np.sqrt(K / 64)
    ref = np.maximum(A.astype(np.float64) @ B.astype(np.float64) + C, 0)
    assert np.abs(split - ref).max() <= bound
    assert np.abs(split - whole).max() <= bound


@pytest.mark.gpu
def test_streamed_elementwise_chain_ragged_is_bit_identical(cuda):
    n = (1 << 22) + 100          # last panel ragged
    rng = np.random.default_rng(7)
    X, Y, Z = (rng.uniform(-1, 1, n).astype(np.float32) for _ in range(3))
    k, g = _kernel(lambda g, X_, Y_, Z_: g.add("relu", [g.add("add", [g.add("mul", [X_, Y_]), Z_])]),
                   ("X", (n,), 0, 0), ("Y", (n,), 0, 0), ("Z", (n,), 0, 0))
    whole, split = _both(k, (X, Y, Z), 5)
    assert split.tobytes() == whole.tobytes()
    want = oracle.evaluate(g.to_list(), dict(zip(g.inputs, (X, Y, Z))), g.output)
    assert split.tobytes() == want.tobytes()


@pytest.mark.gpu
def test_streamed_row_vector_broadcast_is_bit_identical(cuda):
    rng = np.random.default_rng(8)
    X = rng.standard_normal((1000, 96), dtype=np.float32)
    v = rng.standard_normal(96, dtype=np.float32)
    k, g = _kernel(lambda g, X_, v_: g.add("relu", [g.add("add", [X_, v_])]), ("X", (1000, 96), 0, 0),
                   ("v", (96,), 0, 0))
    assert k.row_split() == (1000, [96 * 4, 0], 96 * 4)
    whole, split = _both(k, (X, v), 3)
    assert split.tobytes() == whole.tobytes()
    want = oracle.evaluate(g.to_list(), dict(zip(g.inputs, (X, v))), g.output)
    assert split.tobytes() == want.tobytes()


@pytest.mark.gpu
def test_auto_streaming_on_pinned_buffers(cuda):
    """A call large enough for the automatic split, on pinned host memory
    (the bench's end-to-end path)."""
    torch = cuda
    n = 1 << 25                  # 3 x 128 MiB in, 128 MiB out
    gen = torch.Generator().manual_seed(9)
    X, Y, Z = (torch.rand(n, generator=gen).mul_(2).sub_(1).pin_memory() for _ in range(3))
    out = torch.zeros(n).pin_memory()
    k, g = _kernel(lambda g, X_, Y_, Z_: g.add("relu", [g.add("add", [g.add("mul", [X_, Y_]), Z_])]),
                   ("X", (n,), 0, 0), ("Y", (n,), 0, 0), ("Z", (n,), 0, 0))
    k.call_host_ptrs([t.data_ptr() for t in (X, Y, Z)] + [out.data_ptr()])
    want = torch.relu(X * Y + Z)     # three separately rounded fp32 ops, relu(-0) = 0
    assert torch.equal(out, want)


@pytest.mark.gpu
@pytest.mark.parametrize("panels", ["0", "4"])
def test_host_call_with_a_resident_input(cuda, panels):
    """bafe_cuda_run_host_resident: B already on the device (a multi-GPU
    caller assembles it over NVLink), A, C and the output on the host;
    bit-identical to the plain host call and the oracle, streamed or in one
    piece."""
    torch = cuda
    bafe.set_option("gemm_precision", "exact")
    M, K, N = 1000, 96, 40
    gen = torch.Generator().manual_seed(10)
    A, B, C = (torch.randn(*s, generator=gen) for s in ((M, K), (K, N), (M, N)))
    k, g = _kernel(_gemm_relu_add, ("A", (M, K), 0, 0), ("B", (K, N), 0, 0), ("C", (M, N), 0, 0))
    bafe.set_option("host_panels", panels)
    try:
        want = torch.zeros(M, N)
        k.call_host_ptrs([A.data_ptr(), B.data_ptr(), C.data_ptr(), want.data_ptr()])
        Bd = B.cuda()
        torch.cuda.synchronize()
        got = torch.zeros(M, N)
        k.call_host_resident([A.data_ptr(), Bd.data_ptr(), C.data_ptr(), got.data_ptr()], [False, True, False])
    finally:
        bafe.set_option("host_panels", "auto")
    assert torch.equal(got, want)
    ref = oracle.evaluate(g.to_list(), dict(zip(g.inputs, (A.numpy(), B.numpy(), C.numpy()))), g.output)
    assert got.numpy().tobytes() == ref.reshape(M, N).tobytes()


@pytest.mark.gpu
@pytest.mark.parametrize("shape,dtype,panels", [
    ((1000, 768), np.float32, 4),      # 16-byte kernel; panels of 192 output rows
    ((517, 333), np.float32, 3),       # scalar kernel; panels of 128, 128, 77 rows
    ((300, 260), np.float64, 2),       # 8-byte elements
])
def test_streamed_transpose_is_bit_identical(cuda, shape, dtype, panels):
    """A plan that is one transpose streams by output rows: each panel's
    input is a band of x's columns (one strided copy), so the input and
    output copies overlap.  Same bits as one piece and as x.T."""
    rng = np.random.default_rng(12)
    X = rng.standard_normal(shape).astype(dtype)
    dt = 0 if dtype == np.float32 else 1
    k, g = _kernel(lambda g, X_: g.add("transpose", [X_], perm=[1, 0]), ("X", shape, dt, 0))
    assert k.row_split() is None              # not a row split: x splits by columns
    whole, split = _both(k, (X,), panels)
    assert split.tobytes() == whole.tobytes()
    assert split.tobytes() == np.ascontiguousarray(X.T).tobytes()


@pytest.mark.gpu
@pytest.mark.parametrize("panels", ["0", "4"])
def test_resident_input_filled_after_the_call_starts(cuda, panels):
    """The resident input is written on another stream, behind ~25 ms of
    other work, and the call gets the event recorded after it: the kernels
    wait (reading the buffer early would compute with its zeros)."""
    torch = cuda
    bafe.set_option("gemm_precision", "exact")
    M, K, N = 1000, 96, 40
    gen = torch.Generator().manual_seed(13)
    A, B, C = (torch.randn(*s, generator=gen) for s in ((M, K), (K, N), (M, N)))
    Bpin = B.pin_memory()
    k, _ = _kernel(_gemm_relu_add, ("A", (M, K), 0, 0), ("B", (K, N), 0, 0), ("C", (M, N), 0, 0))
    want = torch.zeros(M, N)
    k.call_host_ptrs([A.data_ptr(), B.data_ptr(), C.data_ptr(), want.data_ptr()])
    Bd = torch.zeros(K, N, device="cuda")
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    ready = torch.cuda.Event()
    with torch.cuda.stream(side):
        torch.cuda._sleep(50_000_000)             # a bounded spin, then the real values
        Bd.copy_(Bpin, non_blocking=True)
        ready.record(side)
    bafe.set_option("host_panels", panels)
    try:
        got = torch.zeros(M, N)
        k.call_host_resident([A.data_ptr(), Bd.data_ptr(), C.data_ptr(), got.data_ptr()], [False, True, False], ready)
    finally:
        bafe.set_option("host_panels", "auto")
    assert torch.equal(got, want)


@pytest.mark.gpu
def test_run_host_shared_on_one_rank(cuda):
    """parallel.run_host_shared without a process group: the shared input is
    copied to the device (one slab), the call reads it in place after the
    ready event; same bits as the plain host call."""
    torch = cuda
    from bafe_b200.parallel import SharedInput, run_host_shared
    bafe.set_option("gemm_precision", "exact")
    M, K, N = 1000, 96, 40
    gen = torch.Generator().manual_seed(14)
    A, B, C = (torch.randn(*s, generator=gen).pin_memory() for s in ((M, K), (K, N), (M, N)))
    k, _ = _kernel(_gemm_relu_add, ("A", (M, K), 0, 0), ("B", (K, N), 0, 0), ("C", (M, N), 0, 0))
    want = torch.zeros(M, N)
    k.call_host_ptrs([A.data_ptr(), B.data_ptr(), C.data_ptr(), want.data_ptr()])
    sh = SharedInput(None)
    for _ in range(2):                               # the device buffer is reused
        got = torch.zeros(M, N).pin_memory()
        run_host_shared(k, [A, B, C], got, {1: sh})
        assert torch.equal(got, want)
