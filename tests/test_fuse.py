"""Cross-call fusion (bafe.fuse) on the backend.

fuse(f, g) concatenates the traced graphs as fuse.c does (f's output feeds
g's first input) and compiles ONE plan, so the intermediate stays on the
device -- and, when it is consumed elementwise, is not stored at all.
CPU tests check the concatenation and the resulting plan (lowering needs no
GPU); GPU tests check results against the unfused calls and the oracle
(bafe/tests/test_fuse.py's cases: fused == sequential)."""
import numpy as np
import pytest

import bafe_b200 as bafe
from bafe_b200.graph import GraphBuilder


@bafe.jit
def mm(A, B):
    return bafe.matmul(A, B)


@bafe.jit
def relu_add(X, C):
    return bafe.relu(bafe.add(X, C))


@bafe.jit
def mul_add(X, Y, Z):
    return bafe.add(bafe.mul(X, Y), Z)


@bafe.jit
def relu1(X):
    return bafe.relu(X)


def test_concat_follows_fuse_c():
    a = GraphBuilder()
    A = a.add_input("A", (8, 4), 0, 0)
    B = a.add_input("B", (4, 6), 0, 0)
    a.set_output(a.add("matmul", [A, B]))
    b = GraphBuilder()
    X = b.add_input("X", (8, 6), 0, 0)
    C = b.add_input("C", (8, 6), 0, 0)
    b.set_output(b.add("relu", [b.add("add", [X, C])]))
    f = GraphBuilder.concat(a, b)
    nodes = f.to_list()
    assert len(nodes) == 3 + 4                    # b's first input node stays, unreferenced
    assert f.inputs == [0, 1, 3 + 1]              # a's inputs + b's inputs[1:]
    add = nodes[3 + 2]
    assert add["op"] == "add" and add["children"] == [2, 4]   # X -> a's output
    assert f.output == 3 + 3 and nodes[f.output]["op"] == "relu"


def test_fused_gemm_and_epilogue_become_one_kernel():
    h = bafe.fuse(mm, relu_add)
    A = np.zeros((256, 128), np.float32)
    B = np.zeros((128, 192), np.float32)
    C = np.zeros((256, 192), np.float32)
    k = h.kernel_for(A, B, C)
    steps = k.describe().strip().splitlines()
    assert len(steps) == 1 and steps[0].startswith("gemm.") and "epi=relu(add(acc,C))" in steps[0]


def test_fused_elementwise_chain_is_one_region():
    h = bafe.fuse(bafe.fuse(mul_add, relu1), relu1)
    X = np.zeros(1024, np.float32)
    assert h.n_args == 3
    steps = h.kernel_for(X, X, X).describe().strip().splitlines()
    assert steps == ["ew n=1024 float relu(relu(add(mul(X,Y),Z))) -> out"]


def test_fuse_rejects_plain_functions_and_bad_arity():
    with pytest.raises(TypeError):
        bafe.fuse(lambda a: a, relu1)
    h = bafe.fuse(mm, relu_add)
    with pytest.raises(TypeError):
        h.kernel_for(np.zeros((4, 4), np.float32), np.zeros((4, 4), np.float32))


@pytest.mark.gpu
def test_fused_equals_sequential_calls(cuda):
    rng = np.random.default_rng(4)
    A = rng.standard_normal((96, 64), dtype=np.float32)
    B = rng.standard_normal((64, 80), dtype=np.float32)
    C = rng.standard_normal((96, 80), dtype=np.float32)
    h = bafe.fuse(mm, relu_add)
    fused = h(A, B, C)
    seq = relu_add(mm(A, B), C)
    assert fused.tobytes() == seq.tobytes()       # exact GEMM path: same sums, same epilogue
    X, Y, Z = (rng.uniform(-1, 1, 1 << 20).astype(np.float32) for _ in range(3))
    h2 = bafe.fuse(bafe.fuse(mul_add, relu1), relu1)
    assert h2(X, Y, Z).tobytes() == relu1(relu1(mul_add(X, Y, Z))).tobytes()


@pytest.mark.gpu
def test_fused_large_gemm_epilogue_matches_unfused(cuda):
    rng = np.random.default_rng(5)
    M, K, N = 1024, 512, 768
    A = rng.standard_normal((M, K), dtype=np.float32)
    B = rng.standard_normal((K, N), dtype=np.float32)
    C = rng.standard_normal((M, N), dtype=np.float32)
    fused = bafe.fuse(mm, relu_add)(A, B, C)
    seq = relu_add(mm(A, B), C)                   # 3xTF32: same products, one rounding less in the middle
    ref = np.maximum(A.astype(np.float64) @ B.astype(np.float64) + C, 0)
    bound = 1e-4 * np.sqrt(K / 64)
    assert np.abs(fused - ref).max() <= bound and np.abs(seq - ref).max() <= bound


# ---- pinned to the reference: tests/golden/fuse_*.npz hold the output of
# the reference's own fused kernel (f and g optimized apart,
# bafe_fuse_concat, optimized again, its JIT) on seeded inputs ------------

@bafe.jit
def mm_x(X, C):
    return bafe.matmul(X, C)


@bafe.jit
def relu_x(X):
    return bafe.relu(X)


@bafe.jit
def relu_add_x(X, C):
    return bafe.relu(X + C)


FNS = {"matmul": (mm, mm_x), "relu": (None, relu_x), "relu_add": (None, relu_add_x)}


def _fuse_case_args(name):
    import cases
    meta, stored, golden = cases.load(name)
    args = []
    for spec in meta["inputs"]:
        if spec["name"] in stored:
            args.append(stored[spec["name"]])
        else:
            t = (spec["name"], tuple(spec["shape"]), spec["dtype"], spec["fortran"], spec["layout"], spec["spec"])
            args.append(cases.make_input(t))
    f_name, g_name = meta["fuse"]
    return bafe.fuse(FNS[f_name][0], FNS[g_name][1]), args, golden


FUSE_CASES = ["fuse_two_matmuls", "fuse_matmul_then_relu", "fuse_matmul_then_add_bias",
              "fuse_matmul_then_relu_64x64", "fuse_gemm_then_relu_add_c_256"]


@pytest.mark.gpu
@pytest.mark.parametrize("name", FUSE_CASES)
def test_fused_call_is_bit_exact_to_reference_fuse(cuda, name):
    """h = bafe.fuse(f, g) called with numpy arrays, `exact` GEMM precision:
    the device-resident fused plan reproduces the reference's fused kernel
    bit for bit."""
    bafe.set_option("gemm_precision", "exact")
    try:
        h, args, golden = _fuse_case_args(name)
        out = h(*args)
    finally:
        bafe.set_option("gemm_precision", "auto")
    assert out.shape == golden.shape
    assert out.tobytes() == np.ascontiguousarray(golden).tobytes(), h.kernel_for(*args).describe()


@pytest.mark.gpu
def test_fused_tensor_core_plan_matches_reference_fuse(cuda):
    """The 256 x 320 x 256 fused case with 3xTF32 requested runs one
    tensor-core kernel with the epilogue fused; it stays within
    1e-4 * sqrt(K/64) * rms(A) * rms(B) of the reference's fused output."""
    bafe.set_option("gemm_precision", "3xtf32")
    try:
        h, args, golden = _fuse_case_args("fuse_gemm_then_relu_add_c_256")
        k = h.kernel_for(*args)
        steps = k.describe().strip().splitlines()
        assert "gemm.tc.3xtf32" in steps[-1] and "epi=relu(add(acc,C))" in steps[-1], k.describe()
        out = h(*args)
    finally:
        bafe.set_option("gemm_precision", "auto")
    A, B = (a.astype(np.float64) for a in args[:2])
    bound = 1e-4 * np.sqrt(A.shape[1] / 64) * np.sqrt(np.mean(A * A)) * np.sqrt(np.mean(B * B))
    err = float(np.abs(out.astype(np.float64) - golden).max())
    print(f"fused 3xTF32 vs the reference's fused kernel: max |err| {err:.3e} (bound {bound:.3e})")
    assert err <= bound
