"""Tensor-core GEMM (tcgen05, kind::tf32) parity.

Bounds (inputs N(0,1) unless stated; K = inner dimension):
  * 3xTF32: max |out - reference| <= 1e-4 * sqrt(K/64), the north-star
    bound, against both an fp64 evaluation and the reference's own fp32
    result (golden row panels, exact reference summation order);
  * 1xTF32: max |out - fp64| <= TF32_TOL * sqrt(K/64) with
    TF32_TOL = 4e-2, and the relative tolerance
    |out - fp64| <= 2^-9 * (|A| |B|) elementwise (measured maxima are
    printed by the tests).
Operands are device-resident (torch); column-major operands are passed as
their transposed row-major storage with the COL_MAJOR tag.
"""
import math

import numpy as np
import pytest

import bafe_b200 as bafe
import cases

pytestmark = pytest.mark.gpu

TF32_TOL = 4e-2
# 1xTF32 relative tolerance, elementwise against |A| |B| (the sum of the
# products' magnitudes): both operands lose up to 2^-10 of their value to
# tf32's 10-bit mantissa, so each product is within 2^-9 of its exact value.
TF32_REL_TOL = 2.0 ** -9


def _graph(M, N, K, a_col, b_col, epi):
    g = bafe.GraphBuilder()
    a = g.add_input("A", (M, K), 0, 1 if a_col else 0)
    b = g.add_input("B", (K, N), 0, 1 if b_col else 0)
    mm = g.add("matmul", [a, b])
    if epi == "none":
        root = mm
    elif epi == "relu_add_c":
        c = g.add_input("C", (M, N), 0, 0)
        root = g.add("relu", [g.add("add", [mm, c])])
    elif epi == "relu_add_mul":
        c = g.add_input("C", (M, N), 0, 0)
        d = g.add_input("D", (M, N), 0, 0)
        root = g.add("relu", [g.add("add", [mm, g.add("mul", [c, d])])])
    elif epi == "relu_bias":
        c = g.add_input("bias", (N,), 0, 0)
        root = g.add("relu", [g.add("add", [mm, c])])
    else:
        raise ValueError(epi)
    g.set_output(root)
    return g


def _run(torch, M, N, K, a_col, b_col, epi, prec, seed=0, scale=1.0):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn(M, K, device="cuda", generator=gen) * scale
    B = torch.randn(K, N, device="cuda", generator=gen) * scale
    extra = []
    if epi in ("relu_add_c", "relu_add_mul"):
        extra.append(torch.randn(M, N, device="cuda", generator=gen))
    if epi == "relu_add_mul":
        extra.append(torch.randn(M, N, device="cuda", generator=gen))
    if epi == "relu_bias":
        extra.append(torch.randn(N, device="cuda", generator=gen))
    bafe.set_option("gemm_precision", prec)
    k = bafe.compile_graph(_graph(M, N, K, a_col, b_col, epi))
    a_store = A.t().contiguous() if a_col else A
    b_store = B.t().contiguous() if b_col else B
    out = torch.empty(M, N, device="cuda")
    k.run_torch([a_store, b_store] + extra, out)
    bafe.synchronize()
    ref = A.double() @ B.double()
    if epi == "relu_add_c":
        ref = torch.relu(ref + extra[0].double())
    elif epi == "relu_add_mul":
        ref = torch.relu(ref + (extra[0] * extra[1]).double())
    elif epi == "relu_bias":
        ref = torch.relu(ref + extra[0].double())
    err = float((out.double() - ref).abs().max())
    scale = A.double().abs() @ B.double().abs()
    rel = float(((out.double() - ref).abs() / scale).max())
    _run.last_rel = rel
    return k, out, err


SHAPES = [(128, 256, 32), (256, 256, 256), (300, 520, 100), (1000, 768, 1024), (132, 260, 36)]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("a_col,b_col", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_3xtf32_layouts_and_shapes(cuda, shape, a_col, b_col):
    M, N, K = shape
    k, out, err = _run(cuda, M, N, K, a_col, b_col, "none", "3xtf32")
    assert "gemm.tc.3xtf32" in k.describe()
    bound = 1e-4 * math.sqrt(K / 64)
    print(f"3xtf32 {shape} a_col={a_col} b_col={b_col}: max err {err:.3e} (bound {bound:.1e})")
    assert err <= bound


@pytest.mark.parametrize("epi", ["relu_add_c", "relu_add_mul", "relu_bias"])
def test_3xtf32_fused_epilogues(cuda, epi):
    k, out, err = _run(cuda, 512, 512, 512, 0, 0, epi, "3xtf32", seed=3)
    steps = k.describe().strip().splitlines()
    # residual pre-passes for A and B, then one GEMM carrying the epilogue
    assert [l.split()[0].replace(".pair", "") for l in steps] == ["ew", "ew", "gemm.tc.3xtf32"], steps
    assert "tf32_split(A)" in steps[0] and "tf32_residual(B)" in steps[1]
    bound = 1e-4 * math.sqrt(512 / 64)
    print(f"3xtf32 epilogue {epi}: max err {err:.3e}")
    assert err <= bound


@pytest.mark.parametrize("shape", [(256, 256, 256), (1000, 768, 1024), (2048, 2048, 2048)])
@pytest.mark.parametrize("a_col,b_col", [(0, 0), (1, 1)])
def test_tf32(cuda, shape, a_col, b_col):
    M, N, K = shape
    k, out, err = _run(cuda, M, N, K, a_col, b_col, "relu_add_c", "tf32", seed=5)
    assert "gemm.tc.tf32" in k.describe()
    bound = TF32_TOL * math.sqrt(K / 64)
    rel = _run.last_rel
    print(f"tf32 {shape} a_col={a_col} b_col={b_col}: max err {err:.3e} (bound {bound:.1e}), "
          f"max |err| / (|A||B|) {rel:.3e} (tolerance {TF32_REL_TOL:.3e})")
    assert err <= bound
    assert rel <= TF32_REL_TOL


def test_3xtf32_large_many_tiles(cuda):
    """4096^3 (512 tiles over 148 persistent CTAs, both accumulators cycling)."""
    k, out, err = _run(cuda, 4096, 4096, 4096, 0, 0, "relu_add_mul", "3xtf32", seed=9)
    bound = 1e-4 * math.sqrt(4096 / 64)
    print(f"3xtf32 4096^3 relu(add(mm, C*D)): max err {err:.3e} (bound {bound:.1e})")
    assert err <= bound


def test_host_pointer_path_tensor_cores(cuda):
    """The legacy host-pointer function on a tensor-core plan."""
    rng = np.random.default_rng(1)
    A = rng.standard_normal((512, 384), dtype=np.float32)
    B = np.asfortranarray(rng.standard_normal((384, 640), dtype=np.float32))
    C = rng.standard_normal((512, 640), dtype=np.float32)

    @bafe.jit
    def f(A, B, C):
        return bafe.relu(bafe.matmul(A, B) + C)

    bafe.set_option("gemm_precision", "3xtf32")
    out = f(A, B, C)
    ref = np.maximum(A.astype(np.float64) @ B.astype(np.float64) + C, 0)
    assert "a=row b=col" in f.kernel_for(A, B, C).describe()
    assert np.max(np.abs(out - ref)) <= 1e-4 * math.sqrt(384 / 64)


# ---------------------------------------------------------------- batched --
# Rank-3 products (the emitter's batched loop, codegen.c:215-236): each batch
# item is its own GEMM; an operand without a batch dimension is shared.  The
# tensor-core kernels take the batch index as the third TMA coordinate.

@pytest.mark.parametrize("batch,M,N,K,a_col,b_col,b_shared", [
    (3, 256, 320, 192, 0, 0, False),
    (4, 300, 260, 520, 1, 1, False),
    (5, 512, 256, 256, 0, 1, True),
    (2, 128, 1024, 2048, 1, 0, True),
])
@pytest.mark.parametrize("prec", ["3xtf32", "tf32"])
@pytest.mark.parametrize("pair", ["1", "0"])
def test_batched_gemm_on_tensor_cores(cuda, batch, M, N, K, a_col, b_col, b_shared, prec, pair):
    torch = cuda
    gen = torch.Generator(device="cuda").manual_seed(batch * 131 + M)
    A = torch.randn(batch, M, K, device="cuda", generator=gen)
    B = torch.randn(K, N, device="cuda", generator=gen) if b_shared else \
        torch.randn(batch, K, N, device="cuda", generator=gen)
    C = torch.randn(batch, M, N, device="cuda", generator=gen)
    g = bafe.GraphBuilder()
    a = g.add_input("A", (batch, M, K), 0, 1 if a_col else 0)
    b = g.add_input("B", tuple(B.shape), 0, 1 if b_col else 0)
    c = g.add_input("C", (batch, M, N), 0, 0)
    g.set_output(g.add("relu", [g.add("add", [g.add("matmul", [a, b]), c])]))
    bafe.set_option("gemm_precision", prec)
    bafe.set_option("tc_pair", pair)
    try:
        k = bafe.compile_graph(g)
        assert ("gemm.tc.3xtf32" if prec == "3xtf32" else "gemm.tc.tf32") in k.describe()
        assert f"batch={batch}" in k.describe()
        a_store = A.transpose(1, 2).contiguous() if a_col else A
        b_store = B.transpose(-1, -2).contiguous() if b_col else B
        out = torch.full((batch, M, N), float("nan"), device="cuda")
        k.run_torch([a_store, b_store, C], out)
        bafe.synchronize()
    finally:
        bafe.set_option("tc_pair", "1")
    ref = torch.relu(torch.matmul(A.double(), B.double()) + C.double())
    err = float((out.double() - ref).abs().max())
    tol = (1e-4 if prec == "3xtf32" else TF32_TOL) * math.sqrt(K / 64)
    print(f"batched {prec} pair={pair} {batch}x{M}x{N}x{K}: max err {err:.3e} (bound {tol:.3e})")
    assert err <= tol


# ------------------------------------------------- in-kernel residuals --
# tc_convert=1: the kernel makes the tf32 residuals in shared memory (no
# pre-pass, no scratch); same products, same bound.

@pytest.mark.parametrize("shape,a_col,b_col", [((512, 512, 512), 0, 0), ((300, 260, 1000), 1, 1),
                                               ((1024, 768, 4096), 0, 1), ((4096, 4096, 4096), 0, 0)])
@pytest.mark.parametrize("pair", ["1", "0"])
def test_3xtf32_in_kernel_residuals(cuda, shape, a_col, b_col, pair):
    M, N, K = shape
    bafe.set_option("tc_convert", "1")
    bafe.set_option("tc_pair", pair)
    try:
        k, out, err = _run(cuda, M, N, K, a_col, b_col, "relu_add_c", "3xtf32", seed=11)
    finally:
        bafe.set_option("tc_convert", "auto")
        bafe.set_option("tc_pair", "1")
    steps = k.describe().strip().splitlines()
    assert len(steps) == 1 and steps[0].startswith("gemm.tc.3xtf32"), steps
    bound = 1e-4 * math.sqrt(K / 64)
    print(f"3xtf32 in-kernel residuals {shape} pair={pair}: max err {err:.3e} (bound {bound:.1e})")
    assert err <= bound


def test_prepared_launch_follows_new_buffers(cuda):
    """The runtime reuses a step's prepared tensor maps while its buffers stay
    the same; new input / epilogue / output buffers must be picked up."""
    torch = cuda
    bafe.set_option("gemm_precision", "3xtf32")
    k = bafe.compile_graph(_graph(512, 384, 256, 0, 0, "relu_add_c"))
    gen = torch.Generator(device="cuda").manual_seed(21)
    outs = []
    for it in range(3):
        A = torch.randn(512, 256, device="cuda", generator=gen)
        B = torch.randn(256, 384, device="cuda", generator=gen)
        C = torch.randn(512, 384, device="cuda", generator=gen)
        out = torch.empty(512, 384, device="cuda")
        for _ in range(2):                               # second call reuses the prepared launch
            k.run_torch([A, B, C], out)
        bafe.synchronize()
        ref = torch.relu(A.double() @ B.double() + C.double())
        assert float((out.double() - ref).abs().max()) <= 1e-4 * math.sqrt(256 / 64), it
        outs.append(out)


# ------------------------------------------------------------ epilogue --
# Epilogue operands are read as 4-element vectors when every one is aligned
# for that (16 bytes; 8 for 16-bit operands), element by element otherwise;
# the output is written by TMA stores from shared memory, which clip rows
# >= M and columns >= N.

@pytest.mark.parametrize("prec", ["tf32", "3xtf32"])
@pytest.mark.parametrize("pair", ["1", "0"])
def test_epilogue_operands_off_vector_alignment(cuda, prec, pair):
    """C at a 4-byte and the bias at a 12-byte offset: element reads."""
    torch = cuda
    M, N, K = 300, 516, 256
    gen = torch.Generator(device="cuda").manual_seed(31)
    A = torch.randn(M, K, device="cuda", generator=gen)
    B = torch.randn(K, N, device="cuda", generator=gen)
    C = torch.randn(M * N + 1, device="cuda", generator=gen)[1:].view(M, N)
    bias = torch.randn(N + 3, device="cuda", generator=gen)[3:]
    assert C.data_ptr() % 16 == 4 and bias.data_ptr() % 16 == 12
    g = bafe.GraphBuilder()
    a = g.add_input("A", (M, K), 0, 0)
    b = g.add_input("B", (K, N), 0, 0)
    c = g.add_input("C", (M, N), 0, 0)
    v = g.add_input("bias", (N,), 0, 0)
    g.set_output(g.add("relu", [g.add("add", [g.add("add", [g.add("matmul", [a, b]), c]), v])]))
    bafe.set_option("gemm_precision", prec)
    bafe.set_option("tc_pair", pair)
    try:
        k = bafe.compile_graph(g)
        assert "gemm.tc" in k.describe()
        out = torch.full((M, N), float("nan"), device="cuda")
        k.run_torch([A, B, C, bias], out)
        bafe.synchronize()
    finally:
        bafe.set_option("tc_pair", "1")
    ref = torch.relu(A.double() @ B.double() + C.double() + bias.double())
    err = float((out.double() - ref).abs().max())
    tol = (1e-4 if prec == "3xtf32" else TF32_TOL) * math.sqrt(K / 64)
    print(f"misaligned epilogue operands {prec} pair={pair}: max err {err:.3e}")
    assert err <= tol


@pytest.mark.parametrize("pair", ["1", "0"])
def test_epilogue_half_operands(cuda, pair):
    """f16 and bf16 epilogue operands (8-byte vectors), f32 output, ragged tiles."""
    torch = cuda
    M, N, K = 520, 388, 320
    gen = torch.Generator(device="cuda").manual_seed(37)
    A = torch.randn(M, K, device="cuda", generator=gen)
    B = torch.randn(K, N, device="cuda", generator=gen)
    C = torch.randn(M, N, device="cuda", generator=gen).to(torch.float16)
    D = torch.randn(N, device="cuda", generator=gen).to(torch.bfloat16)
    g = bafe.GraphBuilder()
    a = g.add_input("A", (M, K), 0, 0)
    b = g.add_input("B", (K, N), 0, 0)
    c = g.add_input("C", (M, N), 4, 0)
    d = g.add_input("D", (N,), 5, 0)
    g.set_output(g.add("mul", [g.add("add", [g.add("matmul", [a, b]), c]), d]))
    bafe.set_option("gemm_precision", "3xtf32")
    bafe.set_option("tc_pair", pair)
    try:
        k = bafe.compile_graph(g)
        assert "gemm.tc.3xtf32" in k.describe()
        out = torch.full((M, N), float("nan"), device="cuda")
        k.run_torch([A, B, C.view(torch.int16), D.view(torch.int16)], out)
        bafe.synchronize()
    finally:
        bafe.set_option("tc_pair", "1")
    ref = (A.double() @ B.double() + C.double()) * D.double()
    err = float((out.double() - ref).abs().max())
    print(f"half epilogue operands pair={pair}: max err {err:.3e}")
    assert err <= 1e-4 * math.sqrt(K / 64) * float(D.double().abs().max())


# ------------------------------------------------------------ split tail --
# When the last wave of tiles would leave CTAs idle, its tiles are split
# into up to 4 ranges of K whose fp32 partials a fixup kernel adds (in
# order) before the epilogue: one more launch.  Same bounds; the split
# result differs from the unsplit one only by summation order.

SPLIT_CASES = [
    # (batch, M, N, K, prec, pair, elem): tiles = 74 (pairs) or 148 + a short tail
    (1, 1790, 3068, 4096, "3xtf32", "1", 0),     # 7 x 12 = 84 pair tiles: 10 split 4 ways, ragged edges
    (1, 1792, 3072, 4096, "tf32", "0", 0),       # 14 x 12 = 168 single-CTA tiles: 20 split 4 ways
    (3, 512, 1536, 8192, "tf32", "1", 0),        # 3 x 2 x 6 = 36 batched pair tiles, all split 2 ways
    (1, 1792, 3072, 8192, "bf16", "1", 1),       # bf16 operands
]


@pytest.mark.parametrize("batch,M,N,K,prec,pair,elem", SPLIT_CASES)
def test_split_tail_tiles(cuda, monkeypatch, batch, M, N, K, prec, pair, elem):
    torch = cuda
    gen = torch.Generator(device="cuda").manual_seed(M + N + K)
    dt = torch.bfloat16 if elem else torch.float32
    shape_a, shape_b, shape_o = ((batch,) if batch > 1 else ()) + (M, K), ((batch,) if batch > 1 else ()) + (K, N), \
        ((batch,) if batch > 1 else ()) + (M, N)
    A = torch.randn(*shape_a, device="cuda", generator=gen).to(dt)
    B = torch.randn(*shape_b, device="cuda", generator=gen).to(dt)
    C = torch.randn(*shape_o, device="cuda", generator=gen)
    D = torch.randn(*shape_o, device="cuda", generator=gen)
    g = bafe.GraphBuilder()
    a = g.add_input("A", shape_a, 5 if elem else 0, 0)
    b = g.add_input("B", shape_b, 5 if elem else 0, 0)
    c = g.add_input("C", shape_o, 0, 0)
    d = g.add_input("D", shape_o, 0, 0)
    g.set_output(g.add("relu", [g.add("add", [g.add("matmul", [a, b]), g.add("mul", [c, d])])]))
    bafe.set_option("gemm_precision", "auto" if elem else prec)
    bafe.set_option("tc_pair", pair)
    ins = [A.view(torch.int16), B.view(torch.int16), C, D] if elem else [A, B, C, D]
    outs, launches = {}, {}
    try:
        for split in ("1", "0"):
            monkeypatch.setenv("BAFE_TC_SPLIT", split)
            k = bafe.compile_graph(g)
            assert "gemm.tc" in k.describe()
            # bf16 operands give a bf16 result (its bits in int16)
            out = torch.zeros(shape_o, dtype=torch.int16, device="cuda") if elem else \
                torch.full(shape_o, float("nan"), device="cuda")
            n0 = bafe.launch_count()
            k.run_torch(ins, out)
            bafe.synchronize()
            launches[split] = bafe.launch_count() - n0
            # a new output each time: the launch is prepared anew
            outs[split] = ((out.to(torch.int32) & 0xFFFF) << 16).view(torch.float32) if elem else out
    finally:
        bafe.set_option("tc_pair", "1")
        bafe.set_option("gemm_precision", "auto")
    assert launches["1"] == launches["0"] + 1, launches        # the fixup kernel ran
    ref = torch.relu(torch.matmul(A.double(), B.double()) + C.double() * D.double())
    tol = (1e-4 if prec == "3xtf32" else TF32_TOL) * math.sqrt(K / 64)
    if elem:                                  # one bf16 ulp of the value + the f32 summation error
        tol = torch.exp2(torch.floor(torch.log2(ref.abs().clamp_min(1e-30))) - 7) + 1e-4 * math.sqrt(K / 64)
    for split, out in outs.items():
        err = (out.double() - ref).abs()
        print(f"split={split} {prec} pair={pair} {batch}x{M}x{N}x{K}: max err {float(err.max()):.3e}")
        assert bool((err <= tol).all())
    assert bool(((outs["1"].double() - outs["0"].double()).abs() <= 2 * tol).all())


def test_wave_alignment_changes_no_bit(cuda, monkeypatch):
    """The pair kernel's producers align their waves (for two or more whole
    waves of tiles with K >= 128 k-blocks); it reorders no sum, so the
    result is bit for bit the unaligned one."""
    torch = cuda
    M, N, K = 4096, 2560, 4096               # 16 x 10 = 160 pair tiles: 148 whole, 12 split
    gen = torch.Generator(device="cuda").manual_seed(41)
    A = torch.randn(M, K, device="cuda", generator=gen)
    B = torch.randn(K, N, device="cuda", generator=gen)
    C = torch.randn(M, N, device="cuda", generator=gen)
    bafe.set_option("gemm_precision", "3xtf32")
    k = bafe.compile_graph(_graph(M, N, K, 0, 0, "relu_add_c"))
    outs = {}
    for on in ("1", "0"):
        monkeypatch.setenv("BAFE_TC_WAVE_SYNC", on)
        out = torch.full((M, N), float("nan"), device="cuda")   # a new output: prepared anew
        k.run_torch([A, B, C], out)
        bafe.synchronize()
        outs[on] = out
    assert torch.equal(outs["1"], outs["0"])
    ref = torch.relu(A.double() @ B.double() + C.double())
    assert float((outs["1"].double() - ref).abs().max()) <= 1e-4 * math.sqrt(K / 64)
