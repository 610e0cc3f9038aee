"""bf16 GEMMs on the tensor cores (kind::f16), against the exact kernel.

(The exact kernel and the tensor-core plan are also pinned to the
reference's own bf16 outputs: tests/golden/bf16_*.npz, checked in
test_gpu_parity.py bit for bit and within the bound below.)

The reference converts bf16 operands to f32 exactly, multiplies in f32
(exact for bf16 x bf16) and sums in f32 in 32-wide chunks, then rounds the
epilogue result to bf16 (codegen.c:85-127, 191-293).  The tensor-core path
has the same products and a different f32 summation order, so after the
rounding to bf16 it differs from the reference -- the exact kernel, which
is bit-identical to it -- where the two f32 sums straddle a bf16 rounding
boundary.  Bound (N(0,1) inputs): |tc - exact| <= 1 bf16 ulp of the value
+ 1e-4 * sqrt(K/64) (the f32 summation error of either order; it dominates
only under cancellation, where the value is far below the terms), the
same against an fp64 evaluation, and >= 99.9 % of outputs bit-identical
(measured: 99.99 %)."""
import numpy as np
import pytest

import bafe_b200 as bafe

pytestmark = pytest.mark.gpu

BF16 = 5


def _bits_to_f32(t):
    return (t.to(dtype=__import__("torch").int32) & 0xFFFF).bitwise_left_shift(16).view(__import__("torch").float32)


def _graph(shape_a, shape_b, a_col, b_col, epi):
    g = bafe.GraphBuilder()
    a = g.add_input("A", shape_a, BF16, 1 if a_col else 0)
    b = g.add_input("B", shape_b, BF16, 1 if b_col else 0)
    mm = g.add("matmul", [a, b])
    if epi == "relu_add_c":
        out_shape = tuple(shape_a[:-1]) + (shape_b[-1],)
        c = g.add_input("C", out_shape, BF16, 0)
        mm = g.add("relu", [g.add("add", [mm, c])])
    g.set_output(mm)
    return g


@pytest.mark.parametrize("shape,a_col,b_col,epi", [
    ((512, 384, 256), 0, 0, "none"),
    ((512, 384, 256), 1, 1, "relu_add_c"),
    ((304, 264, 520), 0, 1, "relu_add_c"),
    ((304, 264, 520), 1, 0, "none"),
    ((304, 260, 520), 0, 1, "relu_add_c"),      # 520-byte rows: plain stores, no TMA
    ((1024, 2048, 1024), 0, 0, "relu_add_c"),
    ((3, 256, 512, 128), 0, 0, "relu_add_c"),
    ((512, 512, 16384), 0, 0, "relu_add_c"),     # several TMEM promotion chunks
])
@pytest.mark.parametrize("pair", ["1", "0"])
def test_bf16_tensor_core_gemm_within_one_ulp(cuda, shape, a_col, b_col, epi, pair):
    torch = cuda
    batch = shape[:-3]
    M, N, K = shape[-3:]
    gen = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.randn(*batch, M, K, device="cuda", generator=gen).to(torch.bfloat16)
    B = torch.randn(*batch, K, N, device="cuda", generator=gen).to(torch.bfloat16)
    ins = [A.transpose(-1, -2).contiguous() if a_col else A, B.transpose(-1, -2).contiguous() if b_col else B]
    C = None
    if epi == "relu_add_c":
        C = torch.randn(*batch, M, N, device="cuda", generator=gen).to(torch.bfloat16)
        ins.append(C)
    g = _graph(tuple(A.shape), tuple(B.shape), a_col, b_col, epi)
    outs = {}
    bafe.set_option("tc_pair", pair)
    try:
        for prec in ("auto", "exact"):
            bafe.set_option("gemm_precision", prec)
            k = bafe.compile_graph(g)
            assert ("gemm.tc.bf16" in k.describe()) == (prec == "auto"), k.describe()
            out = torch.zeros(*batch, M, N, dtype=torch.int16, device="cuda")
            k.run_torch([t.view(torch.int16) for t in ins], out)
            bafe.synchronize()
            outs[prec] = out
    finally:
        bafe.set_option("tc_pair", "1")
        bafe.set_option("gemm_precision", "auto")
    tc, ex = _bits_to_f32(outs["auto"]), _bits_to_f32(outs["exact"])
    # one bf16 ulp at the larger magnitude (8 significant bits)
    ulp = torch.maximum(tc.abs(), ex.abs()).clamp_min(1e-30)
    ulp = torch.exp2(torch.floor(torch.log2(ulp)) - 7)
    acc_err = 1e-4 * (K / 64) ** 0.5
    assert bool(((tc - ex).abs() <= ulp + acc_err).all())
    same = float((outs["auto"] == outs["exact"]).float().mean())
    ref = torch.matmul(A.double(), B.double())
    if C is not None:
        ref = torch.relu(ref + C.double())
    excess = float(((tc.double() - ref).abs() - ulp.double() - acc_err).max())
    print(f"bf16 {shape} pair={pair}: {100 * same:.3f} % bit-identical to the exact kernel")
    assert same > 0.999
    assert excess <= 0.0
