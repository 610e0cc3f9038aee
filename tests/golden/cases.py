"""Golden cases: the reference's own numeric tests and the workload configs,
with seeded inputs.  make_golden.py runs each through the reference
(optimizer + generated C kernel) and stores the optimized graph and the
output in <name>.npz; the tests rebuild that exact graph and feed it to the
backend.

Each case: name, cite (the reference test or config it restates), build
(GraphBuilder -> root, using the builder's input order = the arguments'),
inputs [(name, shape, dtype, fortran, layout, spec)], optional panel
(rows [r0, r1) of a large problem: the reference runs the same expression
on the row panel, whose per-row results equal the full problem's because
matmul's summation order does not depend on M).
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

GOLDEN_DIR = Path(__file__).resolve().parent

N01 = lambda seed, std=1.0: {"kind": "normal", "seed": seed, "std": std}
U11 = lambda seed: {"kind": "uniform", "seed": seed}
RINT = lambda seed: {"kind": "randint", "seed": seed, "lo": -100, "hi": 100}
SPECIAL = lambda seed: {"kind": "special", "seed": seed}


def _ew3(g, X, Y, Z):
    return g.add("relu", [g.add("add", [g.add("mul", [X, Y]), Z])])


CASES = [
    # ---- bafe/tests/test_e2e.py -------------------------------------------
    dict(name="e2e_matmul", cite="bafe/tests/test_e2e.py:14",
         build=lambda g, A, B: g.add("matmul", [A, B]),
         inputs=[("A", (16, 32), "float32", False, 0, N01(101)), ("B", (32, 24), "float32", False, 0, N01(102))]),
    dict(name="e2e_relu", cite="bafe/tests/test_e2e.py:26",
         build=lambda g, X: g.add("relu", [X]),
         inputs=[("X", (32, 32), "float32", False, 0, N01(103, 2.0))]),
    dict(name="e2e_add", cite="bafe/tests/test_e2e.py:37",
         build=lambda g, A, B: g.add("add", [A, B]),
         inputs=[("A", (16, 16), "float32", False, 0, N01(104)), ("B", (16, 16), "float32", False, 0, N01(105))]),
    dict(name="e2e_relu_matmul", cite="bafe/tests/test_e2e.py:49",
         build=lambda g, A, B: g.add("relu", [g.add("matmul", [A, B])]),
         inputs=[("A", (16, 32), "float32", False, 0, N01(106)), ("B", (32, 24), "float32", False, 0, N01(107))]),
    dict(name="e2e_relu_matmul_plus_c", cite="bafe/tests/test_e2e.py:61",
         build=lambda g, A, B, C: g.add("relu", [g.add("add", [g.add("matmul", [A, B]), C])]),
         inputs=[("A", (16, 32), "float32", False, 0, N01(108)), ("B", (32, 24), "float32", False, 0, N01(109)),
                 ("C", (16, 24), "float32", False, 0, N01(110))]),
    dict(name="e2e_relu_matmul_bias", cite="bafe/tests/test_e2e.py:75",
         build=lambda g, A, B, b: g.add("relu", [g.add("add", [g.add("matmul", [A, B]), b])]),
         inputs=[("A", (16, 32), "float32", False, 0, N01(111)), ("B", (32, 24), "float32", False, 0, N01(112)),
                 ("bias", (24,), "float32", False, 0, N01(113))]),
    dict(name="e2e_matmul_bias", cite="bafe/tests/test_e2e.py:92",
         build=lambda g, A, B, b: g.add("add", [g.add("matmul", [A, B]), b]),
         inputs=[("A", (16, 32), "float32", False, 0, N01(114)), ("B", (32, 24), "float32", False, 0, N01(115)),
                 ("bias", (24,), "float32", False, 0, N01(116))]),
    dict(name="e2e_relu_sigmoid_tanh", cite="bafe/tests/test_e2e.py:196",
         build=lambda g, X: g.add("tanh", [g.add("sigmoid", [g.add("relu", [X])])]),
         inputs=[("X", (32, 32), "float32", False, 0, N01(117, 2.0))]),
    dict(name="e2e_bias_add", cite="bafe/tests/test_e2e.py:207",
         build=lambda g, X, b: g.add("bias_add", [X, b]),
         inputs=[("X", (16, 32), "float32", False, 0, N01(118)), ("bias", (32,), "float32", False, 0, N01(119))]),
    # ---- bafe/tests/test_layout.py ----------------------------------------
    dict(name="layout_col_b", cite="bafe/tests/test_layout.py:214",
         build=lambda g, A, B: g.add("matmul", [A, B]),
         inputs=[("A", (16, 32), "float32", False, 0, N01(120)), ("B", (32, 24), "float32", True, 1, N01(121))]),
    dict(name="layout_both_col", cite="bafe/tests/test_layout.py:231",
         build=lambda g, A, B: g.add("matmul", [A, B]),
         inputs=[("A", (16, 32), "float32", True, 1, N01(122)), ("B", (32, 24), "float32", True, 1, N01(123))]),
    # ---- bafe/tests/test_dtypes.py ----------------------------------------
    dict(name="f16_matmul", cite="bafe/tests/test_dtypes.py:11",
         build=lambda g, A, B: g.add("matmul", [A, B]),
         inputs=[("A", (8, 8), "float16", False, 0, N01(124)), ("B", (8, 8), "float16", False, 0, N01(125))]),
    dict(name="f16_relu", cite="bafe/tests/test_dtypes.py:23",
         build=lambda g, X: g.add("relu", [X]),
         inputs=[("X", (16, 16), "float16", False, 0, N01(126, 2.0))]),
    dict(name="f16_matmul_relu", cite="bafe/tests/test_dtypes.py:34",
         build=lambda g, A, B: g.add("relu", [g.add("matmul", [A, B])]),
         inputs=[("A", (8, 8), "float16", False, 0, N01(127)), ("B", (8, 8), "float16", False, 0, N01(128))]),
    dict(name="f16_add", cite="bafe/tests/test_dtypes.py:46",
         build=lambda g, A, B: g.add("add", [A, B]),
         inputs=[("A", (16, 16), "float16", False, 0, N01(129)), ("B", (16, 16), "float16", False, 0, N01(130))]),
    dict(name="f16_matmul_bias_relu", cite="bafe/tests/test_dtypes.py:58",
         build=lambda g, A, B, b: g.add("relu", [g.add("add", [g.add("matmul", [A, B]), b])]),
         inputs=[("A", (8, 8), "float16", False, 0, N01(131)), ("B", (8, 8), "float16", False, 0, N01(132)),
                 ("bias", (8,), "float16", False, 0, N01(133))]),
    dict(name="f64_matmul", cite="bafe/tests/test_dtypes.py:77",
         build=lambda g, A, B: g.add("matmul", [A, B]),
         inputs=[("A", (8, 8), "float64", False, 0, N01(134)), ("B", (8, 8), "float64", False, 0, N01(135))]),
    dict(name="f64_relu", cite="bafe/tests/test_dtypes.py:89",
         build=lambda g, X: g.add("relu", [X]),
         inputs=[("X", (16, 16), "float64", False, 0, N01(136, 2.0))]),
    dict(name="f64_sigmoid", cite="bafe/tests/test_dtypes.py:100",
         build=lambda g, X: g.add("sigmoid", [X]),
         inputs=[("X", (8, 8), "float64", False, 0, N01(137))]),
    dict(name="batched_matmul_3d", cite="bafe/tests/test_dtypes.py:133",
         build=lambda g, A, B: g.add("matmul", [A, B]),
         inputs=[("A", (2, 4, 8), "float32", False, 0, N01(138)), ("B", (2, 8, 6), "float32", False, 0, N01(139))]),
    dict(name="batched_matmul_relu_3d", cite="bafe/tests/test_dtypes.py:146",
         build=lambda g, A, B: g.add("relu", [g.add("matmul", [A, B])]),
         inputs=[("A", (2, 4, 8), "float32", False, 0, N01(140)), ("B", (2, 8, 6), "float32", False, 0, N01(141))]),
    dict(name="dot_1x8_8x1", cite="bafe/tests/test_dtypes.py:158",
         build=lambda g, A, B: g.add("matmul", [A, B]),
         inputs=[("A", (1, 8), "float32", False, 0, N01(142)), ("B", (8, 1), "float32", False, 0, N01(143))]),
    dict(name="tall_matmul", cite="bafe/tests/test_dtypes.py:172",
         build=lambda g, A, B: g.add("matmul", [A, B]),
         inputs=[("A", (64, 4), "float32", False, 0, N01(144)), ("B", (4, 64), "float32", False, 0, N01(145))]),
    dict(name="wide_matmul", cite="bafe/tests/test_dtypes.py:185",
         build=lambda g, A, B: g.add("matmul", [A, B]),
         inputs=[("A", (4, 64), "float32", False, 0, N01(146)), ("B", (64, 4), "float32", False, 0, N01(147))]),
    dict(name="i32_add", cite="bafe/tests/test_dtypes.py:202",
         build=lambda g, A, B: g.add("add", [A, B]),
         inputs=[("A", (8, 8), "int32", False, 0, RINT(148)), ("B", (8, 8), "int32", False, 0, RINT(149))]),
    dict(name="i64_add", cite="bafe/tests/test_dtypes.py:213",
         build=lambda g, A, B: g.add("add", [A, B]),
         inputs=[("A", (8, 8), "int64", False, 0, RINT(150)), ("B", (8, 8), "int64", False, 0, RINT(151))]),
    # ---- BF16 through the C API: inputs are raw bf16 words, the kernel
    # widens them exactly and rounds its result back to nearest-even with the
    # emitter's bias trick (codegen.c:113-127, 157-169) ----------------------
    dict(name="bf16_matmul", cite="bafe/src/codegen.c:113-127,191-293 (bf16 in, bf16 out)",
         build=lambda g, A, B: g.add("matmul", [A, B]),
         inputs=[("A", (8, 8), "bfloat16", False, 0, N01(186)), ("B", (8, 8), "bfloat16", False, 0, N01(187))]),
    dict(name="bf16_relu", cite="bafe/src/codegen.c:113-127,338-344",
         build=lambda g, X: g.add("relu", [X]),
         inputs=[("X", (16, 16), "bfloat16", False, 0, N01(188, 2.0))]),
    dict(name="bf16_add", cite="bafe/src/codegen.c:113-127,294-326",
         build=lambda g, A, B: g.add("add", [A, B]),
         inputs=[("A", (16, 16), "bfloat16", False, 0, N01(189)), ("B", (16, 16), "bfloat16", False, 0, N01(190))]),
    dict(name="bf16_matmul_relu", cite="bafe/src/codegen.c:113-127,467-486 (fused at 8x8)",
         build=lambda g, A, B: g.add("relu", [g.add("matmul", [A, B])]),
         inputs=[("A", (8, 8), "bfloat16", False, 0, N01(191)), ("B", (8, 8), "bfloat16", False, 0, N01(192))]),
    dict(name="bf16_matmul_bias_relu", cite="bafe/src/codegen.c:113-127,502-517",
         build=lambda g, A, B, b: g.add("relu", [g.add("add", [g.add("matmul", [A, B]), b])]),
         inputs=[("A", (8, 8), "bfloat16", False, 0, N01(193)), ("B", (8, 8), "bfloat16", False, 0, N01(194)),
                 ("bias", (8,), "bfloat16", False, 0, N01(195))]),
    dict(name="bf16_special_values", cite="bafe/src/codegen.c:113-127,294-344 (NaN / -0 / inf through bf16)",
         build=_ew3,
         inputs=[("X", (4096,), "bfloat16", False, 0, SPECIAL(196)), ("Y", (4096,), "bfloat16", False, 0, SPECIAL(197)),
                 ("Z", (4096,), "bfloat16", False, 0, SPECIAL(198))]),
    dict(name="bf16_relu_matmul_plus_c_256", cite="bafe/src/codegen.c:113-127,191-293,294-344 (tensor-core size)",
         build=lambda g, A, B, C: g.add("relu", [g.add("add", [g.add("matmul", [A, B]), C])]),
         inputs=[("A", (256, 256), "bfloat16", False, 0, N01(199)), ("B", (256, 256), "bfloat16", False, 0, N01(200)),
                 ("C", (256, 256), "bfloat16", False, 0, N01(201))],
         store_inputs=False),
    dict(name="bf16_matmul_col_b_320x384x512", cite="bafe/src/codegen.c:113-127,206-213 (B Fortran order)",
         build=lambda g, A, B: g.add("matmul", [A, B]),
         inputs=[("A", (320, 512), "bfloat16", False, 0, N01(202)), ("B", (512, 384), "bfloat16", True, 1, N01(203))],
         store_inputs=False),
    # ---- bafe.fuse(f, g): the graph FusedFunction compiles (f and g optimized
    # apart, bafe_fuse_concat, optimized again; __init__.py:844-885,
    # fuse.c:12-125).  fuse = (f, g) names the jitted functions the tests
    # rebuild; na = f's argument count ---------------------------------------
    dict(name="fuse_two_matmuls", cite="bafe/tests/test_fuse.py:14", fuse=("matmul", "matmul"), na=2,
         build_a=lambda g, A, B: g.add("matmul", [A, B]),
         build_b=lambda g, X, C: g.add("matmul", [X, C]),
         inputs=[("A", (8, 16), "float32", False, 0, N01(204)), ("B", (16, 32), "float32", False, 0, N01(205)),
                 ("C", (32, 24), "float32", False, 0, N01(206))]),
    dict(name="fuse_matmul_then_relu", cite="bafe/tests/test_fuse.py:35", fuse=("matmul", "relu"), na=2,
         build_a=lambda g, A, B: g.add("matmul", [A, B]),
         build_b=lambda g, X: g.add("relu", [X]),
         inputs=[("A", (16, 32), "float32", False, 0, N01(207)), ("B", (32, 24), "float32", False, 0, N01(208))]),
    dict(name="fuse_matmul_then_add_bias", cite="bafe/tests/test_fuse.py:54", fuse=("matmul", "relu_add"), na=2,
         build_a=lambda g, A, B: g.add("matmul", [A, B]),
         build_b=lambda g, X, b: g.add("relu", [g.add("add", [X, b])]),
         inputs=[("A", (32, 32), "float32", False, 0, N01(209)), ("B", (32, 32), "float32", False, 0, N01(210)),
                 ("bias", (32,), "float32", False, 0, N01(211))]),
    dict(name="fuse_matmul_then_relu_64x64", cite="bafe/tests/test_fuse.py:113 (largest shape)", fuse=("matmul", "relu"),
         na=2, build_a=lambda g, A, B: g.add("matmul", [A, B]),
         build_b=lambda g, X: g.add("relu", [X]),
         inputs=[("A", (64, 64), "float32", False, 0, N01(212)), ("B", (64, 64), "float32", False, 0, N01(213))]),
    dict(name="fuse_gemm_then_relu_add_c_256", cite="bafe/tests/test_fuse.py:243 (fused == sequential), tensor-core size",
         fuse=("matmul", "relu_add"), na=2,
         build_a=lambda g, A, B: g.add("matmul", [A, B]),
         build_b=lambda g, X, C: g.add("relu", [g.add("add", [X, C])]),
         inputs=[("A", (256, 320), "float32", False, 0, N01(214)), ("B", (320, 256), "float32", False, 0, N01(215)),
                 ("C", (256, 256), "float32", False, 0, N01(216))],
         store_inputs=False),
    # ---- tensor-core layouts at sizes where auto picks the tensor cores --
    dict(name="col_a_relu_matmul_plus_c_320x384x512", cite="bafe/src/codegen.c:206-213 (A Fortran order), 240-290",
         build=lambda g, A, B, C: g.add("relu", [g.add("add", [g.add("matmul", [A, B]), C])]),
         inputs=[("A", (320, 512), "float32", True, 1, N01(217)), ("B", (512, 384), "float32", False, 0, N01(218)),
                 ("C", (320, 384), "float32", False, 0, N01(219))],
         store_inputs=False),
    dict(name="batched_matmul_4x256x320x256", cite="bafe/src/codegen.c:215-236 (batched rank-3 matmul)",
         build=lambda g, A, B: g.add("matmul", [A, B]),
         inputs=[("A", (4, 256, 320), "float32", False, 0, N01(220)), ("B", (4, 320, 256), "float32", False, 0, N01(221))],
         store_inputs=False),
    # ---- scripts/test_smoke.c (deterministic pattern) ----------------------
    dict(name="smoke_c_pattern", cite="scripts/test_smoke.c:11-24,54-56",
         build=lambda g, A, B, b: g.add("relu", [g.add("add", [g.add("matmul", [A, B]), b])]),
         inputs=[("A", (32, 32), "float32", False, 0, {"kind": "pattern", "mod": 7, "scale": 0.1}),
                 ("B", (32, 32), "float32", False, 0, {"kind": "pattern", "mod": 5, "scale": 0.1}),
                 ("bias", (32,), "float32", False, 0, {"kind": "pattern", "mod": 1 << 30, "scale": 0.01})]),
    # ---- fused forms the extractor picks at tiny sizes ----------------------
    dict(name="fused_matmul_relu_8", cite="bafe/src/rewrite.c:207-220, codegen.c:467-486",
         build=lambda g, A, B: g.add("relu", [g.add("matmul", [A, B])]),
         inputs=[("A", (8, 8), "float32", False, 0, N01(152)), ("B", (8, 8), "float32", False, 0, N01(153))]),
    dict(name="fused_matmul_bias_relu_8", cite="bafe/src/rewrite.c:258-278, codegen.c:502-517",
         build=lambda g, A, B, b: g.add("relu", [g.add("add", [g.add("matmul", [A, B]), b])]),
         inputs=[("A", (8, 8), "float32", False, 0, N01(154)), ("B", (8, 8), "float32", False, 0, N01(155)),
                 ("bias", (8,), "float32", False, 0, N01(156))]),
    # ---- transpose materialisation ------------------------------------------
    dict(name="transpose_64x48", cite="bafe/src/codegen.c:360-369",
         build=lambda g, X: g.add("transpose", [X], perm=[1, 0]),
         inputs=[("X", (64, 48), "float32", False, 0, N01(157))]),
    dict(name="transpose_then_relu", cite="bafe/src/codegen.c:360-369,338-344",
         build=lambda g, X: g.add("relu", [g.add("transpose", [X], perm=[1, 0])]),
         inputs=[("X", (40, 72), "float32", False, 0, N01(158))]),
    # ---- elementwise edge values (relu of NaN/-0, inf arithmetic) -----------
    dict(name="ew_special_values", cite="bafe/src/codegen.c:294-344",
         build=_ew3,
         inputs=[("X", (4096,), "float32", False, 0, SPECIAL(159)), ("Y", (4096,), "float32", False, 0, SPECIAL(160)),
                 ("Z", (4096,), "float32", False, 0, SPECIAL(161))]),
    # ---- zero-size dimensions (shapes may hold 0: types.c:70-73; the
    # emitted loops then run zero times over a zeroed node buffer) ----------
    dict(name="empty_k_matmul_plus_c", cite="bafe/src/types.c:70-73, codegen.c:241-247 (K=0: relu(0 + C))",
         build=lambda g, A, B, C: g.add("relu", [g.add("add", [g.add("matmul", [A, B]), C])]),
         inputs=[("A", (8, 0), "float32", False, 0, N01(162)), ("B", (0, 12), "float32", False, 0, N01(163)),
                 ("C", (8, 12), "float32", False, 0, N01(164))]),
    dict(name="empty_m_matmul", cite="bafe/src/types.c:70-73, codegen.c:241-247 (M=0)",
         build=lambda g, A, B: g.add("matmul", [A, B]),
         inputs=[("A", (0, 16), "float32", False, 0, N01(165)), ("B", (16, 12), "float32", False, 0, N01(166))]),
    dict(name="empty_batch_matmul", cite="bafe/src/types.c:70-73, codegen.c:231-235 (batch of 0)",
         build=lambda g, A, B: g.add("matmul", [A, B]),
         inputs=[("A", (0, 4, 8), "float32", False, 0, N01(167)), ("B", (0, 8, 4), "float32", False, 0, N01(168))]),
    dict(name="empty_ew_chain", cite="bafe/src/types.c:70-73, codegen.c:294-344 (n=0)",
         build=_ew3,
         inputs=[("X", (0,), "float32", False, 0, U11(169)), ("Y", (0,), "float32", False, 0, U11(170)),
                 ("Z", (0,), "float32", False, 0, U11(171))]),
    dict(name="empty_transpose", cite="bafe/src/types.c:70-73, codegen.c:360-369 (0x7 -> 7x0)",
         build=lambda g, X: g.add("transpose", [X], perm=[1, 0]),
         inputs=[("X", (0, 7), "float32", False, 0, N01(172))]),
    # ---- single-axis reductions, sequential per output (codegen.c:405-452) --
    dict(name="reduce_sum_axis0", cite="bafe/src/codegen.c:419-428",
         build=lambda g, X: g.add("reduce_sum", [X], axes=[0]),
         inputs=[("X", (37, 53), "float32", False, 0, N01(173))]),
    dict(name="reduce_sum_axis1", cite="bafe/src/codegen.c:429-434",
         build=lambda g, X: g.add("reduce_sum", [X], axes=[1]),
         inputs=[("X", (37, 53), "float32", False, 0, N01(174))]),
    dict(name="reduce_sum_axis_neg1", cite="bafe/src/codegen.c:418 (axis % 2 of -1 is -1: the row branch)",
         build=lambda g, X: g.add("reduce_sum", [X], axes=[-1]),
         inputs=[("X", (16, 40), "float32", False, 0, N01(175))]),
    dict(name="reduce_max_axis0", cite="bafe/src/codegen.c:424-427",
         build=lambda g, X: g.add("reduce_max", [X], axes=[0]),
         inputs=[("X", (37, 53), "float32", False, 0, N01(176))]),
    dict(name="reduce_max_axis1_keepdims", cite="bafe/src/codegen.c:435-438, types.c:113-136",
         build=lambda g, X: g.add("reduce_max", [X], axes=[1], keepdims=True),
         inputs=[("X", (37, 53), "float32", False, 0, N01(177))]),
    dict(name="reduce_sum_1d", cite="bafe/src/codegen.c:409-415",
         build=lambda g, X: g.add("reduce_sum", [X], axes=[0]),
         inputs=[("X", (1000,), "float32", False, 0, U11(178))]),
    dict(name="reduce_max_1d_special_values", cite="bafe/src/codegen.c:413-415 (NaN / -0 / inf: first wins ties)",
         build=lambda g, X: g.add("reduce_max", [X], axes=[0]),
         inputs=[("X", (4096,), "float32", False, 0, SPECIAL(179))]),
    dict(name="reduce_sum_rows_special_values", cite="bafe/src/codegen.c:429-434",
         build=lambda g, X: g.add("reduce_sum", [X], axes=[1]),
         inputs=[("X", (64, 64), "float32", False, 0, SPECIAL(180))]),
    dict(name="reduce_sum_i32", cite="bafe/src/codegen.c:419-423",
         build=lambda g, X: g.add("reduce_sum", [X], axes=[0]),
         inputs=[("X", (50, 30), "int32", False, 0, RINT(181))]),
    dict(name="reduce_max_f64", cite="bafe/src/codegen.c:435-438",
         build=lambda g, X: g.add("reduce_max", [X], axes=[1]),
         inputs=[("X", (20, 33), "float64", False, 0, N01(182))]),
    dict(name="reduce_sum_of_relu", cite="bafe/src/codegen.c:338-344,429-434",
         build=lambda g, X: g.add("reduce_sum", [g.add("relu", [X])], axes=[1]),
         inputs=[("X", (48, 70), "float32", False, 0, N01(183))]),
    dict(name="reduce_sum_two_axes_zero_fill", cite="bafe/src/codegen.c:442-451 (generic reduce: zero fill)",
         build=lambda g, X: g.add("reduce_sum", [X], axes=[0, 1]),
         inputs=[("X", (4, 6), "float32", False, 0, N01(184))]),
    dict(name="reduce_max_rank3_zero_fill", cite="bafe/src/codegen.c:442-451 (generic reduce: zero fill)",
         build=lambda g, X: g.add("reduce_max", [X], axes=[2]),
         inputs=[("X", (3, 4, 5), "float32", False, 0, N01(185))]),
    # ---- workload configs -----------------------------------------------------
    dict(name="cfg1_seed0", cite="benchmark configuration: relu(matmul(A,B)+C) 64x64x64",
         build=lambda g, A, B, C: g.add("relu", [g.add("add", [g.add("matmul", [A, B]), C])]),
         inputs=[("A", (64, 64), "float32", False, 0, N01(0)), ("B", (64, 64), "float32", False, 0, N01(1)),
                 ("C", (64, 64), "float32", False, 0, N01(2))]),
    dict(name="cfg2_row_col", cite="benchmark configuration: matmul 256^3, B Fortran order",
         build=lambda g, A, B: g.add("matmul", [A, B]),
         inputs=[("A", (256, 256), "float32", False, 0, N01(10)), ("B", (256, 256), "float32", True, 1, N01(11))],
         store_inputs=False),
    dict(name="cfg2_row_row", cite="benchmark configuration: matmul 256^3, B row-major",
         build=lambda g, A, B: g.add("matmul", [A, B]),
         inputs=[("A", (256, 256), "float32", False, 0, N01(10)), ("B", (256, 256), "float32", False, 0, N01(11))],
         store_inputs=False),
    dict(name="cfg3_panel_top", cite="benchmark configuration: relu(add(matmul(A,B), mul(C,D))) 4096^3, rows 0:8",
         build=lambda g, A, B, C, D: g.add("relu", [g.add("add", [g.add("matmul", [A, B]), g.add("mul", [C, D])])]),
         inputs=[("A", (4096, 4096), "float32", False, 0, N01(20)), ("B", (4096, 4096), "float32", False, 0, N01(21)),
                 ("C", (4096, 4096), "float32", False, 0, N01(22)), ("D", (4096, 4096), "float32", False, 0, N01(23))],
         panel=(0, 8), panel_inputs=("A", "C", "D"), store_inputs=False),
    dict(name="cfg3_panel_bottom", cite="benchmark configuration: relu(add(matmul(A,B), mul(C,D))) 4096^3, rows 4088:4096",
         build=lambda g, A, B, C, D: g.add("relu", [g.add("add", [g.add("matmul", [A, B]), g.add("mul", [C, D])])]),
         inputs=[("A", (4096, 4096), "float32", False, 0, N01(20)), ("B", (4096, 4096), "float32", False, 0, N01(21)),
                 ("C", (4096, 4096), "float32", False, 0, N01(22)), ("D", (4096, 4096), "float32", False, 0, N01(23))],
         panel=(4088, 4096), panel_inputs=("A", "C", "D"), store_inputs=False),
    dict(name="cfg4_chunk", cite="benchmark configuration: relu(add(mul(X,Y),Z)) U(-1,1), first 2^17 of each vector",
         build=_ew3,
         inputs=[("X", (1 << 17,), "float32", False, 0, U11(30)), ("Y", (1 << 17,), "float32", False, 0, U11(31)),
                 ("Z", (1 << 17,), "float32", False, 0, U11(32))],
         store_inputs=False),
    dict(name="cfg5_panel_top", cite="benchmark configuration: relu(matmul(A,B)+C) 16384^3, B BLOCKED, std 1/sqrt(K), rows 0:4",
         build=lambda g, A, B, C: g.add("relu", [g.add("add", [g.add("matmul", [A, B]), C])]),
         inputs=[("A", (16384, 16384), "float32", False, 0, N01(40, 0.0078125)),
                 ("B", (16384, 16384), "float32", False, 2, N01(41, 0.0078125)),
                 ("C", (16384, 16384), "float32", False, 0, N01(42, 0.0078125))],
         panel=(0, 4), panel_inputs=("A", "C"), store_inputs=False),
    dict(name="cfg5_panel_mid", cite="benchmark configuration: relu(matmul(A,B)+C) 16384^3, B TENSOR_CORE, rows 8190:8194",
         build=lambda g, A, B, C: g.add("relu", [g.add("add", [g.add("matmul", [A, B]), C])]),
         inputs=[("A", (16384, 16384), "float32", False, 0, N01(40, 0.0078125)),
                 ("B", (16384, 16384), "float32", False, 3, N01(41, 0.0078125)),
                 ("C", (16384, 16384), "float32", False, 0, N01(42, 0.0078125))],
         panel=(8190, 8194), panel_inputs=("A", "C"), store_inputs=False),
    dict(name="cfg5_panel_bottom", cite="benchmark configuration: relu(matmul(A,B)+C) 16384^3, B BLOCKED, rows 16380:16384",
         build=lambda g, A, B, C: g.add("relu", [g.add("add", [g.add("matmul", [A, B]), C])]),
         inputs=[("A", (16384, 16384), "float32", False, 0, N01(40, 0.0078125)),
                 ("B", (16384, 16384), "float32", False, 2, N01(41, 0.0078125)),
                 ("C", (16384, 16384), "float32", False, 0, N01(42, 0.0078125))],
         panel=(16380, 16384), panel_inputs=("A", "C"), store_inputs=False),
]

CASE_BY_NAME = {c["name"]: c for c in CASES}


_BIG_CACHE: dict = {}


def make_input(name_shape_spec, full: bool = True, rows: int | None = None) -> np.ndarray:
    """Materialise one input of a case from its spec (seeded).  rows: only
    the first `rows` rows of a row-major 2-D normal / uniform input (the
    seeded generator fills arrays in order, so they equal the full array's
    first rows).  The last two arrays of 256 MiB or more are kept, read-only,
    for the next request (the large configurations' shared operands)."""
    name, shape, dtype, fortran, layout, spec = name_shape_spec
    if (rows is not None and len(shape) == 2 and not fortran and dtype != "bfloat16"
            and spec["kind"] in ("normal", "uniform") and rows < shape[0]):
        from inputs import generate
        return generate(spec, (rows, shape[1]), dtype, fortran)
    if int(np.prod(shape)) * 4 < (256 << 20):
        return _make_input(name_shape_spec)
    key = (tuple(shape), dtype, fortran, json.dumps(spec, sort_keys=True))
    if key not in _BIG_CACHE:
        if len(_BIG_CACHE) >= 2:
            _BIG_CACHE.pop(next(iter(_BIG_CACHE)))
        a = _make_input(name_shape_spec)
        a.setflags(write=False)
        _BIG_CACHE[key] = a
    return _BIG_CACHE[key]


def _make_input(name_shape_spec) -> np.ndarray:
    from inputs import generate, special_values
    name, shape, dtype, fortran, layout, spec = name_shape_spec
    kind = spec["kind"]
    if kind == "pattern":
        n = int(np.prod(shape))
        a = ((np.arange(n) % spec["mod"]).astype(np.float32) * np.float32(spec["scale"])).reshape(shape)
        return a.astype(dtype)
    if dtype == "bfloat16":
        # drawn in fp32, then rounded to bf16 words (nearest-even)
        base = (name, shape, "float32", fortran, layout, spec)
        return f32_to_bf16_bits(make_input(base))
    if kind == "special":
        return special_values(int(np.prod(shape)), spec["seed"]).reshape(shape).astype(dtype)
    return generate(spec, shape, dtype, fortran)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 words, round to nearest-even by adding 0x7FFF plus the
    kept lsb (the emitter's own rounding, codegen.c:119-125); keeps the
    array's memory order."""
    bits = np.asarray(a, np.float32).view(np.uint32).astype(np.uint64)
    bits = (bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFFFFFF
    out = (bits >> 16).astype(np.uint16)
    return np.asfortranarray(out) if np.isfortran(a) else np.ascontiguousarray(out)


def bf16_bits_to_f64(a: np.ndarray) -> np.ndarray:
    """bf16 words -> their exact values (as float64)."""
    return (np.asarray(a, np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)


DTYPE_CODE = {"float32": 0, "float64": 1, "int32": 2, "int64": 3, "float16": 4, "bfloat16": 5}


def traced_graph(case: dict):
    """The case's graph as the front end traces it, at its declared (full)
    shapes and layout tags; for a fuse case, f's and g's traced graphs
    concatenated as bafe.fuse does (fuse.c:12-106: f's output feeds g's
    first input)."""
    from bafe_b200.graph import GraphBuilder
    specs = case["inputs"]
    if not case.get("fuse"):
        g = GraphBuilder()
        ids = [g.add_input(s[0], s[1], DTYPE_CODE[s[2]], s[4]) for s in specs]
        g.set_output(case["build"](g, *ids))
        return g
    na = case["na"]
    ga = GraphBuilder()
    ids_a = [ga.add_input(s[0], s[1], DTYPE_CODE[s[2]], s[4]) for s in specs[:na]]
    ra = case["build_a"](ga, *ids_a)
    ga.set_output(ra)
    gb = GraphBuilder()
    x = gb.add_input("X", ga.shape(ra), ga.dtype(ra), 0)
    ids_b = [gb.add_input(s[0], s[1], DTYPE_CODE[s[2]], s[4]) for s in specs[na:]]
    gb.set_output(case["build_b"](gb, x, *ids_b))
    return GraphBuilder.concat(ga, gb)


def load(name: str):
    """-> (meta dict, {input name: array or None}, golden output)."""
    z = np.load(GOLDEN_DIR / f"{name}.npz", allow_pickle=False)
    meta = json.loads(str(z["meta"]))
    ins = {k[3:]: z[k] for k in z.files if k.startswith("in_")}
    return meta, ins, z["out"]


def graph_from_nodes(nodes: list, input_ids: list, root: int):
    """Rebuild a BafeGraph struct from a node list (reference-optimized graph)."""
    import ctypes
    from bafe_b200._binding import BafeGraph
    from bafe_b200.graph import _OPNAME
    g = BafeGraph()
    ctypes.memset(ctypes.byref(g), 0, ctypes.sizeof(g))
    for i, n in enumerate(nodes):
        x = g.nodes[i]
        x.id = i
        x.op_name = _OPNAME[n["op"]]
        x.n_children = len(n["children"])
        for k, c in enumerate(n["children"]):
            x.children[k] = c
        x.shape.rank = len(n["shape"])
        for d, v in enumerate(n["shape"]):
            x.shape.dims[d] = v
        x.dtype = n["dtype"]
        x.layout = n["layout"]
        x.is_input = n["is_input"]
        if n["is_input"]:
            x.input_name = n["name"].encode()
        for f, key in (("perm", "perm"), ("axes", "axes"), ("shape", "tshape")):
            vals = n.get(key, [])
            setattr(x.attrs, "n_" + f, len(vals))
            for k, v in enumerate(vals):
                getattr(x.attrs, f)[k] = v
        x.attrs.keepdims = n.get("keepdims", False)
        x.attrs.name = n.get("attr_name", n["name"] if n["is_input"] else "").encode()
    g.n_nodes = len(nodes)
    for k, i in enumerate(input_ids):
        g.inputs[k] = i
    g.n_inputs = len(input_ids)
    g.outputs[0] = root
    g.n_outputs = 1
    return g
