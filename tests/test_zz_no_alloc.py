"""The GEMM entry point that allocates no device memory.

bafe_cuda_gemm_3xtf32_static_scratch serves callers that cannot call
cudaMalloc (strict memory budgets or custom allocators that forbid hidden
device allocations, code that must avoid cudaMalloc's implicit device-wide
synchronisation): its scratch --
the tf32 residuals of A and B -- lives in a fixed 64 MiB array inside the
library instead of device buffers allocated on first use.  These tests call
it through the C ABI and compare it with the planned entry point
(bafe_cuda_jit_get_or_compile + bafe_cuda_run_device on a 3xTF32 plan),
within the 3xTF32 bound the other tests use, on two calls in a row (the
second with new operands, so stale scratch contents would show).

This file is collected last so that a run stopping at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""
import ctypes
import math

import pytest

import bafe_b200 as bafe
from bafe_b200 import _binding

pytestmark = pytest.mark.gpu


def _planned(torch, A, B, a_col, b_col):
    M, K = A.shape
    N = B.shape[1]
    g = bafe.GraphBuilder()
    a = g.add_input("A", (M, K), 0, 1 if a_col else 0)
    b = g.add_input("B", (K, N), 0, 1 if b_col else 0)
    g.set_output(g.add("matmul", [a, b]))
    bafe.set_option("gemm_precision", "3xtf32")
    k = bafe.compile_graph(g)
    assert "gemm.tc.3xtf32" in k.describe()
    out = torch.empty(M, N, device="cuda")
    k.run_torch([A.t().contiguous() if a_col else A, B.t().contiguous() if b_col else B], out)
    bafe.synchronize()
    return out


def _static(torch, A, B, a_col, b_col):
    """One call; returns (output, device bytes free before the call minus
    after it), the operands and the output allocated before measuring."""
    M, K = A.shape
    N = B.shape[1]
    a_store = A.t().contiguous() if a_col else A
    b_store = B.t().contiguous() if b_col else B
    out = torch.full((M, N), float("nan"), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    rc = _binding.lib.bafe_cuda_gemm_3xtf32_static_scratch(
        ctypes.c_void_p(a_store.data_ptr()), ctypes.c_void_p(b_store.data_ptr()), ctypes.c_void_p(out.data_ptr()),
        M, N, K, a_col, b_col, ctypes.c_void_p(stream))
    assert rc == 0, _binding.last_error()
    torch.cuda.synchronize()
    return out, free0 - torch.cuda.mem_get_info()[0]


@pytest.mark.parametrize("shape,a_col,b_col", [((1024, 768, 512), 0, 0), ((640, 520, 1000), 1, 1)])
def test_static_scratch_matches_planned_entry_two_calls(cuda, shape, a_col, b_col):
    torch = cuda
    M, N, K = shape
    bound = 1e-4 * math.sqrt(K / 64)
    gen = torch.Generator(device="cuda").manual_seed(17)
    for call in range(2):
        A = torch.randn(M, K, device="cuda", generator=gen)
        B = torch.randn(K, N, device="cuda", generator=gen)
        want = _planned(torch, A, B, a_col, b_col)
        got, taken = _static(torch, A, B, a_col, b_col)
        if call > 0:
            # the device's free memory is the same after the call as before
            # it: no allocation on the caller's behalf (the first call of the
            # process may load the library's kernels)
            assert taken == 0, f"call {call}: {taken} bytes of device memory taken"
        err = float((got - want).abs().max())
        assert err <= bound, f"call {call}: max |static - planned| = {err}"
        ref = A.double() @ B.double()
        assert float((got.double() - ref).abs().max()) <= bound


def test_static_scratch_rejects_problems_larger_than_the_array(cuda):
    torch = cuda
    A = torch.empty(4096, 4096, device="cuda")
    B = torch.empty(4096, 4096, device="cuda")
    out = torch.empty(4096, 4096, device="cuda")
    rc = _binding.lib.bafe_cuda_gemm_3xtf32_static_scratch(
        ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(B.data_ptr()), ctypes.c_void_p(out.data_ptr()),
        4096, 4096, 4096, 0, 0, None)
    assert rc != 0
    assert "static scratch" in _binding.last_error()[1]
