"""Failure detection on the device, without a GPU fault.

Every pipeline wait of the tensor-core GEMMs is bounded: when it runs out
the kernel raises its abort flag, writes a role code into a device error
word and returns, and the host turns the code into an error (13).  The
self-test entry point runs that same wait on an mbarrier nothing arrives
at -- no copies or MMAs in flight -- and these tests check that the code
arrives within the deadline and that the context keeps working."""
import ctypes

import numpy as np
import pytest

import bafe_b200 as bafe
from bafe_b200._binding import last_error, lib


def _selftest(us):
    code = ctypes.c_uint(0)
    ms = ctypes.c_double(0.0)
    rc = lib.bafe_cuda_selftest_wait_timeout(us, ctypes.byref(code), ctypes.byref(ms))
    return rc, code.value, ms.value


def test_selftest_rejects_bad_deadlines_on_the_host():
    for us in (0, -5, 10**8):
        rc, code, _ = _selftest(us)
        assert rc == 8 and code == 0
        assert "timeout_us" in last_error()[1]


@pytest.mark.gpu
@pytest.mark.parametrize("us", [1000, 20000])
def test_bounded_wait_runs_out_and_reports(cuda, us):
    rc, code, ms = _selftest(us)
    assert rc == 0, last_error()
    assert code == 0x5E1F7E57
    assert us / 1000.0 <= ms < us / 1000.0 + 2000.0      # waited its deadline, then returned


@pytest.mark.gpu
def test_context_keeps_working_after_a_timeout(cuda):
    torch = cuda
    assert _selftest(5000)[0] == 0
    g = bafe.GraphBuilder()
    a = g.add_input("A", (512, 256), 0, 0)
    b = g.add_input("B", (256, 384), 0, 0)
    g.set_output(g.add("relu", [g.add("matmul", [a, b])]))
    bafe.set_option("gemm_precision", "3xtf32")
    k = bafe.compile_graph(g)
    assert "gemm.tc.3xtf32" in k.describe()
    A = torch.randn(512, 256, device="cuda")
    B = torch.randn(256, 384, device="cuda")
    out = torch.empty(512, 384, device="cuda")
    k.run_torch([A, B], out)
    bafe.synchronize()                              # no stale error word either
    ref = torch.relu(A.double() @ B.double())
    assert float((out.double() - ref).abs().max()) <= 1e-4 * np.sqrt(256 / 64)
