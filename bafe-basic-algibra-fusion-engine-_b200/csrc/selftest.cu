// selftest.cu -- exercises the bounded mbarrier wait that every pipeline
// role of the tensor-core GEMMs uses, on a barrier nothing arrives at.
//
// The GEMM kernels never spin without a deadline: a wait that runs out
// raises the CTA's abort flag and writes a role code into a device error
// word, every role leaves its loop, and the host reports the code after the
// launch (error 13).  Making a real GEMM time out would leave TMA copies
// and MMAs in flight; this kernel times out with no asynchronous work
// issued at all, so it can run on a shared GPU, and the caller can check
// that the code arrives and that the context still runs work afterwards.
#include "bafe_cuda.h"
#include "internal.h"

#include "bafe_dev.cuh"
#include "gemm_tc.cuh"

#include <cuda_runtime.h>

#include <chrono>
#include <string>

namespace {

__global__ void __launch_bounds__(32) bafe_selftest_wait_kernel(unsigned* err, unsigned long long timeout_ns,
                                                                 unsigned code) {
    using namespace bafe::tc;
    __shared__ __align__(8) unsigned long long bar;
    __shared__ bafe::tc::Shared sh;
    const u32 b = smem_u32(&bar);
    if (threadIdx.x == 0) {
        mbar_init(b, 1);          // one arrival expected, none will come
        sh.abort = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    bafe::TcArgs g;
    g.err = err;
    g.timeout_ns = timeout_ns;
    wait(b, 0u, &sh, g, code);    // runs out, sets sh.abort and *err
}

int fail(int code, const std::string& msg) {
    bafe_cuda::set_error(code, msg);
    return code;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int bafe_cuda_selftest_wait_timeout(int timeout_us, unsigned* code_out,
                                                                                       double* elapsed_ms) {
    if (code_out) *code_out = 0;
    if (timeout_us < 1 || timeout_us > 10000000) return fail(8, "timeout_us must be in [1, 10^7]");
    unsigned* word = nullptr;
    if (cudaMalloc(&word, sizeof(unsigned)) != cudaSuccess) {
        cudaGetLastError();
        return fail(6, "cudaMalloc(4) failed");
    }
    int rc = 0;
    const unsigned kCode = 0x5e1f7e57u;
    const auto t0 = std::chrono::steady_clock::now();
    if (cudaMemset(word, 0, sizeof(unsigned)) != cudaSuccess) rc = fail(7, "cudaMemset failed");
    if (!rc) {
        bafe_selftest_wait_kernel<<<1, 32>>>(word, (unsigned long long)timeout_us * 1000ull, kCode);
        cudaError_t e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) rc = fail(9, std::string("self-test kernel: ") + cudaGetErrorString(e));
    }
    unsigned got = 0;
    if (!rc && cudaMemcpy(&got, word, sizeof(unsigned), cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = fail(9, "reading the error word failed");
    const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    cudaFree(word);
    cudaGetLastError();
    if (rc) return rc;
    if (code_out) *code_out = got;
    if (elapsed_ms) *elapsed_ms = ms;
    return got == kCode ? 0 : fail(13, "the bounded wait did not report its timeout code");
}
