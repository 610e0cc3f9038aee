// static_scratch.cu -- 3xTF32 tensor-core GEMM (out = A . B) whose scratch
// memory is a fixed array inside this library, so the call allocates
// nothing.
//
// Who needs this: callers that cannot call cudaMalloc -- code under a
// strict memory budget or a custom allocator that forbids hidden device
// allocations, and code that must not hit the implicit device-wide
// synchronisation cudaMalloc/cudaFree can cause.  The regular plans keep
// their scratch (the tf32 residuals of A and B) in device buffers the
// library allocates on first use; this entry point puts it in g_scratch
// instead.  The call is synchronous: it waits for its stream and reads the
// status word back before returning.
//
// Limits and sharing:
//   * capacity kStaticScratchBytes (64 MiB): 256 bytes of status, then
//     M*K + K*N floats of residuals -- larger problems are rejected;
//   * the array lives on every GPU that loads the library until the process
//     exits;
//   * every call shares the one array and it keeps the last call's contents:
//     the status word is cleared at each call, the residuals are fully
//     rewritten; calls that overlap on the GPU (different streams, or
//     several host threads) race on it;
//   * the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current) and sets the
//     kernel's shared-memory limit; make that first call before any stream
//     capture.
#include "bafe_cuda.h"
#include "internal.h"
#include "tc_launch.h"

#include "bafe_dev.cuh"
#include "gemm_tc.cuh"

#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

namespace {

constexpr size_t kStaticScratchBytes = size_t(64) << 20;
constexpr size_t kStatusBytes = 256;

// The scratch.  In host code `g_scratch` names a host-side stand-in, not a
// device address: kernels are only ever given the address looked up with
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_scratch[kStaticScratchBytes];

// out = acc: the plain product, no epilogue.
struct PlainSpec {
    typedef float TA;
    typedef float TB;
    typedef float T;
    typedef float P;
    typedef float S;
    typedef float Out;
    template <class G>
    static __device__ __forceinline__ float apply(float acc, const G&, i64, i64, i64) { return acc; }
    template <class G>
    static __device__ __forceinline__ void apply4(const float* acc4, const G&, i64, i64, i64, bafe::Vec4<float>& o4) {
        for (int e = 0; e < 4; ++e) o4.v[e] = acc4[e];
    }
};

__global__ void __launch_bounds__(bafe::TcCfg<3>::THREADS, 1)
bafe_gemm_tc3_static_scratch(const __grid_constant__ bafe::TcArgs g) {
    bafe::gemm_tc<PlainSpec, 3>(g);
}

__global__ void __launch_bounds__(256) bafe_tf32_residual_static_scratch(const float* __restrict__ in,
                                                                         float* __restrict__ out, long long n) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = bafe::tf32_lo(in[i]);
}

struct DeviceSetup {
    bool done = false;
    unsigned char* scratch = nullptr;   // device address of g_scratch
    int sm_count = 0;
};
DeviceSetup g_setup[64];
std::mutex g_setup_mu;

int fail(int code, const std::string& msg) {
    bafe_cuda::set_error(code, msg);
    return code;
}

int setup_device(int dev, DeviceSetup*& out) {
    std::lock_guard<std::mutex> lk(g_setup_mu);
    if (dev < 0 || dev >= 64) return fail(4, "device ordinal out of range");
    DeviceSetup& s = g_setup[dev];
    if (!s.done) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            return fail(14, std::string("cudaGetSymbolAddress(static scratch): ") + cudaGetErrorString(e));
        }
        e = cudaFuncSetAttribute(bafe_gemm_tc3_static_scratch, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 bafe_cuda::tc_smem_bytes(3, false));
        if (e != cudaSuccess) {
            cudaGetLastError();
            return fail(14, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
        }
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        s.scratch = static_cast<unsigned char*>(p);
        s.sm_count = sms > 0 ? sms : 148;
        s.done = true;
    }
    out = &s;
    return 0;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int bafe_cuda_gemm_3xtf32_static_scratch(
    const float* A, const float* B, float* out, int64_t M, int64_t N, int64_t K, int a_col, int b_col,
    void* stream) {
    if (!A || !B || !out) return fail(8, "null operand");
    if (M < 1 || N < 1 || K < 1) return fail(8, "M, N and K must be >= 1");
    // Element counts are compared with the capacity before any product is
    // formed, so no size can wrap around (M, N, K are each >= 1 here).
    const int64_t cap_floats = (int64_t)((kStaticScratchBytes - kStatusBytes - 256) / 4);
    if (M > cap_floats / K || N > cap_floats / K || M * K + K * N > cap_floats)
        return fail(15, "problem needs more scratch than the static scratch holds: " +
                            std::to_string((unsigned long long)kStaticScratchBytes) +
                            " bytes (M*K + K*N <= " + std::to_string((long long)cap_floats) + " floats)");
    const int64_t a_ld = a_col ? M : K, b_ld = b_col ? K : N;
    if ((a_ld * 4) % 16 || (b_ld * 4) % 16 || N % 4)
        return fail(8, "tensor-core GEMM needs 16-byte row strides (A, B) and N % 4 == 0");
    const size_t a_bytes = (size_t)(M * K) * 4, b_bytes = (size_t)(K * N) * 4;
    const size_t a_off = kStatusBytes, b_off = a_off + ((a_bytes + 255) & ~size_t(255));
    if (b_off + b_bytes > kStaticScratchBytes) return fail(15, "static scratch too small for this problem");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return fail(4, "no CUDA device available");
    }
    DeviceSetup* ds = nullptr;
    if (int rc = setup_device(dev, ds)) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned* status = reinterpret_cast<unsigned*>(ds->scratch);
    float* a_lo = reinterpret_cast<float*>(ds->scratch + a_off);
    float* b_lo = reinterpret_cast<float*>(ds->scratch + b_off);
    // The status word must start at zero; the residuals are overwritten.
    if (cudaMemsetAsync(status, 0, sizeof(unsigned), st) != cudaSuccess) {
        cudaGetLastError();
        return fail(7, "cudaMemsetAsync(status)");
    }
    const int grid = ds->sm_count * 8;
    bafe_tf32_residual_static_scratch<<<grid, 256, 0, st>>>(A, a_lo, (long long)(M * K));
    bafe_tf32_residual_static_scratch<<<grid, 256, 0, st>>>(B, b_lo, (long long)(K * N));
    bafe_cuda::Step s;
    s.kind = bafe_cuda::StepKind::GemmTc;
    s.M = M;
    s.N = N;
    s.K = K;
    s.a_col = a_col ? 1 : 0;
    s.b_col = b_col ? 1 : 0;
    s.tc_variant = 3;
    s.tc_pair = false;
    bafe_cuda::TcLaunch L;
    std::string err;
    if (int rc = bafe_cuda::tc_prepare(s, A, B, a_lo, b_lo, out, {}, ds->sm_count, status, nullptr, 0, nullptr, L, err))
        return fail(rc, err);
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(L.grid, 1, 1);
    cfg.blockDim = dim3(L.block, 1, 1);
    cfg.dynamicSmemBytes = L.smem;
    cfg.stream = st;
    void* args[] = {L.args};
    cudaError_t e = cudaLaunchKernelExC(&cfg, (const void*)bafe_gemm_tc3_static_scratch, args);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(7, std::string("launch: ") + cudaGetErrorString(e));
    }
    bafe_cuda::g_launch_count += 3;
    // Synchronous like BAFE's kernels: the result is in `out` on return and a
    // pipeline wait that ran out of time is reported here.
    e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(9, std::string("device error: ") + cudaGetErrorString(e));
    }
    unsigned code = 0;
    if (cudaMemcpy(&code, status, sizeof(unsigned), cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        return fail(9, "reading the status word failed");
    }
    if (code) return fail(13, "tensor-core GEMM timed out on a pipeline barrier; the output is invalid");
    return 0;
}
