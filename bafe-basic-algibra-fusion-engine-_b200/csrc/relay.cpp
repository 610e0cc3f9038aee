// relay.cpp -- copy-engine relay of an operand down a chain of ranks.
//
// A row-panel-sharded GEMM needs all of B on every rank.  When B changes
// from call to call it crosses NVLink inside the call, and an SM-based
// collective cannot run beside the persistent GEMM (which holds one CTA on
// every SM until it ends).  The relay moves B without SMs: rank r's copy
// engine pushes chunk c of its B into rank r+1's B (a cudaMemcpyAsync into
// the successor's buffer, mapped through CUDA IPC), then raises the
// successor's flag c to the step number with a fenced stream write
// (cuStreamWriteValue32).  Rank r+1 forwards chunk c once its own flag c
// reaches the step (cuStreamWaitValue32 on its copy stream), and its GEMM
// slices wait on the same flags.  Both waits are executed by the GPU's
// front end: no kernel spins, no SM is held.
//
// Flags count steps, so they never need resetting: step s waits for >= s.
// A sender overwrites its successor's B for step s+1 only after the
// successor acknowledged step s (the successor writes the ack word in the
// sender's flag block once its GEMM and its own forwarding of step s are
// done); the caller enqueues that wait with bafe_cuda_signal_wait.
#include "internal.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <string>

#define BAFE_API extern "C" __attribute__((visibility("default")))

namespace bafe_cuda {
namespace {

struct MemOps {
    bool ok = false;
    std::string why;
    decltype(&cuStreamWaitValue32) wait32 = nullptr;
    decltype(&cuStreamWriteValue32) write32 = nullptr;
};

MemOps& memops() {
    static MemOps m;
    static bool init = false;
    if (init) return m;
    init = true;
    auto get = [&](const char* name, void** fn) {
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint(name, fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !*fn) {
            cudaGetLastError();
            m.why = std::string("driver entry point missing: ") + name;
            return false;
        }
        return true;
    };
    if (!get("cuStreamWaitValue32", (void**)&m.wait32)) return m;
    if (!get("cuStreamWriteValue32", (void**)&m.write32)) return m;
    m.ok = true;
    return m;
}

int fail(const char* what, cudaError_t e) {
    set_error(11, std::string(what) + ": " + cudaGetErrorString(e));
    cudaGetLastError();
    return 11;
}

int fail_cu(const char* what, CUresult r) {
    set_error(11, std::string(what) + ": CUresult " + std::to_string((int)r));
    return 11;
}

}  // namespace
}  // namespace bafe_cuda

using namespace bafe_cuda;

static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handles are 64 bytes");

BAFE_API int bafe_cuda_relay_alloc(int device, int64_t bytes, uint64_t* dptr, void* ipc_handle) {
    if (bytes <= 0 || !dptr) { set_error(11, "relay_alloc: bad size or pointer"); return 11; }
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return fail("relay_alloc: cudaSetDevice", e);
    void* p = nullptr;
    if ((e = cudaMalloc(&p, (size_t)bytes)) != cudaSuccess) return fail("relay_alloc: cudaMalloc", e);
    if ((e = cudaMemset(p, 0, (size_t)bytes)) != cudaSuccess) { cudaFree(p); return fail("relay_alloc: cudaMemset", e); }
    if (ipc_handle) {
        cudaIpcMemHandle_t h;
        if ((e = cudaIpcGetMemHandle(&h, p)) != cudaSuccess) { cudaFree(p); return fail("relay_alloc: cudaIpcGetMemHandle", e); }
        memcpy(ipc_handle, &h, sizeof(h));
    }
    *dptr = (uint64_t)(uintptr_t)p;
    return 0;
}

BAFE_API int bafe_cuda_relay_free(uint64_t dptr) {
    cudaError_t e = cudaFree((void*)(uintptr_t)dptr);
    return e == cudaSuccess ? 0 : fail("relay_free: cudaFree", e);
}

BAFE_API int bafe_cuda_relay_open(int device, const void* ipc_handle, uint64_t* dptr) {
    if (!ipc_handle || !dptr) { set_error(11, "relay_open: null argument"); return 11; }
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return fail("relay_open: cudaSetDevice", e);
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    void* p = nullptr;
    if ((e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess)
        return fail("relay_open: cudaIpcOpenMemHandle", e);
    *dptr = (uint64_t)(uintptr_t)p;
    return 0;
}

BAFE_API int bafe_cuda_relay_close(uint64_t dptr) {
    cudaError_t e = cudaIpcCloseMemHandle((void*)(uintptr_t)dptr);
    return e == cudaSuccess ? 0 : fail("relay_close: cudaIpcCloseMemHandle", e);
}

BAFE_API int bafe_cuda_signal_wait(uint64_t addr, uint32_t value, void* stream) {
    MemOps& m = memops();
    if (!m.ok) { set_error(11, m.why); return 11; }
    CUresult r = m.wait32((CUstream)stream, (CUdeviceptr)addr, value, CU_STREAM_WAIT_VALUE_GEQ);
    return r == CUDA_SUCCESS ? 0 : fail_cu("cuStreamWaitValue32", r);
}

BAFE_API int bafe_cuda_signal_write(uint64_t addr, uint32_t value, void* stream) {
    MemOps& m = memops();
    if (!m.ok) { set_error(11, m.why); return 11; }
    CUresult r = m.write32((CUstream)stream, (CUdeviceptr)addr, value, CU_STREAM_WRITE_VALUE_DEFAULT);
    return r == CUDA_SUCCESS ? 0 : fail_cu("cuStreamWriteValue32", r);
}

BAFE_API int bafe_cuda_relay_step(uint64_t buf, uint64_t flags, uint64_t next_buf, uint64_t next_flags,
                                  const int64_t* bounds, int n_chunks, uint32_t step, int have, void* stream) {
    if (!bounds || n_chunks <= 0 || bounds[0] < 0) { set_error(11, "relay_step: bad chunk bounds"); return 11; }
    for (int c = 0; c < n_chunks; ++c)
        if (bounds[c + 1] <= bounds[c]) { set_error(11, "relay_step: chunk bounds must increase"); return 11; }
    if (!have && !flags) { set_error(11, "relay_step: a receiving rank needs its flag block"); return 11; }
    if (next_buf && !next_flags) { set_error(11, "relay_step: a forwarding rank needs its successor's flags"); return 11; }
    for (int c = 0; c < n_chunks; ++c) {
        if (!have) {
            int rc = bafe_cuda_signal_wait(flags + 4ull * (uint64_t)c, step, stream);
            if (rc) return rc;
        }
        if (!next_buf) continue;
        const uint64_t off = (uint64_t)bounds[c], n = (uint64_t)(bounds[c + 1] - bounds[c]);
        cudaError_t e = cudaMemcpyAsync((void*)(uintptr_t)(next_buf + off), (const void*)(uintptr_t)(buf + off),
                                        (size_t)n, cudaMemcpyDeviceToDevice, (cudaStream_t)stream);
        if (e != cudaSuccess) return fail("relay_step: cudaMemcpyAsync", e);
        int rc = bafe_cuda_signal_write(next_flags + 4ull * (uint64_t)c, step, stream);
        if (rc) return rc;
    }
    return 0;
}
