// gemm_tc.cuh -- tensor-core (tcgen05) GEMM with a generated epilogue.
#pragma once
#include "bafe_dev.cuh"

#define BAFE_TC_THREADS 256

namespace bafe {

struct TcArgs {
    const void* a;
    const void* b;
    void* out;
    i64 M, N, K;
    i64 o_bstride;
    const void* ep[8];
};

template <class Spec, int VARIANT>
__device__ __forceinline__ void gemm_tc(const TcArgs& g) {}

}  // namespace bafe
