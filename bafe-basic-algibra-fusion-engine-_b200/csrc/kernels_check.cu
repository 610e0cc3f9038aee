// kernels_check.cu -- nvcc sm_100a compile check of the device templates
// that NVRTC instantiates at run time (built by `make check`, never loaded).
// It instantiates each template once with a representative generated spec
// so that `-Xptxas -v` reports registers / spills / shared memory.
#include "bafe_dev.cuh"
#include "layout.cuh"
#include "gemm_exact.cuh"
#include "gemm_tc.cuh"

// relu(matmul(A,B) + C), all f32, as the lowering emits it.
struct CheckSpec {
    typedef float TA; typedef float TB; typedef float T; typedef float P; typedef float S;
    typedef float Out;
    static __device__ __forceinline__ TA loadA(const void* p, i64 i) { return reinterpret_cast<const float*>(p)[i]; }
    static __device__ __forceinline__ TB loadB(const void* p, i64 i) { return reinterpret_cast<const float*>(p)[i]; }
    template <class G> static __device__ __forceinline__ Out apply(T acc, const G& g, i64 b, i64 i, i64 j) {
        const i64 flat = b * g.o_bstride + i * g.N + j;
        const float x0 = reinterpret_cast<const float*>(g.ep[0])[flat];
        return bafe::relu(bafe::add(acc, x0));
    }
    template <class G> static __device__ __forceinline__ void apply4(const T* acc4, const G& g, i64 b, i64 i, i64 j, bafe::Vec4<Out>& o4) {
        const i64 flat = b * g.o_bstride + i * g.N + j;
        const bafe::Vec4<float> v0 = bafe::ld4(reinterpret_cast<const float*>(g.ep[0]) + flat);
#pragma unroll
        for (int e = 0; e < 4; ++e) o4.v[e] = bafe::relu(bafe::add(acc4[e], v0.v[e]));
    }
    template <class G> static __device__ __forceinline__ void prefetch(const G& g, i64 b, i64 i, i64 j0) {
        if (i >= g.M) return;
        for (int l = 0; l < 4; ++l) {
            const i64 j = j0 + l * 32;
            if (j < g.N) bafe::prefetch_l2(reinterpret_cast<const char*>(g.ep[0]) + (b * g.o_bstride + i * g.N + j) * 4);
        }
    }
};

extern "C" __global__ void __launch_bounds__(256) check_gemm_exact(const bafe::GemmArgs g) {
    bafe::gemm_exact<CheckSpec, false>(g);
}
extern "C" __global__ void __launch_bounds__(256) check_gemm_exact_tile32(const bafe::GemmArgs g) {
    bafe::gemm_exact<CheckSpec, false, 2>(g);
}
extern "C" __global__ void __launch_bounds__(256) check_gemm_exact_tile16(const bafe::GemmArgs g) {
    bafe::gemm_exact<CheckSpec, false, 1>(g);
}
extern "C" __global__ void __launch_bounds__(bafe::TcCfg<3>::THREADS, 1) check_gemm_tc3(const __grid_constant__ bafe::TcArgs g) {
    bafe::gemm_tc<CheckSpec, 3>(g);
}
extern "C" __global__ void __launch_bounds__(bafe::TcCfg<1>::THREADS, 1) check_gemm_tc1(const __grid_constant__ bafe::TcArgs g) {
    bafe::gemm_tc<CheckSpec, 1>(g);
}
extern "C" __global__ void __launch_bounds__(bafe::TcPairCfg<3>::THREADS, 1) check_gemm_tc3_pair(const __grid_constant__ bafe::TcArgs g) {
    bafe::gemm_tc_pair<CheckSpec, 3>(g);
}
extern "C" __global__ void __launch_bounds__(bafe::TcPairCfg<1>::THREADS, 1) check_gemm_tc1_pair(const __grid_constant__ bafe::TcArgs g) {
    bafe::gemm_tc_pair<CheckSpec, 1>(g);
}
extern "C" __global__ void __launch_bounds__(256) check_gemm_tc_fixup_pair(const __grid_constant__ bafe::TcArgs g) {
    bafe::gemm_tc_fixup<CheckSpec, 256>(g);
}
extern "C" __global__ void __launch_bounds__(bafe::TcPairCfg<3>::THREADS, 1) check_gemm_tc3_pair_conv(const __grid_constant__ bafe::TcArgs g) {
    bafe::gemm_tc_pair<CheckSpec, 3, bafe::ElemTf32, true>(g);
}
extern "C" __global__ void __launch_bounds__(bafe::TcCfg<3>::THREADS, 1) check_gemm_tc3_conv(const __grid_constant__ bafe::TcArgs g) {
    bafe::gemm_tc<CheckSpec, 3, bafe::ElemTf32, true>(g);
}
// bf16 operands (kind::f16), bf16 output through the emitter's conversion.
struct CheckSpecBf16 {
    typedef float TA; typedef float TB; typedef float T; typedef float P; typedef float S;
    typedef u16 Out;
    template <class G> static __device__ __forceinline__ Out apply(T acc, const G& g, i64 b, i64 i, i64 j) {
        return bafe::f32_to_bf16(bafe::relu(acc));
    }
    template <class G> static __device__ __forceinline__ void apply4(const T* acc4, const G&, i64, i64, i64, bafe::Vec4<Out>& o4) {
#pragma unroll
        for (int e = 0; e < 4; ++e) o4.v[e] = bafe::f32_to_bf16(bafe::relu(acc4[e]));
    }
    template <class G> static __device__ __forceinline__ void prefetch(const G&, i64, i64, i64) {}
};
extern "C" __global__ void __launch_bounds__(bafe::TcPairCfg<1>::THREADS, 1) check_gemm_bf16_pair(const __grid_constant__ bafe::TcArgs g) {
    bafe::gemm_tc_pair<CheckSpecBf16, 1, bafe::ElemBf16>(g);
}
extern "C" __global__ void __launch_bounds__(bafe::TcCfg<1>::THREADS, 1) check_gemm_bf16(const __grid_constant__ bafe::TcArgs g) {
    bafe::gemm_tc<CheckSpecBf16, 1, bafe::ElemBf16>(g);
}
extern "C" __global__ void __launch_bounds__(256) check_gemm_tc_fixup_bf16(const __grid_constant__ bafe::TcArgs g) {
    bafe::gemm_tc_fixup<CheckSpecBf16, 128>(g);
}
extern "C" __global__ void __launch_bounds__(256) check_transpose(const float* x, float* out, i64 M, i64 N, i64 ldx) {
    bafe::transpose2d<float>(x, out, M, N, ldx);
}
extern "C" __global__ void __launch_bounds__(256) check_transpose_w4(const float* x, float* out, i64 M, i64 N, i64 ldx) {
    bafe::transpose2d_w4<float>(x, out, M, N, ldx);
}
extern "C" __global__ void __launch_bounds__(256) check_gather(const float* x, float* out, const bafe::GatherArgs g) {
    bafe::gather_nd<float>(x, out, g);
}
extern "C" __global__ void __launch_bounds__(256) check_reduce(const float* x, float* out, i64 M, i64 N, int axis) {
    bafe::reduce_axis<float, false>(x, out, M, N, axis);
}
// relu(add(mul(X,Y),Z)) streaming kernel body as generated (4-wide).
extern "C" __global__ void __launch_bounds__(256) check_ew(const float* __restrict__ x, const float* __restrict__ y,
                                                          const float* __restrict__ z, float* __restrict__ o, i64 n) {
    const i64 ng = n >> 2;
    for (i64 g = (i64)blockIdx.x * blockDim.x + threadIdx.x; g < ng; g += (i64)gridDim.x * blockDim.x) {
        const auto a = bafe::ld4(x + 4 * g), b = bafe::ld4(y + 4 * g), c = bafe::ld4(z + 4 * g);
        bafe::Vec4<float> r;
#pragma unroll
        for (int l = 0; l < 4; ++l) r.v[l] = bafe::relu(bafe::add(bafe::mul(a.v[l], b.v[l]), c.v[l]));
        bafe::st4(o + 4 * g, r);
    }
}
