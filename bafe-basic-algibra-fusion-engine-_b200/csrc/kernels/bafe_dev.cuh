// bafe_dev.cuh -- device helpers shared by every generated kernel.
//
// Compiled by NVRTC for sm_100a as part of each plan's generated source
// (the host embeds this file as a string).  No CUDA or C++ standard headers
// are included: NVRTC provides the builtins and math functions.
#pragma once

typedef long long i64;
typedef unsigned long long u64;
typedef unsigned int u32;
typedef unsigned short u16;
typedef int i32;

namespace bafe {

// relu as BAFE's emitter writes it: `v > 0 ? v : 0` (codegen.c:338-344).
// NaN and -0 map to +0 because the comparison is false for them.  A select,
// never fmaxf (which would return -0 for -0 and the other operand for NaN).
__device__ __forceinline__ float relu(float v) { return v > 0.0f ? v : 0.0f; }
__device__ __forceinline__ double relu(double v) { return v > 0.0 ? v : 0.0; }
__device__ __forceinline__ i32 relu(i32 v) { return v > 0 ? v : 0; }
__device__ __forceinline__ i64 relu(i64 v) { return v > 0 ? v : 0; }

// Each arithmetic op rounds separately: the reference's generated C is
// compiled without contraction (-std=c11), so a*b+c must never become an FMA.
__device__ __forceinline__ float add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float sub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float mul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double add(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double sub(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ double mul(double a, double b) { return __dmul_rn(a, b); }
// Integer ops wrap (two's complement), which is what the reference's
// compiled C does in practice for int32_t/int64_t.
__device__ __forceinline__ i32 add(i32 a, i32 b) { return (i32)((u32)a + (u32)b); }
__device__ __forceinline__ i32 sub(i32 a, i32 b) { return (i32)((u32)a - (u32)b); }
__device__ __forceinline__ i32 mul(i32 a, i32 b) { return (i32)((u32)a * (u32)b); }
__device__ __forceinline__ i64 add(i64 a, i64 b) { return (i64)((u64)a + (u64)b); }
__device__ __forceinline__ i64 sub(i64 a, i64 b) { return (i64)((u64)a - (u64)b); }
__device__ __forceinline__ i64 mul(i64 a, i64 b) { return (i64)((u64)a * (u64)b); }

// a + b with the NaN results of the host's scalar SSE add (`addss a, b`,
// which the reference's sequential `acc += x` loops compile to): a NaN
// operand propagates quieted, the first one winning, and an invalid sum
// (inf - inf) gives the negative default NaN.  The device add returns one
// canonical NaN instead, which differs in sign and payload bits.
__device__ __forceinline__ float add_host_nan(float a, float b) {
    const float r = __fadd_rn(a, b);
    if (r == r) return r;
    if (a != a) return __uint_as_float(__float_as_uint(a) | 0x00400000u);
    if (b != b) return __uint_as_float(__float_as_uint(b) | 0x00400000u);
    return __uint_as_float(0xffc00000u);
}
__device__ __forceinline__ double add_host_nan(double a, double b) {
    const double r = __dadd_rn(a, b);
    if (r == r) return r;
    if (a != a) return __longlong_as_double(__double_as_longlong(a) | 0x0008000000000000ll);
    if (b != b) return __longlong_as_double(__double_as_longlong(b) | 0x0008000000000000ll);
    return __longlong_as_double((long long)0xfff8000000000000ull);
}
__device__ __forceinline__ i32 add_host_nan(i32 a, i32 b) { return add(a, b); }
__device__ __forceinline__ i64 add_host_nan(i64 a, i64 b) { return add(a, b); }

// sigmoid / tanh as emitted (codegen.c:345-356): `1.0f / (1.0f + expf(-x))`
// and `tanhf(x)` -- float libm calls and float literals whatever the buffer
// type, so the argument is converted to float first.  These go through
// CUDA's expf/tanhf and are tolerance-checked, not bit-exact.
__device__ __forceinline__ float sigmoid_of_neg(float neg_x) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(neg_x)));
}
__device__ __forceinline__ float tanh_f(float x) { return tanhf(x); }

// F16 / BF16 boundary conversions, restating the emitter's own helpers
// (codegen.c:91-127) bit for bit -- including their quirks (no subnormal
// input handling, truncating f32->f16, NaN -> inf) -- so that half-precision
// graphs reproduce the reference exactly.
__device__ __forceinline__ float f16_to_f32(u16 h) {
    u32 sign = ((u32)(h & 0x8000u)) << 16;
    u32 ex = ((u32)((h >> 10) & 0x1Fu)) + 112u;
    u32 mant = ((u32)(h & 0x3FFu)) << 13;
    if ((h & 0x7FFFu) == 0) return __uint_as_float(sign);
    if ((h & 0x7C00u) == 0x7C00u) return __uint_as_float(sign | 0x7F800000u | mant);
    return __uint_as_float(sign | (ex << 23) | mant);
}
__device__ __forceinline__ u16 f32_to_f16(float f) {
    u32 bits = __float_as_uint(f);
    u16 sign = (u16)((bits >> 16) & 0x8000u);
    i32 ex = (i32)((bits >> 23) & 0xFFu) - 127 + 15;
    u32 mant = (bits >> 13) & 0x3FFu;
    if (ex <= 0) {
        if (ex < -10) return sign;
        mant = (mant | 0x400u) >> (1 - ex);
        return (u16)(sign | mant);
    }
    if (ex >= 31) return (u16)(sign | 0x7C00u);
    return (u16)(sign | ((u32)ex << 10) | mant);
}
__device__ __forceinline__ float bf16_to_f32(u16 b) { return __uint_as_float(((u32)b) << 16); }
__device__ __forceinline__ u16 f32_to_bf16(float f) {
    u32 bits = __float_as_uint(f);
    bits += 0x7FFFu + ((bits >> 16) & 1u);
    return (u16)(bits >> 16);
}

// An L2 prefetch hint of the 128-byte line holding p (no register result,
// nothing to wait for).
__device__ __forceinline__ void prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// ---------------------------------------------------------------------------
// Streaming loads / stores.  Generated elementwise kernels move every
// operand once, so loads bypass L1 allocation and stores are marked
// evict-first; 16-byte vectors where alignment allows.
// ---------------------------------------------------------------------------
template <class T> struct Vec4 { T v[4]; };

__device__ __forceinline__ Vec4<float> ld4(const float* p) {
    float4 x = __ldcs(reinterpret_cast<const float4*>(p));
    Vec4<float> r; r.v[0] = x.x; r.v[1] = x.y; r.v[2] = x.z; r.v[3] = x.w; return r;
}
__device__ __forceinline__ Vec4<i32> ld4(const i32* p) {
    int4 x = __ldcs(reinterpret_cast<const int4*>(p));
    Vec4<i32> r; r.v[0] = x.x; r.v[1] = x.y; r.v[2] = x.z; r.v[3] = x.w; return r;
}
__device__ __forceinline__ Vec4<double> ld4(const double* p) {
    double2 a = __ldcs(reinterpret_cast<const double2*>(p));
    double2 b = __ldcs(reinterpret_cast<const double2*>(p) + 1);
    Vec4<double> r; r.v[0] = a.x; r.v[1] = a.y; r.v[2] = b.x; r.v[3] = b.y; return r;
}
__device__ __forceinline__ Vec4<i64> ld4(const i64* p) {
    longlong2 a = __ldcs(reinterpret_cast<const longlong2*>(p));
    longlong2 b = __ldcs(reinterpret_cast<const longlong2*>(p) + 1);
    Vec4<i64> r; r.v[0] = a.x; r.v[1] = a.y; r.v[2] = b.x; r.v[3] = b.y; return r;
}
__device__ __forceinline__ Vec4<u16> ld4(const u16* p) {
    uint2 x = __ldcs(reinterpret_cast<const uint2*>(p));
    Vec4<u16> r;
    r.v[0] = (u16)(x.x & 0xFFFFu); r.v[1] = (u16)(x.x >> 16);
    r.v[2] = (u16)(x.y & 0xFFFFu); r.v[3] = (u16)(x.y >> 16);
    return r;
}

__device__ __forceinline__ void st4(float* p, const Vec4<float>& r) {
    __stcs(reinterpret_cast<float4*>(p), make_float4(r.v[0], r.v[1], r.v[2], r.v[3]));
}
__device__ __forceinline__ void st4(i32* p, const Vec4<i32>& r) {
    __stcs(reinterpret_cast<int4*>(p), make_int4(r.v[0], r.v[1], r.v[2], r.v[3]));
}
__device__ __forceinline__ void st4(double* p, const Vec4<double>& r) {
    __stcs(reinterpret_cast<double2*>(p), make_double2(r.v[0], r.v[1]));
    __stcs(reinterpret_cast<double2*>(p) + 1, make_double2(r.v[2], r.v[3]));
}
__device__ __forceinline__ void st4(i64* p, const Vec4<i64>& r) {
    __stcs(reinterpret_cast<longlong2*>(p), make_longlong2(r.v[0], r.v[1]));
    __stcs(reinterpret_cast<longlong2*>(p) + 1, make_longlong2(r.v[2], r.v[3]));
}
__device__ __forceinline__ void st4(u16* p, const Vec4<u16>& r) {
    __stcs(reinterpret_cast<uint2*>(p),
           make_uint2((u32)r.v[0] | ((u32)r.v[1] << 16), (u32)r.v[2] | ((u32)r.v[3] << 16)));
}

}  // namespace bafe
