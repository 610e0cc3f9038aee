/* bafe_oracle.c -- CPU restatement of BAFE's generated-kernel arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the oracle the CUDA backend is
 * checked against; nothing in the product links it.  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg load the shared
 * object built from it.
 *
 * Every function restates one loop nest that BAFE's C99 emitter writes
 * (bafe/src/codegen.c, reference version 0.3.1) with the same per-element
 * operation order, so that compiled with -ffp-contract=off (no FMA), as the
 * reference's JIT effectively is (jit.c:275-280 passes -std=c11, which
 * implies -ffp-contract=off), it reproduces the reference bit for bit.
 * Parity is pinned: tests/golden holds outputs produced by the reference's
 * own generated kernels (see tests/golden/make_golden.py) and the CPU test
 * suite checks this file against them.
 *
 * Element types: f32 (float), f64 (double), i32, i64.  F16/BF16 inputs are
 * converted to f32 with the reference's own helpers (restated below) and
 * computed as f32, exactly like codegen.c:85-127,157-169.
 */
#include <stddef.h>
#include <stdint.h>
#include <string.h>
#include <math.h>

#define OR_ADD 0
#define OR_SUB 1
#define OR_MUL 2

/* ---------------------------------------------------------------------- */
/* elementwise binary ops                                                  */
/* ---------------------------------------------------------------------- */

/* Same-shape: v[i] = a[i] op b[i]  (codegen.c:322-325).
 * Row broadcast (M,N) op (N,): v[i*N+j] = a[i*N+j] op b[j] (codegen.c:304-312).
 * Row broadcast (N,) op (M,N): v[i*N+j] = a[j] op b[i*N+j] (codegen.c:313-321).
 * mode: 0 same shape over n=M*N elements, 1 = b is the row vector,
 *       2 = a is the row vector. */
#define DEF_BINARY(T, SFX)                                                     \
void oracle_binary_##SFX(int op, int mode, const T *a, const T *b, T *v,     \
                         int64_t M, int64_t N) {                               \
    if (mode == 0) {                                                           \
        int64_t n = M * N;                                                     \
        for (int64_t i = 0; i < n; i++) {                                      \
            T x = a[i], y = b[i];                                              \
            v[i] = op == OR_ADD ? (T)(x + y) : op == OR_SUB ? (T)(x - y)       \
                                             : (T)(x * y);                     \
        }                                                                      \
        return;                                                                \
    }                                                                          \
    for (int64_t i = 0; i < M; i++)                                            \
        for (int64_t j = 0; j < N; j++) {                                      \
            T x = mode == 1 ? a[i * N + j] : a[j];                             \
            T y = mode == 1 ? b[j] : b[i * N + j];                             \
            v[i * N + j] = op == OR_ADD ? (T)(x + y)                           \
                         : op == OR_SUB ? (T)(x - y) : (T)(x * y);             \
        }                                                                      \
}
DEF_BINARY(float, f32)
DEF_BINARY(double, f64)
DEF_BINARY(int32_t, i32)
DEF_BINARY(int64_t, i64)

/* relu: `T v = x[i]; y[i] = v > 0 ? v : 0;` (codegen.c:338-344).
 * NaN and -0 both become +0 because the comparison is false for them.
 * neg: y[i] = -x[i] (codegen.c:357-359). */
#define DEF_UNARY(T, SFX)                                                      \
void oracle_relu_##SFX(const T *x, T *y, int64_t n) {                          \
    for (int64_t i = 0; i < n; i++) { T v = x[i]; y[i] = v > 0 ? v : 0; }      \
}                                                                              \
void oracle_neg_##SFX(const T *x, T *y, int64_t n) {                           \
    for (int64_t i = 0; i < n; i++) y[i] = -x[i];                              \
}
DEF_UNARY(float, f32)
DEF_UNARY(double, f64)
DEF_UNARY(int32_t, i32)
DEF_UNARY(int64_t, i64)

/* sigmoid `1.0f / (1.0f + expf(-x))` and tanh `tanhf(x)` (codegen.c:345-356).
 * The emitter uses the float literals and float libm calls even for f64
 * buffers; the f64 variants restate that (double -> float call -> double). */
void oracle_sigmoid_f32(const float *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = 1.0f / (1.0f + expf(-x[i]));
}
void oracle_tanh_f32(const float *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = tanhf(x[i]);
}
void oracle_sigmoid_f64(const double *x, double *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = 1.0f / (1.0f + expf(-x[i]));
}
void oracle_tanh_f64(const double *x, double *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = tanhf(x[i]);
}

/* ---------------------------------------------------------------------- */
/* transpose                                                               */
/* ---------------------------------------------------------------------- */

/* Rank-2: output shape (M,N) = (x.cols, x.rows);
 * v[i*N+j] = x[j*M+i]  (codegen.c:363-369).  esize bytes per element. */
void oracle_transpose2d(const void *x, void *v, int64_t M, int64_t N, int esize) {
    const char *xs = (const char *)x; char *vs = (char *)v;
    for (int64_t i = 0; i < M; i++)
        for (int64_t j = 0; j < N; j++)
            memcpy(vs + (i * N + j) * esize, xs + (j * M + i) * esize, (size_t)esize);
}

/* Rank-R with permutation perm (codegen.c:371-404): for every output index
 * (o_0..o_{R-1}) in row-major order, in_idx = sum_d o_{perm[d]} * in_stride[d]
 * and out_idx = sum_d o_d * out_stride[d].  Note the emitter indexes the
 * INPUT strides with d and the loop variable with perm[d]; this is the
 * inverse permutation for non-involutive perms and is restated as is. */
void oracle_transpose_nd(const void *x, void *v, int R, const int32_t *out_dims,
                         const int32_t *in_dims, const int32_t *perm, int esize) {
    int64_t in_stride[8], out_stride[8], idx[8];
    int64_t numel = 1;
    for (int d = R - 1; d >= 0; d--) {
        in_stride[d] = 1; out_stride[d] = 1;
        for (int j = d + 1; j < R; j++) { in_stride[d] *= in_dims[j]; out_stride[d] *= out_dims[j]; }
    }
    for (int d = 0; d < R; d++) { numel *= out_dims[d]; idx[d] = 0; }
    const char *xs = (const char *)x; char *vs = (char *)v;
    for (int64_t t = 0; t < numel; t++) {
        int64_t rem = t;
        for (int d = R - 1; d >= 0; d--) { idx[d] = rem % out_dims[d]; rem /= out_dims[d]; }
        int64_t in_idx = 0, out_idx = 0;
        for (int d = 0; d < R; d++) {
            in_idx += idx[perm[d]] * in_stride[d];
            out_idx += idx[d] * out_stride[d];
        }
        memcpy(vs + out_idx * esize, xs + in_idx * esize, (size_t)esize);
    }
}

/* ---------------------------------------------------------------------- */
/* matmul                                                                  */
/* ---------------------------------------------------------------------- */

/* Tiled matmul (codegen.c:191-293): v = 0; for ii, jj, kk tiles of 32
 * (MATMUL_TILE, codegen.c:23), for i, j in the tile: acc = 0 (accumulator
 * type T); acc += A*B over k in the tile; v[i*N+j] += acc.
 * Each output is therefore ((0 + s_0) + s_1) + ... over 32-wide k chunks in
 * increasing k, each s_c summed left to right from 0.
 * A index: row `A[i*K+k]`, col `A[i + M*k]`; B index: row `B[k*N+j]`,
 * col `B[K*j + k]` (codegen.c:206-213).  Batched (codegen.c:215-236):
 * `batch` independent problems at offsets b*M*K, b*K*N, b*M*N.
 * chunk = 32 restates `matmul`; chunk = K (>= 1) restates the plain
 * i-j-k loop of the fused forms (codegen.c:477-485), where the output is
 * acc itself rather than 0 + acc (so pass direct = 1). */
#define DEF_MATMUL(T, SFX)                                                     \
void oracle_matmul_##SFX(const T *A, const T *B, T *v, int64_t batch,          \
                         int64_t M, int64_t N, int64_t K, int a_col,           \
                         int b_col, int64_t chunk, int direct) {               \
    for (int64_t b = 0; b < batch; b++) {                                      \
        const T *Ab = A + b * M * K; const T *Bb = B + b * K * N;              \
        T *vb = v + b * M * N;                                                 \
        if (direct) {                                                          \
            for (int64_t i = 0; i < M; i++)                                    \
                for (int64_t j = 0; j < N; j++) {                              \
                    T acc = 0;                                                 \
                    for (int64_t k = 0; k < K; k++) {                          \
                        T a = a_col ? Ab[i + M * k] : Ab[i * K + k];           \
                        T bb = b_col ? Bb[K * j + k] : Bb[k * N + j];          \
                        acc += a * bb;                                         \
                    }                                                          \
                    vb[i * N + j] = acc;                                       \
                }                                                              \
            continue;                                                          \
        }                                                                      \
        for (int64_t i = 0; i < M * N; i++) vb[i] = 0;                         \
        for (int64_t ii = 0; ii < M; ii += 32)                                 \
            for (int64_t jj = 0; jj < N; jj += 32)                             \
                for (int64_t kk = 0; kk < K; kk += chunk)                      \
                    for (int64_t i = ii; i < ii + 32 && i < M; i++)            \
                        for (int64_t j = jj; j < jj + 32 && j < N; j++) {      \
                            T acc = 0;                                         \
                            for (int64_t k = kk; k < kk + chunk && k < K; k++) { \
                                T a = a_col ? Ab[i + M * k] : Ab[i * K + k];   \
                                T bb = b_col ? Bb[K * j + k] : Bb[k * N + j];  \
                                acc += a * bb;                                 \
                            }                                                  \
                            vb[i * N + j] += acc;                              \
                        }                                                      \
    }                                                                          \
}
DEF_MATMUL(float, f32)
DEF_MATMUL(double, f64)
DEF_MATMUL(int32_t, i32)
DEF_MATMUL(int64_t, i64)

/* Row-panel matmul for large problems: rows [r0, r1) of the chunked matmul.
 * The chunk order of every element is independent of M (the ii loop only
 * groups rows), so a panel reproduces the full-size rows bit for bit.
 * out has (r1-r0)*N elements. */
void oracle_matmul_panel_f32(const float *A, const float *B, float *out,
                             int64_t M, int64_t N, int64_t K, int a_col, int b_col,
                             int64_t r0, int64_t r1) {
    for (int64_t i = r0; i < r1; i++)
        for (int64_t j = 0; j < N; j++) {
            float v = 0;
            for (int64_t kk = 0; kk < K; kk += 32) {
                float acc = 0;
                for (int64_t k = kk; k < kk + 32 && k < K; k++) {
                    float a = a_col ? A[i + M * k] : A[i * K + k];
                    float bb = b_col ? B[K * j + k] : B[k * N + j];
                    acc += a * bb;
                }
                v += acc;
            }
            out[(i - r0) * N + j] = v;
        }
}

/* ---------------------------------------------------------------------- */
/* reductions (codegen.c:406-452)                                          */
/* ---------------------------------------------------------------------- */

/* 1-D: sum `v[0] = 0; v[0] += x[i]`; max `v[0] = x[0]; if (x[i] > v[0]) ...`.
 * 2-D over axis ax (ax = axes[0] % 2): axis 0 reduces rows per column j,
 * axis 1 reduces columns per row i, same sequential order.
 * is_max selects reduce_max.  For 1-D pass M = 1, N = length, ax = 1. */
#define DEF_REDUCE(T, SFX)                                                     \
void oracle_reduce_##SFX(const T *x, T *v, int64_t M, int64_t N, int ax,       \
                         int is_max) {                                         \
    if (ax == 0) {                                                             \
        for (int64_t j = 0; j < N; j++) {                                      \
            if (!is_max) { v[j] = 0; for (int64_t i = 0; i < M; i++) v[j] += x[i * N + j]; } \
            else { v[j] = x[j]; for (int64_t i = 1; i < M; i++) if (x[i * N + j] > v[j]) v[j] = x[i * N + j]; } \
        }                                                                      \
    } else {                                                                   \
        for (int64_t i = 0; i < M; i++) {                                      \
            if (!is_max) { v[i] = 0; for (int64_t j = 0; j < N; j++) v[i] += x[i * N + j]; } \
            else { v[i] = x[i * N]; for (int64_t j = 1; j < N; j++) if (x[i * N + j] > v[i]) v[i] = x[i * N + j]; } \
        }                                                                      \
    }                                                                          \
}
DEF_REDUCE(float, f32)
DEF_REDUCE(double, f64)
DEF_REDUCE(int32_t, i32)
DEF_REDUCE(int64_t, i64)

/* ---------------------------------------------------------------------- */
/* F16 / BF16 boundary conversions (codegen.c:91-127)                      */
/* ---------------------------------------------------------------------- */

/* The emitter's own half helpers, restated: f16 -> f32 rebiases the
 * exponent by +112 without special-casing subnormals; f32 -> f16 truncates
 * the mantissa, flushes exponents below -10 to signed zero, shifts small
 * ones into subnormals and maps exponent >= 31 (including NaN) to inf.
 * bf16 -> f32 is a shift; f32 -> bf16 rounds to nearest even by adding
 * 0x7FFF + lsb (NaN payloads are not special-cased). */
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

float oracle_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)(h & 0x8000)) << 16;
    uint32_t ex = ((uint32_t)((h >> 10) & 0x1F)) + 112;
    uint32_t mant = ((uint32_t)(h & 0x3FF)) << 13;
    if ((h & 0x7FFF) == 0) return u2f(sign);
    if ((h & 0x7C00) == 0x7C00) return u2f(sign | 0x7F800000 | mant);
    return u2f(sign | (ex << 23) | mant);
}
uint16_t oracle_f32_to_f16(float f) {
    uint32_t bits = f2u(f);
    uint16_t sign = (bits >> 16) & 0x8000;
    int32_t ex = (int32_t)((bits >> 23) & 0xFF) - 127 + 15;
    uint32_t mant = (bits >> 13) & 0x3FF;
    if (ex <= 0) {
        if (ex < -10) return sign;
        mant = (mant | 0x400) >> (1 - ex);
        return (uint16_t)(sign | mant);
    }
    if (ex >= 31) return sign | 0x7C00;
    return (uint16_t)(sign | (ex << 10) | mant);
}
float oracle_bf16_to_f32(uint16_t b) { return u2f(((uint32_t)b) << 16); }
uint16_t oracle_f32_to_bf16(float f) {
    uint32_t bits = f2u(f);
    bits += 0x7FFF + ((bits >> 16) & 1);
    return (uint16_t)(bits >> 16);
}
void oracle_f16_to_f32_n(const uint16_t *h, float *f, int64_t n) {
    for (int64_t i = 0; i < n; i++) f[i] = oracle_f16_to_f32(h[i]);
}
void oracle_f32_to_f16_n(const float *f, uint16_t *h, int64_t n) {
    for (int64_t i = 0; i < n; i++) h[i] = oracle_f32_to_f16(f[i]);
}
void oracle_bf16_to_f32_n(const uint16_t *h, float *f, int64_t n) {
    for (int64_t i = 0; i < n; i++) f[i] = oracle_bf16_to_f32(h[i]);
}
void oracle_f32_to_bf16_n(const float *f, uint16_t *h, int64_t n) {
    for (int64_t i = 0; i < n; i++) h[i] = oracle_f32_to_bf16(f[i]);
}
