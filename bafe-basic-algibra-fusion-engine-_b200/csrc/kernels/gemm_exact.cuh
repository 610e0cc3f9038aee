// gemm_exact.cuh -- CUDA-core GEMM that reproduces BAFE's summation order
// bit for bit, with a generated elementwise epilogue.
//
// BAFE's matmul (codegen.c:240-290) accumulates each output as
//     v = 0; for each 32-wide k chunk c (increasing k): acc = 0;
//     acc += A*B over the chunk (left to right); v += acc
// with every multiply and add rounded separately (no FMA).  The fused
// forms (codegen.c:477-517) use one plain loop over all K: v = acc.
// Each thread here owns a 4x4 block of outputs and walks k in exactly that
// order with __fmul_rn/__fadd_rn, so the result equals the reference's
// compiled C for any shape.  This is the path for shapes the tensor-core
// kernel cannot take (TMA stride alignment), for integer and f64 graphs,
// and for gemm_precision=exact.
//
// Tiling: a (16 TM) x (16 TM) output tile per 256-thread block, TM = 4, 2
// or 1 (64, 32 or 16 wide: the lowering takes the largest that still
// gives the GPU enough blocks, so small problems are spread over more
// SMs), k staged 32 at a time through shared memory (the chunk width, so a
// chunk never spans two stages).  Thread (tx, ty) owns rows TM ty .. TM ty
// + TM-1 and columns TM tx .. TM tx + TM-1, so each k-step reads its TM A
// and TM B values as two contiguous runs (vector shared-memory loads; rows
// padded by 4 elements keep them 16-byte aligned).  On the 16- and 32-wide
// tiles the next stage's global loads are issued before the current stage's
// arithmetic and land in registers meanwhile (stored to shared memory after
// it), so their latency overlaps the k-loop instead of adding to it.
#pragma once
#include "bafe_dev.cuh"

namespace bafe {

struct GemmArgs {
    const void* a;
    const void* b;
    void* out;
    i64 M, N, K, batch;
    i64 a_bstride, b_bstride, o_bstride;   // elements between batch items
    int a_col, b_col;                      // operand stored column-major
    const void* ep[8];                     // epilogue operands
    i64 z0, y0;                            // first batch item / row tile of this launch
                                           // (a grid's y and z stop at 65535: larger
                                           // problems take several launches)
};

// Spec (generated per step) provides the operand value types TA/TB, the
// accumulator type T (the matmul node's buffer type), the C product and sum
// types P = TA*TB and S = T+P, loaders that read and convert one stored
// element, and apply(acc, g, batch, i, j) -> stored output element (the
// fused elementwise epilogue).  With all-f32 operands P = S = T = float.
template <class Spec, bool DIRECT, int TM = 4>
__device__ __forceinline__ void gemm_exact(const GemmArgs& g) {
    typedef typename Spec::TA TA;
    typedef typename Spec::TB TB;
    typedef typename Spec::T T;
    typedef typename Spec::P P;
    typedef typename Spec::S S;
    constexpr int TILE = 16 * TM;              // output tile edge
    constexpr int LD = TILE * 32 / 256;        // elements of each operand a thread stages per k-block
    __shared__ __align__(16) TA As[32][TILE + 4];   // As[k][m]
    __shared__ __align__(16) TB Bs[32][TILE + 4];   // Bs[k][n]
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const i64 bz = g.z0 + blockIdx.z;
    const i64 m0 = (g.y0 + (i64)blockIdx.y) * TILE, n0 = (i64)blockIdx.x * TILE;
    const i64 M = g.M, N = g.N, K = g.K;
    const i64 aoff = bz * g.a_bstride, boff = bz * g.b_bstride;

    T v[TM][TM], acc[TM][TM];
#pragma unroll
    for (int r = 0; r < TM; ++r)
#pragma unroll
        for (int c = 0; c < TM; ++c) { v[r][c] = (T)0; acc[r][c] = (T)0; }

    // Stage A[m0:m0+TILE, k0:k0+32] and B[k0:k0+32, n0:n0+TILE].  Elements
    // outside the matrices are zero on BOTH sides, so padded products are
    // +0 and leave every partial sum unchanged (an accumulator that starts
    // at +0 never holds -0, and x + +0 == x for every other x).  The loads
    // are branch-free (an element outside the matrix reads the matrix's
    // first element and is replaced by zero), so they are in flight together.
    TA av[LD];
    TB bv[LD];
    auto load_stage = [&](i64 k0) {
#pragma unroll
        for (int t = 0; t < LD; ++t) {
            const int e = tid + 256 * t;
            const int mm = g.a_col ? (e % TILE) : (e >> 5), kk = g.a_col ? (e / TILE) : (e & 31);
            const i64 gm = m0 + mm, gk = k0 + kk;
            const bool ina = gm < M && gk < K;
            av[t] = Spec::loadA(g.a, aoff + (ina ? (g.a_col ? gm + M * gk : gm * K + gk) : 0));
            if (!ina) av[t] = (TA)0;
            const int nn = g.b_col ? (e >> 5) : (e % TILE), kb = g.b_col ? (e & 31) : (e / TILE);
            const i64 gn = n0 + nn, gkb = k0 + kb;
            const bool inb = gn < N && gkb < K;
            bv[t] = Spec::loadB(g.b, boff + (inb ? (g.b_col ? K * gn + gkb : gkb * N + gn) : 0));
            if (!inb) bv[t] = (TB)0;
        }
    };
    auto store_stage = [&]() {
#pragma unroll
        for (int t = 0; t < LD; ++t) {
            const int e = tid + 256 * t;
            As[g.a_col ? (e / TILE) : (e & 31)][g.a_col ? (e % TILE) : (e >> 5)] = av[t];
            Bs[g.b_col ? (e & 31) : (e / TILE)][g.b_col ? (e >> 5) : (e % TILE)] = bv[t];
        }
    };
    if (K > 0) {
        load_stage(0);
        store_stage();
        __syncthreads();
    }
    // The 64-wide tile has enough independent work per stage to hide its
    // loads (and double-buffering them cost it 6 % at 1024^3): it loads
    // each stage after the previous one's arithmetic instead.
    constexpr bool AHEAD = TM < 4;
    for (i64 k0 = 0; k0 < K; k0 += 32) {
        const bool more = k0 + 32 < K;
        if (AHEAD && more) load_stage(k0 + 32);   // in flight during this stage's arithmetic
#pragma unroll 4
        for (int k = 0; k < 32; ++k) {
            TA a[TM];
            TB b[TM];
#pragma unroll
            for (int r = 0; r < TM; ++r) a[r] = As[k][TM * ty + r];
#pragma unroll
            for (int c = 0; c < TM; ++c) b[c] = Bs[k][TM * tx + c];
#pragma unroll
            for (int r = 0; r < TM; ++r)
#pragma unroll
                for (int c = 0; c < TM; ++c)
                    acc[r][c] = (T)add((S)acc[r][c], (S)mul((P)a[r], (P)b[c]));
        }
        if (!DIRECT) {
#pragma unroll
            for (int r = 0; r < TM; ++r)
#pragma unroll
                for (int c = 0; c < TM; ++c) { v[r][c] = add(v[r][c], acc[r][c]); acc[r][c] = (T)0; }
        }
        __syncthreads();                       // every thread is done reading this stage
        if (more) {
            if (!AHEAD) load_stage(k0 + 32);
            store_stage();
            __syncthreads();
        }
    }
    // Epilogue in two passes: every apply (operand loads only), then every
    // store -- an operand load cannot move above a store to `out` that may
    // alias it, so interleaved the 16 outputs' loads ran one after another
    // (a 64^3 relu(matmul + C) took 16 us, nearly all of it there).
    typedef typename Spec::Out Out;
    Out* out = reinterpret_cast<Out*>(g.out) + bz * g.o_bstride;
    Out res[TM][TM];
#pragma unroll
    for (int r = 0; r < TM; ++r) {
        const i64 i = m0 + TM * ty + r;
#pragma unroll
        for (int c = 0; c < TM; ++c) {
            const i64 j = n0 + TM * tx + c;
            if (i < M && j < N) res[r][c] = Spec::apply(DIRECT ? acc[r][c] : v[r][c], g, bz, i, j);
        }
    }
#pragma unroll
    for (int r = 0; r < TM; ++r) {
        const i64 i = m0 + TM * ty + r;
        if (i >= M) continue;
#pragma unroll
        for (int c = 0; c < TM; ++c) {
            const i64 j = n0 + TM * tx + c;
            if (j < N) out[i * N + j] = res[r][c];
        }
    }
}

}  // namespace bafe
