// layout.cuh -- data-movement kernels: rank-2 transpose, strided gather
// (rank-N transpose / broadcast), single-axis reductions.
//
// Instantiated by generated code with the element type; results are bit
// copies (transpose, gather) or follow BAFE's sequential summation order
// (reductions), so they match the reference exactly.
#pragma once
#include "bafe_dev.cuh"

namespace bafe {

// Rank-2 transpose materialisation: out has shape (M, N) and
// out[i*N + j] = x[j*ldx + i] (codegen.c:363-369; x is (N, M) row-major,
// ldx = M; a panel of output rows [r0, r0 + M') is the launch with x moved
// r0 columns, out moved r0 rows, M = M' and ldx the full row length).
// 32x32 tiles staged through shared memory so that both the global read
// (along x's rows) and the global write (along out's rows) are coalesced;
// the +1 column pad keeps the transposed shared-memory read conflict-free.
// Block (32, 8): each thread moves 4 elements per tile.  Grid covers
// (ceil(N/32), ceil(M/32)) tiles, batched over blockIdx.z.
template <class T>
__device__ __forceinline__ void transpose2d(const T* __restrict__ x, T* __restrict__ out,
                                            i64 M, i64 N, i64 ldx) {
    __shared__ T tile[32][33];
    const i64 b = blockIdx.z;
    x += b * ldx * N;
    out += b * M * N;
    const i64 j0 = (i64)blockIdx.x * 32;   // output column block == x row block
    const i64 i0 = (i64)blockIdx.y * 32;   // output row block == x column block
    const int tx = threadIdx.x, ty = threadIdx.y;
#pragma unroll
    for (int r = 0; r < 32; r += 8) {
        const i64 xr = j0 + ty + r, xc = i0 + tx;       // x[xr][xc], x is (N, M)
        if (xr < N && xc < M) tile[ty + r][tx] = x[xr * ldx + xc];
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 32; r += 8) {
        const i64 oi = i0 + ty + r, oj = j0 + tx;       // out[oi][oj] = x[oj][oi]
        if (oi < M && oj < N) out[oi * N + oj] = tile[tx][ty + r];
    }
}

// The same transpose for 4-byte element types with 16-byte global accesses
// (M, N and ldx multiples of 4, 16-byte aligned buffers): a CTA of 256
// threads moves a 64 x 64 tile.  Each thread first issues its four 16-byte
// loads (four rows of x, 64 B in flight), then scatters the 16 elements into
// the tile stored transposed -- S[c][r] for x's row r, column c -- and after
// the barrier reads four consecutive S[c][..] as one 16-byte vector, which
// is four consecutive elements of out's row c, stored with one 16-byte
// store.  The 16-byte chunks of each S row are XOR-swizzled with (c / 4) so
// that the scattering stores spread over the banks (2-way at most) while
// every vector read stays one aligned chunk.
template <class T>
__device__ __forceinline__ void transpose2d_w4(const T* __restrict__ x, T* __restrict__ out, i64 M, i64 N, i64 ldx) {
    static_assert(sizeof(T) == 4, "4-byte element types only");
    __shared__ __align__(16) u32 S[64 * 64];
    x += (i64)blockIdx.z * ldx * N;        // batched: one (N, ldx) x / (M, N) out per z
    out += (i64)blockIdx.z * M * N;
    const i64 j0 = (i64)blockIdx.x * 64;   // x row block == out column block
    const i64 i0 = (i64)blockIdx.y * 64;   // x column block == out row block
    const int t = threadIdx.x;
    const int q = t & 15, r0 = t >> 4;
    uint4 v[4];
#pragma unroll
    for (int pass = 0; pass < 4; ++pass) {
        const i64 xr = j0 + r0 + 16 * pass, xc = i0 + 4 * q;
        if (xr < N && xc < M) v[pass] = __ldcs(reinterpret_cast<const uint4*>(x + xr * ldx + xc));
        else v[pass] = make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int pass = 0; pass < 4; ++pass) {
        const int r = r0 + 16 * pass;
        const u32 e[4] = {v[pass].x, v[pass].y, v[pass].z, v[pass].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int c = 4 * q + k;               // (c / 4) & 15 == q
            S[c * 64 + 4 * ((r >> 2) ^ q) + (r & 3)] = e[k];
        }
    }
    __syncthreads();
    const int p = t & 15, c0 = t >> 4;
#pragma unroll
    for (int pass = 0; pass < 4; ++pass) {
        const int c = c0 + 16 * pass;
        const i64 oi = i0 + c, oj = j0 + 4 * p;
        const uint4 w = *reinterpret_cast<const uint4*>(&S[c * 64 + 4 * (p ^ ((c >> 2) & 15))]);
        if (oi < M && oj < N) __stcs(reinterpret_cast<uint4*>(out + oi * N + oj), w);
    }
}

// Strided gather over a rank-R output: out[o] = x[sum_d coord_d(o) * stride[d]]
// where coord_d is o's row-major coordinate.  Used for rank-N transposes
// (stride = input stride of the permuted axis) and for broadcast_to
// (stride 0 on broadcast axes).  Grid-stride, one element per step.
struct GatherArgs {
    i64 numel;
    int rank;
    i64 dims[8];
    i64 stride[8];
};

template <class T>
__device__ __forceinline__ void gather_nd(const T* __restrict__ x, T* __restrict__ out,
                                          const GatherArgs& g) {
    for (i64 o = (i64)blockIdx.x * blockDim.x + threadIdx.x; o < g.numel;
         o += (i64)gridDim.x * blockDim.x) {
        i64 rem = o, src = 0;
        for (int d = g.rank - 1; d >= 0; --d) {
            const i64 c = rem % g.dims[d];
            rem /= g.dims[d];
            src += c * g.stride[d];
        }
        out[o] = x[src];
    }
}

// The same gather when the innermost output axis is contiguous in x
// (stride 1) and a multiple of 4 long, every other stride a multiple of 4
// (or 0): four consecutive outputs are four consecutive, aligned inputs --
// one address computation and one vector load / store per four elements.
// x and out 16-byte aligned.
template <class T>
__device__ __forceinline__ void gather_nd_v4(const T* __restrict__ x, T* __restrict__ out,
                                             const GatherArgs& g) {
    const i64 L4 = g.dims[g.rank - 1] / 4;
    const i64 n4 = g.numel / 4;
    for (i64 q = (i64)blockIdx.x * blockDim.x + threadIdx.x; q < n4; q += (i64)gridDim.x * blockDim.x) {
        const i64 row = q / L4;
        i64 rem = row, src = (q - row * L4) * 4;
        for (int d = g.rank - 2; d >= 0; --d) {
            const i64 c = rem % g.dims[d];
            rem /= g.dims[d];
            src += c * g.stride[d];
        }
        st4(out + q * 4, ld4(x + src));
    }
}

// Single-axis reduction of an (M, N) tensor, sequential per output element
// exactly as codegen.c:410-445 loops: axis 0 -> one output per column j
// (consecutive threads read consecutive columns: coalesced), axis 1 -> one
// output per row i.  Sum starts from 0 and accumulates with the host's NaN
// results (acc first, as `out[i] += x[...]`); max starts from the first
// element and replaces on a strict `>`.
template <class T, bool IS_MAX>
__device__ __forceinline__ void reduce_axis(const T* __restrict__ x, T* __restrict__ out,
                                            i64 M, i64 N, int axis) {
    const i64 t = (i64)blockIdx.x * blockDim.x + threadIdx.x;
    if (axis == 0) {
        if (t >= N) return;
        T v = IS_MAX ? x[t] : (T)0;
        for (i64 i = IS_MAX ? 1 : 0; i < M; ++i) {
            const T e = x[i * N + t];
            if (IS_MAX) { if (e > v) v = e; } else { v = add_host_nan(v, e); }
        }
        out[t] = v;
    } else {
        if (t >= M) return;
        const T* row = x + t * N;
        T v = IS_MAX ? row[0] : (T)0;
        for (i64 j = IS_MAX ? 1 : 0; j < N; ++j) {
            const T e = row[j];
            if (IS_MAX) { if (e > v) v = e; } else { v = add_host_nan(v, e); }
        }
        out[t] = v;
    }
}

}  // namespace bafe
