// gemm_tc.cuh -- tcgen05 tensor-core GEMM (sm_100a) with a generated
// elementwise epilogue: out = epi(A . B), fp32 in/out.
//
// Structure (one CTA per SM, persistent over 128 x 256 output tiles):
//   warp 0        TMA producer: k-blocks of A and B (and, for 3xTF32, of
//                 their residuals A_lo, B_lo) into a STAGES-deep ring of
//                 swizzled shared-memory stages.  No multicast.
//   warp 1        allocates TMEM; one lane issues tcgen05.mma (kind::tf32,
//                 M=128, N=256, K=8 per instruction).  The K loop is cut
//                 into chunks (KC k-blocks: TcCfg / TcPairCfg, or the
//                 element trait's KB_CHUNK); each chunk accumulates into
//                 one of two TMEM buffers, starting from zero.
//   warps 2-9     accumulate: each thread owns one tile row (TMEM lane) and
//                 128 columns; after every chunk it tcgen05.ld's the chunk
//                 partial sums and adds them into 128 fp32 registers with
//                 round-to-nearest (packed fp32x2 adds), then releases the
//                 TMEM buffer to the
//                 MMA warp.  After the last chunk it applies the generated
//                 epilogue (Spec::apply4: relu(acc + C), ...) and stores
//                 through TMA (tc_epilogue).
//                 For 3xTF32 with CONVERT the same threads also write the
//                 tf32 residuals of every stage, one chunk ahead of the
//                 drain they wait for (see below).
//
// Why chunks: the tensor core's fp32 accumulator truncates at every
// accumulation step, which biases long sums (measured: the 3xTF32 error
// grew like K^1.5 with a single TMEM accumulator, 1.1e-2 at K=4096).
// Summing short partial sums in registers with round-to-nearest keeps the
// error a random walk over chunks (~KC * K^0.5), inside the 3xTF32 bound.
//
// kind::tf32 reads the top 19 bits of each fp32 operand (the low 13
// mantissa bits are ignored).  3xTF32 operands: A is split to nearest,
// A_hi = rn_tf32(x), A_lo = rn_tf32(x - A_hi); B's raw values are its "hi"
// part (truncated by the tensor core) and B_lo = rn_tf32(x - trunc_tf32(x)).
// With one side rounded to nearest the dropped A_lo.B_lo term has no
// systematic sign (with both sides truncated it always had the product's
// sign and biased sums toward zero: mean error -1.9e-9 at 16384^3, now ~0).
// Rounding A rather than B: a sharded GEMM's rank holds a row panel of A
// but all of B, so it writes one copy of B (B_lo) instead of two.  The
// stage holds [A_hi][B][A_lo][B_lo]; each k-step
//     acc += A_hi.B_lo + A_lo.B, then acc += A_hi.B   (three MMAs)
// By default streaming pre-passes (tf32_split for A, tf32_residual for B)
// write the parts to memory and TMA loads them.  With CONVERT the producer
// loads only the raw operands and the accumulate threads write the parts
// into the stage in shared memory (lo into the second half, A_hi over the
// raw A; elementwise, so the swizzle needs no index
// mapping), releasing each stage to the MMA issuer on LO(s): no pre-pass,
// no scratch, half the operand bytes from L2 and HBM -- but 64 KB more
// shared-memory traffic per k-block and CTA, which costs throughput on B200.
//
// Operand layouts (BAFE layout tags): A row-major = K-major, A col-major =
// M-major; B col-major = K-major, B row-major = N-major.  K-major tiles are
// loaded as one [rows x 32] box (128 B per row, 128B swizzle); MN-major
// tiles as 32-wide boxes [k 32 x mn 32] side by side, written by TMA with
// the 128B-swizzle-32B-atom mode that MN-major tf32 UMMA operands require.
//
// Every wait is bounded by a wall-clock deadline (globaltimer): a role that
// times out raises the CTA's abort flag and the caller-visible error word,
// every role then leaves its loop, in-flight TMA copies and MMAs are drained
// (bounded again), TMEM is freed and the kernel returns.
#pragma once
#include "bafe_dev.cuh"

namespace bafe {

struct __align__(64) TmaDesc { unsigned long long v[16]; };   // CUtensorMap

struct TcArgs {
    TmaDesc tmap_a;
    TmaDesc tmap_b;
    TmaDesc tmap_a_lo;             // 3xTF32 residuals (same layouts as A, B)
    TmaDesc tmap_b_lo;
    TmaDesc tmap_out;              // output, for TMA stores (valid when out_tma)
    TmaDesc tmap_ws;               // split partials [parts x tile rows][256] f32 (valid when split > 1)
    void* out;
    i64 M, N, K;
    i64 o_bstride;
    const void* ep[8];
    unsigned* err;                 // error word (0 = ok); set on timeout
    int a_mn, b_mn;                // operand is MN-major
    int num_m, num_n, num_tiles;
    int group_m;                   // rasterisation group along M
    unsigned long long timeout_ns; // per-wait deadline
    int batch;                     // independent products (tiles: batch x num_m x num_n)
    int a_batched, b_batched;      // operand has its own matrix per batch item
    int out_tma;                   // epilogue stores through tmap_out
    int ep_vec;                    // epilogue operands load as 4-element vectors
    float* ws;                     // split partials (see unit_range)
    int split;                     // K ranges per tail tile (1: no split)
    int split_first;               // first split tile: tiles [split_first, num_tiles) are split
    int num_units;                 // split_first + (num_tiles - split_first) * split
    unsigned* wave_ctr;            // wave alignment counter (zero at launch), or null
    // K slices (CTA-pair kernel): this launch covers k-blocks [kb_first,
    // kb_last), kb_first a multiple of the promotion chunk, so every output
    // still sums the same chunk partials in the same order.  acc_in: each
    // tile's sums start from the fp32 values in `out` (the previous slice's);
    // acc_raw: the sums are stored to `out` as they are, without the
    // epilogue (a later slice continues them).  A whole-K launch has
    // kb_first 0, kb_last 0 (all k-blocks) and both flags 0.
    int kb_first, kb_last;
    int acc_in, acc_raw;
};
static_assert(sizeof(TcArgs) == 1024, "TcArgs layout (mirrored by the host)");

// Work units of the persistent kernels.  Tiles [0, split_first) are whole
// units; when the last wave would leave CTAs idle, each tile from
// split_first on becomes `split` units over consecutive ranges of whole
// TMEM chunks [c0, c1) of K, which store their fp32 partial tile to ws
// (part p of split tile s at rows (s * split + p) * tile rows); the fixup
// kernel (gemm_tc_fixup) adds the parts in order and applies the epilogue.
// part = -1 for a whole tile.
__device__ __forceinline__ void unit_range(const TcArgs& g, int u, int n_chunks, int& t, int& c0, int& c1, int& part) {
    if (u < g.split_first) {
        t = u; c0 = 0; c1 = n_chunks; part = -1;
        return;
    }
    const int v = u - g.split_first;
    t = g.split_first + v / g.split;
    part = v % g.split;
    c0 = (int)((long long)part * n_chunks / g.split);
    c1 = (int)((long long)(part + 1) * n_chunks / g.split);
}

template <int VARIANT> struct TcCfg;
// KB_PER_CHUNK k-blocks (of 32) per TMEM partial sum: the 3xTF32 variant,
// whose accuracy bound is tight, promotes twice as often.
template <> struct TcCfg<1> {      // 1xTF32
    static constexpr int BN = 256, STAGES = 4, THREADS = 320, KB_PER_CHUNK = 4;
};
template <> struct TcCfg<3> {      // 3xTF32
    static constexpr int BN = 256, STAGES = 2, THREADS = 320, KB_PER_CHUNK = 2;
};
// CTA-pair variants (gemm_tc_pair): each CTA stages its 128 rows of A and
// half (128 columns) of B per k-block, so a stage is a third smaller and
// the ring deeper.
template <int VARIANT> struct TcPairCfg;
// 1xTF32 pair: 1024-deep chunks (its error is the operands' tf32
// rounding; promoting every 256 k cost 5 % under the power cap).
template <> struct TcPairCfg<1> {
    static constexpr int STAGES = 6, THREADS = 320, KB_PER_CHUNK = 32;
};
// 3xTF32 pair: 96-deep chunks.  With 64-deep ones the MMA issuer waited
// on a TMEM buffer still being drained for part of its time; 96-deep
// chunks run 4.4-4.6 % faster on two B200s under the power cap (A/B on the
// same box, the SM clock no lower), 128-deep ones 5.3 %, for an error that
// grows with the chunk: max |err| at 4096^3 1.87e-4 (64), 2.63e-4 (96),
// 3.40e-4 (128) against the bound 8e-4.  96 keeps most of the gain and
// fits the converting form's look-ahead (KB_PER_CHUNK <= STAGES).  (An
// older form of this kernel lost 11 % net with 96-deep chunks on a box
// whose power cap then pulled the clock from 1.49 to 1.19 GHz.)
template <> struct TcPairCfg<3> {
    static constexpr int STAGES = 3, THREADS = 320, KB_PER_CHUNK = 3;
};

// Two IEEE round-to-nearest fp32 additions in one instruction (Blackwell
// packed fp32): a0 += b0, a1 += b1, the same results as two __fadd_rn.
__device__ __forceinline__ void fadd2_rn(float& a0, float& a1, u32 b0, u32 b1) {
    asm("{\n\t.reg .b64 x, y;\n\tmov.b64 x, {%0, %1};\n\tmov.b64 y, {%2, %3};\n\tadd.rn.f32x2 x, x, y;\n\tmov.b64 {%0, %1}, x;\n\t}"
        : "+f"(a0), "+f"(a1) : "r"(b0), "r"(b1));
}

// x rounded to the nearest tf32 value (ties to even on the 10-bit
// mantissa; the low 13 bits come out clear).  Rounding the bit pattern's
// magnitude is symmetric in the sign.  A value whose rounding would
// overflow is truncated instead (it stays finite; a residual carries the
// rest); inf and NaN are returned unchanged.
__device__ __forceinline__ float tf32_rn(float x) {
    const u32 b = __float_as_uint(x);
    if ((b & 0x7F800000u) == 0x7F800000u) return x;
    const u32 r = (b + 0x0FFFu + ((b >> 13) & 1u)) & 0xFFFFE000u;
    return __uint_as_float((r & 0x7F800000u) == 0x7F800000u ? (b & 0xFFFFE000u) : r);
}

// Residual of the tf32 truncation, x - (x with the low 13 mantissa bits
// cleared) -- exact in fp32 -- rounded to the nearest tf32 value, so the
// tensor core, which ignores those 13 bits, reads it rounded rather than
// truncated.  0 for inf / NaN (the raw operand, the hi part, carries them).
// Used where the raw operand itself is the hi part (kind::tf32 truncates
// it); lo then has the sign of x.
__device__ __forceinline__ float tf32_lo(float x) {
    const u32 bits = __float_as_uint(x);
    if ((bits & 0x7F800000u) == 0x7F800000u) return 0.0f;
    return tf32_rn(__fsub_rn(x, __uint_as_float(bits & 0xFFFFE000u)));
}

// Round-to-nearest split x ~ hi + lo: hi = tf32_rn(x), lo = tf32_rn(x - hi)
// (x - hi is exact in fp32).  |lo| <= 2^-11 |x| and its sign is independent
// of x's, so the dropped lo_a * lo_b product of the 3xTF32 scheme no longer
// has the sign of a * b (with a truncated hi on both sides it always did,
// which biased every sum toward zero).
__device__ __forceinline__ void tf32_split(float x, float& hi, float& lo) {
    hi = tf32_rn(x);
    lo = ((__float_as_uint(x) & 0x7F800000u) == 0x7F800000u) ? 0.0f : tf32_rn(__fsub_rn(x, hi));
}

namespace tc {

constexpr int BM = 128, BK = 32;

__device__ __forceinline__ u32 smem_u32(const void* p) {
    return static_cast<u32>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ u64 now_ns() {
    u64 t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(u32 bar, u32 count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ bool mbar_try(u32 bar, u32 parity) {
    u32 ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
__device__ __forceinline__ void mbar_arrive(u32 bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(u32 bar, u32 bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// TMA tile load of a 3-D map (x, y, batch) into this CTA's shared memory,
// completing on the mbarrier at `bar`.
__device__ __forceinline__ void tma_load_3d(u32 dst, const TmaDesc* map, u32 bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<u64>(map)), "r"(bar), "r"(x), "r"(y), "r"(z) : "memory");
}
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(u32 bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_mma_tf32(u32 tmem_d, u64 adesc, u64 bdesc, u32 idesc, u32 accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate),
          "r"(0u), "r"(0u), "r"(0u), "r"(0u) : "memory");
}
__device__ __forceinline__ void tc_mma_f16kind(u32 tmem_d, u64 adesc, u64 bdesc, u32 idesc, u32 accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate),
          "r"(0u), "r"(0u), "r"(0u), "r"(0u) : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp gets row
// (lane base + t), columns [col, col+32).  tmem_ld32_nowait issues the load
// only; tmem_wait_ld waits for every load issued before it.
__device__ __forceinline__ void tmem_ld32_nowait(u32 taddr, u32 (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
// The wait names the loaded registers as operands so that no use of them can
// be scheduled between the asynchronous load and its completion.
__device__ __forceinline__ void tmem_wait_ld(u32 (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;" : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31]) :: "memory");
}
__device__ __forceinline__ void tmem_wait_ld(u32 (&a)[32], u32 (&b)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;" : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]), "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]), "+r"(a[12]), "+r"(a[13]), "+r"(a[14]), "+r"(a[15]), "+r"(a[16]), "+r"(a[17]), "+r"(a[18]), "+r"(a[19]), "+r"(a[20]), "+r"(a[21]), "+r"(a[22]), "+r"(a[23]), "+r"(a[24]), "+r"(a[25]), "+r"(a[26]), "+r"(a[27]), "+r"(a[28]), "+r"(a[29]), "+r"(a[30]), "+r"(a[31]), "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7]), "+r"(b[8]), "+r"(b[9]), "+r"(b[10]), "+r"(b[11]), "+r"(b[12]), "+r"(b[13]), "+r"(b[14]), "+r"(b[15]), "+r"(b[16]), "+r"(b[17]), "+r"(b[18]), "+r"(b[19]), "+r"(b[20]), "+r"(b[21]), "+r"(b[22]), "+r"(b[23]), "+r"(b[24]), "+r"(b[25]), "+r"(b[26]), "+r"(b[27]), "+r"(b[28]), "+r"(b[29]), "+r"(b[30]), "+r"(b[31]) :: "memory");
}
__device__ __forceinline__ void tmem_ld32(u32 taddr, u32 (&r)[32]) {
    tmem_ld32_nowait(taddr, r);
    tmem_wait_ld(r);
}

// UMMA shared-memory descriptor, version 1; lbo / sbo in bytes.
// K-major operands use the 128B swizzle (layout type 2): 8-row groups
// (SBO = 1024 B), K advances inside the 128-byte row.  MN-major tf32
// operands must use the 128B swizzle with 32-byte atoms (layout type 1,
// "128B_BASE32B"): 32 elements along MN per 128-byte row, 4-row K groups
// (SBO = 512 B), MN atoms LBO apart.
__device__ __forceinline__ u64 smem_desc(u32 addr, u32 lbo, u32 sbo, u32 layout) {
    u64 d = 0;
    d |= (u64)((addr >> 4) & 0x3FFFu);
    d |= (u64)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (u64)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (u64)1 << 46;
    d |= (u64)(layout & 7u) << 61;
    return d;
}

// Instruction descriptor: D f32, A/B format (kind::tf32: 2 = TF32;
// kind::f16: 0 = F16, 1 = BF16), majors, N, M (128, or 256 for a CTA pair).
__device__ __forceinline__ u32 instr_desc(int a_mn, int b_mn, int n, int m = BM, u32 fmt = 2u) {
    return (1u << 4) | (fmt << 7) | (fmt << 10) | ((u32)a_mn << 15) | ((u32)b_mn << 16) |
           ((u32)(n >> 3) << 17) | ((u32)(m >> 4) << 24);
}

// Shared state of one CTA.
struct Shared {
    u32 abort;
    u32 tmem_base;
};

// try_wait with cluster-scope acquire: the phase completes with arrivals
// released by the peer CTA of a pair (their shared-memory writes included).
__device__ __forceinline__ bool mbar_try_cluster(u32 bar, u32 parity) {
    u32 ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint4 lds128(u32 addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ void sts128(u32 addr, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
// Writes the tf32 residual of PER x NT 16-byte chunks (chunk i of thread ct
// at (ct + i * NT) * 16 bytes) from `hi` to the same offsets at `lo`, four
// chunks per round (four shared-memory loads in flight; the callers hold
// 128 accumulators, so a wider round spills).
// The first A_PER rounds cover the stage's A tile: hi and lo come from the
// round-to-nearest split (tf32_split) and hi is written back over the raw
// operand.  The remaining rounds cover B: the raw operand stays the hi part
// and lo = tf32_lo(x) -- the same operands the pre-passes give the kernel.
template <int PER, int NT, int A_PER>
__device__ __forceinline__ void convert_stage(u32 hi, u32 lo, int ct) {
    constexpr int R = 4;
    static_assert(PER % R == 0 && A_PER % R == 0, "rounds of four chunks");
#pragma unroll
    for (int r = 0; r < PER; r += R) {
        uint4 v[R];
#pragma unroll
        for (int j = 0; j < R; ++j) v[j] = lds128(hi + 16u * (u32)(ct + (r + j) * NT));
        if (r >= A_PER) {
#pragma unroll
            for (int j = 0; j < R; ++j) {
                v[j].x = __float_as_uint(tf32_lo(__uint_as_float(v[j].x)));
                v[j].y = __float_as_uint(tf32_lo(__uint_as_float(v[j].y)));
                v[j].z = __float_as_uint(tf32_lo(__uint_as_float(v[j].z)));
                v[j].w = __float_as_uint(tf32_lo(__uint_as_float(v[j].w)));
            }
        } else {
#pragma unroll
            for (int j = 0; j < R; ++j) {
                float h[4], l[4];
                tf32_split(__uint_as_float(v[j].x), h[0], l[0]);
                tf32_split(__uint_as_float(v[j].y), h[1], l[1]);
                tf32_split(__uint_as_float(v[j].z), h[2], l[2]);
                tf32_split(__uint_as_float(v[j].w), h[3], l[3]);
                sts128(hi + 16u * (u32)(ct + (r + j) * NT),
                       make_uint4(__float_as_uint(h[0]), __float_as_uint(h[1]), __float_as_uint(h[2]),
                                  __float_as_uint(h[3])));
                v[j] = make_uint4(__float_as_uint(l[0]), __float_as_uint(l[1]), __float_as_uint(l[2]),
                                  __float_as_uint(l[3]));
            }
        }
#pragma unroll
        for (int j = 0; j < R; ++j) sts128(lo + 16u * (u32)(ct + (r + j) * NT), v[j]);
    }
}

// Bounded wait on an mbarrier phase; returns false (and raises the abort
// flag / error word) on timeout or when another role has aborted.
__device__ __forceinline__ bool wait(u32 bar, u32 parity, volatile Shared* sh, const TcArgs& g, u32 code) {
    if (mbar_try(bar, parity)) return true;
    const u64 t0 = now_ns();
    while (true) {
        if (mbar_try(bar, parity)) return true;
        if (sh->abort) return false;
        if (now_ns() - t0 > g.timeout_ns) {
            sh->abort = 1u;
            atomicCAS(g.err, 0u, code);
            return false;
        }
    }
}

// Limit of the final drains (copies in flight, MMAs before TMEM is freed):
// never below 200 ms, so that a short wait deadline cannot cut them off --
// asynchronous work that is already issued finishes in microseconds.
__device__ __forceinline__ u64 drain_ns(const TcArgs& g) {
    return g.timeout_ns > 200000000ull ? g.timeout_ns : 200000000ull;
}

// The same wait with cluster-scope acquire (mbar_try_cluster).
__device__ __forceinline__ bool wait_cluster(u32 bar, u32 parity, volatile Shared* sh, const TcArgs& g, u32 code) {
    if (mbar_try_cluster(bar, parity)) return true;
    const u64 t0 = now_ns();
    while (true) {
        if (mbar_try_cluster(bar, parity)) return true;
        if (sh->abort) return false;
        if (now_ns() - t0 > g.timeout_ns) {
            sh->abort = 1u;
            atomicCAS(g.err, 0u, code);
            return false;
        }
    }
}

__device__ __forceinline__ u32 cluster_rank() {
    u32 r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Arrive on the mbarrier at the same shared-memory offset in CTA `rank` of
// the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(u32 bar, u32 rank) {
    u32 remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(bar), "r"(rank));
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on the
// pair leader's mbarrier (same offset); no multicast.
__device__ __forceinline__ void tma_load_2d_pair(u32 dst, const TmaDesc* map, u32 bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<u64>(map)), "r"(bar & 0xFEFFFFFFu), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(u32 dst, const TmaDesc* map, u32 bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<u64>(map)), "r"(bar & 0xFEFFFFFFu), "r"(x), "r"(y), "r"(z) : "memory");
}
__device__ __forceinline__ void tc_mma_tf32_pair(u32 tmem_d, u64 adesc, u64 bdesc, u32 idesc, u32 accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate),
          "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u) : "memory");
}
__device__ __forceinline__ void tc_mma_f16kind_pair(u32 tmem_d, u64 adesc, u64 bdesc, u32 idesc, u32 accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate),
          "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u) : "memory");
}
// Completion of the pair's prior MMAs signalled on the barrier at offset
// `bar` in both CTAs of the pair (tcgen05.commit, not a load).
__device__ __forceinline__ void tc_commit_pair(u32 bar) {
    asm volatile(
        "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}"
        ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tile_coords(const TcArgs& g, int t, int& mb, int& nb, int& bi) {
    const int per_batch = g.num_m * g.num_n;
    bi = t / per_batch;
    t -= bi * per_batch;
    const int per_group = g.group_m * g.num_n;
    const int group = t / per_group;
    const int first_m = group * g.group_m;
    int gsize = g.num_m - first_m;
    if (gsize > g.group_m) gsize = g.group_m;
    const int local = t - group * per_group;
    mb = first_m + local % gsize;
    nb = local / gsize;
}

}  // namespace tc

// Epilogue of one accumulate warp: rows i0 .. i0+31 (lane r holds row
// i0 + r in acc), columns n0 .. n0+127.  Lane r's loads and stores touch 32
// rows per warp instruction, one L1 transaction per row, so:
//   * pass 1 applies the generated epilogue with 16-byte operand loads
//     (Spec::apply4, when every operand is aligned for them: ep_vec), all
//     loads and no stores, so they are in flight together -- an operand
//     load cannot move above a store to `out` that may alias it;
//   * pass 2 stores through TMA: each 32-row x 128-byte sub-tile is written
//     to this warp's 4 KB staging buffer in shared memory (128B swizzle,
//     conflict-free 16-byte stores) and one lane issues a bulk tensor store,
//     which writes whole rows and clips rows >= M and columns >= N (L2
//     evict-first, like streaming stores).
// Measured on a 256^3 tf32 pair tile: relu(acc + C) 41k -> 12k cycles,
// plain stores 9.3k -> 4.5k.  Results of at most 4 bytes are kept, as
// bits, in the accumulator registers between the passes.
template <class T> struct tc_is_f32 { static constexpr bool value = false; };
template <> struct tc_is_f32<float> { static constexpr bool value = true; };
constexpr u32 EPI_OFFSET = 1024;                 // staging: after the ring's mbarriers and Shared words
constexpr u32 EPI_WARP_BYTES = 4096;             // 32 rows x 128 bytes per accumulate warp
__device__ __forceinline__ float tc_pack_bits(float x) { return x; }
__device__ __forceinline__ float tc_pack_bits(i32 x) { return __int_as_float(x); }
__device__ __forceinline__ float tc_pack_bits(u16 x) { return __uint_as_float(x); }
template <class T> __device__ __forceinline__ T tc_unpack_bits(float f);
template <> __device__ __forceinline__ float tc_unpack_bits<float>(float f) { return f; }
template <> __device__ __forceinline__ i32 tc_unpack_bits<i32>(float f) { return __float_as_int(f); }
template <> __device__ __forceinline__ u16 tc_unpack_bits<u16>(float f) { return (u16)__float_as_uint(f); }
// 16 bytes of results (4 x 4-byte or 8 x 2-byte) from their bits in acc
template <class Out>
__device__ __forceinline__ uint4 tc_chunk(const float* a) {
    if constexpr (sizeof(Out) == 4) {
        return make_uint4(__float_as_uint(a[0]), __float_as_uint(a[1]), __float_as_uint(a[2]), __float_as_uint(a[3]));
    } else {
        u32 w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) w[e] = (__float_as_uint(a[2 * e]) & 0xFFFFu) | (__float_as_uint(a[2 * e + 1]) << 16);
        return make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// TMA store of one accumulate warp's 32 rows x 128 results (their bits in
// acc): 32-row x 128-byte sub-tiles through the warp's staging buffer
// (128B swizzle: lane r writes its 16-byte chunk c at chunk c ^ (r & 7) of
// row r, conflict-free), one bulk tensor store each, at map coordinates
// (x0 + sub-tile column, y0, z); sub-tiles from x_end on are skipped.
// EVICT_FIRST: the rows are not read again soon (final output).
template <class Out, bool EVICT_FIRST>
__device__ __forceinline__ void tc_store_rows(const float (&acc)[128], const TmaDesc* map, i64 x0, i64 y0, i64 z, i64 x_end,
                                              u32 stg, int lane) {
    constexpr int SUB = 128 / sizeof(Out);            // columns per 128-byte sub-tile
    constexpr int PER = 16 / sizeof(Out);             // results per 16-byte chunk
#pragma unroll
    for (int sb = 0; sb < 128 / SUB; ++sb) {
        if (x0 + sb * SUB >= x_end) break;            // warp-uniform
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");   // buffer free
        __syncwarp();
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const uint4 w = tc_chunk<Out>(acc + sb * SUB + c * PER);
            const u32 addr = stg + (u32)lane * 128u + (u32)((c ^ (lane & 7)) * 16);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w.x), "r"(w.y), "r"(w.z), "r"(w.w)
                         : "memory");
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // visible to the TMA unit
        __syncwarp();
        if (lane == 0) {
            if (EVICT_FIRST) {
                // like streaming stores: the output must not push the
                // operand panels out of L2
                u64 policy;
                asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
                asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group.L2::cache_hint"
                             " [%0, {%1, %2, %3}], [%4], %5;"
                             ::"l"(map), "r"((int)(x0 + sb * SUB)), "r"((int)y0), "r"((int)z), "r"(stg), "l"(policy)
                             : "memory");
            } else {
                asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];"
                             ::"l"(map), "r"((int)(x0 + sb * SUB)), "r"((int)y0), "r"((int)z), "r"(stg) : "memory");
            }
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
    }
}

// Called by all 32 lanes of the warp; stg: its staging buffer (1024-aligned).
template <class Spec>
__device__ __forceinline__ void tc_epilogue(float (&acc)[128], const TcArgs& g, i64 bi, i64 i0, i64 n0,
                                            typename Spec::Out* out, u32 stg, int lane) {
    using namespace tc;
    typedef typename Spec::Out Out;
    const i64 i = i0 + lane;
    if constexpr (sizeof(Out) > 4) {
        // 8-byte results: apply and store per element group
        if (i < g.M) {
            Out* row = out + bi * g.o_bstride + i * g.N + n0;
#pragma unroll
            for (int v = 0; v < 128; v += 4) {
                if (n0 + v < g.N) {
                    Vec4<Out> o;
#pragma unroll
                    for (int e = 0; e < 4; ++e) o.v[e] = Spec::apply(acc[v + e], g, bi, i, n0 + v + e);
                    st4(row + v, o);
                }
            }
        }
        return;
    } else {
        // pass 1 (N % 4 == 0: a 4-column group is in range or not at all)
        if (i < g.M) {
            if (g.ep_vec) {
#pragma unroll
                for (int v = 0; v < 128; v += 4) {
                    if (n0 + v < g.N) {
                        Vec4<Out> o;
                        Spec::apply4(acc + v, g, bi, i, n0 + v, o);
#pragma unroll
                        for (int e = 0; e < 4; ++e) acc[v + e] = tc_pack_bits(o.v[e]);
                    }
                }
            } else {
#pragma unroll
                for (int v = 0; v < 128; v += 4) {
                    if (n0 + v < g.N) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) acc[v + e] = tc_pack_bits(Spec::apply(acc[v + e], g, bi, i, n0 + v + e));
                    }
                }
            }
        }
        // pass 2
        if (g.out_tma) {
            tc_store_rows<Out, true>(acc, &g.tmap_out, n0, i0, bi, g.N, stg, lane);
        } else if (i < g.M) {
            Out* row = out + bi * g.o_bstride + i * g.N + n0;
#pragma unroll
            for (int v = 0; v < 128; v += 4) {
                if (n0 + v < g.N) {
                    Vec4<Out> o;
#pragma unroll
                    for (int e = 0; e < 4; ++e) o.v[e] = tc_unpack_bits<Out>(acc[v + e]);
                    st4(row + v, o);
                }
            }
        }
    }
}
// Before the CTA exits or its staging is reused by another kernel role:
// the warp's bulk stores have completed.
__device__ __forceinline__ void tc_epilogue_flush(int lane) {
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// K slices: lane r's row i0 + r, columns n0 .. n0+127, of the fp32 sums a
// previous slice left in `out` (16-byte loads; N % 4 == 0 keeps the rows
// 16-byte aligned), rows >= M and columns >= N read as 0.
__device__ __forceinline__ void tc_load_sums(float (&acc)[128], const TcArgs& g, i64 bi, i64 i0, i64 n0, int lane) {
    const i64 i = i0 + lane;
    if (i >= g.M) return;
    const float* row = reinterpret_cast<const float*>(g.out) + bi * g.o_bstride + i * g.N + n0;
#pragma unroll
    for (int v = 0; v < 128; v += 4) {
        if (n0 + v < g.N) {
            const float4 x = *reinterpret_cast<const float4*>(row + v);
            acc[v] = x.x; acc[v + 1] = x.y; acc[v + 2] = x.z; acc[v + 3] = x.w;
        }
    }
}
// ... and the sums stored back unchanged (no epilogue) for the next slice:
// through the output's TMA map (kept in L2: the next slice reads them), or
// plain 16-byte stores.
__device__ __forceinline__ void tc_store_sums(const float (&acc)[128], const TcArgs& g, i64 bi, i64 i0, i64 n0,
                                              u32 stg, int lane) {
    if (g.out_tma) {
        tc_store_rows<float, false>(acc, &g.tmap_out, n0, i0, bi, g.N, stg, lane);
        return;
    }
    const i64 i = i0 + lane;
    if (i >= g.M) return;
    float* row = reinterpret_cast<float*>(g.out) + bi * g.o_bstride + i * g.N + n0;
#pragma unroll
    for (int v = 0; v < 128; v += 4)
        if (n0 + v < g.N) *reinterpret_cast<float4*>(row + v) = make_float4(acc[v], acc[v + 1], acc[v + 2], acc[v + 3]);
}

// Split tail tiles: out = epi(sum of the K-range partials in ws, in part
// order), 4 columns per thread (N % 4 == 0), rows of TILE_M-row tiles.
template <class Spec, int TILE_M>
__device__ __forceinline__ void gemm_tc_fixup(const TcArgs& g) {
    typedef typename Spec::Out Out;
    const i64 per_tile = (i64)TILE_M * 64;           // 4-column groups of a tile
    const i64 part_elems = (i64)TILE_M * 256;
    const i64 total = (i64)(g.num_tiles - g.split_first) * per_tile;
    Out* out = reinterpret_cast<Out*>(g.out);
    for (i64 x = (i64)blockIdx.x * blockDim.x + threadIdx.x; x < total; x += (i64)gridDim.x * blockDim.x) {
        const int tl = (int)(x / per_tile);
        const int r = (int)(x % per_tile / 64), c = (int)(x % 64) * 4;
        int mb, nb, bi;
        tc::tile_coords(g, g.split_first + tl, mb, nb, bi);
        const i64 i = (i64)mb * TILE_M + r, j = (i64)nb * 256 + c;
        if (i >= g.M || j >= g.N) continue;
        const float* p = g.ws + (i64)tl * g.split * part_elems + (i64)r * 256 + c;
        float4 sum = __ldcs(reinterpret_cast<const float4*>(p));
        for (int q = 1; q < g.split; ++q) {
            const float4 v = __ldcs(reinterpret_cast<const float4*>(p + q * part_elems));
            sum.x = __fadd_rn(sum.x, v.x);
            sum.y = __fadd_rn(sum.y, v.y);
            sum.z = __fadd_rn(sum.z, v.z);
            sum.w = __fadd_rn(sum.w, v.w);
        }
        const float a[4] = {sum.x, sum.y, sum.z, sum.w};
        Vec4<Out> o;
        if (g.ep_vec) {
            Spec::apply4(a, g, bi, i, j, o);
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) o.v[e] = Spec::apply(a[e], g, bi, i, j + e);
        }
        st4(out + bi * g.o_bstride + i * g.N + j, o);
    }
}

// Operand element types.  A k-block is one 128-byte swizzle row of K: 32
// tf32 or 64 bf16 elements; an MMA consumes 32 bytes of K (8 tf32 under
// kind::tf32, 16 bf16 under kind::f16), four MMAs per k-block, so stage
// sizes and K-major descriptors are the same in bytes.  MN-major tiles
// differ: tf32 needs the 128B swizzle with 32-byte atoms (32 elements per
// row, 4-row K groups), bf16 uses the plain 128B swizzle (64 elements per
// row, 8-row K groups).
struct ElemTf32 {
    static constexpr int BYTES = 4, BKE = 32;       // elements per k-block
    static constexpr u32 FMT = 2u;                   // instruction-descriptor a/b format
    static constexpr int MN_ATOM = 32;               // MN elements per swizzle row
    static constexpr u32 MN_LT = 1u, MN_SBO = 512u, MN_KK = 1024u;   // layout, K-group stride, per-MMA advance
    static constexpr int KB_CHUNK = 0;               // promotion chunk: the config's
    __device__ static __forceinline__ void mma(u32 d, u64 a, u64 b, u32 idesc, u32 acc) { tc::tc_mma_tf32(d, a, b, idesc, acc); }
    __device__ static __forceinline__ void mma_pair(u32 d, u64 a, u64 b, u32 idesc, u32 acc) { tc::tc_mma_tf32_pair(d, a, b, idesc, acc); }
};
struct ElemBf16 {
    static constexpr int BYTES = 2, BKE = 64;
    static constexpr u32 FMT = 1u;
    static constexpr int MN_ATOM = 64;
    static constexpr u32 MN_LT = 2u, MN_SBO = 1024u, MN_KK = 2048u;
    // Products are exact; the accumulator truncates toward zero at each
    // MMA, a bias that grows with the chunk.  Each promotion moves the
    // tile's partial sums out of TMEM and adds them on the CUDA cores,
    // which under the 1 kW power cap costs throughput.  Measured on one
    // B200 (16384^3 TFLOP/s; share of 512x512x16384 results bit-identical
    // to the exact kernel): every 512 k 965 / 99.975 %, every 2048 k 1083 /
    // 99.929 %, every 4096 k 1153 / 99.860 %.  2048 k keeps > 99.9 %.
    static constexpr int KB_CHUNK = 32;
    __device__ static __forceinline__ void mma(u32 d, u64 a, u64 b, u32 idesc, u32 acc) { tc::tc_mma_f16kind(d, a, b, idesc, acc); }
    __device__ static __forceinline__ void mma_pair(u32 d, u64 a, u64 b, u32 idesc, u32 acc) { tc::tc_mma_f16kind_pair(d, a, b, idesc, acc); }
};

template <class Spec, int VARIANT, class E = ElemTf32, bool CONVERT = false>
__device__ __forceinline__ void gemm_tc(const TcArgs& g) {
    using namespace tc;
    typedef TcCfg<VARIANT> Cfg;
    constexpr int BN = Cfg::BN, STAGES = Cfg::STAGES;
    constexpr bool SPLIT = VARIANT == 3;
    constexpr bool CONV = SPLIT && CONVERT;          // residuals made in shared memory
    static_assert(!SPLIT || E::BYTES == 4, "the 3-product split is for fp32 operands");
    constexpr int KB_PER_CHUNK = E::KB_CHUNK ? E::KB_CHUNK : Cfg::KB_PER_CHUNK;
    // the conversion look-ahead (one chunk) must fit in the stage ring, or
    // the converters wait on loads that wait on MMAs that wait on them
    static_assert(!CONV || KB_PER_CHUNK <= STAGES, "conversion look-ahead exceeds the stages");
    constexpr int BKE = E::BKE;                      // elements per k-block
    constexpr u32 MN_BOX = BKE * 128u;              // one MN-major box: a k-block of 128-byte rows
    constexpr u32 A_BYTES = BM * BK * 4;            // 16 KB (128 rows x 128 B)
    constexpr u32 B_BYTES = BN * BK * 4;            // 32 KB
    constexpr u32 STAGE_BYTES = (A_BYTES + B_BYTES) * (SPLIT ? 2 : 1);
    constexpr u32 TMEM_COLS = 2 * BN;
    constexpr int ACC_THREADS = 256;

    extern __shared__ unsigned char smem_raw[];
    // 1024-byte aligned stage ring (the swizzle pattern is address based)
    const u32 raw_addr = smem_u32(smem_raw);
    const u32 base = (raw_addr + 1023u) & ~1023u;
    unsigned char* smem = smem_raw + (base - raw_addr);
    const u32 bars = base + STAGES * STAGE_BYTES;   // mbarriers follow the ring
    // barrier layout: full[S], empty[S], tfull[2], tempty[2], drain
    auto FULL = [&](int s) { return bars + 8u * s; };
    auto EMPTY = [&](int s) { return bars + 8u * (STAGES + s); };
    auto TFULL = [&](int b) { return bars + 8u * (2 * STAGES + b); };
    auto TEMPTY = [&](int b) { return bars + 8u * (2 * STAGES + 2 + b); };
    const u32 DRAIN = bars + 8u * (2 * STAGES + 4);
    auto LO = [&](int s) { return bars + 8u * (2 * STAGES + 5 + s); };   // residuals of stage s ready
    volatile Shared* sh = reinterpret_cast<volatile Shared*>(smem + STAGES * STAGE_BYTES + 8 * (3 * STAGES + 5));
    static_assert(8 * (3 * STAGES + 5) + sizeof(Shared) <= EPI_OFFSET, "mbarriers overlap the epilogue staging");

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(FULL(s), 1);
            mbar_init(EMPTY(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(TFULL(b), 1);
            mbar_init(TEMPTY(b), ACC_THREADS);
        }
        mbar_init(DRAIN, 1);
        for (int s = 0; s < STAGES; ++s) mbar_init(LO(s), ACC_THREADS);
        sh->abort = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32((const void*)&sh->tmem_base)), "r"(TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const u32 tmem = sh->tmem_base;
    const int k_blocks = (int)((g.K + BKE - 1) / BKE);
    const int n_chunks = (k_blocks + KB_PER_CHUNK - 1) / KB_PER_CHUNK;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer --
        if (lane == 0) {
            int s = 0;
            u32 phase = 0;
            u32 armed[STAGES];
            for (int i = 0; i < STAGES; ++i) armed[i] = 0xFFFFFFFFu;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < g.num_units; u += gridDim.x) {
                int t, c0, c1, part;
                unit_range(g, u, n_chunks, t, c0, c1, part);
                int mb, nb, bi;
                tile_coords(g, t, mb, nb, bi);
                const int m0 = mb * BM, n0 = nb * BN;
                const int kb_stop = c1 * KB_PER_CHUNK < k_blocks ? c1 * KB_PER_CHUNK : k_blocks;
                // Every operand map is 3-D (batch extent 1 when the operand
                // is shared): the batch coordinate is fixed per tile, so the
                // k-loop issues one load form without a branch.
                const int za = g.a_batched ? bi : 0, zb = g.b_batched ? bi : 0;
                auto load_a = [&](u32 dst, const TmaDesc* m, u32 bar, int x, int y) { tma_load_3d(dst, m, bar, x, y, za); };
                auto load_b = [&](u32 dst, const TmaDesc* m, u32 bar, int x, int y) { tma_load_3d(dst, m, bar, x, y, zb); };
                for (int kb = c0 * KB_PER_CHUNK; kb < kb_stop; ++kb) {
                    if (!wait(EMPTY(s), phase ^ 1u, sh, g, 1u)) { ok = false; break; }
                    const u32 a_dst = base + s * STAGE_BYTES;
                    const u32 b_dst = a_dst + A_BYTES;
                    mbar_expect_tx(FULL(s), CONV ? A_BYTES + B_BYTES : STAGE_BYTES);
                    armed[s] = phase;
                    const int k0 = kb * BKE;
#pragma unroll
                    for (int part = 0; part < (SPLIT && !CONV ? 2 : 1); ++part) {
                        const TmaDesc* ma = part ? &g.tmap_a_lo : &g.tmap_a;
                        const TmaDesc* mbp = part ? &g.tmap_b_lo : &g.tmap_b;
                        const u32 ad = a_dst + part * (A_BYTES + B_BYTES);
                        const u32 bd = b_dst + part * (A_BYTES + B_BYTES);
                        if (g.a_mn) {
                            for (int j = 0; j < BM / E::MN_ATOM; ++j)
                                load_a(ad + j * MN_BOX, ma, FULL(s), m0 + E::MN_ATOM * j, k0);
                        } else {
                            load_a(ad, ma, FULL(s), k0, m0);
                        }
                        if (g.b_mn) {
                            for (int j = 0; j < BN / E::MN_ATOM; ++j)
                                load_b(bd + j * MN_BOX, mbp, FULL(s), n0 + E::MN_ATOM * j, k0);
                        } else {
                            load_b(bd, mbp, FULL(s), k0, n0);
                        }
                    }
                    if (++s == STAGES) { s = 0; phase ^= 1u; }
                }
            }
            // Drain: wait for every copy this thread issued (bounded).
            for (int i = 0; i < STAGES; ++i) {
                if (armed[i] == 0xFFFFFFFFu) continue;
                const u64 t0 = now_ns();
                while (!mbar_try(FULL(i), armed[i]) && now_ns() - t0 < drain_ns(g)) {}
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------- MMA issuer --
        if (lane == 0) {
            const u32 idesc = instr_desc(g.a_mn, g.b_mn, BN, BM, E::FMT);
            const u32 a_lbo = g.a_mn ? MN_BOX : 16u, b_lbo = g.b_mn ? MN_BOX : 16u;
            const u32 a_sbo = g.a_mn ? E::MN_SBO : 1024u, b_sbo = g.b_mn ? E::MN_SBO : 1024u;
            const u32 a_lt = g.a_mn ? E::MN_LT : 2u, b_lt = g.b_mn ? E::MN_LT : 2u;
            int s = 0;
            u32 phase = 0;
            u32 chunk = 0;                              // chunks issued by this CTA
            bool ok = true;
            for (int u = blockIdx.x; ok && u < g.num_units; u += gridDim.x) {
                int t, c0, c1, part;
                unit_range(g, u, n_chunks, t, c0, c1, part);
                for (int c = c0; ok && c < c1; ++c, ++chunk) {
                    const int buf = (int)(chunk & 1u);
                    const u32 use = (chunk >> 1) & 1u;
                    if (!wait(TEMPTY(buf), use ^ 1u, sh, g, 2u)) { ok = false; break; }
                    tc_fence_after();
                    const u32 d = tmem + (u32)(buf * BN);
                    const int kb_end = (c + 1) * KB_PER_CHUNK < k_blocks ? (c + 1) * KB_PER_CHUNK : k_blocks;
                    for (int kb = c * KB_PER_CHUNK; kb < kb_end; ++kb) {
                        if (!wait(CONV ? LO(s) : FULL(s), phase, sh, g, 3u)) { ok = false; break; }
                        tc_fence_after();
                        const u32 a_hi = base + s * STAGE_BYTES;
                        const u32 b_hi = a_hi + A_BYTES;
                        const u32 a_lo = a_hi + A_BYTES + B_BYTES;
                        const u32 b_lo = a_lo + A_BYTES;
                        // 3xTF32: the k-block's eight cross-term MMAs (hi.lo,
                        // lo.hi) go first, then its four hi.hi MMAs, so the
                        // small terms are summed while the accumulator is
                        // small (its additions truncate: fewer full-size
                        // truncations per chunk; measured rms error -25 %).
                        // K-major: 32 B further along the row; MN-major:
                        // the next 8 (tf32) / 16 (bf16) k-rows.
                        if (SPLIT) {
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk) {
                                const u32 ao = g.a_mn ? kk * E::MN_KK : kk * 32u;
                                const u32 bo = g.b_mn ? kk * E::MN_KK : kk * 32u;
                                const u32 acc = (kb > c * KB_PER_CHUNK || kk > 0) ? 1u : 0u;
                                E::mma(d, smem_desc(a_hi + ao, a_lbo, a_sbo, a_lt),
                                       smem_desc(b_lo + bo, b_lbo, b_sbo, b_lt), idesc, acc);
                                E::mma(d, smem_desc(a_lo + ao, a_lbo, a_sbo, a_lt),
                                       smem_desc(b_hi + bo, b_lbo, b_sbo, b_lt), idesc, 1u);
                            }
                        }
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {
                            const u32 ao = g.a_mn ? kk * E::MN_KK : kk * 32u;
                            const u32 bo = g.b_mn ? kk * E::MN_KK : kk * 32u;
                            const u32 acc = (SPLIT || kb > c * KB_PER_CHUNK || kk > 0) ? 1u : 0u;
                            E::mma(d, smem_desc(a_hi + ao, a_lbo, a_sbo, a_lt), smem_desc(b_hi + bo, b_lbo, b_sbo, b_lt),
                                   idesc, acc);
                        }
                        tc_commit(EMPTY(s));           // stage free once these MMAs finish
                        if (++s == STAGES) { s = 0; phase ^= 1u; }
                    }
                    if (!ok) break;
                    tc_commit(TFULL(buf));             // chunk partial sums ready
                }
            }
            // Drain outstanding MMAs before TMEM is released (bounded).
            tc_commit(DRAIN);
            const u64 t0 = now_ns();
            while (!mbar_try(DRAIN, 0u) && now_ns() - t0 < drain_ns(g)) {}
        }
    } else {
        // ------------------------------------ accumulate + epilogue --
        const int q = warp & 3;                        // TMEM lane quadrant
        const int half = (warp - 2) >> 2;              // column half of the tile
        const u32 lane_addr = (u32)(q * 32) << 16;
        typename Spec::Out* out = reinterpret_cast<typename Spec::Out*>(g.out);
        const u32 stg = base + STAGES * STAGE_BYTES + EPI_OFFSET + (u32)(warp - 2) * EPI_WARP_BYTES;
        u32 chunk = 0;
        bool ok = true;
        // 3xTF32 with converted residuals: these threads also write the tf32
        // residuals of every stage (each its 1/256 share), one
        // TMEM chunk ahead of the drain they wait for, and release it on the
        // MMA issuer through LO(s).
        // conv counts converted k-blocks from the current tile's first; the
        // look-ahead may run into the next tiles but never past this CTA's
        // last k-block, nor more than KB_PER_CHUNK <= STAGES k-blocks beyond
        // the chunk being drained (so producer, converters and MMA issuer
        // never wait on one another in a circle).
        const int at = threadIdx.x - 64;
        int conv = 0, cs = 0;
        u32 cph = 0;
        auto convert_until = [&](int target) -> bool {
            if constexpr (CONV) {
                while (conv < target) {
                    if (!wait(FULL(cs), cph, sh, g, 5u)) return false;
                    const u32 hi = base + cs * STAGE_BYTES;
                    convert_stage<(A_BYTES + B_BYTES) / 16 / ACC_THREADS, ACC_THREADS, A_BYTES / 16 / ACC_THREADS>(
                        hi, hi + A_BYTES + B_BYTES, at);
                    fence_async_smem();                    // visible to the tensor core
                        mbar_arrive(LO(cs));
                    if (++cs == STAGES) { cs = 0; cph ^= 1u; }
                    ++conv;
                }
            }
            return true;
        };
        for (int u = blockIdx.x; ok && u < g.num_units; u += gridDim.x) {
            int t, c0, c1, part;
            unit_range(g, u, n_chunks, t, c0, c1, part);
            // k-blocks this CTA still has after the current tile, capped
            // (with converted residuals the tiles are never split: u == t)
            const long long after = (long long)(g.num_units - 1 - u) / (int)gridDim.x * k_blocks;
            const int limit = k_blocks + (after < KB_PER_CHUNK ? (int)after : KB_PER_CHUNK);
            float acc[128];
#pragma unroll
            for (int e = 0; e < 128; ++e) acc[e] = 0.0f;
            for (int c = c0; c < c1; ++c, ++chunk) {
                const int buf = (int)(chunk & 1u);
                const u32 use = (chunk >> 1) & 1u;
                const int c_end = (c + 1) * KB_PER_CHUNK < k_blocks ? (c + 1) * KB_PER_CHUNK : k_blocks;
                const bool conv_ok = convert_until(c_end + KB_PER_CHUNK < limit ? c_end + KB_PER_CHUNK : limit);
                // warp-uniform: tcgen05.ld below needs all 32 lanes converged
                const bool ready = conv_ok && wait(TFULL(buf), use, sh, g, 4u);
                if (!__all_sync(0xFFFFFFFFu, ready)) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    u32 r[32];
                    tmem_ld32(tmem + lane_addr + (u32)(buf * BN + half * 128 + 32 * j), r);
#pragma unroll
                    for (int e = 0; e < 32; e += 2) fadd2_rn(acc[32 * j + e], acc[32 * j + e + 1], r[e], r[e + 1]);
                }
                tc_fence_before();
                mbar_arrive(TEMPTY(buf));
            }
            if (!ok) break;
            if (CONV) conv -= k_blocks;                // counted from the next tile's first k-block
            int mb, nb, bi;
            tile_coords(g, t, mb, nb, bi);
            const i64 i0 = (i64)mb * BM + q * 32;
            const i64 n0 = (i64)nb * BN + half * 128;
            if (part < 0) tc_epilogue<Spec>(acc, g, bi, i0, n0, out, stg, lane);
            else tc_store_rows<float, false>(acc, &g.tmap_ws, half * 128, ((i64)(t - g.split_first) * g.split + part) * BM + q * 32,
                                             0, 256, stg, lane);
        }
        tc_epilogue_flush(lane);
    }

    // ------------------------------------------------------- teardown --
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}


// CTA-pair (cta_group::2) variant.  A cluster of two CTAs on two SMs
// computes a 256 x 256 output tile: CTA r owns rows [128r, 128r+128) of the
// tile (its A tile and TMEM accumulator) and stages columns [128r, 128r+128)
// of B; one tcgen05.mma.cta_group::2 (M=256, N=256, K=8) issued by the
// leader (CTA 0) reads A from each CTA's shared memory and both halves of B,
// so per SM a k-block moves 32 KB (1xTF32) instead of 48 KB.  Both CTAs'
// TMA loads complete on the leader's FULL barrier; MMA completion is
// committed to the barriers of both CTAs; the accumulate warps of both
// CTAs release a TMEM chunk buffer by arriving on the leader's barrier.
// Roles, chunked register accumulation, bounded waits as in gemm_tc.
template <class Spec, int VARIANT, class E = ElemTf32, bool CONVERT = false>
__device__ __forceinline__ void gemm_tc_pair(const TcArgs& g) {
    using namespace tc;
    typedef TcPairCfg<VARIANT> Cfg;
    constexpr int BN = 256, STAGES = Cfg::STAGES;
    constexpr bool SPLIT = VARIANT == 3;
    constexpr bool CONV = SPLIT && CONVERT;          // residuals made in shared memory
    static_assert(!SPLIT || E::BYTES == 4, "the 3-product split is for fp32 operands");
    constexpr int KB_PER_CHUNK = E::KB_CHUNK ? E::KB_CHUNK : Cfg::KB_PER_CHUNK;
    // the conversion look-ahead (one chunk) must fit in the stage ring, or
    // the converters wait on loads that wait on MMAs that wait on them
    static_assert(!CONV || KB_PER_CHUNK <= STAGES, "conversion look-ahead exceeds the stages");
    constexpr int BKE = E::BKE;
    constexpr u32 MN_BOX = BKE * 128u;
    constexpr u32 A_BYTES = BM * BK * 4;            // 16 KB: this CTA's 128 rows
    constexpr u32 B_BYTES = (BN / 2) * BK * 4;      // 16 KB: this CTA's half of B
    constexpr u32 STAGE_BYTES = (A_BYTES + B_BYTES) * (SPLIT ? 2 : 1);
    constexpr u32 TMEM_COLS = 2 * BN;
    constexpr int ACC_THREADS = 256;

    extern __shared__ unsigned char smem_raw[];
    const u32 raw_addr = smem_u32(smem_raw);
    const u32 base = (raw_addr + 1023u) & ~1023u;
    unsigned char* smem = smem_raw + (base - raw_addr);
    const u32 bars = base + STAGES * STAGE_BYTES;
    auto FULL = [&](int s) { return bars + 8u * s; };
    auto EMPTY = [&](int s) { return bars + 8u * (STAGES + s); };
    auto TFULL = [&](int b) { return bars + 8u * (2 * STAGES + b); };
    auto TEMPTY = [&](int b) { return bars + 8u * (2 * STAGES + 2 + b); };
    const u32 DRAIN = bars + 8u * (2 * STAGES + 4);
    auto LO = [&](int s) { return bars + 8u * (2 * STAGES + 5 + s); };   // residuals of stage s ready
    volatile Shared* sh = reinterpret_cast<volatile Shared*>(smem + STAGES * STAGE_BYTES + 8 * (3 * STAGES + 5));
    static_assert(8 * (3 * STAGES + 5) + sizeof(Shared) <= EPI_OFFSET, "mbarriers overlap the epilogue staging");

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const u32 cta = cluster_rank();
    const int pair = (int)(blockIdx.x >> 1);
    const int num_pairs = (int)(gridDim.x >> 1);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(FULL(s), 1);
            mbar_init(EMPTY(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(TFULL(b), 1);
            mbar_init(TEMPTY(b), 2 * ACC_THREADS);
        }
        mbar_init(DRAIN, 1);
        for (int s = 0; s < STAGES; ++s) mbar_init(LO(s), 2 * ACC_THREADS);   // both CTAs' converting threads
        sh->abort = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32((const void*)&sh->tmem_base)), "r"(TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();                                  // both CTAs' barriers exist
    tc_fence_after();
    const u32 tmem = sh->tmem_base;
    const int k_blocks = (int)((g.K + BKE - 1) / BKE);
    // this launch's K slice: k-blocks [kb_first, kb_hi), chunks from c_first
    const int kb_hi = g.kb_last > 0 && g.kb_last < k_blocks ? g.kb_last : k_blocks;   // 0: all
    const int c_first = g.kb_first / KB_PER_CHUNK;
    const int n_chunks = (kb_hi + KB_PER_CHUNK - 1) / KB_PER_CHUNK - c_first;
    auto unit_chunks = [&](int u, int& t, int& c0, int& c1, int& part) {
        unit_range(g, u, n_chunks, t, c0, c1, part);
        c0 += c_first;
        c1 += c_first;
    };

    if (warp == 0) {
        // ---------------------------------------- TMA producer (both CTAs) --
        if (lane == 0) {
            int s = 0;
            u32 phase = 0;
            u32 armed[STAGES];
            for (int i = 0; i < STAGES; ++i) armed[i] = 0xFFFFFFFFu;
            bool ok = true;
            bool align_on = true;
            for (int u = pair; ok && u < g.num_units; u += num_pairs) {
                int t, c0, c1, part;
                unit_chunks(u, t, c0, c1, part);
                int mb, nb, bi;
                tile_coords(g, t, mb, nb, bi);
                const int m0 = mb * 2 * BM + (int)cta * BM, n0 = nb * BN + (int)cta * (BN / 2);
                const int kb_stop = c1 * KB_PER_CHUNK < kb_hi ? c1 * KB_PER_CHUNK : kb_hi;
                const int za = g.a_batched ? bi : 0, zb = g.b_batched ? bi : 0;
                // Wave alignment (advisory): the leader's producer starts the
                // loads of wave w once every pair has issued all of wave
                // w-1's, so the pairs of a wave walk K together and share the
                // operand panels' slices in L2 instead of re-reading them
                // from HBM as they drift apart.  The wait is bounded (100 us;
                // aligned pairs stay microseconds apart, and a pair that is not
                // resident -- other kernels holding SMs -- costs one such wait);
                // when it runs out this CTA stops aligning (results do not
                // depend on it).
                const bool aligned = g.wave_ctr && cta == 0 && u < g.split_first;
                if (aligned && align_on && u >= num_pairs) {
                    const unsigned need = (unsigned)(u - pair);   // pairs x waves before this one
                    const u64 t0 = now_ns();
                    for (;;) {
                        unsigned v;
                        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(g.wave_ctr) : "memory");
                        if (v >= need) break;
                        if (now_ns() - t0 > 100000ull) { align_on = false; break; }
                        __nanosleep(256);
                    }
                }
                // With converted residuals each CTA's copies complete on its
                // own FULL barrier (its converting threads wait there);
                // otherwise on the leader's, which the MMA issuer waits on.
                auto load_a = [&](u32 dst, const TmaDesc* m, u32 bar, int x, int y) {
                    if (CONV) tma_load_3d(dst, m, bar, x, y, za);
                    else tma_load_3d_pair(dst, m, bar, x, y, za);
                };
                auto load_b = [&](u32 dst, const TmaDesc* m, u32 bar, int x, int y) {
                    if (CONV) tma_load_3d(dst, m, bar, x, y, zb);
                    else tma_load_3d_pair(dst, m, bar, x, y, zb);
                };
                for (int kb = c0 * KB_PER_CHUNK; kb < kb_stop; ++kb) {
                    if (!wait(EMPTY(s), phase ^ 1u, sh, g, 1u)) { ok = false; break; }
                    const u32 a_dst = base + s * STAGE_BYTES;
                    const u32 b_dst = a_dst + A_BYTES;
                    if (CONV) {
                        mbar_expect_tx(FULL(s), A_BYTES + B_BYTES);   // this CTA's raw operands
                        armed[s] = phase;
                    } else if (cta == 0) {
                        mbar_expect_tx(FULL(s), 2 * STAGE_BYTES);     // both CTAs' bytes
                        armed[s] = phase;
                    }
                    const int k0 = kb * BKE;
#pragma unroll
                    for (int part = 0; part < (SPLIT && !CONV ? 2 : 1); ++part) {
                        const TmaDesc* ma = part ? &g.tmap_a_lo : &g.tmap_a;
                        const TmaDesc* mbp = part ? &g.tmap_b_lo : &g.tmap_b;
                        const u32 ad = a_dst + part * (A_BYTES + B_BYTES);
                        const u32 bd = b_dst + part * (A_BYTES + B_BYTES);
                        if (g.a_mn) {
                            for (int j = 0; j < BM / E::MN_ATOM; ++j)
                                load_a(ad + j * MN_BOX, ma, FULL(s), m0 + E::MN_ATOM * j, k0);
                        } else {
                            load_a(ad, ma, FULL(s), k0, m0);
                        }
                        if (g.b_mn) {
                            for (int j = 0; j < (BN / 2) / E::MN_ATOM; ++j)
                                load_b(bd + j * MN_BOX, mbp, FULL(s), n0 + E::MN_ATOM * j, k0);
                        } else {
                            load_b(bd, mbp, FULL(s), k0, n0);
                        }
                    }
                    if (++s == STAGES) { s = 0; phase ^= 1u; }
                }
                if (aligned && ok) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(g.wave_ctr) : "memory");
            }
            // Drain (bounded): wait for the copies on this CTA's armed FULL
            // phases (the leader's count both CTAs' copies unless converting).
            for (int i = 0; i < STAGES; ++i) {
                const u64 t0 = now_ns();
                if (CONV || cta == 0) {
                    if (armed[i] == 0xFFFFFFFFu) continue;
                    while (!mbar_try(FULL(i), armed[i]) && now_ns() - t0 < drain_ns(g)) {}
                }
            }
        }
    } else if (warp == 1) {
        // --------------------------------------- MMA issuer (leader CTA) --
        if (lane == 0 && cta == 0) {
            const u32 idesc = instr_desc(g.a_mn, g.b_mn, BN, 2 * BM, E::FMT);
            const u32 a_lbo = g.a_mn ? MN_BOX : 16u, b_lbo = g.b_mn ? MN_BOX : 16u;
            const u32 a_sbo = g.a_mn ? E::MN_SBO : 1024u, b_sbo = g.b_mn ? E::MN_SBO : 1024u;
            const u32 a_lt = g.a_mn ? E::MN_LT : 2u, b_lt = g.b_mn ? E::MN_LT : 2u;
            int s = 0;
            u32 phase = 0;
            u32 chunk = 0;
            bool ok = true;
            for (int u = pair; ok && u < g.num_units; u += num_pairs) {
                int t, c0, c1, part;
                unit_chunks(u, t, c0, c1, part);
                for (int c = c0; ok && c < c1; ++c, ++chunk) {
                    const int buf = (int)(chunk & 1u);
                    const u32 use = (chunk >> 1) & 1u;
                    if (!wait(TEMPTY(buf), use ^ 1u, sh, g, 2u)) { ok = false; break; }
                    tc_fence_after();
                    const u32 d = tmem + (u32)(buf * BN);
                    const int kb_end = (c + 1) * KB_PER_CHUNK < kb_hi ? (c + 1) * KB_PER_CHUNK : kb_hi;
                    for (int kb = c * KB_PER_CHUNK; kb < kb_end; ++kb) {
                        const bool ready = CONV ? wait_cluster(LO(s), phase, sh, g, 3u) : wait(FULL(s), phase, sh, g, 3u);
                        if (!ready) { ok = false; break; }
                        tc_fence_after();
                        const u32 a_hi = base + s * STAGE_BYTES;
                        const u32 b_hi = a_hi + A_BYTES;
                        const u32 a_lo = a_hi + A_BYTES + B_BYTES;
                        const u32 b_lo = a_lo + A_BYTES;
                        // 3xTF32: cross terms first, then hi.hi (see gemm_tc)
                        if (SPLIT) {
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk) {
                                const u32 ao = g.a_mn ? kk * E::MN_KK : kk * 32u;
                                const u32 bo = g.b_mn ? kk * E::MN_KK : kk * 32u;
                                const u32 acc = (kb > c * KB_PER_CHUNK || kk > 0) ? 1u : 0u;
                                E::mma_pair(d, smem_desc(a_hi + ao, a_lbo, a_sbo, a_lt),
                                            smem_desc(b_lo + bo, b_lbo, b_sbo, b_lt), idesc, acc);
                                E::mma_pair(d, smem_desc(a_lo + ao, a_lbo, a_sbo, a_lt),
                                            smem_desc(b_hi + bo, b_lbo, b_sbo, b_lt), idesc, 1u);
                            }
                        }
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {
                            const u32 ao = g.a_mn ? kk * E::MN_KK : kk * 32u;
                            const u32 bo = g.b_mn ? kk * E::MN_KK : kk * 32u;
                            const u32 acc = (SPLIT || kb > c * KB_PER_CHUNK || kk > 0) ? 1u : 0u;
                            E::mma_pair(d, smem_desc(a_hi + ao, a_lbo, a_sbo, a_lt),
                                        smem_desc(b_hi + bo, b_lbo, b_sbo, b_lt), idesc, acc);
                        }
                        tc_commit_pair(EMPTY(s));      // both CTAs' stage s is free
                        if (++s == STAGES) { s = 0; phase ^= 1u; }
                    }
                    if (!ok) break;
                    tc_commit_pair(TFULL(buf));        // both CTAs' partial sums ready
                }
            }
            tc_commit_pair(DRAIN);
            const u64 t0 = now_ns();
            while (!mbar_try(DRAIN, 0u) && now_ns() - t0 < drain_ns(g)) {}
        }
    } else {
        // ------------------------- accumulate + epilogue (both CTAs) --
        const int q = warp & 3;
        const int half = (warp - 2) >> 2;
        const u32 lane_addr = (u32)(q * 32) << 16;
        typename Spec::Out* out = reinterpret_cast<typename Spec::Out*>(g.out);
        const u32 stg = base + STAGES * STAGE_BYTES + EPI_OFFSET + (u32)(warp - 2) * EPI_WARP_BYTES;
        u32 chunk = 0;
        bool ok = true;
        // 3xTF32 with converted residuals: these threads also write the tf32
        // residuals of every stage of their CTA (each its 1/256 share), one
        // TMEM chunk ahead of the drain they wait for, and release it on the
        // leader's LO(s) (the MMA reads both CTAs' stages).
        // conv counts converted k-blocks from the current tile's first; the
        // look-ahead may run into the next tiles but never past this CTA's
        // last k-block, nor more than KB_PER_CHUNK <= STAGES k-blocks beyond
        // the chunk being drained (so producer, converters and MMA issuer
        // never wait on one another in a circle).
        const int at = threadIdx.x - 64;
        int conv = 0, cs = 0;
        u32 cph = 0;
        auto convert_until = [&](int target) -> bool {
            if constexpr (CONV) {
                while (conv < target) {
                    if (!wait(FULL(cs), cph, sh, g, 5u)) return false;
                    const u32 hi = base + cs * STAGE_BYTES;
                    convert_stage<(A_BYTES + B_BYTES) / 16 / ACC_THREADS, ACC_THREADS, A_BYTES / 16 / ACC_THREADS>(
                        hi, hi + A_BYTES + B_BYTES, at);
                    fence_async_smem();                    // visible to the tensor core
                        if (cta == 0) mbar_arrive(LO(cs));
                        else mbar_arrive_cluster(LO(cs), 0u);
                    if (++cs == STAGES) { cs = 0; cph ^= 1u; }
                    ++conv;
                }
            }
            return true;
        };
        for (int u = pair; ok && u < g.num_units; u += num_pairs) {
            int t, c0, c1, part;
            unit_chunks(u, t, c0, c1, part);
            // k-blocks this CTA still has after the current tile, capped
            // (with converted residuals the tiles are never split: u == t,
            // and never sliced: the launch covers all k-blocks)
            const long long after = (long long)(g.num_units - 1 - u) / num_pairs * k_blocks;
            const int limit = k_blocks + (after < KB_PER_CHUNK ? (int)after : KB_PER_CHUNK);
            float acc[128];
#pragma unroll
            for (int e = 0; e < 128; ++e) acc[e] = 0.0f;
            // a K slice after the first continues the sums the previous one
            // stored (the first K range of a split tile carries them)
            if constexpr (tc_is_f32<typename Spec::Out>::value) {
                if (g.acc_in && part <= 0) {
                    int mb, nb, bi;
                    tile_coords(g, t, mb, nb, bi);
                    tc_load_sums(acc, g, bi, (i64)mb * 2 * BM + (i64)cta * BM + q * 32, (i64)nb * BN + half * 128, lane);
                }
            }
            for (int c = c0; c < c1; ++c, ++chunk) {
                const int buf = (int)(chunk & 1u);
                const u32 use = (chunk >> 1) & 1u;
                const int c_end = (c + 1) * KB_PER_CHUNK < kb_hi ? (c + 1) * KB_PER_CHUNK : kb_hi;
                const bool conv_ok = convert_until(c_end + KB_PER_CHUNK < limit ? c_end + KB_PER_CHUNK : limit);
                // two chunks before a whole tile's epilogue: its operand rows
                // into L2 (the epilogue's loads would otherwise stall these
                // threads, which also drain TMEM for the MMA issuer)
                if (part < 0 && !g.acc_raw && c == (c1 - 2 > c0 ? c1 - 2 : c0)) {
                    int mb, nb, bi;
                    tile_coords(g, t, mb, nb, bi);
                    Spec::prefetch(g, bi, (i64)mb * 2 * BM + (i64)cta * BM + q * 32 + lane, (i64)nb * BN + half * 128);
                }
                // ... and in a K slice that continues earlier sums, the sums
                // this pair's next tile starts from (read when it begins)
                if (g.acc_in && c == (c1 - 2 > c0 ? c1 - 2 : c0) && u + num_pairs < g.num_units) {
                    int tn, c0n, c1n, partn;
                    unit_chunks(u + num_pairs, tn, c0n, c1n, partn);
                    if (partn <= 0) {
                        int mb, nb, bi;
                        tile_coords(g, tn, mb, nb, bi);
                        const i64 i = (i64)mb * 2 * BM + (i64)cta * BM + q * 32 + lane;
                        const i64 j0 = (i64)nb * BN + half * 128;
                        if (i < g.M) {
                            const char* row = reinterpret_cast<const char*>(g.out) + (bi * g.o_bstride + i * g.N) * 4;
#pragma unroll
                            for (int l = 0; l < 4; ++l)
                                if (j0 + 32 * l < g.N) prefetch_l2(row + (j0 + 32 * l) * 4);
                        }
                    }
                }
                const bool ready = conv_ok && wait(TFULL(buf), use, sh, g, 4u);
                if (!__all_sync(0xFFFFFFFFu, ready)) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int j = 0; j < 4; j += 2) {
                    u32 r0[32], r1[32];
                    tmem_ld32_nowait(tmem + lane_addr + (u32)(buf * BN + half * 128 + 32 * j), r0);
                    tmem_ld32_nowait(tmem + lane_addr + (u32)(buf * BN + half * 128 + 32 * (j + 1)), r1);
                    tmem_wait_ld(r0, r1);
#pragma unroll
                    for (int e = 0; e < 32; e += 2) {
                        fadd2_rn(acc[32 * j + e], acc[32 * j + e + 1], r0[e], r0[e + 1]);
                        fadd2_rn(acc[32 * (j + 1) + e], acc[32 * (j + 1) + e + 1], r1[e], r1[e + 1]);
                    }
                }
                tc_fence_before();
                if (cta == 0) mbar_arrive(TEMPTY(buf));
                else mbar_arrive_cluster(TEMPTY(buf), 0u);
            }
            if (!ok) break;
            if (CONV) conv -= k_blocks;                // counted from the next tile's first k-block
            int mb, nb, bi;
            tile_coords(g, t, mb, nb, bi);
            const i64 i0 = (i64)mb * 2 * BM + (i64)cta * BM + q * 32;
            const i64 n0 = (i64)nb * BN + half * 128;
            bool raw = false;
            if constexpr (tc_is_f32<typename Spec::Out>::value) raw = g.acc_raw != 0;
            if (part < 0 && raw) tc_store_sums(acc, g, bi, i0, n0, stg, lane);
            else if (part < 0) tc_epilogue<Spec>(acc, g, bi, i0, n0, out, stg, lane);
            else tc_store_rows<float, false>(acc, &g.tmap_ws, half * 128,
                                             ((i64)(t - g.split_first) * g.split + part) * 2 * BM + cta * BM + q * 32, 0, 256,
                                             stg, lane);
        }
        tc_epilogue_flush(lane);
    }

    // ------------------------------------------------------- teardown --
    tc_fence_before();
    __syncthreads();
    cluster_sync();                                  // the peer is done with our barriers / TMEM
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

}  // namespace bafe
