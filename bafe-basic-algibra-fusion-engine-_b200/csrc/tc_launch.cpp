// tc_launch.cpp -- host side of the tensor-core GEMM (kernels/gemm_tc.cuh):
// TMA tensor maps for the operand layouts, the by-value argument block,
// persistent grid size.
#include "tc_launch.h"

#include <cuda.h>

#include <cstdlib>
#include <cstring>

namespace bafe_cuda {

namespace {

constexpr int BM = 128, BK = 32, BN = 256;

// Mirror of bafe::TcArgs (kernels/gemm_tc.cuh); field order and types must match.
struct alignas(64) TcArgsHost {
    CUtensorMap tmap_a;
    CUtensorMap tmap_b;
    CUtensorMap tmap_a_lo;
    CUtensorMap tmap_b_lo;
    CUtensorMap tmap_out;
    CUtensorMap tmap_ws;
    void* out;
    int64_t M, N, K;
    int64_t o_bstride;
    const void* ep[8];
    unsigned* err;
    int32_t a_mn, b_mn;
    int32_t num_m, num_n, num_tiles;
    int32_t group_m;
    unsigned long long timeout_ns;
    int32_t batch;
    int32_t a_batched, b_batched;
    int32_t out_tma;
    int32_t ep_vec;
    float* ws;
    int32_t split, split_first, num_units;
    unsigned* wave_ctr;
    int32_t kb_first, kb_last;     // K slice in k-blocks (kb_last 0: all)
    int32_t acc_in, acc_raw;       // continue / leave the sums in the output
};
static_assert(sizeof(CUtensorMap) == 128, "CUtensorMap size");
static_assert(sizeof(TcArgsHost) == 1024, "TcArgs layout");
static_assert(sizeof(TcArgsHost) <= sizeof(TcLaunch::args), "TcArgs fits the launch block");

int threads_of(int) { return 320; }
// k-blocks (one 128-byte row of K) per TMEM promotion chunk, as the kernels
// have it: bf16 32; tf32 pair 32 (1x) / 3 (3x), single 4 / 2
int chunk_kblocks(const Step& s) {
    if (s.tc_elem == 1) return 32;
    if (s.tc_variant == 3) return s.tc_pair ? 3 : 2;
    return s.tc_pair ? 32 : 4;
}
int stages_of(int variant, bool pair) { return pair ? (variant == 3 ? 3 : 6) : (variant == 3 ? 2 : 4); }
int stage_bytes(int variant, bool pair) {
    return (BM * BK * 4 + (pair ? BN / 2 : BN) * BK * 4) * (variant == 3 ? 2 : 1);
}

}  // namespace

bool tc_kernel_enabled() {
    const char* e = getenv("BAFE_DISABLE_TC");
    return !(e && *e && *e != '0');
}

int tc_smem_bytes(int variant, bool pair) {
    // alignment slack + stage ring + mbarriers and shared words (1 KB, so
    // the epilogue staging stays 1024-aligned) + the epilogue staging of
    // the 8 accumulate warps (4 KB each)
    return 1024 + stages_of(variant, pair) * stage_bytes(variant, pair) + 1024 + 8 * 4096;
}

TcSplit tc_split_of(const Step& s, int sm_count) {
    TcSplit sp;
    if (s.tc_convert) return sp;                 // the conversion look-ahead assumes whole tiles
    const char* e = getenv("BAFE_TC_SPLIT");
    if (e && *e == '0') return sp;
    const int64_t tile_m = s.tc_pair ? 2 * BM : BM;
    const int64_t batch = s.batch > 1 ? s.batch : 1;
    const int64_t tiles = (s.M + tile_m - 1) / tile_m * ((s.N + BN - 1) / BN) * batch;
    const int64_t units = s.tc_pair ? sm_count / 2 : sm_count;
    const int64_t rem = units > 0 ? tiles % units : 0;
    if (rem == 0) return sp;
    const int64_t kb = (s.K + (s.tc_elem == 1 ? 64 : 32) - 1) / (s.tc_elem == 1 ? 64 : 32);
    const int64_t chunks = (kb + chunk_kblocks(s) - 1) / chunk_kblocks(s);
    // up to 4 K ranges per tail tile, as many as the idle units take, each
    // of at least 2 chunks and 32 k-blocks (shorter ones lose more to the
    // extra partial store, fixup launch and pipeline fill than they save)
    int64_t parts = units / rem;
    if (parts > 4) parts = 4;
    if (parts > chunks / 2) parts = chunks / 2;
    while (parts >= 2 && kb / parts < 32) --parts;
    if (parts < 2) return sp;
    sp.parts = (int)parts;
    sp.first = (int)(tiles - rem);
    sp.ws_bytes = (size_t)rem * parts * tile_m * BN * 4;
    return sp;
}

int tc_prepare(const Step& s, const void* a, const void* b, const void* a_lo, const void* b_lo, void* out,
               const std::vector<const void*>& ep, int sm_count, unsigned* err_word, void* ws, size_t ws_bytes,
               unsigned* wave_ctr, TcLaunch& L, std::string& err) {
    const bool split = s.tc_variant == 3;
    const bool lo_maps = split && !s.tc_convert;     // residuals read from memory
    if (lo_maps && (!a_lo || !b_lo)) {
        err = "tensor-core GEMM: 3xTF32 needs the residual operands";
        return 12;
    }
    if (((uintptr_t)a | (uintptr_t)b | (uintptr_t)a_lo | (uintptr_t)b_lo) % 16) {
        err = "tensor-core GEMM: A and B must be 16-byte aligned (TMA)";
        return 12;
    }
    if ((uintptr_t)out % 16) {
        err = "tensor-core GEMM: the output must be 16-byte aligned";
        return 12;
    }
    TcArgsHost h;
    memset(&h, 0, sizeof(h));
    const uint64_t M = (uint64_t)s.M, N = (uint64_t)s.N, K = (uint64_t)s.K;
    const uint64_t batch = (uint64_t)(s.batch > 1 ? s.batch : 1);
    // Element size and the k-block width in elements (one 128-byte row):
    // f32 32, bf16 64.  K-major boxes: k-block x rows; MN-major boxes:
    // 128 B of MN (32 f32 with 32-byte atoms, 64 bf16 plain 128B swizzle)
    // x k-block rows.
    const bool bf16 = s.tc_elem == 1;
    const uint64_t es = bf16 ? 2 : 4;
    const uint32_t bke = bf16 ? 64 : 32, mn_atom = bf16 ? 64 : 32;
    const int elem = bf16 ? 2 : 1, mn_swz = bf16 ? 1 : 2;
    // Every map is 3-D: an operand with its own matrix per batch item has
    // the batch as third dimension, one shared by all items (or an
    // unbatched product) extent 1 there, read at batch coordinate 0.
    const bool a3 = batch > 1 && s.a_bstride != 0, b3 = batch > 1 && s.b_bstride != 0;
    const uint64_t a_batch = a3 ? batch : 1, b_batch = b3 ? batch : 1;
    // A: row-major = K-major (box 32 k x 128 rows, 128B swizzle); col-major =
    // M-major (stored [K][M]; boxes of 32 m x 32 k, 128B swizzle, 32B atoms).
    auto map_a = [&](CUtensorMap* m, const void* p) {
        if (s.a_col) {
            uint64_t dims[3] = {M, K, a_batch}, strides[2] = {M * es, M * K * es};
            uint32_t box[3] = {mn_atom, bke, 1};
            return tc_encode_tensor_map(m, elem, 3, const_cast<void*>(p), dims, strides, box, mn_swz, err);
        }
        uint64_t dims[3] = {K, M, a_batch}, strides[2] = {K * es, M * K * es};
        uint32_t box[3] = {bke, (uint32_t)BM, 1};
        return tc_encode_tensor_map(m, elem, 3, const_cast<void*>(p), dims, strides, box, 1, err);
    };
    // B: col-major = K-major (stored [N][K]; box 32 k x 256 cols);
    // row-major = N-major (stored [K][N]; boxes of 32 n x 32 k, 32B atoms).
    auto map_b = [&](CUtensorMap* m, const void* p) {
        if (s.b_col) {
            uint64_t dims[3] = {K, N, b_batch}, strides[2] = {K * es, K * N * es};
            uint32_t box[3] = {bke, (uint32_t)(s.tc_pair ? BN / 2 : BN), 1};
            return tc_encode_tensor_map(m, elem, 3, const_cast<void*>(p), dims, strides, box, 1, err);
        }
        uint64_t dims[3] = {N, K, b_batch}, strides[2] = {N * es, K * N * es};
        uint32_t box[3] = {mn_atom, bke, 1};
        return tc_encode_tensor_map(m, elem, 3, const_cast<void*>(p), dims, strides, box, mn_swz, err);
    };
    if (int rc = map_a(&h.tmap_a, a)) return rc;
    if (int rc = map_b(&h.tmap_b, b)) return rc;
    if (lo_maps) {
        if (int rc = map_a(&h.tmap_a_lo, a_lo)) return rc;
        if (int rc = map_b(&h.tmap_b_lo, b_lo)) return rc;
    }
    // Epilogue: stores through a TMA map of the output when its results are
    // 2 or 4 bytes and its rows whole 16-byte units (box: 32 rows x 128
    // bytes, the accumulate warps' staging sub-tile); 16-byte operand loads
    // when every epilogue operand is aligned for them (columns come in
    // groups of 4 from a multiple of 4, and N % 4 == 0).
    const uint64_t oes = (uint64_t)s.dst_esize;
    if ((oes == 4 || oes == 2) && (N * oes) % 16 == 0) {
        uint64_t dims[3] = {N, M, batch}, strides[2] = {N * oes, M * N * oes};
        uint32_t box[3] = {(uint32_t)(128 / oes), 32, 1};
        if (int rc = tc_encode_tensor_map(&h.tmap_out, oes == 4 ? 1 : 2, 3, out, dims, strides, box, 1, err)) return rc;
        h.out_tma = 1;
    }
    h.ep_vec = 1;
    for (size_t k = 0; k < ep.size(); ++k) {
        const int es = k + 2 < s.src_esize.size() ? s.src_esize[k + 2] : 8;
        const uintptr_t need = es >= 4 ? 16 : (uintptr_t)(4 * es);
        if ((uintptr_t)ep[k] % need) h.ep_vec = 0;
    }
    h.out = out;
    h.M = s.M;
    h.N = s.N;
    h.K = s.K;
    h.o_bstride = s.M * s.N;
    for (size_t k = 0; k < ep.size() && k < 8; ++k) h.ep[k] = ep[k];
    h.err = err_word;
    h.a_mn = s.a_col ? 1 : 0;
    h.b_mn = s.b_col ? 0 : 1;
    const int tile_m = s.tc_pair ? 2 * BM : BM;   // a CTA pair covers 256 rows
    h.num_m = (int)((s.M + tile_m - 1) / tile_m);
    h.num_n = (int)((s.N + BN - 1) / BN);
    h.batch = (int32_t)batch;
    h.a_batched = a3 ? 1 : 0;
    h.b_batched = b3 ? 1 : 0;
    int64_t tiles = (int64_t)h.num_m * h.num_n * (int64_t)batch;
    if (tiles > (1LL << 30)) {
        err = "tensor-core GEMM: too many tiles";
        return 12;
    }
    h.num_tiles = (int)tiles;
    // The last wave's tiles split along K when that fills idle CTAs (and
    // the caller gave the workspace for their partials).
    h.split = 1;
    h.split_first = h.num_tiles;
    L.fix_grid = 0;
    const TcSplit sp = tc_split_of(s, sm_count);
    if (sp.parts > 1 && ws && ws_bytes >= sp.ws_bytes && (uintptr_t)ws % 16 == 0) {
        const uint64_t rows = sp.ws_bytes / (BN * 4);
        uint64_t dims[3] = {(uint64_t)BN, rows, 1}, strides[2] = {(uint64_t)BN * 4, rows * BN * 4};
        uint32_t box[3] = {32, 32, 1};
        if (int rc = tc_encode_tensor_map(&h.tmap_ws, 1, 3, ws, dims, strides, box, 1, err)) return rc;
        h.ws = (float*)ws;
        h.split = sp.parts;
        h.split_first = sp.first;
        const int64_t groups = (int64_t)(h.num_tiles - sp.first) * (s.tc_pair ? 2 * BM : BM) * (BN / 4);
        const int64_t fg = (groups + 255) / 256;
        L.fix_grid = (unsigned)(fg < (int64_t)sm_count * 8 ? fg : (int64_t)sm_count * 8);
    }
    h.num_units = h.split_first + (h.num_tiles - h.split_first) * h.split;
    // Wave alignment of the pair kernel's producers (advisory, bounded):
    // for GEMMs of at least two whole waves of long tiles, where pairs that
    // drift apart along K re-read shared operand panels from HBM.
    L.wave_sync = false;
    {
        const char* ws_env = getenv("BAFE_TC_WAVE_SYNC");
        const int64_t pairs = sm_count / 2;
        const int64_t kb = (s.K + (s.tc_elem == 1 ? 64 : 32) - 1) / (s.tc_elem == 1 ? 64 : 32);
        if (wave_ctr && s.tc_pair && !(ws_env && *ws_env == '0') && pairs > 0 && h.split_first >= 2 * pairs &&
            kb >= 128) {
            h.wave_ctr = wave_ctr;
            L.wave_sync = true;
        }
    }
    // Tiles are walked in groups of group_m M-tiles (all N-tiles of a group
    // before the next).  One wave of concurrent tiles then reads about
    // group_m A panels and waves/group_m B panels; their sum is smallest for
    // a square footprint: 8 x 9.25 for 74 CTA pairs, 16 x 9.25 for 148 CTAs
    // (whose B panels are twice as wide as their A panels).
    h.group_m = s.tc_pair ? 8 : 16;
    const char* to = getenv("BAFE_TC_TIMEOUT_MS");
    h.timeout_ns = (unsigned long long)(to ? atof(to) : 2000.0) * 1000000ull;
    memcpy(L.args, &h, sizeof(h));
    const int64_t work = h.num_units;
    if (s.tc_pair) {
        const int64_t pairs = sm_count / 2;
        L.grid = (unsigned)(2 * (work < pairs ? work : pairs));
        L.cluster = 2;
    } else {
        L.grid = (unsigned)(work < sm_count ? work : sm_count);
        L.cluster = 1;
    }
    L.block = (unsigned)threads_of(s.tc_variant);
    L.smem = (unsigned)tc_smem_bytes(s.tc_variant, s.tc_pair);
    return 0;
}

int tc_k_slice_align(const Step& s) {
    if (s.kind != StepKind::GemmTc || !s.tc_pair || s.tc_convert || s.dst_esize != 4 || s.batch > 1 || s.b_col)
        return 0;
    return chunk_kblocks(s) * (s.tc_elem == 1 ? 64 : 32);
}

void tc_set_k_slice(TcLaunch& L, int64_t k0, int64_t k1, int64_t K, bool acc_in, bool acc_raw, bool elem_bf16) {
    TcArgsHost h;
    memcpy(&h, L.args, sizeof(h));
    const int64_t bke = elem_bf16 ? 64 : 32;
    h.kb_first = (int32_t)(k0 / bke);
    h.kb_last = k1 >= K ? 0 : (int32_t)(k1 / bke);
    h.acc_in = acc_in ? 1 : 0;
    h.acc_raw = acc_raw ? 1 : 0;
    memcpy(L.args, &h, sizeof(h));
}

}  // namespace bafe_cuda
