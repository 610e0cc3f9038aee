// tc_launch.h -- host side of the tensor-core GEMM: tensor maps, grid and
// the by-value argument block of bafe::gemm_tc (kernels/gemm_tc.cuh).
#pragma once
#include "internal.h"

namespace bafe_cuda {

struct TcLaunch {
    alignas(64) unsigned char args[1024];
    unsigned grid = 0, block = 0, smem = 0;
    unsigned cluster = 1;          // CTAs per cluster (2 for the CTA-pair kernel)
    unsigned fix_grid = 0;         // > 0: split tail tiles; launch the fixup kernel (256 threads) after
    bool wave_sync = false;        // the wave counter must be zeroed before the launch
};

// K split of the tail tiles (gemm_tc.cuh, unit_range): parts per tile (1:
// none), the first split tile and the partials' workspace bytes.
struct TcSplit {
    int parts = 1;
    int first = 0;
    size_t ws_bytes = 0;
};
TcSplit tc_split_of(const Step& s, int sm_count);

bool tc_kernel_enabled();
int tc_smem_bytes(int variant, bool pair = false);
// a_lo / b_lo: 3xTF32 residual operands (same layouts as a / b), or null.
// ws / ws_bytes: workspace for split tail tiles (tc_split_of), or null: no split.
// wave_ctr: a device word for the pair kernel's wave alignment, or null: none.
int tc_prepare(const Step& s, const void* a, const void* b, const void* a_lo, const void* b_lo, void* out,
               const std::vector<const void*>& ep, int sm_count, unsigned* err_word, void* ws, size_t ws_bytes,
               unsigned* wave_ctr, TcLaunch& L, std::string& err);
// K slices of a CTA-pair GEMM whose output is fp32 (its sums are carried
// through the output between slices): the multiple of K, in elements, that
// slice boundaries must be (one promotion chunk, so that the summation
// order is the whole launch's), or 0 when the step cannot be sliced
// (single-CTA or converting kernel, batched, col-major B, other output type).
int tc_k_slice_align(const Step& s);
// Makes a prepared launch (no split tail: ws null) cover K range [k0, k1):
// acc_in continues the sums in the output, acc_raw leaves them there.
void tc_set_k_slice(TcLaunch& L, int64_t k0, int64_t k1, int64_t K, bool acc_in, bool acc_raw, bool elem_bf16);
// elem: 0 = u8, 1 = f32, 2 = bf16; swizzle: 0 none, 1 = 128B, 2 = 128B with 32-byte atoms
int tc_encode_tensor_map(void* map, int elem, int rank, void* gaddr, const uint64_t* dims,
                         const uint64_t* strides_bytes, const uint32_t* box, int swizzle, std::string& err);

}  // namespace bafe_cuda
