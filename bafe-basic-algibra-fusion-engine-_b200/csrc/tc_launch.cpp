// tc_launch.cpp -- host side of the tensor-core GEMM.
#include "tc_launch.h"

namespace bafe_cuda {

bool tc_kernel_enabled() { return false; }
int tc_smem_bytes(int) { return 0; }
int tc_prepare(const Step&, const void*, const void*, void*, const std::vector<const void*>&, int, TcLaunch&,
               std::string& err) {
    err = "tensor-core GEMM not available";
    return 11;
}

}  // namespace bafe_cuda
