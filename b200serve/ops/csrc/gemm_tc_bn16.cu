// Instantiations of the tcgen05 GEMM for a token tile of 16 (see gemm_tc.cuh).
#include "gemm_tc.cuh"

namespace b200 {

template <>
void launch_gemm_bn<16>(int epi, const CUtensorMap& tw, const CUtensorMap& ta, const GemmParams& p, int grid,
                         cudaStream_t stream) {
  switch (epi) {
    case EPI_BF16: launch_gemm<16, EPI_BF16>(tw, ta, p, grid, stream); break;
    case EPI_F32: launch_gemm<16, EPI_F32>(tw, ta, p, grid, stream); break;
    case EPI_SWIGLU: launch_gemm<16, EPI_SWIGLU>(tw, ta, p, grid, stream); break;
    case EPI_PUSH: launch_gemm<16, EPI_PUSH>(tw, ta, p, grid, stream); break;
    case EPI_QKV: launch_gemm<16, EPI_QKV>(tw, ta, p, grid, stream); break;
    case EPI_PARTIAL: launch_gemm<16, EPI_PARTIAL>(tw, ta, p, grid, stream); break;
    default: TORCH_CHECK(false, "bad epilogue");
  }
}

}  // namespace b200
