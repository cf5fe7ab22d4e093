// Swap-AB (<= 32 token rows) instantiations of the tcgen05 GEMM.
#include "gemm_kernel.cuh"

namespace q38 {
void launch_swap(int epi, const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& g, dim3 grid, cudaStream_t st) {
  switch (epi) {
    case EPI_BF16: launch_gemm<32, SKINNY_STAGES, EPI_BF16, true>(ma, mb, g, grid, st); break;
    case EPI_F32: launch_gemm<32, SKINNY_STAGES, EPI_F32, true>(ma, mb, g, grid, st); break;
    case EPI_ADD_F32: launch_gemm<32, SKINNY_STAGES, EPI_ADD_F32, true>(ma, mb, g, grid, st); break;
    case EPI_SWIGLU: launch_gemm<32, SKINNY_STAGES, EPI_SWIGLU, true>(ma, mb, g, grid, st); break;
    case EPI_ARGMAX: launch_gemm<32, SKINNY_STAGES, EPI_ARGMAX, true>(ma, mb, g, grid, st); break;
    case EPI_PUSH_F32: launch_gemm<32, SKINNY_STAGES, EPI_PUSH_F32, true>(ma, mb, g, grid, st); break;
    case EPI_SPLIT_F32: launch_gemm<32, SKINNY_STAGES, EPI_SPLIT_F32, true>(ma, mb, g, grid, st); break;
    default: TORCH_CHECK(false, "bad epilogue");
  }
}
}  // namespace q38
