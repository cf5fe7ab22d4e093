// Prefill (128 x 256 tile) instantiations of the tcgen05 GEMM.
#include "gemm_kernel.cuh"

namespace q38 {
void launch_prefill(int epi, const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& g, dim3 grid,
                    cudaStream_t st) {
  switch (epi) {
    case EPI_BF16: launch_gemm<PREFILL_BN, PREFILL_STAGES, EPI_BF16, false>(ma, mb, g, grid, st); break;
    case EPI_F32: launch_gemm<PREFILL_BN, PREFILL_STAGES, EPI_F32, false>(ma, mb, g, grid, st); break;
    case EPI_ADD_F32: launch_gemm<PREFILL_BN, PREFILL_STAGES, EPI_ADD_F32, false>(ma, mb, g, grid, st); break;
    case EPI_SWIGLU: launch_gemm<PREFILL_BN, PREFILL_STAGES, EPI_SWIGLU, false>(ma, mb, g, grid, st); break;
    case EPI_RS_F32: launch_gemm<PREFILL_BN, PREFILL_STAGES, EPI_RS_F32, false>(ma, mb, g, grid, st); break;
    default: TORCH_CHECK(false, "bad epilogue");
  }
}
}  // namespace q38
