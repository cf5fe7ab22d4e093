// Swap-AB (<= 64 token rows) instantiations of the tcgen05 GEMM with block-scaled e4m3 weights
// (MXFP8: one E8M0 scale per 32 elements of a row) and bf16 activations.  The weight crosses HBM
// at one byte per element; two converter warps expand each tile in shared memory to the exact
// bf16 values (e4m3 x power of two) the bf16 kernel would read, and the MMA, split-K plan and
// epilogues are those of the bf16 kernel, so the output has the same bits as the bf16 GEMM over
// the dequantised weight.
#include "gemm_kernel.cuh"

namespace q38 {
void launch_swap_mx(int epi, const CUtensorMap& mb, const GemmArgs& g, dim3 grid, cudaStream_t st) {
  switch (epi) {
    case EPI_BF16: launch_gemm<32, SKINNY_STAGES, EPI_BF16, true, true>(mb, mb, g, grid, st); break;
    case EPI_F32: launch_gemm<32, SKINNY_STAGES, EPI_F32, true, true>(mb, mb, g, grid, st); break;
    case EPI_ADD_F32: launch_gemm<32, SKINNY_STAGES, EPI_ADD_F32, true, true>(mb, mb, g, grid, st); break;
    case EPI_SWIGLU: launch_gemm<32, SKINNY_STAGES, EPI_SWIGLU, true, true>(mb, mb, g, grid, st); break;
    case EPI_PUSH_F32: launch_gemm<32, SKINNY_STAGES, EPI_PUSH_F32, true, true>(mb, mb, g, grid, st); break;
    case EPI_SPLIT_F32: launch_gemm<32, SKINNY_STAGES, EPI_SPLIT_F32, true, true>(mb, mb, g, grid, st); break;
    default: TORCH_CHECK(false, "epilogue not served with MX weights");
  }
}
}  // namespace q38
