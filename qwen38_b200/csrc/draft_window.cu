// Kernels of the windowed block drafter (DFlash2 family): the dynamic grouped causal convolution
// that frames each layer branch, and the learned candidate selector.
//
// Convolution (scripts/ci/draft_convolution.py:17-37): each output row r of a block mixes its own
// row and the previous row of the block, per channel c, with a static base weight plus a dynamic
// weight that the row itself produced (one dynamic weight per group of `group` channels):
//   y[r, c] = (base[0, c] + dyn[r, t0, c / group]) * x[r, c] + (base[1, c] + dyn[r, t0 + 1, c / group]) * x[r - 1, c]
// with x[-1] = 0.  The reference sums the four products in this order with fp32 intermediates and
// rounds fp32 inputs to bf16 first; so does this kernel.  Output: a bf16 row, or an add into the
// fp32 residual (the branch's closing convolution).
//
// Selector (scripts/ci/draft_selector.py:37-56): for block rows i = 1..R-1 in order, every
// candidate c of row i scores unary[i, c] + sum_k pred[prev, k] * f[i, k] * succ[c, k]; the best
// (first on ties) becomes the proposal and the next `prev`, starting from the anchor.  One CTA runs
// the whole chain (a warp per candidate), so a proposal needs no host round trip.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace q38 {

__device__ __forceinline__ float conv_in(float v) { return __bfloat162float(__float2bfloat16(v)); }
__device__ __forceinline__ float conv_in(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename TX>
__global__ void __launch_bounds__(256)
draft_conv_kernel(const TX* __restrict__ x, const __nv_bfloat16* __restrict__ dyn, long long ldd, int tap0,
                  const float* __restrict__ base, int H, int group, __nv_bfloat16* __restrict__ out,
                  float* __restrict__ resid) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= H) return;
  const int G = H / group;
  const __nv_bfloat16* drow = dyn + (long long)r * ldd + (long long)tap0 * G + c / group;
  const float x0 = conv_in(x[(size_t)r * H + c]);
  const float x1 = r > 0 ? conv_in(x[(size_t)(r - 1) * H + c]) : 0.f;
  float y = 0.f;
  y = __fadd_rn(y, __fmul_rn(base[c], x0));
  y = __fadd_rn(y, __fmul_rn(__bfloat162float(drow[0]), x0));
  y = __fadd_rn(y, __fmul_rn(base[H + c], x1));
  y = __fadd_rn(y, __fmul_rn(__bfloat162float(drow[G]), x1));
  if (resid) resid[(size_t)r * H + c] += y;
  else out[(size_t)r * H + c] = __float2bfloat16(y);
}

constexpr int SEL_MAX_C = 32;

__global__ void __launch_bounds__(1024)
draft_select_kernel(const __nv_bfloat16* __restrict__ feats, long long ldf, const int64_t* __restrict__ cand,
                    const float* __restrict__ unary, int R, int C, const int64_t* __restrict__ anchor,
                    const __nv_bfloat16* __restrict__ pred, const __nv_bfloat16* __restrict__ succ, long long V,
                    int rank, int64_t* __restrict__ out, int* err) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float pf[];                 // [rank]: pred[prev] * f[i]
  __shared__ float score[SEL_MAX_C];
  __shared__ long long prev;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    long long a0 = anchor[0];
    if (a0 < 0 || a0 >= V) {
      record_error(err, kErrShape);
      a0 = 0;
    }
    prev = a0;
  }
  __syncthreads();
  for (int i = 1; i < R; ++i) {
    const long long p = prev;
    for (int k = threadIdx.x; k < rank; k += blockDim.x)
      pf[k] = __bfloat162float(pred[p * rank + k]) * __bfloat162float(feats[(long long)i * ldf + k]);
    __syncthreads();
    if (warp < C) {
      const long long c = cand[(long long)i * C + warp];
      const bool ok = c >= 0 && c < V;
      float acc = 0.f;
      if (ok)
        for (int k = lane; k < rank; k += 32) acc += pf[k] * __bfloat162float(succ[c * rank + k]);
      acc = warp_sum(acc);
      if (lane == 0) score[warp] = ok ? unary[(long long)i * C + warp] + acc : -INFINITY;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int best = 0;
      float bv = score[0];
      for (int j = 1; j < C; ++j)
        if (score[j] > bv) {
          bv = score[j];
          best = j;
        }
      long long nxt = cand[(long long)i * C + best];
      if (nxt < 0 || nxt >= V) {
        record_error(err, kErrShape);
        nxt = 0;
      }
      out[i - 1] = nxt;
      prev = nxt;
    }
    __syncthreads();
  }
}

}  // namespace q38

// x [R, H] bf16 or fp32 (contiguous); dyn [R, >= (tap0 + 2) * H / group] bf16 (row stride dyn.stride(0));
// base [2, H] fp32; exactly one of out (bf16 [R, H]) and resid (fp32 [R, H], added into).
void q38_draft_conv(torch::Tensor x, torch::Tensor dyn, int64_t tap0, torch::Tensor base, int64_t group,
                    c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> resid) {
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.dim() == 2 && x.is_contiguous(), "contiguous x [R, H]");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kFloat, "bf16 or fp32 x");
  const int64_t R = x.size(0), H = x.size(1);
  TORCH_CHECK(R >= 1 && R <= 65535 && H >= 1, "1..65535 rows");
  TORCH_CHECK(group >= 1 && H % group == 0, "hidden size must be a multiple of the group");
  const int64_t G = H / group;
  TORCH_CHECK(dyn.scalar_type() == at::kBFloat16 && dyn.dim() == 2 && dyn.stride(1) == 1 && dyn.size(0) == R,
              "bf16 row-major dynamic kernels [R, ...]");
  TORCH_CHECK(tap0 >= 0 && (tap0 + 2) * G <= dyn.size(1), "dynamic kernel columns out of range");
  TORCH_CHECK(base.scalar_type() == at::kFloat && base.is_contiguous() && base.numel() == 2 * H, "fp32 base [2, H]");
  TORCH_CHECK(out.has_value() != resid.has_value(), "exactly one of out / resid");
  if (out) TORCH_CHECK(out->scalar_type() == at::kBFloat16 && out->is_contiguous() && out->numel() == R * H, "bf16 out [R, H]");
  if (resid) TORCH_CHECK(resid->scalar_type() == at::kFloat && resid->is_contiguous() && resid->numel() == R * H, "fp32 resid [R, H]");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const dim3 grid((unsigned)((H + 255) / 256), (unsigned)R);
  __nv_bfloat16* op = out ? reinterpret_cast<__nv_bfloat16*>(out->data_ptr()) : nullptr;
  float* rp = resid ? resid->data_ptr<float>() : nullptr;
  const auto* dp = reinterpret_cast<const __nv_bfloat16*>(dyn.data_ptr());
  if (x.scalar_type() == at::kFloat)
    q38::launch_pdl(q38::draft_conv_kernel<float>, grid, dim3(256), 0, st, (const float*)x.data_ptr<float>(), dp,
                    (long long)dyn.stride(0), (int)tap0, (const float*)base.data_ptr<float>(), (int)H, (int)group, op, rp);
  else
    q38::launch_pdl(q38::draft_conv_kernel<__nv_bfloat16>, grid, dim3(256), 0, st,
                    reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), dp, (long long)dyn.stride(0), (int)tap0,
                    (const float*)base.data_ptr<float>(), (int)H, (int)group, op, rp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// feats [R, >= rank] bf16 (row stride feats.stride(0)); cand [R, C] int64 global ids; unary [R, C]
// fp32; anchor [1] int64; pred / succ [V, rank] bf16; out [R - 1] int64.
void q38_draft_select(torch::Tensor feats, torch::Tensor cand, torch::Tensor unary, torch::Tensor anchor,
                      torch::Tensor pred, torch::Tensor succ, torch::Tensor out, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(cand.device());
  TORCH_CHECK(cand.scalar_type() == at::kLong && cand.dim() == 2 && cand.is_contiguous(), "int64 cand [R, C]");
  const int64_t R = cand.size(0), C = cand.size(1);
  TORCH_CHECK(R >= 2 && R <= 1024 && C >= 1 && C <= q38::SEL_MAX_C, "2..1024 rows, 1..32 candidates");
  TORCH_CHECK(unary.scalar_type() == at::kFloat && unary.is_contiguous() && unary.sizes() == cand.sizes(),
              "fp32 unary [R, C]");
  TORCH_CHECK(pred.scalar_type() == at::kBFloat16 && pred.is_contiguous() && pred.dim() == 2, "bf16 pred [V, rank]");
  TORCH_CHECK(succ.scalar_type() == at::kBFloat16 && succ.is_contiguous() && succ.sizes() == pred.sizes(),
              "bf16 succ [V, rank]");
  const int64_t V = pred.size(0), rank = pred.size(1);
  TORCH_CHECK(rank >= 1 && rank <= 4096, "rank 1..4096");
  TORCH_CHECK(feats.scalar_type() == at::kBFloat16 && feats.dim() == 2 && feats.stride(1) == 1 &&
                  feats.size(0) == R && feats.size(1) >= rank,
              "bf16 feats [R, >= rank]");
  TORCH_CHECK(anchor.scalar_type() == at::kLong && anchor.numel() >= 1, "int64 anchor");
  TORCH_CHECK(out.scalar_type() == at::kLong && out.is_contiguous() && out.numel() >= R - 1, "int64 out [R - 1]");
  TORCH_CHECK(err.scalar_type() == at::kInt, "int32 error word");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  q38::launch_pdl(q38::draft_select_kernel, dim3(1), dim3((unsigned)(32 * C)), (size_t)rank * sizeof(float), st,
                  reinterpret_cast<const __nv_bfloat16*>(feats.data_ptr()), (long long)feats.stride(0),
                  (const int64_t*)cand.data_ptr<int64_t>(), (const float*)unary.data_ptr<float>(), (int)R, (int)C,
                  (const int64_t*)anchor.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(pred.data_ptr()),
                  reinterpret_cast<const __nv_bfloat16*>(succ.data_ptr()), (long long)V, (int)rank,
                  out.data_ptr<int64_t>(), err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
