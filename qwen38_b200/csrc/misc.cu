// Small fused ops: RMSNorm (+ residual read in fp32), embedding gather into the fp32 residual,
// Markov-selector steps, and the pinned-acceptance / greedy-accept helpers.
//
// Markov selector (K-MARKOV): step i scores logits[i] + pred[prev] . succ^T over the (local) vocab
// and takes the argmax, which becomes prev for step i+1 (scripts/ci/dspark_markov.py:4-29,
// scripts/ci/dspark_markov_device.py).  `prev` lives in device memory so the 15 steps need no
// host round trip.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace q38 {

// One CTA per row; the row stays in registers between the sum of squares and the scaling.
template <typename TIn, int VPT>
__global__ void __launch_bounds__(256)
rms_norm_kernel(const TIn* __restrict__ x, long long ldx, const float* __restrict__ w, int H, float eps,
                __nv_bfloat16* __restrict__ out, long long ldo) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  const TIn* xr = x + (size_t)r * ldx;
  __shared__ float red[32];
  float v[VPT], wv[VPT];
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < VPT; ++u) {             // row and weight loads share one memory round trip
    const int i = threadIdx.x + u * blockDim.x;
    float f = 0.f;
    wv[u] = 0.f;
    if (i < H) {
      if constexpr (std::is_same<TIn, float>::value) f = xr[i];
      else f = __bfloat162float(xr[i]);
      wv[u] = w[i];
    }
    v[u] = f;
    ss += f * f;
  }
  ss = warp_sum(ss);
  const int w_ = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w_] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[31] = rsqrtf(t / H + eps);
  }
  __syncthreads();
  const float inv = red[31];
  __nv_bfloat16* o = out + (size_t)r * ldo;
#pragma unroll
  for (int u = 0; u < VPT; ++u) {
    const int i = threadIdx.x + u * blockDim.x;
    if (i < H) o[i] = __float2bfloat16(v[u] * inv * wv[u]);
  }
}

// The second half of the pushed tensor-parallel all-reduce (the GEMM half is EPI_PUSH_F32): one
// CTA per token row reads every rank's {value, epoch} words of its row, spinning (bounded) on each
// until this use's epoch appears, adds the W partials in rank order 0..W-1 to the fp32 residual row
// (identical bits on every rank), writes the row back, advances the row's epoch, and - when a norm
// weight is given - emits its RMSNorm in bf16.
constexpr int AR_RANKS = 8;
constexpr int AR_ROWS = 32;

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* addr) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(addr) : "memory");
  return v;
}

template <int VPT>
__global__ void __launch_bounds__(256)
rms_norm_ar_kernel(float* __restrict__ x, int H, const float* __restrict__ w, float eps,
                   __nv_bfloat16* __restrict__ out, long long ldo, const unsigned long long* __restrict__ recv,
                   int* __restrict__ epochs, int slot, int world, long long block_words, int* err) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  __shared__ int ok_s;
  __shared__ float red[32];
  if (threadIdx.x == 0) ok_s = 1;
  const uint32_t e = (uint32_t)epochs[(size_t)slot * AR_ROWS + r] + 1u;
  __syncthreads();
  const unsigned long long* base = recv + (size_t)slot * world * block_words + (size_t)r * H;
  float psum[VPT];                         // rank-ordered sums: ((0 + p_0) + p_1) + ...
  bool ok = true;
  const unsigned long long t0 = globaltimer();
#pragma unroll
  for (int u = 0; u < VPT; ++u) psum[u] = 0.f;
#pragma unroll
  for (int q = 0; q < AR_RANKS; ++q) {
    if (q >= world) break;
    unsigned long long wv4[VPT];
#pragma unroll
    for (int u = 0; u < VPT; ++u) {          // issue every load of this source before spinning
      const int i = threadIdx.x + u * blockDim.x;
      wv4[u] = i < H ? ld_relaxed_sys_u64(base + (size_t)q * block_words + i) : ((unsigned long long)e << 32);
    }
#pragma unroll
    for (int u = 0; u < VPT; ++u) {
      const int i = threadIdx.x + u * blockDim.x;
      while (ok && (uint32_t)(wv4[u] >> 32) != e) {
        if (globaltimer() - t0 > kWaitLimitNs) {
          ok = false;
          break;
        }
        wv4[u] = ld_relaxed_sys_u64(base + (size_t)q * block_words + i);
      }
      if (i < H) psum[u] += __uint_as_float((uint32_t)wv4[u]);
    }
  }
  if (!ok) {
    record_error(err, kErrPeer);
    ok_s = 0;
  }
  __syncthreads();
  if (!ok_s) return;                       // a peer never published: residual and epoch untouched
  float* xr = x + (size_t)r * H;
  float v[VPT], wv[VPT];
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < VPT; ++u) {
    const int i = threadIdx.x + u * blockDim.x;
    float xv = 0.f;
    wv[u] = 0.f;
    if (i < H) {
      xv = xr[i];
      if (w) wv[u] = w[i];
    }
    v[u] = xv + psum[u];
    if (i < H) xr[i] = v[u];
    ss += v[u] * v[u];
  }
  if (threadIdx.x == 0) epochs[(size_t)slot * AR_ROWS + r] = (int)e;
  if (!out) return;
  ss = warp_sum(ss);
  const int w_ = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w_] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[31] = rsqrtf(t / H + eps);
  }
  __syncthreads();
  const float inv = red[31];
  __nv_bfloat16* o = out + (size_t)r * ldo;
#pragma unroll
  for (int u = 0; u < VPT; ++u) {
    const int i = threadIdx.x + u * blockDim.x;
    if (i < H) o[i] = __float2bfloat16(v[u] * inv * wv[u]);
  }
}

__global__ void embed_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ table, int H,
                             float* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  const int64_t id = ids[r];
  const __nv_bfloat16* src = table + (size_t)id * H;
  float* dst = out + (size_t)r * H;
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(src + i);
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float2 f = __bfloat1622float2(b[u]);
      dst[i + 2 * u] = f.x;
      dst[i + 2 * u + 1] = f.y;
    }
  }
}

// One Markov step over a vocab tile of 256 rows: per-tile (max, argmax) of logits + bias.
__global__ void __launch_bounds__(256)
markov_step_kernel(const float* __restrict__ logits, const __nv_bfloat16* __restrict__ pred,
                   const __nv_bfloat16* __restrict__ succ, int V, int R, const int64_t* __restrict__ prev,
                   float* __restrict__ part_val, int* __restrict__ part_idx) {
  extern __shared__ float pp[];   // [R]
  __shared__ float sv[8];
  __shared__ int si[8];
  pdl_wait();
  pdl_trigger();
  const int64_t pv = *prev;
  for (int i = threadIdx.x; i < R; i += blockDim.x) pp[i] = __bfloat162float(pred[(size_t)pv * R + i]);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  const int v0 = blockIdx.x * 256;
  for (int rr = warp; rr < 256; rr += 8) {
    const int v = v0 + rr;
    if (v >= V) break;
    const __nv_bfloat16* srow = succ + (size_t)v * R;
    float d = 0.f;
    for (int k = lane * 8; k < R; k += 256) {
      const uint4 u = *reinterpret_cast<const uint4*>(srow + k);
      const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(b[q]);
        d = fmaf(f.x, pp[k + 2 * q], d);
        d = fmaf(f.y, pp[k + 2 * q + 1], d);
      }
    }
    d = warp_sum(d);
    const float sc = logits[v] + d;
    if (sc > best || (sc == best && v < bi)) { best = sc; bi = v; }
  }
  if (lane == 0) { sv[warp] = best; si[warp] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 8; ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < bi)) { best = sv[w]; bi = si[w]; }
    part_val[blockIdx.x] = best;
    part_idx[blockIdx.x] = bi;
  }
}

// Reduce tile partials -> (value, global index); writes prev (next step's anchor) and out.
__global__ void markov_finalize_kernel(const float* __restrict__ part_val, const int* __restrict__ part_idx,
                                       int tiles, long long vocab_offset, int64_t* __restrict__ prev,
                                       int64_t* __restrict__ out, float* __restrict__ out_val) {
  pdl_wait();
  pdl_trigger();
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int t = threadIdx.x; t < tiles; t += blockDim.x) {
    const float v = part_val[t];
    const int i = part_idx[t];
    if (v > best || (v == best && i < bi)) { best = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    if (v2 > best || (v2 == best && i2 < bi)) { best = v2; bi = i2; }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) { sv[w] = best; si[w] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < (int)(blockDim.x >> 5); ++k)
      if (sv[k] > best || (sv[k] == best && si[k] < bi)) { best = sv[k]; bi = si[k]; }
    const int64_t g = (int64_t)bi + vocab_offset;
    if (prev) *prev = g;
    out[0] = g;
    if (out_val) out_val[0] = best;
  }
}

}  // namespace q38

void q38_rms_norm(torch::Tensor x, torch::Tensor w, double eps, torch::Tensor out) {
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kFloat, "bf16 out, fp32 weight");
  const int R = (int)x.size(0), H = (int)x.size(1);
  if (R == 0) return;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  TORCH_CHECK(H <= 256 * 32, "rms_norm: hidden too large");
  const int vpt = (H + 255) / 256;
#define Q38_NORM(VV)                                                                                        \
  if (x.scalar_type() == at::kFloat)                                                                        \
    q38::launch_pdl(q38::rms_norm_kernel<float, VV>, dim3(R), dim3(256), 0, st, (const float*)x.data_ptr<float>(), \
        (long long)x.stride(0), (const float*)w.data_ptr<float>(), H, (float)eps,                          \
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), (long long)out.stride(0));                        \
  else                                                                                                      \
    q38::launch_pdl(q38::rms_norm_kernel<__nv_bfloat16, VV>, dim3(R), dim3(256), 0, st,                     \
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), (long long)x.stride(0),                       \
        (const float*)w.data_ptr<float>(), H, (float)eps, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),  \
        (long long)out.stride(0));
  if (vpt <= 1) { Q38_NORM(1) }
  else if (vpt <= 4) { Q38_NORM(4) }
  else if (vpt <= 8) { Q38_NORM(8) }
  else if (vpt <= 20) { Q38_NORM(20) }
  else { Q38_NORM(32) }
#undef Q38_NORM
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void q38_embedding(torch::Tensor ids, torch::Tensor table, torch::Tensor out) {
  c10::cuda::CUDAGuard guard(ids.device());
  TORCH_CHECK(ids.scalar_type() == at::kLong && table.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kFloat, "int64 ids, bf16 table, fp32 out");
  const int R = (int)ids.numel(), H = (int)table.size(1);
  TORCH_CHECK(H % 8 == 0, "hidden must be a multiple of 8");
  if (R == 0) return;
  q38::launch_pdl(q38::embed_kernel, dim3(R), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
                  (const int64_t*)ids.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()),
                  H, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// One Markov step: out[0] <- argmax_v logits[v] + pred[prev] . succ[v]; prev <- out (global id).
void q38_markov_step(torch::Tensor logits_row, torch::Tensor pred, torch::Tensor succ, torch::Tensor prev,
                     torch::Tensor out, c10::optional<torch::Tensor> out_val, torch::Tensor part_val,
                     torch::Tensor part_idx, int64_t vocab_offset, bool write_prev) {
  c10::cuda::CUDAGuard guard(pred.device());
  const int V = (int)succ.size(0), R = (int)succ.size(1);
  TORCH_CHECK(R % 8 == 0, "Markov rank must be a multiple of 8");
  const int tiles = (V + 255) / 256;
  TORCH_CHECK(part_val.numel() >= tiles, "partial buffer too small");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  q38::launch_pdl(q38::markov_step_kernel, dim3(tiles), dim3(256), R * sizeof(float), st,
      (const float*)logits_row.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(pred.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(succ.data_ptr()), V, R, (const int64_t*)prev.data_ptr<int64_t>(),
      part_val.data_ptr<float>(), part_idx.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  q38::launch_pdl(q38::markov_finalize_kernel, dim3(1), dim3(256), 0, st, (const float*)part_val.data_ptr<float>(),
                  (const int*)part_idx.data_ptr<int>(), tiles, (long long)vocab_offset,
                  write_prev ? prev.data_ptr<int64_t>() : (int64_t*)nullptr, out.data_ptr<int64_t>(),
                  out_val ? out_val->data_ptr<float>() : (float*)nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// x [R, H] fp32 residual (updated in place); w / out optional (absent: reduce only).
void q38_rms_norm_ar(torch::Tensor x, c10::optional<torch::Tensor> w, double eps, c10::optional<torch::Tensor> out,
                     int64_t recv_local, torch::Tensor epochs, int64_t slot, int64_t world, int64_t block_words,
                     torch::Tensor err) {
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous() && x.dim() == 2, "contiguous fp32 residual");
  TORCH_CHECK((bool)w == (bool)out, "norm weight and output go together");
  if (out) TORCH_CHECK(out->scalar_type() == at::kBFloat16 && out->stride(1) == 1, "bf16 row-major output");
  TORCH_CHECK(world >= 1 && world <= q38::AR_RANKS, "1..8 ranks");
  const int R = (int)x.size(0), H = (int)x.size(1);
  TORCH_CHECK(R <= q38::AR_ROWS && (int64_t)R * H <= block_words, "residual larger than a receive block");
  TORCH_CHECK(epochs.scalar_type() == at::kInt && epochs.numel() >= (slot + 1) * q38::AR_ROWS, "epoch array too small");
  TORCH_CHECK(H <= 256 * 20, "hidden too large");
  if (R == 0) return;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const float* wp = w ? w->data_ptr<float>() : nullptr;
  __nv_bfloat16* op = out ? reinterpret_cast<__nv_bfloat16*>(out->data_ptr()) : nullptr;
  const long long ldo = out ? out->stride(0) : 0;
  const int vpt = (H + 255) / 256;
#define Q38_NORM_AR(VV)                                                                                          \
  q38::launch_pdl(q38::rms_norm_ar_kernel<VV>, dim3(R), dim3(256), 0, st, x.data_ptr<float>(), H, wp, (float)eps,  \
                  op, ldo, reinterpret_cast<const unsigned long long*>(recv_local), epochs.data_ptr<int>(),     \
                  (int)slot, (int)world, (long long)block_words, err.data_ptr<int>());
  if (vpt <= 4) { Q38_NORM_AR(4) }
  else if (vpt <= 8) { Q38_NORM_AR(8) }
  else { Q38_NORM_AR(20) }
#undef Q38_NORM_AR
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
