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

// RMSNorm rows are spread over a cluster of NORM_CPR CTAs (128 threads each): CTA c of row r owns
// the 128-column chunks c, c + NORM_CPR, c + 2 NORM_CPR, ... of the row, so a [16, 5120] residual
// runs on 128 CTAs instead of 16 and each CTA touches 640 columns.  The sum of squares is reduced
// in a fixed order (per thread over its chunks, xor butterfly in the warp, the four warps in order,
// then the cluster's CTAs in rank order through distributed shared memory), so every kernel that
// normalises with this core - the plain norm and the all-reduce norm - produces the same bits for
// the same row.
constexpr int NORM_CPR = 8;
constexpr int NORM_NT = 128;

__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Store `v` into CTA `rank`'s copy of the shared variable at `local`.
__device__ __forceinline__ void st_cluster_f32(const float* local, uint32_t rank, float v) {
  uint32_t a = smem_u32(local), ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(v) : "memory");
}

// Row total of the per-thread partial `ss` over the whole cluster (every CTA gets the same bits).
// `flag` is exchanged alongside (all CTAs learn the minimum); the caller has issued
// cluster_arrive_relaxed() once at kernel start, which this matches before the first remote store.
__device__ __forceinline__ float norm_row_total(float ss, int& flag) {
  __shared__ float red[NORM_NT / 32];
  __shared__ float xch[NORM_CPR];
  __shared__ float okx[NORM_CPR];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  cluster_wait();                                  // every CTA of the cluster has started
  if (threadIdx.x < NORM_CPR) {
    const float t = ((red[0] + red[1]) + red[2]) + red[3];
    const uint32_t me = cluster_rank();
    st_cluster_f32(&xch[me], threadIdx.x, t);
    st_cluster_f32(&okx[me], threadIdx.x, (float)flag);
  }
  cluster_sync_all();
  float tot = 0.f;
#pragma unroll
  for (int p = 0; p < NORM_CPR; ++p) {
    tot += xch[p];
    flag = min(flag, (int)okx[p]);
  }
  return tot;
}

template <typename TIn, int VPT>
__global__ void __launch_bounds__(NORM_NT)
rms_norm_kernel(const TIn* __restrict__ x, long long ldx, const float* __restrict__ w, int H, float eps,
                __nv_bfloat16* __restrict__ out, long long ldo) {
  cluster_arrive_relaxed();
  pdl_wait();
  pdl_trigger();
  const int c = (int)cluster_rank(), r = blockIdx.y;
  const TIn* xr = x + (size_t)r * ldx;
  float v[VPT], wv[VPT];
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < VPT; ++u) {             // row and weight loads share one memory round trip
    const int i = (u * NORM_CPR + c) * NORM_NT + threadIdx.x;
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
  int flag = 1;
  const float inv = rsqrtf(norm_row_total(ss, flag) / H + eps);
  __nv_bfloat16* o = out + (size_t)r * ldo;
#pragma unroll
  for (int u = 0; u < VPT; ++u) {
    const int i = (u * NORM_CPR + c) * NORM_NT + threadIdx.x;
    if (i < H) o[i] = __float2bfloat16(v[u] * inv * wv[u]);
  }
}

// Deferred split-K reduction + residual add + RMSNorm (<= 64 rows, the cluster-spread layout of
// rms_norm_kernel).  parts holds S fp32 slices [S][R][H] of a row-parallel GEMM (EPI_SPLIT_F32);
// every element becomes x + (((0 + p_0) + p_1) + ... + p_{S-1}), the split-order sum and residual
// add of the GEMM's own fix-up, and is written back to the residual x.  With a weight the updated
// row is normalised into `out` with the norm core shared by rms_norm_kernel (same bits); without
// one (w == nullptr) only the residual is completed.
constexpr int MAX_SPLITS = 8;

template <int VPT>
__global__ void __launch_bounds__(NORM_NT)
rms_norm_split_kernel(float* __restrict__ x, const float* __restrict__ parts, int S, const float* __restrict__ w,
                      int H, float eps, __nv_bfloat16* __restrict__ out, long long ldo) {
  cluster_arrive_relaxed();
  pdl_wait();
  pdl_trigger();
  const int c = (int)cluster_rank(), r = blockIdx.y, R = gridDim.y;
  float* xr = x + (size_t)r * H;
  const size_t pstride = (size_t)R * H;
  const float* pr = parts + (size_t)r * H;
  float v[VPT], wv[VPT], acc[VPT];
#pragma unroll
  for (int u = 0; u < VPT; ++u) {               // residual and weight loads in one round trip
    const int i = (u * NORM_CPR + c) * NORM_NT + threadIdx.x;
    v[u] = i < H ? xr[i] : 0.f;
    wv[u] = (w != nullptr && i < H) ? w[i] : 0.f;
    acc[u] = 0.f;
  }
#pragma unroll
  for (int k = 0; k < MAX_SPLITS; ++k) {        // slices in split order
    if (k < S) {
#pragma unroll
      for (int u = 0; u < VPT; ++u) {
        const int i = (u * NORM_CPR + c) * NORM_NT + threadIdx.x;
        if (i < H) acc[u] += __ldcg(pr + k * pstride + i);
      }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < VPT; ++u) {
    const int i = (u * NORM_CPR + c) * NORM_NT + threadIdx.x;
    v[u] = v[u] + acc[u];
    if (i < H) xr[i] = v[u];
    ss += v[u] * v[u];
  }
  if (w == nullptr) {
    cluster_wait();                             // matches the arrive above; no exchange needed
    return;
  }
  int flag = 1;
  const float inv = rsqrtf(norm_row_total(ss, flag) / H + eps);
  __nv_bfloat16* o = out + (size_t)r * ldo;
#pragma unroll
  for (int u = 0; u < VPT; ++u) {
    const int i = (u * NORM_CPR + c) * NORM_NT + threadIdx.x;
    if (i < H) o[i] = __float2bfloat16(v[u] * inv * wv[u]);
  }
}

// Many rows (prefill chunks): one CTA of 256 threads per row, row kept in registers between the
// sum of squares and the scaling.  Row counts above NORM_CLUSTER_ROWS take this kernel; its
// reduction order differs from the cluster kernel's, which only rows of decode / verify size
// (where the all-reduce norm must reproduce the plain norm bit for bit) need.
constexpr int NORM_CLUSTER_ROWS = 64;

template <typename TIn, int VPT>
__global__ void __launch_bounds__(256)
rms_norm_rows_kernel(const TIn* __restrict__ x, long long ldx, const float* __restrict__ w, int H, float eps,
                     __nv_bfloat16* __restrict__ out, long long ldo) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  const TIn* xr = x + (size_t)r * ldx;
  __shared__ float red[8];
  float v[VPT], wv[VPT];
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < VPT; ++u) {
    const int i = threadIdx.x + u * 256;
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
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) t += red[k];
  const float inv = rsqrtf(t / H + eps);
  __nv_bfloat16* o = out + (size_t)r * ldo;
#pragma unroll
  for (int u = 0; u < VPT; ++u) {
    const int i = threadIdx.x + u * 256;
    if (i < H) o[i] = __float2bfloat16(v[u] * inv * wv[u]);
  }
}

// The second half of the pushed tensor-parallel all-reduce (the GEMM half is EPI_PUSH_F32): the
// CTAs of a row read every rank's {value, epoch} words of their chunks - all ranks' loads in flight
// at once - and spin (bounded) on each until this use's epoch appears, add the W partials in rank
// order 0..W-1 to the fp32 residual (identical bits on every rank), and - when a norm weight is
// given - emit the row's RMSNorm in bf16.  The residual, the row's epoch and the output are
// written only when every CTA of the row saw every word: a peer that never published leaves them
// untouched (the error word records it).
constexpr int AR_RANKS = 8;
constexpr int AR_ROWS = 64;          // = AR_MAX_ROWS of the pushing GEMM (gemm_kernel.cuh)

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* addr) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(addr) : "memory");
  return v;
}

template <int VPT, int WORLD>
__global__ void __launch_bounds__(NORM_NT)
rms_norm_ar_kernel(float* __restrict__ x, int H, const float* __restrict__ w, float eps,
                   __nv_bfloat16* __restrict__ out, long long ldo, const unsigned long long* __restrict__ recv,
                   int* __restrict__ epochs, int slot, long long block_words, int* err) {
  cluster_arrive_relaxed();
  pdl_wait();
  pdl_trigger();
  const int c = (int)cluster_rank(), r = blockIdx.y;
  const uint32_t e = (uint32_t)epochs[(size_t)slot * AR_ROWS + r] + 1u;
  const unsigned long long* base = recv + (size_t)slot * WORLD * block_words + (size_t)r * H;
  unsigned long long wd[WORLD][VPT];
#pragma unroll
  for (int q = 0; q < WORLD; ++q)             // every rank's words of this thread's columns in flight
#pragma unroll
    for (int u = 0; u < VPT; ++u) {
      const int i = (u * NORM_CPR + c) * NORM_NT + threadIdx.x;
      wd[q][u] = i < H ? ld_relaxed_sys_u64(base + (size_t)q * block_words + i) : ((unsigned long long)e << 32);
    }
  int flag = 1;
  const unsigned long long t0 = globaltimer();
#pragma unroll
  for (int q = 0; q < WORLD; ++q)
#pragma unroll
    for (int u = 0; u < VPT; ++u) {
      const int i = (u * NORM_CPR + c) * NORM_NT + threadIdx.x;
      while (flag && (uint32_t)(wd[q][u] >> 32) != e) {
        if (globaltimer() - t0 > kWaitLimitNs) {
          flag = 0;
          break;
        }
        wd[q][u] = ld_relaxed_sys_u64(base + (size_t)q * block_words + i);
      }
    }
  if (!flag) record_error(err, kErrPeer);
  flag = __syncthreads_and(flag);
  float* xr = x + (size_t)r * H;
  float v[VPT], wv[VPT];
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < VPT; ++u) {
    const int i = (u * NORM_CPR + c) * NORM_NT + threadIdx.x;
    float psum = 0.f;                          // rank-ordered: ((0 + p_0) + p_1) + ...
#pragma unroll
    for (int q = 0; q < WORLD; ++q) psum += __uint_as_float((uint32_t)wd[q][u]);
    float xv = 0.f;
    wv[u] = 0.f;
    if (i < H) {
      xv = xr[i];
      if (w) wv[u] = w[i];
    }
    v[u] = xv + psum;
    ss += v[u] * v[u];
  }
  const float tot = norm_row_total(ss, flag);
  if (!flag) return;                          // some CTA of the row missed a word: nothing written
#pragma unroll
  for (int u = 0; u < VPT; ++u) {
    const int i = (u * NORM_CPR + c) * NORM_NT + threadIdx.x;
    if (i < H) xr[i] = v[u];
  }
  if (c == 0 && threadIdx.x == 0) epochs[(size_t)slot * AR_ROWS + r] = (int)e;
  if (!out) return;
  const float inv = rsqrtf(tot / H + eps);
  __nv_bfloat16* o = out + (size_t)r * ldo;
#pragma unroll
  for (int u = 0; u < VPT; ++u) {
    const int i = (u * NORM_CPR + c) * NORM_NT + threadIdx.x;
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

// One Markov step over a vocab tile of 256 rows: per-tile (max, argmax) of logits + bias.  The row
// scores use markov_row_dot (common.cuh), the arithmetic of the one-launch selector (markov.cu).

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
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, grp = threadIdx.x >> 3, j = threadIdx.x & 7;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  const int v0 = blockIdx.x * 256;
  for (int r0 = 0; r0 < 256 && v0 + r0 < V; r0 += 32) {     // uniform trip count over the CTA
    const int v = v0 + r0 + grp;
    const bool valid = v < V;
    const int vr = valid ? v : v0;                              // invalid groups score a row, discard it
    const float sc = logits[vr] + markov_row_dot(succ + (size_t)vr * R, pp, R, j);
    if (valid && (sc > best || (sc == best && v < bi))) { best = sc; bi = v; }
  }
#pragma unroll
  for (int o = 16; o >= 8; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    if (v2 > best || (v2 == best && i2 < bi)) { best = v2; bi = i2; }
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

// Per-row chunk count of the cluster-spread norms: VPT 128-column chunks per CTA.
static int norm_vpt(int H) { return (((H + q38::NORM_NT - 1) / q38::NORM_NT) + q38::NORM_CPR - 1) / q38::NORM_CPR; }

void q38_rms_norm(torch::Tensor x, torch::Tensor w, double eps, torch::Tensor out) {
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kFloat, "bf16 out, fp32 weight");
  const int R = (int)x.size(0), H = (int)x.size(1);
  if (R == 0) return;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (R > q38::NORM_CLUSTER_ROWS) {
    const int v2 = (H + 255) / 256;
    TORCH_CHECK(v2 <= 32, "rms_norm: hidden above 8192");
#define Q38_NORM_ROWS(VV)                                                                                   \
  if (x.scalar_type() == at::kFloat) {                                                                      \
    q38::launch_pdl(q38::rms_norm_rows_kernel<float, VV>, dim3(R), dim3(256), 0, st,                         \
                    (const float*)x.data_ptr<float>(), (long long)x.stride(0), (const float*)w.data_ptr<float>(), \
                    H, (float)eps, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), (long long)out.stride(0)); \
  } else {                                                                                                  \
    q38::launch_pdl(q38::rms_norm_rows_kernel<__nv_bfloat16, VV>, dim3(R), dim3(256), 0, st,                 \
                    reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), (long long)x.stride(0),             \
                    (const float*)w.data_ptr<float>(), H, (float)eps,                                        \
                    reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), (long long)out.stride(0));             \
  }
    if (v2 <= 4) { Q38_NORM_ROWS(4) }
    else if (v2 <= 8) { Q38_NORM_ROWS(8) }
    else if (v2 <= 20) { Q38_NORM_ROWS(20) }
    else { Q38_NORM_ROWS(32) }
#undef Q38_NORM_ROWS
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  const int vpt = norm_vpt(H);
  TORCH_CHECK(vpt <= 8, "rms_norm: hidden above 8192");
  const dim3 grid(q38::NORM_CPR, R), cl(q38::NORM_CPR, 1, 1);
#define Q38_NORM(VV)                                                                                          \
  if (x.scalar_type() == at::kFloat) {                                                                        \
    TORCH_CHECK(q38::launch_pdl_cluster(q38::rms_norm_kernel<float, VV>, grid, dim3(q38::NORM_NT), 0, st, cl,  \
        (const float*)x.data_ptr<float>(), (long long)x.stride(0), (const float*)w.data_ptr<float>(), H,     \
        (float)eps, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), (long long)out.stride(0)) == cudaSuccess, \
        "rms_norm launch");                                                                                    \
  } else {                                                                                                    \
    TORCH_CHECK(q38::launch_pdl_cluster(q38::rms_norm_kernel<__nv_bfloat16, VV>, grid, dim3(q38::NORM_NT), 0,  \
        st, cl, reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), (long long)x.stride(0),               \
        (const float*)w.data_ptr<float>(), H, (float)eps, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),  \
        (long long)out.stride(0)) == cudaSuccess, "rms_norm launch");                                         \
  }
  if (vpt <= 1) { Q38_NORM(1) }
  else if (vpt <= 2) { Q38_NORM(2) }
  else if (vpt <= 5) { Q38_NORM(5) }
  else { Q38_NORM(8) }
#undef Q38_NORM
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Completes a deferred split-K row-parallel GEMM (q38_linear_split) into the residual x and, with a
// weight, normalises the updated rows into out (see rms_norm_split_kernel).
void q38_rms_norm_split(torch::Tensor x, torch::Tensor parts, int64_t S, c10::optional<torch::Tensor> w, double eps,
                        c10::optional<torch::Tensor> out) {
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous() && x.dim() == 2, "contiguous fp32 residual");
  const int R = (int)x.size(0), H = (int)x.size(1);
  TORCH_CHECK(R >= 1 && R <= q38::NORM_CLUSTER_ROWS, "deferred split-K serves 1..64 rows");
  TORCH_CHECK(S >= 1 && S <= q38::MAX_SPLITS, "1..8 split slices");
  TORCH_CHECK(parts.scalar_type() == at::kFloat && parts.is_contiguous() && parts.numel() >= S * R * H,
              "split partial buffer too small");
  TORCH_CHECK(w.has_value() == out.has_value(), "weight and output go together");
  const float* wp = nullptr;
  __nv_bfloat16* op = nullptr;
  long long ldo = 0;
  if (w.has_value()) {
    TORCH_CHECK(w->scalar_type() == at::kFloat && w->numel() == H, "fp32 weight [H]");
    TORCH_CHECK(out->scalar_type() == at::kBFloat16 && out->stride(1) == 1 && out->size(0) == R, "bf16 out [R, H]");
    wp = w->data_ptr<float>();
    op = reinterpret_cast<__nv_bfloat16*>(out->data_ptr());
    ldo = out->stride(0);
  }
  const int vpt = norm_vpt(H);
  TORCH_CHECK(vpt <= 8, "rms_norm: hidden above 8192");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const dim3 grid(q38::NORM_CPR, R), cl(q38::NORM_CPR, 1, 1);
  cudaError_t e;
#define Q38_NSPLIT(VV)                                                                                        \
  e = q38::launch_pdl_cluster(q38::rms_norm_split_kernel<VV>, grid, dim3(q38::NORM_NT), 0, st, cl,            \
                              x.data_ptr<float>(), (const float*)parts.data_ptr<float>(), (int)S, wp, H,      \
                              (float)eps, op, ldo);
  if (vpt <= 1) { Q38_NSPLIT(1) }
  else if (vpt <= 2) { Q38_NSPLIT(2) }
  else if (vpt <= 5) { Q38_NSPLIT(5) }
  else { Q38_NSPLIT(8) }
#undef Q38_NSPLIT
  TORCH_CHECK(e == cudaSuccess, "rms_norm_split launch");
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
  const int vpt = norm_vpt(H);
  TORCH_CHECK(vpt <= 5, "hidden above 5120 not served by the all-reduce norm");
  if (R == 0) return;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const float* wp = w ? w->data_ptr<float>() : nullptr;
  __nv_bfloat16* op = out ? reinterpret_cast<__nv_bfloat16*>(out->data_ptr()) : nullptr;
  const long long ldo = out ? out->stride(0) : 0;
  const dim3 grid(q38::NORM_CPR, R), cl(q38::NORM_CPR, 1, 1);
  cudaError_t e = cudaErrorInvalidValue;
#define Q38_AR(VV, WW)                                                                                         \
  e = q38::launch_pdl_cluster(q38::rms_norm_ar_kernel<VV, WW>, grid, dim3(q38::NORM_NT), 0, st, cl,              \
                              x.data_ptr<float>(), H, wp, (float)eps, op, ldo,                                 \
                              reinterpret_cast<const unsigned long long*>(recv_local), epochs.data_ptr<int>(), \
                              (int)slot, (long long)block_words, err.data_ptr<int>());
#define Q38_AR_W(VV)                                                                                           \
  switch (world) {                                                                                             \
    case 1: Q38_AR(VV, 1) break;                                                                               \
    case 2: Q38_AR(VV, 2) break;                                                                               \
    case 4: Q38_AR(VV, 4) break;                                                                               \
    case 8: Q38_AR(VV, 8) break;                                                                               \
    case 3: Q38_AR(VV, 3) break;                                                                               \
    case 5: Q38_AR(VV, 5) break;                                                                               \
    case 6: Q38_AR(VV, 6) break;                                                                               \
    default: Q38_AR(VV, 7) break;                                                                              \
  }
  if (vpt <= 1) { Q38_AR_W(1) }
  else if (vpt <= 2) { Q38_AR_W(2) }
  else { Q38_AR_W(5) }
#undef Q38_AR_W
#undef Q38_AR
  TORCH_CHECK(e == cudaSuccess, "rms_norm_ar launch failed");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
