// Fused tensor-parallel all-reduce of prefill out-projections (K-GEMMRS for prefill chunks).
//
// The reference fuses its prefill out-projections with the collective
// (matmul_reduce_scatter_async, docker/qwen-c2-graft/graft/gdn/tp.py:711-723, fp32 partials) and the
// following all-gather into the next projection (graft/mlp.py:440-446).  Here the residual stays
// replicated in fp32 and the all-reduce is split over the three kernels that already touch the data:
//
//  1. the out-projection GEMM (EPI_RS_F32, gemm_kernel.cuh) writes each 128-row fp32 tile into the
//     reduce-scatter area of the rank that owns those rows (tile t -> rank t % W) and bumps that
//     rank's arrival counter: the partials cross NVLink tile by tile while later tiles compute;
//  2. `rs_reduce_bcast_kernel` on every rank waits (bounded) for all W sources of its own rows,
//     adds them in rank order to the residual rows (identical bits whichever rank does it) and
//     stores each finished row once through the NVSwitch multicast address of the symmetric
//     residual buffer, so every rank's replica receives it; each CTA then adds 1 to every rank's
//     completion flag with one multicast release reduction;
//  3. the next consumer of the residual (the RMSNorm, or a plain wait before a tap read) waits
//     (bounded) until the flag reaches this use's count.
//
// Each rank sends (W-1)/W of its partial point to point and receives (W-1)/W of the reduced rows
// through the switch: the bytes of a ring reduce-scatter + all-gather, with no separate collective
// launch, no copy of the partial and no extra pass for the residual add.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace q38 {
namespace pfar {

constexpr int BM = 128;      // rows per tile (the prefill GEMM's token tile)
constexpr int NT = 256;

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void multimem_st_v4(float* mc, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void multimem_red_release_add_u64(unsigned long long* mc, unsigned long long v) {
  asm volatile("multimem.red.release.sys.global.add.u64 [%0], %1;" ::"l"(mc), "l"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

// Bounded wait of thread 0 until *flag >= target; then every thread may read what the flag
// publishes (the data arrived through a multicast alias of the same memory).
__device__ __forceinline__ bool wait_count(const unsigned long long* flag, unsigned long long target, int* err) {
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    bool ok = true;
    const unsigned long long t0 = globaltimer();
    while (ld_acquire_sys_u64(flag) < target) {
      if (globaltimer() - t0 > kWaitLimitNs) {
        record_error(err, kErrPeer);
        ok = false;
        break;
      }
    }
    ok_s = ok;
  }
  __syncthreads();
  fence_proxy_alias();     // every reading thread: the data came through the multicast alias
  return ok_s != 0;
}

struct RedArgs {
  const float* recv;                // this rank's area [W][rows_cap][H]
  const unsigned long long* count;  // this rank's arrival counter
  unsigned long long count_target;
  const float* x;                   // this rank's residual replica [T, H]
  float* x_mc;                      // multicast address of the residual buffer
  unsigned long long* flag_mc;      // multicast address of the completion flag
  int rank, world, rows_cap, T, H;   // rows_cap: local rows per source block (the area's stride)
  int* err;
};

// One CTA per local row slot of this rank (every rank launches the same number of slots for a
// chunk; slots past the chunk only signal).
__global__ void __launch_bounds__(NT) rs_reduce_bcast_kernel(RedArgs a) {
  const int lr = blockIdx.x;
  const int grow = ((lr / BM) * a.world + a.rank) * BM + lr % BM;   // global row of this slot
  const bool ok = wait_count(a.count, a.count_target, a.err);   // also orders this thread's x reads
  if (ok && grow < a.T) {
    const int h4 = a.H / 4;
    const float4* xr = reinterpret_cast<const float4*>(a.x + (size_t)grow * a.H);
    for (int c = threadIdx.x; c < h4; c += NT) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int s = 0; s < a.world; ++s) {           // rank order: the same bits on every rank
        const float4 p = __ldcg(reinterpret_cast<const float4*>(a.recv + ((size_t)s * a.rows_cap + lr) * a.H) + c);
        acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
      }
      const float4 xv = xr[c];
      multimem_st_v4(a.x_mc + (size_t)grow * a.H + 4 * c,
                     make_float4(xv.x + acc.x, xv.y + acc.y, xv.z + acc.z, xv.w + acc.w));
    }
  }
  fence_proxy_alias();     // every storing thread, before the CTA's release below
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    multimem_red_release_add_u64(a.flag_mc, 1ull);
  }
}

// Plain wait for the completion flag (before the residual is read raw, e.g. a tap).
__global__ void rs_wait_kernel(const unsigned long long* flag, unsigned long long target, int* err) {
  pdl_wait();
  pdl_trigger();
  wait_count(flag, target, err);
}

// RMSNorm of prefill rows after waiting for the residual's completion flag (one CTA per row, the
// arithmetic of rms_norm_rows_kernel in misc.cu).
template <int VPT>
__global__ void __launch_bounds__(256)
rms_norm_wait_kernel(const float* __restrict__ x, const float* __restrict__ w, int H, float eps,
                     __nv_bfloat16* __restrict__ out, long long ldo, const unsigned long long* flag,
                     unsigned long long target, int* err) {
  pdl_wait();
  pdl_trigger();
  wait_count(flag, target, err);
  const int r = blockIdx.x;
  const float* xr = x + (size_t)r * H;
  __shared__ float red[8];
  float v[VPT], wv[VPT];
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < VPT; ++u) {
    const int i = threadIdx.x + u * 256;
    v[u] = i < H ? xr[i] : 0.f;
    wv[u] = i < H ? w[i] : 0.f;
    ss += v[u] * v[u];
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

}  // namespace pfar
}  // namespace q38

// Reduce this rank's rows of a prefill all-reduce and broadcast them (see the file comment).
// Launched without programmatic dependent launch: its CTAs spin on peers, and must not hold SMs the
// preceding GEMM still needs.
void q38_rs_reduce_bcast(int64_t recv_local, int64_t count_local, int64_t count_target, torch::Tensor x,
                         int64_t x_mc, int64_t flag_mc, int64_t rank, int64_t world, int64_t rows_cap,
                         int64_t slots, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous() && x.dim() == 2, "contiguous fp32 residual");
  const int T = (int)x.size(0), H = (int)x.size(1);
  TORCH_CHECK(H % 4 == 0, "hidden must be a multiple of 4");
  q38::pfar::RedArgs a{};
  a.recv = reinterpret_cast<const float*>(recv_local);
  a.count = reinterpret_cast<const unsigned long long*>(count_local);
  a.count_target = (unsigned long long)count_target;
  a.x = x.data_ptr<float>();
  a.x_mc = reinterpret_cast<float*>(x_mc);
  a.flag_mc = reinterpret_cast<unsigned long long*>(flag_mc);
  a.rank = (int)rank;
  a.world = (int)world;
  a.rows_cap = (int)rows_cap;
  a.T = T;
  a.H = H;
  a.err = err.data_ptr<int>();
  TORCH_CHECK(slots >= 1 && slots <= rows_cap, "row slots outside the area");
  q38::pfar::rs_reduce_bcast_kernel<<<(unsigned)slots, q38::pfar::NT, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void q38_rs_wait(int64_t flag_local, int64_t target, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(err.device());
  q38::launch_pdl(q38::pfar::rs_wait_kernel, dim3(1), dim3(32), 0, at::cuda::getCurrentCUDAStream(),
                  reinterpret_cast<const unsigned long long*>(flag_local), (unsigned long long)target,
                  err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void q38_rms_norm_wait(torch::Tensor x, torch::Tensor w, double eps, torch::Tensor out, int64_t flag_local,
                       int64_t target, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous() && out.scalar_type() == at::kBFloat16 &&
                  out.stride(1) == 1, "fp32 residual, bf16 output");
  const int R = (int)x.size(0), H = (int)x.size(1);
  if (R == 0) return;
  const int v = (H + 255) / 256;
  TORCH_CHECK(v <= 32, "hidden above 8192");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto f = reinterpret_cast<const unsigned long long*>(flag_local);
#define Q38_NW(VV)                                                                                            \
  q38::launch_pdl(q38::pfar::rms_norm_wait_kernel<VV>, dim3(R), dim3(256), 0, st, (const float*)x.data_ptr<float>(), \
                  (const float*)w.data_ptr<float>(), H, (float)eps,                                              \
                  reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), (long long)out.stride(0), f,               \
                  (unsigned long long)target, err.data_ptr<int>());
  if (v <= 4) { Q38_NW(4) }
  else if (v <= 8) { Q38_NW(8) }
  else if (v <= 20) { Q38_NW(20) }
  else { Q38_NW(32) }
#undef Q38_NW
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
