// K-MARKOV: the drafter's sequential Markov selector in one persistent launch.
//
// Step i of a block picks  prev_{i+1} = argmax_v  logits[i][v] + pred[prev_i] . succ[v]
// (the DSpark selector: scripts/ci/dspark_markov.py:4-29; the reference pins one device program
// for the 15 steps, scripts/ci/dspark_markov_device.py:22-53).  pred [V, R] is replicated,
// succ [V_l, R] and the logits [P, V_l] are this rank's vocabulary shard.
//
// One CTA per SM stays resident for all P steps.  Per step every CTA stages pred[prev] (R fp32)
// in shared memory, scores its contiguous slice of the local vocabulary (a warp per row, 16-byte
// succ loads, the row's dot product reduced with a fixed xor butterfly), and publishes its best
// (value, index) record (double-buffered by step parity); one grid barrier later every CTA
// reduces the grid's records in the same order, so all hold the rank's winner: one barrier per
// step.  With W > 1 ranks, CTA 0 stores
// the winner into every rank's receive word for this step as one 64-bit word
// {value bits | 24-bit index | 8-bit epoch of this step's slot} (a 64-bit store is observed whole:
// no fence or flag; each step slot counts its own uses, so a slot never matches a stale epoch),
// and every CTA spins (bounded) on its local copies of the W words, then takes the global winner
// (ties: lowest index) as the next prev.  The per-step scoring arithmetic is the one of the
// two-launch step kernel it replaces (same dot-product order), so the selected ids are the same.
//
// Co-residency: the grid is at most one CTA per SM and the kernel is launched without
// programmatic dependent launch and never triggers its dependents early, so every CTA can be
// resident at once.  Every wait (grid barrier, peer words) is bounded by %globaltimer (2 s): on
// timeout the kernel records an error code and finishes its steps with what it has; the host reads
// the error word.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace q38 {
namespace markov {

constexpr int NT = 1024;
constexpr int MAX_RANKS = 8;
constexpr int SLICE_SMEM_MAX = 160 * 1024;   // succ slice kept in shared memory up to this size
constexpr int MAX_STEPS = 32;

struct Args {
  const float* logits;                 // [P, V_l], row stride ld
  long long ld;
  const __nv_bfloat16* pred;           // [V, R]
  const __nv_bfloat16* succ;           // [V_l, R]
  const int64_t* anchor;               // [1] global id
  int64_t* out;                        // [P] global ids
  int P, V_l, R;
  long long vocab_off;
  float* rec_val;                      // [2][gridDim] per-CTA records, double-buffered by step parity
  int* rec_idx;
  unsigned int* bar_count;             // grid barrier: arrivals (returns to 0) and generation
  unsigned int* bar_gen;
  // cross-rank exchange (world > 1): receive words [MAX_STEPS][MAX_RANKS] of every rank
  long long recv[MAX_RANKS];
  int rank, world;
  int* epoch;                          // [MAX_STEPS] per-step write counters of this rank's words
  int* err;
};

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

__device__ __forceinline__ unsigned ld_acquire_gpu_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64_m(const unsigned long long* a) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys_u64_m(unsigned long long* a, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}

// Sense-by-generation grid barrier (all CTAs resident).  Returns false when it gave up.
__device__ bool grid_barrier(const Args& a, bool ok) {
  __shared__ int ok_s;
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned g = ld_acquire_gpu_u32(a.bar_gen);
    __threadfence();
    if (atomicAdd(a.bar_count, 1u) == gridDim.x - 1) {
      *a.bar_count = 0;
      __threadfence();
      atomicAdd(a.bar_gen, 1u);
    } else if (ok) {                 // after a failure nobody waits again (the error is recorded)
      const unsigned long long t0 = globaltimer();
      while (ld_acquire_gpu_u32(a.bar_gen) == g) {
        if (globaltimer() - t0 > kWaitLimitNs) {
          record_error(a.err, kErrPeer);
          ok = false;
          break;
        }
      }
    }
    ok_s = ok;
  }
  __syncthreads();
  return ok_s != 0;
}

__global__ void __launch_bounds__(NT) markov_select_kernel(Args a, int slice_in_smem) {
  extern __shared__ float pp[];                        // pred[prev] as fp32 [R], then the succ slice
  __shared__ float wv[NT / 32];
  __shared__ int wi[NT / 32];
  __shared__ long long prev_s;
  __shared__ uint32_t ep_s[MAX_STEPS];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid < a.P) ep_s[tid] = (uint32_t)(a.epoch[tid] + 1) & 0xffu;   // read before the first barrier
  const int per = (a.V_l + gridDim.x - 1) / gridDim.x;
  const int v0 = blockIdx.x * per, v1 = min(a.V_l, v0 + per);
  long long prev = *a.anchor;
  bool ok = true;
  // this CTA's succ rows, staged once in shared memory when they fit (tensor-parallel shards)
  __nv_bfloat16* slice = reinterpret_cast<__nv_bfloat16*>(pp + a.R);
  if (slice_in_smem) {
    const int n16 = (v1 - v0) * a.R / 8;
    const uint4* src = reinterpret_cast<const uint4*>(a.succ + (size_t)v0 * a.R);
    for (int k = tid; k < n16; k += NT) reinterpret_cast<uint4*>(slice)[k] = src[k];
  }
  const int grp = tid >> 3, j = tid & 7;               // 8 lanes per row, NT / 8 rows in flight
  for (int i = 0; i < a.P; ++i) {
    for (int k = tid; k < a.R; k += NT) pp[k] = __bfloat162float(a.pred[(size_t)prev * a.R + k]);
    __syncthreads();
    const float* lrow = a.logits + (size_t)i * a.ld;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    // the trip count is uniform over the CTA (row groups past the slice score row v0 and discard
    // it): every lane of a warp reaches the row group's shuffles together
    for (int base = v0; base < v1; base += NT / 8) {
      const int v = base + grp;
      const bool valid = v < v1;
      const int vr = valid ? v : v0;
      const __nv_bfloat16* srow = slice_in_smem ? slice + (size_t)(vr - v0) * a.R : a.succ + (size_t)vr * a.R;
      const float sc = lrow[vr] + markov_row_dot(srow, pp, a.R, j);
      const int gv = (int)(vr + a.vocab_off);
      if (valid && better(sc, gv, best, bi)) { best = sc; bi = gv; }
    }
#pragma unroll
    for (int o = 16; o >= 8; o >>= 1) {                // the warp's four row groups
      const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(v2, i2, best, bi)) { best = v2; bi = i2; }
    }
    if (lane == 0) { wv[warp] = best; wi[warp] = bi; }
    __syncthreads();
    const int buf = (i & 1) * gridDim.x;
    if (tid == 0) {
      for (int w = 1; w < NT / 32; ++w)
        if (better(wv[w], wi[w], best, bi)) { best = wv[w]; bi = wi[w]; }
      a.rec_val[buf + blockIdx.x] = best;
      a.rec_idx[buf + blockIdx.x] = bi;
    }
    ok = grid_barrier(a, ok);
    // the rank's winner: every CTA reduces the records in the same order (warp 0)
    if (warp == 0) {
      float b = -INFINITY;
      int x = 0x7fffffff;
      for (int c = lane; c < (int)gridDim.x; c += 32) {
        const float v = __ldcg(a.rec_val + buf + c);
        const int id = __ldcg(a.rec_idx + buf + c);
        if (better(v, id, b, x)) { b = v; x = id; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, b, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, x, o);
        if (better(v2, i2, b, x)) { b = v2; x = i2; }
      }
      if (a.world > 1) {
        const uint32_t ep = ep_s[i];                                // this step slot's next use
        if (blockIdx.x == 0 && lane < a.world) {
          const unsigned long long w = ((unsigned long long)__float_as_uint(b) << 32) |
                                       ((unsigned long long)(x & 0xffffff) << 8) | ep;
          st_relaxed_sys_u64_m(reinterpret_cast<unsigned long long*>(a.recv[lane]) + i * MAX_RANKS + a.rank, w);
        }
        float gb = -INFINITY;
        int gx = 0x7fffffff;
        if (lane < a.world) {
          const unsigned long long* mine = reinterpret_cast<const unsigned long long*>(a.recv[a.rank]) +
                                           i * MAX_RANKS + lane;
          unsigned long long w = ld_relaxed_sys_u64_m(mine);
          const unsigned long long t0 = globaltimer();
          while ((uint32_t)(w & 0xffu) != ep) {
            if (globaltimer() - t0 > kWaitLimitNs) {
              record_error(a.err, kErrPeer);
              ok = false;
              break;
            }
            w = ld_relaxed_sys_u64_m(mine);
          }
          gb = __uint_as_float((uint32_t)(w >> 32));
          gx = (int)((w >> 8) & 0xffffff);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float v2 = __shfl_xor_sync(0xffffffffu, gb, o);
          const int i2 = __shfl_xor_sync(0xffffffffu, gx, o);
          if (better(v2, i2, gb, gx)) { gb = v2; gx = i2; }
        }
        b = gb;
        x = gx;
      }
      if (lane == 0) prev_s = x;
    }
    __syncthreads();
    prev = prev_s;
    if (blockIdx.x == 0 && tid == 0) a.out[i] = prev;
    // records are double-buffered by step parity: step i + 2 rewrites this step's buffer only
    // after every CTA has passed step i + 1's barrier, i.e. finished reading this step's records
  }
  // every CTA read the per-step epochs before the first step's barrier
  if (blockIdx.x == 0 && tid < a.P && a.world > 1) a.epoch[tid] = a.epoch[tid] + 1;
}

}  // namespace markov
}  // namespace q38

// logits [P, V_l] fp32, pred [V, R] bf16, succ [V_l, R] bf16, anchor [1] int64 (global id);
// out [P] int64.  state: int32 [4 + 32] scratch (barrier count, generation, 2 spare, per-step
// epochs of the cross-rank words), zeroed once.
// recv_ptrs: every rank's receive words (empty at one rank).
void q38_markov_select(torch::Tensor logits, torch::Tensor pred, torch::Tensor succ, torch::Tensor anchor,
                       torch::Tensor out, int64_t vocab_offset, torch::Tensor rec_val, torch::Tensor rec_idx,
                       torch::Tensor state, std::vector<int64_t> recv_ptrs, int64_t rank, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(logits.device());
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1, "fp32 logits, unit column stride");
  TORCH_CHECK(pred.scalar_type() == at::kBFloat16 && succ.scalar_type() == at::kBFloat16 && pred.is_contiguous() &&
                  succ.is_contiguous(), "contiguous bf16 pred / succ");
  const int P = (int)logits.size(0), V_l = (int)logits.size(1), R = (int)succ.size(1);
  TORCH_CHECK(succ.size(0) == V_l && pred.size(1) == R && R % 8 == 0 && R <= 4096, "pred/succ shapes");
  TORCH_CHECK(P >= 1 && P <= q38::markov::MAX_STEPS, "1..32 steps");
  TORCH_CHECK(pred.size(0) + 0 < (1 << 24), "vocabulary ids must fit in 24 bits");
  TORCH_CHECK(anchor.scalar_type() == at::kLong && out.scalar_type() == at::kLong && out.numel() >= P, "int64 ids");
  TORCH_CHECK(state.scalar_type() == at::kInt && state.numel() >= 4 + q38::markov::MAX_STEPS, "int32 state [36]");
  const int world = recv_ptrs.empty() ? 1 : (int)recv_ptrs.size();
  TORCH_CHECK(world <= q38::markov::MAX_RANKS, "1..8 ranks");
  int grid = std::min(q38::device_sms(), std::max(1, (V_l + 63) / 64));
  TORCH_CHECK(rec_val.numel() >= 2 * grid && rec_idx.numel() >= 2 * grid, "record buffers too small");
  q38::markov::Args a{};
  a.logits = logits.data_ptr<float>();
  a.ld = logits.stride(0);
  a.pred = reinterpret_cast<const __nv_bfloat16*>(pred.data_ptr());
  a.succ = reinterpret_cast<const __nv_bfloat16*>(succ.data_ptr());
  a.anchor = anchor.data_ptr<int64_t>();
  a.out = out.data_ptr<int64_t>();
  a.P = P;
  a.V_l = V_l;
  a.R = R;
  a.vocab_off = vocab_offset;
  a.rec_val = rec_val.data_ptr<float>();
  a.rec_idx = rec_idx.data_ptr<int>();
  int* st = state.data_ptr<int>();
  a.bar_count = reinterpret_cast<unsigned int*>(st);
  a.bar_gen = reinterpret_cast<unsigned int*>(st + 1);
  a.epoch = st + 4;
  for (int p = 0; p < world && !recv_ptrs.empty(); ++p) a.recv[p] = recv_ptrs[p];
  a.rank = (int)rank;
  a.world = world;
  a.err = err.data_ptr<int>();
  const int per = (V_l + grid - 1) / grid;
  const size_t slice_bytes = (size_t)per * R * 2;
  const int in_smem = slice_bytes <= (size_t)q38::markov::SLICE_SMEM_MAX ? 1 : 0;
  const size_t smem = (size_t)R * sizeof(float) + (in_smem ? slice_bytes : 0);
  TORCH_CHECK(q38::set_smem_once<q38::markov::markov_select_kernel>((int)(R * sizeof(float) +
                                                                         q38::markov::SLICE_SMEM_MAX)) == cudaSuccess,
              "cudaFuncSetAttribute failed");
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  // plain launch: no programmatic dependent launch, so no later kernel takes an SM this grid needs
  q38::markov::markov_select_kernel<<<grid, q38::markov::NT, smem, s>>>(a, in_smem);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
