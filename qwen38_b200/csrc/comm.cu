// In-kernel tensor-parallel collectives over NVLink / NVSwitch peer memory.
//
// Every rank owns one cudaMalloc'd "peer buffer" whose CUDA IPC handle is exchanged once over the
// process group; each rank maps every peer's buffer and keeps the W base pointers on the device.
// A buffer holds data slots (one per collective call site, so a slot is reused only after a full
// step has gone by on every rank) and flag words.
//
// allreduce_residual: the row-parallel GEMM wrote this rank's fp32 partial [rows, H] into its own
// slot; the kernel runs a per-CTA barrier (each CTA stores its epoch into every peer's flag word
// for (slot, cta, this rank) with release semantics at system scope, then waits with acquire loads
// until all W flags for (slot, cta) reach the epoch), then sums the W partials in rank order
// 0..W-1 (identical bits on every rank) and adds the sum into the replicated fp32 residual.
// argmax_allreduce: the same barrier on (value, index) pairs; ties take the lowest index.
//
// Waits are bounded by %globaltimer (2 s); on timeout the CTA records kErrPeer in the device error
// word and returns without touching the output.  The reference's TT-CCL all-reduce / all-gather
// calls (graft/gdn/tp.py:1399, graft/mlp.py:619, qwen36_model.py:495-510) map onto these.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace q38 {
namespace comm {

constexpr int MAX_RANKS = 8;
constexpr int AR_CTAS = 32;          // CTAs per all-reduce launch (flag words per slot and rank)

struct PeerPtrs {
  int64_t p[MAX_RANKS];
};


// Per-CTA barrier across ranks for (slot, cta).  flag word layout in every rank's buffer:
// flags[(slot * AR_CTAS + cta) * MAX_RANKS + src].  Returns false on timeout.
__device__ bool cta_barrier(const PeerPtrs& flag_base, int rank, int world, int slot, int cta, int* epochs,
                            int* err) {
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    const int e = epochs[slot * AR_CTAS + cta] + 1;
    __threadfence_system();
    for (int p = 0; p < world; ++p) {
      int* f = reinterpret_cast<int*>(flag_base.p[p]) + (slot * AR_CTAS + cta) * MAX_RANKS + rank;
      st_release_sys(f, e);
    }
    const int* mine = reinterpret_cast<const int*>(flag_base.p[rank]) + (slot * AR_CTAS + cta) * MAX_RANKS;
    bool ok = true;
    unsigned long long t0 = globaltimer();
    for (int p = 0; p < world && ok; ++p) {
      while (ld_acquire_sys(mine + p) < e) {
        if (globaltimer() - t0 > kWaitLimitNs) {
          record_error(err, kErrPeer);
          ok = false;
          break;
        }
      }
    }
    if (ok) epochs[slot * AR_CTAS + cta] = e;
    ok_s = ok;
  }
  __syncthreads();
  return ok_s != 0;
}

__global__ void __launch_bounds__(256) allreduce_residual_kernel(PeerPtrs data, PeerPtrs flags, int rank, int world,
                                                                 int slot, size_t slot_floats, int n,
                                                                 float* __restrict__ residual, int* epochs,
                                                                 int* err) {
  pdl_wait();
  pdl_trigger();
  if (!cta_barrier(flags, rank, world, slot, blockIdx.x, epochs, err)) return;
  const int n4 = n / 4;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < MAX_RANKS; ++p) {
      if (p >= world) break;
      const float4 v = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(data.p[p]) +
                                                       (size_t)slot * slot_floats)[i];
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    float4 r = reinterpret_cast<float4*>(residual)[i];
    r.x += acc.x; r.y += acc.y; r.z += acc.z; r.w += acc.w;
    reinterpret_cast<float4*>(residual)[i] = r;
  }
}

// (value, index) per row: every rank writes its pair into its own slot, barrier, then picks the
// best over ranks (ties -> lowest index).  `out` gets the global index (int64).
__global__ void argmax_allreduce_kernel(PeerPtrs data, PeerPtrs flags, int rank, int world, int slot,
                                        size_t slot_floats, int rows, const float* __restrict__ val,
                                        const int64_t* __restrict__ idx, int64_t* __restrict__ out, int* epochs,
                                        int* err) {
  pdl_wait();
  pdl_trigger();
  float* mine = reinterpret_cast<float*>(data.p[rank]) + (size_t)slot * slot_floats;
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    mine[2 * r] = val[r];
    reinterpret_cast<int*>(mine)[2 * r + 1] = (int)idx[r];
  }
  __syncthreads();
  if (!cta_barrier(flags, rank, world, slot, 0, epochs, err)) return;
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int p = 0; p < world; ++p) {
      const float* s = reinterpret_cast<const float*>(data.p[p]) + (size_t)slot * slot_floats;
      const float v = s[2 * r];
      const int i = reinterpret_cast<const int*>(s)[2 * r + 1];
      if (v > best || (v == best && i < bi)) { best = v; bi = i; }
    }
    out[r] = bi;
  }
}

}  // namespace comm
}  // namespace q38

// ----------------------------------------------------------------------------- host side
torch::Tensor q38_peer_alloc(int64_t bytes, int64_t device) {
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  void* p = nullptr;
  TORCH_CHECK(cudaMalloc(&p, (size_t)bytes) == cudaSuccess, "cudaMalloc of the peer buffer failed");
  TORCH_CHECK(cudaMemset(p, 0, (size_t)bytes) == cudaSuccess, "cudaMemset failed");
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device);
  return torch::from_blob(p, {bytes}, [](void* q) { cudaFree(q); }, opts);
}

torch::Tensor q38_ipc_handle(torch::Tensor buf) {
  cudaIpcMemHandle_t h;
  TORCH_CHECK(cudaIpcGetMemHandle(&h, buf.data_ptr()) == cudaSuccess, "cudaIpcGetMemHandle failed");
  auto t = torch::empty({(int64_t)sizeof(h)}, torch::kUInt8);
  memcpy(t.data_ptr(), &h, sizeof(h));
  return t;
}

int64_t q38_ipc_open(torch::Tensor handle, int64_t device) {
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  cudaIpcMemHandle_t h;
  TORCH_CHECK(handle.numel() == sizeof(h), "bad IPC handle");
  memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  TORCH_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess,
              "cudaIpcOpenMemHandle failed");
  return reinterpret_cast<int64_t>(p);
}

void q38_ipc_close(int64_t ptr) { cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)); }

static q38::comm::PeerPtrs to_ptrs(const std::vector<int64_t>& v, int64_t add) {
  TORCH_CHECK(v.size() <= q38::comm::MAX_RANKS, "at most 8 ranks");
  q38::comm::PeerPtrs p{};
  for (size_t i = 0; i < v.size(); ++i) p.p[i] = v[i] + add;
  return p;
}

// data_ptrs / flag_ptrs: base addresses (peer buffers mapped into this process) of every rank's
// data and flag regions.  `residual` [rows, H] fp32 gets += sum over ranks of slot `slot`.
void q38_allreduce_residual(std::vector<int64_t> data_ptrs, std::vector<int64_t> flag_ptrs, int64_t rank,
                            int64_t slot, int64_t slot_floats, torch::Tensor residual, torch::Tensor epochs,
                            torch::Tensor err) {
  c10::cuda::CUDAGuard guard(residual.device());
  TORCH_CHECK(residual.scalar_type() == at::kFloat && residual.is_contiguous(), "contiguous fp32 residual");
  const int n = (int)residual.numel();
  TORCH_CHECK(n % 4 == 0 && n <= slot_floats, "residual larger than a slot");
  const int world = (int)data_ptrs.size();
  q38::launch_pdl(q38::comm::allreduce_residual_kernel, dim3(q38::comm::AR_CTAS), dim3(256), 0,
                  at::cuda::getCurrentCUDAStream(), to_ptrs(data_ptrs, 0), to_ptrs(flag_ptrs, 0), (int)rank, world,
                  (int)slot, (size_t)slot_floats, n, residual.data_ptr<float>(), epochs.data_ptr<int>(),
                  err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void q38_argmax_allreduce(std::vector<int64_t> data_ptrs, std::vector<int64_t> flag_ptrs, int64_t rank,
                          int64_t slot, int64_t slot_floats, torch::Tensor val, torch::Tensor idx, torch::Tensor out,
                          torch::Tensor epochs, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(val.device());
  const int rows = (int)val.numel();
  TORCH_CHECK(2 * rows <= slot_floats, "too many rows for a slot");
  const int world = (int)data_ptrs.size();
  q38::launch_pdl(q38::comm::argmax_allreduce_kernel, dim3(1), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
                  to_ptrs(data_ptrs, 0), to_ptrs(flag_ptrs, 0), (int)rank, world, (int)slot, (size_t)slot_floats,
                  rows, (const float*)val.data_ptr<float>(), (const int64_t*)idx.data_ptr<int64_t>(),
                  out.data_ptr<int64_t>(), epochs.data_ptr<int>(), err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
