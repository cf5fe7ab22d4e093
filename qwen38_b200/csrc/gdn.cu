// Gated DeltaNet recurrence kernels (K-GDN-DECODE / commit / sequential prefill).
//
// Per value head h (one CTA) and row t:
//   conv:  u_t = silu(sum_j w[c, j] * x[t - (K-1) + j, c])  over the head's q, k (shared by the
//          GQA group) and v channels, x = [window (K-1 rows) ; projected rows]
//   q_t = l2norm(u_q) * Dk^-0.5, k_t = l2norm(u_k), v_t = u_v
//   g_t = -exp(A_log[h]) * softplus(a_t + dt_bias[h]),  beta_t = sigmoid(b_t)
//   S <- exp(g_t) S;  S <- S + k_t (beta_t (v_t - S^T k_t))^T;  o_t = S^T q_t
//   out_t = rmsnorm(o_t) * norm_w * silu(z_t)
// (reference: docker/qwen-c2-graft/graft/gdn/tp.py:540-730 prefill, :1176-1408 decode;
//  scripts/ci/gdn_seq_block_device_test.py:431-456 fp64 recurrence).
//
// Layout: 4 threads per value column c; thread (c, p) keeps S[p*D/4 .. p*D/4 + D/4)[c] in
// registers.  S^T k and S^T q are reduced across the 4 threads with a fixed xor butterfly, so the
// arithmetic of row t is identical whether it runs inside a verify block, a commit replay or a
// single-row decode: verify outputs match sequential decode bit for bit and commit publishes
// exactly the state sequential decode would have produced.
//
// Modes: WRITE_OUT (verify, prefill) and WRITE_STATE (commit, prefill).  Rows are processed in
// sub-blocks of SUB rows staged in shared memory.  The row count may come from device memory
// (commit: the accepted prefix length, so the launch can live inside a CUDA graph).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace q38 {

struct GdnArgs {
  const __nv_bfloat16* proj;   // [rows, in_width] layer 0; + layer * proj_layer_stride
  long long proj_ld, proj_layer_stride;
  const __nv_bfloat16* window; // [K-1, C] (+ layer stride)
  long long win_layer_stride;
  float* state;                // [nv, D, D] (+ layer stride)
  long long state_layer_stride;
  const float* conv_w;         // [C, K] (+ layer stride)
  long long convw_layer_stride;
  const float* A_log;          // [nv] (+ layer stride nv)
  const float* dt_bias;
  const float* norm_w;         // [D] (+ layer stride D)
  __nv_bfloat16* out;          // [rows, nv*D]
  long long out_ld;
  int rows;                    // used when rows_dev == nullptr
  const int* rows_dev;         // device row count (commit)
  int nk, nv, C;               // local key heads, value heads, conv channels
  float eps;
};

template <int D, int KC, int SUB, bool WRITE_OUT, bool WRITE_STATE>
__global__ void __launch_bounds__(4 * D)
gdn_recurrent_kernel(GdnArgs a) {
  constexpr int NT = 4 * D;
  constexpr int RPT = D / 4;     // state rows per thread
  const int h = blockIdx.x;
  const int layer = blockIdx.y;
  const int tid = threadIdx.x;
  const int col = tid >> 2, part = tid & 3;
  const int rep = a.nv / a.nk;
  const int kh = h / rep;

  const __nv_bfloat16* __restrict__ proj = a.proj + layer * a.proj_layer_stride;
  const __nv_bfloat16* __restrict__ window = a.window + layer * a.win_layer_stride;
  float* __restrict__ state = a.state + layer * a.state_layer_stride + (size_t)h * D * D;
  const float* __restrict__ conv_w = a.conv_w + layer * a.convw_layer_stride;
  __nv_bfloat16* __restrict__ outp = a.out;
  const float A = -__expf(a.A_log[layer * a.nv + h]);
  const float dtb = a.dt_bias[layer * a.nv + h];
  const float* norm_w = a.norm_w + layer * D;

  // channel offsets of this head inside [q | k | v | z | b | a]
  const int cq = kh * D, ck = a.nk * D + kh * D, cv = 2 * a.nk * D + h * D;
  const int cz = a.C + h * D, cb = a.C + a.nv * D + h, ca = a.C + a.nv * D + a.nv + h;

  // q/k rows are read by the 4 threads of a column at quarter offsets: pad each quarter by 4 floats
  // so the quarters fall in different banks.
  constexpr int QP = RPT + 4;
  __shared__ __align__(16) float q_s[SUB][4 * QP], k_s[SUB][4 * QP];
  __shared__ float v_s[SUB][D];
  __shared__ float g_s[SUB], b_s[SUB];
  __shared__ float o_s[SUB][D];
  __shared__ float red_s[SUB][2][NT / 32];

  // conv taps are static; everything else may come from the previous kernel
  float wq[KC], wk[KC], wv[KC];
#pragma unroll
  for (int j = 0; j < KC; ++j) {
    wq[j] = conv_w[(size_t)(cq + col) * KC + j];
    wk[j] = conv_w[(size_t)(ck + col) * KC + j];
    wv[j] = conv_w[(size_t)(cv + col) * KC + j];
  }
  pdl_wait();
  pdl_trigger();
  const int rows = a.rows_dev ? *a.rows_dev : a.rows;

  // state registers
  float S[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) S[i] = state[(size_t)(part * RPT + i) * D + col];


  auto x_at = [&](int r, int ch) -> float {   // r in [-(K-1), rows)
    if (r < 0) return __bfloat162float(window[(size_t)(r + KC - 1) * a.C + ch]);
    return __bfloat162float(proj[(size_t)r * a.proj_ld + ch]);
  };

  const int qidx = (col / RPT) * QP + (col % RPT);   // padded slot of channel `col`
  for (int r0 = 0; r0 < rows; r0 += SUB) {
    const int nsub = min(SUB, rows - r0);
    // ---- prologue: conv + silu for q/k/v channel `col`, split rows over the 4 parts
#pragma unroll
    for (int tt = 0; tt < SUB / 4; ++tt) {
      const int t = part + 4 * tt;
      if (t >= nsub) break;
      const int r = r0 + t;
      float xq[KC], xk[KC], xv[KC];
#pragma unroll
      for (int j = 0; j < KC; ++j) {          // issue all loads before the arithmetic
        const int rr = r - (KC - 1) + j;
        xq[j] = x_at(rr, cq + col);
        xk[j] = x_at(rr, ck + col);
        xv[j] = x_at(rr, cv + col);
      }
      float sq = 0.f, sk = 0.f, sv = 0.f;
#pragma unroll
      for (int j = 0; j < KC; ++j) {
        sq += wq[j] * xq[j];
        sk += wk[j] * xk[j];
        sv += wv[j] * xv[j];
      }
      q_s[t][qidx] = silu_f(sq);
      k_s[t][qidx] = silu_f(sk);
      v_s[t][col] = silu_f(sv);
    }
    if (tid < nsub) {
      const int r = r0 + tid;
      const float av = __bfloat162float(proj[(size_t)r * a.proj_ld + ca]);
      const float bv = __bfloat162float(proj[(size_t)r * a.proj_ld + cb]);
      const float sp = (av + dtb) > 20.f ? (av + dtb) : log1pf(__expf(av + dtb));
      g_s[tid] = A * sp;
      b_s[tid] = 1.f / (1.f + __expf(-bv));
    }
    __syncthreads();
    // ---- L2 norms of q and k per row (fixed-order block reduction)
    {
      const int warp = tid >> 5, lane = tid & 31;
      for (int t = 0; t < nsub; ++t) {
        float pq = 0.f, pk = 0.f;
        for (int c = tid; c < D; c += NT) {
          const int ci = (c / RPT) * QP + (c % RPT);
          pq += q_s[t][ci] * q_s[t][ci];
          pk += k_s[t][ci] * k_s[t][ci];
        }
        pq = warp_sum(pq);
        pk = warp_sum(pk);
        if (lane == 0) { red_s[t][0][warp] = pq; red_s[t][1][warp] = pk; }
      }
      __syncthreads();
      if (tid < nsub) {
        float sq = 0.f, sk = 0.f;
        for (int w = 0; w < NT / 32; ++w) { sq += red_s[tid][0][w]; sk += red_s[tid][1][w]; }
        red_s[tid][0][0] = rsqrtf(sq + 1e-6f) * rsqrtf((float)D);
        red_s[tid][1][0] = rsqrtf(sk + 1e-6f);
      }
      __syncthreads();
      for (int t = 0; t < nsub; ++t) {
        for (int c = tid; c < D; c += NT) {
          const int ci = (c / RPT) * QP + (c % RPT);
          q_s[t][ci] *= red_s[t][0][0];
          k_s[t][ci] *= red_s[t][1][0];
        }
      }
      __syncthreads();
    }
    // ---- sequential recurrence
    for (int t = 0; t < nsub; ++t) {
      const float decay = __expf(g_s[t]);
      float kv = 0.f;
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        S[i] *= decay;
        kv += S[i] * k_s[t][part * QP + i];
      }
      kv += __shfl_xor_sync(0xffffffffu, kv, 1);
      kv += __shfl_xor_sync(0xffffffffu, kv, 2);
      const float delta = (v_s[t][col] - kv) * b_s[t];
      float o = 0.f;
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        S[i] += k_s[t][part * QP + i] * delta;
        o += S[i] * q_s[t][part * QP + i];
      }
      if constexpr (WRITE_OUT) {
        o += __shfl_xor_sync(0xffffffffu, o, 1);
        o += __shfl_xor_sync(0xffffffffu, o, 2);
        if (part == 0) o_s[t][col] = o;
      }
    }
    if constexpr (WRITE_OUT) {
      __syncthreads();
      // ---- gated RMSNorm epilogue
      const int warp = tid >> 5, lane = tid & 31;
      for (int t = 0; t < nsub; ++t) {
        float ss = 0.f;
        for (int c = tid; c < D; c += NT) ss += o_s[t][c] * o_s[t][c];
        ss = warp_sum(ss);
        if (lane == 0) red_s[t][0][warp] = ss;
      }
      __syncthreads();
      if (tid < nsub) {
        float s = 0.f;
        for (int w = 0; w < NT / 32; ++w) s += red_s[tid][0][w];
        red_s[tid][1][0] = rsqrtf(s / D + a.eps);
      }
      __syncthreads();
      constexpr int PER = (SUB * D + NT - 1) / NT;
      float zv[PER];
#pragma unroll
      for (int u = 0; u < PER; ++u) {            // issue every z load before any store
        const int idx = tid + u * NT;
        const int t = idx / D, c = idx % D;
        zv[u] = (t < nsub) ? __bfloat162float(proj[(size_t)(r0 + t) * a.proj_ld + cz + c]) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int idx = tid + u * NT;
        const int t = idx / D, c = idx % D;
        if (t < nsub) {
          const float y = o_s[t][c] * red_s[t][1][0] * norm_w[c] * silu_f(zv[u]);
          outp[(size_t)(r0 + t) * a.out_ld + (size_t)h * D + c] = __float2bfloat16(y);
        }
      }
    }
    __syncthreads();
  }
  if constexpr (WRITE_STATE) {
#pragma unroll
    for (int i = 0; i < RPT; ++i) state[(size_t)(part * RPT + i) * D + col] = S[i];
  }
}

// Conv window after consuming `rows` projected rows: the last K-1 inputs of [window ; proj].
template <int KC>
__global__ void gdn_window_kernel(const __nv_bfloat16* __restrict__ proj, long long proj_ld,
                                  long long proj_layer_stride, __nv_bfloat16* window, long long win_layer_stride,
                                  int C, int rows, const int* rows_dev) {
  const int layer = blockIdx.y;
  const int ch = blockIdx.x * blockDim.x + threadIdx.x;
  pdl_wait();
  pdl_trigger();
  if (ch >= C) return;
  const int n = rows_dev ? *rows_dev : rows;
  if (n <= 0) return;
  const __nv_bfloat16* p = proj + layer * proj_layer_stride;
  __nv_bfloat16* w = window + layer * win_layer_stride;
  __nv_bfloat16 full[2 * KC];
#pragma unroll
  for (int j = 0; j < KC - 1; ++j) {
    const int r = n - (KC - 1) + j;   // index into [window ; proj]
    full[j] = r < 0 ? w[(size_t)(r + KC - 1) * C + ch] : p[(size_t)r * proj_ld + ch];
  }
#pragma unroll
  for (int j = 0; j < KC - 1; ++j) w[(size_t)j * C + ch] = full[j];
}

}  // namespace q38

// ----------------------------------------------------------------------------- bindings
// mode: 0 = verify (outputs, state untouched), 1 = commit (state + window, rows from rows_dev),
//       2 = prefill (outputs + state + window)
void q38_gdn_recurrent(int64_t mode, torch::Tensor proj, torch::Tensor window, torch::Tensor state,
                       torch::Tensor conv_w, torch::Tensor A_log, torch::Tensor dt_bias, torch::Tensor norm_w,
                       c10::optional<torch::Tensor> out, int64_t rows, c10::optional<torch::Tensor> rows_dev,
                       int64_t nk, int64_t nv, int64_t D, double eps) {
  c10::cuda::CUDAGuard guard(proj.device());
  // Per-layer tensors may carry a leading layer dimension (commit of every layer in one launch).
  const bool multi = state.dim() == 4;
  const int layers = multi ? (int)state.size(0) : 1;
  TORCH_CHECK(proj.scalar_type() == at::kBFloat16 && window.scalar_type() == at::kBFloat16, "bf16 proj/window");
  TORCH_CHECK(state.scalar_type() == at::kFloat, "fp32 state");
  const int KC = (int)conv_w.size(-1);
  const int C = (int)conv_w.size(-2);
  q38::GdnArgs a{};
  a.proj = reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr());
  a.proj_ld = proj.stride(-2);
  a.proj_layer_stride = multi ? proj.stride(0) : 0;
  a.window = reinterpret_cast<const __nv_bfloat16*>(window.data_ptr());
  a.win_layer_stride = multi ? window.stride(0) : 0;
  a.state = state.data_ptr<float>();
  a.state_layer_stride = multi ? state.stride(0) : 0;
  a.conv_w = conv_w.data_ptr<float>();
  a.convw_layer_stride = multi ? conv_w.stride(0) : 0;
  a.A_log = A_log.data_ptr<float>();
  a.dt_bias = dt_bias.data_ptr<float>();
  a.norm_w = norm_w.data_ptr<float>();
  a.out = out ? reinterpret_cast<__nv_bfloat16*>(out->data_ptr()) : nullptr;
  a.out_ld = out ? out->stride(0) : 0;
  a.rows = (int)rows;
  a.rows_dev = rows_dev ? rows_dev->data_ptr<int>() : nullptr;
  a.nk = (int)nk;
  a.nv = (int)nv;
  a.C = C;
  a.eps = (float)eps;
  TORCH_CHECK(KC == 4, "conv kernel size 4 supported");
  TORCH_CHECK(mode != 0 || out, "verify needs an output");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  dim3 grid((unsigned)nv, (unsigned)layers);
#define Q38_GDN_LAUNCH(DD)                                                                              \
  if (mode == 0) q38::launch_pdl(q38::gdn_recurrent_kernel<DD, 4, 16, true, false>, grid, dim3(4 * DD), 0, st, a); \
  else if (mode == 1) q38::launch_pdl(q38::gdn_recurrent_kernel<DD, 4, 16, false, true>, grid, dim3(4 * DD), 0, st, a); \
  else q38::launch_pdl(q38::gdn_recurrent_kernel<DD, 4, 16, true, true>, grid, dim3(4 * DD), 0, st, a);
  if (D == 128) { Q38_GDN_LAUNCH(128) }
  else if (D == 32) { Q38_GDN_LAUNCH(32) }
  else TORCH_CHECK(false, "GDN head dim 32 or 128 supported");
#undef Q38_GDN_LAUNCH
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (mode != 0) {
    dim3 g2((unsigned)((C + 255) / 256), (unsigned)layers);
    q38::launch_pdl(q38::gdn_window_kernel<4>, g2, dim3(256), 0, st, a.proj, a.proj_ld, a.proj_layer_stride,
                    reinterpret_cast<__nv_bfloat16*>(window.data_ptr()), a.win_layer_stride, C, (int)rows,
                    a.rows_dev);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}
