// Gated DeltaNet recurrence kernels (K-GDN-DECODE / commit / sequential prefill).
//
// Per value head h (a cluster of CTAs, one slice of value columns each) and row t:
//   conv:  u_t = silu(sum_j w[c, j] * x[t - (K-1) + j, c])  over the head's q, k (shared by the
//          GQA group) and v channels, x = [window (K-1 rows) ; projected rows]
//   q_t = l2norm(u_q) * Dk^-0.5, k_t = l2norm(u_k), v_t = u_v
//   g_t = -exp(A_log[h]) * softplus(a_t + dt_bias[h]),  beta_t = sigmoid(b_t)
//   S <- exp(g_t) S;  S <- S + k_t (beta_t (v_t - S^T k_t))^T;  o_t = S^T q_t
//   out_t = rmsnorm(o_t) * norm_w * silu(z_t)
// (reference: docker/qwen-c2-graft/graft/gdn/tp.py:540-730 prefill, :1176-1408 decode;
//  scripts/ci/gdn_seq_block_device_test.py:431-456 fp64 recurrence).
//
// Layout: a head's D value columns are split over SPLIT CTAs of one thread-block cluster (D=128:
// 4 CTAs of 32 columns, so a layer's 48 heads fill 192 SMs' worth of CTAs instead of 48).  The
// columns of the state evolve independently; only the gated RMSNorm needs whole-row statistics,
// which the cluster exchanges through distributed shared memory (each CTA stores its partial sum
// of squares into every peer's buffer, one cluster barrier, then every CTA adds the SPLIT
// partials in cluster-rank order).  Inside a CTA, 4 threads own a value column c; thread (c, p)
// keeps S[p*D/4 .. p*D/4 + D/4)[c] in registers.  S^T k and S^T q are reduced with a fixed xor
// butterfly and a fixed 4-way partial-sum split, so the arithmetic of row t is identical whether
// it runs inside a verify block, a commit replay or a single-row decode: verify outputs match
// sequential decode bit for bit and commit publishes exactly the state sequential decode would
// have produced.
//
// Each sub-block of SUB rows first stages its raw projected rows (q and k channels of the head's
// key group, this CTA's v and z columns, for rows r0-(K-1) .. r0+SUB-1) in shared memory with
// 16-byte asynchronous copies (4-byte ones when a row is not 16-byte aligned), so the conv, the
// norms and the epilogue read only shared memory.  Thread c < D convolves q channel c and k
// channel c for every row in registers and the row L2 norms come from one butterfly per row, so q
// and k reach shared memory once, normalised.  The recurrence folds the decay into the state
// update: S <- decay S + k (beta (v - decay S^T k))^T.
//
// Modes: WRITE_OUT (verify, prefill) and WRITE_STATE (commit, prefill).  The row count may come
// from device memory (commit: the accepted prefix length, so the launch can live inside a CUDA
// graph).
#include <cooperative_groups.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace q38 {

namespace cg = cooperative_groups;

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
  unsigned long long* trace;   // optional per-CTA %globaltimer stamps [grid][8] (micro-benchmarks)
  int vec16;                   // rows and channel groups 16-byte aligned: stage with 16-byte copies
};

// trace points: 0 entry, 1 past the PDL wait, 2 first sub-block staged, 3 conv + norms done,
// 4 recurrence done, 5 norm statistics exchanged, 6 outputs written, 7 exit
#define Q38_GSTAMP(k)                                                                                  \
  do {                                                                                                 \
    if (a.trace && threadIdx.x == 0 && (r0 == 0 || (k) >= 7))                                          \
      a.trace[((size_t)blockIdx.y * gridDim.x + blockIdx.x) * 8 + (k)] = globaltimer();                \
  } while (0)

template <int D, int SPLIT>
struct GdnShape {
  static constexpr int COLS = D / SPLIT;     // value columns per CTA
  static constexpr int NT = 4 * COLS;        // threads per CTA
  static constexpr int RPT = D / 4;          // state rows per thread
  static constexpr int QP = RPT + 4;         // padded quarter of a q/k row (bank spread)
  static constexpr int RAWW = 2 * D + 2 * COLS;   // staged channels: q | k | v slice | z slice
};

template <int D, int KC, int SUB, bool WRITE_OUT, bool WRITE_STATE, int SPLIT>
__global__ void __launch_bounds__(GdnShape<D, SPLIT>::NT)
gdn_recurrent_kernel(GdnArgs a) {
  using G = GdnShape<D, SPLIT>;
  constexpr int COLS = G::COLS, NT = G::NT, RPT = G::RPT, QP = G::QP, RAWW = G::RAWW;
  static_assert(NT == 128 && SUB * 8 == NT, "128 threads: 16 rows x 8 lanes in the row reductions");
  constexpr int NPR = 8;                       // threads per row in row reductions
  const int h = blockIdx.x / SPLIT, sl = blockIdx.x % SPLIT;   // sl == rank in the cluster
  const int layer = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int col = tid >> 2, part = tid & 3;
  const int gcol = sl * COLS + col;            // value column inside the head
  const int rep = a.nv / a.nk;
  const int kh = h / rep;

  const __nv_bfloat16* __restrict__ proj = a.proj + layer * a.proj_layer_stride;
  const __nv_bfloat16* __restrict__ window = a.window + layer * a.win_layer_stride;
  float* __restrict__ state = a.state + layer * a.state_layer_stride + (size_t)h * D * D;
  const float* __restrict__ conv_w = a.conv_w + layer * a.convw_layer_stride;
  const float A = -__expf(a.A_log[layer * a.nv + h]);
  const float dtb = a.dt_bias[layer * a.nv + h];
  const float* norm_w = a.norm_w + layer * D;

  // channel offsets inside [q | k | v | z | b | a]
  const int cq = kh * D, ck = a.nk * D + kh * D, cv = 2 * a.nk * D + h * D + sl * COLS;
  const int cz = a.C + h * D + sl * COLS, cb = a.C + a.nv * D + h, ca = a.C + a.nv * D + a.nv + h;

  __shared__ __align__(16) __nv_bfloat16 raw[SUB + KC - 1][RAWW];
  __shared__ __align__(16) float q_s[SUB][4 * QP], k_s[SUB][4 * QP];
  __shared__ float v_s[SUB][COLS];
  __shared__ float o_s[SUB][COLS];
  __shared__ float g_s[SUB], b_s[SUB], rs_s[SUB];
  __shared__ float ssq_s[SUB][4], ssk_s[SUB][4];   // per-warp row sums of squares of q and k
  __shared__ float ss_part[2][SPLIT][SUB];     // DSMEM targets, double-buffered by sub-block parity

  // conv taps are static; everything else may come from the previous kernel
  static_assert(D <= NT && D % 32 == 0, "thread c < D owns q channel c and k channel c");
  float wq[KC], wk[KC], wv[KC];            // conv taps: this thread's q and k channels, v column
#pragma unroll
  for (int j = 0; j < KC; ++j) {
    wq[j] = tid < D ? conv_w[(size_t)(cq + tid) * KC + j] : 0.f;
    wk[j] = tid < D ? conv_w[(size_t)(ck + tid) * KC + j] : 0.f;
  }
#pragma unroll
  for (int j = 0; j < KC; ++j) wv[j] = conv_w[(size_t)(cv + col) * KC + j];
  // The recurrent state is written only by commit / prefill launches that completed before the
  // kernel this one follows began its own wait (every kernel of a step waits on its predecessor
  // before triggering its successor, except the GEMM, whose predecessor does), so it is read
  // before griddepcontrol.wait: its DRAM round trip overlaps the previous kernel's tail.
  int r0 = 0;
  Q38_GSTAMP(0);
  float S[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) S[i] = state[(size_t)(part * RPT + i) * D + gcol];
  pdl_wait();
  Q38_GSTAMP(1);
  pdl_trigger();
  const int rows = a.rows_dev ? *a.rows_dev : a.rows;

  cg::cluster_group cluster = cg::this_cluster();
  int parity = 0;
  for (r0 = 0; r0 < rows; r0 += SUB, parity ^= 1) {
    const int nsub = min(SUB, rows - r0);
    // ---- 1. stage raw rows r0-(K-1) .. r0+nsub-1 with 16-byte asynchronous copies (channel
    //         groups of 8 are 16-byte aligned in proj and window); z only for rows >= 0
    constexpr int V8 = RAWW / 8;
    if (!a.vec16) {                               // rows not 16-byte aligned: 4-byte copies
      constexpr int PAIRS = RAWW / 2;
      for (int idx = tid; idx < (nsub + KC - 1) * PAIRS; idx += NT) {
        const int i = idx / PAIRS, c2 = 2 * (idx % PAIRS);
        const int r = r0 - (KC - 1) + i;
        int ch;
        if (c2 < D) ch = cq + c2;
        else if (c2 < 2 * D) ch = ck + (c2 - D);
        else if (c2 < 2 * D + COLS) ch = cv + (c2 - 2 * D);
        else ch = cz + (c2 - 2 * D - COLS);
        if (r >= 0) cp_async4(&raw[i][c2], proj + (size_t)r * a.proj_ld + ch);
        else if (c2 < 2 * D + COLS) cp_async4(&raw[i][c2], window + (size_t)(r + KC - 1) * a.C + ch);
        else *reinterpret_cast<uint32_t*>(&raw[i][c2]) = 0u;
      }
    }
    for (int idx = tid; a.vec16 && idx < (nsub + KC - 1) * V8; idx += NT) {
      const int i = idx / V8, c8 = (idx % V8) * 8;   // staged channel of the group
      const int r = r0 - (KC - 1) + i;
      int ch;
      if (c8 < D) ch = cq + c8;
      else if (c8 < 2 * D) ch = ck + (c8 - D);
      else if (c8 < 2 * D + COLS) ch = cv + (c8 - 2 * D);
      else ch = cz + (c8 - 2 * D - COLS);
      if (r >= 0) cp_async16(&raw[i][c8], proj + (size_t)r * a.proj_ld + ch);
      else if (c8 < 2 * D + COLS) cp_async16(&raw[i][c8], window + (size_t)(r + KC - 1) * a.C + ch);
      else *reinterpret_cast<uint4*>(&raw[i][c8]) = make_uint4(0u, 0u, 0u, 0u);
    }
    cp_async_commit();
    if (tid < nsub) {
      const int r = r0 + tid;
      const float av = __bfloat162float(proj[(size_t)r * a.proj_ld + ca]);
      const float bv = __bfloat162float(proj[(size_t)r * a.proj_ld + cb]);
      const float sp = (av + dtb) > 20.f ? (av + dtb) : log1pf(__expf(av + dtb));
      g_s[tid] = __expf(A * sp);                   // the row's decay
      b_s[tid] = 1.f / (1.f + __expf(-bv));
    }
    cp_async_wait<0>();
    __syncthreads();
    Q38_GSTAMP(2);
    // ---- 2. conv + SiLU and L2 norms in registers: thread c < D owns q channel c and k channel c
    //         for every row of the sub-block; row sums of squares by xor butterfly in the warp,
    //         then over the warps in order
    {
      static_assert(KC == 4, "four conv taps");
      float qv[SUB], kv[SUB], sq[SUB], sk[SUB];
#pragma unroll
      for (int t = 0; t < SUB; ++t) {
        float aq = 0.f, ak = 0.f;
        if (tid < D && t < nsub) {
#pragma unroll
          for (int j = 0; j < KC; ++j) {
            aq += wq[j] * __bfloat162float(raw[t + j][tid]);
            ak += wk[j] * __bfloat162float(raw[t + j][D + tid]);
          }
          aq = silu_f(aq);
          ak = silu_f(ak);
        }
        qv[t] = aq;
        kv[t] = ak;
        sq[t] = aq * aq;
        sk[t] = ak * ak;
      }
      // the rows' butterflies level by level, so the 2 x SUB independent shuffles of a level
      // pipeline instead of running row after row
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int t = 0; t < SUB; ++t) {
          sq[t] += __shfl_xor_sync(0xffffffffu, sq[t], o);
          sk[t] += __shfl_xor_sync(0xffffffffu, sk[t], o);
        }
      }
      if (lane == 0 && warp < D / 32) {
#pragma unroll
        for (int t = 0; t < SUB; ++t) { ssq_s[t][warp] = sq[t]; ssk_s[t][warp] = sk[t]; }
      }
      for (int t = part; t < nsub; t += 4) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < KC; ++j) acc += wv[j] * __bfloat162float(raw[t + j][2 * D + col]);
        v_s[t][col] = silu_f(acc);
      }
      __syncthreads();
      if (tid < D) {
        const int pi = (tid / RPT) * QP + (tid % RPT);
#pragma unroll
        for (int t = 0; t < SUB; ++t) {
          if (t < nsub) {
            float pq = 0.f, pk = 0.f;
#pragma unroll
            for (int w = 0; w < D / 32; ++w) { pq += ssq_s[t][w]; pk += ssk_s[t][w]; }
            q_s[t][pi] = qv[t] * (rsqrtf(pq + 1e-6f) * rsqrtf((float)D));
            k_s[t][pi] = kv[t] * rsqrtf(pk + 1e-6f);
          }
        }
      }
    }
    __syncthreads();
    Q38_GSTAMP(3);
    // ---- 3. sequential recurrence: S <- decay S + k (beta (v - decay S^T k))^T, o = S^T q, with
    //         float4 shared-memory operands, a fixed 4-way partial-sum split and an xor butterfly
    //         over the column's 4 threads
    for (int t = 0; t < nsub; ++t) {
      const float decay = g_s[t];
      const float4* kr = reinterpret_cast<const float4*>(&k_s[t][part * QP]);
      const float4* qr = reinterpret_cast<const float4*>(&q_s[t][part * QP]);
      float kv4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i4 = 0; i4 < RPT / 4; ++i4) {
        const float4 k4 = kr[i4];
        kv4[0] = fmaf(S[4 * i4 + 0], k4.x, kv4[0]);
        kv4[1] = fmaf(S[4 * i4 + 1], k4.y, kv4[1]);
        kv4[2] = fmaf(S[4 * i4 + 2], k4.z, kv4[2]);
        kv4[3] = fmaf(S[4 * i4 + 3], k4.w, kv4[3]);
      }
      float kvs = (kv4[0] + kv4[1]) + (kv4[2] + kv4[3]);
      kvs += __shfl_xor_sync(0xffffffffu, kvs, 1);
      kvs += __shfl_xor_sync(0xffffffffu, kvs, 2);
      const float delta = (v_s[t][col] - decay * kvs) * b_s[t];
      float o4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i4 = 0; i4 < RPT / 4; ++i4) {
        const float4 k4 = kr[i4], q4 = qr[i4];
        S[4 * i4 + 0] = fmaf(decay, S[4 * i4 + 0], k4.x * delta);
        S[4 * i4 + 1] = fmaf(decay, S[4 * i4 + 1], k4.y * delta);
        S[4 * i4 + 2] = fmaf(decay, S[4 * i4 + 2], k4.z * delta);
        S[4 * i4 + 3] = fmaf(decay, S[4 * i4 + 3], k4.w * delta);
        o4[0] = fmaf(S[4 * i4 + 0], q4.x, o4[0]);
        o4[1] = fmaf(S[4 * i4 + 1], q4.y, o4[1]);
        o4[2] = fmaf(S[4 * i4 + 2], q4.z, o4[2]);
        o4[3] = fmaf(S[4 * i4 + 3], q4.w, o4[3]);
      }
      if constexpr (WRITE_OUT) {
        float o = (o4[0] + o4[1]) + (o4[2] + o4[3]);
        o += __shfl_xor_sync(0xffffffffu, o, 1);
        o += __shfl_xor_sync(0xffffffffu, o, 2);
        if (part == 0) o_s[t][col] = o;
      }
    }
    Q38_GSTAMP(4);
    if constexpr (WRITE_OUT) {
      __syncthreads();
      // ---- 5. gated RMSNorm: partial sums of squares over this CTA's columns, exchanged in the
      // cluster through DSMEM, summed in cluster-rank order
      {
        const int t = tid / NPR, j = tid % NPR;
        float ss = 0.f;
#pragma unroll
        for (int m = 0; m < COLS / NPR; ++m) {
          const float v = o_s[t][j * (COLS / NPR) + m];
          ss += v * v;
        }
#pragma unroll
        for (int o = 1; o < NPR; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (j == 0) {
#pragma unroll
          for (int p = 0; p < SPLIT; ++p) {
            float* dst = cluster.map_shared_rank(&ss_part[parity][sl][t], p);
            *dst = ss;
          }
        }
      }
      cluster.sync();
      Q38_GSTAMP(5);
      if (tid < nsub) {
        float s = 0.f;
#pragma unroll
        for (int p = 0; p < SPLIT; ++p) s += ss_part[parity][p][tid];
        rs_s[tid] = rsqrtf(s / D + a.eps);
      }
      __syncthreads();
      for (int idx = tid; idx < nsub * COLS; idx += NT) {
        const int t = idx / COLS, c = idx % COLS;
        const float z = __bfloat162float(raw[t + KC - 1][2 * D + COLS + c]);
        const float y = o_s[t][c] * rs_s[t] * norm_w[sl * COLS + c] * silu_f(z);
        a.out[(size_t)(r0 + t) * a.out_ld + (size_t)h * D + sl * COLS + c] = __float2bfloat16(y);
      }
      Q38_GSTAMP(6);
    }
    __syncthreads();
  }
  if constexpr (WRITE_STATE) {
#pragma unroll
    for (int i = 0; i < RPT; ++i) state[(size_t)(part * RPT + i) * D + gcol] = S[i];
  }
  Q38_GSTAMP(7);
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

static unsigned long long* g_gdn_trace = nullptr;   // micro-benchmark stamps (kbench gdn --trace)

// ----------------------------------------------------------------------------- bindings
void q38_gdn_set_trace(c10::optional<torch::Tensor> trace) {
  g_gdn_trace = trace ? reinterpret_cast<unsigned long long*>(trace->data_ptr<int64_t>()) : nullptr;
}

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
  a.trace = g_gdn_trace;
  a.vec16 = (a.proj_ld % 8 == 0 && C % 8 == 0 && (reinterpret_cast<uintptr_t>(a.proj) & 15) == 0 &&
             (reinterpret_cast<uintptr_t>(a.window) & 15) == 0 && (!multi || (a.proj_layer_stride % 8 == 0 &&
                                                                              a.win_layer_stride % 8 == 0)))
                ? 1 : 0;
  TORCH_CHECK(KC == 4, "conv kernel size 4 supported");
  TORCH_CHECK(mode != 0 || out, "verify needs an output");
  TORCH_CHECK(a.proj_ld % 2 == 0 && C % 2 == 0 && (reinterpret_cast<uintptr_t>(a.proj) & 3) == 0 &&
                  (reinterpret_cast<uintptr_t>(a.window) & 3) == 0,
              "GDN rows are staged as bf16 pairs: even row strides and 4-byte aligned bases required");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto launch = [&](auto kern, int split) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(nv * split), (unsigned)layers);
    cfg.blockDim = dim3(128);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int n = 0;
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = split;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
    if (q38::pdl_enabled()) {
      attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[n].val.programmaticStreamSerializationAllowed = 1;
      ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    TORCH_CHECK(cudaLaunchKernelEx(&cfg, kern, a) == cudaSuccess, "GDN recurrence launch failed");
  };
#define Q38_GDN_LAUNCH(DD, SP)                                                                   \
  if (mode == 0) launch(q38::gdn_recurrent_kernel<DD, 4, 16, true, false, SP>, SP);             \
  else if (mode == 1) launch(q38::gdn_recurrent_kernel<DD, 4, 16, false, true, SP>, SP);        \
  else launch(q38::gdn_recurrent_kernel<DD, 4, 16, true, true, SP>, SP);
  if (D == 128) { Q38_GDN_LAUNCH(128, 4) }
  else if (D == 32) { Q38_GDN_LAUNCH(32, 1) }
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
