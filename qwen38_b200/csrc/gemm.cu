// GEMM host side: tensor maps, split-K planning, dispatch and bindings (kernel: gemm_kernel.cuh).
#include <c10/cuda/CUDAGuard.h>

#include <mutex>
#include <unordered_map>

#include "gemm_kernel.cuh"

namespace q38 {

bool pdl_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("Q38_PDL");      // on by default; Q38_PDL=0 launches without the attribute
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

// Final reduction of per-tile argmax partials: out_idx[n] = argmax over tiles (ties -> lower index)
__global__ void argmax_finalize_kernel(const float* __restrict__ val, const int* __restrict__ idx, int tiles, int N,
                                       long long vocab_offset, float* __restrict__ out_val,
                                       int64_t* __restrict__ out_idx) {
  pdl_wait();
  pdl_trigger();
  const int n = blockIdx.x;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int t = threadIdx.x; t < tiles; t += blockDim.x) {
    const float v = val[(size_t)t * N + n];
    const int i = idx[(size_t)t * N + n];
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
    out_val[n] = best;
    out_idx[n] = (int64_t)bi + vocab_offset;
  }
}


// ============================================================================= host side
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn get_encode() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && p != nullptr, "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

// Row-major [rows, cols] bf16 matrix -> TMA map with box {64 cols, box_rows rows}, 128-B swizzle.
CUtensorMap make_map_2d(const void* ptr, int64_t rows, int64_t cols, int64_t row_stride_elems, int box_rows) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((row_stride_elems * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(row_stride_elems * 2)};
  cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = get_encode()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return map;
}

// Weight maps are reused across calls: cache by (pointer, shape, box).
static std::mutex g_map_mu;
static std::unordered_map<std::string, CUtensorMap> g_map_cache;

static CUtensorMap cached_map(const torch::Tensor& t, int box_rows, bool cache) {
  const int64_t rows = t.size(0), cols = t.size(1), ld = t.stride(0);
  if (!cache) return make_map_2d(t.data_ptr(), rows, cols, ld, box_rows);
  std::string key = std::to_string(reinterpret_cast<uintptr_t>(t.data_ptr())) + ":" + std::to_string(rows) + ":" +
                    std::to_string(cols) + ":" + std::to_string(ld) + ":" + std::to_string(box_rows);
  std::lock_guard<std::mutex> lk(g_map_mu);
  auto it = g_map_cache.find(key);
  if (it != g_map_cache.end()) return it->second;
  CUtensorMap m = make_map_2d(t.data_ptr(), rows, cols, ld, box_rows);
  g_map_cache.emplace(key, m);
  return m;
}

void clear_map_cache() {
  std::lock_guard<std::mutex> lk(g_map_mu);
  g_map_cache.clear();
}

// Split count for a weight of `m_tiles` row tiles and `kblocks` K blocks: a function of the weight
// shape only (never of the token count), about two CTAs per SM, at most one portable cluster.
int pick_splits(int m_tiles, int kblocks, int sms) {
  int s = (2 * sms) / std::max(1, m_tiles);
  s = std::max(1, std::min(std::min(s, kblocks / 4), MAX_CLUSTER_SPLITS));
  return s;
}

struct SampleArgs {
  const float* scale;
  const unsigned long long* key;
  long long vocab_off;
};

struct Scratch {
  float* ws;
  int64_t ws_floats;
  int* counters;
  int64_t n_counters;
  int* err;
};

static Scratch scratch_of(torch::Tensor ws, torch::Tensor counters, torch::Tensor err) {
  return Scratch{ws.data_ptr<float>(), ws.numel(), counters.data_ptr<int>(), counters.numel(), err.data_ptr<int>()};
}

static int num_sms() { return device_sms(); }

static bool splitk_cluster() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("Q38_SPLITK");
    v = (e && std::string(e) == "cluster") ? 1 : 0;
  }
  return v == 1;
}

// MX weight: e4m3 bytes tiled like a bf16 weight ([tiles * 128, 64] uint8) and E8M0 scales
// ([tiles * 128, 2] uint8), see mx_tile_weight in qwen38_b200/ops/native.py.
struct MxW {
  const uint8_t* q;
  const uint8_t* s;
};

static MxW mx_of(const torch::Tensor& wq, const torch::Tensor& wsc) {
  TORCH_CHECK(wq.scalar_type() == at::kByte && wsc.scalar_type() == at::kByte && wq.is_contiguous() &&
                  wsc.is_contiguous() && wq.is_cuda() && wsc.is_cuda(), "MX weight: contiguous uint8 values and scales");
  TORCH_CHECK(wsc.numel() * 32 == wq.numel(), "MX weight: one scale per 32 values");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(wq.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(wsc.data_ptr()) % 16 == 0,
              "MX weight: 16-byte aligned storage");
  return MxW{reinterpret_cast<const uint8_t*>(wq.data_ptr()), reinterpret_cast<const uint8_t*>(wsc.data_ptr())};
}

// out (m, n) layout: swap -> out[n * ldo + m]; prefill -> out[m * ldo + n]
// `w` is a tile-contiguous weight ([ceil(N/128) * ceil(K/64) * 128, 64], see tile_weight in
// qwen38_b200/ops/native.py) of logical shape [N, K].
void gemm_dispatch(const torch::Tensor& x, const torch::Tensor& w, int N, torch::Tensor& out, int epi,
                   const Scratch& sc, float* amax_val = nullptr, int* amax_idx = nullptr, int* amax_tiles = nullptr,
                   const ArArgs* ar = nullptr, unsigned long long* trace = nullptr, int64_t ldo_override = -1,
                   const SampleArgs* samp = nullptr, const RsArgs* rs = nullptr, const MxW* mx = nullptr) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && out.is_cuda(), "CUDA tensors required");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == (mx ? at::kByte : at::kBFloat16),
              "bf16 activations and bf16 (or MX e4m3) weights required");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x [T, K] K-contiguous required");
  const int T = (int)x.size(0), K = (int)x.size(1);
  TORCH_CHECK(w.dim() == 2 && w.size(1) == BK && w.is_contiguous(), "tile-contiguous weight [rows, 64] required");
  TORCH_CHECK(w.size(0) == (int64_t)((N + BM - 1) / BM) * ((K + BK - 1) / BK) * BM, "weight tiling mismatch");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  GemmArgs g{};
  g.K = K;
  g.kblocks = (K + BK - 1) / BK;
  g.out = out.data_ptr();
  g.ldo = ldo_override >= 0 ? ldo_override : out.stride(0);
  g.err = sc.err;
  g.ws = sc.ws;
  g.counters = sc.counters;
  g.trace = trace;
  TORCH_CHECK(epi != EPI_RS_F32 || (T > 32 && rs != nullptr), "the reduce-scatter epilogue serves prefill tiles");
  TORCH_CHECK(mx == nullptr || (T <= SWAP_MAX_ROWS && epi != EPI_ARGMAX && epi != EPI_RS_F32),
              "MX weights stream through the swap-mode GEMM (<= 64 rows)");
  if (T <= SWAP_MAX_ROWS) {
    // swap-AB streaming: M = weight rows, N = tokens in 32-token tiles (grid y).  Each token
    // column's result depends on its own column and the split plan (a function of N, K and the SM
    // count) only, so a row gets the same bits alone or packed with other requests' rows.
    g.M = N;
    g.N = T;
    const int m_tiles = (N + BM - 1) / BM;
    const int n_tiles = (T + 31) / 32;
    int splits = pick_splits(m_tiles, g.kblocks, num_sms());
    int kps = (g.kblocks + splits - 1) / splits;
    splits = (g.kblocks + kps - 1) / kps;
    g.splits = splits;
    g.kps = kps;
    // Split-K fix-up: the last-arriving CTA through global memory by default; Q38_SPLITK=cluster
    // reduces through DSMEM inside a cluster of the tile's splits (same bits).  Measured on B200
    // the cluster form was slower: clusters of up to 8 CTAs at two CTAs per SM no longer fit the
    // grid into one wave once GPC boundaries are respected.  ARGMAX always uses the global form.
    g.cluster_k = epi != EPI_ARGMAX && epi != EPI_SPLIT_F32 && n_tiles == 1 && mx == nullptr && splitk_cluster();
    if (splits > 1 && !g.cluster_k && epi != EPI_SPLIT_F32) {
      TORCH_CHECK((int64_t)m_tiles * n_tiles * splits * BM * 32 <= sc.ws_floats, "split-K workspace too small");
      TORCH_CHECK(m_tiles * n_tiles <= sc.n_counters, "split-K counter array too small");
    }
    if (epi == EPI_PUSH_F32) {
      TORCH_CHECK(ar != nullptr && (int64_t)T * N <= ar->block_words, "pushed all-reduce: block too small");
      g.ar = *ar;
    }
    if (epi == EPI_ARGMAX) {
      if (samp) {
        g.samp_scale = samp->scale;
        g.samp_key = samp->key;
        g.vocab_off = samp->vocab_off;
      }
      g.amax_val = amax_val;
      g.amax_idx = amax_idx;
      *amax_tiles = m_tiles;
    }
    CUtensorMap mb = cached_map(x, 32, false);
    dim3 grid(m_tiles, n_tiles, splits);
    if (mx) {
      g.mxq = mx->q;
      g.mxs = mx->s;
      launch_swap_mx(epi, mb, g, grid, st);
    } else {
      CUtensorMap ma = cached_map(w, BM, true);    // one 16 KB weight tile per box
      launch_swap(epi, ma, mb, g, grid, st);
    }
  } else {
    TORCH_CHECK(epi != EPI_ARGMAX && epi != EPI_PUSH_F32, "argmax / pushed all-reduce epilogues serve <= 64 rows");
    g.M = T;
    g.N = N;
    g.splits = 1;
    g.kps = g.kblocks;
    if (epi == EPI_SWIGLU) TORCH_CHECK(N % PREFILL_BN == 0, "SwiGLU prefill needs N % 256 == 0");
    if (epi == EPI_RS_F32) {
      TORCH_CHECK(N % PREFILL_BN == 0, "reduce-scatter prefill needs N % 256 == 0");
      const int tiles = (T + BM - 1) / BM;
      TORCH_CHECK((int64_t)((tiles + rs->world - 1) / rs->world) * BM <= rs->rows_cap,
                  "reduce-scatter area too small for this chunk");
      g.rs = *rs;
    }
    CUtensorMap ma = cached_map(x, BM, false);
    CUtensorMap mb = cached_map(w, BM, true);      // two 16 KB weight tiles per 256-row stage
    dim3 grid((T + BM - 1) / BM, (N + PREFILL_BN - 1) / PREFILL_BN, 1);
    launch_prefill(epi, ma, mb, g, grid, st);
  }
}

}  // namespace q38

// ----------------------------------------------------------------------------- bindings
void q38_linear(torch::Tensor x, torch::Tensor w, int64_t N, torch::Tensor out, int64_t epi, torch::Tensor ws,
                torch::Tensor counters, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(x.device());
  auto sc = q38::scratch_of(ws, counters, err);
  if (epi == q38::EPI_BF16 || epi == q38::EPI_SWIGLU) {
    TORCH_CHECK(out.scalar_type() == at::kBFloat16, "bf16 output required");
  } else {
    TORCH_CHECK(out.scalar_type() == at::kFloat, "fp32 output required");
  }
  TORCH_CHECK(out.stride(1) == 1, "row-contiguous output required");
  q38::gemm_dispatch(x, w, (int)N, out, (int)epi, sc);
}

// q38_linear with an MX weight (wq e4m3 bytes, wsc E8M0 scales; <= 64 rows, not argmax).
void q38_linear_mx(torch::Tensor x, torch::Tensor wq, torch::Tensor wsc, int64_t N, torch::Tensor out, int64_t epi,
                   torch::Tensor ws, torch::Tensor counters, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(x.device());
  auto sc = q38::scratch_of(ws, counters, err);
  const q38::MxW mx = q38::mx_of(wq, wsc);
  if (epi == q38::EPI_BF16 || epi == q38::EPI_SWIGLU) {
    TORCH_CHECK(out.scalar_type() == at::kBFloat16, "bf16 output required");
  } else {
    TORCH_CHECK(out.scalar_type() == at::kFloat, "fp32 output required");
  }
  TORCH_CHECK(out.stride(1) == 1, "row-contiguous output required");
  q38::gemm_dispatch(x, wq, (int)N, out, (int)epi, sc, nullptr, nullptr, nullptr, nullptr, nullptr, -1, nullptr,
                     nullptr, &mx);
}

// Row-parallel out-projection whose epilogue pushes this rank's fp32 partial [T, N] (T <= 64)
// into every rank's receive block of `slot` as {value, epoch} words (EPI_PUSH_F32); the reduction
// into the residual happens in q38_rms_norm_ar.  recv_ptrs: every rank's receive area mapped into
// this process; epochs: this rank's [slots][32] per-row epochs.
void q38_linear_push(torch::Tensor x, torch::Tensor w, int64_t N, torch::Tensor ws, torch::Tensor counters,
                     torch::Tensor err, std::vector<int64_t> recv_ptrs, int64_t rank, int64_t slot,
                     int64_t block_words, torch::Tensor epochs, int64_t mc_ptr,
                     c10::optional<torch::Tensor> mx_scales) {
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.size(0) <= q38::AR_MAX_ROWS, "the pushed all-reduce serves <= 64 rows");
  TORCH_CHECK(x.size(0) * N <= block_words, "partial larger than a receive block");
  const int world = (int)recv_ptrs.size();
  TORCH_CHECK(world >= 1 && world <= q38::AR_MAX_RANKS, "1..8 ranks");
  TORCH_CHECK(rank >= 0 && rank < world, "bad rank");
  TORCH_CHECK(epochs.scalar_type() == at::kInt && epochs.numel() >= (slot + 1) * q38::AR_MAX_ROWS,
              "epoch array too small");
  q38::ArArgs a{};
  for (int p = 0; p < world; ++p) a.recv[p] = recv_ptrs[p];
  a.block_words = block_words;
  a.mc = mc_ptr;
  a.rank = (int)rank;
  a.world = world;
  a.slot = (int)slot;
  a.epochs = epochs.data_ptr<int>();
  auto sc = q38::scratch_of(ws, counters, err);
  // no local output tensor: the epilogue writes the receive blocks, laid out [T, N] (ldo = N)
  torch::Tensor unused = x;
  q38::MxW mx{};
  if (mx_scales) mx = q38::mx_of(w, *mx_scales);
  q38::gemm_dispatch(x, w, (int)N, unused, q38::EPI_PUSH_F32, sc, nullptr, nullptr, nullptr, &a, nullptr, N, nullptr,
                     nullptr, mx_scales ? &mx : nullptr);
}

// Split-K slices of the swap-AB plan for an [N, K] weight (the count q38_linear would use).
int64_t q38_swap_splits(int64_t N, int64_t K) {
  const int m_tiles = (int)((N + q38::BM - 1) / q38::BM), kblocks = (int)((K + q38::BK - 1) / q38::BK);
  const int s = q38::pick_splits(m_tiles, kblocks, q38::num_sms());
  const int kps = (kblocks + s - 1) / s;
  return (kblocks + kps - 1) / kps;
}

// Row-parallel out-projection of <= 64 rows whose split-K reduction is left to the consumer:
// with S > 1 slices every slice stores its fp32 partial into parts ([S][T][N], contiguous from the
// start of `parts`) and nothing else; the next RMSNorm of the residual (q38_rms_norm_split) adds the
// slices in split order and then the residual, the same arithmetic as the in-kernel fix-up, so the
// residual gets the same bits one launch later without the fix-up's serial tail.  With one slice
// the GEMM adds into `residual` directly.  Returns S (1: nothing pending).
int64_t q38_linear_split(torch::Tensor x, torch::Tensor w, int64_t N, torch::Tensor residual, torch::Tensor parts,
                         torch::Tensor ws, torch::Tensor counters, torch::Tensor err,
                         c10::optional<torch::Tensor> mx_scales) {
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t T = x.size(0);
  TORCH_CHECK(T >= 1 && T <= q38::SWAP_MAX_ROWS, "deferred split-K serves 1..64 rows");
  TORCH_CHECK(residual.scalar_type() == at::kFloat && residual.is_contiguous() && residual.size(0) == T &&
                  residual.size(1) == N, "fp32 residual [T, N]");
  auto sc = q38::scratch_of(ws, counters, err);
  q38::MxW mxw{};
  const q38::MxW* mx = nullptr;
  if (mx_scales) {
    mxw = q38::mx_of(w, *mx_scales);
    mx = &mxw;
  }
  const int64_t S = q38_swap_splits(N, x.size(1));
  if (S == 1) {
    q38::gemm_dispatch(x, w, (int)N, residual, q38::EPI_ADD_F32, sc, nullptr, nullptr, nullptr, nullptr, nullptr, -1,
                       nullptr, nullptr, mx);
    return 1;
  }
  TORCH_CHECK(parts.scalar_type() == at::kFloat && parts.is_contiguous() && parts.numel() >= S * T * N,
              "split partial buffer too small");
  q38::gemm_dispatch(x, w, (int)N, parts, q38::EPI_SPLIT_F32, sc, nullptr, nullptr, nullptr, nullptr, nullptr, N,
                     nullptr, nullptr, mx);
  return S;
}

// Prefill out-projection whose tiles go to their owning rank's reduce-scatter area (EPI_RS_F32):
// recv_ptrs / count_ptrs are every rank's area and arrival counter, rows_cap the local rows per
// source block.  The owner's q38_rs_reduce_bcast completes the all-reduce.
void q38_linear_rs(torch::Tensor x, torch::Tensor w, int64_t N, torch::Tensor ws, torch::Tensor counters,
                   torch::Tensor err, std::vector<int64_t> recv_ptrs, std::vector<int64_t> count_ptrs, int64_t rank,
                   int64_t rows_cap) {
  c10::cuda::CUDAGuard guard(x.device());
  const int world = (int)recv_ptrs.size();
  TORCH_CHECK(world >= 1 && world <= q38::AR_MAX_RANKS && (int)count_ptrs.size() == world, "1..8 ranks");
  q38::RsArgs r{};
  for (int p = 0; p < world; ++p) {
    r.recv[p] = recv_ptrs[p];
    r.count[p] = count_ptrs[p];
  }
  r.rank = (int)rank;
  r.world = world;
  r.rows_cap = (int)rows_cap;
  auto sc = q38::scratch_of(ws, counters, err);
  torch::Tensor unused = x;
  q38::gemm_dispatch(x, w, (int)N, unused, q38::EPI_RS_F32, sc, nullptr, nullptr, nullptr, nullptr, nullptr, N,
                     nullptr, &r);
}

// Micro-benchmark entry: q38_linear with per-CTA phase stamps written to `trace` ([grid][8] int64).
// Returns the grid size.
int64_t q38_linear_trace(torch::Tensor x, torch::Tensor w, int64_t N, torch::Tensor out, int64_t epi,
                         torch::Tensor ws, torch::Tensor counters, torch::Tensor err, torch::Tensor trace,
                         c10::optional<torch::Tensor> mx_scales) {
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(trace.scalar_type() == at::kLong && trace.is_contiguous(), "int64 trace buffer");
  TORCH_CHECK(epi == q38::EPI_BF16 || epi == q38::EPI_F32 || epi == q38::EPI_ADD_F32 || epi == q38::EPI_SWIGLU,
              "traced epilogues: bf16, f32, add, swiglu");
  auto sc = q38::scratch_of(ws, counters, err);
  const int T = (int)x.size(0), K = (int)x.size(1);
  const int64_t m_tiles = (T <= q38::SWAP_MAX_ROWS) ? ((N + 127) / 128) * ((T + 31) / 32)
                                                    : ((T + 127) / 128) * ((N + q38::PREFILL_BN - 1) / q38::PREFILL_BN);
  const int64_t kb = (K + 63) / 64;
  // MX: 4 more words per CTA after the stamps (converter / MMA wait and work cycles)
  TORCH_CHECK(trace.numel() >= m_tiles * kb * (mx_scales ? 12 : 8), "trace buffer too small");
  q38::MxW mx{};
  if (mx_scales) mx = q38::mx_of(w, *mx_scales);
  q38::gemm_dispatch(x, w, (int)N, out, (int)epi, sc, nullptr, nullptr, nullptr, nullptr,
                     reinterpret_cast<unsigned long long*>(trace.data_ptr<int64_t>()), -1, nullptr, nullptr,
                     mx_scales ? &mx : nullptr);
  return m_tiles;
}

void q38_lm_head_argmax(torch::Tensor x, torch::Tensor w, int64_t N, torch::Tensor out_val, torch::Tensor out_idx,
                        int64_t vocab_offset, torch::Tensor part_val, torch::Tensor part_idx, torch::Tensor ws,
                        torch::Tensor counters, torch::Tensor err, c10::optional<torch::Tensor> samp_scale,
                        c10::optional<torch::Tensor> samp_key) {
  c10::cuda::CUDAGuard guard(x.device());
  auto sc = q38::scratch_of(ws, counters, err);
  const int T = (int)x.size(0);
  TORCH_CHECK(T <= q38::SWAP_MAX_ROWS, "LM-head argmax serves <= 64 rows");
  const int tiles_needed = (int)((N + 127) / 128);
  TORCH_CHECK(part_val.numel() >= (int64_t)tiles_needed * T && part_idx.numel() >= (int64_t)tiles_needed * T,
              "argmax partial buffers too small");
  int tiles = 0;
  torch::Tensor dummy = out_val;  // not written by the argmax epilogue
  q38::SampleArgs sa{};
  if (samp_scale) {
    TORCH_CHECK(samp_key && samp_scale->scalar_type() == at::kFloat && samp_key->scalar_type() == at::kLong &&
                    samp_scale->numel() >= T && samp_key->numel() >= T, "sampling: fp32 scale [T] and int64 key [T]");
    sa.scale = samp_scale->data_ptr<float>();
    sa.key = reinterpret_cast<const unsigned long long*>(samp_key->data_ptr<int64_t>());
  }
  sa.vocab_off = vocab_offset;
  q38::gemm_dispatch(x, w, (int)N, dummy, q38::EPI_ARGMAX, sc, part_val.data_ptr<float>(), part_idx.data_ptr<int>(),
                     &tiles, nullptr, nullptr, -1, &sa);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  q38::launch_pdl(q38::argmax_finalize_kernel, dim3(T), dim3(256), 0, st, (const float*)part_val.data_ptr<float>(),
                  (const int*)part_idx.data_ptr<int>(), tiles, T, (long long)vocab_offset, out_val.data_ptr<float>(),
                  out_idx.data_ptr<int64_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void q38_clear_map_cache() { q38::clear_map_cache(); }
