// Allocation-free entry point for the skinny tcgen05 GEMM (<= 32 token rows).
//
// This entry point has no counterpart in the reference.
//
// Who it is for: callers that cannot allocate device memory at call time.  A caller running
// inside another framework's memory pool that forbids stray cudaMalloc / cudaFree, an embedded
// serving loop whose memory is fixed at start-up, or code that must not touch an allocator on its
// hot path (allocation can synchronise the device or fail under fragmentation) can still run this
// GEMM: the caller passes only its inputs and outputs, and the kernel's scratch memory (split-K
// partial tiles, per-tile arrival counters and the error word) lives in the file-scope array
// `g_scratch` below, a fixed 8 MiB + 16 KiB that every GPU loading this library holds until the
// process exits.
//
// C interface (prototypes, return codes, limits): q38_noalloc.h.
//
//   int q38_linear_noalloc(x, T, K, w_tiled, N, out, ldo, epi, stream)
//     x        bf16 [T, K] row-major, T <= 32, K % 8 == 0, 16-byte aligned
//     w_tiled  bf16 weight of logical shape [N, K] in the tile-contiguous layout of
//              qwen38_b200.ops.native.tile_weight (tile (n/128, k/64) is one 16 KB block)
//     out      [T, ldo] row-major; epi 0: bf16 store, 1: fp32 store, 2: fp32 accumulate (out += x w^T)
//     returns  0 on success, Q38_NOALLOC_E* otherwise (nothing is launched on error)
//
// Set-up: the first call on a device (with that device current) looks up the device address of
// `g_scratch` with cudaGetSymbolAddress; make that first call before any stream capture.  The
// entry point itself calls no cudaMalloc, cudaFree or other allocating routine.
//
// Sharing: every call on a device uses the same scratch array, which keeps the previous call's
// contents.  Each call clears the arrival counters and the error word it uses (cudaMemsetAsync on
// its stream) before launching.  Calls that overlap on the GPU (different streams, or a second
// host thread) race on the scratch: serialise them.
#include "gemm_kernel.cuh"
#include "q38_noalloc.h"

#include <mutex>

namespace q38 {
namespace noalloc {

constexpr size_t kPartialFloats = size_t(1) << 21;   // 8 MiB of split-K partials
constexpr int kCounters = 4096;                      // per-tile arrival counters
constexpr size_t kScratchBytes = kPartialFloats * 4 + kCounters * 4 + 256;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

static void* g_scratch_dev[kMaxDevices];
static std::once_flag g_once[kMaxDevices];
static cudaError_t g_setup_err[kMaxDevices];

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

static bool encode(CUtensorMap* map, const void* ptr, uint64_t rows, uint64_t cols, uint64_t row_bytes, int box_rows) {
  EncodeFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int EPI>
static cudaError_t launch(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& g, dim3 grid,
                          cudaStream_t st) {
  auto kern = gemm_tn_kernel<32, SKINNY_STAGES, EPI, true>;
  constexpr int smem = Smem<32, SKINNY_STAGES>::TOTAL;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, 128, smem, st>>>(ma, mb, g);
  return cudaGetLastError();
}

}  // namespace noalloc
}  // namespace q38

static_assert(q38::noalloc::kCounters == Q38_NOALLOC_MAX_TILES, "header limit out of date");
static_assert(q38::noalloc::kPartialFloats == Q38_NOALLOC_MAX_PARTIAL_FLOATS, "header limit out of date");
static_assert(Q38_NOALLOC_EPI_BF16 == q38::EPI_BF16 && Q38_NOALLOC_EPI_F32 == q38::EPI_F32 &&
                  Q38_NOALLOC_EPI_ADD_F32 == q38::EPI_ADD_F32, "header epilogue codes out of date");

// Declared in q38_noalloc.h (the C interface); the definitions below must match it.
extern "C" __attribute__((visibility("default"))) int q38_linear_noalloc(const void* x, int T, int K,
                                                                          const void* w_tiled, int N, void* out,
                                                                          int ldo, int epi, cudaStream_t stream) {
  using namespace q38;
  using namespace q38::noalloc;
  if (!x || !w_tiled || !out || T < 1 || T > 32 || K < 1 || N < 1 || ldo < N) return Q38_NOALLOC_EARG;
  if (K % 8 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w_tiled) & 15))
    return Q38_NOALLOC_EARG;
  if (epi != EPI_BF16 && epi != EPI_F32 && epi != EPI_ADD_F32) return Q38_NOALLOC_EARG;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return Q38_NOALLOC_ECUDA;
  std::call_once(g_once[dev], [dev] {
    g_setup_err[dev] = cudaGetSymbolAddress(&g_scratch_dev[dev], g_scratch);
  });
  if (g_setup_err[dev] != cudaSuccess || g_scratch_dev[dev] == nullptr) return Q38_NOALLOC_ECUDA;

  // split plan: the policy of the allocating entry point (weight shape only), so both produce the
  // same bits
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return Q38_NOALLOC_ECUDA;
  const int kblocks = (K + BK - 1) / BK;
  const int m_tiles = (N + BM - 1) / BM;
  int splits = pick_splits(m_tiles, kblocks, sms);
  int kps = (kblocks + splits - 1) / splits;
  splits = (kblocks + kps - 1) / kps;
  if (m_tiles > kCounters) return Q38_NOALLOC_ESIZE;
  if (splits > 1 && (size_t)m_tiles * splits * BM * 32 > kPartialFloats) return Q38_NOALLOC_ESIZE;

  unsigned char* base = static_cast<unsigned char*>(g_scratch_dev[dev]);
  float* partials = reinterpret_cast<float*>(base);
  int* counters = reinterpret_cast<int*>(base + kPartialFloats * 4);
  int* err = counters + kCounters;
  // counters and the error word must start at zero for this call
  if (cudaMemsetAsync(counters, 0, (size_t)(kCounters + 1) * sizeof(int), stream) != cudaSuccess)
    return Q38_NOALLOC_ECUDA;

  CUtensorMap ma, mb;
  const uint64_t wrows = (uint64_t)m_tiles * kblocks * BM;
  if (!encode(&ma, w_tiled, wrows, BK, BK * 2, BM)) return Q38_NOALLOC_ECUDA;
  if (!encode(&mb, x, (uint64_t)T, (uint64_t)K, (uint64_t)K * 2, 32)) return Q38_NOALLOC_ECUDA;

  GemmArgs g{};
  g.M = N;
  g.N = T;
  g.K = K;
  g.kblocks = kblocks;
  g.kps = kps;
  g.splits = splits;
  g.out = out;
  g.ldo = ldo;
  g.ws = partials;
  g.counters = counters;
  g.err = err;
  const dim3 grid(m_tiles, 1, splits);
  cudaError_t e;
  if (epi == EPI_BF16) e = launch<EPI_BF16>(ma, mb, g, grid, stream);
  else if (epi == EPI_F32) e = launch<EPI_F32>(ma, mb, g, grid, stream);
  else e = launch<EPI_ADD_F32>(ma, mb, g, grid, stream);
  return e == cudaSuccess ? Q38_NOALLOC_OK : Q38_NOALLOC_ECUDA;
}

// Error word of the last call on the current device (wait timeouts, see csrc/common.cuh); copies one
// int to the host after synchronising the device.  Returns -1 if the scratch is not set up.
extern "C" __attribute__((visibility("default"))) int q38_linear_noalloc_status(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= q38::noalloc::kMaxDevices) return -1;
  if (q38::noalloc::g_scratch_dev[dev] == nullptr) return -1;
  int v = 0;
  const unsigned char* base = static_cast<const unsigned char*>(q38::noalloc::g_scratch_dev[dev]);
  const int* err = reinterpret_cast<const int*>(base + q38::noalloc::kPartialFloats * 4) + q38::noalloc::kCounters;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpy(&v, err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  return v;
}
