// Decode / verify attention on the 5th-generation tensor cores (K-ATTN-DECODE/VERIFY, head dim 256).
//
// The work split is the one of the mma.sync kernel in attention.cu: one CTA per (KV head, key
// group) over the fixed absolute partition of the key axis (attention.cu `groups_for`), a
// (max, sum, unnormalised O) partial per query vector and group, merged in group order by
// `attn_combine_kernel` (which also applies the sigmoid gate).  What changes is how a CTA works:
//
//  * the GQA group's query vectors (rep heads x T rows, up to 128 per pass) are the M = 128 side
//    of `tcgen05.mma`; Q is staged once in shared memory in the 128-byte-swizzled K-major layout;
//  * each 128-key tile of K and V arrives by TMA (plain 2-D tiled loads of this GPU's own paged
//    cache, one 16-key page x 64 columns per box, no multicast) straight into the swizzled
//    operand layouts: K as the K-major B operand of S = Q K^T, V as the MN-major B operand of
//    O += P V;
//  * S (128 x 128 fp32) and O (128 x 256 fp32) accumulate in tensor memory; one thread per query
//    row (its TMEM lane) applies the mask and the online softmax, writes P in bf16 as the A operand
//    of the second MMA, and rescales its O row in TMEM when its running max grows;
//  * tiles whose keys were all committed before this step are requested before the
//    programmatic-dependent-launch wait (the previous kernel only writes this step's rows), so
//    their HBM round trip overlaps the previous kernel's tail.
//
// Batch invariance (a verify row gives the bits of the same row decoded alone) holds as in the
// mma.sync kernel: each S / O element depends only on its own query row, the key tiles are fixed
// absolute ranges, and a tile past a row's position adds exact zeros with a rescale of exactly 1.
//
// Reference: the paged flash-decode SDPA the reference runs per verify block
// (optimisation/ttnn-op/k64j/kernels/compute/sdpa_flash_decode_qwen.cpp) and its call site
// (docker/qwen-c2-graft/graft/attention/tp.py:645).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "attn_groups.cuh"
#include "common.cuh"

namespace q38 {

CUtensorMap make_map_2d(const void* ptr, int64_t rows, int64_t cols, int64_t row_stride_elems, int box_rows);

namespace attn_tc {

constexpr int D = 256;              // head dim
constexpr int M = 128;              // query vectors per pass (UMMA M, TMEM lanes)
constexpr int KT = 128;             // keys per tile (one 128-key chunk of the partition)
constexpr int PAGE = 16;            // keys per TMA box (one KV-cache block)
constexpr int PANEL = 64;           // bf16 columns per 128-byte swizzled row
constexpr int PANEL_BYTES = 128 * 128;             // 128 rows x 128 B
constexpr int Q_OFF = 0;                           // Q: 4 panels (D)
constexpr int K_OFF = Q_OFF + (D / PANEL) * PANEL_BYTES;       // K: 4 panels (D) of 128 keys
constexpr int V_OFF = K_OFF + (D / PANEL) * PANEL_BYTES;       // V: 4 panels (D) of 128 keys
constexpr int P_OFF = V_OFF + (D / PANEL) * PANEL_BYTES;       // P: 2 panels (keys) of 128 rows
constexpr int BAR_OFF = P_OFF + (KT / PANEL) * PANEL_BYTES;
constexpr int SMEM = BAR_OFF + 64 + 1024;          // barriers + slack for 1024-byte alignment
constexpr int TILE_TX = (KT / PAGE) * (D / PANEL) * PAGE * PANEL * 2;   // bytes per K or V tile
constexpr int TMEM_COLS = 512;      // S: columns [0, 128), O: [256, 512)
constexpr int S_COL = 0, O_COL = 256;
constexpr int NT = 128;

// byte offset of 16-byte chunk c (0..7) of row r inside a 128B-swizzled panel
__device__ __forceinline__ uint32_t sw128(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// MN-major operand descriptor, 128-byte swizzle: atoms of 8 K-rows x 64 MN elements (1024 B);
// `lbo` = byte distance between 64-element MN blocks, `sbo` = between 8-row K groups.
__device__ __forceinline__ uint64_t smem_desc_sw128_mn(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// kind::f16 instruction descriptor, bf16 inputs, fp32 accumulate, A K-major, B K- or MN-major
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn_major ? (1u << 16) : 0u) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

struct Args {
  const __nv_bfloat16* q;      // [T, nq, D]
  const int* block_table;      // paged cache (PAGE-key blocks) or nullptr: contiguous rows
  int cache_rows;              // rows of the 2-D cache view (blocks x PAGE, or positions)
  const int* qpos;             // [T]
  int T, nq, nkv;
  float scale;
  int causal;
  float* part_o;               // [nkv, max_splits, nqv, D]
  float* part_ml;              // [nkv, max_splits, nqv, 2]
  int max_splits;
  int* err;
};

// Issues the TMA boxes of one 128-key tile of K (or V) into `dst` (4 panels x 128 keys x 128 B):
// page i of the tile (keys k0 + 16 i ..) comes from cache block block_table[(k0 + 16 i) / 16];
// pages past the last key load the sequence's first block instead (finite data, masked to p = 0).
__device__ __forceinline__ void load_tile(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, const Args& a,
                                          int g, int k0, int n_keys) {
#pragma unroll 1
  for (int i = 0; i < KT / PAGE; ++i) {
    const int kp = k0 + i * PAGE;
    int row;
    if (a.block_table) row = a.block_table[(kp < n_keys ? kp : 0) / PAGE] * PAGE;
    else row = kp < n_keys ? kp : 0;
#pragma unroll
    for (int p = 0; p < D / PANEL; ++p)
      tma_load_2d(dst + p * PANEL_BYTES + i * PAGE * 128, map, bar, g * D + p * PANEL, row);
  }
}

__global__ void __launch_bounds__(NT, 1)
attn_decode_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* kbar = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* vbar = kbar + 1;
  uint64_t* sbar = kbar + 2;
  uint64_t* obar = kbar + 3;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(kbar + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int g = blockIdx.x, grp = blockIdx.y;
  const int rep = a.nq / a.nkv, nqv = rep * a.T;
  const int n_keys = a.qpos[a.T - 1] + 1;                // positions are inputs of the whole step
  const int c0 = group_first_chunk(grp);
  const int k_begin = c0 * CH;
  if (k_begin >= n_keys) return;                         // CTA-uniform: before any barrier or TMEM
  const int k_end = min(n_keys, (c0 + group_chunks(grp)) * CH);
  const int ntiles = (k_end - k_begin + KT - 1) / KT;
  const int first_new = a.qpos[0];                       // keys >= this are written by this step

  if (tid == 0) {
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
    for (int i = 0; i < 4; ++i) mbar_init(kbar + i, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // the first tile's K and V before the wait when none of its keys is written by this step
  const bool early = k_begin + KT <= first_new && k_begin + KT <= k_end;
  if (tid == 0 && early) {
    mbar_expect_tx(kbar, TILE_TX);
    load_tile(smem + K_OFF, &kmap, kbar, a, g, k_begin, n_keys);
    mbar_expect_tx(vbar, TILE_TX);
    load_tile(smem + V_OFF, &vmap, vbar, a, g, k_begin, n_keys);
  }
  pdl_wait();
  pdl_trigger();

  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);      // this warp's TMEM lanes
  constexpr uint32_t IDESC_S = idesc_bf16(M, KT, false);
  constexpr uint32_t IDESC_O = idesc_bf16(M, D, true);
  int phase = 0;                                                   // tiles issued so far (all passes)
  for (int qb = 0; qb < nqv; qb += M) {
    // ---- this pass's query vectors into the swizzled K-major Q operand (zeros past nqv)
    for (int idx = tid; idx < M * (D / 8); idx += NT) {
      const int r = idx / (D / 8), ch = idx % (D / 8);
      uint8_t* dst = smem + Q_OFF + (ch / 8) * PANEL_BYTES + sw128(r, ch % 8);
      const int qv = qb + r;
      if (qv < nqv) {
        const int hq = g * rep + qv / a.T, t = qv % a.T;
        cp_async16(dst, reinterpret_cast<const uint4*>(a.q + ((size_t)t * a.nq + hq) * D) + ch);
      } else {
        *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    cp_async_commit();
    cp_async_wait<0>();
    fence_proxy_async_smem();
    // this thread's query row (TMEM lane == row)
    const int qv = qb + tid;
    const bool rv = qv < nqv;
    const int p_row = rv ? (a.causal ? a.qpos[qv % a.T] : n_keys - 1) : -1;
    float m_run = -INFINITY, l_run = 0.f;
    // this pass's first tile: K and V (unless requested before the PDL wait); the previous pass's
    // last P V must be done before V, P and O are reused
    if (phase > 0) {
      mbar_wait(obar, (uint32_t)((phase - 1) & 1), a.err, kErrMmaWait, abort_flag);
      tc_fence_after();
    }
    if (tid == 0 && !(early && phase == 0)) {
      mbar_expect_tx(kbar, TILE_TX);
      load_tile(smem + K_OFF, &kmap, kbar, a, g, k_begin, n_keys);
      mbar_expect_tx(vbar, TILE_TX);
      load_tile(smem + V_OFF, &vmap, vbar, a, g, k_begin, n_keys);
    }
    for (int kt = 0; kt < ntiles; ++kt, ++phase) {
      const int k0 = k_begin + kt * KT;
      const uint32_t par = (uint32_t)(phase & 1);
      __syncthreads();                                  // Q staged / previous tile's P published
      if (tid == 32) {
        // ---- S = Q K^T (M = 128 queries, N = 128 keys, K = 256)
        if (mbar_wait(kbar, par, a.err, kErrTmaWait, abort_flag)) {
          tc_fence_after();
          const uint32_t qs = smem_u32(smem + Q_OFF), ks = smem_u32(smem + K_OFF);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk / 4) * PANEL_BYTES + (kk % 4) * 32;
            umma_bf16(tmem + S_COL, smem_desc_sw128(qs + off), smem_desc_sw128(ks + off), IDESC_S,
                      kk > 0 ? 1u : 0u);
          }
        }
        umma_commit(sbar);
      }
      __syncwarp();
      mbar_wait(sbar, par, a.err, kErrMmaWait, abort_flag);
      tc_fence_after();
      // K is free once S is computed: the next tile's K streams in under this tile's softmax
      if (tid == 0 && kt + 1 < ntiles) {
        mbar_expect_tx(kbar, TILE_TX);
        load_tile(smem + K_OFF, &kmap, kbar, a, g, k0 + KT, n_keys);
      }
      // V, P and O are free once the previous tile's P V is done: this tile's V streams in under
      // the softmax
      if (kt > 0) {
        mbar_wait(obar, par ^ 1u, a.err, kErrMmaWait, abort_flag);
        tc_fence_after();
        if (tid == 0) {
          mbar_expect_tx(vbar, TILE_TX);
          load_tile(smem + V_OFF, &vmap, vbar, a, g, k0, n_keys);
        }
      }
      // ---- online softmax of this thread's query row over the tile (two passes over S in TMEM:
      //      the tile max, then p = exp(s - m) into the bf16 P operand and the row sum)
      float tmax = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < KT / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(trow + S_COL + c * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int kp = k0 + c * 32 + j;
          if (kp < k_end && kp <= p_row) tmax = fmaxf(tmax, __uint_as_float(v[j]) * a.scale);
        }
      }
      const float m_new = fmaxf(m_run, tmax);
      const float mz = m_new == -INFINITY ? 0.f : m_new;
      const float corr = __expf(m_run - mz);          // 0 before any key, exactly 1 if unchanged
      float lt = 0.f;
#pragma unroll 1
      for (int c = 0; c < KT / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(trow + S_COL + c * 32, v);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const int kp = k0 + c * 32 + j;
          const float p0 = (kp < k_end && kp <= p_row) ? __expf(__uint_as_float(v[j]) * a.scale - mz) : 0.f;
          const float p1 = (kp + 1 < k_end && kp + 1 <= p_row) ? __expf(__uint_as_float(v[j + 1]) * a.scale - mz)
                                                               : 0.f;
          lt += p0;
          lt += p1;
          __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
          pk[j / 2] = *reinterpret_cast<uint32_t*>(&b2);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {              // 8 keys per 16-byte chunk
          const int kk = c * 32 + u * 8;
          *reinterpret_cast<uint4*>(smem + P_OFF + (kk / PANEL) * PANEL_BYTES + sw128(tid, (kk % PANEL) / 8)) =
              make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
      }
      l_run = l_run * corr + lt;
      m_run = m_new;
      // ---- O *= corr where a row's max grew (later tiles of a multi-chunk group; warp-uniform)
      if (kt > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(trow + O_COL + c * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) * corr);
          tmem_st_32x32b_x32(trow + O_COL + c * 32, v);
        }
        tmem_st_wait();
      }
      fence_proxy_async_smem();                      // P (generic stores) -> the MMA's async reads
      tc_fence_before();
      __syncthreads();
      if (tid == 32) {
        // ---- O += P V (M = 128 queries, N = 256, K = 128 keys; V MN-major)
        tc_fence_after();
        if (mbar_wait(vbar, par, a.err, kErrTmaWait, abort_flag)) {
          tc_fence_after();
          const uint32_t ps = smem_u32(smem + P_OFF), vs = smem_u32(smem + V_OFF);
#pragma unroll
          for (int kk = 0; kk < KT / 16; ++kk) {
            const uint64_t da = smem_desc_sw128(ps + (kk / 4) * PANEL_BYTES + (kk % 4) * 32);
            const uint64_t db = smem_desc_sw128_mn(vs + kk * 16 * 128, PANEL_BYTES, 1024);
            umma_bf16(tmem + O_COL, da, db, IDESC_O, (kt > 0 || kk > 0) ? 1u : 0u);
          }
        }
        umma_commit(obar);
      }
      __syncwarp();
    }
    // ---- the pass's partials: (m, l) and the unnormalised O row of every query vector
    mbar_wait(obar, (uint32_t)((phase - 1) & 1), a.err, kErrMmaWait, abort_flag);
    tc_fence_after();
    const size_t prow = ((size_t)g * a.max_splits + grp) * nqv + qv;
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(trow + O_COL + c * 32, v);
      tmem_ld_wait();
      if (rv) {
        float4* dst = reinterpret_cast<float4*>(a.part_o + prow * D + c * 32);
#pragma unroll
        for (int u = 0; u < 8; ++u)
          dst[u] = make_float4(__uint_as_float(v[4 * u]), __uint_as_float(v[4 * u + 1]),
                               __uint_as_float(v[4 * u + 2]), __uint_as_float(v[4 * u + 3]));
      }
    }
    if (rv) {
      a.part_ml[prow * 2] = m_run;
      a.part_ml[prow * 2 + 1] = l_run;
    }
    tc_fence_before();
    __syncthreads();                                 // O read out before the next pass reuses it
    tc_fence_after();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace attn_tc
}  // namespace q38

// Launches the tcgen05 decode kernel for the partial (m, l, O) of every (KV head, key group) and
// query vector; the caller runs the combine kernel.  Returns false when this shape is not served
// (head dim, block size or alignment), so the caller takes the mma.sync kernel.
bool q38_attn_decode_tc(const torch::Tensor& q, const torch::Tensor& kcache, const torch::Tensor& vcache,
                        const int* block_table, int block_size, const int* qpos, int T, int nq, int nkv, float scale,
                        int causal, float* part_o, float* part_ml, int max_splits, int* err, cudaStream_t st) {
  using namespace q38::attn_tc;
  const int Dq = (int)q.size(2);
  if (Dq != D || (block_table && block_size != PAGE)) return false;
  if (!kcache.is_contiguous() || !vcache.is_contiguous() || !q.is_contiguous()) return false;
  if (((reinterpret_cast<uintptr_t>(kcache.data_ptr()) | reinterpret_cast<uintptr_t>(vcache.data_ptr())) & 15) != 0)
    return false;
  static int enabled = -1;
  if (enabled < 0) {
    const char* e = getenv("Q38_ATTN_TC");
    enabled = (e && e[0] == '0') ? 0 : 1;
  }
  if (!enabled) return false;
  const int64_t cols = (int64_t)nkv * D;
  const int64_t rows = kcache.numel() / cols;
  CUtensorMap km = q38::make_map_2d(kcache.data_ptr(), rows, cols, cols, PAGE);
  CUtensorMap vm = q38::make_map_2d(vcache.data_ptr(), rows, cols, cols, PAGE);
  Args a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.block_table = block_table;
  a.cache_rows = (int)rows;
  a.qpos = qpos;
  a.T = T;
  a.nq = nq;
  a.nkv = nkv;
  a.scale = scale;
  a.causal = causal;
  a.part_o = part_o;
  a.part_ml = part_ml;
  a.max_splits = max_splits;
  a.err = err;
  TORCH_CHECK(q38::set_smem_once<attn_decode_tc_kernel>(SMEM) == cudaSuccess, "cudaFuncSetAttribute failed");
  const dim3 grid((unsigned)nkv, (unsigned)q38::groups_for(max_splits));
  TORCH_CHECK(q38::launch_pdl(attn_decode_tc_kernel, grid, dim3(NT), (size_t)SMEM, st, km, vm, a) == cudaSuccess,
              "tcgen05 decode attention launch failed");
  return true;
}
