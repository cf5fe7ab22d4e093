// tcgen05 GEMM family for the hybrid target: D[m, n] = sum_k A[m, k] * B[n, k]  (both K-major bf16).
//
// One warp-specialised kernel, two roles:
//  * swap-AB streaming (decode / verify, <= 32 token rows): A = weight [N_out, K] (the 128-row
//    UMMA M side), B = token rows [T, K] (N = 32).  Weight tiles stream through a TMA ring at HBM
//    rate; split-K over K blocks is reduced by the last-arriving CTA of each tile in a fixed order,
//    so a token row's result never depends on how many rows ran with it (verify rows are bit-
//    identical to single-row decode).
//  * prefill tiles (> 32 rows): A = tokens [T, K], B = weight [N_out, K], 128 x 256 tiles.
// Roles inside a 128-thread CTA: thread 0 issues TMA loads, thread 32 issues tcgen05.mma (one
// elected thread), all four warps drain TMEM with tcgen05.ld in the epilogue.  Epilogues: bf16
// store, fp32 store, fp32 accumulate into the residual stream, SwiGLU over [gate 64 | up 64] row
// blocks, per-tile argmax (LM head), and (swap mode) the fused tensor-parallel all-reduce:
//
// EPI_PUSH_F32 - the GEMM half of the tensor-parallel all-reduce of a row-parallel out-projection
// (TP > 1).  As soon as a tile's split-K fix-up is done, the fixing CTA stores its fp32 partial
// tile into its own block of every rank's receive area over NVLink (tile t crosses NVLink while
// later tiles are still in the MMA), each value as one 8-byte word {value, epoch}: a single
// 64-bit store is observed whole, so the reader needs no fence or flag - it spins (bounded) on
// each word until the epoch of this use of the slot appears.  The GEMM never waits; the kernel
// that consumes the residual next (`rms_norm_ar_kernel`, misc.cu) completes the reduction.
#pragma once
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include <cooperative_groups.h>

#include "common.cuh"

namespace q38 {

enum Epi : int {
  EPI_BF16 = 0, EPI_F32 = 1, EPI_ADD_F32 = 2, EPI_SWIGLU = 3, EPI_ARGMAX = 4, EPI_PUSH_F32 = 5,
  EPI_RS_F32 = 6,   // prefill tiles: fp32 partial straight into the owning rank's reduce-scatter area
  EPI_SPLIT_F32 = 7,  // swap mode: every split-K slice stores its own fp32 partial ([split][token][N] at
                      // g.out, token stride ldo); no fix-up: the consumer adds the slices in split order
};

constexpr int AR_MAX_RANKS = 8;

// Peer buffers of the pushed all-reduce.  Receive area of every rank: blocks [slot][src rank]
// of `block_words` 8-byte words {fp32 value, epoch}, each a [tokens, ldo] partial.
constexpr int SWAP_MAX_ROWS = 64;  // token rows the swap-AB (weight-streaming) GEMM serves, in 32-row tiles
constexpr int AR_MAX_ROWS = 64;   // rows of one pushed all-reduce (a packed verify of up to 4 x 16)

struct ArArgs {
  long long recv[AR_MAX_RANKS];    // every rank's receive area (8-byte words), mapped into this process
  long long mc;                    // NVLS multicast address of the receive areas (0: per-rank stores)
  long long block_words;           // words per (slot, source rank) block: [AR_MAX_ROWS][ldo]
  int rank, world, slot;
  const int* epochs;               // this rank's [slots][AR_MAX_ROWS] epochs (advanced by the reader)
};

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* addr, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(addr), "l"(v) : "memory");
}
// One 8-byte store through the NVSwitch multicast object: every rank's copy receives the word.
__device__ __forceinline__ void multimem_st_u64(unsigned long long* mc_addr, unsigned long long v) {
  asm volatile("multimem.st.relaxed.sys.global.u64 [%0], %1;" ::"l"(mc_addr), "l"(v) : "memory");
}

// Push of one {value, epoch} word to every rank's copy of this rank's receive block: a single
// multicast store when the areas are bound to an NVLS multicast object, else one store per rank.
__device__ __forceinline__ void push_word(const ArArgs& a, size_t word, unsigned long long v) {
  if (a.mc) {
    multimem_st_u64(reinterpret_cast<unsigned long long*>(a.mc) + word, v);
  } else {
    for (int p = 0; p < a.world; ++p) st_relaxed_sys_u64(reinterpret_cast<unsigned long long*>(a.recv[p]) + word, v);
  }
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* addr) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(addr) : "memory");
  return v;
}

// Reduce-scatter of a prefill out-projection (EPI_RS_F32, tile mode): 128-row token tile t belongs
// to rank t % world, which keeps its tiles at local rows (t / world) * 128 ..; a source writes its
// fp32 tile into [source rank][local row][ldo] of the owner's area, then adds 1 to the owner's
// arrival counter with a system-scope release (prefill_ar.cu reduces and broadcasts the rows).
struct RsArgs {
  long long recv[AR_MAX_RANKS];    // every rank's reduce-scatter area, mapped into this process
  long long count[AR_MAX_RANKS];   // every rank's arrival counter (u64)
  int rank, world, rows_cap;       // rows_cap: local rows per source block
};

constexpr int BM = 128;
constexpr int BK = 64;

struct GemmArgs {
  int M, N, K;
  int kblocks, kps;           // total 64-wide K blocks, K blocks per split
  int splits;
  void* out;
  long long ldo;
  float* ws;                  // split-K partials
  int* counters;              // split-K arrival counters (left at zero)
  int* err;
  float* amax_val;            // EPI_ARGMAX partials [m_tiles, N]
  int* amax_idx;
  ArArgs ar;                  // EPI_PUSH_F32 only
  RsArgs rs;                  // EPI_RS_F32 only
  unsigned long long* trace;  // optional per-CTA %globaltimer stamps [grid][8] (micro-benchmarks)
  const float* samp_scale;    // EPI_ARGMAX: per token row 1/temperature (0: greedy), or nullptr
  const unsigned long long* samp_key;   // per token row noise key
  long long vocab_off;        // global vocabulary index of weight row 0 (noise index)
  int cluster_k;              // swap mode, splits > 1: the splits of a tile form one cluster and
                              // reduce through DSMEM (the launch sets cluster dims (1, 1, splits));
                              // 0: partials through `ws` and the last-arriving CTA (`counters`)
  const uint8_t* mxq;         // MX weights (swap mode): e4m3 bytes, tile (t, kb) = [128 rows][64] at
                              // ((t * kblocks + kb) * 8192)
  const uint8_t* mxs;         // their E8M0 scales, tile (t, kb) = [128 rows][2] at ((t * kblocks + kb) * 256)
};

// trace points: 0 entry, 1 setup done, 2 first stage landed, 3 last MMA issued, 4 accumulator
// ready, 5 split-K partial published, 6 epilogue done, 7 exit
#define Q38_STAMP(k)                                                                                   \
  do {                                                                                                 \
    if (g.trace)                                                                                       \
      g.trace[((size_t)(blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x) * 8 + (k)] =    \
          globaltimer();                                                                               \
  } while (0)

template <int BN, int STAGES>
struct Smem {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int NST = STAGES;                // operand ring slots
  static constexpr int RS = 0;                      // MX load ring slots (none)
  static constexpr int R_OFF = 0, RSLOT = 0;       // (MX load ring only)
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = RING_BYTES;
  static constexpr int TOTAL = BAR_OFF + (2 * STAGES + 2) * 8 + 16 + 1024;  // + alignment slack
};

// MX (block-scaled e4m3 weight) swap-mode layout.  A load ring of RS slots {activation tile (the
// MMA's B operand, written swizzled by TMA), 8 KB of e4m3 weight bytes, 256 B of E8M0 scales} that
// one barrier covers, and an operand ring of NST bf16 weight tiles in the 128-byte-swizzled K-major
// layout the MMA reads, written by two converter warps.  A load slot is free once the converters
// and the MMA are both done with it; the producer never waits for a conversion, so RS stages of
// weight bytes stay in flight.  The whole region is also the split-K fix-up's staging area.
struct SmemMx {
  static constexpr int A_BYTES = BM * BK * 2;       // one bf16 weight tile (operand ring slot)
  static constexpr int B_BYTES = 32 * BK * 2;       // one activation tile
  static constexpr int RAW_Q = BM * BK;             // e4m3 bytes of one weight tile
  static constexpr int RAW_S = BM * (BK / 32);      // its scales
  static constexpr int RSLOT = 13 * 1024;           // B | q | scales, 1024-aligned slots
  static constexpr int NST = 3;
  static constexpr int RS = 4;
  static constexpr int PF = 12;                     // stages prefetched into L2 beyond the load ring
  static constexpr int STAGE_BYTES = A_BYTES;
  static constexpr int R_OFF = NST * A_BYTES;
  static constexpr int RING_BYTES = R_OFF + RS * RSLOT;
  static constexpr int BAR_OFF = RING_BYTES;
  static constexpr int TOTAL = BAR_OFF + (2 * NST + 2 * RS + 2) * 8 + 16 + 1024;
  static_assert(B_BYTES + RAW_Q + RAW_S <= RSLOT, "load slot too small");
};

// Four e4m3 bytes -> four bf16 values times 2^-120 (two bf16x2 words), exact for every finite e4m3
// including subnormals: the e4m3 sign moves to bit 15 and its 7 exponent+mantissa bits to bits
// 10..4, so the bf16 exponent field equals the e4m3 one and the bf16 bias (127) is 120 above the
// e4m3 bias (7).  The multiply by a power of two m2 (bf16x2) restores the block scale.
__device__ __forceinline__ void e4m3x4_to_bf16x4_scaled(uint32_t w, uint32_t m2, uint32_t& lo, uint32_t& hi) {
  const uint32_t t0 = __byte_perm(w, 0u, 0x1404u);  // [0, b0, 0, b1]
  const uint32_t t1 = __byte_perm(w, 0u, 0x3424u);  // [0, b2, 0, b3]
  const uint32_t f0 = (t0 & 0x80008000u) | ((t0 >> 4) & 0x07F007F0u);
  const uint32_t f1 = (t1 & 0x80008000u) | ((t1 >> 4) & 0x07F007F0u);
  // exact products (a power-of-two factor, no rounding; bf16 arithmetic keeps subnormal inputs)
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(lo) : "r"(f0), "r"(m2));
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(hi) : "r"(f1), "r"(m2));
}

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
// AND of `pred` over the `n` threads of named barrier `id` (every one of them calls it).
__device__ __forceinline__ bool named_bar_and(int id, int n, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

// Swap-mode split-K through distributed shared memory.  The `splits` CTAs of one weight tile are
// one thread-block cluster (cluster rank = split).  Each CTA parks its fp32 accumulator tile
// [32 tokens][128 rows] in its own (now idle) operand ring; after one cluster barrier, CTA c sums
// every split's values for its slice of the tile's output units in split order 0, 1, .. (the
// same additions, in the same order, as the last-arriving-CTA fix-up, so the bits do not depend on
// the path) and runs the epilogue for that slice; a second barrier keeps each CTA's tile alive
// until its peers have read it.  Compared with the global-memory fix-up this drops the partial
// round trip through L2, the fence, the arrival counter and the serial tail in one CTA, and the
// epilogue (the residual update or the NVLink push of EPI_PUSH_F32) runs on every CTA of the tile.
// Output units: one weight row (128 per tile), or for SwiGLU one [gate, up] row pair (64 per tile).
// A CTA whose mbarrier wait gave up contributes zeros; the error word already carries the failure.
template <int EPI>
__device__ __forceinline__ void swap_cluster_epilogue(const GemmArgs& g, float* tile_s, uint32_t trow, bool have,
                                                      int m_tile, int split, int row) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  {
    uint32_t r[32];
    if (have) {
      tmem_ld_32x32b_x32(trow, r);
      tmem_ld_wait();
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) tile_s[j * BM + row] = have ? __uint_as_float(r[j]) : 0.f;
  }
  cluster.sync();
  if (threadIdx.x == 0) Q38_STAMP(5);
  constexpr bool SW = EPI == EPI_SWIGLU;
  constexpr int UNITS = SW ? BM / 2 : BM;
  constexpr int EMAX = (UNITS / 2) * 32 / 128;       // elements per thread at splits >= 2
  const int S = g.splits;
  const int per = (UNITS + S - 1) / S;
  const int u0 = min(UNITS, split * per), nu = min(UNITS, u0 + per) - u0;
  const int nvalid = min(32, g.N);
  const int nel = nu * nvalid;
  const float* peer[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) peer[q] = q < S ? cluster.map_shared_rank(tile_s, q) : tile_s;
  // every element's split sum first (all DSMEM loads in flight), then the memory epilogue with
  // every global load issued before any dependent store
  float v[EMAX];
  int off[EMAX];
#pragma unroll
  for (int k = 0; k < EMAX; ++k) {
    const int e = threadIdx.x + k * 128;
    const int u = u0 + (e < nel ? e % nu : 0), j = e < nel ? e / nu : 0;
    float acc = 0.f, up = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (q < S && e < nel) {
        acc += peer[q][j * BM + u];
        if constexpr (SW) up += peer[q][j * BM + u + BM / 2];
      }
    }
    if constexpr (SW) {
      v[k] = silu_f(acc) * up;
      off[k] = e < nel ? (int)(j * g.ldo + m_tile * (BM / 2) + u) : -1;
    } else {
      v[k] = acc;
      off[k] = (e < nel && m_tile * BM + u < g.M) ? (int)(j * g.ldo + m_tile * BM + u) : -1;
    }
  }
  if constexpr (EPI == EPI_ADD_F32) {
    float* o = reinterpret_cast<float*>(g.out);
    float r[EMAX];
#pragma unroll
    for (int k = 0; k < EMAX; ++k) r[k] = off[k] >= 0 ? o[off[k]] : 0.f;
#pragma unroll
    for (int k = 0; k < EMAX; ++k)
      if (off[k] >= 0) o[off[k]] = r[k] + v[k];
  } else if constexpr (EPI == EPI_BF16 || SW) {
#pragma unroll
    for (int k = 0; k < EMAX; ++k)
      if (off[k] >= 0) reinterpret_cast<__nv_bfloat16*>(g.out)[off[k]] = __float2bfloat16(v[k]);
  } else if constexpr (EPI == EPI_F32) {
#pragma unroll
    for (int k = 0; k < EMAX; ++k)
      if (off[k] >= 0) reinterpret_cast<float*>(g.out)[off[k]] = v[k];
  } else if constexpr (EPI == EPI_PUSH_F32) {
    const ArArgs& a = g.ar;
    const size_t mine = (size_t)(a.slot * a.world + a.rank) * a.block_words;
#pragma unroll
    for (int k = 0; k < EMAX; ++k) {
      if (off[k] < 0) continue;
      const int j = off[k] / (int)g.ldo;
      const unsigned long long w =
          ((unsigned long long)((uint32_t)a.epochs[(size_t)a.slot * AR_MAX_ROWS + j] + 1u) << 32) |
          __float_as_uint(v[k]);
      push_word(a, mine + off[k], w);
    }
  }
  cluster.sync();
}

template <int BN, int STAGES, int EPI, bool SWAP, bool MX = false>
__global__ void __launch_bounds__(MX ? 256 : 128, MX ? 2 : 1)
gemm_tn_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, GemmArgs g) {
  static_assert(!MX || (SWAP && BN == 32), "MX weights stream through the swap-mode kernel");
  using S = typename std::conditional<MX, SmemMx, Smem<BN, STAGES>>::type;
  constexpr int NST = S::NST;
  // CTA barrier of the epilogue threads: in the MX kernel warps 4-7 (converters) have left by then
  auto cta_sync = [] {
    if constexpr (MX) named_bar_sync(2, 128);
    else __syncthreads();
  };
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint64_t* empty_bar = full_bar + NST;
  uint64_t* rfull_bar = empty_bar + NST;         // MX load ring: activation, weight bytes, scales landed
  uint64_t* rempty_bar = rfull_bar + S::RS;      // MX load ring: converted and consumed by the MMA
  uint64_t* acc_bar = rempty_bar + S::RS;
  uint64_t* fix_bar = acc_bar + 1;                // split-K fix-up: staged partials landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 2);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) Q38_STAMP(0);
  const int m_tile = blockIdx.x, n_tile = blockIdx.y, split = blockIdx.z;
  const int m0 = m_tile * BM, n0 = n_tile * BN;
  const int kb0 = split * g.kps;
  const int kb1 = min(g.kblocks, kb0 + g.kps);
  const int nk = kb1 - kb0;
  constexpr int TMEM_COLS = BN < 32 ? 32 : BN;

  if (tid == 0) {
    if constexpr (!MX) tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full_bar[s], 1);                // MX: the converters' arrival
      mbar_init(&empty_bar[s], 1);
    }
    for (int s = 0; s < S::RS; ++s) {
      mbar_init(&rfull_bar[s], 1);
      mbar_init(&rempty_bar[s], 2);              // the converters and the MMA's commit
    }
    mbar_init(acc_bar, 1);
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
  if (tid == 0) {
    Q38_STAMP(1);
    pdl_trigger();
  }

  if (tid == 0) {
    // ---------------- TMA producer
    // Weights are stored tile-contiguous (wtile row (t * kblocks + kb) * 128 + r holds weight row
    // 128 t + r, columns 64 kb ..): every weight tile is one contiguous 16 KB block.  The weight
    // operand (A in swap mode, B otherwise) is static, so its first STAGES tiles are requested
    // before waiting for the previous kernel; activation tiles after.
    const uint64_t pol_w = policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    auto load_w = [&](int stage, int kb) {
      uint8_t* sa = smem + stage * S::STAGE_BYTES;
      if constexpr (SWAP) {
        tma_load_2d_hint(sa, &map_a, &full_bar[stage], 0, (m_tile * g.kblocks + kb) * BM, pol_w);
      } else {
        uint8_t* sb = sa + S::A_BYTES;
#pragma unroll
        for (int j = 0; j < BN / BM; ++j)
          tma_load_2d_hint(sb + j * (BM * BK * 2), &map_b, &full_bar[stage], 0,
                           ((n_tile * (BN / BM) + j) * g.kblocks + kb) * BM, pol_w);
      }
    };
    auto load_x = [&](int stage, int kb) {
      uint8_t* sa = smem + stage * S::STAGE_BYTES;
      if constexpr (SWAP) tma_load_2d_hint(sa + S::A_BYTES, &map_b, &full_bar[stage], kb * BK, n0, pol_x);
      else tma_load_2d_hint(sa, &map_a, &full_bar[stage], kb * BK, m0, pol_x);
    };
    if constexpr (!MX) {
      const int pre = nk < STAGES ? nk : STAGES;
      for (int i = 0; i < pre; ++i) {
        mbar_expect_tx(&full_bar[i], S::STAGE_BYTES);
        load_w(i, kb0 + i);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) load_x(i, kb0 + i);
      for (int i = pre; i < nk; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(&empty_bar[s], ((i / STAGES) - 1) & 1, g.err, kErrTmaWait, abort_flag)) break;
        mbar_expect_tx(&full_bar[s], S::STAGE_BYTES);
        load_w(s, kb0 + i);
        load_x(s, kb0 + i);
      }
    } else {
      // MX: K block kb0 + i goes to load slot i % RS: its e4m3 tile and scales by two bulk copies
      // (static: the first RS are requested before the PDL wait) and its activation tile by TMA.
      const uint8_t* wq = g.mxq + (size_t)m_tile * g.kblocks * S::RAW_Q;
      const uint8_t* wsc = g.mxs + (size_t)m_tile * g.kblocks * S::RAW_S;
      auto load_q = [&](int i) {
        const int r = i % S::RS;
        uint8_t* slot = smem + S::R_OFF + r * S::RSLOT;
        mbar_expect_tx(&rfull_bar[r], S::B_BYTES + S::RAW_Q + S::RAW_S);
        bulk_load_hint(slot + S::B_BYTES, wq + (size_t)(kb0 + i) * S::RAW_Q, S::RAW_Q, &rfull_bar[r], pol_w);
        bulk_load_hint(slot + S::B_BYTES + S::RAW_Q, wsc + (size_t)(kb0 + i) * S::RAW_S, S::RAW_S, &rfull_bar[r],
                       pol_w);
      };
      auto load_act = [&](int i) {
        const int r = i % S::RS;
        tma_load_2d_hint(smem + S::R_OFF + r * S::RSLOT, &map_b, &rfull_bar[r], (kb0 + i) * BK, n0, pol_x);
      };
      // Weight bytes also go to L2 PF stages ahead of the ring, so the ring's copies find them there:
      // the ring holds 4 x 8 KB of weight, too few bytes in flight to cover HBM latency by itself.
      auto prefetch = [&](int i) {
        if (i < nk) {
          bulk_prefetch_l2(wq + (size_t)(kb0 + i) * S::RAW_Q, S::RAW_Q);
          bulk_prefetch_l2(wsc + (size_t)(kb0 + i) * S::RAW_S, S::RAW_S);
        }
      };
      const int pre = nk < S::RS ? nk : S::RS;
      for (int i = 0; i < pre; ++i) load_q(i);
      for (int i = pre; i < pre + S::PF; ++i) prefetch(i);
      pdl_wait();
      for (int i = 0; i < pre; ++i) load_act(i);
      for (int i = pre; i < nk; ++i) {
        if (!mbar_wait(&rempty_bar[i % S::RS], ((i / S::RS) - 1) & 1, g.err, kErrTmaWait, abort_flag)) break;
        load_q(i);
        load_act(i);
        prefetch(i + S::PF);
      }
    }
  } else {
    if constexpr (MX) {
      if (warp >= 4) {
        // ---------------- MX converters (warps 4-7, which exist only in the MX kernel and leave
        // after the main loop: every later barrier names the 128 threads of warps 0-3): e4m3 x 2^(scale - 127) -> bf16, written into
        // the operand slot in the 128-byte-swizzled K-major layout (16-byte chunk c of row r at
        // c ^ (r % 8)).  Every value is exact (an e4m3 value times a power of two fits bf16), so the
        // MMA sees exactly the dequantised weight.  The weight is static: conversion starts before
        // the PDL wait.
        const int ct = tid - 128;
        long long c_raw = 0, c_empty = 0, c_work = 0;   // cycle totals (micro-benchmark trace only)
        for (int i = 0; i < nk; ++i) {
          const int r = i % S::RS, s = i % NST;
          const long long t0 = clock64();
          bool ok = mbar_wait(&rfull_bar[r], (i / S::RS) & 1, g.err, kErrTmaWait, abort_flag);
          const long long t1 = clock64();
          if (ok && i >= NST) ok = mbar_wait(&empty_bar[s], ((i / NST) - 1) & 1, g.err, kErrTmaWait, abort_flag);
          const long long t2 = clock64();
          c_raw += t2 - t0;
          (void)t1;
          if (!named_bar_and(1, 128, ok)) break;     // all converter threads leave together
          const uint8_t* raw = smem + S::R_OFF + r * S::RSLOT + S::B_BYTES;
          uint8_t* a_tile = smem + s * S::A_BYTES;
          // Thread ct handles the 16-byte chunks ct, ct + 64, ... (row = chunk / 4, quarter = chunk % 4):
          // every load is issued before any conversion or store, so the eight chunks' shared-memory
          // latencies overlap (one converter warp per scheduler has no other warps to hide them).
          constexpr int CH = (BM * BK) / (16 * 128);
          uint4 v[CH];
          uint32_t e[CH];
#pragma unroll
          for (int q = 0; q < CH; ++q) {
            const int chunk = ct + 128 * q, row = chunk >> 2, c16 = chunk & 3;
            v[q] = *reinterpret_cast<const uint4*>(raw + row * BK + c16 * 16);
            e[q] = raw[S::RAW_Q + row * (BK / 32) + (c16 >> 1)];   // scale of this 32-group
          }
#pragma unroll
          for (int q = 0; q < CH; ++q) {
            const int chunk = ct + 128 * q, row = chunk >> 2, c16 = chunk & 3;
            const uint32_t m = (e[q] + 120u) << 7;     // bf16 2^(e - 127 + 120)
            const uint32_t m2 = m | (m << 16);
            uint32_t o[8];
            e4m3x4_to_bf16x4_scaled(v[q].x, m2, o[0], o[1]);
            e4m3x4_to_bf16x4_scaled(v[q].y, m2, o[2], o[3]);
            e4m3x4_to_bf16x4_scaled(v[q].z, m2, o[4], o[5]);
            e4m3x4_to_bf16x4_scaled(v[q].w, m2, o[6], o[7]);
            uint8_t* rowp = a_tile + row * 128;
            const int sw = row & 7;
            *reinterpret_cast<uint4*>(rowp + (((2 * c16) ^ sw) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<uint4*>(rowp + (((2 * c16 + 1) ^ sw) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
          }
          const long long t3 = clock64();
          c_work += t3 - t2;
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic writes -> tensor core reads
          named_bar_sync(1, 128);
          if (ct == 0) {
            mbar_arrive(&full_bar[s]);
            mbar_arrive(&rempty_bar[r]);
          }
          c_empty += clock64() - t3;
        }
        if (g.trace && ct == 0) {
          // after the [grid][8] stamps: per CTA {converter cycles waiting for the load and a free
          // operand slot, converting (loads, expansion, stores), publishing (proxy fence, barrier,
          // arrivals); MMA thread cycles waiting for a converted tile}
          unsigned long long* mt = g.trace + (size_t)gridDim.x * gridDim.y * gridDim.z * 8 +
                                   ((size_t)(blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x) * 4;
          mt[0] = (unsigned long long)c_raw;
          mt[1] = (unsigned long long)c_work;
          mt[2] = (unsigned long long)c_empty;
        }
        return;                                   // the epilogue belongs to warps 0-3
      }
    }
    pdl_wait();     // nothing upstream is read or written before this point
  }
  if (tid == 32) {
    // ---------------- MMA issuer (single thread)
    constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
    long long c_full = 0;
    for (int i = 0; i < nk; ++i) {
      const int s = i % NST;
      const long long tw = MX ? clock64() : 0;
      if (!mbar_wait(&full_bar[s], (i / NST) & 1, g.err, kErrTmaWait, abort_flag)) break;
      if constexpr (MX) c_full += clock64() - tw;
      if constexpr (MX) {            // the activation tile of this K block (landed before the conversion)
        if (!mbar_wait(&rfull_bar[i % S::RS], (i / S::RS) & 1, g.err, kErrTmaWait, abort_flag)) break;
      }
      if (i == 0) Q38_STAMP(2);
      tc_fence_after();
      const uint32_t sa = smem_u32(smem + s * S::STAGE_BYTES);
      const uint32_t sb = MX ? smem_u32(smem + S::R_OFF + (i % S::RS) * S::RSLOT) : sa + S::A_BYTES;
      const uint64_t da = smem_desc_sw128(sa), db = smem_desc_sw128(sb);
#pragma unroll
      for (int k = 0; k < BK / 16; ++k) {
        // advance 16 bf16 (32 B) along K inside the 128-B swizzle atom
        umma_bf16(tmem, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, (i > 0 || k > 0) ? 1u : 0u);
      }
      umma_commit(&empty_bar[s]);
      if constexpr (MX) umma_commit(&rempty_bar[i % S::RS]);
    }
    if constexpr (MX) {
      if (g.trace)
        g.trace[(size_t)gridDim.x * gridDim.y * gridDim.z * 8 +
                ((size_t)(blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x) * 4 + 3] =
            (unsigned long long)c_full;
    }
    Q38_STAMP(3);
    umma_commit(acc_bar);
  }

  // ---------------- epilogue: all warps
  __syncwarp();
  mbar_wait(acc_bar, 0, g.err, kErrMmaWait, abort_flag);
  tc_fence_after();
  cta_sync();
  if (tid == 0) Q38_STAMP(4);
  const bool ok = (*abort_flag == 0);   // CTA-uniform after the barrier

  const int row = warp * 32 + lane;   // TMEM lane == tile row m
  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);

  bool clustered = false;
  if constexpr (SWAP && !MX && EPI != EPI_ARGMAX && EPI != EPI_SPLIT_F32) {
    clustered = g.splits > 1 && g.cluster_k;
    if (clustered)
      swap_cluster_epilogue<EPI>(g, reinterpret_cast<float*>(smem), trow, ok && nk > 0, m_tile, split, row);
  }
  if (ok && nk > 0 && !clustered) {
    if constexpr (SWAP) {
      // Each thread owns output feature m0+row, tokens n0 .. n0+BN-1 (BN == 32).
      static_assert(BN == 32, "swap mode uses 32 token columns");
      uint32_t r[32];
      tmem_ld_32x32b_x32(trow, r);
      tmem_ld_wait();
      float acc[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) acc[j] = __uint_as_float(r[j]);

      bool do_epi = true;
      if (g.splits > 1 && EPI != EPI_SPLIT_F32) {
        const int tile = n_tile * gridDim.x + m_tile;   // (feature tile, 32-token tile)
        float* part = g.ws + ((size_t)tile * g.splits + split) * (BM * BN);
#pragma unroll
        for (int j = 0; j < 32; ++j) part[j * BM + row] = acc[j];
        __threadfence();
        cta_sync();
        if (tid == 0) {
          const int prev = atomicAdd(&g.counters[tile], 1);
          *last_flag = (prev == g.splits - 1);
          Q38_STAMP(5);
        }
        cta_sync();
        do_epi = *last_flag != 0;
        if (do_epi) {
          __threadfence();
          // Sum the partials in split order (the fixing CTA's own from registers).  The other
          // splits' 16 KB partials are requested at once: up to RING_PARTS by bulk copies into the
          // idle operand ring (one round trip for all of them), any beyond that by direct L2 loads
          // issued before the wait.  The partials were written by other CTAs' generic stores and
          // published by the counter; the proxy fence orders the bulk (async-proxy) reads after.
          constexpr int PART = BM * BN;                                  // floats per partial
          constexpr int RING_PARTS = S::RING_BYTES / (PART * 4);
          const float* base = g.ws + (size_t)tile * g.splits * PART;
          float* stage = reinterpret_cast<float*>(smem);
          asm volatile("fence.proxy.async.global;" ::: "memory");
          if (tid == 0) {
            mbar_init(fix_bar, 1);
            fence_mbar_init();
            int k = 0;
            const int nb = min(g.splits - 1, RING_PARTS);
            mbar_expect_tx(fix_bar, (uint32_t)(nb * PART * 4));
            for (int s = 0; s < g.splits && k < nb; ++s) {
              if (s == split) continue;
              bulk_load(stage + (size_t)k * PART, base + (size_t)s * PART, PART * 4, fix_bar);
              ++k;
            }
          }
          float extra[32];                 // the one direct-loaded partial (splits - 1 > RING_PARTS)
          int extra_s = -1;
          if (g.splits - 1 > RING_PARTS) {
            extra_s = g.splits - 1 == split ? g.splits - 2 : g.splits - 1;
#pragma unroll
            for (int j = 0; j < 32; ++j) extra[j] = __ldcg(base + (size_t)extra_s * PART + j * BM + row);
          }
          cta_sync();                 // fix_bar initialised before anyone waits on it
          const bool staged = mbar_wait(fix_bar, 0, g.err, kErrSplitK, abort_flag);
          float own[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) { own[j] = acc[j]; acc[j] = 0.f; }
          if (staged) {
            int k = 0;
            for (int s = 0; s < g.splits; ++s) {
              if (s == split) {
#pragma unroll
                for (int j = 0; j < 32; ++j) acc[j] += own[j];
              } else if (s == extra_s) {
#pragma unroll
                for (int j = 0; j < 32; ++j) acc[j] += extra[j];
              } else {
                const float* sp = stage + (size_t)k * PART;
#pragma unroll
                for (int j = 0; j < 32; ++j) acc[j] += sp[j * BM + row];
                ++k;
              }
            }
          }
          cta_sync();                 // the epilogue may reuse the ring the partials sat in
          if (tid == 0) g.counters[tile] = 0;
        }
      }
      if (do_epi) {
        const int m = m0 + row;
        const int nvalid = min(32, g.N - n0);
        if constexpr (EPI == EPI_SWIGLU) {
          // rows [0,64) gate, [64,128) up of feature block m_tile; exchange up through smem
          float* up_s = reinterpret_cast<float*>(smem);   // ring is idle now
          if (row >= 64) {
#pragma unroll
            for (int j = 0; j < 32; ++j) up_s[j * 64 + (row - 64)] = acc[j];
          }
          cta_sync();
          if (row < 64) {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(g.out);
            const int f = m_tile * 64 + row;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (j < nvalid) {
                const float u = up_s[j * 64 + row];
                o[(size_t)(n0 + j) * g.ldo + f] = __float2bfloat16(silu_f(acc[j]) * u);
              }
            }
          }
        } else if constexpr (EPI == EPI_ARGMAX) {
          // per token column: max over the 128 rows of this tile, ties -> lowest row
          float* sv = reinterpret_cast<float*>(smem);
          int* si = reinterpret_cast<int*>(smem + 4 * 32 * 4);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (j >= nvalid) break;
            float v = (m < g.M) ? acc[j] : -INFINITY;
            if (g.samp_scale != nullptr && m < g.M) {      // Gumbel-max sampling rows
              const float sc = g.samp_scale[n0 + j];
              if (sc > 0.f) v = acc[j] * sc + gumbel_noise(g.samp_key[n0 + j], (unsigned long long)(g.vocab_off + m));
            }
            int idx = m;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
              const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
              const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
              if (v2 > v || (v2 == v && i2 < idx)) { v = v2; idx = i2; }
            }
            if (lane == 0) { sv[warp * 32 + j] = v; si[warp * 32 + j] = idx; }
          }
          cta_sync();
          if (tid < nvalid) {
            float v = sv[tid];
            int idx = si[tid];
#pragma unroll
            for (int w = 1; w < 4; ++w) {
              const float v2 = sv[w * 32 + tid];
              const int i2 = si[w * 32 + tid];
              if (v2 > v || (v2 == v && i2 < idx)) { v = v2; idx = i2; }
            }
            g.amax_val[(size_t)m_tile * g.N + n0 + tid] = v;
            g.amax_idx[(size_t)m_tile * g.N + n0 + tid] = idx;
          }
        } else if constexpr (EPI == EPI_PUSH_F32) {
          const ArArgs& a = g.ar;
          if (m < g.M) {
            uint32_t ep[32];
#pragma unroll
            for (int j = 0; j < 32; ++j)
              ep[j] = j < nvalid ? (uint32_t)a.epochs[(size_t)a.slot * AR_MAX_ROWS + n0 + j] + 1u : 0u;
            const size_t mine = (size_t)(a.slot * a.world + a.rank) * a.block_words;
            if (a.mc) {                                  // one multicast store reaches every rank
              unsigned long long* dst = reinterpret_cast<unsigned long long*>(a.mc) + mine;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < nvalid)
                  multimem_st_u64(dst + (size_t)(n0 + j) * g.ldo + m,
                                  ((unsigned long long)ep[j] << 32) | __float_as_uint(acc[j]));
            } else {
              for (int p = 0; p < a.world; ++p) {        // push: this rank's block in every rank
                unsigned long long* dst = reinterpret_cast<unsigned long long*>(a.recv[p]) + mine;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (j < nvalid)
                    st_relaxed_sys_u64(dst + (size_t)(n0 + j) * g.ldo + m,
                                       ((unsigned long long)ep[j] << 32) | __float_as_uint(acc[j]));
              }
            }
          }
        } else {
          // Fully unrolled over the 32 token columns (predicated), so acc[] stays in registers;
          // the residual accumulate issues every load before any add.
          if (m < g.M) {
            if constexpr (EPI == EPI_SPLIT_F32) {
              float* __restrict__ o = reinterpret_cast<float*>(g.out) + (size_t)split * g.N * g.ldo;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < nvalid) o[(size_t)(n0 + j) * g.ldo + m] = acc[j];
            } else if constexpr (EPI == EPI_ADD_F32) {
              float* __restrict__ o = reinterpret_cast<float*>(g.out);
              float r[32];
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < nvalid) r[j] = o[(size_t)(n0 + j) * g.ldo + m];
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < nvalid) o[(size_t)(n0 + j) * g.ldo + m] = r[j] + acc[j];
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (j < nvalid) {
                  const size_t off = (size_t)(n0 + j) * g.ldo + m;
                  if constexpr (EPI == EPI_BF16) reinterpret_cast<__nv_bfloat16*>(g.out)[off] = __float2bfloat16(acc[j]);
                  else reinterpret_cast<float*>(g.out)[off] = acc[j];
                }
              }
            }
          }
        }
      }
    } else {
      // Non-swap: thread owns token row m0+row, features n0 .. n0+BN-1.
      const int m = m0 + row;
      const bool rv = m < g.M;
      if constexpr (EPI == EPI_SWIGLU) {
        // BN = 256 columns = two [gate 64 | up 64] blocks -> 128 output features
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(g.out) + (size_t)m * g.ldo;
#pragma unroll 1
        for (int blk = 0; blk < BN / 128; ++blk) {
#pragma unroll 1
          for (int half = 0; half < 2; ++half) {
            uint32_t rg[32], ru[32];
            tmem_ld_32x32b_x32(trow + blk * 128 + half * 32, rg);
            tmem_ld_32x32b_x32(trow + blk * 128 + 64 + half * 32, ru);
            tmem_ld_wait();
            const int f0 = (n0 / 2) + blk * 64 + half * 32;
            if (rv && f0 < g.N / 2) {
              __align__(16) __nv_bfloat16 vals[32];
#pragma unroll
              for (int j = 0; j < 32; ++j)
                vals[j] = __float2bfloat16(silu_f(__uint_as_float(rg[j])) * __uint_as_float(ru[j]));
#pragma unroll
              for (int q = 0; q < 4; ++q)
                reinterpret_cast<uint4*>(o + f0)[q] = reinterpret_cast<const uint4*>(vals)[q];
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(trow + c * 32, r);
          tmem_ld_wait();
          const int nb = n0 + c * 32;
          if (!rv || nb >= g.N) continue;
          const bool full = nb + 32 <= g.N;
          if constexpr (EPI == EPI_BF16) {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(g.out) + (size_t)m * g.ldo + nb;
            if (full) {
              __align__(16) __nv_bfloat16 vals[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) vals[j] = __float2bfloat16(__uint_as_float(r[j]));
#pragma unroll
              for (int q = 0; q < 4; ++q) reinterpret_cast<uint4*>(o)[q] = reinterpret_cast<const uint4*>(vals)[q];
            } else {
              for (int j = 0; j < g.N - nb; ++j) o[j] = __float2bfloat16(__uint_as_float(r[j]));
            }
          } else {
            float* o = reinterpret_cast<float*>(g.out) + (size_t)m * g.ldo + nb;
            if constexpr (EPI == EPI_RS_F32) {
              const int owner = m_tile % g.rs.world;
              const size_t lrow = (size_t)(m_tile / g.rs.world) * BM + row;
              o = reinterpret_cast<float*>(g.rs.recv[owner]) + ((size_t)g.rs.rank * g.rs.rows_cap + lrow) * g.ldo + nb;
            }
            if (full) {
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                float4 v = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                       __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
                if constexpr (EPI == EPI_ADD_F32) {
                  const float4 p = reinterpret_cast<float4*>(o)[q];
                  v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
                }
                reinterpret_cast<float4*>(o)[q] = v;
              }
            } else {
              for (int j = 0; j < g.N - nb; ++j) {
                if constexpr (EPI == EPI_ADD_F32) o[j] += __uint_as_float(r[j]);
                else o[j] = __uint_as_float(r[j]);
              }
            }
          }
        }
      }
    }
  }

  if constexpr (!SWAP && EPI == EPI_RS_F32) {
    // every thread's stores of the tile are done: one system-scope release increment of the
    // owner's arrival counter (also after a failed wait, so the owner's wait ends; the error word
    // carries the failure)
    cta_sync();
    if (tid == 0) {
      __threadfence_system();
      atomicAdd_system(reinterpret_cast<unsigned long long*>(g.rs.count[m_tile % g.rs.world]), 1ull);
    }
  }

  // ---------------- teardown
  if (tid == 0) Q38_STAMP(6);
  tc_fence_before();
  cta_sync();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  if (tid == 0) Q38_STAMP(7);
}

template <int BN, int STAGES, int EPI, bool SWAP, bool MX = false>
void launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& g, dim3 grid, cudaStream_t st) {
  auto kern = gemm_tn_kernel<BN, STAGES, EPI, SWAP, MX>;
  constexpr int smem = std::conditional<MX, SmemMx, Smem<BN, STAGES>>::type::TOTAL;
  const cudaError_t attr = set_smem_once<gemm_tn_kernel<BN, STAGES, EPI, SWAP, MX>>(smem);
  TORCH_CHECK(attr == cudaSuccess, "cudaFuncSetAttribute failed");
  const unsigned cz = (SWAP && !MX && g.cluster_k && g.splits > 1) ? (unsigned)g.splits : 1u;
  TORCH_CHECK(launch_pdl_cluster(kern, grid, dim3(MX ? 256 : 128), (size_t)smem, st, dim3(1, 1, cz), ma, mb, g) ==
                  cudaSuccess,
              "GEMM launch failed");
}

constexpr int SKINNY_STAGES = 5;   // 5 x 20 KB ring: two CTAs per SM
constexpr int MAX_CLUSTER_SPLITS = 8;   // split-K CTAs of one tile: one portable cluster
constexpr int PREFILL_BN = 256;
constexpr int PREFILL_STAGES = 4;  // 4 x 48 KB ring

// Split-K count of the skinny GEMM for a weight shape (gemm.cu; shared by every entry point so
// they produce the same bits).
int pick_splits(int m_tiles, int kblocks, int sms);

// epilogue-dispatched launchers, one translation unit each
void launch_swap(int epi, const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& g, dim3 grid, cudaStream_t st);
// MX-weight swap GEMM (g.mxq / g.mxs set; mb: the activation map)
void launch_swap_mx(int epi, const CUtensorMap& mb, const GemmArgs& g, dim3 grid, cudaStream_t st);
void launch_prefill(int epi, const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& g, dim3 grid,
                    cudaStream_t st);

}  // namespace q38
