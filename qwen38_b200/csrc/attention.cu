// Attention kernels for the gated full-attention layers and the block drafter.
//
// attn_prep  : per (row, head): RMSNorm of q / k heads (weight = multiplier, 1+w for the target),
//              partial RoPE (half-split, first rd channels, optional YaRN scale), q to a staging
//              buffer, k / v rows written into the KV cache at each row's position (paged through
//              a block table, or contiguous).  (graft/attention/tp.py:547-641 attn_decode_prep +
//              paged_update_cache, :779-838 prefill fill.)
// attn_decode: split-K flash decode for <= 32 query rows (verify / decode / drafter block).  The key
//              axis is cut into fixed absolute groups of 128-key chunks (1, 4 or 8 chunks per
//              group, growing with key position), one CTA per (KV head, group) with an online
//              softmax over its 64-key tiles, so a row's result depends only on its own position,
//              never on how many rows ran with it.  GQA: all q heads of one KV head run in one CTA
//              against one staged K/V tile.  Causal (target) or full (drafter).
// attn_combine: merges the per-group (max, sum, o) partials in group order, applies
//              sigmoid(gate) (graft/attention/tp.py:121-237 gated output), writes bf16.
// attn_prefill: causal flash attention of a prefill chunk over the paged cache (K-ATTN-PREFILL;
//              the reference's chunked / paged SDPA, graft/attention/tp.py:476,645).  One CTA per
//              (16 query positions, KV head): warp w owns q head w of the GQA group, so each
//              64-key K/V tile is staged once (cp.async, double-buffered) for all its heads;
//              online softmax in registers, sigmoid(gate) epilogue, bf16 out.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "attn_groups.cuh"
#include "common.cuh"

namespace q38 {

struct PrepArgs {
  const __nv_bfloat16* proj;   // [T, width]
  long long proj_ld;
  int q_off, k_off, v_off;     // column offsets of q, k, v head blocks (q_off < 0: no q)
  int nq, nkv, D, rd;
  const float* qn;             // [D] multiplier
  const float* kn;
  const float* inv_freq;       // [rd/2]
  float rope_scale, eps;
  const int* pos;              // [T]
  __nv_bfloat16* q_out;        // [T, nq, D]
  __nv_bfloat16* kcache;       // paged [nb, bs, nkv, D] or contiguous [cap, nkv, D]
  __nv_bfloat16* vcache;
  const int* block_table;      // nullptr: contiguous
  int block_size;
  long long table_len;         // paged: block-table entries; contiguous: cache rows
  long long cache_blocks;      // paged: blocks in the cache
  int* err;                    // bad positions are recorded here and their rows skipped
};

__global__ void attn_prep_kernel(PrepArgs a) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int hh = blockIdx.y;        // [0, nq) q heads, [nq, nq+nkv) kv heads
  const int c = threadIdx.x;        // channel
  const int D = a.D;
  extern __shared__ float xs[];     // [D]
  __shared__ float red[32];
  const bool is_q = hh < a.nq;
  const int head = is_q ? hh : hh - a.nq;
  const int col = (is_q ? a.q_off : a.k_off) + head * D + c;
  const float x = __bfloat162float(a.proj[(size_t)t * a.proj_ld + col]);
  // RMSNorm over D
  float ss = warp_sum(x * x);
  const int w = c >> 5, l = c & 31;
  if (l == 0) red[w] = ss;
  __syncthreads();
  if (c == 0) {
    float s = 0.f;
    for (int i = 0; i < (D + 31) / 32; ++i) s += red[i];
    red[31] = rsqrtf(s / D + a.eps);
  }
  __syncthreads();
  const float y = x * red[31] * (is_q ? a.qn[c] : a.kn[c]);
  xs[c] = y;
  __syncthreads();
  float out = y;
  const int p = a.pos[t];
  if (c < a.rd) {
    const int half = a.rd >> 1;
    const int i = c < half ? c : c - half;
    const float ang = (float)p * a.inv_freq[i];
    float sn, cs;
    sincosf(ang, &sn, &cs);
    cs *= a.rope_scale;
    sn *= a.rope_scale;
    const float rot = c < half ? -xs[c + half] : xs[c - half];
    out = y * cs + rot * sn;
  }
  if (is_q) {
    a.q_out[((size_t)t * a.nq + head) * D + c] = __float2bfloat16(out);
  } else {
    // a position outside the cache (a corrupted position or block table) is recorded and its
    // row skipped instead of written out of bounds
    size_t base;
    if (a.block_table) {
      if (p < 0 || (long long)(p / a.block_size) >= a.table_len) {
        if (c == 0) record_error(a.err, kErrShape);
        return;
      }
      const int blk = a.block_table[p / a.block_size];
      if (blk < 0 || blk >= a.cache_blocks) {
        if (c == 0) record_error(a.err, kErrShape);
        return;
      }
      base = ((size_t)blk * a.block_size + (p % a.block_size)) * a.nkv + head;
    } else {
      if (p < 0 || p >= a.table_len) {
        if (c == 0) record_error(a.err, kErrShape);
        return;
      }
      base = (size_t)p * a.nkv + head;
    }
    a.kcache[base * D + c] = __float2bfloat16(out);
    const float v = __bfloat162float(a.proj[(size_t)t * a.proj_ld + a.v_off + head * D + c]);
    a.vcache[base * D + c] = __float2bfloat16(v);
  }
}

// ------------------------------------------------------------------------------- decode
constexpr int MAXW = 8;      // warps per CTA: one 16-row query tile each

struct DecodeArgs {
  const __nv_bfloat16* q;      // [T, nq, D]
  const __nv_bfloat16* kcache;
  const __nv_bfloat16* vcache;
  const int* block_table;      // nullptr: contiguous
  int block_size;
  const int* qpos;             // [T]
  int T, nq, nkv, D;
  float scale;
  int causal;
  float* part_o;               // [nkv, splits, nqv, D]
  float* part_ml;              // [nkv, splits, nqv, 2]
  int max_splits;
  int window;                  // > 0: row at position p sees keys k with p - k < window
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

constexpr int DK_T = 64;       // keys per staged tile inside a group

// One CTA per (KV head g, key group).  All query vectors of the GQA group (rep heads x T rows) run
// against 64-key K/V tiles staged once in shared memory (cp.async, double-buffered): warp w owns
// query rows 16w..16w+15 of the current row group of up to 16 x warps rows.  S = Q K^T and O = P V
// on tensor cores (m16n8k16, fp32 accumulate) with an online softmax over the group's tiles in key
// order; the (max, sum, unnormalised O) partial of the group is merged across groups in group
// order by the combine kernel.  A tile beyond a row's own position changes nothing: its
// probabilities are exact zeros and its rescale factor is exactly 1, so row t gives the same bits
// in a 16-row verify as in a 1-row decode.  WIN adds a sliding-window lower bound per row (the
// windowed block drafter): keys below it are masked the same exact-zero way.
template <int D, bool WIN>
__global__ void __launch_bounds__(256, 1)
attn_decode_kernel(DecodeArgs a) {
  constexpr int DP = D + 8;                 // padded row: conflict-free ldmatrix
  constexpr int NT_K = DK_T / 8;            // key n-tiles per tile
  constexpr int NT_D = D / 8;               // output n-tiles
  pdl_wait();
  pdl_trigger();
  const int g = blockIdx.x, grp = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int rep = a.nq / a.nkv;
  const int nqv = rep * a.T;
  const int n_keys = a.qpos[a.T - 1] + 1;
  const int c0 = group_first_chunk(grp);
  const int k_begin = c0 * CH;
  if (k_begin >= n_keys) return;
  const int k_end = min(n_keys, (c0 + group_chunks(grp)) * CH);
  const int ntiles = (k_end - k_begin + DK_T - 1) / DK_T;

  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(smem);                 // [nwarps*16][DP]
  __nv_bfloat16* KV = Qs + nwarps * 16 * DP;                                  // [2 bufs][K, V][DK_T][DP]
  auto Ks = [&](int b) { return KV + (size_t)(2 * b) * DK_T * DP; };
  auto Vs = [&](int b) { return KV + (size_t)(2 * b + 1) * DK_T * DP; };
  __shared__ long long kv_row[2][DK_T];

  auto load_tile = [&](int kt, int b) {
    const int t0 = k_begin + kt * DK_T;
    // one block-table lookup per key, not per 16-byte copy
    for (int j = threadIdx.x; j < DK_T; j += blockDim.x) {
      const int kp = t0 + j;
      long long base = -1;
      if (kp < k_end) {
        if (a.block_table) {
          const int blk = a.block_table[kp / a.block_size];
          base = (((long long)blk * a.block_size + (kp % a.block_size)) * a.nkv + g) * D;
        } else {
          base = ((long long)kp * a.nkv + g) * D;
        }
      }
      kv_row[b][j] = base;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < DK_T * (D / 8); idx += blockDim.x) {
      const int j = idx / (D / 8), ch = idx % (D / 8);
      uint4* dk = reinterpret_cast<uint4*>(Ks(b) + j * DP) + ch;
      uint4* dv = reinterpret_cast<uint4*>(Vs(b) + j * DP) + ch;
      const long long base = kv_row[b][j];
      if (base >= 0) {
        cp_async16(dk, reinterpret_cast<const uint4*>(a.kcache + base) + ch);
        cp_async16(dv, reinterpret_cast<const uint4*>(a.vcache + base) + ch);
      } else {
        *dk = make_uint4(0, 0, 0, 0);
        *dv = make_uint4(0, 0, 0, 0);
      }
    }
  };

  for (int qb = 0; qb < nqv; qb += nwarps * 16) {
    __syncthreads();                           // previous row group done with Q and the tiles
    // ---- this row group's query vectors (zeros for padding rows)
    for (int idx = threadIdx.x; idx < nwarps * 16 * (D / 8); idx += blockDim.x) {
      const int qi = idx / (D / 8), ch = idx % (D / 8);
      const int gq = qb + qi;
      uint4* dst = reinterpret_cast<uint4*>(Qs + qi * DP) + ch;
      if (gq < nqv) {
        const int hq = g * rep + gq / a.T, t = gq % a.T;
        cp_async16(dst, reinterpret_cast<const uint4*>(a.q + ((size_t)t * a.nq + hq) * D) + ch);
      } else {
        *dst = make_uint4(0, 0, 0, 0);
      }
    }
    load_tile(0, 0);
    cp_async_commit();
    if (ntiles > 1) {
      load_tile(1, 1);
      cp_async_commit();
    }
    const int row0 = qb + warp * 16;
    const bool active = row0 < nqv;
    const int r_lo = row0 + (lane >> 2), r_hi = r_lo + 8;
    const int p_lo = (active && r_lo < nqv) ? (a.causal ? a.qpos[r_lo % a.T] : n_keys - 1) : -1;
    const int p_hi = (active && r_hi < nqv) ? (a.causal ? a.qpos[r_hi % a.T] : n_keys - 1) : -1;
    int w_lo = 0, w_hi = 0;                    // lowest visible key of each row (WIN only)
    if constexpr (WIN) {
      w_lo = (active && r_lo < nqv) ? a.qpos[r_lo % a.T] - a.window + 1 : 0;
      w_hi = (active && r_hi < nqv) ? a.qpos[r_hi % a.T] - a.window + 1 : 0;
    }
    float O[NT_D][4];
#pragma unroll
    for (int n = 0; n < NT_D; ++n) O[n][0] = O[n][1] = O[n][2] = O[n][3] = 0.f;
    float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
    const uint32_t qbase = smem_u32(Qs + (warp * 16) * DP);

    for (int kt = 0; kt < ntiles; ++kt) {
      const int b = kt & 1;
      if (kt + 1 < ntiles) cp_async_wait<1>();
      else cp_async_wait<0>();
      __syncthreads();
      if (active) {
        const int t0 = k_begin + kt * DK_T;
        float S[NT_K][4];
#pragma unroll
        for (int n = 0; n < NT_K; ++n) S[n][0] = S[n][1] = S[n][2] = S[n][3] = 0.f;
        const uint32_t kbase = smem_u32(Ks(b));
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4(qbase + (uint32_t)(((lane & 15) * DP + kk * 16 + (lane >> 4) * 8) * 2), a0, a1, a2, a3);
#pragma unroll
          for (int n = 0; n < NT_K; ++n) {
            uint32_t b0, b1;
            ldsm_x2(kbase + (uint32_t)(((n * 8 + (lane & 7)) * DP + kk * 16 + ((lane >> 3) & 1) * 8) * 2), b0, b1);
            mma_bf16_16816(S[n], a0, a1, a2, a3, b0, b1);
          }
        }
        float tm_lo = -INFINITY, tm_hi = -INFINITY;
#pragma unroll
        for (int n = 0; n < NT_K; ++n) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int kp = t0 + n * 8 + (lane & 3) * 2 + e;
            bool ok_lo = kp < k_end && kp <= p_lo, ok_hi = kp < k_end && kp <= p_hi;
            if constexpr (WIN) {
              ok_lo = ok_lo && kp >= w_lo;
              ok_hi = ok_hi && kp >= w_hi;
            }
            S[n][e] = ok_lo ? S[n][e] * a.scale : -INFINITY;
            S[n][2 + e] = ok_hi ? S[n][2 + e] * a.scale : -INFINITY;
            tm_lo = fmaxf(tm_lo, S[n][e]);
            tm_hi = fmaxf(tm_hi, S[n][2 + e]);
          }
        }
        tm_lo = fmaxf(tm_lo, __shfl_xor_sync(0xffffffffu, tm_lo, 1));
        tm_lo = fmaxf(tm_lo, __shfl_xor_sync(0xffffffffu, tm_lo, 2));
        tm_hi = fmaxf(tm_hi, __shfl_xor_sync(0xffffffffu, tm_hi, 1));
        tm_hi = fmaxf(tm_hi, __shfl_xor_sync(0xffffffffu, tm_hi, 2));
        const float mn_lo = fmaxf(m_lo, tm_lo), mn_hi = fmaxf(m_hi, tm_hi);
        const float mz_lo = mn_lo == -INFINITY ? 0.f : mn_lo;
        const float mz_hi = mn_hi == -INFINITY ? 0.f : mn_hi;
        const float c_lo = __expf(m_lo - mz_lo), c_hi = __expf(m_hi - mz_hi);   // 0 before any key, 1 if unchanged
        m_lo = mn_lo;
        m_hi = mn_hi;
        l_lo *= c_lo;
        l_hi *= c_hi;
#pragma unroll
        for (int n = 0; n < NT_D; ++n) {
          O[n][0] *= c_lo; O[n][1] *= c_lo;
          O[n][2] *= c_hi; O[n][3] *= c_hi;
        }
#pragma unroll
        for (int n = 0; n < NT_K; ++n) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            S[n][e] = __expf(S[n][e] - mz_lo);
            S[n][2 + e] = __expf(S[n][2 + e] - mz_hi);
            l_lo += S[n][e];
            l_hi += S[n][2 + e];
          }
        }
        const uint32_t vbase = smem_u32(Vs(b));
#pragma unroll
        for (int j = 0; j < DK_T / 16; ++j) {
          const uint32_t a0 = pack_bf16(S[2 * j][0], S[2 * j][1]);
          const uint32_t a1 = pack_bf16(S[2 * j][2], S[2 * j][3]);
          const uint32_t a2 = pack_bf16(S[2 * j + 1][0], S[2 * j + 1][1]);
          const uint32_t a3 = pack_bf16(S[2 * j + 1][2], S[2 * j + 1][3]);
#pragma unroll
          for (int n = 0; n < NT_D; ++n) {
            uint32_t b0, b1;
            ldsm_x2_t(vbase + (uint32_t)(((j * 16 + (lane & 15)) * DP + n * 8) * 2), b0, b1);
            mma_bf16_16816(O[n], a0, a1, a2, a3, b0, b1);
          }
        }
      }
      __syncthreads();                         // every warp is done with buffer b
      if (kt + 2 < ntiles) {
        load_tile(kt + 2, b);
        cp_async_commit();
      }
    }
    if (!active) continue;
    // ---- the group's partial: row sums over the quad, then (m, l) and unnormalised O
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
    const size_t plo = ((size_t)g * a.max_splits + grp) * nqv + r_lo;
    const size_t phi = ((size_t)g * a.max_splits + grp) * nqv + r_hi;
#pragma unroll
    for (int n = 0; n < NT_D; ++n) {
      const int d = n * 8 + (lane & 3) * 2;
      if (r_lo < nqv) *reinterpret_cast<float2*>(a.part_o + plo * D + d) = make_float2(O[n][0], O[n][1]);
      if (r_hi < nqv) *reinterpret_cast<float2*>(a.part_o + phi * D + d) = make_float2(O[n][2], O[n][3]);
    }
    if ((lane & 3) == 0) {
      if (r_lo < nqv) { a.part_ml[plo * 2] = m_lo; a.part_ml[plo * 2 + 1] = l_lo; }
      if (r_hi < nqv) { a.part_ml[phi * 2] = m_hi; a.part_ml[phi * 2 + 1] = l_hi; }
    }
  }
}

__global__ void attn_combine_kernel(DecodeArgs a, const __nv_bfloat16* gate, long long gate_ld, int gate_off,
                                    __nv_bfloat16* out, long long out_ld) {
  pdl_wait();
  pdl_trigger();
  const int hq = blockIdx.x, t = blockIdx.y;
  const int D = a.D;
  const int rep = a.nq / a.nkv;
  const int g = hq / rep;
  const int nqv = rep * a.T;
  const int qv = (hq % rep) * a.T + t;
  const int n_keys = a.causal ? a.qpos[t] + 1 : a.qpos[a.T - 1] + 1;
  const int ns = groups_for((n_keys + CH - 1) / CH);        // key groups this row sees
  // 1. every split's (max, sum) into shared memory in parallel, then the global max and the
  //    per-split weights exp(m_s - M) once (fixed split order everywhere)
  extern __shared__ float cm[];                 // [2 * ns]: weight, weighted sum
  __shared__ float red[32];
  __shared__ float Ms;
  float mloc = -INFINITY;
  for (int s = threadIdx.x; s < ns; s += blockDim.x) {
    const size_t pidx = ((size_t)g * a.max_splits + s) * nqv + qv;
    const float ms = a.part_ml[pidx * 2];
    cm[2 * s] = ms;
    cm[2 * s + 1] = a.part_ml[pidx * 2 + 1];
    mloc = fmaxf(mloc, ms);
  }
  mloc = warp_max(mloc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mloc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) M = fmaxf(M, red[w]);
    Ms = M;
  }
  __syncthreads();
  const float M = Ms;
  for (int s = threadIdx.x; s < ns; s += blockDim.x) {
    const float ms = cm[2 * s];
    const float wgt = ms == -INFINITY ? 0.f : __expf(ms - M);
    cm[2 * s] = wgt;
    cm[2 * s + 1] *= wgt;
  }
  __syncthreads();
  float L = 0.f;
  for (int s = 0; s < ns; ++s) L += cm[2 * s + 1];
  // 2. weighted sum of the partial outputs, 32 splits' loads in flight at a time (one round trip
  //    up to 4,096 keys), summed in split order
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float acc = 0.f;
    for (int s0 = 0; s0 < ns; s0 += 32) {
      float v[32];
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const int s = s0 + u;
        v[u] = s < ns ? __ldcg(a.part_o + (((size_t)g * a.max_splits + s) * nqv + qv) * D + c) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 32; ++u)
        if (s0 + u < ns) acc += cm[2 * (s0 + u)] * v[u];
    }
    float y = acc / L;
    if (gate) {
      const float gv = __bfloat162float(gate[(size_t)t * gate_ld + gate_off + (size_t)hq * D + c]);
      y *= 1.f / (1.f + __expf(-gv));
    }
    out[(size_t)t * out_ld + (size_t)hq * D + c] = __float2bfloat16(y);
  }
}

struct PrefillArgs {
  const __nv_bfloat16* q;      // [T, nq, D]
  const __nv_bfloat16* kcache;
  const __nv_bfloat16* vcache;
  const int* block_table;      // nullptr: contiguous
  int block_size;
  const int* qpos;             // [T] absolute positions, increasing
  int T, nq, nkv;
  float scale;
  const __nv_bfloat16* gate;   // [T, gate_ld] (+ head * D), nullptr: no gate
  long long gate_ld;
  __nv_bfloat16* out;          // [T, out_ld]
  long long out_ld;
};

constexpr int PF_QT = 16;      // query positions per CTA
constexpr int PF_KT = 64;      // keys per staged tile

template <int D>
__global__ void __launch_bounds__(256, 1)
attn_prefill_kernel(PrefillArgs a) {
  constexpr int DP = D + 8;
  constexpr int NT_K = PF_KT / 8;
  constexpr int NT_D = D / 8;
  pdl_wait();
  pdl_trigger();
  const int qt = gridDim.x - 1 - blockIdx.x;     // longest (latest) query tiles first
  const int g = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rep = a.nq / a.nkv;                  // == warps per CTA
  const int t0 = qt * PF_QT;
  const int nt = min(PF_QT, a.T - t0);
  const int n_keys = a.qpos[t0 + nt - 1] + 1;
  const int ntiles = (n_keys + PF_KT - 1) / PF_KT;

  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(smem);          // [rep*16][DP]
  __nv_bfloat16* KV = Qs + rep * PF_QT * DP;                            // [2 bufs][K, V][PF_KT][DP]
  auto Ks = [&](int b) { return KV + (size_t)(2 * b) * PF_KT * DP; };
  auto Vs = [&](int b) { return KV + (size_t)(2 * b + 1) * PF_KT * DP; };

  auto kv_base = [&](int kp) -> size_t {
    if (a.block_table) {
      const int blk = a.block_table[kp / a.block_size];
      return ((size_t)blk * a.block_size + (kp % a.block_size)) * a.nkv + g;
    }
    return (size_t)kp * a.nkv + g;
  };
  auto load_tile = [&](int kt, int b) {
    const int k0 = kt * PF_KT;
    for (int idx = threadIdx.x; idx < PF_KT * (D / 8); idx += blockDim.x) {
      const int j = idx / (D / 8), ch = idx % (D / 8);
      const int kp = k0 + j;
      uint4* dk = reinterpret_cast<uint4*>(Ks(b) + j * DP) + ch;
      uint4* dv = reinterpret_cast<uint4*>(Vs(b) + j * DP) + ch;
      if (kp < n_keys) {
        const size_t base = kv_base(kp) * D;
        cp_async16(dk, reinterpret_cast<const uint4*>(a.kcache + base) + ch);
        cp_async16(dv, reinterpret_cast<const uint4*>(a.vcache + base) + ch);
      } else {
        *dk = make_uint4(0, 0, 0, 0);
        *dv = make_uint4(0, 0, 0, 0);
      }
    }
  };
  // Q rows: warp w / row i <- q[t0 + i, g*rep + w, :]
  for (int idx = threadIdx.x; idx < rep * PF_QT * (D / 8); idx += blockDim.x) {
    const int r = idx / (D / 8), ch = idx % (D / 8);
    const int w = r / PF_QT, i = r % PF_QT;
    uint4* dst = reinterpret_cast<uint4*>(Qs + r * DP) + ch;
    if (i < nt) cp_async16(dst, reinterpret_cast<const uint4*>(a.q + ((size_t)(t0 + i) * a.nq + g * rep + w) * D) + ch);
    else *dst = make_uint4(0, 0, 0, 0);
  }
  load_tile(0, 0);
  cp_async_commit();
  if (ntiles > 1) {
    load_tile(1, 1);
    cp_async_commit();
  }

  // rows of this thread inside the warp's 16: lane/4 and lane/4 + 8
  const int i_lo = lane >> 2, i_hi = i_lo + 8;
  const int p_lo = i_lo < nt ? a.qpos[t0 + i_lo] : -1;
  const int p_hi = i_hi < nt ? a.qpos[t0 + i_hi] : -1;
  float O[NT_D][4];
#pragma unroll
  for (int n = 0; n < NT_D; ++n) O[n][0] = O[n][1] = O[n][2] = O[n][3] = 0.f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
  const uint32_t qbase = smem_u32(Qs + (warp * PF_QT) * DP);

  for (int kt = 0; kt < ntiles; ++kt) {
    const int b = kt & 1;
    if (kt + 1 < ntiles) cp_async_wait<1>();
    else cp_async_wait<0>();
    __syncthreads();
    const int k0 = kt * PF_KT;
    {
      float S[NT_K][4];
#pragma unroll
      for (int n = 0; n < NT_K; ++n) S[n][0] = S[n][1] = S[n][2] = S[n][3] = 0.f;
      const uint32_t kbase = smem_u32(Ks(b));
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(qbase + (uint32_t)(((lane & 15) * DP + kk * 16 + (lane >> 4) * 8) * 2), a0, a1, a2, a3);
#pragma unroll
        for (int n = 0; n < NT_K; ++n) {
          uint32_t b0, b1;
          ldsm_x2(kbase + (uint32_t)(((n * 8 + (lane & 7)) * DP + kk * 16 + ((lane >> 3) & 1) * 8) * 2), b0, b1);
          mma_bf16_16816(S[n], a0, a1, a2, a3, b0, b1);
        }
      }
      // causal mask + online softmax
      float tm_lo = -INFINITY, tm_hi = -INFINITY;
#pragma unroll
      for (int n = 0; n < NT_K; ++n) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int kp = k0 + n * 8 + (lane & 3) * 2 + e;
          S[n][e] = kp <= p_lo ? S[n][e] * a.scale : -INFINITY;
          S[n][2 + e] = kp <= p_hi ? S[n][2 + e] * a.scale : -INFINITY;
          tm_lo = fmaxf(tm_lo, S[n][e]);
          tm_hi = fmaxf(tm_hi, S[n][2 + e]);
        }
      }
      tm_lo = fmaxf(tm_lo, __shfl_xor_sync(0xffffffffu, tm_lo, 1));
      tm_lo = fmaxf(tm_lo, __shfl_xor_sync(0xffffffffu, tm_lo, 2));
      tm_hi = fmaxf(tm_hi, __shfl_xor_sync(0xffffffffu, tm_hi, 1));
      tm_hi = fmaxf(tm_hi, __shfl_xor_sync(0xffffffffu, tm_hi, 2));
      const float mn_lo = fmaxf(m_lo, tm_lo), mn_hi = fmaxf(m_hi, tm_hi);
      const float mz_lo = mn_lo == -INFINITY ? 0.f : mn_lo;
      const float mz_hi = mn_hi == -INFINITY ? 0.f : mn_hi;
      const float c_lo = __expf(m_lo - mz_lo), c_hi = __expf(m_hi - mz_hi);   // exp(-inf) = 0 on the first tile
      m_lo = mn_lo;
      m_hi = mn_hi;
      l_lo *= c_lo;
      l_hi *= c_hi;
#pragma unroll
      for (int n = 0; n < NT_D; ++n) {
        O[n][0] *= c_lo; O[n][1] *= c_lo;
        O[n][2] *= c_hi; O[n][3] *= c_hi;
      }
#pragma unroll
      for (int n = 0; n < NT_K; ++n) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          S[n][e] = __expf(S[n][e] - mz_lo);
          S[n][2 + e] = __expf(S[n][2 + e] - mz_hi);
          l_lo += S[n][e];
          l_hi += S[n][2 + e];
        }
      }
      const uint32_t vbase = smem_u32(Vs(b));
#pragma unroll
      for (int j = 0; j < PF_KT / 16; ++j) {
        const uint32_t a0 = pack_bf16(S[2 * j][0], S[2 * j][1]);
        const uint32_t a1 = pack_bf16(S[2 * j][2], S[2 * j][3]);
        const uint32_t a2 = pack_bf16(S[2 * j + 1][0], S[2 * j + 1][1]);
        const uint32_t a3 = pack_bf16(S[2 * j + 1][2], S[2 * j + 1][3]);
#pragma unroll
        for (int n = 0; n < NT_D; ++n) {
          uint32_t b0, b1;
          ldsm_x2_t(vbase + (uint32_t)(((j * 16 + (lane & 15)) * DP + n * 8) * 2), b0, b1);
          mma_bf16_16816(O[n], a0, a1, a2, a3, b0, b1);
        }
      }
    }
    __syncthreads();                       // every warp is done with buffer b
    if (kt + 2 < ntiles) {
      load_tile(kt + 2, b);
      cp_async_commit();
    }
  }
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
  const float inv_lo = l_lo > 0.f ? 1.f / l_lo : 0.f, inv_hi = l_hi > 0.f ? 1.f / l_hi : 0.f;
  const int hq = g * rep + warp;
#pragma unroll
  for (int n = 0; n < NT_D; ++n) {
    const int d = n * 8 + (lane & 3) * 2;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int i = half ? i_hi : i_lo;
      if (i >= nt) continue;
      const float inv = half ? inv_hi : inv_lo;
      float y0 = O[n][2 * half] * inv, y1 = O[n][2 * half + 1] * inv;
      const size_t t = (size_t)(t0 + i);
      if (a.gate) {
        const __nv_bfloat162 gv = *reinterpret_cast<const __nv_bfloat162*>(a.gate + t * a.gate_ld + (size_t)hq * D + d);
        y0 *= 1.f / (1.f + __expf(-__bfloat162float(gv.x)));
        y1 *= 1.f / (1.f + __expf(-__bfloat162float(gv.y)));
      }
      *reinterpret_cast<__nv_bfloat162*>(a.out + t * a.out_ld + (size_t)hq * D + d) = __floats2bfloat162_rn(y0, y1);
    }
  }
}
}  // namespace q38

// ----------------------------------------------------------------------------- bindings
void q38_attn_prep(torch::Tensor proj, int64_t q_off, int64_t k_off, int64_t v_off, int64_t nq, int64_t nkv,
                   int64_t D, int64_t rd, torch::Tensor qn, torch::Tensor kn, torch::Tensor inv_freq,
                   double rope_scale, double eps, torch::Tensor pos, c10::optional<torch::Tensor> q_out,
                   torch::Tensor kcache, torch::Tensor vcache, c10::optional<torch::Tensor> block_table,
                   int64_t block_size, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(proj.device());
  TORCH_CHECK(proj.scalar_type() == at::kBFloat16 && kcache.scalar_type() == at::kBFloat16, "bf16 required");
  TORCH_CHECK(pos.scalar_type() == at::kInt, "int32 positions");
  TORCH_CHECK(D <= 1024 && D % 32 == 0, "head dim must be a multiple of 32");
  q38::PrepArgs a{};
  a.proj = reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr());
  a.proj_ld = proj.stride(0);
  a.q_off = (int)q_off; a.k_off = (int)k_off; a.v_off = (int)v_off;
  a.nq = (int)nq; a.nkv = (int)nkv; a.D = (int)D; a.rd = (int)rd;
  a.qn = nq > 0 ? qn.data_ptr<float>() : nullptr;
  a.kn = kn.data_ptr<float>();
  a.inv_freq = inv_freq.data_ptr<float>();
  a.rope_scale = (float)rope_scale;
  a.eps = (float)eps;
  a.pos = pos.data_ptr<int>();
  a.q_out = q_out ? reinterpret_cast<__nv_bfloat16*>(q_out->data_ptr()) : nullptr;
  a.kcache = reinterpret_cast<__nv_bfloat16*>(kcache.data_ptr());
  a.vcache = reinterpret_cast<__nv_bfloat16*>(vcache.data_ptr());
  a.block_table = block_table ? block_table->data_ptr<int>() : nullptr;
  a.block_size = (int)block_size;
  if (block_table) {
    TORCH_CHECK(kcache.dim() == 4 && block_size == kcache.size(1), "paged cache [blocks, block_size, kv, D]");
    a.table_len = block_table->numel();
    a.cache_blocks = kcache.size(0);
  } else {
    TORCH_CHECK(kcache.dim() == 3, "contiguous cache [rows, kv, D]");
    a.table_len = kcache.size(0);
    a.cache_blocks = 0;
  }
  a.err = err.data_ptr<int>();
  const int T = (int)proj.size(0);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  q38::launch_pdl(q38::attn_prep_kernel, dim3(T, (unsigned)(nq + nkv)), dim3((unsigned)D), D * sizeof(float), st, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

bool q38_attn_decode_tc(const torch::Tensor& q, const torch::Tensor& kcache, const torch::Tensor& vcache,
                        const int* block_table, int block_size, const int* qpos, int T, int nq, int nkv, float scale,
                        int causal, float* part_o, float* part_ml, int max_splits, int* err, cudaStream_t st);

void q38_attn_decode_window(torch::Tensor q, torch::Tensor kcache, torch::Tensor vcache,
                            c10::optional<torch::Tensor> block_table, int64_t block_size, torch::Tensor qpos,
                            double scale, int64_t causal, c10::optional<torch::Tensor> gate, int64_t gate_off,
                            torch::Tensor out, torch::Tensor part_o, torch::Tensor part_ml, int64_t max_keys,
                            int64_t window, c10::optional<torch::Tensor> err) {
  c10::cuda::CUDAGuard guard(q.device());
  const int T = (int)q.size(0), nq = (int)q.size(1), D = (int)q.size(2);
  const int nkv = (int)kcache.size(-2);
  TORCH_CHECK(T <= 32, "decode attention serves <= 32 rows");
  TORCH_CHECK(nq % nkv == 0, "GQA group mismatch");
  q38::DecodeArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.kcache = reinterpret_cast<const __nv_bfloat16*>(kcache.data_ptr());
  a.vcache = reinterpret_cast<const __nv_bfloat16*>(vcache.data_ptr());
  a.block_table = block_table ? block_table->data_ptr<int>() : nullptr;
  a.block_size = (int)block_size;
  a.qpos = qpos.data_ptr<int>();
  a.T = T; a.nq = nq; a.nkv = nkv; a.D = D;
  a.scale = (float)scale;
  a.causal = (int)causal;
  a.max_splits = (int)((max_keys + q38::CH - 1) / q38::CH);
  TORCH_CHECK(window >= 0 && window <= (int64_t)1 << 30, "window out of range");
  a.window = (int)window;
  const int nqv = nq / nkv * T;
  TORCH_CHECK(part_o.numel() >= (int64_t)nkv * a.max_splits * nqv * D, "attention partial buffer too small");
  TORCH_CHECK(part_ml.numel() >= (int64_t)nkv * a.max_splits * nqv * 2, "attention partial buffer too small");
  a.part_o = part_o.data_ptr<float>();
  a.part_ml = part_ml.data_ptr<float>();
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int warps = std::max(4, std::min(q38::MAXW, (nqv + 15) / 16));   // >= 4 warps to stage K/V
  const size_t smem = (size_t)(4 * q38::DK_T + warps * 16) * (D + 8) * 2;
  dim3 grid(nkv, q38::groups_for(a.max_splits));
  // head dim 256 without a window: the tcgen05 kernel (attention_tc.cu); otherwise mma.sync
  const bool tc = window == 0 && q38_attn_decode_tc(q, kcache, vcache, a.block_table, a.block_size, a.qpos, T, nq,
                                                    nkv, a.scale, a.causal, a.part_o, a.part_ml, a.max_splits,
                                                    err ? err->data_ptr<int>() : nullptr, st);
#define Q38_DEC(DD)                                                                                         \
  {                                                                                                         \
    auto k = a.window > 0 ? q38::attn_decode_kernel<DD, true> : q38::attn_decode_kernel<DD, false>;         \
    TORCH_CHECK((a.window > 0 ? q38::set_smem_once<q38::attn_decode_kernel<DD, true>>((int)smem)             \
                              : q38::set_smem_once<q38::attn_decode_kernel<DD, false>>((int)smem)) == cudaSuccess, \
                "cudaFuncSetAttribute failed");                                                             \
    q38::launch_pdl(k, grid, dim3(warps * 32), smem, st, a);                                               \
  }
  if (tc) {
  } else if (D == 256) Q38_DEC(256)
  else if (D == 128) Q38_DEC(128)
  else if (D == 64) Q38_DEC(64)
  else TORCH_CHECK(false, "head dim 64/128/256 supported");
#undef Q38_DEC
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const __nv_bfloat16* gp = gate ? reinterpret_cast<const __nv_bfloat16*>(gate->data_ptr()) : nullptr;
  q38::launch_pdl(q38::attn_combine_kernel, dim3(nq, T), dim3(std::min(D, 256)),
                  (size_t)2 * a.max_splits * sizeof(float), st, a, gp,
                  (long long)(gate ? gate->stride(0) : 0), (int)gate_off,
                  reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), (long long)out.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void q38_attn_decode(torch::Tensor q, torch::Tensor kcache, torch::Tensor vcache,
                     c10::optional<torch::Tensor> block_table, int64_t block_size, torch::Tensor qpos, double scale,
                     int64_t causal, c10::optional<torch::Tensor> gate, int64_t gate_off, torch::Tensor out,
                     torch::Tensor part_o, torch::Tensor part_ml, int64_t max_keys, c10::optional<torch::Tensor> err) {
  q38_attn_decode_window(q, kcache, vcache, block_table, block_size, qpos, scale, causal, gate, gate_off, out, part_o,
                         part_ml, max_keys, 0, err);
}

void q38_attn_prefill(torch::Tensor q, torch::Tensor kcache, torch::Tensor vcache,
                      c10::optional<torch::Tensor> block_table, int64_t block_size, torch::Tensor qpos, double scale,
                      c10::optional<torch::Tensor> gate, torch::Tensor out) {
  c10::cuda::CUDAGuard guard(q.device());
  const int T = (int)q.size(0), nq = (int)q.size(1), D = (int)q.size(2);
  const int nkv = (int)kcache.size(-2);
  TORCH_CHECK(q.is_contiguous() && q.scalar_type() == at::kBFloat16, "contiguous bf16 q [T, nq, D]");
  TORCH_CHECK(nq % nkv == 0 && nq / nkv >= 1 && nq / nkv <= 8, "GQA group of 1..8 heads");
  TORCH_CHECK(qpos.scalar_type() == at::kInt && qpos.numel() == T, "int32 positions [T]");
  TORCH_CHECK(out.stride(1) == 1 && out.size(0) == T && out.size(1) >= (int64_t)nq * D, "out [T, >= nq*D]");
  TORCH_CHECK(!gate || (gate->stride(1) == 1 && gate->stride(0) % 2 == 0), "row-contiguous gate");
  q38::PrefillArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.kcache = reinterpret_cast<const __nv_bfloat16*>(kcache.data_ptr());
  a.vcache = reinterpret_cast<const __nv_bfloat16*>(vcache.data_ptr());
  a.block_table = block_table ? block_table->data_ptr<int>() : nullptr;
  a.block_size = (int)block_size;
  a.qpos = qpos.data_ptr<int>();
  a.T = T; a.nq = nq; a.nkv = nkv;
  a.scale = (float)scale;
  a.gate = gate ? reinterpret_cast<const __nv_bfloat16*>(gate->data_ptr()) : nullptr;
  a.gate_ld = gate ? gate->stride(0) : 0;
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.out_ld = out.stride(0);
  const int rep = nq / nkv;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  dim3 grid((unsigned)((T + q38::PF_QT - 1) / q38::PF_QT), (unsigned)nkv);
#define Q38_PF(DD)                                                                                  \
  {                                                                                                 \
    const size_t smem = (size_t)(rep * q38::PF_QT + 4 * q38::PF_KT) * (DD + 8) * 2;                 \
    auto k = q38::attn_prefill_kernel<DD>;                                                          \
    TORCH_CHECK(q38::set_smem_once<q38::attn_prefill_kernel<DD>>((int)smem) == cudaSuccess,          \
                "cudaFuncSetAttribute failed");                                                     \
    TORCH_CHECK(q38::launch_pdl(k, grid, dim3(rep * 32), smem, st, a) == cudaSuccess, "prefill attention launch"); \
  }
  if (D == 256) Q38_PF(256)
  else if (D == 128) Q38_PF(128)
  else if (D == 64) Q38_PF(64)
  else TORCH_CHECK(false, "head dim 64/128/256 supported");
#undef Q38_PF
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Host view of the decode attention's key-group partition (for tests and planners): one
// (first chunk, chunk count) pair per group covering `nchunks` 128-key chunks.
std::vector<std::pair<int64_t, int64_t>> q38_attn_key_groups(int64_t nchunks) {
  std::vector<std::pair<int64_t, int64_t>> out;
  const int n = q38::groups_for((int)nchunks);
  for (int g = 0; g < n; ++g) {
    const int c0 = q38::group_first_chunk(g);
    const int cnt = std::min(q38::group_chunks(g), (int)nchunks - c0);
    out.emplace_back(c0, cnt);
  }
  return out;
}
