// Attention kernels for the gated full-attention layers and the block drafter.
//
// attn_prep  : per (row, head): RMSNorm of q / k heads (weight = multiplier, 1+w for the target),
//              partial RoPE (half-split, first rd channels, optional YaRN scale), q to a staging
//              buffer, k / v rows written into the KV cache at each row's position (paged through
//              a block table, or contiguous).  (graft/attention/tp.py:547-641 attn_decode_prep +
//              paged_update_cache, :779-838 prefill fill.)
// attn_decode: split-K flash decode for <= 32 query rows (verify / decode / drafter block).  Key
//              chunks are fixed absolute ranges of CH keys, so a row's result depends only on its
//              own position, never on how many rows ran with it.  GQA: all q heads of one KV head
//              run in one CTA against one staged K/V tile.  Causal (target) or full (drafter).
// attn_combine: merges the per-chunk (max, sum, o) partials in chunk order, applies
//              sigmoid(gate) (graft/attention/tp.py:121-237 gated output), writes bf16.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

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
};

__global__ void attn_prep_kernel(PrepArgs a) {
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
    size_t base;
    if (a.block_table) {
      const int blk = a.block_table[p / a.block_size];
      base = ((size_t)blk * a.block_size + (p % a.block_size)) * a.nkv + head;
    } else {
      base = (size_t)p * a.nkv + head;
    }
    a.kcache[base * D + c] = __float2bfloat16(out);
    const float v = __bfloat162float(a.proj[(size_t)t * a.proj_ld + a.v_off + head * D + c]);
    a.vcache[base * D + c] = __float2bfloat16(v);
  }
}

// ------------------------------------------------------------------------------- decode
constexpr int CH = 256;      // keys per split
constexpr int SUBK = 32;     // keys per staged sub-tile
constexpr int MAXQ = 96;     // query vectors per pass (8 warps x 12)

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
  float* part_o;               // [nkv, splits, nq/nkv*T, D]
  float* part_ml;              // [nkv, splits, nq/nkv*T, 2]
  int max_splits;
};

template <int D, int QPW>
__global__ void __launch_bounds__(256)
attn_decode_kernel(DecodeArgs a) {
  constexpr int DP = D + 8;                 // padded row (bf16) -> conflict-free 16-B reads
  constexpr int DPL = D / 32;               // dims per lane in PV
  const int g = blockIdx.x, s = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rep = a.nq / a.nkv;
  const int nqv = rep * a.T;                // query vectors of this KV head
  const int n_keys = a.qpos[a.T - 1] + 1;   // rows are consecutive positions; last sees most
  const int k0 = s * CH;
  if (k0 >= n_keys) return;
  const int k1 = min(n_keys, k0 + CH);

  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* Ks = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* Vs = Ks + SUBK * DP;
  __nv_bfloat16* Qs = Vs + SUBK * DP;       // [MAXQ][DP]

  for (int qb = 0; qb < nqv; qb += MAXQ) {
    const int nqb = min(MAXQ, nqv - qb);
    // stage queries (query vector qi -> head g*rep + qi / T, row qi % T)
    for (int idx = threadIdx.x; idx < nqb * (D / 8); idx += blockDim.x) {
      const int qi = idx / (D / 8), ch = idx % (D / 8);
      const int gq = qb + qi;
      const int hq = g * rep + gq / a.T, t = gq % a.T;
      reinterpret_cast<uint4*>(Qs + qi * DP)[ch] =
          reinterpret_cast<const uint4*>(a.q + ((size_t)t * a.nq + hq) * D)[ch];
    }
    float m[QPW], lsum[QPW], o[QPW][DPL];
    int myq[QPW], mypos[QPW];
#pragma unroll
    for (int i = 0; i < QPW; ++i) {
      m[i] = -INFINITY;
      lsum[i] = 0.f;
#pragma unroll
      for (int d = 0; d < DPL; ++d) o[i][d] = 0.f;
      const int qi = warp * QPW + i;
      myq[i] = qi;
      mypos[i] = qi < nqb ? a.qpos[(qb + qi) % a.T] : -1;
    }
    for (int kb = k0; kb < k1; kb += SUBK) {
      __syncthreads();
      // stage K/V sub-tile
      for (int idx = threadIdx.x; idx < SUBK * (D / 8); idx += blockDim.x) {
        const int j = idx / (D / 8), ch = idx % (D / 8);
        const int kp = kb + j;
        uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
        if (kp < k1) {
          size_t base;
          if (a.block_table) {
            const int blk = a.block_table[kp / a.block_size];
            base = ((size_t)blk * a.block_size + (kp % a.block_size)) * a.nkv + g;
          } else {
            base = (size_t)kp * a.nkv + g;
          }
          kv = reinterpret_cast<const uint4*>(a.kcache + base * D)[ch];
          vv = reinterpret_cast<const uint4*>(a.vcache + base * D)[ch];
        }
        reinterpret_cast<uint4*>(Ks + j * DP)[ch] = kv;
        reinterpret_cast<uint4*>(Vs + j * DP)[ch] = vv;
      }
      __syncthreads();
      const int kp = kb + lane;
#pragma unroll
      for (int i = 0; i < QPW; ++i) {
        if (myq[i] >= nqb) continue;
        // score of key `lane` for query i
        float sc = 0.f;
        const uint4* qrow = reinterpret_cast<const uint4*>(Qs + myq[i] * DP);
        const uint4* krow = reinterpret_cast<const uint4*>(Ks + lane * DP);
#pragma unroll 4
        for (int ch = 0; ch < D / 8; ++ch) {
          const uint4 qa = qrow[ch], kk = krow[ch];
          const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&qa);
          const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&kk);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float2 qf = __bfloat1622float2(q2[u]), kf = __bfloat1622float2(k2[u]);
            sc = fmaf(qf.x, kf.x, sc);
            sc = fmaf(qf.y, kf.y, sc);
          }
        }
        sc *= a.scale;
        const bool valid = kp < k1 && (!a.causal || kp <= mypos[i]);
        if (!valid) sc = -INFINITY;
        const float mt = warp_max(sc);
        const float mn = fmaxf(m[i], mt);
        if (mn == -INFINITY) continue;     // nothing visible yet for this query
        const float pj = valid ? __expf(sc - mn) : 0.f;
        const float corr = __expf(m[i] - mn);
        lsum[i] = lsum[i] * corr + warp_sum(pj);
        m[i] = mn;
#pragma unroll
        for (int d = 0; d < DPL; ++d) o[i][d] *= corr;
        for (int j = 0; j < SUBK; ++j) {
          const float pb = __shfl_sync(0xffffffffu, pj, j);
          if (pb == 0.f) continue;
          const __nv_bfloat16* vrow = Vs + j * DP + lane * DPL;
#pragma unroll
          for (int d = 0; d < DPL; ++d) o[i][d] = fmaf(pb, __bfloat162float(vrow[d]), o[i][d]);
        }
      }
    }
    // write partials
#pragma unroll
    for (int i = 0; i < QPW; ++i) {
      if (myq[i] >= nqb) continue;
      const size_t qv = (size_t)(qb + myq[i]);
      const size_t pidx = ((size_t)g * a.max_splits + s) * nqv + qv;
      float* po = a.part_o + pidx * D + lane * DPL;
#pragma unroll
      for (int d = 0; d < DPL; ++d) po[d] = o[i][d];
      if (lane == 0) {
        a.part_ml[pidx * 2] = m[i];
        a.part_ml[pidx * 2 + 1] = lsum[i];
      }
    }
  }
}

__global__ void attn_combine_kernel(DecodeArgs a, const __nv_bfloat16* gate, long long gate_ld, int gate_off,
                                    __nv_bfloat16* out, long long out_ld) {
  const int hq = blockIdx.x, t = blockIdx.y;
  const int D = a.D;
  const int rep = a.nq / a.nkv;
  const int g = hq / rep;
  const int nqv = rep * a.T;
  const int qv = (hq % rep) * a.T + t;
  const int n_keys = a.causal ? a.qpos[t] + 1 : a.qpos[a.T - 1] + 1;
  const int ns = (n_keys + CH - 1) / CH;
  float M = -INFINITY;
  for (int s = 0; s < ns; ++s) M = fmaxf(M, a.part_ml[(((size_t)g * a.max_splits + s) * nqv + qv) * 2]);
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float acc = 0.f, L = 0.f;
    for (int s = 0; s < ns; ++s) {
      const size_t pidx = ((size_t)g * a.max_splits + s) * nqv + qv;
      const float ms = a.part_ml[pidx * 2];
      if (ms == -INFINITY) continue;
      const float wgt = __expf(ms - M);
      L += wgt * a.part_ml[pidx * 2 + 1];
      acc += wgt * a.part_o[pidx * D + c];
    }
    float y = acc / L;
    if (gate) {
      const float gv = __bfloat162float(gate[(size_t)t * gate_ld + gate_off + (size_t)hq * D + c]);
      y *= 1.f / (1.f + __expf(-gv));
    }
    out[(size_t)t * out_ld + (size_t)hq * D + c] = __float2bfloat16(y);
  }
}

}  // namespace q38

// ----------------------------------------------------------------------------- bindings
void q38_attn_prep(torch::Tensor proj, int64_t q_off, int64_t k_off, int64_t v_off, int64_t nq, int64_t nkv,
                   int64_t D, int64_t rd, torch::Tensor qn, torch::Tensor kn, torch::Tensor inv_freq,
                   double rope_scale, double eps, torch::Tensor pos, c10::optional<torch::Tensor> q_out,
                   torch::Tensor kcache, torch::Tensor vcache, c10::optional<torch::Tensor> block_table,
                   int64_t block_size) {
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
  const int T = (int)proj.size(0);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  q38::attn_prep_kernel<<<dim3(T, (unsigned)(nq + nkv)), (unsigned)D, D * sizeof(float), st>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void q38_attn_decode(torch::Tensor q, torch::Tensor kcache, torch::Tensor vcache,
                     c10::optional<torch::Tensor> block_table, int64_t block_size, torch::Tensor qpos, double scale,
                     int64_t causal, c10::optional<torch::Tensor> gate, int64_t gate_off, torch::Tensor out,
                     torch::Tensor part_o, torch::Tensor part_ml, int64_t max_keys) {
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
  const int nqv = nq / nkv * T;
  TORCH_CHECK(part_o.numel() >= (int64_t)nkv * a.max_splits * nqv * D, "attention partial buffer too small");
  TORCH_CHECK(part_ml.numel() >= (int64_t)nkv * a.max_splits * nqv * 2, "attention partial buffer too small");
  a.part_o = part_o.data_ptr<float>();
  a.part_ml = part_ml.data_ptr<float>();
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int qpw = (std::min(nqv, q38::MAXQ) + 7) / 8;
  const size_t smem = (size_t)(2 * q38::SUBK + q38::MAXQ) * (D + 8) * 2;
  dim3 grid(nkv, a.max_splits);
#define Q38_DEC(DD, QQ)                                                                                     \
  {                                                                                                         \
    auto k = q38::attn_decode_kernel<DD, QQ>;                                                               \
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);                        \
    k<<<grid, 256, smem, st>>>(a);                                                                          \
  }
#define Q38_DEC_D(DD)                                                   \
  if (qpw <= 1) Q38_DEC(DD, 1) else if (qpw <= 2) Q38_DEC(DD, 2)        \
  else if (qpw <= 4) Q38_DEC(DD, 4) else if (qpw <= 8) Q38_DEC(DD, 8)   \
  else Q38_DEC(DD, 12)
  if (D == 256) { Q38_DEC_D(256) }
  else if (D == 128) { Q38_DEC_D(128) }
  else if (D == 64) { Q38_DEC_D(64) }
  else TORCH_CHECK(false, "head dim 64/128/256 supported");
#undef Q38_DEC_D
#undef Q38_DEC
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const __nv_bfloat16* gp = gate ? reinterpret_cast<const __nv_bfloat16*>(gate->data_ptr()) : nullptr;
  q38::attn_combine_kernel<<<dim3(nq, T), std::min(D, 256), 0, st>>>(
      a, gp, gate ? gate->stride(0) : 0, (int)gate_off, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
      out.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
