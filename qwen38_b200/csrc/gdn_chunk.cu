// Chunked gated delta rule for prefill (K-GDN-PREFILL), head dim 128, chunk 64.
//
// For a chunk of C rows with cumulative log-decay G (G_i = sum_{t<=i} g_t), L2-normalised q, k
// (q scaled by Dk^-0.5), values v and write strengths beta:
//   A    = strictly_lower(-(beta_i k_i . k_j) exp(G_i - G_j)),   T = (I - A)^-1
//   U    = T (beta v),   W = T (beta k exp(G))
//   V'   = U - W S
//   O    = (q exp(G)) S + tril(q k^T exp(G_i - G_j)) V'
//   S   <- exp(G_C) S + (k exp(G_C - G))^T V'
// which equals C steps of the sequential rule (the WY / UT form; the reference runs the same
// computation through TT-NN chunk_gated_delta_rule ops, graft/gdn/tp.py:629-652, chunk 128).
//
// gdn_chunk_prep_kernel (grid: chunks x heads) does the conv1d + SiLU, L2 norms, gates and every
// per-chunk product on tensor cores (mma.sync m16n8k16, fp32 accumulate) with an fp32 forward
// substitution for T.  gdn_chunk_scan_kernel (grid: heads x 4 value-column slices) carries the
// fp32 state in MMA accumulators across the chunks of the prefill call.  gdn_out_norm_kernel
// applies the gated RMSNorm times silu(z).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace q38 {
namespace gdnc {

constexpr int D = 128;     // head dim (k and v)
constexpr int C = 64;      // chunk rows
constexpr int KC = 4;      // conv taps
constexpr int DPAD = D + 8;
constexpr int CPAD = C + 8;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t (&r)[2]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t (&r)[2]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// A fragment (16x16) at (m0, k0) of a row-major bf16 matrix with leading dimension ld.
__device__ __forceinline__ void frag_a(const __nv_bfloat16* base, int ld, int m0, int k0, uint32_t (&a)[4]) {
  const int lane = threadIdx.x & 31;
  ldsm_x4(smem_u32(base + (m0 + (lane & 15)) * ld + k0 + (lane >> 4) * 8), a);
}
// A fragment (16x16) of A = X^T where X is row-major [k][m] (ld): transposed load.
__device__ __forceinline__ void frag_a_t(const __nv_bfloat16* base, int ld, int m0, int k0, uint32_t (&a)[4]) {
  const int lane = threadIdx.x & 31;
  ldsm_x4_t(smem_u32(base + (k0 + (lane & 7) + ((lane >> 4) << 3)) * ld + m0 + ((lane >> 3) & 1) * 8), a);
}
// B fragment (16x8) at (k0, n0) where B^T is stored row-major [n][k] (k contiguous).
__device__ __forceinline__ void frag_b_nk(const __nv_bfloat16* base, int ld, int k0, int n0, uint32_t (&b)[2]) {
  const int lane = threadIdx.x & 31;
  ldsm_x2(smem_u32(base + (n0 + (lane & 7)) * ld + k0 + ((lane >> 3) & 1) * 8), b);
}
// B fragment (16x8) at (k0, n0) where B is stored row-major [k][n] (n contiguous).
__device__ __forceinline__ void frag_b_kn(const __nv_bfloat16* base, int ld, int k0, int n0, uint32_t (&b)[2]) {
  const int lane = threadIdx.x & 31;
  ldsm_x2_t(smem_u32(base + (k0 + (lane & 15)) * ld + n0), b);
}

struct PrepArgs {
  const __nv_bfloat16* proj;   // [S, width]
  long long proj_ld;
  const __nv_bfloat16* window; // [K-1, Cch]: inputs before row 0
  int S;                       // rows of this prefill call
  const float* conv_w;         // [Cch, K]
  const float* A_log;          // [nv]
  const float* dt_bias;
  int nk, nv, Cch;
  __nv_bfloat16* U;            // [nchunks, nv, C, D]
  __nv_bfloat16* W;
  __nv_bfloat16* Qp;           // q exp(G)
  __nv_bfloat16* Kp;           // k exp(G_C - G)
  __nv_bfloat16* P;            // [nchunks, nv, C, C]
  float* dec;                  // [nchunks, nv] exp(G_C)
};

// shared-memory plan (bytes): two 51 KB regions reused phase by phase, so two CTAs fit per SM
//   R0: raw rows [C+3][3D] bf16 (conv input)  ->  beta v, beta k exp(G) [C][DPAD] bf16 + A [C][C+4] f32
//   R1: q, k, v [C][DPAD] bf16                ->  N [C][C+4] f32 + T [C][CPAD] bf16
constexpr int RAW_B = (C + KC - 1) * 3 * D * 2;                 // 51,456
constexpr int QKV_B = 3 * C * DPAD * 2;                         // 52,224
constexpr int BVK_B = 2 * C * DPAD * 2;                         // 34,816
constexpr int AM_B = C * (C + 4) * 4;                           // 17,408
constexpr int R0_B = (RAW_B > BVK_B + AM_B ? RAW_B : BVK_B + AM_B);
constexpr int R1_B = QKV_B;
static_assert(R1_B >= AM_B + C * CPAD * 2, "N and T fit in R1");
constexpr int PREP_SMEM = R0_B + R1_B + 5 * C * 4 + 64;
constexpr int FB = 16;                                          // forward-substitution block

__global__ void __launch_bounds__(256, 2) gdn_chunk_prep_kernel(PrepArgs a) {
  extern __shared__ __align__(16) uint8_t sm[];
  __nv_bfloat16* raw = reinterpret_cast<__nv_bfloat16*>(sm);                  // R0
  __nv_bfloat16* bv = reinterpret_cast<__nv_bfloat16*>(sm);                   // R0 after the conv
  __nv_bfloat16* bk = bv + C * DPAD;
  float* Am = reinterpret_cast<float*>(sm + BVK_B);
  __nv_bfloat16* qs = reinterpret_cast<__nv_bfloat16*>(sm + R0_B);            // R1
  __nv_bfloat16* ks = qs + C * DPAD;
  __nv_bfloat16* vs = ks + C * DPAD;
  float* Nm = reinterpret_cast<float*>(sm + R0_B);                            // R1 after Q K^T
  __nv_bfloat16* Tb = reinterpret_cast<__nv_bfloat16*>(Nm + C * (C + 4));
  float* gsh = reinterpret_cast<float*>(sm + R0_B + R1_B);                     // g, then cumulative G
  float* bsh = gsh + C;
  float* nq = bsh + C;
  float* nkk = nq + C;
  float* eg = nkk + C;                                                         // exp(G)

  const int c = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r0 = c * C;
  const int nrows = min(C, a.S - r0);
  const int rep = a.nv / a.nk, kh = h / rep;
  const int chan[3] = {kh * D, a.nk * D + kh * D, 2 * a.nk * D + h * D};

  // conv taps (static weights) before waiting on the previous kernel: thread t owns q/k channel
  // t (q: t < D, k: t >= D) for every row, and v channel t % D for rows (t / D) * C/2 ..
  const int qk_part = tid / D, qk_ch = tid % D;
  float wqk[KC], wv[KC];
#pragma unroll
  for (int j = 0; j < KC; ++j) {
    wqk[j] = a.conv_w[(size_t)(chan[qk_part] + qk_ch) * KC + j];
    wv[j] = a.conv_w[(size_t)(chan[2] + qk_ch) * KC + j];
  }
  pdl_wait();
  pdl_trigger();

  // ---- 1. raw projected rows r0-3 .. r0+C-1 (q, k, v channels of the head), all copies in flight
  for (int idx = tid; idx < (C + KC - 1) * 3 * (D / 8); idx += blockDim.x) {
    const int i = idx / (3 * (D / 8));
    const int rem = idx % (3 * (D / 8));
    const int part = rem / (D / 8), ch8 = rem % (D / 8);
    const int r = r0 - (KC - 1) + i;
    uint4* dst = reinterpret_cast<uint4*>(raw + i * 3 * D + part * D + ch8 * 8);
    if (r < 0) cp_async16(dst, a.window + (size_t)(r + KC - 1) * a.Cch + chan[part] + ch8 * 8);
    else if (r < a.S) cp_async16(dst, a.proj + (size_t)r * a.proj_ld + chan[part] + ch8 * 8);
    else *dst = make_uint4(0, 0, 0, 0);
  }
  cp_async_commit();
  if (tid < C) {
    const int r = r0 + tid;
    float g = 0.f, be = 0.f;
    if (tid < nrows) {
      const int ca = a.Cch + a.nv * D + a.nv + h, cb = a.Cch + a.nv * D + h;
      const float av = __bfloat162float(a.proj[(size_t)r * a.proj_ld + ca]);
      const float bvv = __bfloat162float(a.proj[(size_t)r * a.proj_ld + cb]);
      const float x = av + a.dt_bias[h];
      const float sp = x > 20.f ? x : log1pf(__expf(x));
      g = -__expf(a.A_log[h]) * sp;
      be = 1.f / (1.f + __expf(-bvv));
    }
    gsh[tid] = g;
    bsh[tid] = be;
  }
  cp_async_wait<0>();
  __syncthreads();
  // ---- 2. causal conv + SiLU with a sliding register window; cumulative decay (thread 0)
  {
    __nv_bfloat16* dst = qk_part == 0 ? qs : ks;
    const int col = qk_part * D + qk_ch;
    float x0 = __bfloat162float(raw[0 * 3 * D + col]), x1 = __bfloat162float(raw[1 * 3 * D + col]);
    float x2 = __bfloat162float(raw[2 * 3 * D + col]);
    for (int i = 0; i < C; ++i) {
      const float x3 = __bfloat162float(raw[(i + 3) * 3 * D + col]);
      const float y = wqk[0] * x0 + wqk[1] * x1 + wqk[2] * x2 + wqk[3] * x3;
      dst[i * DPAD + qk_ch] = __float2bfloat16(i < nrows ? silu_f(y) : 0.f);
      x0 = x1; x1 = x2; x2 = x3;
    }
    const int vcol = 2 * D + qk_ch, i0 = qk_part * (C / 2);
    x0 = __bfloat162float(raw[(i0 + 0) * 3 * D + vcol]);
    x1 = __bfloat162float(raw[(i0 + 1) * 3 * D + vcol]);
    x2 = __bfloat162float(raw[(i0 + 2) * 3 * D + vcol]);
    for (int i = i0; i < i0 + C / 2; ++i) {
      const float x3 = __bfloat162float(raw[(i + 3) * 3 * D + vcol]);
      const float y = wv[0] * x0 + wv[1] * x1 + wv[2] * x2 + wv[3] * x3;
      vs[i * DPAD + qk_ch] = __float2bfloat16(i < nrows ? silu_f(y) : 0.f);
      x0 = x1; x1 = x2; x2 = x3;
    }
  }
  if (tid == 0) {
    float acc = 0.f;
    for (int i = 0; i < C; ++i) {
      acc += gsh[i];
      gsh[i] = acc;
    }
  }
  __syncthreads();
  // ---- 3. L2 norms (warp per row, fixed order), exp(G)
  for (int i = warp; i < C; i += 8) {
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int m = 0; m < D / 32; ++m) {
      const float q = __bfloat162float(qs[i * DPAD + lane + 32 * m]);
      const float k = __bfloat162float(ks[i * DPAD + lane + 32 * m]);
      sq += q * q;
      sk += k * k;
    }
    sq = warp_sum(sq);
    sk = warp_sum(sk);
    if (lane == 0) {
      nq[i] = rsqrtf(sq + 1e-6f) * rsqrtf((float)D);
      nkk[i] = rsqrtf(sk + 1e-6f);
    }
  }
  if (tid < C) eg[tid] = __expf(gsh[tid]);
  __syncthreads();
  const float GC = gsh[C - 1];
  const size_t ch_base = ((size_t)c * a.nv + h) * C;
  // ---- 4. normalise in place, q exp(G) and k exp(G_C - G) to global, beta v and beta k exp(G)
  for (int idx = tid; idx < C * (D / 8); idx += blockDim.x) {
    const int i = idx / (D / 8), c8 = (idx % (D / 8)) * 8;
    const uint4 qu = *reinterpret_cast<const uint4*>(qs + i * DPAD + c8);
    const uint4 ku = *reinterpret_cast<const uint4*>(ks + i * DPAD + c8);
    const uint4 vu = *reinterpret_cast<const uint4*>(vs + i * DPAD + c8);
    const __nv_bfloat16* qv = reinterpret_cast<const __nv_bfloat16*>(&qu);
    const __nv_bfloat16* kv = reinterpret_cast<const __nv_bfloat16*>(&ku);
    const __nv_bfloat16* vv = reinterpret_cast<const __nv_bfloat16*>(&vu);
    const float sq = nq[i], sk = nkk[i], e = eg[i], ekc = __expf(GC - gsh[i]), be = bsh[i];
    __align__(16) __nv_bfloat16 qn[8], kn[8], qp[8], kp[8], bvo[8], bko[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float q = __bfloat162float(qv[u]) * sq;
      const float k = __bfloat162float(kv[u]) * sk;
      qn[u] = __float2bfloat16(q);
      kn[u] = __float2bfloat16(k);
      qp[u] = __float2bfloat16(q * e);
      kp[u] = __float2bfloat16(k * ekc);
      bvo[u] = __float2bfloat16(be * __bfloat162float(vv[u]));
      bko[u] = __float2bfloat16(be * __bfloat162float(kn[u]) * e);
    }
    *reinterpret_cast<uint4*>(qs + i * DPAD + c8) = *reinterpret_cast<const uint4*>(qn);
    *reinterpret_cast<uint4*>(ks + i * DPAD + c8) = *reinterpret_cast<const uint4*>(kn);
    *reinterpret_cast<uint4*>(a.Qp + (ch_base + i) * D + c8) = *reinterpret_cast<const uint4*>(qp);
    *reinterpret_cast<uint4*>(a.Kp + (ch_base + i) * D + c8) = *reinterpret_cast<const uint4*>(kp);
    *reinterpret_cast<uint4*>(bv + i * DPAD + c8) = *reinterpret_cast<const uint4*>(bvo);
    *reinterpret_cast<uint4*>(bk + i * DPAD + c8) = *reinterpret_cast<const uint4*>(bko);
  }
  __syncthreads();
  // ---- 5. K K^T -> A (fp32), Q K^T -> P (bf16 to global).  warp: m-tile warp/2, n-tiles 4*(warp%2)..+3
  {
    const int mt = warp >> 1, nt0 = (warp & 1) * 4;
    float kk[4][4], qk[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) kk[n][e] = qk[n][e] = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < D; k0 += 16) {
      uint32_t fa[4], fq[4];
      frag_a(ks, DPAD, mt * 16, k0, fa);
      frag_a(qs, DPAD, mt * 16, k0, fq);
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        uint32_t fb[2];
        frag_b_nk(ks, DPAD, k0, (nt0 + n) * 8, fb);
        mma16816(kk[n], fa, fb);
        mma16816(qk[n], fq, fb);
      }
    }
#pragma unroll
    for (int n = 0; n < 4; ++n) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = mt * 16 + (lane >> 2) + hh * 8;
        const int j = (nt0 + n) * 8 + (lane & 3) * 2;
        float pv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float dec = __expf(gsh[i] - gsh[j + e]);
          Am[i * (C + 4) + j + e] = (j + e < i) ? -bsh[i] * kk[n][2 * hh + e] * dec : 0.f;
          pv[e] = (j + e <= i) ? qk[n][2 * hh + e] * dec : 0.f;
        }
        *reinterpret_cast<__nv_bfloat162*>(a.P + (ch_base + i) * C + j) = __floats2bfloat162_rn(pv[0], pv[1]);
      }
    }
  }
  __syncthreads();
  // ---- 6. T = (I - A)^-1 (strictly lower part N), blocked over 16-row blocks:
  //   diagonal blocks by forward substitution (one warp each), then block rows I = 1..3:
  //   M_IJ = sum_{K=J}^{I-1} A_IK T_KJ,  T_IJ = M_IJ + N_II M_IJ   (T_KK = I + N_KK)
  for (int i = tid; i < C * (C + 4); i += blockDim.x) Nm[i] = 0.f;
  __syncthreads();
  if (warp < C / FB) {
    const int b0 = warp * FB;
    const int j = b0 + (lane & (FB - 1));
    for (int il = 1; il < FB; ++il) {
      const int i = b0 + il;
      if (lane < il) {
        float s = Am[i * (C + 4) + j];
        for (int m = j + 1; m < i; ++m) s += Am[i * (C + 4) + m] * Nm[m * (C + 4) + j];
        Nm[i * (C + 4) + j] = s;
      }
      __syncwarp();
    }
  }
  __syncthreads();
  for (int I = 1; I < C / FB; ++I) {
    // M for every J < I: entries (J, r, cc) spread over the threads, kept in registers
    float mval[3];
    int ment[3];
    int nm = 0;
    for (int e = tid; e < I * FB * FB; e += blockDim.x) {
      const int J = e / (FB * FB), r = (e / FB) % FB, cc = e % FB;
      const int i = I * FB + r, jcol = J * FB + cc;
      float s = 0.f;
      for (int K = J; K < I; ++K) {
#pragma unroll 4
        for (int m = 0; m < FB; ++m) {
          const int km = K * FB + m;
          const float t = (K == J) ? ((m == cc ? 1.f : 0.f) + Nm[km * (C + 4) + jcol]) : Nm[km * (C + 4) + jcol];
          s += Am[i * (C + 4) + km] * t;
        }
      }
      mval[nm] = s;
      ment[nm] = e;
      ++nm;
    }
    __syncthreads();
    for (int q = 0; q < nm; ++q) {               // stage M in the (still zero) T_IJ blocks
      const int e = ment[q];
      const int J = e / (FB * FB), r = (e / FB) % FB, cc = e % FB;
      Nm[(I * FB + r) * (C + 4) + J * FB + cc] = mval[q];
    }
    __syncthreads();
    for (int q = 0; q < nm; ++q) {               // T_IJ = M + N_II M
      const int e = ment[q];
      const int J = e / (FB * FB), r = (e / FB) % FB, cc = e % FB;
      const int i = I * FB + r, jcol = J * FB + cc;
      float s = mval[q];
      for (int m = 0; m < r; ++m) s += Nm[i * (C + 4) + I * FB + m] * Nm[(I * FB + m) * (C + 4) + jcol];
      mval[q] = s;
    }
    __syncthreads();
    for (int q = 0; q < nm; ++q) {
      const int e = ment[q];
      const int J = e / (FB * FB), r = (e / FB) % FB, cc = e % FB;
      Nm[(I * FB + r) * (C + 4) + J * FB + cc] = mval[q];
    }
    __syncthreads();
  }
  for (int idx = tid; idx < C * C; idx += blockDim.x) {
    const int i = idx / C, j = idx % C;
    Tb[i * CPAD + j] = __float2bfloat16(i == j ? 1.f : Nm[i * (C + 4) + j]);
  }
  __syncthreads();
  // ---- 7. U = T (beta v), W = T (beta k exp(G)).  64 x 128 outputs each; warp: m-tile warp/2, 8 n-tiles
  {
    const int mt = warp >> 1, nt0 = (warp & 1) * 8;
    float u[8][4], w[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) u[n][e] = w[n][e] = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < C; k0 += 16) {
      uint32_t ft[4];
      frag_a(Tb, CPAD, mt * 16, k0, ft);
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        uint32_t fv[2], fk[2];
        frag_b_kn(bv, DPAD, k0, (nt0 + n) * 8, fv);
        frag_b_kn(bk, DPAD, k0, (nt0 + n) * 8, fk);
        mma16816(u[n], ft, fv);
        mma16816(w[n], ft, fk);
      }
    }
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int d = (nt0 + n) * 8 + (lane & 3) * 2;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = mt * 16 + (lane >> 2) + hh * 8;
        *reinterpret_cast<__nv_bfloat162*>(a.U + (ch_base + i) * D + d) =
            __floats2bfloat162_rn(u[n][2 * hh], u[n][2 * hh + 1]);
        *reinterpret_cast<__nv_bfloat162*>(a.W + (ch_base + i) * D + d) =
            __floats2bfloat162_rn(w[n][2 * hh], w[n][2 * hh + 1]);
      }
    }
  }
  if (tid == 0) a.dec[(size_t)c * a.nv + h] = __expf(GC);
}

struct ScanArgs {
  const __nv_bfloat16* U;
  const __nv_bfloat16* W;
  const __nv_bfloat16* Qp;
  const __nv_bfloat16* Kp;
  const __nv_bfloat16* P;
  const float* dec;
  float* state;                // [nv, D, D]
  float* O;                    // [S, nv, D] (fp32, before the gated norm)
  int S, nchunks, nv;
};

constexpr int VS = 32;          // value columns per CTA
constexpr int VSP = VS + 8;
constexpr int SCAN_SMEM = (3 * C * DPAD + C * CPAD + C * VSP + D * VSP + C * VSP) * 2;

// grid (nv, D / VS), 128 threads.  Warp w keeps state rows 32w .. 32w+31 x VS columns in MMA
// accumulator fragments (fp32) for the whole call.
__global__ void __launch_bounds__(128, 1) gdn_chunk_scan_kernel(ScanArgs a) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t sm[];
  __nv_bfloat16* Ws = reinterpret_cast<__nv_bfloat16*>(sm);      // [C][DPAD]
  __nv_bfloat16* Qs = Ws + C * DPAD;
  __nv_bfloat16* Ks = Qs + C * DPAD;
  __nv_bfloat16* Ps = Ks + C * DPAD;                              // [C][CPAD]
  __nv_bfloat16* Us = Ps + C * CPAD;                              // [C][VSP]
  __nv_bfloat16* Sb = Us + C * VSP;                               // [D][VSP]
  __nv_bfloat16* Vp = Sb + D * VSP;                               // [C][VSP]
  const int h = blockIdx.x, col0 = blockIdx.y * VS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* st = a.state + (size_t)h * D * D;

  // state fragments: rows 32*warp + 16*mt + (lane>>2) (+8), cols 8*nt + 2*(lane&3) (+1)
  float Sf[2][4][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = warp * 32 + mt * 16 + (lane >> 2) + (e >> 1) * 8;
        const int cc = col0 + nt * 8 + (lane & 3) * 2 + (e & 1);
        Sf[mt][nt][e] = st[(size_t)r * D + cc];
      }

  for (int c = 0; c < a.nchunks; ++c) {
    const size_t base = ((size_t)c * a.nv + h) * C;
    // ---- stage chunk inputs (asynchronous copies: one memory round trip per chunk)
    for (int idx = tid; idx < C * (D / 8); idx += blockDim.x) {
      const int i = idx / (D / 8), ch = idx % (D / 8);
      cp_async16(Ws + i * DPAD + ch * 8, a.W + (base + i) * D + ch * 8);
      cp_async16(Qs + i * DPAD + ch * 8, a.Qp + (base + i) * D + ch * 8);
      cp_async16(Ks + i * DPAD + ch * 8, a.Kp + (base + i) * D + ch * 8);
    }
    for (int idx = tid; idx < C * (C / 8); idx += blockDim.x) {
      const int i = idx / (C / 8), ch = idx % (C / 8);
      cp_async16(Ps + i * CPAD + ch * 8, a.P + (base + i) * C + ch * 8);
    }
    for (int idx = tid; idx < C * (VS / 8); idx += blockDim.x) {
      const int i = idx / (VS / 8), ch = idx % (VS / 8);
      cp_async16(Us + i * VSP + ch * 8, a.U + (base + i) * D + col0 + ch * 8);
    }
    cp_async_commit();
    // state (bf16) as a B operand [D][VS]
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int r = warp * 32 + mt * 16 + (lane >> 2) + hh * 8;
          const int cc = nt * 8 + (lane & 3) * 2;
          *reinterpret_cast<__nv_bfloat162*>(Sb + r * VSP + cc) =
              __floats2bfloat162_rn(Sf[mt][nt][2 * hh], Sf[mt][nt][2 * hh + 1]);
        }
    cp_async_wait<0>();
    __syncthreads();
    // ---- V' = U - W S   (warp: rows 16*warp.., all VS columns)
    float vp[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) vp[nt][e] = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < D; k0 += 16) {
      uint32_t fa[4];
      frag_a(Ws, DPAD, warp * 16, k0, fa);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        uint32_t fb[2];
        frag_b_kn(Sb, VSP, k0, nt * 8, fb);
        mma16816(vp[nt], fa, fb);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = warp * 16 + (lane >> 2) + hh * 8;
        const int cc = nt * 8 + (lane & 3) * 2;
        const float u0 = __bfloat162float(Us[i * VSP + cc]), u1 = __bfloat162float(Us[i * VSP + cc + 1]);
        *reinterpret_cast<__nv_bfloat162*>(Vp + i * VSP + cc) =
            __floats2bfloat162_rn(u0 - vp[nt][2 * hh], u1 - vp[nt][2 * hh + 1]);
      }
    __syncthreads();
    // ---- O = Q' S + P V'
    float o[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[nt][e] = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < D; k0 += 16) {
      uint32_t fa[4];
      frag_a(Qs, DPAD, warp * 16, k0, fa);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        uint32_t fb[2];
        frag_b_kn(Sb, VSP, k0, nt * 8, fb);
        mma16816(o[nt], fa, fb);
      }
    }
#pragma unroll
    for (int k0 = 0; k0 < C; k0 += 16) {
      uint32_t fa[4];
      frag_a(Ps, CPAD, warp * 16, k0, fa);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        uint32_t fb[2];
        frag_b_kn(Vp, VSP, k0, nt * 8, fb);
        mma16816(o[nt], fa, fb);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = warp * 16 + (lane >> 2) + hh * 8;
        const int r = c * C + i;
        if (r < a.S) {
          const int cc = col0 + nt * 8 + (lane & 3) * 2;
          *reinterpret_cast<float2*>(a.O + ((size_t)r * a.nv + h) * D + cc) =
              make_float2(o[nt][2 * hh], o[nt][2 * hh + 1]);
        }
      }
    // ---- S = exp(G_C) S + K'^T V'
    const float d = a.dec[(size_t)c * a.nv + h];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) Sf[mt][nt][e] *= d;
#pragma unroll
    for (int k0 = 0; k0 < C; k0 += 16) {
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        uint32_t fa[4];
        frag_a_t(Ks, DPAD, warp * 32 + mt * 16, k0, fa);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          uint32_t fb[2];
          frag_b_kn(Vp, VSP, k0, nt * 8, fb);
          mma16816(Sf[mt][nt], fa, fb);
        }
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = warp * 32 + mt * 16 + (lane >> 2) + (e >> 1) * 8;
        const int cc = col0 + nt * 8 + (lane & 3) * 2 + (e & 1);
        st[(size_t)r * D + cc] = Sf[mt][nt][e];
      }
}

// out[r, h*D + c] = rmsnorm(O[r, h, :]) * norm_w * silu(z[r, h*D + c]); one warp per (row, head)
__global__ void gdn_out_norm_kernel(const float* __restrict__ O, const __nv_bfloat16* __restrict__ proj,
                                    long long proj_ld, int zoff, const float* __restrict__ norm_w, float eps,
                                    int S, int nv, __nv_bfloat16* __restrict__ out, long long out_ld) {
  pdl_wait();
  pdl_trigger();
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= S * nv) return;
  const int r = gw / nv, h = gw % nv;
  const float* o = O + ((size_t)r * nv + h) * D;
  float v[D / 32];
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < D / 32; ++u) {
    v[u] = o[lane + 32 * u];
    ss += v[u] * v[u];
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / D + eps);
#pragma unroll
  for (int u = 0; u < D / 32; ++u) {
    const int cc = lane + 32 * u;
    const float z = __bfloat162float(proj[(size_t)r * proj_ld + zoff + h * D + cc]);
    out[(size_t)r * out_ld + h * D + cc] = __float2bfloat16(v[u] * inv * norm_w[cc] * silu_f(z));
  }
}

}  // namespace gdnc
}  // namespace q38

// Chunked prefill of one GDN layer: outputs [S, nv*D] (bf16), state / window advanced in place.
void q38_gdn_chunk_prefill(torch::Tensor proj, torch::Tensor window, torch::Tensor state, torch::Tensor conv_w,
                           torch::Tensor A_log, torch::Tensor dt_bias, torch::Tensor norm_w, torch::Tensor out,
                           torch::Tensor work, int64_t nk, int64_t nv, double eps) {
  using namespace q38::gdnc;
  c10::cuda::CUDAGuard guard(proj.device());
  const int S = (int)proj.size(0);
  const int Cch = (int)conv_w.size(0);
  TORCH_CHECK(conv_w.size(1) == KC, "conv kernel 4 required");
  TORCH_CHECK(Cch == 2 * nk * D + nv * D, "chunked GDN prefill serves head dim 128");
  TORCH_CHECK(proj.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(proj.data_ptr()) & 15) == 0,
              "16-byte aligned projection rows required");
  const int nch = (S + C - 1) / C;
  const size_t mat = (size_t)nch * nv * C * D;       // elements per [nch, nv, C, D] buffer
  const size_t need = 4 * mat * 2 + (size_t)nch * nv * C * C * 2 + (size_t)nch * nv * 4 + (size_t)S * nv * D * 4;
  TORCH_CHECK((size_t)work.numel() * work.element_size() >= need, "GDN chunk workspace too small");
  uint8_t* wp = reinterpret_cast<uint8_t*>(work.data_ptr());
  auto take = [&](size_t bytes) { uint8_t* p = wp; wp += (bytes + 255) & ~size_t(255); return p; };
  PrepArgs pa{};
  pa.proj = reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr());
  pa.proj_ld = proj.stride(0);
  pa.window = reinterpret_cast<const __nv_bfloat16*>(window.data_ptr());
  pa.S = S;
  pa.conv_w = conv_w.data_ptr<float>();
  pa.A_log = A_log.data_ptr<float>();
  pa.dt_bias = dt_bias.data_ptr<float>();
  pa.nk = (int)nk; pa.nv = (int)nv; pa.Cch = Cch;
  pa.U = reinterpret_cast<__nv_bfloat16*>(take(mat * 2));
  pa.W = reinterpret_cast<__nv_bfloat16*>(take(mat * 2));
  pa.Qp = reinterpret_cast<__nv_bfloat16*>(take(mat * 2));
  pa.Kp = reinterpret_cast<__nv_bfloat16*>(take(mat * 2));
  pa.P = reinterpret_cast<__nv_bfloat16*>(take((size_t)nch * nv * C * C * 2));
  pa.dec = reinterpret_cast<float*>(take((size_t)nch * nv * 4));
  float* O = reinterpret_cast<float*>(take((size_t)S * nv * D * 4));
  TORCH_CHECK((size_t)(wp - reinterpret_cast<uint8_t*>(work.data_ptr())) <=
                  (size_t)work.numel() * work.element_size(), "GDN chunk workspace too small");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  TORCH_CHECK(q38::set_smem_once<gdn_chunk_prep_kernel>(PREP_SMEM) == cudaSuccess &&
                  q38::set_smem_once<gdn_chunk_scan_kernel>(SCAN_SMEM) == cudaSuccess, "cudaFuncSetAttribute failed");
  gdn_chunk_prep_kernel<<<dim3(nch, (unsigned)nv), 256, PREP_SMEM, st>>>(pa);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  ScanArgs sa{};
  sa.U = pa.U; sa.W = pa.W; sa.Qp = pa.Qp; sa.Kp = pa.Kp; sa.P = pa.P; sa.dec = pa.dec;
  sa.state = state.data_ptr<float>();
  sa.O = O;
  sa.S = S; sa.nchunks = nch; sa.nv = (int)nv;
  gdn_chunk_scan_kernel<<<dim3((unsigned)nv, D / VS), 128, SCAN_SMEM, st>>>(sa);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const int warps = S * (int)nv;
  gdn_out_norm_kernel<<<(warps + 7) / 8, 256, 0, st>>>(O, pa.proj, pa.proj_ld, Cch, norm_w.data_ptr<float>(),
                                                       (float)eps, S, (int)nv,
                                                       reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                                       out.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

size_t q38_gdn_chunk_workspace_bytes(int64_t S, int64_t nv) {
  using namespace q38::gdnc;
  const size_t nch = (S + C - 1) / C;
  const size_t mat = nch * nv * C * D;
  return 4 * ((mat * 2 + 255) & ~size_t(255)) + ((nch * nv * C * C * 2 + 255) & ~size_t(255)) +
         ((nch * nv * 4 + 255) & ~size_t(255)) + ((S * nv * D * 4 + 255) & ~size_t(255)) + 4096;
}
