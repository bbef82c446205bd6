// sf_kv_attention.cu -- decode-phase attention over an int8-quantized KV cache.
//
// Reference: fused_quantized_attention_decode
// (siliconfer/kernels/metal/q4_attention.py:200-260, kernel source 80-175) over
// the cache format of siliconfer/model/kv_cache.py:49-69 (int8 codes, one fp32
// scale per (batch, kv head, token) vector):
//   k = k_code * k_scale,  v = v_code * v_scale             (dequant inline)
//   score_t = (q . k_t) / sqrt(head_dim)
//   out = sum_t softmax(score)_t * v_t                        (fp32)
// split over T_cache into tiles whose partial (m, l, acc) are merged with the
// flash-attention rule M = max m_i, L = sum l_i e^(m_i - M),
// out = sum acc_i e^(m_i - M) / max(L, 1e-20)  (q4_attention.py:248-256).
//
// Two kernels share this file: a tensor-core kernel for head_dim 64/128 and
// GQA groups up to 16 (the default, described before kv_attn_tc_kernel), and
// the CUDA-core kernel below (head_dim 256).
// B200 layout of the work (CUDA-core kernel):
//  * one CTA per (T split, batch, kv head) serves every query head of that kv
//    head (GQA group), so each K/V byte is read once per group, not once per
//    query head as in the reference;
//  * a warp takes 32 consecutive tokens at a time: lane = token for the q.k
//    scores (16-byte loads of the key row; q is in shared memory and read as
//    a broadcast), one online-softmax update per 32 tokens (warp max / sum by
//    shuffles), then lane = slice of head_dim for the value sum (each value
//    row is one coalesced warp load);
//  * the warps of a CTA merge in shared memory and write the split's partial
//    (m, l, acc) into the caller's workspace; a second kernel merges splits.
// Roofline: HBM-bound, 2 * T * head_dim bytes of codes + 8 * T bytes of
// scales per (batch, kv head).
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdlib>

#include "sf_q4.h"
#include "sf_q4_internal.h"

namespace sf {
extern std::atomic<long long> g_launches;

namespace {

constexpr int kAttnWarps = 4;

struct AttnArgs {
  const void* q;          // [B, H, D] of q_dtype
  const int8_t* kc;       // [B, Hkv, T, D]
  const float* ks;        // [B, Hkv, T]
  const int8_t* vc;
  const float* vs;
  float* part;            // workspace: [B, H, nsplit] x (m, l) then [B, H, nsplit, D] acc
  void* out;              // [B, H, D] of out_dtype
  int B, H, Hkv, T, D, G, nsplit, tsplit, q_dtype, out_dtype;
  float inv_sqrt_d;
};

__device__ __forceinline__ float ld_q(const void* q, size_t i, int dt) {
  if (dt == SF_F32) return static_cast<const float*>(q)[i];
  if (dt == SF_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(q)[i]);
  return __half2float(static_cast<const __half*>(q)[i]);
}

template <int D, int G>
__global__ void __launch_bounds__(32 * kAttnWarps) kv_attn_split_kernel(const AttnArgs a) {
  constexpr int DL = D / 32;     // head_dim elements per lane in the value sum
  __shared__ __align__(16) float qs[G][D];
  __shared__ float wm[kAttnWarps][G], wl[kAttnWarps][G];
  __shared__ float wacc[kAttnWarps][G][D];
  const int split = blockIdx.x, bk = blockIdx.y;      // bk = b * Hkv + kv head
  const int b = bk / a.Hkv, kvh = bk % a.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the group's queries, pre-scaled by 1/sqrt(D)
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    const int h = kvh * G + g;
    qs[g][d] = ld_q(a.q, ((size_t)b * a.H + h) * D + d, a.q_dtype) * a.inv_sqrt_d;
  }
  __syncthreads();
  const int t0 = split * a.tsplit, t1 = min(a.T, t0 + a.tsplit);
  const int8_t* kb = a.kc + (size_t)bk * a.T * D;
  const int8_t* vb = a.vc + (size_t)bk * a.T * D;
  const float* ksb = a.ks + (size_t)bk * a.T;
  const float* vsb = a.vs + (size_t)bk * a.T;

  float m[G], l[G], acc[G][DL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < DL; ++e) acc[g][e] = 0.f;
  }
  for (int base = t0 + 32 * warp; base < t1; base += 32 * kAttnWarps) {
    const int t = base + lane;
    const bool valid = t < t1;
    // scores: lane = token
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = 0.f;
    if (valid) {
      const int8_t* krow = kb + (size_t)t * D;
#pragma unroll 2
      for (int d0 = 0; d0 < D; d0 += 16) {
        const int4 kv4 = *reinterpret_cast<const int4*>(krow + d0);
        const int8_t* k8 = reinterpret_cast<const int8_t*>(&kv4);
        float kf[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) kf[e] = (float)k8[e];
#pragma unroll
        for (int g = 0; g < G; ++g) {
#pragma unroll
          for (int e4 = 0; e4 < 16; e4 += 4) {
            const float4 qv = *reinterpret_cast<const float4*>(&qs[g][d0 + e4]);
            s[g] = fmaf(qv.x, kf[e4], s[g]);
            s[g] = fmaf(qv.y, kf[e4 + 1], s[g]);
            s[g] = fmaf(qv.z, kf[e4 + 2], s[g]);
            s[g] = fmaf(qv.w, kf[e4 + 3], s[g]);
          }
        }
      }
      const float sk = ksb[t];
#pragma unroll
      for (int g = 0; g < G; ++g) s[g] *= sk;
    }
    // online softmax over these 32 tokens
    float p[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float bm = valid ? s[g] : -INFINITY;
#pragma unroll
      for (int o = 16; o; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
      const float mn = fmaxf(m[g], bm);
      const float corr = expf(m[g] - mn);   // m = -inf at the start: e^-inf = 0
      p[g] = valid ? expf(s[g] - mn) : 0.f;
      float ps = p[g];
#pragma unroll
      for (int o = 16; o; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      l[g] = l[g] * corr + ps;
      m[g] = mn;
#pragma unroll
      for (int e = 0; e < DL; ++e) acc[g][e] *= corr;
    }
    // value sum: lane = head_dim slice [lane*DL, lane*DL + DL)
    const int nt = min(32, t1 - base);
    for (int i = 0; i < nt; ++i) {
      const int tt = base + i;
      const float sv = vsb[tt];
      const int8_t* vrow = vb + (size_t)tt * D + lane * DL;
      float vf[DL];
      if constexpr (DL == 8) {
        const int2 v2 = *reinterpret_cast<const int2*>(vrow);
        const int8_t* v8 = reinterpret_cast<const int8_t*>(&v2);
#pragma unroll
        for (int e = 0; e < 8; ++e) vf[e] = (float)v8[e] * sv;
      } else if constexpr (DL == 4) {
        const int v1 = *reinterpret_cast<const int*>(vrow);
        const int8_t* v8 = reinterpret_cast<const int8_t*>(&v1);
#pragma unroll
        for (int e = 0; e < 4; ++e) vf[e] = (float)v8[e] * sv;
      } else {
#pragma unroll
        for (int e = 0; e < DL; ++e) vf[e] = (float)vrow[e] * sv;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pi = __shfl_sync(0xffffffffu, p[g], i);
#pragma unroll
        for (int e = 0; e < DL; ++e) acc[g][e] = fmaf(pi, vf[e], acc[g][e]);
      }
    }
  }
  // merge the warps of this CTA, write the split's partial
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) { wm[warp][g] = m[g]; wl[warp][g] = l[g]; }
#pragma unroll
    for (int e = 0; e < DL; ++e) wacc[warp][g][lane * DL + e] = acc[g][e];
  }
  __syncthreads();
  const size_t nbh = (size_t)a.B * a.H;
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    float M = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm[w][g]);
    float L = 0.f, A = 0.f;
    for (int w = 0; w < kAttnWarps; ++w) {
      const float c = M == -INFINITY ? 0.f : expf(wm[w][g] - M);
      L += wl[w][g] * c;
      A += wacc[w][g][d] * c;
    }
    const size_t bhs = ((size_t)b * a.H + kvh * G + g) * a.nsplit + split;
    a.part[2 * nbh * a.nsplit + bhs * D + d] = A;
    if (d == 0) {
      a.part[2 * bhs] = M;
      a.part[2 * bhs + 1] = L;
    }
  }
}

__global__ void __launch_bounds__(256) kv_attn_merge_kernel(const AttnArgs a) {
  const int bh = blockIdx.x;
  const size_t nbh = (size_t)a.B * a.H;
  const float* ml = a.part + 2 * (size_t)bh * a.nsplit;
  const float* acc = a.part + 2 * nbh * a.nsplit + (size_t)bh * a.nsplit * a.D;
  float M = -INFINITY;
  for (int s = 0; s < a.nsplit; ++s) M = fmaxf(M, ml[2 * s]);
  for (int d = threadIdx.x; d < a.D; d += blockDim.x) {
    float L = 0.f, A = 0.f;
    for (int s = 0; s < a.nsplit; ++s) {
      const float c = M == -INFINITY ? 0.f : expf(ml[2 * s] - M);
      L += ml[2 * s + 1] * c;
      A += acc[(size_t)s * a.D + d] * c;
    }
    const float y = A / fmaxf(L, 1e-20f);
    const size_t o = (size_t)bh * a.D + d;
    if (a.out_dtype == SF_F32) static_cast<float*>(a.out)[o] = y;
    else if (a.out_dtype == SF_BF16) static_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(y);
    else static_cast<__half*>(a.out)[o] = __float2half_rn(y);
  }
}

// ---------------------------------------------------------------------------
// Tensor-core variant (head_dim 64 or 128, GQA group <= 8): one warp takes 32
// tokens at a time, with the products transposed so that the tokens, not the
// few query heads of a group, fill the MMA's 16 rows:
//  * S^T = K Q^T on mma.sync m16n8k16 (fp16 in, fp32 accumulate): the int8
//    keys are the A operand (16 tokens x 16 of head_dim), converted exactly
//    (0x6400 | (v + 128) - 1152); the group's query heads, padded to 8, are
//    the B operand, split into an fp16 high and low part (two MMAs) so that q
//    keeps about 22 bits.  Inside each 16-wide block of head_dim the order is
//    permuted the same way in Q and K (logical k 2t, 2t+1, 2t+8, 2t+9 =
//    physical 4t .. 4t+3), which leaves q.k unchanged and lets each lane
//    fetch its key bytes with one 32-bit load;
//  * the scores are scaled per token by k_scale; a lane holds heads 2t, 2t+1
//    of its tokens and keeps their online-softmax state;
//  * O^T += V^T P'^T with P' = p * v_scale * 2^10 (split high/low, the power
//    of two keeps P' clear of fp16 subnormals and is divided out at the end):
//    the values, staged as fp16 in shared memory, are the A operand through
//    ldmatrix.trans, and P' goes through a small shared tile to become the B
//    operand (also ldmatrix.trans).  The accumulators hold O^T[d][head] with
//    the same heads 2t, 2t+1 per lane as the softmax state.
// Per 32 tokens and head_dim 128 this is 32 + 32 MMAs (the untransposed form,
// with at most 8 of 16 rows in use, needs 64 + 64).  With PR (groups of at
// most 4 heads) a head's high and low parts take two adjacent columns (2h, 2h+1)
// of one MMA instead of two MMAs, and each lane's column pair (2t, 2t+1) is then
// one head, t: 16 + 16 MMAs.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
// two signed bytes (b0 low) -> exact half2
__device__ __forceinline__ void i8x4_to_h2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  uint32_t a, b;
  asm("prmt.b32 %0, %1, %2, 0x4140;" : "=r"(a) : "r"(u), "r"(0x64646464u));
  asm("prmt.b32 %0, %1, %2, 0x4342;" : "=r"(b) : "r"(u), "r"(0x64646464u));
  const __half2 off = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
  lo = h2u(__hsub2(*reinterpret_cast<__half2*>(&a), off));
  hi = h2u(__hsub2(*reinterpret_cast<__half2*>(&b), off));
}
__device__ __forceinline__ void split_h2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
  hi = h2u(__halves2half2(h0, h1));
  lo = h2u(__halves2half2(__float2half_rn(x0 - __half2float(h0)), __float2half_rn(x1 - __half2float(h1))));
}

// Per-warp shared memory of the tensor-core kernel: two stages of raw int8
// K and V rows (32 tokens, row pitch D + 16: the 32-bit key-fragment reads of
// 8 rows land on 8 different bank groups), then the block's values as fp16
// (row pitch 2D + 16: conflict-free ldmatrix), then the P'^T tiles.
template <int D>
struct TcAttnLayout {
  static constexpr int RP = D + 16;                 // raw row pitch
  static constexpr int RAW = 32 * RP;               // one K or V block
  static constexpr int STAGE = 2 * RAW;             // K then V
  static constexpr int PITCH = 2 * D + 16;          // fp16 value rows
  static constexpr int PT = 32 * 16;                // P'^T high (then low): [32 tokens][8 heads] fp16
  static constexpr int WARP = 2 * STAGE + 32 * PITCH + 2 * PT;
  static constexpr int SMEM = 4 * WARP;             // kAttnWarps = 4
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}

template <int D, bool PR>
__global__ void __launch_bounds__(32 * kAttnWarps, 2) kv_attn_tc_kernel(const AttnArgs a) {
  using Ly = TcAttnLayout<D>;
  constexpr int KS = D / 16;            // k-steps of S^T (over head_dim)
  constexpr int DM = D / 16;            // 16-row d tiles of O^T
  constexpr int CH = D / 16;            // 16-byte chunks per row
  constexpr float kPScale = 1024.f;
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float wm[kAttnWarps][16], wl[kAttnWarps][16];
  const int split = blockIdx.x, bk = blockIdx.y;
  const int b = bk / a.Hkv, kvh = bk % a.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int G = a.G;
  // B fragments of Q^T (column = head g, pre-scaled by 1/sqrt(D)), permuted as above
  // (PR: column g is the high (g even) or low part of head g / 2)
  uint32_t qh[KS][2], ql[KS][2];
  const int qhead = PR ? (g >> 1) : g;
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (qhead < G) {
      const size_t qo = ((size_t)b * a.H + kvh * G + qhead) * D + 16 * ks + 4 * t;
#pragma unroll
      for (int e = 0; e < 4; ++e) v[e] = ld_q(a.q, qo + e, a.q_dtype) * a.inv_sqrt_d;
    }
    split_h2(v[0], v[1], qh[ks][0], ql[ks][0]);   // b0: logical k 2t, 2t+1
    split_h2(v[2], v[3], qh[ks][1], ql[ks][1]);   // b1: logical k 2t+8, 2t+9
    if (PR && (g & 1)) {
      qh[ks][0] = ql[ks][0];
      qh[ks][1] = ql[ks][1];
    }
  }
  const int t0 = split * a.tsplit, t1 = min(a.T, t0 + a.tsplit);
  const int8_t* kb = a.kc + (size_t)bk * a.T * D;
  const int8_t* vb = a.vc + (size_t)bk * a.T * D;
  const float* ksb = a.ks + (size_t)bk * a.T;
  const float* vsb = a.vs + (size_t)bk * a.T;
  const uint32_t wbase = smem_u32(smem + warp * Ly::WARP);
  const uint32_t vtile = wbase + 2 * Ly::STAGE;
  const uint32_t ptile = vtile + 32 * Ly::PITCH;   // P'^T high, then low at + PT

  // this warp's blocks: base = t0 + 32 * (warp + kAttnWarps * i)
  auto issue = [&](int i) {
    const int base = t0 + 32 * (warp + kAttnWarps * i);
    if (base < t1) {
      const uint32_t st = wbase + (uint32_t)(i & 1) * Ly::STAGE;
#pragma unroll
      for (int c = lane; c < 32 * CH; c += 32) {
        const int tok = c / CH, dp = (c % CH) * 16;
        const bool v = base + tok < t1;
        const size_t go = (size_t)(v ? base + tok : t0) * D + dp;
        cp_async16(st + tok * Ly::RP + dp, kb + go, v);
        cp_async16(st + Ly::RAW + tok * Ly::RP + dp, vb + go, v);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  // softmax state of heads 2t and 2t + 1
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float o[DM][4];   // O^T: d tile md rows 16 md + g (+8), heads 2t, 2t + 1
#pragma unroll
  for (int i = 0; i < DM; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  issue(0);
  issue(1);
  for (int i = 0;; ++i) {
    const int base = t0 + 32 * (warp + kAttnWarps * i);
    if (base >= t1) break;
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    __syncwarp();
    const uint32_t st = wbase + (uint32_t)(i & 1) * Ly::STAGE;
    // the block's values as fp16 (exact)
#pragma unroll
    for (int c = lane; c < 32 * CH; c += 32) {
      const int tok = c / CH, dp = (c % CH) * 16;
      uint32_t w[4];
      asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                   : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
                   : "r"(st + Ly::RAW + tok * Ly::RP + dp));
      uint32_t h[8];
      i8x4_to_h2x2(w[0], h[0], h[1]);
      i8x4_to_h2x2(w[1], h[2], h[3]);
      i8x4_to_h2x2(w[2], h[4], h[5]);
      i8x4_to_h2x2(w[3], h[6], h[7]);
      const uint32_t sa = vtile + tok * Ly::PITCH + dp * 2;
      asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(sa), "r"(h[0]), "r"(h[1]), "r"(h[2]), "r"(h[3]) : "memory");
      asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(sa + 16), "r"(h[4]), "r"(h[5]), "r"(h[6]), "r"(h[7]) : "memory");
    }
    // S^T = K Q^T for two tiles of 16 tokens: s[mt] = rows (tokens) 16 mt + g
    // and + 8, columns (heads) 2t, 2t + 1
    float s[2][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      s[mt][0] = s[mt][1] = s[mt][2] = s[mt][3] = 0.f;
      const uint32_t kr = st + (16 * mt + g) * Ly::RP + 4 * t;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t w0, w1;
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(w0) : "r"(kr + 16 * ks));
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(w1) : "r"(kr + 8 * Ly::RP + 16 * ks));
        uint32_t af[4];
        i8x4_to_h2x2(w0, af[0], af[2]);   // row g: logical k 2t, 2t+1 | 2t+8, 2t+9
        i8x4_to_h2x2(w1, af[1], af[3]);   // row g + 8
        mma16816(s[mt], af, qh[ks][0], qh[ks][1]);
        if (!PR) mma16816(s[mt], af, ql[ks][0], ql[ks][1]);
      }
    }
    if constexpr (PR) {
      // head t's score = its high column + its low column (kept in both)
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int r = 0; r < 2; ++r) s[mt][2 * r] = s[mt][2 * r + 1] = s[mt][2 * r] + s[mt][2 * r + 1];
    }
    // per-token key scale, mask past t1, online softmax per head (column)
    float rmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int tok = base + 16 * mt + g + 8 * r;
        const float sk = tok < t1 ? ksb[tok] : 0.f;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          s[mt][2 * r + e] = tok < t1 ? s[mt][2 * r + e] * sk : -INFINITY;
          rmax[e] = fmaxf(rmax[e], s[mt][2 * r + e]);
        }
      }
    float corr[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      rmax[e] = fmaxf(rmax[e], __shfl_xor_sync(0xffffffffu, rmax[e], 4));
      rmax[e] = fmaxf(rmax[e], __shfl_xor_sync(0xffffffffu, rmax[e], 8));
      rmax[e] = fmaxf(rmax[e], __shfl_xor_sync(0xffffffffu, rmax[e], 16));
      const float mn = fmaxf(m[e], rmax[e]);
      corr[e] = expf(m[e] - mn);
      m[e] = mn;
    }
    float rsum[2] = {0.f, 0.f};
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int tl = 16 * mt + g + 8 * r, tok = base + tl;
        const float sv = tok < t1 ? vsb[tok] * kPScale : 0.f;
        const float p0 = expf(s[mt][2 * r] - m[0]), p1 = expf(s[mt][2 * r + 1] - m[1]);
        rsum[0] += p0;
        rsum[1] += p1;
        uint32_t hi, lo;
        split_h2(p0 * sv, p1 * sv, hi, lo);
        if constexpr (PR) {
          // columns 2t, 2t+1 = high and low part of head t's p' (p0 == p1 here)
          hi = (hi & 0xFFFFu) | (lo << 16);
          asm volatile("st.shared.u32 [%0], %1;" ::"r"(ptile + tl * 16 + 4 * t), "r"(hi) : "memory");
        } else {
          asm volatile("st.shared.u32 [%0], %1;" ::"r"(ptile + tl * 16 + 4 * t), "r"(hi) : "memory");
          asm volatile("st.shared.u32 [%0], %1;" ::"r"(ptile + Ly::PT + tl * 16 + 4 * t), "r"(lo) : "memory");
        }
      }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      rsum[e] += __shfl_xor_sync(0xffffffffu, rsum[e], 4);
      rsum[e] += __shfl_xor_sync(0xffffffffu, rsum[e], 8);
      rsum[e] += __shfl_xor_sync(0xffffffffu, rsum[e], 16);
      l[e] = l[e] * corr[e] + rsum[e];
    }
#pragma unroll
    for (int q = 0; q < DM; ++q) {
      o[q][0] *= corr[0]; o[q][1] *= corr[1];
      o[q][2] *= corr[0]; o[q][3] *= corr[1];
    }
    __syncwarp();
    // O^T += V^T P'^T: per 16-token k-step, B = P'^T (high and low) by one
    // ldmatrix.x4.trans, A = V^T of each 16-row d tile by another
    const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      uint32_t ph0, ph1, pl0, pl1;
      {
        const uint32_t addr = ptile + (uint32_t)(mi >> 1) * Ly::PT + (16 * kk + (mi & 1) * 8 + rr) * 16;
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(ph0), "=r"(ph1), "=r"(pl0), "=r"(pl1)
                     : "r"(addr));
      }
#pragma unroll
      for (int md = 0; md < DM; ++md) {
        const uint32_t addr = vtile + (16 * kk + (mi >> 1) * 8 + rr) * Ly::PITCH + (16 * md + (mi & 1) * 8) * 2;
        uint32_t av[4];
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(av[0]), "=r"(av[1]), "=r"(av[2]), "=r"(av[3])
                     : "r"(addr));
        mma16816(o[md], av, ph0, ph1);
        if (!PR) mma16816(o[md], av, pl0, pl1);
      }
    }
    __syncwarp();          // stage i & 1, the fp16 tile and the P' tiles are free again
    issue(i + 2);
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  // merge the warps of this CTA (rows < G), write the split's partial
  __syncthreads();   // every warp is done with its shared memory
  auto wacc = reinterpret_cast<float (*)[16][D]>(smem);
  if constexpr (PR) {
    // head t: its high and low columns summed
    if (g == 0) { wm[warp][t] = m[0]; wl[warp][t] = l[0]; }
#pragma unroll
    for (int q = 0; q < DM; ++q) {
      const int d = 16 * q + g;
      wacc[warp][t][d] = (o[q][0] + o[q][1]) / kPScale;
      wacc[warp][t][d + 8] = (o[q][2] + o[q][3]) / kPScale;
    }
  } else {
    if (g == 0) {
      wm[warp][2 * t] = m[0]; wl[warp][2 * t] = l[0];
      wm[warp][2 * t + 1] = m[1]; wl[warp][2 * t + 1] = l[1];
    }
#pragma unroll
    for (int q = 0; q < DM; ++q) {
      const int d = 16 * q + g;
      wacc[warp][2 * t][d] = o[q][0] / kPScale;
      wacc[warp][2 * t + 1][d] = o[q][1] / kPScale;
      wacc[warp][2 * t][d + 8] = o[q][2] / kPScale;
      wacc[warp][2 * t + 1][d + 8] = o[q][3] / kPScale;
    }
  }
  __syncthreads();
  const size_t nbh = (size_t)a.B * a.H;
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int gg = i / D, d = i % D;
    float M = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm[w][gg]);
    float L = 0.f, A = 0.f;
    for (int w = 0; w < kAttnWarps; ++w) {
      const float c = M == -INFINITY ? 0.f : expf(wm[w][gg] - M);
      L += wl[w][gg] * c;
      A += wacc[w][gg][d] * c;
    }
    const size_t bhs = ((size_t)b * a.H + kvh * G + gg) * a.nsplit + split;
    a.part[2 * nbh * a.nsplit + bhs * D + d] = A;
    if (d == 0) {
      a.part[2 * bhs] = M;
      a.part[2 * bhs + 1] = L;
    }
  }
}

template <int D, bool PR>
cudaError_t launch_tc_dp(const AttnArgs& a, dim3 grid, cudaStream_t st) {
  using Ly = TcAttnLayout<D>;
  static_assert(Ly::SMEM >= kAttnWarps * 16 * D * 4, "merge buffer must fit");
  cudaError_t e =
      cudaFuncSetAttribute(kv_attn_tc_kernel<D, PR>, cudaFuncAttributeMaxDynamicSharedMemorySize, Ly::SMEM);
  if (e != cudaSuccess) return e;
  kv_attn_tc_kernel<D, PR><<<grid, 32 * kAttnWarps, Ly::SMEM, st>>>(a);
  return cudaGetLastError();
}
template <int D>
cudaError_t launch_tc_d(const AttnArgs& a, dim3 grid, cudaStream_t st) {
  return a.G <= 4 ? launch_tc_dp<D, true>(a, grid, st) : launch_tc_dp<D, false>(a, grid, st);
}

template <int D>
cudaError_t launch_split_d(const AttnArgs& a, dim3 grid, cudaStream_t st) {
  switch (a.G) {
    case 1: kv_attn_split_kernel<D, 1><<<grid, 32 * kAttnWarps, 0, st>>>(a); break;
    case 2: kv_attn_split_kernel<D, 2><<<grid, 32 * kAttnWarps, 0, st>>>(a); break;
    case 4: kv_attn_split_kernel<D, 4><<<grid, 32 * kAttnWarps, 0, st>>>(a); break;
    case 7: kv_attn_split_kernel<D, 7><<<grid, 32 * kAttnWarps, 0, st>>>(a); break;
    case 8: kv_attn_split_kernel<D, 8><<<grid, 32 * kAttnWarps, 0, st>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

int choose_splits(int T, int BHkv, int sms) {
  // about two CTAs per SM (the resident count of the tensor-core kernel), at
  // least 256 tokens per split
  int want = (2 * sms + BHkv - 1) / BHkv;
  int cap = (T + 255) / 256;
  if (want > cap) want = cap;
  return want < 1 ? 1 : want;
}

}  // namespace
}  // namespace sf

using namespace sf;

extern "C" {

size_t sf_kv_attention_workspace_bytes(int B, int H, int D, int n_split) {
  if (B <= 0 || H <= 0 || D <= 0 || n_split <= 0) return 0;
  return (size_t)B * H * n_split * (2 + (size_t)D) * 4;
}

int sf_kv_attention_splits(int B, int Hkv, int T) {
  return choose_splits(T, B * Hkv, device_info().sms);
}

int sf_kv_attention_decode(const void* q, int q_dtype, const int8_t* k_codes, const float* k_scales,
                           const int8_t* v_codes, const float* v_scales, void* out, int out_dtype, int B, int H,
                           int Hkv, int T, int D, int n_split, void* workspace, size_t workspace_bytes,
                           void* stream) {
  if (!q || !k_codes || !k_scales || !v_codes || !v_scales || !out || !workspace)
    return fail(SF_ERR_NULL, "null pointer argument");
  if (q_dtype < 0 || q_dtype > 2 || out_dtype < 0 || out_dtype > 2) return fail(SF_ERR_DTYPE, "unknown dtype code");
  if (B < 1 || H < 1 || Hkv < 1 || T < 1 || H % Hkv)
    return fail(SF_ERR_SHAPE, "need B, H, n_kv_heads, T >= 1 and H divisible by n_kv_heads");
  const int G = H / Hkv;
  if (!(G == 1 || G == 2 || G == 4 || G == 7 || G == 8))
    return fail(SF_ERR_UNSUPPORTED, "GQA group size %d not built (1, 2, 4, 7, 8)", G);
  if (!(D == 64 || D == 128 || D == 256))
    return fail(SF_ERR_UNSUPPORTED, "head_dim %d not built (64, 128, 256)", D);
  if ((reinterpret_cast<uintptr_t>(k_codes) | reinterpret_cast<uintptr_t>(v_codes)) & 15)
    return fail(SF_ERR_ALIGN, "k_codes and v_codes must be 16-byte aligned");
  if (n_split <= 0) n_split = choose_splits(T, B * Hkv, device_info().sms);
  if (n_split > T) n_split = T;
  if (workspace_bytes < sf_kv_attention_workspace_bytes(B, H, D, n_split))
    return fail(SF_ERR_SHAPE, "workspace too small: need %zu bytes", sf_kv_attention_workspace_bytes(B, H, D, n_split));
  AttnArgs a{};
  a.q = q; a.kc = k_codes; a.ks = k_scales; a.vc = v_codes; a.vs = v_scales;
  a.part = static_cast<float*>(workspace); a.out = out;
  a.B = B; a.H = H; a.Hkv = Hkv; a.T = T; a.D = D; a.G = G; a.nsplit = n_split;
  a.tsplit = (T + n_split - 1) / n_split;
  a.q_dtype = q_dtype; a.out_dtype = out_dtype;
  a.inv_sqrt_d = 1.0f / sqrtf((float)D);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)n_split, (unsigned)(B * Hkv));
  cudaError_t e;
  if (D <= 128 && G <= 8) {
    e = D == 64 ? launch_tc_d<64>(a, grid, st) : launch_tc_d<128>(a, grid, st);
  } else {
    e = D == 64 ? launch_split_d<64>(a, grid, st)
                : (D == 128 ? launch_split_d<128>(a, grid, st) : launch_split_d<256>(a, grid, st));
  }
  if (e != cudaSuccess) return cuda_fail(e, "kv_attn_split_kernel launch");
  kv_attn_merge_kernel<<<(unsigned)(B * H), 128, 0, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kv_attn_merge_kernel launch");
  g_launches.fetch_add(2, std::memory_order_relaxed);
  return SF_OK;
}

}  // extern "C"
