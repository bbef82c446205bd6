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
// B200 layout of the work:
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

#include "sf_q4.h"
#include "sf_q4_internal.h"

namespace sf {
extern std::atomic<long long> g_launches;

namespace {

constexpr int kAttnWarps = 4;
constexpr int kMaxD = 256;
constexpr int kMaxGroup = 8;

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
  // enough CTAs for about four per SM, at least 64 tokens per split
  int want = (4 * sms + BHkv - 1) / BHkv;
  int cap = (T + 63) / 64;
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
  cudaError_t e = D == 64 ? launch_split_d<64>(a, grid, st)
                          : (D == 128 ? launch_split_d<128>(a, grid, st) : launch_split_d<256>(a, grid, st));
  if (e != cudaSuccess) return cuda_fail(e, "kv_attn_split_kernel launch");
  kv_attn_merge_kernel<<<(unsigned)(B * H), 128, 0, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kv_attn_merge_kernel launch");
  g_launches.fetch_add(2, std::memory_order_relaxed);
  return SF_OK;
}

}  // extern "C"
