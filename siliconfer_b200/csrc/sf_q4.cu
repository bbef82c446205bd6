// sf_q4.cu -- B200 (sm_100a) kernels behind the siliconfer Q4Linear C ABI.
//
// Kernels in this file:
//   q4_gemv_kernel<T, ASYM>  decode GEMV for T <= 8 tokens (the hot path).
//   q4_gemv_generic_kernel   any legal shape (even group size, K % gs == 0);
//                            also serves the reference's "scalar" entry.
//   q4_dequant_kernel        bit-exact fp32 dequant (+ fp16/bf16 rounding).
//   q4_quantize_pack_kernel  RTN quantize + nibble pack, bit-exact with numpy.
// The tcgen05 prefill GEMM lives in sf_q4_gemm_tc.cu.
//
// Reference algorithm: siliconfer/kernels/neon/q4_gemv.cpp:37-140 (sym),
// :145-238 (asym) and siliconfer/kernels/neon/__init__.py:88-124 (numpy
// oracle).  Per (row, group): sym y += s * sum(sext(q) * x); asym
// y += s * (sum(q * x) - z * sum(x)).

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include <atomic>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "sf_q4.h"
#include "sf_q4_internal.h"

namespace sf {

thread_local char g_last_error[512] = "";
std::atomic<long long> g_launches{0};

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(SF_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

SF_DEFINE_ERROR_READER(take_dev_error_gemv)

DeviceInfo& device_info() {
  static DeviceInfo info[kMaxDevices];
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) dev = 0;
  DeviceInfo& d = info[dev];
  if (!d.ready) {
    std::lock_guard<std::mutex> lock(mu);
    if (!d.ready) {
      cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
      cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
      if (d.sms <= 0) d.sms = 148;
      d.ready = true;
    }
  }
  return d;
}

// ---------------------------------------------------------------------------
// Output / input conversions
// ---------------------------------------------------------------------------
__device__ __forceinline__ void store_y(void* y, size_t idx, float v, int dt) {
  if (dt == SF_F32) reinterpret_cast<float*>(y)[idx] = v;
  else if (dt == SF_F16) reinterpret_cast<__half*>(y)[idx] = __float2half_rn(v);
  else reinterpret_cast<__nv_bfloat16*>(y)[idx] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ float load_x(const void* x, size_t idx, int dt) {
  if (dt == SF_F32) return reinterpret_cast<const float*>(x)[idx];
  if (dt == SF_F16) return __half2float(reinterpret_cast<const __half*>(x)[idx]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[idx]);
}

// Load 8 consecutive activations starting at element idx (idx % 8 == 0, base
// 16-byte aligned) as fp32.
__device__ __forceinline__ void load_x8(const void* x, size_t idx, int dt, float* out) {
  if (dt == SF_F32) {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + idx);
    float4 a = __ldg(p), b = __ldg(p + 1);
    out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
    out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
  } else {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(
        reinterpret_cast<const uint16_t*>(x) + idx));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (dt == SF_F16) {
        float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        out[2 * i] = f.x; out[2 * i + 1] = f.y;
      } else {
        float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
        out[2 * i] = f.x; out[2 * i + 1] = f.y;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Nibble -> exact fp32 without an int->float conversion.
//
// Nibble j of a 32-bit word sits at bits 4j..4j+3.  OR-ing it into the
// mantissa of 2^(23-4j) gives exactly 2^(23-4j) + u; subtracting that magic
// (plus 8 for two's-complement nibbles, whose sign bit is flipped by the same
// single LOP3) leaves the exact small integer.  Nibbles 5..7 are shifted down
// by 12 bits and reuse slots 2..4.  One LOP3 per weight, one FADD2 per pair.
// ---------------------------------------------------------------------------
template <int J, bool ASYM>
__device__ __forceinline__ float nib_magic(uint32_t v) {
  constexpr uint32_t kMask = 0xFu << (4 * J);
  constexpr uint32_t kExp = (127u + 23u - 4u * J) << 23;      // bits of 2^(23-4J)
  constexpr uint32_t kFlip = ASYM ? 0u : (0x8u << (4 * J));   // u ^ 8 for sym
  return __uint_as_float((v & kMask) ^ (kExp | kFlip));
}

template <int J, bool ASYM>
__device__ __forceinline__ constexpr float nib_bias() {
  return (float)(1u << (23 - 4 * J)) + (ASYM ? 0.0f : 8.0f);
}

// acc += dequant_int(word) . x[0..7]   (x given as 4 consecutive float2)
template <bool ASYM>
__device__ __forceinline__ float2 dot8(uint32_t w, const float2* x, float2 acc) {
  const uint32_t h = w >> 12;
  const float2 p0 = __fadd2_rn(make_float2(nib_magic<0, ASYM>(w), nib_magic<1, ASYM>(w)),
                               make_float2(-nib_bias<0, ASYM>(), -nib_bias<1, ASYM>()));
  const float2 p1 = __fadd2_rn(make_float2(nib_magic<2, ASYM>(w), nib_magic<3, ASYM>(w)),
                               make_float2(-nib_bias<2, ASYM>(), -nib_bias<3, ASYM>()));
  const float2 p2 = __fadd2_rn(make_float2(nib_magic<4, ASYM>(w), nib_magic<2, ASYM>(h)),
                               make_float2(-nib_bias<4, ASYM>(), -nib_bias<2, ASYM>()));
  const float2 p3 = __fadd2_rn(make_float2(nib_magic<3, ASYM>(h), nib_magic<4, ASYM>(h)),
                               make_float2(-nib_bias<3, ASYM>(), -nib_bias<4, ASYM>()));
  acc = __ffma2_rn(p0, x[0], acc);
  acc = __ffma2_rn(p1, x[1], acc);
  acc = __ffma2_rn(p2, x[2], acc);
  acc = __ffma2_rn(p3, x[3], acc);
  return acc;
}

// ---------------------------------------------------------------------------
// Decode GEMV: persistent, warp-specialised, bulk-copy pipelined.
//
// CTA b owns output rows [N*b/grid, N*(b+1)/grid).  Its rows are streamed in
// chunks of R full rows (R*K/2 contiguous bytes of W, plus the chunk's scales
// and zeros) by ONE producer thread with cp.async.bulk into an S-stage ring of
// shared-memory buffers guarded by mbarriers.  Consumer warp (slice s, row
// group rg) owns the K-slice [s*32*CK, (s+1)*32*CK): each lane holds its CK
// activations per token in registers for the whole kernel, reads LB packed
// bytes of each of its RW rows per chunk from shared memory, and accumulates
// in fp32.  Partials are reduced across the warp with a butterfly
// reduce-scatter and across K-slices through shared memory; one thread per
// (token, row) adds the bias and writes y.
// ---------------------------------------------------------------------------
template <int T> struct GemvShape {
  static constexpr int LB = (T <= 2) ? 16 : (T <= 4 ? 8 : 4);   // packed bytes per lane per row
  static constexpr int CK = 2 * LB;                              // k values per lane
  static constexpr int NWD = LB / 4;                             // 32-bit words per lane per row
  static constexpr int RW = (T == 1) ? 4 : (T == 2 ? 2 : 1);     // rows per warp per chunk
  static constexpr int V = RW * T;                               // partial sums per lane
  static constexpr int VP = V <= 1 ? 1 : V <= 2 ? 2 : V <= 4 ? 4 : 8;
  static constexpr int LOGV = VP == 1 ? 0 : VP == 2 ? 1 : VP == 4 ? 2 : 3;
};

template <int T, bool ASYM>
__global__ void __launch_bounds__(kGemvMaxThreads) q4_gemv_kernel(const GemvParams p) {
  using Sh = GemvShape<T>;
  constexpr int LB = Sh::LB, CK = Sh::CK, NWD = Sh::NWD, RW = Sh::RW;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  float* red = reinterpret_cast<float*>(smem + kRedOffset);
  uint8_t* stages = smem + p.stage_base;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncons = p.KS * p.RG;
  const int rb = (int)((long long)p.N * blockIdx.x / gridDim.x);
  const int re = (int)((long long)p.N * (blockIdx.x + 1) / gridDim.x);
  const int nchunks = (re - rb + p.R - 1) / p.R;
  const int KH = p.K >> 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.nst; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], ncons); }
    fence_mbar_init();
  }
  __syncthreads();
  // Weights do not depend on the previous kernel: let the next kernel in the
  // stream launch now so that it can start streaming its own weights.
  griddep_launch_dependents();

  if (warp == ncons) {
    // ---------------- producer ----------------
    if (lane == 0) {
      for (int c = 0; c < nchunks; ++c) {
        const int st = c % p.nst, use = c / p.nst;
        if (use > 0 && !mbar_wait(&empty[st], (use - 1) & 1)) break;
        const int r0 = rb + c * p.R;
        const int rows = min(p.R, re - r0);
        uint8_t* buf = stages + (size_t)st * p.stage_bytes;
        const uint32_t wbytes = (uint32_t)rows * KH;           // K % 32 == 0 -> multiple of 16
        // scales/zeros: copy from the 16-byte boundary at or below the chunk start
        const uintptr_t s_src = reinterpret_cast<uintptr_t>(p.S + (size_t)r0 * p.G);
        const uint32_t s_pre = (uint32_t)(s_src & 15);
        const uint32_t s_bytes = (s_pre + (uint32_t)rows * p.G * 4) & ~15u;
        uint32_t tx = wbytes + s_bytes;
        if (ASYM) tx += s_bytes;  // zeros share the scales' geometry
        mbar_arrive_expect_tx(&full[st], tx);
        bulk_g2s(buf, p.W + (size_t)r0 * KH, wbytes, &full[st]);
        if (s_bytes) {
          bulk_g2s(buf + p.s_off, reinterpret_cast<const void*>(s_src - s_pre), s_bytes, &full[st]);
          if (ASYM)
            bulk_g2s(buf + p.z_off,
                     reinterpret_cast<const uint8_t*>(p.Z + (size_t)r0 * p.G) - s_pre, s_bytes,
                     &full[st]);
        }
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  const int s = warp % p.KS, rg = warp / p.KS;
  const int kl = s * 32 * CK + lane * CK;
  const bool active = kl < p.K;
  const int gl = active ? kl / p.gs : 0;

  // The activations are produced by the previous kernel: wait for it.
  griddep_wait();
  float2 xr[T][CK / 2];
  float xs[T];
#pragma unroll
  for (int t = 0; t < T; ++t) {
    xs[t] = 0.f;
#pragma unroll
    for (int i = 0; i < CK; i += 8) {
      float v[8];
      if (active) load_x8(p.X, (size_t)t * p.K + kl + i, p.xdt, v);
      else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) xr[t][i / 2 + j] = make_float2(v[2 * j], v[2 * j + 1]);
      if (ASYM) {
#pragma unroll
        for (int j = 0; j < 8; ++j) xs[t] += v[j];
      }
    }
  }

  const int nthr = ncons * 32;
  bool ok_wait = true;
  for (int c = 0; c < nchunks; ++c) {
    const int st = c % p.nst, use = c / p.nst;
    const int r0 = rb + c * p.R;
    const int rows = min(p.R, re - r0);
    if (ok_wait) ok_wait = mbar_wait(&full[st], use & 1);
    const uint8_t* buf = stages + (size_t)st * p.stage_bytes;
    const uintptr_t s_src = reinterpret_cast<uintptr_t>(p.S + (size_t)r0 * p.G);
    const int s_pre = (int)(s_src & 15) >> 2;
    const int s_cnt = (int)(((s_src & 15) + (uint32_t)rows * p.G * 4) & ~15u) >> 2;
    const float* ss = reinterpret_cast<const float*>(buf + p.s_off);
    const float* zz = reinterpret_cast<const float*>(buf + p.z_off);

    uint32_t wv[RW][NWD];
    float sc[RW], zp[RW];
#pragma unroll
    for (int rr = 0; rr < RW; ++rr) {
      const int lr = rg * RW + rr;
      const bool ok = active && lr < rows && ok_wait;
      if (ok) {
        const uint8_t* src = buf + (size_t)lr * KH + s * 32 * LB + lane * LB;
        if constexpr (NWD == 4) {
          const uint4 v = *reinterpret_cast<const uint4*>(src);
          wv[rr][0] = v.x; wv[rr][1] = v.y; wv[rr][2] = v.z; wv[rr][3] = v.w;
        } else if constexpr (NWD == 2) {
          const uint2 v = *reinterpret_cast<const uint2*>(src);
          wv[rr][0] = v.x; wv[rr][1] = v.y;
        } else {
          wv[rr][0] = *reinterpret_cast<const uint32_t*>(src);
        }
        const int si = s_pre + lr * p.G + gl;
        if (si < s_cnt) {
          sc[rr] = ss[si];
          zp[rr] = ASYM ? zz[si] : 0.f;
        } else {
          sc[rr] = __ldg(p.S + (size_t)(r0 + lr) * p.G + gl);
          zp[rr] = ASYM ? __ldg(p.Z + (size_t)(r0 + lr) * p.G + gl) : 0.f;
        }
      } else {
#pragma unroll
        for (int q = 0; q < NWD; ++q) wv[rr][q] = 0u;  // contributes 0 (scale is 0)
        sc[rr] = 0.f;
        zp[rr] = 0.f;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);

    float part[Sh::VP];
#pragma unroll
    for (int v = 0; v < Sh::VP; ++v) part[v] = 0.f;
#pragma unroll
    for (int rr = 0; rr < RW; ++rr) {
#pragma unroll
      for (int t = 0; t < T; ++t) {
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int q = 0; q < NWD; ++q) acc = dot8<ASYM>(wv[rr][q], &xr[t][4 * q], acc);
        float d = acc.x + acc.y;
        if (ASYM) d = fmaf(-zp[rr], xs[t], d);
        part[rr * T + t] = d * sc[rr];
      }
    }

    // Butterfly reduce-scatter of VP values over 32 lanes.
#pragma unroll
    for (int st2 = 0, n = Sh::VP; st2 < Sh::LOGV; ++st2, n >>= 1) {
      const int off = 16 >> st2;
      const bool upper = (lane & off) != 0;
#pragma unroll
      for (int i = 0; i < n / 2; ++i) {
        const float send = upper ? part[i] : part[i + n / 2];
        const float keep = upper ? part[i + n / 2] : part[i];
        part[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
      }
    }
#pragma unroll
    for (int off = 16 >> Sh::LOGV; off >= 1; off >>= 1)
      part[0] += __shfl_xor_sync(0xffffffffu, part[0], off);

    float* rbuf = red + (c & 1) * (p.KS * T * p.R);
    if ((lane & ((32 >> Sh::LOGV) - 1)) == 0) {
      int vi = 0;
#pragma unroll
      for (int j = 0; j < Sh::LOGV; ++j) vi |= ((lane >> (4 - j)) & 1) << (Sh::LOGV - 1 - j);
      if (vi < Sh::V) {
        const int rr = vi / T, t = vi % T;
        rbuf[(s * T + t) * p.R + rg * RW + rr] = part[0];
      }
    }
    named_barrier_sync(1, nthr);
    for (int idx = threadIdx.x; idx < rows * T; idx += nthr) {
      const int t = idx / rows, r = idx - t * rows;
      float acc = 0.f;
      for (int k = 0; k < p.KS; ++k) acc += rbuf[(k * T + t) * p.R + r];
      if (p.bias) acc += __ldg(p.bias + r0 + r);
      store_y(p.Y, (size_t)t * p.N + r0 + r, acc, p.ydt);
    }
  }
}

// ---------------------------------------------------------------------------
// Generic GEMV (any even group size): one warp per output row, dequantize
// each weight with the reference's formula and accumulate in fp32.
// ---------------------------------------------------------------------------
__global__ void q4_gemv_generic_kernel(const GemvParams p, int T) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  griddep_launch_dependents();
  griddep_wait();
  if (warp >= p.N) return;
  const int KH = p.K >> 1;
  const uint8_t* w = p.W + (size_t)warp * KH;
  for (int t = 0; t < T; ++t) {
    float acc = 0.f;
    for (int j = lane; j < KH; j += 32) {
      const uint8_t b = w[j];
      const int g = (2 * j) / p.gs;
      const float s = __ldg(p.S + (size_t)warp * p.G + g);
      int lo = b & 15, hi = b >> 4;
      float qlo, qhi;
      if (p.Z) {
        const float z = __ldg(p.Z + (size_t)warp * p.G + g);
        qlo = (float)lo - z; qhi = (float)hi - z;
      } else {
        qlo = (float)(lo < 8 ? lo : lo - 16); qhi = (float)(hi < 8 ? hi : hi - 16);
      }
      acc = fmaf(qlo * s, load_x(p.X, (size_t)t * p.K + 2 * j, p.xdt), acc);
      acc = fmaf(qhi * s, load_x(p.X, (size_t)t * p.K + 2 * j + 1, p.xdt), acc);
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) {
      if (p.bias) acc += __ldg(p.bias + warp);
      store_y(p.Y, (size_t)t * p.N + warp, acc, p.ydt);
    }
  }
}

// ---------------------------------------------------------------------------
// Dequant: one thread per packed byte -> two outputs.  fp32 result uses the
// reference's exact operation order: q*s, or (q - z)*s.
// ---------------------------------------------------------------------------
__global__ void q4_dequant_kernel(const uint8_t* __restrict__ W, const float* __restrict__ S,
                                  const float* __restrict__ Z, void* out, int odt, int N,
                                  int K, int gs) {
  const size_t nbytes = (size_t)N * (K / 2);
  const int G = K / gs;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nbytes;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t row = i / (K / 2);
    const int k = (int)(i - row * (K / 2)) * 2;
    const uint8_t b = W[i];
    const int g0 = k / gs, g1 = (k + 1) / gs;
    int lo = b & 15, hi = b >> 4;
    float v0, v1;
    if (Z) {
      v0 = __fmul_rn(__fsub_rn((float)lo, Z[row * G + g0]), S[row * G + g0]);
      v1 = __fmul_rn(__fsub_rn((float)hi, Z[row * G + g1]), S[row * G + g1]);
    } else {
      v0 = __fmul_rn((float)(lo < 8 ? lo : lo - 16), S[row * G + g0]);
      v1 = __fmul_rn((float)(hi < 8 ? hi : hi - 16), S[row * G + g1]);
    }
    const size_t o = row * K + k;
    store_y(out, o, v0, odt);
    store_y(out, o + 1, v1, odt);
  }
}

// ---------------------------------------------------------------------------
// RTN quantize + pack, one warp per (row, group).  Matches
// siliconfer/quant/primitives.py:24-51 / 82-114 bit for bit: IEEE division,
// round-half-to-even, identical clip order.
// ---------------------------------------------------------------------------
__global__ void q4_quantize_pack_kernel(const float* __restrict__ W, uint8_t* __restrict__ P,
                                        float* __restrict__ S, float* __restrict__ Z, int N,
                                        int K, int gs) {
  const int G = K / gs;
  const long long task = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (task >= (long long)N * G) return;
  const int row = (int)(task / G), g = (int)(task % G);
  const float* w = W + (size_t)row * K + (size_t)g * gs;
  float mx = -INFINITY, mn = INFINITY, amax = 0.f;
  for (int i = lane; i < gs; i += 32) {
    const float v = w[i];
    mx = fmaxf(mx, v); mn = fminf(mn, v); amax = fmaxf(amax, fabsf(v));
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  }
  float scale, safe, zero = 0.f;
  if (Z) {
    scale = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
    safe = scale == 0.f ? 1.0f : scale;
    zero = fminf(fmaxf(rintf(__fdiv_rn(-mn, safe)), 0.f), 15.f);
  } else {
    scale = __fdiv_rn(amax, 7.0f);
    safe = scale == 0.f ? 1.0f : scale;
  }
  if (lane == 0) {
    S[(size_t)row * G + g] = scale;
    if (Z) Z[(size_t)row * G + g] = zero;
  }
  uint8_t* out = P + (size_t)row * (K / 2) + (size_t)g * (gs / 2);
  for (int j = lane; j < gs / 2; j += 32) {
    int q[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float r = rintf(__fdiv_rn(w[2 * j + h], safe));
      if (Z) q[h] = (int)fminf(fmaxf(__fadd_rn(r, zero), 0.f), 15.f);
      else q[h] = (int)fminf(fmaxf(r, -8.f), 7.f) & 15;
    }
    out[j] = (uint8_t)(q[0] | (q[1] << 4));
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
template <int T, bool ASYM>
cudaError_t launch_gemv_t(const GemvParams& p, int grid, int threads, size_t smem,
                          cudaStream_t stream, bool pdl) {
  auto* fn = q4_gemv_kernel<T, ASYM>;
  static thread_local int configured_dev = -1;
  static thread_local size_t configured_smem = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev || configured_smem < smem) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
    configured_smem = smem;
  }
  return launch_kernel(fn, grid, threads, smem, stream, pdl, p);
}

template <bool ASYM>
cudaError_t launch_gemv(int T, const GemvParams& p, int grid, int threads, size_t smem,
                        cudaStream_t stream, bool pdl) {
  switch (T) {
    case 1: return launch_gemv_t<1, ASYM>(p, grid, threads, smem, stream, pdl);
    case 2: return launch_gemv_t<2, ASYM>(p, grid, threads, smem, stream, pdl);
    case 3: return launch_gemv_t<3, ASYM>(p, grid, threads, smem, stream, pdl);
    case 4: return launch_gemv_t<4, ASYM>(p, grid, threads, smem, stream, pdl);
    case 5: return launch_gemv_t<5, ASYM>(p, grid, threads, smem, stream, pdl);
    case 6: return launch_gemv_t<6, ASYM>(p, grid, threads, smem, stream, pdl);
    case 7: return launch_gemv_t<7, ASYM>(p, grid, threads, smem, stream, pdl);
    default: return launch_gemv_t<8, ASYM>(p, grid, threads, smem, stream, pdl);
  }
}

static int lane_bytes(int T) { return T <= 2 ? 16 : (T <= 4 ? 8 : 4); }
static int rows_per_warp(int T) { return T == 1 ? 4 : (T == 2 ? 2 : 1); }

// Plan the fast GEMV; returns false when the shape needs the generic kernel.
bool plan_gemv(int N, int K, int T, int gs, bool asym, GemvPlan& pl) {
  if (T < 1 || T > kMaxGemvT || K % 32 || gs % 32 || N < 1) return false;
  const DeviceInfo& di = device_info();
  const int CK = 2 * lane_bytes(T);
  const int KS = (K + 32 * CK - 1) / (32 * CK);
  if (KS > kGemvMaxThreads / 32 - 1) return false;
  const int RW = rows_per_warp(T);
  const int grid = N < di.sms ? N : di.sms;
  const int rows_cta = (N + grid - 1) / grid;
  int rg_max = (kGemvMaxThreads / 32 - 1) / KS;
  int rg_target = (8 + KS - 1) / KS;            // aim for >= 8 consumer warps
  int rg_need = (rows_cta + RW - 1) / RW;       // no more row groups than rows
  int RG = rg_target < rg_need ? rg_target : rg_need;
  if (RG > rg_max) RG = rg_max;
  if (RG < 1) RG = 1;
  const int R = RG * RW;
  const int G = K / gs;
  const size_t wb = (size_t)R * (K / 2);
  const size_t sb = ((size_t)R * G * 4 + 16 + 15) & ~(size_t)15;
  size_t stage = ((wb + 127) & ~(size_t)127) + sb + (asym ? sb : 0);
  stage = (stage + 127) & ~(size_t)127;
  const size_t red_bytes = (size_t)2 * KS * T * R * 4;
  const size_t base = ((size_t)kRedOffset + red_bytes + 127) & ~(size_t)127;
  const int nchunks = (rows_cta + R - 1) / R;
  size_t budget = 112 * 1024;
  if (base + 2 * stage > budget) budget = (size_t)di.smem_optin;
  long long S = (long long)((budget - base) / stage);
  if (S < 1) return false;
  if (S > kMaxStages) S = kMaxStages;
  if (S > nchunks) S = nchunks;
  if (S < 1) S = 1;
  pl.KS = KS; pl.RG = RG; pl.R = R; pl.S = (int)S;
  pl.grid = grid;
  pl.threads = (KS * RG + 1) * 32;
  pl.stage_bytes = stage;
  pl.s_off = (wb + 127) & ~(size_t)127;
  pl.z_off = pl.s_off + sb;
  pl.stage_base = base;
  pl.smem = base + (size_t)S * stage;
  return pl.threads <= kGemvMaxThreads;
}

int run_linear(const uint8_t* W, const float* S, const float* Z, const float* bias,
               const void* X, int xdt, void* Y, int ydt, int N, int K, int T, int gs,
               int flags, cudaStream_t stream, bool force_generic) {
  if (!W || !S || !X || !Y) return fail(SF_ERR_NULL, "null pointer argument");
  if (xdt < 0 || xdt > 2 || ydt < 0 || ydt > 2) return fail(SF_ERR_DTYPE, "unknown dtype code");
  if (N < 0 || K <= 0 || T < 0) return fail(SF_ERR_SHAPE, "invalid N/K/T");
  if (gs <= 0 || gs % 2) return fail(SF_ERR_SHAPE, "group_size must be a positive even number");
  if (K % 2) return fail(SF_ERR_SHAPE, "in_features must be even");
  if (K % gs) return fail(SF_ERR_SHAPE, "in_features must be divisible by group_size");
  if (N == 0 || T == 0) return SF_OK;
  const bool pdl = (flags & SF_FLAG_PDL) != 0;
  const bool aligned = ((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(S) |
                         reinterpret_cast<uintptr_t>(Z) | reinterpret_cast<uintptr_t>(X)) & 15) == 0;
  GemvParams p{};
  p.W = W; p.S = S; p.Z = Z; p.bias = bias; p.X = X; p.Y = Y;
  p.N = N; p.K = K; p.G = K / gs; p.gs = gs; p.xdt = xdt; p.ydt = ydt;
  const size_t xe = xdt == SF_F32 ? 4 : 2, ye = ydt == SF_F32 ? 4 : 2;

  if (!force_generic && T > kMaxGemvT) {
    int rc = run_tc_gemm(W, S, Z, bias, X, xdt, Y, ydt, N, K, T, gs, flags, stream);
    if (rc != SF_ERR_UNSUPPORTED) return rc;
  }
  if (!force_generic && aligned) {
    for (int t0 = 0; t0 < T; t0 += kMaxGemvT) {
      const int tc = T - t0 < kMaxGemvT ? T - t0 : kMaxGemvT;
      GemvPlan pl;
      if (!plan_gemv(N, K, tc, gs, Z != nullptr, pl)) break;
      GemvParams q = p;
      q.X = static_cast<const uint8_t*>(X) + (size_t)t0 * K * xe;
      q.Y = static_cast<uint8_t*>(Y) + (size_t)t0 * N * ye;
      q.KS = pl.KS; q.RG = pl.RG; q.R = pl.R; q.nst = pl.S;
      q.stage_bytes = (uint32_t)pl.stage_bytes; q.s_off = (uint32_t)pl.s_off;
      q.z_off = (uint32_t)pl.z_off; q.stage_base = (uint32_t)pl.stage_base;
      cudaError_t e = Z ? launch_gemv<true>(tc, q, pl.grid, pl.threads, pl.smem, stream, pdl)
                        : launch_gemv<false>(tc, q, pl.grid, pl.threads, pl.smem, stream, pdl);
      if (e != cudaSuccess) return cuda_fail(e, "q4_gemv_kernel launch");
      g_launches.fetch_add(1, std::memory_order_relaxed);
      if (t0 + tc == T) return SF_OK;
    }
  }
  // Generic path: every legal shape.
  const int threads = 256;
  const int blocks = (int)(((long long)N * 32 + threads - 1) / threads);
  cudaError_t e = launch_kernel(q4_gemv_generic_kernel, blocks, threads, 0, stream, pdl, p, T);
  if (e != cudaSuccess) return cuda_fail(e, "q4_gemv_generic_kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return SF_OK;
}

}  // namespace sf

// ===========================================================================
// C ABI
// ===========================================================================
using namespace sf;

extern "C" {

const char* sf_status_string(int status) {
  switch (status) {
    case SF_OK: return "ok";
    case SF_ERR_NULL: return "null pointer";
    case SF_ERR_SHAPE: return "shape mismatch";
    case SF_ERR_DTYPE: return "bad dtype";
    case SF_ERR_ALIGN: return "misaligned pointer";
    case SF_ERR_CUDA: return "CUDA error";
    case SF_ERR_UNSUPPORTED: return "unsupported";
    case SF_ERR_TIMEOUT: return "device wait timed out";
    case SF_ERR_COMM: return "peer exchange failed";
    default: return "unknown status";
  }
}

const char* sf_last_error(void) { return g_last_error; }
int sf_version(void) { return 10000; }
long long sf_q4_launch_count(void) { return g_launches.load(); }

int sf_q4_linear(const uint8_t* W, const float* scales, const float* zeros, const float* bias,
                 const void* X, int x_dtype, void* Y, int y_dtype, int N, int K, int T,
                 int group_size, int flags, void* stream) {
  return run_linear(W, scales, zeros, bias, X, x_dtype, Y, y_dtype, N, K, T, group_size, flags,
                    static_cast<cudaStream_t>(stream), false);
}

int sf_q4_gemv_sym(const uint8_t* W, const float* scales, const float* x, float* y, int out_f,
                   int in_f, int group_size, void* stream) {
  return run_linear(W, scales, nullptr, nullptr, x, SF_F32, y, SF_F32, out_f, in_f, 1,
                    group_size, 0, static_cast<cudaStream_t>(stream), false);
}

int sf_q4_gemv_scalar(const uint8_t* W, const float* scales, const float* x, float* y,
                      int out_f, int in_f, int group_size, void* stream) {
  return run_linear(W, scales, nullptr, nullptr, x, SF_F32, y, SF_F32, out_f, in_f, 1,
                    group_size, 0, static_cast<cudaStream_t>(stream), true);
}

int sf_q4_gemv_asym(const uint8_t* W, const float* scales, const float* zeros, const float* x,
                    float* y, int out_f, int in_f, int group_size, void* stream) {
  if (!zeros) return fail(SF_ERR_NULL, "zeros must not be NULL for the asymmetric kernel");
  return run_linear(W, scales, zeros, nullptr, x, SF_F32, y, SF_F32, out_f, in_f, 1,
                    group_size, 0, static_cast<cudaStream_t>(stream), false);
}

int sf_q4_gemm_sym(const uint8_t* W, const float* scales, const float* X, float* Y, int out_f,
                   int in_f, int T, int group_size, void* stream) {
  return run_linear(W, scales, nullptr, nullptr, X, SF_F32, Y, SF_F32, out_f, in_f, T,
                    group_size, 0, static_cast<cudaStream_t>(stream), false);
}

int sf_q4_gemm_asym(const uint8_t* W, const float* scales, const float* zeros, const float* X,
                    float* Y, int out_f, int in_f, int T, int group_size, void* stream) {
  if (!zeros) return fail(SF_ERR_NULL, "zeros must not be NULL for the asymmetric kernel");
  return run_linear(W, scales, zeros, nullptr, X, SF_F32, Y, SF_F32, out_f, in_f, T,
                    group_size, 0, static_cast<cudaStream_t>(stream), false);
}

int sf_q4_dequant(const uint8_t* W, const float* scales, const float* zeros, void* out,
                  int out_dtype, int N, int K, int group_size, void* stream) {
  if (!W || !scales || !out) return fail(SF_ERR_NULL, "null pointer argument");
  if (out_dtype < 0 || out_dtype > 2) return fail(SF_ERR_DTYPE, "unknown dtype code");
  if (N < 0 || K <= 0 || K % 2 || group_size <= 0 || group_size % 2 || K % group_size)
    return fail(SF_ERR_SHAPE, "in_features must be divisible by group_size");
  if (N == 0) return SF_OK;
  const size_t nbytes = (size_t)N * (K / 2);
  const int threads = 256;
  long long blocks = (long long)((nbytes + threads - 1) / threads);
  if (blocks > 148 * 64) blocks = 148 * 64;
  q4_dequant_kernel<<<(int)blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      W, scales, zeros, out, out_dtype, N, K, group_size);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "q4_dequant_kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return SF_OK;
}

int sf_q4_quantize_pack(const float* W, uint8_t* packed, float* scales, float* zeros, int N,
                        int K, int group_size, void* stream) {
  if (!W || !packed || !scales) return fail(SF_ERR_NULL, "null pointer argument");
  if (N < 0 || K <= 0 || K % 2 || group_size <= 0 || group_size % 2 || K % group_size)
    return fail(SF_ERR_SHAPE, "cols=%d not divisible by group_size=%d", K, group_size);
  if (N == 0) return SF_OK;
  const long long tasks = (long long)N * (K / group_size);
  const int threads = 256;
  const long long blocks = (tasks * 32 + threads - 1) / threads;
  if (blocks > 0x7fffffffLL) return fail(SF_ERR_SHAPE, "matrix too large");
  q4_quantize_pack_kernel<<<(int)blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      W, packed, scales, zeros, N, K, group_size);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "q4_quantize_pack_kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return SF_OK;
}

int sf_q4_check_device_error(void) {
  const unsigned int a = take_dev_error_gemv(), b = take_dev_error_tc();
  if (a == 0xffffffffu || b == 0xffffffffu)
    return fail(SF_ERR_CUDA, "reading the device error word failed");
  if (a | b) return fail(SF_ERR_TIMEOUT, "a device-side wait expired (code %u)", a | b);
  return SF_OK;
}

}  // extern "C"
