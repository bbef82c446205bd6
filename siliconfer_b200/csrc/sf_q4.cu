// sf_q4.cu -- B200 (sm_100a) kernels behind the siliconfer Q4Linear C ABI.
//
// Kernels in this file:
//   (the decode GEMV, q4_tile_kernel, lives in sf_q4_tile.cu)
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
#include <cstdlib>
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
    // Decode GEMV as independent warp units; T above kMaxGemvT that the GEMM
    // path declined is cut into chunks of kMaxGemvT tokens (weights re-read).
    // Up to 16 tokens: one launch (9-16 tokens need group size >= 64 and use
    // the two-digit activation grid).  17-47 tokens: chunks of 8 on the
    // three-digit grid, which keeps the reference's elementwise tolerances.
    int rc = SF_OK;
    const int tmax = (T <= kMaxGemvT && gs % 64 == 0) ? kMaxGemvT : 8;
    for (int t0 = 0; t0 < T && rc == SF_OK; t0 += tmax) {
      const int tc = T - t0 < tmax ? T - t0 : tmax;
      rc = run_tile_linear(W, S, Z, bias, static_cast<const uint8_t*>(X) + (size_t)t0 * K * xe, xdt,
                           static_cast<uint8_t*>(Y) + (size_t)t0 * N * ye, ydt, N, K, tc, gs, stream);
    }
    if (rc != SF_ERR_UNSUPPORTED) return rc;
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
    case SF_ERR_CAPTURE: return "scratch must grow during stream capture";
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
  const unsigned int a = take_dev_error_gemv(), b = take_dev_error_tc(),
                     c = take_dev_error_tile() | take_dev_error_tp();
  if (a == 0xffffffffu || b == 0xffffffffu || c == 0xffffffffu)
    return fail(SF_ERR_CUDA, "reading the device error word failed");
  if ((a | b | c) & kErrPoisoned)
    return fail(SF_ERR_COMM,
                "a tensor-parallel exchange met a poisoned communicator (a rank's bounded wait expired in an "
                "earlier call; create the communicator again) (code %u)", a | b | c);
  if (a | b | c) return fail(SF_ERR_TIMEOUT, "a device-side wait expired (code %u)", a | b | c);
  return SF_OK;
}

}  // extern "C"
