// sf_q4_tile.cu -- decode GEMV (T <= 8 tokens) as independent warp work units
// on the sm_100a tensor cores, exact integer arithmetic.
//
// Reference semantics (siliconfer/kernels/neon/q4_gemv.cpp:37-140, 145-238;
// siliconfer/kernels/neon/__init__.py:88-124): per output row i and group g,
//   sym : y += s[i,g] * sum_k sext(q[i,k]) * x[k]
//   asym: y += s[i,g] * (sum_k q[i,k] * x[k] - z[i,g] * sum_k x[k])
//
// Arithmetic (unchanged from the reference's algebra, exact where it can be):
//  * weights are UNSIGNED int8 A operands; symmetric nibbles are flipped
//    (u ^ 8 = q + 8) by the LOP3 that masks them, so both layouts become
//    s * (sum u*x - zeff * sum x) with zeff = 8 (sym) or z (asym);
//  * activations: per (token, group) x_fix = rint(x * 2^(22-E)), E the binary
//    exponent of the group's max |x|, split into three signed int8 digits
//    (x_fix = d0 + 256 d1 + 65536 d2) by a pre-pass (or, for a task that
//    depends on earlier ones, by the first warp that reaches it);
//  * mma.sync m16n8k32 u8 x s8 -> s32 sums u*d exactly; one fp32 epilogue per
//    (row, group, token) recombines the digits, removes zeff * sum(x_fix) and
//    applies s * 2^(E-22).
//
// Work decomposition (the B200 part):
//  * A launch owns a list of tasks (GEMVs).  Each task is cut into units of
//    32 rows x one k-range; all units of all tasks form one global sequence.
//  * Every warp is independent: warp w takes units w, w + W, w + 2W, ...
//    (W = warps in the grid).  There is no block-level synchronisation at all:
//    a unit's operands (packed weights, activation digits, scales, zeros) are
//    streamed by the warp's own cp.async ring of D stages, each lane copying
//    exactly the bytes it feeds to its own MMA fragments, so a lane only waits
//    for its own copies.  Units of consecutive tasks run concurrently on
//    different warps, which hides every per-task latency.
//  * Dependencies (a task that reads what earlier tasks wrote) are per-task
//    completion counters: a warp starting a unit of such a task waits until
//    every unit of the tasks it depends on has been published.  All warps are
//    resident (cooperative launch, grid <= SMs) and take units in increasing
//    order, so a wait never blocks a unit it depends on.  Waits are bounded.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <cstdlib>
#include <map>
#include <mutex>
#include <vector>

#include "sf_q4.h"
#include "sf_q4_internal.h"

namespace sf {
extern std::atomic<long long> g_launches;

SF_DEFINE_ERROR_READER(take_dev_error_tile)

namespace {

constexpr int kD = 4;                  // cp.async ring depth per warp (segments)
constexpr int kTileMaxThreads = 512;
// More than 4 tokens doubles the accumulators; those launches hold at most 8
// warps (their stages are larger) and get 255 registers per thread instead.
__host__ __device__ constexpr int tile_max_threads(int T) { return T > 4 ? 256 : kTileMaxThreads; }
constexpr int kUnitRows = 32;          // rows per unit (two m16 tiles)

// One GEMV of a launch.  16-byte aligned: copied and indexed in device memory.
struct alignas(16) TileTask {
  const uint8_t* W;
  const float* S;
  const float* Z;
  const float* bias;
  const void* X;
  void* Y;
  uint8_t* xd;        // activation digits [T][3][K], then gsc [T][G], xsum [T][G]
  float* part;        // k-split partial sums [ksplit][T][N] (ksplit > 1) or null
  long long ubase;    // index of the task's first unit in the launch
  int N, K, G, lg2gs, xdt, ydt;
  int ntile, ksplit, kper;   // 32-row tiles, k-splits, k per split (whole groups)
  int xpre;                  // digits were written by the pre-pass
  int wait_from, wait_to;    // tasks [wait_from, wait_to) finish before this one reads X
};

struct TileLaunch {
  const TileTask* tasks;  // device table, or null: use `single`
  TileTask single;
  int ntasks;
  long long total;        // units in the launch
  unsigned int* done;     // per task: units finished (zeroed before each launch) or null
  unsigned int* xflag;    // per task: 0 digits missing, 1 being written, 2 ready
};

__device__ __forceinline__ const TileTask& tile_task(const TileLaunch& L, int i) {
  return L.tasks ? L.tasks[i] : L.single;
}

__device__ __forceinline__ void ld_x8(const void* x, size_t idx, int dt, float* v) {
  if (dt == SF_F32) {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + idx);
    const float4 a = __ldcg(p), b = __ldcg(p + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 u = __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(x) + idx));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f;
      if (dt == SF_F16) f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      else f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}

__device__ __forceinline__ void st_y(void* y, size_t idx, float v, int dt) {
  if (dt == SF_F32) reinterpret_cast<float*>(y)[idx] = v;
  else if (dt == SF_F16) reinterpret_cast<__half*>(y)[idx] = __float2half_rn(v);
  else reinterpret_cast<__nv_bfloat16*>(y)[idx] = __float2bfloat16_rn(v);
}

// D += A(u8, 16x32) * B(s8, 32x8), s32 accumulate (no side effects: not volatile).
__device__ __forceinline__ void imma(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                     uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <bool ASYM>
__device__ __forceinline__ uint32_t nib_lo(uint32_t w) {
  return (w & 0x0F0F0F0Fu) ^ (ASYM ? 0u : 0x08080808u);
}
template <bool ASYM>
__device__ __forceinline__ uint32_t nib_hi(uint32_t w) {
  return ((w >> 4) & 0x0F0F0F0Fu) ^ (ASYM ? 0u : 0x08080808u);
}

// Low bytes of d[0..7] in B-operand order: word 0 = k offsets {0,2,4,6},
// word 1 = {1,3,5,7} (matching the low / high nibbles of the A operand).
__device__ __forceinline__ uint2 pack_digits(const int* d) {
  uint2 r;
  r.x = (uint32_t)(d[0] & 255) | ((uint32_t)(d[2] & 255) << 8) | ((uint32_t)(d[4] & 255) << 16) |
        ((uint32_t)(d[6] & 255) << 24);
  r.y = (uint32_t)(d[1] & 255) | ((uint32_t)(d[3] & 255) << 8) | ((uint32_t)(d[5] & 255) << 16) |
        ((uint32_t)(d[7] & 255) << 24);
  return r;
}

// Fixed-point digit split of 8 activations of one lane.  Lanes [lpg-aligned
// blocks] form one quantization group.  Writes the three digit words and
// returns (through gsc_out / sum_out) the group scale and sum.
__device__ __forceinline__ void digits8(const float* v, int lpg, uint2* dig, float& gsc_out,
                                        int& sum_out) {
  float m = 0.f;
  int bad = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    m = fmaxf(m, fabsf(v[j]));
    bad |= !(fabsf(v[j]) <= 3.402823466e38f);
  }
  for (int off = 1; off < lpg; off <<= 1) {
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    bad |= __shfl_xor_sync(0xffffffffu, bad, off);
  }
  // binary exponent field of the group max; groups below 2^-105 are zero
  const int be = (int)(__float_as_uint(m) >> 23);
  const bool zero = bad || be < 22;
  const float scl = zero ? 0.f : __uint_as_float((uint32_t)(275 - be) << 23);   // 2^(22-E)
  int d[3][8];
  int s = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int xf = __float2int_rn(v[j] * scl);
    s += xf;
    const int d0 = (xf << 24) >> 24;
    const int r1 = (xf - d0) >> 8;
    const int d1 = (r1 << 24) >> 24;
    d[0][j] = d0;
    d[1][j] = d1;
    d[2][j] = (r1 - d1) >> 8;
  }
  for (int off = 1; off < lpg; off <<= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  dig[0] = pack_digits(d[0]);
  dig[1] = pack_digits(d[1]);
  dig[2] = pack_digits(d[2]);
  gsc_out = bad ? __int_as_float(0x7fc00000)
                : (zero ? 0.f : __uint_as_float((uint32_t)(be - 21) << 23));   // 2^(E-22)
  sum_out = s;
}

// Activation digits of one task, written by the threads [tid0, tid0 + nthr)
// (a whole CTA in the pre-pass, one warp inside the GEMV kernel).
template <int T>
__device__ __forceinline__ void write_digits(const TileTask& p, int tid, int nthr) {
  const int lane = tid & 31;
  const int octs = p.K >> 3, total = T * octs;
  const int lpg = 1 << (p.lg2gs - 3);
  float* gsc = reinterpret_cast<float*>(p.xd + (size_t)3 * T * p.K);
  float* xsm = gsc + T * p.G;
  for (int ob = tid - lane; ob < total; ob += nthr) {
    const int o = ob + lane;
    const bool ok = o < total;
    const int tok = ok ? o / octs : 0;
    const int oo = ok ? o - tok * octs : 0;
    float v[8];
    if (ok) ld_x8(p.X, (size_t)tok * p.K + (size_t)oo * 8, p.xdt, v);
    else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = 0.f;
    }
    uint2 dig[3];
    float gs_;
    int s;
    digits8(v, lpg, dig, gs_, s);
    if (ok) {
#pragma unroll
      for (int dg = 0; dg < 3; ++dg)
        *reinterpret_cast<uint2*>(p.xd + (size_t)(tok * 3 + dg) * p.K + (size_t)oo * 8) = dig[dg];
      if ((lane & (lpg - 1)) == 0) {
        const int gi = (oo * 8) >> p.lg2gs;
        gsc[tok * p.G + gi] = gs_;
        xsm[tok * p.G + gi] = (float)s;
      }
    }
  }
}

// ---- cp.async helpers (each lane copies only what it later reads itself) ----
template <int BYTES>
__device__ __forceinline__ void cpa(uint32_t dst, const void* src) {
  if constexpr (BYTES == 16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(dst), "l"(src), "n"(BYTES)
                 : "memory");
}
__device__ __forceinline__ void cpa_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cpa_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}

template <int NB>   // NB bytes from shared memory into NB/4 words
__device__ __forceinline__ void lds_n(uint32_t a, uint32_t* w) {
  if constexpr (NB == 32) {
    const uint4 u = lds128(a), v = lds128(a + 16);
    w[0] = u.x; w[1] = u.y; w[2] = u.z; w[3] = u.w; w[4] = v.x; w[5] = v.y; w[6] = v.z; w[7] = v.w;
  } else if constexpr (NB == 16) {
    const uint4 u = lds128(a);
    w[0] = u.x; w[1] = u.y; w[2] = u.z; w[3] = u.w;
  } else if constexpr (NB == 8) {
    const uint2 u = lds64(a);
    w[0] = u.x; w[1] = u.y;
  } else {
    w[0] = lds32(a);
  }
}

// Bounded spin on a global counter (one thread).  false on timeout.
__device__ __forceinline__ bool spin_geq(const unsigned int* p, unsigned int target, unsigned int code) {
  const long long t0 = clock64();
  while (true) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    if (v >= target) return true;
    if (clock64() - t0 > kWaitCycles) {
      atomicOr(&g_dev_error, code);
      return false;
    }
    __nanosleep(128);
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// Per-warp shared-memory stage (bytes), lane-major inside each operand:
//   A  [4 row slots][32 lanes][LB]        rows g, g+8 of tiles 0 and 1
//   B  [NT tiles][32 lanes][2*LB]         the lane's digit column
//   S  [4 row slots][32 lanes][4]         scales (Z: zeros, asym only)
//   X  [NTG][32 lanes][8]                 group scale 2^(E-22) and sum(x_fix)
// ---------------------------------------------------------------------------
template <int T, bool ASYM, int LB>
struct TileStage {
  static constexpr int NTG = (T + 3) / 4;
  static constexpr int NT = 2 * NTG;
  static constexpr int A = 0;
  static constexpr int B = A + 4 * 32 * LB;
  static constexpr int S = B + NT * 32 * 2 * LB;
  static constexpr int Z = S + 4 * 32 * 4;
  static constexpr int X = Z + (ASYM ? 4 * 32 * 4 : 0);
  static constexpr int BYTES = X + NTG * 32 * 8;
};

template <int T, bool ASYM, int LB>
__global__ void __launch_bounds__(tile_max_threads(T), 1)
    q4_tile_kernel(const __grid_constant__ TileLaunch L) {
  using St = TileStage<T, ASYM, LB>;
  constexpr int NTG = St::NTG, NT = St::NT, WPL = LB / 4, SEGK = 8 * LB;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int wpc = blockDim.x >> 5;
  const uint32_t ring = (uint32_t)__cvta_generic_to_shared(smem) + (uint32_t)warp * kD * St::BYTES;
  const long long W_all = (long long)gridDim.x * wpc;
  int ti = 0;
  bool ok = true;

  for (long long u = (long long)warp * gridDim.x + blockIdx.x; u < L.total && ok; u += W_all) {
    while (ti + 1 < L.ntasks && u >= tile_task(L, ti + 1).ubase) ++ti;
    const TileTask& p = tile_task(L, ti);
    const int N = p.N, K = p.K, G = p.G, lg2gs = p.lg2gs, ntile = p.ntile;
    const int lu = (int)(u - p.ubase);
    const int tile = lu % ntile, ks = lu / ntile;

    // ---- dependencies and activation digits ------------------------------
    if (p.wait_to > p.wait_from) {
      int okw = 1;
      if (lane == 0)
        for (int i = p.wait_from; i < p.wait_to && okw; ++i) {
          const TileTask& q = tile_task(L, i);
          okw = spin_geq(L.done + i, (unsigned)(q.ntile * q.ksplit), 0x200u);
        }
      ok = __shfl_sync(0xffffffffu, okw, 0) != 0;
      if (!ok) break;
    }
    if (!p.xpre) {   // the first warp to reach the task writes its digits
      int state = 0;
      if (lane == 0) state = (int)atomicCAS(L.xflag + ti, 0u, 1u);
      state = __shfl_sync(0xffffffffu, state, 0);
      if (state == 0) {
        write_digits<T>(p, lane, 32);
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicExch(L.xflag + ti, 2u);
      } else {
        int okx = 1;
        if (lane == 0) okx = spin_geq(L.xflag + ti, 2u, 0x400u);
        ok = __shfl_sync(0xffffffffu, okx, 0) != 0;
        if (!ok) break;
      }
    }

    // ---- operand sources of this lane --------------------------------------
    const int r0 = tile * kUnitRows;
    const int kb = ks * p.kper;
    const int ke = min(K, kb + p.kper);
    const int nseg = (ke - kb) / SEGK;
    const uint8_t* asrc[4];
    const float* ssrc[4];
    const float* zsrc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = min(r0 + (i >> 1) * 16 + g + 8 * (i & 1), N - 1);
      asrc[i] = p.W + (size_t)row * (K >> 1) + (kb >> 1) + t * LB;
      ssrc[i] = p.S + (size_t)row * G;
      zsrc[i] = ASYM ? p.Z + (size_t)row * G : nullptr;
    }
    const uint8_t* bsrc[NT];
    bool bval[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int tok = (nt >> 1) * 4 + (g >> 1);
      const int dg = (nt & 1) ? ((g & 1) ? -1 : 2) : (g & 1);
      bval[nt] = tok < T && dg >= 0;
      bsrc[nt] = p.xd + (size_t)(bval[nt] ? tok * 3 + dg : 0) * K + kb + t * 2 * LB;
    }
    const float* xgsc = reinterpret_cast<const float*>(p.xd + (size_t)3 * T * K);
    const float* xsum = xgsc + T * G;

    auto issue = [&](int seg) {
      const uint32_t st = ring + (uint32_t)(seg % kD) * St::BYTES;
      const int gi = (kb + seg * SEGK) >> lg2gs;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        cpa<LB>(st + St::A + (i * 32 + lane) * LB, asrc[i] + seg * (SEGK >> 1));
        cpa<4>(st + St::S + (i * 32 + lane) * 4, ssrc[i] + gi);
        if (ASYM) cpa<4>(st + St::Z + (i * 32 + lane) * 4, zsrc[i] + gi);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        if (bval[nt]) {
          const uint32_t d = st + St::B + (nt * 32 + lane) * 2 * LB;
          const uint8_t* sp = bsrc[nt] + seg * SEGK;
          if constexpr (LB == 16) {
            cpa<16>(d, sp);
            cpa<16>(d + 16, sp + 16);
          } else {
            cpa<2 * LB>(d, sp);
          }
        }
      }
#pragma unroll
      for (int tg = 0; tg < NTG; ++tg) {
        const int tok = min(tg * 4 + t, T - 1);
        cpa<4>(st + St::X + (tg * 32 + lane) * 8, xgsc + tok * G + gi);
        cpa<4>(st + St::X + (tg * 32 + lane) * 8 + 4, xsum + tok * G + gi);
      }
    };

#pragma unroll
    for (int s = 0; s < kD - 1; ++s) {
      if (s < nseg) issue(s);
      cpa_commit();
    }

    float acc[2][NTG][2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int tg = 0; tg < NTG; ++tg) acc[mt][tg][0] = acc[mt][tg][1] = 0.f;
    int C[2][NT][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) C[mt][nt][0] = C[mt][nt][1] = C[mt][nt][2] = C[mt][nt][3] = 0;
    const int segs_per_group = (1 << lg2gs) / SEGK;

    for (int seg = 0; seg < nseg; ++seg) {
      cpa_wait<kD - 2>();   // this lane's copies of segment `seg` have landed
      const uint32_t st = ring + (uint32_t)(seg % kD) * St::BYTES;
      uint32_t w[4][WPL];
#pragma unroll
      for (int i = 0; i < 4; ++i) lds_n<LB>(st + St::A + (i * 32 + lane) * LB, w[i]);
      uint32_t bq[NT][2 * WPL];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        lds_n<2 * LB>(st + St::B + (nt * 32 + lane) * 2 * LB, bq[nt]);
        if (!bval[nt]) {
#pragma unroll
          for (int j = 0; j < 2 * WPL; ++j) bq[nt][j] = 0u;
        }
      }
#pragma unroll
      for (int q = 0; q < WPL; ++q)
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          const uint32_t a0 = nib_lo<ASYM>(w[2 * mt][q]), a2 = nib_hi<ASYM>(w[2 * mt][q]);
          const uint32_t a1 = nib_lo<ASYM>(w[2 * mt + 1][q]), a3 = nib_hi<ASYM>(w[2 * mt + 1][q]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            imma(C[mt][nt], a0, a1, a2, a3, bq[nt][2 * q], bq[nt][2 * q + 1]);
        }
      if ((seg + 1) % segs_per_group == 0 || seg + 1 == nseg) {
        // epilogue of this group: recombine digits, remove zeff * sum(x), scale.
        // Lanes whose token does not exist compute on token T-1 and never store.
#pragma unroll
        for (int tg = 0; tg < NTG; ++tg) {
          const uint2 xv = lds64(st + St::X + (tg * 32 + lane) * 8);
          const float gsc = __uint_as_float(xv.x), xs = __uint_as_float(xv.y);
#pragma unroll
          for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const float sc = __uint_as_float(lds32(st + St::S + ((2 * mt + h) * 32 + lane) * 4));
              const float zp = ASYM ? __uint_as_float(lds32(st + St::Z + ((2 * mt + h) * 32 + lane) * 4))
                                    : 8.f;
              const int i01 = C[mt][2 * tg][2 * h] + 256 * C[mt][2 * tg][2 * h + 1];
              float f = fmaf(65536.f, (float)C[mt][2 * tg + 1][2 * h], (float)i01);
              f = fmaf(-zp, xs, f);
              acc[mt][tg][h] = fmaf(f, sc * gsc, acc[mt][tg][h]);
            }
        }
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) C[mt][nt][0] = C[mt][nt][1] = C[mt][nt][2] = C[mt][nt][3] = 0;
      }
      if (seg + kD - 1 < nseg) issue(seg + kD - 1);
      cpa_commit();
    }
    cpa_wait<0>();

    // ---- results -----------------------------------------------------------
#pragma unroll
    for (int tg = 0; tg < NTG; ++tg) {
      const int tok = tg * 4 + t;
      if (tok < T) {
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int row = r0 + mt * 16 + g + 8 * h;
            if (row < N) {
              const float a = acc[mt][tg][h];
              if (p.ksplit == 1) {
                st_y(p.Y, (size_t)tok * N + row, p.bias ? a + __ldg(p.bias + row) : a, p.ydt);
              } else {
                p.part[((size_t)ks * T + tok) * N + row] = a;
              }
            }
          }
      }
    }
    if (L.done) {   // publish this unit
      __threadfence();
      __syncwarp();
      if (lane == 0) atomicAdd(L.done + ti, 1u);
    }
  }
  cpa_wait<0>();
}

// Activation digits of the pre-converted tasks: one CTA per task.
template <int T>
__global__ void __launch_bounds__(256) q4_digits_kernel(const __grid_constant__ TileLaunch L) {
  const TileTask& p = tile_task(L, blockIdx.x);
  if (!p.xpre) return;
  write_digits<T>(p, threadIdx.x, blockDim.x);
}

// y[t, n] = sum_k part[k][t][n] (+ bias), for k-split tasks.
__global__ void q4_splitk_reduce_kernel(const float* __restrict__ part, const float* __restrict__ bias,
                                        void* Y, int ydt, int N, int T, int ksplit) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N * T) return;
  const int n = i % N;
  float a = 0.f;
  for (int k = 0; k < ksplit; ++k) a += part[(size_t)k * N * T + i];
  if (bias) a += __ldg(bias + n);
  st_y(Y, i, a, ydt);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {

int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return v && *v ? atoi(v) : dflt;
}

int lb_for(int gs) { return (gs % 128 == 0) ? 16 : (gs % 64 == 0 ? 8 : 4); }

int stage_bytes(int T, bool asym, int LB) {
  const int ntg = (T + 3) / 4, nt = 2 * ntg;
  return 4 * 32 * LB + nt * 32 * 2 * LB + 4 * 32 * 4 + (asym ? 4 * 32 * 4 : 0) + ntg * 32 * 8;
}

size_t digit_bytes(int T, int K, int G) {
  return (((size_t)3 * T * K + (size_t)8 * T * G) + 127) & ~(size_t)127;
}

struct TileConfig {
  int T, LB, wpc, grid;
  bool asym;
  size_t smem;
};

bool shape_ok(int N, int K, int gs) {
  return N >= 1 && K % 32 == 0 && gs >= 32 && gs <= 256 && (gs & (gs - 1)) == 0 && K % gs == 0;
}

bool make_config(int T, bool asym, int gs, TileConfig& c) {
  const DeviceInfo& di = device_info();
  c.T = T; c.asym = asym; c.LB = lb_for(gs);
  const size_t per_warp = (size_t)kD * stage_bytes(T, asym, c.LB);
  const size_t cap = (size_t)env_int("SF_TILE_SMEM_KB", 224) * 1024 < (size_t)di.smem_optin
                         ? (size_t)env_int("SF_TILE_SMEM_KB", 224) * 1024
                         : (size_t)di.smem_optin;
  int wpc = (int)(cap / per_warp);
  const int want = env_int("SF_TILE_WARPS", 16);
  if (wpc > want) wpc = want;
  if (wpc > tile_max_threads(T) / 32) wpc = tile_max_threads(T) / 32;
  if (wpc < 1) return false;
  c.wpc = wpc;
  c.smem = per_warp * wpc;
  c.grid = di.sms;
  return true;
}

void fill_task(TileTask& q, int N, int K, int gs, int ksplit) {
  q.N = N; q.K = K; q.G = K / gs; q.lg2gs = __builtin_ctz((unsigned)gs);
  q.ntile = (N + kUnitRows - 1) / kUnitRows;
  const int G = K / gs;
  if (ksplit < 1) ksplit = 1;
  if (ksplit > G) ksplit = G;
  const int gper = (G + ksplit - 1) / ksplit;
  q.kper = gper * gs;
  q.ksplit = (G + gper - 1) / gper;
}

template <int T, bool ASYM, int LB>
cudaError_t launch_tile_t(const TileConfig& c, const TileLaunch& L, bool coop, cudaStream_t st) {
  auto* fn = q4_tile_kernel<T, ASYM, LB>;
  static int configured[kMaxDevices] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < kMaxDevices && configured[dev] < (int)c.smem) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c.smem);
    if (e != cudaSuccess) return e;
    configured[dev] = (int)c.smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)c.grid);
  cfg.blockDim = dim3((unsigned)(c.wpc * 32));
  cfg.dynamicSmemBytes = c.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = coop ? attr : nullptr;
  cfg.numAttrs = coop ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, fn, L);
}

template <bool ASYM, int LB>
cudaError_t launch_tile_lb(const TileConfig& c, const TileLaunch& L, bool coop, cudaStream_t st) {
  switch (c.T) {
    case 1: return launch_tile_t<1, ASYM, LB>(c, L, coop, st);
    case 2: return launch_tile_t<2, ASYM, LB>(c, L, coop, st);
    case 3: return launch_tile_t<3, ASYM, LB>(c, L, coop, st);
    case 4: return launch_tile_t<4, ASYM, LB>(c, L, coop, st);
    case 5: return launch_tile_t<5, ASYM, LB>(c, L, coop, st);
    case 6: return launch_tile_t<6, ASYM, LB>(c, L, coop, st);
    case 7: return launch_tile_t<7, ASYM, LB>(c, L, coop, st);
    default: return launch_tile_t<8, ASYM, LB>(c, L, coop, st);
  }
}

cudaError_t launch_tile(const TileConfig& c, const TileLaunch& L, bool coop, cudaStream_t st) {
  if (c.asym) {
    if (c.LB == 16) return launch_tile_lb<true, 16>(c, L, coop, st);
    if (c.LB == 8) return launch_tile_lb<true, 8>(c, L, coop, st);
    return launch_tile_lb<true, 4>(c, L, coop, st);
  }
  if (c.LB == 16) return launch_tile_lb<false, 16>(c, L, coop, st);
  if (c.LB == 8) return launch_tile_lb<false, 8>(c, L, coop, st);
  return launch_tile_lb<false, 4>(c, L, coop, st);
}

cudaError_t launch_digits(int T, int ntasks, const TileLaunch& L, cudaStream_t st) {
  switch (T) {
    case 1: q4_digits_kernel<1><<<ntasks, 256, 0, st>>>(L); break;
    case 2: q4_digits_kernel<2><<<ntasks, 256, 0, st>>>(L); break;
    case 3: q4_digits_kernel<3><<<ntasks, 256, 0, st>>>(L); break;
    case 4: q4_digits_kernel<4><<<ntasks, 256, 0, st>>>(L); break;
    case 5: q4_digits_kernel<5><<<ntasks, 256, 0, st>>>(L); break;
    case 6: q4_digits_kernel<6><<<ntasks, 256, 0, st>>>(L); break;
    case 7: q4_digits_kernel<7><<<ntasks, 256, 0, st>>>(L); break;
    default: q4_digits_kernel<8><<<ntasks, 256, 0, st>>>(L); break;
  }
  return cudaGetLastError();
}

// Library-owned scratch of the single-GEMV entry (activation digits and k-split
// partial sums), one buffer per (device, stream) so that concurrent streams do
// not share it.  Grows on demand; never shrinks.
struct Scratch {
  void* ptr = nullptr;
  size_t bytes = 0;
};
std::mutex g_scratch_mu;
std::map<std::pair<int, cudaStream_t>, Scratch> g_scratch;

int get_scratch(cudaStream_t st, size_t bytes, void** out) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  Scratch& s = g_scratch[{dev, st}];
  if (s.bytes < bytes) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    if (cs != cudaStreamCaptureStatusNone)
      return fail(SF_ERR_UNSUPPORTED,
                  "scratch must grow during stream capture: run the same shape once before capturing");
    if (s.ptr) cudaFree(s.ptr);
    s.ptr = nullptr;
    s.bytes = 0;
    const size_t nb = (bytes + ((size_t)1 << 20) - 1) & ~(((size_t)1 << 20) - 1);
    cudaError_t e = cudaMalloc(&s.ptr, nb);
    if (e != cudaSuccess) return cuda_fail(e, "allocating GEMV scratch");
    s.bytes = nb;
  }
  *out = s.ptr;
  return SF_OK;
}

}  // namespace

// One GEMV (T <= 8): digits pre-pass, tile kernel with a k-split sized to fill
// the GPU, then a reduce when the k-split is > 1.  SF_ERR_UNSUPPORTED when the
// shape is not one this kernel takes.
int run_tile_linear(const uint8_t* W, const float* S, const float* Z, const float* bias,
                    const void* X, int xdt, void* Y, int ydt, int N, int K, int T, int gs,
                    cudaStream_t stream) {
  if (T < 1 || T > kMaxGemvT || !shape_ok(N, K, gs)) return SF_ERR_UNSUPPORTED;
  TileConfig c;
  if (!make_config(T, Z != nullptr, gs, c)) return SF_ERR_UNSUPPORTED;
  TileLaunch L{};
  TileTask& q = L.single;
  q.W = W; q.S = S; q.Z = Z; q.bias = bias; q.X = X; q.Y = Y; q.xdt = xdt; q.ydt = ydt;
  const int ntile = (N + kUnitRows - 1) / kUnitRows;
  const int warps = c.grid * c.wpc;
  fill_task(q, N, K, gs, (warps + ntile - 1) / ntile);
  const size_t dbytes = digit_bytes(T, K, K / gs);
  const size_t pbytes = q.ksplit > 1 ? (size_t)q.ksplit * T * N * 4 : 0;
  void* scr = nullptr;
  int rc = get_scratch(stream, dbytes + pbytes, &scr);
  if (rc != SF_OK) return rc;
  q.xd = static_cast<uint8_t*>(scr);
  q.part = pbytes ? reinterpret_cast<float*>(static_cast<uint8_t*>(scr) + dbytes) : nullptr;
  q.xpre = 1;
  q.ubase = 0;
  L.tasks = nullptr; L.ntasks = 1; L.total = (long long)q.ntile * q.ksplit;
  L.done = nullptr; L.xflag = nullptr;
  const int need = (int)((L.total + c.wpc - 1) / c.wpc);
  if (c.grid > need) c.grid = need;
  cudaError_t e = launch_digits(T, 1, L, stream);
  if (e != cudaSuccess) return cuda_fail(e, "activation digits launch");
  e = launch_tile(c, L, false, stream);
  if (e != cudaSuccess) return cuda_fail(e, "q4_tile_kernel launch");
  g_launches.fetch_add(2, std::memory_order_relaxed);
  if (q.ksplit > 1) {
    const int n = N * T;
    q4_splitk_reduce_kernel<<<(n + 255) / 256, 256, 0, stream>>>(q.part, bias, Y, ydt, N, T, q.ksplit);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "k-split reduce launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
  }
  return SF_OK;
}

}  // namespace sf

// ===========================================================================
// C ABI: a prepared list of GEMVs run as one persistent launch.
// ===========================================================================
using namespace sf;

namespace {
// workspace: [done counters | ready flags] (256-aligned) [task table] [digit arena]
size_t step_header(int n) { return ((size_t)8 * (n > 0 ? n : 0) + 255) & ~(size_t)255; }
size_t step_table(int n) { return (size_t)(n > 0 ? n : 0) * sizeof(TileTask); }

struct StepHandle {
  TileConfig cfg;
  TileLaunch L;
  void* workspace;
  bool coop, prepass;
};
}  // namespace

extern "C" {

size_t sf_q4_step_workspace_bytes(const sf_q4_task* tasks, int ntasks) {
  if (!tasks || ntasks < 1) return 0;
  size_t n = step_header(ntasks) + ((step_table(ntasks) + 127) & ~(size_t)127);
  for (int i = 0; i < ntasks; ++i) {
    const sf_q4_task& a = tasks[i];
    const int G = a.group_size > 0 ? a.K / a.group_size : 0;
    n += digit_bytes(a.T, a.K, G);
  }
  return n;
}

int sf_q4_step_create(const sf_q4_task* tasks, int ntasks, void* workspace, size_t workspace_bytes,
                      void** handle_out) {
  if (!tasks || !workspace || !handle_out) return fail(SF_ERR_NULL, "null pointer argument");
  if (ntasks < 1) return fail(SF_ERR_SHAPE, "ntasks must be >= 1");
  const size_t need = sf_q4_step_workspace_bytes(tasks, ntasks);
  if (workspace_bytes < need) return fail(SF_ERR_SHAPE, "workspace too small: need %zu bytes", need);
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return fail(SF_ERR_ALIGN, "workspace must be 256-byte aligned");
  const int T = tasks[0].T;
  const bool asym = tasks[0].zeros != nullptr;
  if (T < 1 || T > kMaxGemvT) return fail(SF_ERR_UNSUPPORTED, "step tasks need 1 <= T <= %d", kMaxGemvT);
  TileConfig c;
  if (!make_config(T, asym, tasks[0].group_size, c))
    return fail(SF_ERR_UNSUPPORTED, "no launch configuration for T=%d", T);
  std::vector<TileTask> h(ntasks);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  size_t arena = step_header(ntasks) + ((step_table(ntasks) + 127) & ~(size_t)127);
  long long ub = 0;
  int phase = 0, prev_phase = 0;   // first task of the current / previous phase
  bool any_wait = false, any_pre = false;
  for (int i = 0; i < ntasks; ++i) {
    const sf_q4_task& a = tasks[i];
    if (!a.W || !a.scales || !a.X || !a.Y) return fail(SF_ERR_NULL, "task %d: null pointer", i);
    if (a.T != T || (a.zeros != nullptr) != asym || lb_for(a.group_size) != c.LB)
      return fail(SF_ERR_UNSUPPORTED, "task %d: all tasks need the same T, layout and group class", i);
    if (!shape_ok(a.N, a.K, a.group_size))
      return fail(SF_ERR_UNSUPPORTED, "task %d: shape N=%d K=%d gs=%d not supported by the step kernel",
                  i, a.N, a.K, a.group_size);
    if (a.x_dtype < 0 || a.x_dtype > 2 || a.y_dtype < 0 || a.y_dtype > 2)
      return fail(SF_ERR_DTYPE, "task %d: unknown dtype code", i);
    if ((reinterpret_cast<uintptr_t>(a.W) | reinterpret_cast<uintptr_t>(a.scales) |
         reinterpret_cast<uintptr_t>(a.zeros) | reinterpret_cast<uintptr_t>(a.X)) & 15)
      return fail(SF_ERR_ALIGN, "task %d: W, scales, zeros and X must be 16-byte aligned", i);
    TileTask& q = h[i];
    q = TileTask{};
    q.W = a.W; q.S = a.scales; q.Z = a.zeros; q.bias = a.bias; q.X = a.X; q.Y = a.Y;
    q.xdt = a.x_dtype; q.ydt = a.y_dtype;
    fill_task(q, a.N, a.K, a.group_size, 1);
    q.part = nullptr;
    q.xd = ws + arena;
    arena += digit_bytes(T, q.K, q.G);
    // A task with wait_before opens a phase; every task of a phase reads X only
    // after the whole previous phase has finished (and, transitively, all
    // earlier ones).  Only phase-0 inputs exist before the launch.
    if (i > 0 && a.wait_before) {
      prev_phase = phase;
      phase = i;
    }
    q.wait_from = prev_phase;
    q.wait_to = phase;
    q.xpre = phase == 0 ? 1 : 0;
    any_wait |= phase > 0;
    any_pre |= q.xpre != 0;
    q.ubase = ub;
    ub += (long long)q.ntile * q.ksplit;
  }
  StepHandle* hd = new StepHandle{};
  hd->cfg = c;
  hd->workspace = workspace;
  hd->coop = any_wait;
  hd->prepass = any_pre;
  TileLaunch& L = hd->L;
  L.tasks = reinterpret_cast<const TileTask*>(ws + step_header(ntasks));
  L.ntasks = ntasks;
  L.total = ub;
  L.done = reinterpret_cast<unsigned int*>(ws);
  L.xflag = L.done + ntasks;
  cudaError_t e = cudaMemcpy(const_cast<TileTask*>(L.tasks), h.data(), step_table(ntasks),
                             cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    delete hd;
    return cuda_fail(e, "uploading the task table");
  }
  *handle_out = hd;
  return SF_OK;
}

int sf_q4_step_run(void* handle, void* stream) {
  if (!handle) return fail(SF_ERR_NULL, "null handle");
  StepHandle* hd = static_cast<StepHandle*>(handle);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(hd->workspace, 0, step_header(hd->L.ntasks), st);
  if (e != cudaSuccess) return cuda_fail(e, "clearing the completion counters");
  if (hd->prepass) {
    e = launch_digits(hd->cfg.T, hd->L.ntasks, hd->L, st);
    if (e != cudaSuccess) return cuda_fail(e, "activation digits launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
  }
  e = launch_tile(hd->cfg, hd->L, hd->coop, st);
  if (e != cudaSuccess) return cuda_fail(e, "q4 step launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return SF_OK;
}

void sf_q4_step_destroy(void* handle) { delete static_cast<StepHandle*>(handle); }

}  // extern "C"
