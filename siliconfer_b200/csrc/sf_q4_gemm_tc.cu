// sf_q4_gemm_tc.cu -- prefill GEMM Y[T,N] = X[T,K] @ dequant(W)^T on the
// sm_100a tcgen05 tensor cores (bf16 operands, fp32 accumulation in TMEM).
//
// Reference semantics: q4_gemm_sym_neon / q4_gemm_asym_neon
// (siliconfer/kernels/neon/q4_gemm.cpp:12-51) run the GEMV of q4_gemv.cpp
// once per token; the numpy fallback (siliconfer/kernels/neon/__init__.py:
// 191-197, 221-227) computes the same product.  The weight value that enters
// the product is dequantize_sym / dequantize_asym
// (siliconfer/quant/primitives.py:54-75, 117-140): w = q*s and w = (q - z)*s
// in fp32.  Here every weight is that fp32 value rounded to bf16 (nearest
// even), and X is bf16 (converted from fp32/fp16 by a pre-pass), so outputs
// agree with the fp32 reference to the bf16 tolerance.
//
// Kernel structure (one persistent CTA per SM, 14 warps):
//  * warp 4  (producer): per k-block of 64, one TMA tile copy of each
//    128-token slice of X (128-byte swizzle, the tcgen05 K-major layout) and
//    one TMA tile copy of the packed weight bytes [BN rows x 32 bytes];
//  * warps 6-13 (dequant): turn the packed bytes into bf16 weights
//    (q - z) * s in fp32, rounded to bf16, written into shared memory in the
//    same 128-byte swizzled K-major layout, then fence to the async proxy;
//  * warp 5  (MMA): allocates TMEM, one elected thread issues
//    tcgen05.mma.kind::f16 (M = 128 tokens, N = BN weight rows, K = 16) for
//    each of the MT token slices, and releases each stage with
//    tcgen05.commit;
//  * warps 0-3 (epilogue): tcgen05.ld the fp32 accumulators (warp w reads
//    TMEM lanes 32w..32w+31 = tokens), add the bias, convert, store Y.
//  The accumulators are double-buffered in TMEM when MT*BN <= 256 columns,
//  so a tile's epilogue overlaps the next tile's main loop.
//  Every wait is bounded; on expiry the kernel records a bit in the device
//  error word, raises a block-wide abort flag, drains its own copies and
//  MMAs (bounded), frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <map>
#include <mutex>

#include "sf_q4.h"
#include "sf_q4_internal.h"

namespace sf {
SF_DEFINE_ERROR_READER(take_dev_error_tc)
extern std::atomic<long long> g_launches;

namespace {

constexpr int kBK = 64;                 // k per stage: 64 bf16 = one 128-byte swizzle row
constexpr int kSliceBytes = 128 * 128;  // one 128-token slice of X per stage
constexpr int kEpiWarps = 4, kProdWarp = 4, kMmaWarp = 5, kDqWarp0 = 6, kDqWarps = 8;
constexpr int kThreads = 32 * (kDqWarp0 + kDqWarps);
constexpr int kSmemLimit = 232448;      // 227 KB opt-in per block
constexpr int kTcMinT = 48;             // below this the GEMV kernel (weights re-read per 8 tokens) wins

// error-word bits of this kernel
constexpr unsigned kErrProd = 1u << 8, kErrDq = 1u << 9, kErrMma = 1u << 10, kErrEpi = 1u << 11,
                   kErrDrain = 1u << 12;

struct TcParams {
  const float* S;
  const float* Z;
  const float* bias;
  void* Y;
  int T, N, K, G, gs, ydt;
  int mtiles, ntiles, kblocks, stages;
};

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool bar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}

// Bounded wait that also gives up when another role raised the abort flag.
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity, unsigned code,
                                         volatile int* abort_flag) {
  if (bar_try(bar, parity)) return true;
  const long long t0 = clock64();
  while (!bar_try(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) {
      atomicOr(&g_dev_error, code);
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void bar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void prefetch_map(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(m) : "memory");
}

// Shared-memory matrix descriptor of a K-major bf16 tile with 128-byte rows in
// the 128-byte swizzle (8-row atoms of 1024 bytes; stride between atoms 1024):
// start address >> 4 in bits 0-13, leading offset 16 B (unused for swizzled
// K-major), stride offset 1024 B in bits 32-45, descriptor version 1 at bit
// 46, swizzle mode 2 (128 B) in bits 61-63.  Moving 16 k (32 bytes) inside
// the atom adds 2 to the start-address field.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::f16: D fp32 (bits 4-5 = 1), A and B bf16
// (bits 7-9 = 1, 10-12 = 1), both K-major, N >> 3 in bits 17-22, M >> 4 in
// bits 24-28.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// Eight nibbles of one packed word (k order: lo nibble of byte 0 first) to
// eight bf16 weights RNE((q - z) * s), as four bf16x2 words.
//  * u: the nibbles as unsigned 0..15 (symmetric nibbles already flipped
//    with ^8, so that u - 8 is the two's-complement value);
//  * 2^23 + u is built exactly as a float from the byte (prmt);
//  * zint: the zero point is an integer, so 2^23 + z is exact and one
//    subtraction gives u - z exactly; otherwise u and u - z are formed in two
//    steps, rounding exactly as the reference's fp32 (q - z).
template <bool ZINT>
__device__ __forceinline__ uint4 dequant8(uint32_t w, bool sym, float zc, float z, float s) {
  uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
  if (sym) { lo ^= 0x08080808u; hi ^= 0x08080808u; }
  float f[8];
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    f[2 * b] = __uint_as_float(prmt(lo, 0x4B000000u, 0x7440u + b));
    f[2 * b + 1] = __uint_as_float(prmt(hi, 0x4B000000u, 0x7440u + b));
  }
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float a, c;
    if (ZINT) {
      a = __fmul_rn(__fsub_rn(f[2 * j], zc), s);
      c = __fmul_rn(__fsub_rn(f[2 * j + 1], zc), s);
    } else {
      a = __fmul_rn(__fsub_rn(__fsub_rn(f[2 * j], 8388608.f), z), s);
      c = __fmul_rn(__fsub_rn(__fsub_rn(f[2 * j + 1], 8388608.f), z), s);
    }
    o[j] = pack_bf16(a, c);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

template <int MT, int BN>
struct TcLayout {
  static constexpr uint32_t X = MT * kSliceBytes;
  static constexpr uint32_t WQ = BN * 128;     // dequantized bf16 tile
  static constexpr uint32_t P = BN * 32;       // packed bytes
  static constexpr uint32_t STAGE = X + WQ + P;  // multiple of 1024
  static constexpr int ACC_COLS = MT * BN;
  static constexpr int NBUF = ACC_COLS <= 256 ? 2 : 1;
  static constexpr uint32_t TMEM_COLS = ACC_COLS * NBUF <= 256 ? 256 : 512;
  static_assert(STAGE % 1024 == 0, "stage must keep 1024-byte alignment");
};

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
template <int MT, int BN, bool ASYM>
__global__ void __launch_bounds__(kThreads, 1)
    q4_gemm_tc_kernel(const __grid_constant__ CUtensorMap mapX, const __grid_constant__ CUtensorMap mapW,
                      const TcParams p) {
  using L = TcLayout<MT, BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const int S = p.stages;
  // control block after the stages: barriers, TMEM address, abort flag
  const uint32_t ctl = base + (uint32_t)S * L::STAGE;
  const uint32_t full0 = ctl, dq0 = ctl + 8 * 8, empty0 = ctl + 16 * 8;
  const uint32_t accf0 = ctl + 24 * 8, acce0 = ctl + 26 * 8, drain = ctl + 28 * 8;
  uint8_t* ctl_gen = smem_raw + (ctl - raw);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(ctl_gen + 30 * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(ctl_gen + 31 * 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      bar_init(full0 + 8 * s, 1);
      bar_init(dq0 + 8 * s, kDqWarps);
      bar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      bar_init(accf0 + 8 * b, 1);
      bar_init(acce0 + 8 * b, kEpiWarps);
    }
    bar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kProdWarp && lane == 0) {
    prefetch_map(&mapX);
    prefetch_map(&mapW);
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32((const void*)tmem_slot)),
                 "r"(L::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int ntiles_total = p.mtiles * p.ntiles;
  const int KB = p.kblocks;

  if (warp == kProdWarp) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles_total && ok; tile += gridDim.x) {
        const int m0 = (tile % p.mtiles) * (128 * MT), n0 = (tile / p.mtiles) * BN;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1;
          if (!bar_wait(empty0 + 8 * s, ph ^ 1, kErrProd, abort_flag)) { ok = false; break; }
          const uint32_t st = base + s * L::STAGE;
          bar_expect_tx(full0 + 8 * s, L::X + L::P);
#pragma unroll
          for (int m = 0; m < MT; ++m) tma_2d(st + m * kSliceBytes, &mapX, kb * kBK, m0 + m * 128, full0 + 8 * s);
          tma_2d(st + L::X + L::WQ, &mapW, kb * (kBK / 2), n0, full0 + 8 * s);
        }
      }
      // Drain: every issued copy must have landed before the block exits.
      const uint32_t pending = it < (uint32_t)S ? it : (uint32_t)S;
      for (uint32_t j = it - pending; j < it; ++j) {
        const uint32_t s = j % S, ph = (j / S) & 1;
        if (!bar_try(full0 + 8 * s, ph)) {
          const long long t0 = clock64();
          while (!bar_try(full0 + 8 * s, ph))
            if (clock64() - t0 > kWaitCycles) { atomicOr(&g_dev_error, kErrDrain); break; }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(128, BN);
      uint32_t it = 0, issued = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles_total && ok; tile += gridDim.x, ++local) {
        const int b = L::NBUF == 2 ? (local & 1) : 0;
        const uint32_t use = L::NBUF == 2 ? (uint32_t)(local >> 1) : (uint32_t)local;
        if (!bar_wait(acce0 + 8 * b, (use & 1) ^ 1, kErrMma, abort_flag)) break;
        tc_fence_after();
        const uint32_t dcol = tmem + (uint32_t)(b * L::ACC_COLS);
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1;
          if (!bar_wait(full0 + 8 * s, ph, kErrMma, abort_flag) ||
              !bar_wait(dq0 + 8 * s, ph, kErrMma, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t st = base + s * L::STAGE;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t bdesc = sw128_desc(st + L::X + kk * 32);
#pragma unroll
            for (int m = 0; m < MT; ++m)
              mma_bf16(dcol + m * BN, sw128_desc(st + m * kSliceBytes + kk * 32), bdesc, idesc,
                       (kb | kk) != 0);
          }
          issued = 1;
          mma_commit(empty0 + 8 * s);
        }
        if (ok) mma_commit(accf0 + 8 * b);
      }
      // Drain: wait until every issued MMA has completed before TMEM is freed.
      if (issued) {
        mma_commit(drain);
        if (!bar_try(drain, 0)) {
          const long long t0 = clock64();
          while (!bar_try(drain, 0))
            if (clock64() - t0 > kWaitCycles) { atomicOr(&g_dev_error, kErrDrain); break; }
        }
      }
    }
  } else if (warp >= kDqWarp0) {
    // ---------------- dequant: packed bytes -> bf16 swizzled tile ----------------
    const int dt = threadIdx.x - 32 * kDqWarp0;  // 0..255
    constexpr int kUnits = BN * 2;               // (row, 32-k half) pairs per stage
    constexpr int kPer = kUnits / (32 * kDqWarps);
    static_assert(kUnits % (32 * kDqWarps) == 0, "units must divide evenly");
    uint32_t it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles_total && ok; tile += gridDim.x) {
      const int n0 = (tile / p.mtiles) * BN;
      for (int kb = 0; kb < KB; ++kb, ++it) {
        const uint32_t s = it % S, ph = (it / S) & 1;
        // the unit's scale and zero point, fetched before the wait
        float sc[kPer], zz[kPer];
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
          const int u = dt + j * 32 * kDqWarps, r = u >> 1, h = u & 1;
          const int n = n0 + r, g = (kb * kBK + h * 32) / p.gs;
          const bool in = n < p.N;
          sc[j] = in ? __ldg(p.S + (size_t)n * p.G + g) : 0.f;
          zz[j] = (ASYM && in) ? __ldg(p.Z + (size_t)n * p.G + g) : 0.f;
        }
        if (!bar_wait(full0 + 8 * s, ph, kErrDq, abort_flag)) { ok = false; break; }
        const uint32_t st = base + s * L::STAGE;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
          const int u = dt + j * 32 * kDqWarps, r = u >> 1, h = u & 1;
          uint4 wq;
          asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(wq.x), "=r"(wq.y), "=r"(wq.z), "=r"(wq.w)
                       : "r"(st + L::X + L::WQ + r * 32 + h * 16));
          const float z = ASYM ? zz[j] : 8.f;
          const bool zint = !ASYM || (z == rintf(z) && fabsf(z) < 4194304.f);
          const float zc = 8388608.f + z;
          const uint32_t w4[4] = {wq.x, wq.y, wq.z, wq.w};
          const uint32_t row = st + L::X + r * 128;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint4 o = zint ? dequant8<true>(w4[c], !ASYM, zc, z, sc[j])
                                 : dequant8<false>(w4[c], !ASYM, zc, z, sc[j]);
            const uint32_t chunk = (uint32_t)(h * 4 + c) ^ (uint32_t)(r & 7);
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(row + chunk * 16), "r"(o.x), "r"(o.y),
                         "r"(o.z), "r"(o.w)
                         : "memory");
          }
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) bar_arrive(dq0 + 8 * s);
      }
    }
  } else {
    // ---------------- epilogue: TMEM -> Y ----------------
    const int q = warp;  // TMEM lanes 32q..32q+31
    int local = 0;
    const size_t ye = p.ydt == SF_F32 ? 4 : 2;
    for (int tile = blockIdx.x; tile < ntiles_total; tile += gridDim.x, ++local) {
      const int m0 = (tile % p.mtiles) * (128 * MT), n0 = (tile / p.mtiles) * BN;
      const int b = L::NBUF == 2 ? (local & 1) : 0;
      const uint32_t use = L::NBUF == 2 ? (uint32_t)(local >> 1) : (uint32_t)local;
      if (!bar_wait(accf0 + 8 * b, use & 1, kErrEpi, abort_flag)) break;
      tc_fence_after();
#pragma unroll 1
      for (int m = 0; m < MT; ++m) {
        const int t = m0 + m * 128 + q * 32 + lane;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          float v[32];
          tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * L::ACC_COLS + m * BN + c0), v);
          const int nb = n0 + c0;
          if (t < p.T && nb < p.N) {  // rows past T and columns past N store nothing
          const int nv = p.N - nb < 32 ? p.N - nb : 32;
          if (p.bias) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < nv) v[i] += __ldg(p.bias + nb + i);
          }
          uint8_t* yrow = static_cast<uint8_t*>(p.Y) + ((size_t)t * p.N + nb) * ye;
          const bool vec = nv == 32 && ((reinterpret_cast<uintptr_t>(yrow) & 15) == 0);
          if (p.ydt == SF_F32) {
            float* y = reinterpret_cast<float*>(yrow);
            if (vec) {
#pragma unroll
              for (int i = 0; i < 32; i += 4)
                *reinterpret_cast<float4*>(y + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (i < nv) y[i] = v[i];
            }
          } else if (p.ydt == SF_BF16) {
            __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(yrow);
            if (vec) {
#pragma unroll
              for (int i = 0; i < 32; i += 8) {
                uint4 o;
                o.x = pack_bf16(v[i], v[i + 1]); o.y = pack_bf16(v[i + 2], v[i + 3]);
                o.z = pack_bf16(v[i + 4], v[i + 5]); o.w = pack_bf16(v[i + 6], v[i + 7]);
                *reinterpret_cast<uint4*>(y + i) = o;
              }
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (i < nv) y[i] = __float2bfloat16_rn(v[i]);
            }
          } else {
            __half* y = reinterpret_cast<__half*>(yrow);
            if (vec) {
#pragma unroll
              for (int i = 0; i < 32; i += 8) {
                __half2 h0 = __floats2half2_rn(v[i], v[i + 1]), h1 = __floats2half2_rn(v[i + 2], v[i + 3]),
                        h2 = __floats2half2_rn(v[i + 4], v[i + 5]), h3 = __floats2half2_rn(v[i + 6], v[i + 7]);
                uint4 o;
                o.x = *reinterpret_cast<uint32_t*>(&h0); o.y = *reinterpret_cast<uint32_t*>(&h1);
                o.z = *reinterpret_cast<uint32_t*>(&h2); o.w = *reinterpret_cast<uint32_t*>(&h3);
                *reinterpret_cast<uint4*>(y + i) = o;
              }
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (i < nv) y[i] = __float2half_rn(v[i]);
            }
          }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(acce0 + 8 * b);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::TMEM_COLS)
                 : "memory");
  }
}

// fp32 / fp16 activations -> bf16 (round to nearest even), 8 per thread.
__global__ void x_to_bf16_kernel(const void* __restrict__ X, int xdt, __nv_bfloat16* __restrict__ out,
                                 long long n) {
  const long long i0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (i0 >= n) return;
  if (i0 + 8 <= n && xdt == SF_F32 && ((reinterpret_cast<uintptr_t>(X) & 15) == 0)) {
    const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(X) + i0);
    const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(X) + i0 + 4);
    uint4 o;
    o.x = pack_bf16(a.x, a.y); o.y = pack_bf16(a.z, a.w);
    o.z = pack_bf16(b.x, b.y); o.w = pack_bf16(b.z, b.w);
    *reinterpret_cast<uint4*>(out + i0) = o;
    return;
  }
  for (long long i = i0; i < i0 + 8 && i < n; ++i) {
    const float v = xdt == SF_F32 ? static_cast<const float*>(X)[i]
                                  : __half2float(static_cast<const __half*>(X)[i]);
    out[i] = __float2bfloat16_rn(v);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

bool make_map(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t rows,
              uint64_t stride_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// bf16 copy of X for fp32/fp16 inputs: library-owned, one per (device,
// stream), grown on demand.
std::mutex g_xbuf_mu;
std::map<std::pair<int, cudaStream_t>, std::pair<void*, size_t>> g_xbuf;

int xbuf_get(cudaStream_t st, size_t bytes, void** out) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_xbuf_mu);
  auto& e = g_xbuf[{dev, st}];
  if (e.second < bytes) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    if (cs != cudaStreamCaptureStatusNone)
      return fail(SF_ERR_UNSUPPORTED,
                  "prefill activation buffer must grow during stream capture: run the same shape once before capturing");
    if (e.first) {
      cudaStreamSynchronize(st);
      cudaFree(e.first);
      e.first = nullptr;
      e.second = 0;
    }
    const size_t nb = (bytes + ((size_t)1 << 20) - 1) & ~(((size_t)1 << 20) - 1);
    cudaError_t err = cudaMalloc(&e.first, nb);
    if (err != cudaSuccess) return cuda_fail(err, "allocating the prefill activation buffer");
    e.second = nb;
  }
  *out = e.first;
  return SF_OK;
}

struct TcChoice {
  int MT, BN;
};

// Tile shape: fewest tile-rounds per SM, weighing a 128-token tile (MT = 1)
// by the extra dequant work per MAC and a 128-column tile by its extra
// shared-memory operand traffic.
TcChoice choose_tile(int T, int N, int sms) {
  const int cand[4][2] = {{2, 256}, {2, 128}, {1, 256}, {1, 128}};
  TcChoice best{2, 128};
  double best_cost = 1e300;
  for (auto& c : cand) {
    if (c[0] == 2 && T <= 128) continue;  // a second 128-token slice would hold no tokens
    const long long mt = (T + 128 * c[0] - 1) / (128 * c[0]), nt = (N + c[1] - 1) / c[1];
    const long long rounds = (mt * nt + sms - 1) / sms;
    double cost = (double)rounds * 128.0 * c[0] * c[1];
    if (c[0] == 1) cost *= 1.25;
    if (c[1] == 128) cost *= 1.1;
    if (cost < best_cost) { best_cost = cost; best = {c[0], c[1]}; }
  }
  return best;
}

template <int MT, int BN, bool ASYM>
int launch_tc(const CUtensorMap& mx, const CUtensorMap& mw, TcParams& p, int sms, cudaStream_t st) {
  using L = TcLayout<MT, BN>;
  int S = (int)((kSmemLimit - 1024 - 512) / L::STAGE);
  if (S > 6) S = 6;
  if (S < 2) return SF_ERR_UNSUPPORTED;
  p.stages = S;
  const size_t smem = 1024 + (size_t)S * L::STAGE + 512;
  auto* fn = q4_gemm_tc_kernel<MT, BN, ASYM>;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return cuda_fail(e, "q4_gemm_tc_kernel smem attribute");
  const int tiles = p.mtiles * p.ntiles;
  const int grid = tiles < sms ? tiles : sms;
  fn<<<grid, kThreads, smem, st>>>(mx, mw, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "q4_gemm_tc_kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return SF_OK;
}

}  // namespace

int run_tc_gemm(const uint8_t* W, const float* S, const float* Z, const float* bias, const void* X, int xdt,
                void* Y, int ydt, int N, int K, int T, int gs, int flags, cudaStream_t stream) {
  (void)flags;
  if (getenv("SF_TC_DISABLE")) return SF_ERR_UNSUPPORTED;
  if (T < kTcMinT && !getenv("SF_TC_FORCE")) return SF_ERR_UNSUPPORTED;
  // Shapes this kernel takes: whole 64-k blocks, a group size that keeps each
  // 32-k half inside one group, 16-byte aligned weights and activations.
  if (K % kBK || gs % 32 || ((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(X)) & 15))
    return SF_ERR_UNSUPPORTED;
  DeviceInfo& di = device_info();
  if (di.smem_optin < kSmemLimit) return SF_ERR_UNSUPPORTED;

  const void* xb = X;
  if (xdt != SF_BF16) {
    void* buf = nullptr;
    const long long n = (long long)T * K;
    int rc = xbuf_get(stream, (size_t)n * 2, &buf);
    if (rc != SF_OK) return rc;
    const int threads = 256;
    const long long blocks = (n / 8 + threads) / threads;
    x_to_bf16_kernel<<<(unsigned)blocks, threads, 0, stream>>>(X, xdt, static_cast<__nv_bfloat16*>(buf), n);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "x_to_bf16_kernel launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
    xb = buf;
  }

  const TcChoice c = choose_tile(T, N, di.sms);
  CUtensorMap mx, mw;
  if (!make_map(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, xb, (uint64_t)K, (uint64_t)T, (uint64_t)K * 2, kBK, 128,
                CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(SF_ERR_CUDA, "cuTensorMapEncodeTiled failed for the prefill activations (T=%d K=%d)", T, K);
  if (!make_map(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, W, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2, kBK / 2,
                (uint32_t)c.BN, CU_TENSOR_MAP_SWIZZLE_NONE))
    return fail(SF_ERR_CUDA, "cuTensorMapEncodeTiled failed for the prefill weights (N=%d K=%d)", N, K);

  TcParams p{};
  p.S = S; p.Z = Z; p.bias = bias; p.Y = Y;
  p.T = T; p.N = N; p.K = K; p.G = K / gs; p.gs = gs; p.ydt = ydt;
  p.mtiles = (T + 128 * c.MT - 1) / (128 * c.MT);
  p.ntiles = (N + c.BN - 1) / c.BN;
  p.kblocks = K / kBK;
  const bool asym = Z != nullptr;
#define SF_TC_CASE(MT_, BN_)                                                         \
  if (c.MT == MT_ && c.BN == BN_)                                                    \
    return asym ? launch_tc<MT_, BN_, true>(mx, mw, p, di.sms, stream)               \
                : launch_tc<MT_, BN_, false>(mx, mw, p, di.sms, stream);
  SF_TC_CASE(2, 256)
  SF_TC_CASE(2, 128)
  SF_TC_CASE(1, 256)
  SF_TC_CASE(1, 128)
#undef SF_TC_CASE
  return SF_ERR_UNSUPPORTED;
}

}  // namespace sf
