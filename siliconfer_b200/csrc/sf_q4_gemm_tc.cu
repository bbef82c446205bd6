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
// Kernel structure (one persistent CTA per SM, 18 warps):
//  * warp 4 (producer): per k-block of 64, one TMA tile copy of the BT-token
//    slice of X (128-byte swizzle, the tcgen05 K-major layout) and one TMA
//    tile copy of the packed weight bytes [128 rows x 32 bytes];
//  * warps 6-17 (dequant, three per TMEM lane quarter, each taking every
//    third k-block): turn the packed bytes into bf16 weights RNE((q - z) * s)
//    and write them straight into TMEM with tcgen05.st, where they are the
//    MMA's A operand (M = 128 weight rows);
//  * warp 5 (MMA): allocates TMEM; one elected thread issues
//    tcgen05.mma.cta_group::1.kind::f16 (A = weights from TMEM, B = X from
//    shared memory, N = BT tokens, K = 16) and releases stages with
//    tcgen05.commit;
//  * warps 0-3 (epilogue): tcgen05.ld the fp32 accumulators (lanes = weight
//    rows, columns = tokens), add the bias, convert, and store Y through a
//    [token][row] staging tile in shared memory with one TMA bulk store per
//    32-token chunk (two staging tiles alternate).
//  BT = 256 tokens (one accumulator buffer) or 128 (two, so that a tile's
//  epilogue overlaps the next tile's main loop), chosen by tile rounds per SM.
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
#include <cstring>
#include <map>
#include <mutex>

#include "sf_q4.h"
#include "sf_q4_internal.h"


namespace sf {
SF_DEFINE_ERROR_READER(take_dev_error_tc)
extern std::atomic<long long> g_launches;

namespace {

constexpr int kBK = 64;                 // k per stage: 64 bf16 = one 128-byte swizzle row
constexpr int kEpiWarps = 4, kProdWarp = 4, kMmaWarp = 5, kDqWarp0 = 6;
constexpr int kDqLanes = 3;   // dequant warps per TMEM lane quarter, one per in-flight k-block
constexpr int kDqWarps = 4 * kDqLanes;
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
  int T, N, K, G, gs, lg2gs, ydt;
  int mtiles, ntiles, kblocks, stages;
  int tma_store;  // epilogue writes Y with TMA stores (Y 16-byte aligned, N * elem % 16 == 0)
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

// Two fp32 lanes per instruction (sm_100 packed f32x2 arithmetic).
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t v;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(lo), "f"(hi));
  return v;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint32_t pack_bf16x2(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return pack_bf16(lo, hi);
}

// Eight nibbles of one packed word (k order: lo nibble of byte 0 first) to
// eight bf16 weights RNE((q - z) * s), as four bf16x2 words (k pairs).
//  * u: the nibbles as unsigned 0..15 (symmetric nibbles flipped with ^8, so
//    that u - 8 is the two's-complement value and sym is the case z = 8);
//  * 2^23 + u is built exactly as a float from the byte (prmt);
//  * ZINT (integer zero point): negzc = -(2^23 + z) is exact, so one addition
//    gives u - z exactly, then one multiply rounds (u - z) * s once, as the
//    reference's fp32 arithmetic does;
//  * otherwise u is recovered exactly, then u - z and (u - z) * s each round
//    once, again as in the reference.
template <bool ZINT>
__device__ __forceinline__ void dequant8(uint32_t w, bool sym, uint64_t negzc2, uint64_t negz2, uint64_t s2,
                                         uint32_t (&o)[4]) {
  uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
  if (sym) { lo ^= 0x08080808u; hi ^= 0x08080808u; }
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    uint64_t v = f2(__uint_as_float(prmt(lo, 0x4B000000u, 0x7440u + b)),
                    __uint_as_float(prmt(hi, 0x4B000000u, 0x7440u + b)));
    if (ZINT) {
      v = add2(v, negzc2);
    } else {
      v = add2(add2(v, f2(-8388608.f, -8388608.f)), negz2);
    }
    o[b] = pack_bf16x2(mul2(v, s2));
  }
}

// 32 consecutive 32-bit TMEM columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T: A (128 x 16 bf16) in TMEM, one row per
// lane, two k per 32-bit column.
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Shared-memory and TMEM plan of a BT-token tile:
//  * stage s: X tile [BT tokens x 64 k] bf16 in the 128-byte swizzle, then
//    the packed weight tile [128 rows x 32 bytes] in the 32-byte swizzle
//    (rows r and r+4 land in different banks for the dequant reads);
//  * TMEM: the fp32 accumulators (BT columns, two buffers when BT <= 128),
//    then one 32-column slot of dequantized weights per stage.
template <int BT>
struct TcLayout {
  static constexpr uint32_t X = BT * 128;
  static constexpr uint32_t P = 128 * 32;
  static constexpr uint32_t STAGE = X + P;
  // two staging buffers of the epilogue's TMA stores: [32 tokens][128 rows], fp32 at most
  static constexpr uint32_t OUT = 32 * 128 * 4;
  static constexpr int S_SMEM = (kSmemLimit - 1024 - 512 - 2 * (int)OUT) / (int)STAGE;
  static constexpr int S = S_SMEM > 6 ? 6 : S_SMEM;
  static constexpr int NBUF = BT <= 128 ? 2 : 1;
  static constexpr uint32_t A_COL = NBUF * BT;  // first weight slot column
  static constexpr uint32_t TMEM_COLS = 512;
  static_assert(STAGE % 1024 == 0, "stage must keep 1024-byte alignment");
  static_assert(A_COL + 32 * S <= TMEM_COLS, "TMEM plan exceeds 512 columns");
  static constexpr size_t SMEM = 1024 + (size_t)S * STAGE + 2 * OUT + 512;
};

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(x),
               "r"(y), "r"(src)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// ---------------------------------------------------------------------------
// The kernel: one CTA computes Y[t0 : t0+BT, n0 : n0+128] tiles in turn.
// ---------------------------------------------------------------------------
template <int BT, bool ASYM>
__global__ void __launch_bounds__(kThreads, 1)
    q4_gemm_tc_kernel(const __grid_constant__ CUtensorMap mapX, const __grid_constant__ CUtensorMap mapW,
                      const __grid_constant__ CUtensorMap mapY, const TcParams p) {
  using L = TcLayout<BT>;
  constexpr int S = L::S;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t out0 = base + (uint32_t)S * L::STAGE;   // epilogue staging, 2 x OUT
  // control block after the staging: barriers, TMEM address, abort flag
  const uint32_t ctl = out0 + 2 * L::OUT;
  const uint32_t full0 = ctl, dq0 = ctl + 8 * 8, empty0 = ctl + 16 * 8;
  const uint32_t accf0 = ctl + 24 * 8, acce0 = ctl + 26 * 8, drain = ctl + 28 * 8;
  uint8_t* ctl_gen = smem_raw + (ctl - raw);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(ctl_gen + 30 * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(ctl_gen + 31 * 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      bar_init(full0 + 8 * s, 1);
      bar_init(dq0 + 8 * s, 4);  // one warp per lane quarter
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
        const int m0 = (tile % p.mtiles) * BT, n0 = (tile / p.mtiles) * 128;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1;
          if (!bar_wait(empty0 + 8 * s, ph ^ 1, kErrProd, abort_flag)) { ok = false; break; }
          const uint32_t st = base + s * L::STAGE;
          bar_expect_tx(full0 + 8 * s, L::X + L::P);
          tma_2d(st, &mapX, kb * kBK, m0, full0 + 8 * s);
          tma_2d(st + L::X, &mapW, kb * (kBK / 2), n0, full0 + 8 * s);
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
      const uint32_t idesc = idesc_bf16(128, BT);
      uint32_t it = 0, issued = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles_total && ok; tile += gridDim.x, ++local) {
        const int b = L::NBUF == 2 ? (local & 1) : 0;
        const uint32_t use = L::NBUF == 2 ? (uint32_t)(local >> 1) : (uint32_t)local;
        if (!bar_wait(acce0 + 8 * b, (use & 1) ^ 1, kErrMma, abort_flag)) break;
        tc_fence_after();
        const uint32_t dcol = tmem + (uint32_t)(b * BT);
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1;
          if (!bar_wait(full0 + 8 * s, ph, kErrMma, abort_flag) ||
              !bar_wait(dq0 + 8 * s, ph, kErrMma, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t st = base + s * L::STAGE;
          const uint32_t acol = tmem + L::A_COL + 32 * s;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_bf16_ts(dcol, acol + 8 * kk, sw128_desc(st + kk * 32), idesc, (kb | kk) != 0);
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
    // ------- dequant: packed bytes -> bf16 weights in this stage's TMEM slot -------
    // Warp w serves TMEM lanes 32*(w%4)... (weight rows r = one per thread)
    // and every kDqLanes-th stage (stage lane j): all 64 weights of its row
    // for that k-block.  kDqLanes k-blocks are dequantized concurrently per
    // lane quarter, which hides the latency of each one.
    const int q = warp & 3, j = (warp - kDqWarp0) >> 2;
    const int r = 32 * q + lane;
    uint32_t it0 = 0;  // global stage index of the current tile's k-block 0
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles_total && ok; tile += gridDim.x, it0 += KB) {
      const int n = (tile / p.mtiles) * 128 + r;
      const bool in = n < p.N;
      const float* srow = p.S + (size_t)(in ? n : 0) * p.G;
      const float* zrow = ASYM ? p.Z + (size_t)(in ? n : 0) * p.G : nullptr;
      // first k-block of this tile that belongs to stage lane j
      const int kb0 = (int)(((uint32_t)j + kDqLanes - it0 % kDqLanes) % kDqLanes);
      // scales / zero points of both 32-k halves, loaded one own k-block ahead
      auto ld2 = [&](const float* row, int kb, float (&v)[2]) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
          v[hh] = (in && kb < KB) ? __ldg(row + ((kb * kBK + 32 * hh) >> p.lg2gs)) : 0.f;
      };
      float sn[2], zn[2] = {8.f, 8.f};
      ld2(srow, kb0, sn);
      if (ASYM) ld2(zrow, kb0, zn);
      for (int kb = kb0; kb < KB; kb += kDqLanes) {
        const uint32_t it = it0 + kb;
        const uint32_t s = it % S, ph = (it / S) & 1;
        const float sc[2] = {sn[0], sn[1]}, zc[2] = {zn[0], zn[1]};
        ld2(srow, kb + kDqLanes, sn);
        if (ASYM) ld2(zrow, kb + kDqLanes, zn);
        if (!bar_wait(full0 + 8 * s, ph, kErrDq, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t st = base + s * L::STAGE;
        // packed row r: 32 bytes in the 32-byte swizzle (16-byte chunk c at c ^ ((r >> 2) & 1))
        uint32_t w8[8];
        const uint32_t prow = st + L::X + r * 32, sw = (uint32_t)((r >> 2) & 1) << 4;
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(w8[0]), "=r"(w8[1]), "=r"(w8[2]), "=r"(w8[3]) : "r"(prow + sw));
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(w8[4]), "=r"(w8[5]), "=r"(w8[6]), "=r"(w8[7]) : "r"(prow + (sw ^ 16)));
        uint32_t o[32];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const float z = ASYM ? zc[hh] : 8.f;
          const bool zint = !ASYM || (z == rintf(z) && fabsf(z) < 4194304.f);
          const uint64_t s2 = f2(sc[hh], sc[hh]), negzc2 = f2(-(8388608.f + z), -(8388608.f + z)),
                         negz2 = f2(-z, -z);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t oc[4];
            if (zint) dequant8<true>(w8[4 * hh + c], !ASYM, negzc2, negz2, s2, oc);
            else dequant8<false>(w8[4 * hh + c], !ASYM, negzc2, negz2, s2, oc);
#pragma unroll
            for (int e = 0; e < 4; ++e) o[16 * hh + 4 * c + e] = oc[e];
          }
        }
        tmem_st32(tmem + ((uint32_t)(32 * q) << 16) + L::A_COL + 32 * s, o);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) bar_arrive(dq0 + 8 * s);
      }
    }
  } else {
    // ---------------- epilogue: TMEM -> Y ----------------
    // Warp q reads TMEM lanes 32q.. = weight rows; each register column is a
    // token.  With TMA stores (p.tma_store): every 32-token chunk is written
    // into a [32 tokens][128 rows] staging tile (lane = row: conflict-free)
    // and stored by one TMA bulk copy that clips rows past N and tokens past
    // T; two staging tiles alternate.  Otherwise each warp store writes 32
    // consecutive outputs of one token row.
    const int q = warp;
    const int es = p.ydt == SF_F32 ? 4 : 2;
    int local = 0, chunk = 0;
    for (int tile = blockIdx.x; tile < ntiles_total; tile += gridDim.x, ++local) {
      const int m0 = (tile % p.mtiles) * BT, n0 = (tile / p.mtiles) * 128, n = n0 + 32 * q + lane;
      const int b = L::NBUF == 2 ? (local & 1) : 0;
      const uint32_t use = L::NBUF == 2 ? (uint32_t)(local >> 1) : (uint32_t)local;
      if (!bar_wait(accf0 + 8 * b, use & 1, kErrEpi, abort_flag)) break;
      tc_fence_after();
      const bool nin = n < p.N;
      const float bv = (p.bias && nin) ? __ldg(p.bias + n) : 0.f;
#pragma unroll 1
      for (int c0 = 0; c0 < BT; c0 += 32, ++chunk) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * BT + c0), v);
        if (p.tma_store) {
          const uint32_t ob = out0 + (uint32_t)(chunk & 1) * L::OUT;
          // the store that last read this staging tile (two chunks ago) has finished reading it
          if (threadIdx.x == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          named_barrier_sync(1, 32 * kEpiWarps);
          const uint32_t rb = ob + (uint32_t)(32 * q + lane) * es;
          const uint32_t pitch = 128u * es;
          if (p.ydt == SF_F32) {
#pragma unroll
            for (int jj = 0; jj < 32; ++jj)
              asm volatile("st.shared.f32 [%0], %1;" ::"r"(rb + jj * pitch), "f"(v[jj] + bv) : "memory");
          } else if (p.ydt == SF_BF16) {
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) {
              const __nv_bfloat16 h = __float2bfloat16_rn(v[jj] + bv);
              asm volatile("st.shared.b16 [%0], %1;" ::"r"(rb + jj * pitch), "h"(*reinterpret_cast<const unsigned short*>(&h))
                           : "memory");
            }
          } else {
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) {
              const __half h = __float2half_rn(v[jj] + bv);
              asm volatile("st.shared.b16 [%0], %1;" ::"r"(rb + jj * pitch), "h"(*reinterpret_cast<const unsigned short*>(&h))
                           : "memory");
            }
          }
          fence_async_smem();
          named_barrier_sync(1, 32 * kEpiWarps);
          if (threadIdx.x == 0) tma_store_2d(&mapY, n0, m0 + c0, ob);
        } else if (nin) {
          const int t0 = m0 + c0;
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            if (t0 + jj < p.T) {
              const size_t o = (size_t)(t0 + jj) * p.N + n;
              const float y = v[jj] + bv;
              if (p.ydt == SF_F32) static_cast<float*>(p.Y)[o] = y;
              else if (p.ydt == SF_BF16) static_cast<__nv_bfloat16*>(p.Y)[o] = __float2bfloat16_rn(y);
              else static_cast<__half*>(p.Y)[o] = __float2half_rn(y);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(acce0 + 8 * b);
    }
    // every TMA store of this CTA has completed before the block exits
    if (threadIdx.x == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
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
      return fail(SF_ERR_CAPTURE,
                  "prefill activation buffer must grow during stream capture: run the same shape once on the "
                  "capturing stream before capturing");
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

// Token-tile width: fewest tile rounds per SM, weighing a 128-token tile by
// its double dequant work per MAC (each weight tile is dequantized once per
// token tile) and a 256-token tile by its epilogue, which does not overlap
// the next tile's main loop (one accumulator buffer).
int choose_bt(int T, int N, int sms) {
  const long long nt = (N + 127) / 128;
  const long long r128 = ((T + 127) / 128 * nt + sms - 1) / sms;
  const long long r256 = ((T + 255) / 256 * nt + sms - 1) / sms;
  const double c128 = (double)r128 * 128 * 1.3, c256 = (double)r256 * 256 * 1.05;
  return (T > 128 && c256 <= c128) ? 256 : 128;
}

template <int BT, bool ASYM>
int launch_tc(const CUtensorMap& mx, const CUtensorMap& mw, const CUtensorMap& my, TcParams& p, int sms,
              cudaStream_t st) {
  using L = TcLayout<BT>;
  p.stages = L::S;
  auto* fn = q4_gemm_tc_kernel<BT, ASYM>;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::SMEM);
  if (e != cudaSuccess) return cuda_fail(e, "q4_gemm_tc_kernel smem attribute");
  const int tiles = p.mtiles * p.ntiles;
  const int grid = tiles < sms ? tiles : sms;
  fn<<<grid, kThreads, L::SMEM, st>>>(mx, mw, my, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "q4_gemm_tc_kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return SF_OK;
}

}  // namespace

int run_tc_gemm(const uint8_t* W, const float* S, const float* Z, const float* bias, const void* X, int xdt,
                void* Y, int ydt, int N, int K, int T, int gs, int flags, cudaStream_t stream) {
  (void)flags;
  if (T < kTcMinT) return SF_ERR_UNSUPPORTED;
  // Shapes this kernel takes: whole 64-k blocks, a group size that keeps each
  // 32-k half inside one group, 16-byte aligned weights and activations.
  if (K % kBK || gs % 32 || (gs & (gs - 1)) || ((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(X)) & 15))
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

  const int BT = choose_bt(T, N, di.sms);
  CUtensorMap mx, mw;
  if (!make_map(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, xb, (uint64_t)K, (uint64_t)T, (uint64_t)K * 2, kBK,
                (uint32_t)BT, CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(SF_ERR_CUDA, "cuTensorMapEncodeTiled failed for the prefill activations (T=%d K=%d)", T, K);
  if (!make_map(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, W, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2, kBK / 2,
                128, CU_TENSOR_MAP_SWIZZLE_32B))
    return fail(SF_ERR_CUDA, "cuTensorMapEncodeTiled failed for the prefill weights (N=%d K=%d)", N, K);

  TcParams p{};
  p.S = S; p.Z = Z; p.bias = bias; p.Y = Y;
  p.T = T; p.N = N; p.K = K; p.G = K / gs; p.gs = gs; p.lg2gs = __builtin_ctz((unsigned)gs); p.ydt = ydt;
  p.mtiles = (T + BT - 1) / BT;
  p.ntiles = (N + 127) / 128;
  p.kblocks = K / kBK;
  const bool asym = Z != nullptr;
  CUtensorMap my;
  const int ye = ydt == SF_F32 ? 4 : 2;
  p.tma_store = (reinterpret_cast<uintptr_t>(Y) & 15) == 0 &&
                ((size_t)N * ye) % 16 == 0 &&
                make_map(&my, ydt == SF_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                              : (ydt == SF_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16),
                         Y, (uint64_t)N, (uint64_t)T, (uint64_t)N * ye, 128, 32, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!p.tma_store) memset(&my, 0, sizeof(my));
  if (BT == 256)
    return asym ? launch_tc<256, true>(mx, mw, my, p, di.sms, stream)
                : launch_tc<256, false>(mx, mw, my, p, di.sms, stream);
  return asym ? launch_tc<128, true>(mx, mw, my, p, di.sms, stream)
              : launch_tc<128, false>(mx, mw, my, p, di.sms, stream);
}

}  // namespace sf
