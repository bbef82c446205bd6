// sf_q4_tile.cu -- decode GEMV (T <= 16 tokens) as independent warp work units
// on the sm_100a tensor cores, exact integer arithmetic.
//
// Reference semantics (siliconfer/kernels/neon/q4_gemv.cpp:37-140, 145-238;
// siliconfer/kernels/neon/__init__.py:88-124): per output row i and group g,
//   sym : y += s[i,g] * sum_k sext(q[i,k]) * x[k]
//   asym: y += s[i,g] * (sum_k q[i,k] * x[k] - z[i,g] * sum_k x[k])
//
// Arithmetic (the reference's algebra, exact where it can be):
//  * weights are UNSIGNED int8 A operands; symmetric nibbles are flipped
//    (u ^ 8 = q + 8) by the LOP3 that masks them, so both layouts become
//    s * (sum u*x - zeff * sum x) with zeff = 8 (sym) or z (asym);
//  * activations: per (token, group) x_fix = rint(x * 2^(22-E)), E the binary
//    exponent of the group's max |x| (the grid step is 2^-22 of the group
//    max), split into three signed int8 digits (x_fix = d0 + 256 d1 + 65536 d2).
//    Above 8 tokens two digits on a 2^(14-E) grid (rounding at most 2^-15 of
//    the group max, normwise about 1e-5 of y): they halve the MMAs.  Up to 8
//    tokens three are kept: two digits would miss the reference's own
//    elementwise test tolerances on its unit cases (1 and 4 tokens).
//  * mma.sync m16n8k32 u8 x s8 -> s32 sums u*d exactly.  Up to 2 tokens a
//    token's digits are adjacent B columns of one n tile (4 per token, the
//    fourth empty), so a lane's accumulator pair holds digits (0, 1) or
//    (2, -) of one token; each lane scales its pair and the two lanes of a
//    token are added once, at the end of the unit.  From 3 tokens on, n tile
//    2i holds digits (0, 1) and tile 2i + 1 digit 2 of tokens 4i .. 4i + 3, so
//    one lane holds all three digits of its token.  One fp32 epilogue per
//    (row, group, token[, lane]) recombines the digits, removes
//    zeff * sum(x_fix) and applies s * 2^(E-22).
//
// Work decomposition:
//  * A launch owns a list of tasks (GEMVs).  Each task is cut into units of
//    32 rows x one k-range; all units of all tasks form one global sequence.
//  * Every warp is independent: warp w takes units w, w + W, w + 2W, ...
//    (W = warps in the grid); there is no block-level synchronisation.  A warp
//    streams its unit through its own ring of shared-memory stages, each
//    guarded by its own mbarrier: lane 0 issues one TMA tile copy of the
//    weights (32 rows x one k-segment, straight from the reference's row-major
//    [N, K/2] bytes) and one bulk copy of the segment's activation block.
//  * Activations are converted once per task into that block layout (digits
//    in MMA B-fragment order, then the group scales 2^(E-22) and sums), by a
//    pre-pass kernel for tasks whose input exists at launch, and otherwise in
//    parallel by the warps that reach the task, in 32-octet chunks.
//  * A unit that covers part of K writes fp32 partial sums; the last unit of
//    a 32-row tile to finish (per-tile arrival counter) adds the partials in
//    k order -- deterministic -- and writes Y.
//  * Dependencies (a task that reads what earlier tasks wrote) are phases: a
//    warp starting a unit of a later phase first issues its first stages'
//    weight copies (they do not depend on anything), then waits until every
//    tile of the previous phase has been written (per-CTA flag lines) and the
//    phase's inputs converted.  All warps are resident (cooperative launch)
//    and take units in increasing order, so a wait never blocks a unit it
//    depends on.  Waits are bounded.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include <algorithm>
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

// Stages per warp ring: 3; 2 above 4 tokens, whose activation blocks are
// as large as a stage's weights or larger (so that 8 warps per CTA, or 6
// above 8 tokens, still fit in shared memory).
__host__ __device__ constexpr int tile_kd(int T) { return T > 4 ? 2 : 3; }
constexpr int kUnitRows = 32;          // rows per unit (two m16 tiles)
constexpr int kEpiSwiGLU = 1;          // TileTask::epi
constexpr int kRedTiles = 4;           // 32-row tiles summed by one unit of an all-reduce task
// At most 12 warps per CTA (168 registers per thread); more than 4 tokens
// doubles the accumulators, and those launches hold at most 8 warps (their
// stages are larger) with 255 registers per thread.
__host__ __device__ constexpr int tile_max_threads(int T) { return T > 4 ? 256 : 384; }
// Segments whose loads, nibble splits and MMAs are interleaved (one
// accumulator set each): two up to 8 tokens, one above (registers).
__host__ __device__ constexpr int tile_pair(int T) { return T <= 8 ? 2 : 1; }

// Bytes of one segment's activation block: [T][3 digits][4 lanes][2*LB] digit
// bytes, then [T] x (group scale 2^(E-22), sum of x_fix) as two fp32.
__host__ __device__ constexpr int tile_nd(int T) { return T > 8 ? 2 : 3; }   // activation digits
__host__ __device__ constexpr int xblock_bytes(int T, int LB) { return (T * (8 * tile_nd(T) * LB + 8) + 15) & ~15; }

// Shared memory of a CTA: first the weight stages of every warp (1024-byte
// aligned, as the 128-byte TMA swizzle needs), then each warp's other areas.
// One stage = 32 rows x 128 bytes of W (256 k at 4 bits, 512 k at 2 bits) =
// SPS k-segments of 8*LB k (LB: activation bytes per lane and digit).
template <int T, bool ASYM, int LB, int BITS>
struct TileLayout {
  static constexpr int SPS = 128 / (LB * BITS);         // k-segments per stage
  static constexpr int XB = xblock_bytes(T, LB);         // activation block of one segment
  static constexpr int ASTAGE = 32 * 128;                // weight tile of one stage
  static constexpr int SBW = LB == 4 ? 8 : 4;            // groups in one stage's scale box
  static constexpr int SBYTES = 32 * SBW * 4;            // [32 rows][SBW] fp32
  static constexpr int XSTAGE = (SPS * XB + 127) & ~127;
  static constexpr int kD = tile_kd(T);
  // per-warp area: [mbarriers 64 B][zeros 64 B][kD x activations][kD x scales][kD x zeros]
  static constexpr int XOFF = 128;
  static constexpr int SOFF = XOFF + kD * XSTAGE;
  static constexpr int ZOFF = SOFF + kD * SBYTES;
  static constexpr int MISC = ZOFF + (ASYM ? kD * SBYTES : 0);
  static constexpr int WARP = kD * ASTAGE + MISC;        // shared bytes per warp
};

// Rows of a 32-row unit held by lane group g (slot i: tile i>>1, +8 when i is
// odd).  With 128-byte swizzled rows (16-byte chunk c of row r stored at
// c ^ (r & 7)), the rows that one shared-memory phase of fragment loads reads
// must land on different banks: for LB=16 the two rows of a phase differ in
// bit 2, for LB=8 the four rows differ in bits 1-2, for LB=4 any order works.
__device__ __forceinline__ int lane_row(int g, int LB) {
  return LB == 16 ? ((g >> 1) | ((g & 1) << 2)) : (LB == 8 ? (((g & 3) << 1) | (g >> 2)) : g);
}

// One GEMV of a launch.  The tensor maps come first (64-byte aligned).
struct alignas(64) TileTask {
  CUtensorMap tmW;    // packed weights [N][K/2] u8, box {SEGK/2, 32}
  CUtensorMap tmS;    // scales [N][G] f32, box {4, 32} (when stma)
  CUtensorMap tmZ;    // zeros, same
  const uint8_t* W;
  const float* S;
  const float* Z;
  const float* bias;
  const void* X;
  void* Y;
  uint8_t* xd;        // activation blocks, one per k-segment
  float* part;        // k-split partial sums [ksplit][T][N] (ksplit > 1)
  unsigned int* tcnt; // per-tile arrival counters (ksplit > 1)
  long long ubase;    // index of the task's first unit in the launch
  int N, K, G, lg2gs, xdt, ydt;
  int ntile, ksplit, kper;   // 32-row tiles, k-splits, k per split (whole groups)
  int xpre;                  // activation blocks were written by the pre-pass
  int stma;                  // scales (and zeros) by TMA; else per-lane copies
  int nchunk;                // 32-octet conversion chunks
  // Phase of this task: a run of tasks that read X only after the previous
  // phase has written all its tiles.  Phase 0 reads inputs that exist at launch.
  int phase, ph_first, ph_tiles, ph_chunks, ph_last;
  int ph_cbase;              // the phase's first entry in the launch's chunk map
  long long ph_ubase, ph_units;
  // Tensor-parallel exchange (row-parallel projections), see sf_q4_step_create_tp:
  //  kind 0: GEMV; push != 0: its fp32 tiles go to every rank's exchange
  //          region (data[parity][src rank][T][N]) instead of Y, each tile
  //          followed by flag[tile][src] = launch epoch in every rank;
  //  kind 1: all-reduce of a pushed task: waits for flag[tile][*] >= epoch in
  //          this rank's region, sums the ranks in order (+ bias), writes Y.
  int kind, push, tp_rank, tp_world;
  int epi;                             // kEpiSwiGLU: interleaved gate/up rows, Y = silu(gate) * up
  size_t xpar;                         // bytes of one parity half of a region's data
  uint8_t* xdata[8];                   // region data of every rank, as mapped here
  unsigned long long* xflag[8];        // region flags of every rank, as mapped here
};

struct TileLaunch {
  TileTask single;        // used when `tasks` is null
  const TileTask* tasks;  // device table
  unsigned int* phctr;    // per phase: [tiles written, chunks converted, -, -] or null
  unsigned int* flags;    // per CTA, one 128-byte line: [phases written, phases converted]
  long long total;        // units in the launch
  int ntasks;
  unsigned long long* epoch;   // last finished launch (tensor-parallel exchange epoch), or null
  unsigned int* done;          // CTAs finished (step launches: the last one resets the counters), or null
  const unsigned int* cmap;    // per phase, its conversion chunks in order: (task << 16) | chunk of the task
  const long long* ubase;      // first unit of every task, compact (read through L1), or null: single task
  int nphase;                  // phases of the step (phctr has 4 words per phase)
  unsigned long long* poison;  // the communicator's sticky poison word (tensor-parallel steps), or null
};

__device__ __forceinline__ const TileTask* tile_task(const TileLaunch& L, int i) {
  return L.tasks ? L.tasks + i : &L.single;
}

// ---- PTX wrappers -----------------------------------------------------------
__device__ __forceinline__ void bar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// Arrives on `bar` once every cp.async this thread issued so far has landed;
// the barrier's expected count is raised by one first, so the arrival does
// not count against the count it was initialised with.
__device__ __forceinline__ void bar_arrive_cpasync(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool bar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity, unsigned int code) {
  if (bar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!bar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) {
      atomicOr(&g_dev_error, code);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void bulk_copy(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void cpa4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
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

__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Bounded spin on a global counter (one thread).  false on timeout.
__device__ __forceinline__ bool spin_geq(const unsigned int* p, unsigned int target, unsigned int code) {
  if (ld_acquire(p) >= target) return true;
  const long long t0 = clock64();
  while (ld_acquire(p) < target) {
    if (clock64() - t0 > kWaitCycles) {
      atomicOr(&g_dev_error, code);
      return false;
    }
    __nanosleep(64);
  }
  return true;
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

// SwiGLU activation of the gate: silu(x) = x / (1 + e^-x)
// (siliconfer/model/layers.py:144, down_proj(silu(gate(x)) * up(x))).
__device__ __forceinline__ float silu(float x) { return x / (1.f + expf(-x)); }

// D (+)= A(u8, 16x32) * B(s8, 32x8), s32.  Not volatile: no side effects, so
// the compiler may interleave independent chains.
__device__ __forceinline__ void imma(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                     uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void imma0(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                      uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

template <bool ASYM>
__device__ __forceinline__ uint32_t nib_lo(uint32_t w) {
  return (w & 0x0F0F0F0Fu) ^ (ASYM ? 0u : 0x08080808u);
}
template <bool ASYM>
__device__ __forceinline__ uint32_t nib_hi(uint32_t w) {
  return ((w >> 4) & 0x0F0F0F0Fu) ^ (ASYM ? 0u : 0x08080808u);
}
// 2-bit field f (0..3) of each byte as unsigned bytes; the symmetric layout's
// two's-complement q in [-2, 1] becomes q + 2 (flip of the field's top bit).
template <bool ASYM>
__device__ __forceinline__ uint32_t fld2(uint32_t w, int f) {
  return ((w >> (2 * f)) & 0x03030303u) ^ (ASYM ? 0u : 0x02020202u);
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

// Fixed-point digit split of 8 activations of one lane; lanes in aligned
// blocks of `lpg` form one quantization group.  d[i][j]: digit i of input j.
template <int ND>
__device__ __forceinline__ void digits8_raw(const float* v, int lpg, int (&d)[3][8], float& gsc_out,
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
  // biased binary exponent `be` of the group max m: m < 2^(be-126), so
  // x * 2^(126+F-be) stays within +-2^F: three int8 digits for F = 22, two for
  // F = 14 (d1 = (x_fix - d0) / 256 lies in [-64, 64]).  Groups whose max is
  // below 2^-105 are zero.
  constexpr int F = ND == 3 ? 22 : 14;
  const int be = (int)(__float_as_uint(m) >> 23);
  const bool zero = bad || be < 22;
  const float scl = zero ? 0.f : __uint_as_float((uint32_t)(253 + F - be) << 23);   // 2^(126+F-be)
  int s = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int xf = __float2int_rn(v[j] * scl);
    s += xf;
    const int d0 = (xf << 24) >> 24;
    const int r1 = (xf - d0) >> 8;
    d[0][j] = d0;
    if constexpr (ND == 3) {
      const int d1 = (r1 << 24) >> 24;
      d[1][j] = d1;
      d[2][j] = (r1 - d1) >> 8;
    } else {
      d[1][j] = r1;
      d[2][j] = 0;
    }
  }
  for (int off = 1; off < lpg; off <<= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  gsc_out = bad ? __int_as_float(0x7fc00000)
                : (zero ? 0.f : __uint_as_float((uint32_t)(be + 1 - F) << 23));   // 2^(be-126-F)
  sum_out = s;
}

// Converts chunk `c` (32 consecutive octets of the [T][K] input) of a task
// into its activation blocks.  Called by a whole warp.
//
// Byte order of a lane's digits (each 8-byte run = one MMA k-step's two B
// words), matching how the kernel unpacks the packed weights:
//  * 4 bits: octet j (k 8j .. 8j+7) -> words {0,2,4,6}, {1,3,5,7} (the low and
//    high nibbles of 4 packed bytes);
//  * 2 bits: a 16-k block (octets 2q, 2q+1) -> 4 words, word r = k {r, r+4,
//    r+8, r+12} (the 2-bit field r of 4 packed bytes); the two lanes of a
//    block swap half-words and write 8 bytes each.
template <int T, int LB, int BITS>
__device__ __forceinline__ void convert_chunk(const TileTask* p, int c, int lane) {
  constexpr int SEGK = 8 * LB, XB = xblock_bytes(T, LB);
  const int K = p->K, lg2gs = p->lg2gs;
  const int octs = K >> 3, total = T * octs;
  const int lpg = 1 << (lg2gs - 3);
  const int o = c * 32 + lane;
  const bool ok = o < total;
  const int tok = ok ? o / octs : 0;
  const int oo = ok ? o - tok * octs : 0;
  float v[8];
  if (ok) ld_x8(p->X, (size_t)tok * K + (size_t)oo * 8, p->xdt, v);
  else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = 0.f;
  }
  constexpr int ND = tile_nd(T);
  uint2 dig[ND];
  float gsc;
  int s;
  {
    int d[3][8];
    digits8_raw<ND>(v, lpg, d, gsc, s);
    if constexpr (BITS == 4) {
#pragma unroll
      for (int i = 0; i < ND; ++i) dig[i] = pack_digits(d[i]);
    } else {
      const bool odd = (lane & 1) != 0;   // second octet of a 16-k block
#pragma unroll
      for (int i = 0; i < ND; ++i) {
        uint32_t hw[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) hw[r] = (uint32_t)(d[i][r] & 255) | ((uint32_t)(d[i][4 + r] & 255) << 8);
        // the even lane keeps words 0-1 and sends 2-3, the odd lane the reverse
        const uint32_t mine0 = odd ? (hw[2] | hw[3] << 16) : (hw[0] | hw[1] << 16);
        const uint32_t send = odd ? (hw[0] | hw[1] << 16) : (hw[2] | hw[3] << 16);
        const uint32_t got = __shfl_xor_sync(0xffffffffu, send, 1);
        // word r = [k r, r+4 from the even lane][k r+8, r+12 from the odd lane]
        const uint32_t lo = odd ? got : mine0, hi = odd ? mine0 : got;
        dig[i].x = (lo & 0xFFFFu) | (hi << 16);
        dig[i].y = (lo >> 16) | (hi & 0xFFFF0000u);
      }
    }
  }
  if (!ok) return;
  const int k0 = oo * 8;
  const int seg = k0 / SEGK, within = k0 - seg * SEGK;
  const int tt = within / (2 * LB), j = (within - tt * 2 * LB) >> 3;
  uint8_t* blk = p->xd + (size_t)seg * XB;
#pragma unroll
  for (int dg = 0; dg < ND; ++dg)
    *reinterpret_cast<uint2*>(blk + ((tok * ND + dg) * 4 + tt) * 2 * LB + j * 8) = dig[dg];
  if ((lane & (lpg - 1)) == 0) {
    // every segment of the group carries the group's scale and sum
    const int gs = 1 << lg2gs;
    const int s0 = ((k0 >> lg2gs) << lg2gs) / SEGK;
    const float2 gv = make_float2(gsc, (float)s);
    for (int sg = s0; sg < s0 + gs / SEGK; ++sg)
      *reinterpret_cast<float2*>(p->xd + (size_t)sg * XB + T * 8 * ND * LB + tok * 8) = gv;
  }
}

// Writes `val` into word `word` of every CTA's flag line (whole warp).
__device__ __forceinline__ void publish(unsigned int* flags, int word, unsigned int val, int lane) {
  __threadfence();
  for (int c = lane; c < (int)gridDim.x; c += 32)
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(flags + c * 32 + word), "r"(val) : "memory");
}

__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long launch_epoch(const TileLaunch& L) {
  return *reinterpret_cast<volatile const unsigned long long*>(L.epoch);
}
// One fp32 value of a pushed task's tile into every rank's region (peer stores).
__device__ __forceinline__ void push_val(const TileTask* p, unsigned long long ep, int T, int tok, int row, float v) {
  const size_t off = (size_t)(ep & 1) * p->xpar + (((size_t)p->tp_rank * T + tok) * p->N + row) * 4;
  for (int q = 0; q < p->tp_world; ++q) __stcg(reinterpret_cast<float*>(p->xdata[q] + off), v);
}
// The warp's pushes of one tile are complete: flag it in every rank (whole warp).
// The warp barrier orders every lane's pushes before the flag lanes' stores,
// and a system-scope release makes them visible to a peer that acquires the
// flag (release is cumulative over the stores ordered before it).
__device__ __forceinline__ void push_flag(const TileTask* p, unsigned long long ep, int tile, int lane) {
  __syncwarp();
  if (lane < p->tp_world) st_release_sys_u64(p->xflag[lane] + (size_t)tile * p->tp_world + p->tp_rank, ep);
  __syncwarp();
}

// A 32-row tile of task p has been written (whole warp): count it towards its
// phase; the tile that completes the phase tells every CTA.
__device__ __forceinline__ void tile_written(const TileLaunch& L, const TileTask* p, int lane) {
  if (!L.phctr || p->ph_last) return;
  __threadfence();
  __syncwarp();
  unsigned int old = 0;
  if (lane == 0) old = atomicAdd(L.phctr + 4 * p->phase, 1u);
  old = __shfl_sync(0xffffffffu, old, 0);
  if (old + 1 == (unsigned)p->ph_tiles) publish(L.flags, 0, (unsigned)p->phase + 1, lane);
}

}  // namespace

// ---------------------------------------------------------------------------
// The GEMV kernel
// ---------------------------------------------------------------------------
template <int T, bool ASYM, int LB, int BITS>
__global__ void __launch_bounds__(tile_max_threads(T), 1)
    q4_tile_kernel(const __grid_constant__ TileLaunch L) {
  using Ly = TileLayout<T, ASYM, LB, BITS>;
  // CMP (T <= 2): one n tile, token t in columns 4t .. 4t + 3 (digits 0-2, empty);
  // 3..8 tokens: NG groups of 4 tokens, n tiles (2i, 2i + 1) = digits (0, 1) and 2
  // of group i; 9..16 tokens: two digits, n tile i = digits (0, 1) of group i
  constexpr bool CMP = T <= 2;
  constexpr int ND = tile_nd(T), NG = CMP ? 1 : (T + 3) / 4, NT = CMP ? 1 : (ND == 3 ? 2 * NG : NG);
  constexpr int WPL = LB / 4, SEGK = 8 * LB, SPS = Ly::SPS, PS = tile_pair(T);
  constexpr int LBA = LB * BITS / 4;             // packed weight bytes of a lane's row slice per segment
  constexpr int KST = SPS * SEGK;                // k of one stage (128 bytes of every row)
  constexpr int GOFF = T * 8 * ND * LB;          // group scales / sums inside a segment's block
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int wpc = blockDim.x >> 5;
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem);
  if (sbase & 1023) {   // the swizzled TMA tiles need 1024-byte alignment
    if (threadIdx.x == 0) atomicOr(&g_dev_error, 0x800u);
    return;
  }
  constexpr int kD = Ly::kD;
  const uint32_t astage0 = sbase + (uint32_t)warp * kD * Ly::ASTAGE;
  const uint32_t wb = sbase + (uint32_t)wpc * kD * Ly::ASTAGE + (uint32_t)warp * Ly::MISC;
  const uint32_t bar0 = wb, zblk = wb + 64, xstage0 = wb + Ly::XOFF, sstage0 = wb + Ly::SOFF,
                 zstage0 = wb + Ly::ZOFF;

  // one arrival per stage: lane 0's expect_tx.  Per-lane scale copies add
  // their own (cp.async.mbarrier.arrive raises the expected count first).
  if (lane < kD) bar_init(bar0 + lane * 8, 1);
  if (lane < 16) asm volatile("st.shared.u32 [%0], %1;" ::"r"(zblk + lane * 4), "r"(0u) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();

  // B fragment sources: column g of tile nt is (token, digit) or absent.
  // Accumulator columns 2t, 2t+1 of a lane are then (CMP) digits (0, 1) or
  // (2, -) of token t >> 1, else digits (0, 1) of token 4i + t in tile 2i and
  // digit 2 of the same token in tile 2i + 1.
  int bslot[NT];
  bool bval[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    int tok, dg;
    if (CMP) {
      tok = g >> 2;
      dg = g & 3;
    } else if (ND == 3) {
      tok = (nt >> 1) * 4 + (g >> 1);
      dg = (nt & 1) ? ((g & 1) ? 3 : 2) : (g & 1);
    } else {
      tok = nt * 4 + (g >> 1);
      dg = g & 1;
    }
    bval[nt] = tok < T && dg < ND;
    bslot[nt] = bval[nt] ? ((tok * ND + dg) * 4 + t) * 2 * LB : 0;
  }
  const int ltok = CMP ? (t >> 1) : t;            // this lane's token inside a group
  const bool dlead = CMP ? (t & 1) == 0 : true;   // holds digits (0, 1): carries zeff * sum(x)
  const float lmul = dlead ? 1.f : 65536.f;       // weight of the lane's digit pair (CMP)
  // rows of this lane inside a unit and their byte offsets in a swizzled stage
  int rloc[4];
  uint32_t aoff[4][SPS];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    rloc[i] = (i >> 1) * 16 + lane_row(g, LB) + 8 * (i & 1);
#pragma unroll
    for (int sub = 0; sub < SPS; ++sub) {
      const int b = sub * 4 * LBA + t * LBA;   // byte of the row this lane reads for segment `sub`
      aoff[i][sub] = (uint32_t)(rloc[i] * 128 + ((((b >> 4) ^ (rloc[i] & 7)) << 4) | (b & 15)));
    }
  }

  const long long W_all = (long long)gridDim.x * (blockDim.x >> 5);
  // this launch's exchange epoch: one more than the last finished launch's
  const unsigned long long ep = L.epoch ? launch_epoch(L) + 1 : 0ull;
  if (L.poison && *reinterpret_cast<volatile const unsigned long long*>(L.poison)) {
    // An earlier step gave up on a peer: compute nothing, and poison every
    // pushed tile's flag in every peer so that their reduce tasks fail at once.
    if (warp == 0 && blockIdx.x == 0 && lane == 0) atomicOr(&g_dev_error, kErrPoisoned);
    for (int ti2 = 0; ti2 < L.ntasks; ++ti2) {
      const TileTask* p = tile_task(L, ti2);
      if (!p->push) continue;
      for (long long t2 = (long long)warp * gridDim.x + blockIdx.x; t2 < p->ntile; t2 += W_all)
        if (lane < p->tp_world)
          st_release_sys_u64(p->xflag[lane] + (size_t)t2 * p->tp_world + p->tp_rank, kFlagPoison);
    }
    return;
  }
  uint32_t cslot = 0, cpar = 0;   // this warp's ring: next slot to consume and its phase parity
  int seen_phase = -1;            // last phase whose inputs this warp has seen converted
  int ti = 0;
  bool ok = true;

  for (long long u = (long long)warp * gridDim.x + blockIdx.x; u < L.total && ok; u += W_all) {
    while (ti + 1 < L.ntasks && u >= __ldg(L.ubase + ti + 1)) ++ti;
    const TileTask* p = tile_task(L, ti);
    const int N = p->N, K = p->K, G = p->G, lg2gs = p->lg2gs, ntile = p->ntile;
    const int ksplit = p->ksplit, kper = p->kper, stma = p->stma;
    const int lu = (int)(u - p->ubase);
    const int tile = lu % ntile, ks = lu / ntile;
    const int r0 = tile * kUnitRows;
    const int kb = ks * kper;
    const int ke = min(K, kb + kper);
    const int nseg = (ke - kb) / SEGK;
    const int g0 = kb >> lg2gs, gend = ke >> lg2gs;
    const int lg2spg = lg2gs - (31 - __clz(SEGK));   // segments per group = 1 << lg2spg
    const int spg_mask = (1 << lg2spg) - 1;

    // ---- operand streaming (set-up) ------------------------------------------
    // Stage j holds k [kb + 256 j, kb + 256 j + 256): the weight tile, the
    // activation blocks of its segments and the scale box of its groups.
    // Ring position: `cslot` / `cpar` are the slot and phase parity of the
    // next stage to consume, `islot` the slot of the next stage to issue.
    const int nstage = (nseg + SPS - 1) / SPS;
    const uint8_t* xsrc = p->xd + (size_t)(kb / SEGK) * Ly::XB;
    const float* Sb = p->S;
    const float* Zb = p->Z;
    uint32_t islot = cslot;
    // issue_w: the stage's barrier expectation (weights, scales AND activations)
    // and its weight / scale copies; issue_x: its activation copy.  Weights do
    // not depend on earlier tasks, so a unit that must wait for its inputs
    // starts its first stages' weights before the wait.
    auto slot_of = [&](int j) {   // ring slot of stage j of this unit
      const uint32_t s2 = cslot + (uint32_t)j;
      return s2 >= (uint32_t)kD ? s2 - kD : s2;
    };
    auto issue_w = [&](int j) {
      const uint32_t slot = islot;
      islot = islot + 1 == (uint32_t)kD ? 0u : islot + 1;
      const uint32_t bar = bar0 + slot * 8;
      const int nsub = min(SPS, nseg - j * SPS);
      const int fg = (kb + j * KST) >> lg2gs;                   // first group of the stage
      // scale box origin: TMA boxes start on SBW-group boundaries (units are
      // cut in whole boxes, so the stage's groups stay inside); per-lane
      // copies start at the stage's first group
      const int sx = stma ? (fg & ~(Ly::SBW - 1)) : fg;
      if (!stma) {
#pragma unroll
        for (int c = t; c < Ly::SBW; c += 4) {
          const int grp = sx + c;
          if (grp >= g0 && grp < gend) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int row = min(r0 + rloc[i], N - 1);
              const uint32_t o = (uint32_t)(rloc[i] * Ly::SBW + c) * 4;
              cpa4(sstage0 + slot * Ly::SBYTES + o, Sb + (size_t)row * G + grp);
              if (ASYM) cpa4(zstage0 + slot * Ly::SBYTES + o, Zb + (size_t)row * G + grp);
            }
          }
        }
        // each lane's copies count as one more arrival on the stage's barrier;
        // they are registered before lane 0's arrival below can end the phase
        bar_arrive_cpasync(bar);
        __syncwarp();
      }
      if (lane == 0) {
        const uint32_t sbytes = stma ? (uint32_t)Ly::SBYTES * (ASYM ? 2 : 1) : 0u;
        bar_expect_tx(bar, (uint32_t)Ly::ASTAGE + nsub * Ly::XB + sbytes);
        tma_2d(astage0 + slot * Ly::ASTAGE, &p->tmW, (kb * BITS >> 3) + j * 128, r0, bar);
        if (stma) {
          tma_2d(sstage0 + slot * Ly::SBYTES, &p->tmS, sx, r0, bar);
          if (ASYM) tma_2d(zstage0 + slot * Ly::SBYTES, &p->tmZ, sx, r0, bar);
        }
      }
    };
    auto issue_x = [&](int j, uint32_t slot) {
      const int nsub = min(SPS, nseg - j * SPS);
      if (lane == 0) {
        bulk_copy(xstage0 + slot * Ly::XSTAGE, xsrc + (size_t)j * SPS * Ly::XB, nsub * Ly::XB, bar0 + slot * 8);
      }
    };
    const int npro = min(kD - 1, nstage);   // stages issued before the main loop
    // a wait that expired after issue_w: complete and wait out the copies in
    // flight (bounded) so that none lands after the CTA has exited
    auto drain = [&]() {
      for (int j = 0; j < npro; ++j) issue_x(j, slot_of(j));
      for (int j = 0; j < npro; ++j) {
        const uint32_t sl = slot_of(j);
        bar_wait(bar0 + sl * 8, cpar ^ (sl < cslot ? 1u : 0u), 0x10u);
      }
    };
    const bool gemv = p->kind == 0;
    if (gemv) {
      __syncwarp();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      for (int j = 0; j < npro; ++j) issue_w(j);
    }
    // ---- dependencies and activation blocks --------------------------------
    // A warp takes its units in increasing order and phases never go back, so
    // only its first unit of a phase waits (and converts its share); the later
    // ones find the phase's inputs ready.
    if (!p->xpre && p->phase > seen_phase) {
      const int ph = p->phase;
      seen_phase = ph;
      const unsigned int* fl = L.flags + blockIdx.x * 32;
      int okw = 1;
      if (lane == 0) okw = spin_geq(fl, (unsigned)ph, 0x200u);   // previous phase written
      ok = __shfl_sync(0xffffffffu, okw, 0) != 0;
      if (!ok) {
        if (gemv) drain();
        break;
      }
      // The first units of the phase convert its inputs: unit i takes chunks
      // i, i + CS, ... over all tasks of the phase.  Every warp has at most
      // one such unit per phase and reaches it before any other unit of the
      // phase, so no converting warp waits on its own conversion.
      const long long CS = min(W_all, p->ph_units);
      const long long i = u - p->ph_ubase;
      if (i < CS && i < p->ph_chunks) {
        int n = 0;
        for (long long c = i; c < p->ph_chunks; c += CS) {
          const unsigned int e = __ldg(L.cmap + p->ph_cbase + c);
          convert_chunk<T, LB, BITS>(tile_task(L, (int)(e >> 16)), (int)(e & 0xFFFFu), lane);
          ++n;
        }
        asm volatile("fence.proxy.async.global;" ::: "memory");
        __threadfence();
        __syncwarp();
        unsigned int old = 0;
        if (lane == 0) old = atomicAdd(L.phctr + 4 * ph + 1, (unsigned)n);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old + n == (unsigned)p->ph_chunks) publish(L.flags, 1, (unsigned)ph + 1, lane);
      }
      int okx = 1;
      if (lane == 0 && p->ph_chunks > 0) {   // (a phase with nothing to convert has no such flag)
        okx = spin_geq(fl + 1, (unsigned)ph + 1, 0x400u);            // this phase's inputs converted
        asm volatile("fence.proxy.async.global;" ::: "memory");
      }
      ok = __shfl_sync(0xffffffffu, okx, 0) != 0;
      if (!ok) {
        if (gemv) drain();
        break;
      }
    }

    if (p->kind == 1) {
      // ---- all-reduce of a pushed task: unit lu sums kRedTiles 32-row tiles ----
      // lane l polls the flag of tile 4 lu + l / world from rank l % world
      const int W_ = p->tp_world, ntl = (N + kUnitRows - 1) / kUnitRows;
      const int t32 = lu * kRedTiles + lane / W_, src_rank = lane % W_;
      const bool poll = lane < kRedTiles * W_ && t32 < ntl;
      int okf = 1;
      if (poll) {
        const unsigned long long* fl = p->xflag[p->tp_rank] + (size_t)t32 * W_ + src_rank;
        unsigned long long v = ld_acquire_sys_u64(fl);
        const long long t0 = clock64();
        while (v < ep) {
          if (clock64() - t0 > kWaitCycles) {
            atomicOr(&g_dev_error, 0x2000u);
            okf = 0;
            break;
          }
          __nanosleep(32);
          v = ld_acquire_sys_u64(fl);
        }
        if (v == kFlagPoison) {   // that rank gave up on an earlier step
          atomicOr(&g_dev_error, kErrPoisoned);
          okf = 0;
        }
      }
      // the acquiring lanes' loads are ordered before the other lanes' reads below
      __syncwarp();
      ok = __all_sync(0xffffffffu, okf) != 0;
      if (!ok) {
        // the ranks are out of step for good: poison the communicator and these
        // tiles' flags in every peer, so that no peer sums a stale region
        if (lane == 0 && L.poison) *reinterpret_cast<volatile unsigned long long*>(L.poison) = 1ull;
        if (poll) {
          __threadfence_system();
          st_release_sys_u64(p->xflag[src_rank] + (size_t)t32 * W_ + p->tp_rank, kFlagPoison);
        }
        break;
      }
      const float* src = reinterpret_cast<const float*>(p->xdata[p->tp_rank] + (size_t)(ep & 1) * p->xpar);
#pragma unroll 1
      for (int i = 0; i < kRedTiles; ++i) {
        const int row = (lu * kRedTiles + i) * kUnitRows + lane;
        if (row >= N) break;
        const float bv = p->bias ? __ldg(p->bias + row) : 0.f;
        for (int tok = 0; tok < T; ++tok) {
          float v[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) v[q] = q < W_ ? __ldcv(src + ((size_t)q * T + tok) * N + row) : 0.f;
          float a2 = 0.f;
#pragma unroll
          for (int q = 0; q < 8; ++q) a2 += v[q];   // rank order: every rank gets the same bits
          st_y(p->Y, (size_t)tok * N + row, a2 + bv, p->ydt);
        }
      }
      tile_written(L, p, lane);
      continue;
    }
    for (int j = 0; j < npro; ++j) issue_x(j, slot_of(j));

    float acc[2][NG][2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int tg = 0; tg < NG; ++tg) acc[mt][tg][0] = acc[mt][tg][1] = 0.f;
    int C[PS][2][NT][4];   // [segment of the pair][m tile][n tile][fragment]: one segment's sums
    int carry[2][NT][4];   // sums of the earlier segments of a group longer than one segment

    // epilogue of the group that ends with segment s: recombine the digits,
    // remove zeff * sum(x), scale.  Lanes whose token does not exist compute
    // on token T-1 and never store.
    auto epilogue = [&](const int (&Cs)[2][NT][4], int s, uint32_t xs0, uint32_t sst, uint32_t zst, int sx) {
      const uint32_t soff = (uint32_t)(((kb + s * SEGK) >> lg2gs) - sx) * 4;   // inside the stage's box
      float sc[2][2], zp[2][2];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = rloc[2 * mt + h];
          sc[mt][h] = __uint_as_float(lds32(sst + r * (Ly::SBW * 4) + soff));
          zp[mt][h] = ASYM ? __uint_as_float(lds32(zst + r * (Ly::SBW * 4) + soff)) : (BITS == 4 ? 8.f : 2.f);
        }
#pragma unroll
      for (int tg = 0; tg < NG; ++tg) {
        const uint2 xv = lds64(xs0 + GOFF + min(tg * 4 + ltok, T - 1) * 8);
        const float gsc = __uint_as_float(xv.x), xsum = dlead ? __uint_as_float(xv.y) : 0.f;
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float v;
            if (CMP) {
              v = lmul * (float)(Cs[mt][0][2 * h] + 256 * Cs[mt][0][2 * h + 1]);
            } else if (ND == 2) {
              v = (float)(Cs[mt][tg][2 * h] + 256 * Cs[mt][tg][2 * h + 1]);
            } else {
              const int i01 = Cs[mt][2 * tg][2 * h] + 256 * Cs[mt][2 * tg][2 * h + 1];
              v = fmaf(65536.f, (float)Cs[mt][2 * tg + 1][2 * h], (float)i01);
            }
            const float f = fmaf(-zp[mt][h], xsum, v);
            acc[mt][tg][h] = fmaf(f, sc[mt][h] * gsc, acc[mt][tg][h]);
          }
      }
    };

    for (int j = 0; j < nstage; ++j) {
      const uint32_t slot = cslot;
      const uint32_t ast = astage0 + slot * Ly::ASTAGE, xst = xstage0 + slot * Ly::XSTAGE;
      const uint32_t sst = sstage0 + slot * Ly::SBYTES, zst = zstage0 + slot * Ly::SBYTES;
      if (!bar_wait(bar0 + slot * 8, cpar, 0x10u)) {
        ok = false;
        break;
      }
      if (++cslot == (uint32_t)kD) {
        cslot = 0;
        cpar ^= 1u;
      }
      const int fgj = (kb + j * KST) >> lg2gs;
      const int sx = stma ? (fgj & ~(Ly::SBW - 1)) : fgj;
      // The stage's segments are taken in pairs (PS = 2) with one accumulator
      // set each, so that the two halves' loads, nibble splits and MMAs
      // interleave; one at a time (PS = 1) above 8 tokens.  Every segment's
      // sums start from zero; a group that spans several segments carries its
      // earlier segments' sums in `carry` (integers: exact).
#pragma unroll
      for (int pr = 0; pr < SPS; pr += PS) {
        const int s0 = j * SPS + pr;
        if (s0 >= nseg) break;
        uint32_t w[PS][4][LBA / 4];
        uint32_t bq[PS][NT][2 * WPL];
#pragma unroll
        for (int h2 = 0; h2 < PS; ++h2) {
          const uint32_t xs0 = xst + (pr + h2) * Ly::XB;
#pragma unroll
          for (int i = 0; i < 4; ++i) lds_n<LBA>(ast + aoff[i][pr + h2], w[h2][i]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) lds_n<2 * LB>(bval[nt] ? xs0 + bslot[nt] : zblk, bq[h2][nt]);
        }
#pragma unroll
        for (int q = 0; q < WPL; ++q)
#pragma unroll
          for (int h2 = 0; h2 < PS; ++h2)
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
              uint32_t a0, a1, a2, a3;
              if constexpr (BITS == 4) {
                a0 = nib_lo<ASYM>(w[h2][2 * mt][q]);
                a2 = nib_hi<ASYM>(w[h2][2 * mt][q]);
                a1 = nib_lo<ASYM>(w[h2][2 * mt + 1][q]);
                a3 = nib_hi<ASYM>(w[h2][2 * mt + 1][q]);
              } else {
                // 2-bit fields 2f, 2f + 1 of packed word q / 2 (16 weights)
                const int f = 2 * (q & 1);
                a0 = fld2<ASYM>(w[h2][2 * mt][q >> 1], f);
                a2 = fld2<ASYM>(w[h2][2 * mt][q >> 1], f + 1);
                a1 = fld2<ASYM>(w[h2][2 * mt + 1][q >> 1], f);
                a3 = fld2<ASYM>(w[h2][2 * mt + 1][q >> 1], f + 1);
              }
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) {
                if (q == 0) imma0(C[h2][mt][nt], a0, a1, a2, a3, bq[h2][nt][0], bq[h2][nt][1]);
                else imma(C[h2][mt][nt], a0, a1, a2, a3, bq[h2][nt][2 * q], bq[h2][nt][2 * q + 1]);
              }
            }
#pragma unroll
        for (int h2 = 0; h2 < PS; ++h2) {
          const int sg = s0 + h2;
          if (h2 > 0 && sg >= nseg) break;
          if (spg_mask == 0) {   // one segment per group (the common case)
            epilogue(C[h2], sg, xst + (pr + h2) * Ly::XB, sst, zst, sx);
            continue;
          }
          const bool gfirst = (sg & spg_mask) == 0, glast = (sg & spg_mask) == spg_mask;
#pragma unroll
          for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int v = gfirst ? C[h2][mt][nt][e] : C[h2][mt][nt][e] + carry[mt][nt][e];
                if (glast) C[h2][mt][nt][e] = v;
                else carry[mt][nt][e] = v;
              }
          if (glast) epilogue(C[h2], sg, xst + (pr + h2) * Ly::XB, sst, zst, sx);
        }
      }
      __syncwarp();
      if (j + kD - 1 < nstage) {
        const uint32_t sl = islot;
        issue_w(j + kD - 1);
        issue_x(j + kD - 1, sl);
      }
    }
    if (!ok) break;

    // ---- results ---------------------------------------------------------------
    if constexpr (CMP) {
      // a token's two lanes (digits 0-1, digit 2) hold halves of its sums
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int tg = 0; tg < NG; ++tg)
#pragma unroll
          for (int h = 0; h < 2; ++h) acc[mt][tg][h] += __shfl_xor_sync(0xffffffffu, acc[mt][tg][h], 1);
    }
    if (ksplit == 1) {
#pragma unroll
      for (int tg = 0; tg < NG; ++tg) {
        const int tok = tg * 4 + ltok;
        if (dlead && tok < T) {
          if (p->epi == kEpiSwiGLU) {
            // rows 0-15 of the tile are gate rows, 16-31 the matching up rows
            // (m tiles 0 and 1): output row 16 * tile + rloc
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int rg = r0 + rloc[h], ru = r0 + rloc[2 + h];
              const float gv = acc[0][tg][h] + (p->bias ? __ldg(p->bias + rg) : 0.f);
              const float uv = acc[1][tg][h] + (p->bias ? __ldg(p->bias + ru) : 0.f);
              st_y(p->Y, (size_t)tok * (N >> 1) + (tile << 4) + rloc[h], silu(gv) * uv, p->ydt);
            }
            continue;
          }
#pragma unroll
          for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int row = r0 + rloc[2 * mt + h];
              if (row < N) {
                const float a = acc[mt][tg][h];
                if (p->push) push_val(p, ep, T, tok, row, a);
                else st_y(p->Y, (size_t)tok * N + row, p->bias ? a + __ldg(p->bias + row) : a, p->ydt);
              }
            }
        }
      }
      if (p->push) push_flag(p, ep, tile, lane);
      tile_written(L, p, lane);
    } else {
#pragma unroll
      for (int tg = 0; tg < NG; ++tg) {
        const int tok = tg * 4 + ltok;
        if (dlead && tok < T) {
#pragma unroll
          for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int row = r0 + rloc[2 * mt + h];
              if (row < N) __stcg(p->part + ((size_t)ks * T + tok) * N + row, acc[mt][tg][h]);
            }
        }
      }
      __threadfence();
      __syncwarp();
      unsigned int old = 0;
      if (lane == 0) old = atomicAdd(p->tcnt + tile, 1u);
      old = __shfl_sync(0xffffffffu, old, 0);
      if (old == (unsigned)ksplit - 1) {
        // last unit of this tile: add the partial sums in k order
        __threadfence();
        if (lane == 0) p->tcnt[tile] = 0;   // ready for the next launch
        const int row = r0 + lane;
        if (p->epi == kEpiSwiGLU) {
          // N is a multiple of 32 here: every lane has a row.  Lane i < 16 holds
          // gate row 16 * tile + i, lane i + 16 the matching up row.
          const float bv = p->bias ? __ldg(p->bias + row) : 0.f;
          for (int tok = 0; tok < T; ++tok) {
            const float* src = p->part + (size_t)tok * N + row;
            const size_t kstride = (size_t)T * N;
            float a = 0.f;
            for (int kc = 0; kc < ksplit; ++kc) a += __ldcg(src + (size_t)kc * kstride);
            a += bv;
            const float up = __shfl_down_sync(0xffffffffu, a, 16);
            if (lane < 16) st_y(p->Y, (size_t)tok * (N >> 1) + (tile << 4) + lane, silu(a) * up, p->ydt);
          }
        } else if (row < N) {
          const float bv = p->bias ? __ldg(p->bias + row) : 0.f;
          for (int tok = 0; tok < T; ++tok) {
            // loads first (eight in flight), then the sum in k order
            const float* src = p->part + (size_t)tok * N + row;
            const size_t kstride = (size_t)T * N;
            float a = 0.f;
            for (int kc = 0; kc < ksplit; kc += 8) {
              float v[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) v[j] = kc + j < ksplit ? __ldcg(src + (size_t)(kc + j) * kstride) : 0.f;
#pragma unroll
              for (int j = 0; j < 8; ++j) a += v[j];
            }
            if (p->push) push_val(p, ep, T, tok, row, a);
            else st_y(p->Y, (size_t)tok * N + row, a + bv, p->ydt);
          }
        }
        if (p->push) push_flag(p, ep, tile, lane);
        tile_written(L, p, lane);
      }
    }
  }
  // ---- end of a step launch: the last CTA to finish resets the cross-CTA
  // counters and flag lines for the next launch on the stream, and advances
  // the exchange epoch (so no clearing launch is needed between steps).
  if (L.done) {
    __syncthreads();
    unsigned int old = 0;
    if (threadIdx.x == 0) {
      __threadfence();
      old = atomicAdd(L.done, 1u);
    }
    if (__syncthreads_or(threadIdx.x == 0 && old == gridDim.x - 1)) {
      __threadfence();
      // flag lines use words 0 (phases written) and 1 (phases converted)
      for (int i = threadIdx.x; i < 2 * (int)gridDim.x; i += blockDim.x) L.flags[(i >> 1) * 32 + (i & 1)] = 0u;
      for (int i = threadIdx.x; i < 4 * L.nphase; i += blockDim.x) L.phctr[i] = 0u;
      __syncthreads();
      if (threadIdx.x == 0) {
        if (L.epoch) *reinterpret_cast<volatile unsigned long long*>(L.epoch) = ep;
        __threadfence();
        *L.done = 0u;
      }
    }
  }
}

// Activation blocks of the tasks whose input exists at launch: one CTA per task.
template <int T, int LB, int BITS>
__global__ void __launch_bounds__(256) q4_xblocks_kernel(const __grid_constant__ TileLaunch L) {
  const TileTask* p = tile_task(L, blockIdx.x);
  if (!p->xpre) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // blockIdx.y spreads one task's chunks over several CTAs
  const int wpb = blockDim.x >> 5;
  for (int c = blockIdx.y * wpb + warp; c < p->nchunk; c += gridDim.y * wpb) convert_chunk<T, LB, BITS>(p, c, lane);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {


int lb_for(int gs) { return (gs % 128 == 0) ? 16 : (gs % 64 == 0 ? 8 : 4); }

// Shared bytes per warp: TileLayout<T, ASYM, LB, BITS>::WARP.
int warp_bytes(int T, bool asym, int LB, int bits) {
  const int sps = 128 / (LB * bits), sbw = LB == 4 ? 8 : 4, kD = tile_kd(T);
  const int xstage = (sps * xblock_bytes(T, LB) + 127) & ~127;
  return kD * 32 * 128 + 128 + kD * xstage + kD * 32 * sbw * 4 * (asym ? 2 : 1);
}

size_t xblocks_bytes(int T, int K, int gs) {
  const int LB = lb_for(gs);
  return (((size_t)K / (8 * LB)) * xblock_bytes(T, LB) + 127) & ~(size_t)127;
}

struct TileConfig {
  int T, LB, bits, wpc, grid;
  bool asym;
  size_t smem;
};

// Shapes of the decode kernel.  4 bits: K % 32, group size a power of two in
// 32..256.  2 bits: K % 64 (16-byte rows for TMA), group size 128 or 256.
bool shape_ok(int N, int K, int gs, int bits = 4) {
  if (bits == 2) return N >= 1 && K % 64 == 0 && (gs == 128 || gs == 256) && K % gs == 0;
  return bits == 4 && N >= 1 && K % 32 == 0 && gs >= 32 && gs <= 256 && (gs & (gs - 1)) == 0 && K % gs == 0;
}

constexpr int kTileWarps = 12;   // warps per CTA at most (fewer when shared memory runs out)

bool make_config(int T, bool asym, int gs, TileConfig& c, int bits = 4) {
  const DeviceInfo& di = device_info();
  c.T = T; c.asym = asym; c.LB = lb_for(gs); c.bits = bits;
  if (T < 1 || T > kMaxGemvT || (T > 8 && c.LB == 4)) return false;   // 9-16 tokens need group size >= 64
  if (bits == 2 && c.LB != 16) return false;
  const size_t per_warp = (size_t)warp_bytes(T, asym, c.LB, bits);
  const size_t cap = (size_t)di.smem_optin;
  int wpc = (int)(cap / per_warp);
  if (wpc > kTileWarps) wpc = kTileWarps;
  if (wpc > tile_max_threads(T) / 32) wpc = tile_max_threads(T) / 32;
  // whole multiples of the 4 schedulers: an odd warp would carry a 3-warp
  // scheduler and, since every warp gets the same share of units, slow all
  // (above 8 tokens shared memory allows only 5-6 warps: all of them run)
  if (wpc > 4 && T <= 8) wpc &= ~3;
  if (wpc < 1) return false;
  c.wpc = wpc;
  c.smem = per_warp * wpc;
  c.grid = di.sms;
  return true;
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
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Groups per unit for a wanted number of k-ranges: whole groups, at least 4
// (a few segments per unit), in whole scale boxes (4 groups, 8 at group size
// 32) when the scales come by TMA, so that every stage's box is aligned.
int groups_per_unit(int G, long long want, bool stma, int gs) {
  if (want < 1) want = 1;
  const int sbw = gs == 32 ? 8 : 4;
  int gper = (int)((G + want - 1) / want);
  if (gper < 4) gper = 4;
  if (stma) gper = (gper + sbw - 1) / sbw * sbw;
  if (gper > G) gper = G;
  return gper;
}

// Fills the shape fields and the tensor maps of a task (W, S, Z set).
int fill_task(TileTask& q, int N, int K, int gs, int T, long long ksplit_want, int bits = 4) {
  const int LB = lb_for(gs);
  q.N = N; q.K = K; q.G = K / gs; q.lg2gs = __builtin_ctz((unsigned)gs);
  q.ntile = (N + kUnitRows - 1) / kUnitRows;
  const int G = q.G;
  q.stma = (G % 4 == 0) && ((reinterpret_cast<uintptr_t>(q.S) | reinterpret_cast<uintptr_t>(q.Z)) & 15) == 0;
  const int gper = groups_per_unit(G, ksplit_want, q.stma != 0, gs);
  q.kper = gper * gs;
  q.ksplit = (G + gper - 1) / gper;
  q.nchunk = (T * (K / 8) + 31) / 32;
  (void)LB;
  const uint64_t row_bytes = (uint64_t)K * bits / 8;
  if (!make_map(&q.tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, q.W, row_bytes, (uint64_t)N, row_bytes,
                128, kUnitRows, CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(SF_ERR_CUDA, "cuTensorMapEncodeTiled failed for the weights (N=%d K=%d)", N, K);
  if (q.stma) {
    const uint32_t sbw = gs == 32 ? 8 : 4;
    if (!make_map(&q.tmS, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, q.S, (uint64_t)G, (uint64_t)N, (uint64_t)G * 4, sbw,
                  kUnitRows, CU_TENSOR_MAP_SWIZZLE_NONE))
      return fail(SF_ERR_CUDA, "cuTensorMapEncodeTiled failed for the scales");
    if (q.Z && !make_map(&q.tmZ, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, q.Z, (uint64_t)G, (uint64_t)N,
                         (uint64_t)G * 4, sbw, kUnitRows, CU_TENSOR_MAP_SWIZZLE_NONE))
      return fail(SF_ERR_CUDA, "cuTensorMapEncodeTiled failed for the zeros");
  }
  return SF_OK;
}

template <int T, bool ASYM, int LB, int BITS>
cudaError_t launch_tile_t(const TileConfig& c, const TileLaunch& L, bool coop, cudaStream_t st) {
  auto* fn = q4_tile_kernel<T, ASYM, LB, BITS>;
  if (warp_bytes(T, ASYM, LB, BITS) != TileLayout<T, ASYM, LB, BITS>::WARP) return cudaErrorInvalidConfiguration;
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

template <bool ASYM, int LB, int BITS>
cudaError_t launch_tile_lb(const TileConfig& c, const TileLaunch& L, bool coop, cudaStream_t st) {
  switch (c.T) {
    case 1: return launch_tile_t<1, ASYM, LB, BITS>(c, L, coop, st);
    case 2: return launch_tile_t<2, ASYM, LB, BITS>(c, L, coop, st);
    case 3: return launch_tile_t<3, ASYM, LB, BITS>(c, L, coop, st);
    case 4: return launch_tile_t<4, ASYM, LB, BITS>(c, L, coop, st);
    case 5: return launch_tile_t<5, ASYM, LB, BITS>(c, L, coop, st);
    case 6: return launch_tile_t<6, ASYM, LB, BITS>(c, L, coop, st);
    case 7: return launch_tile_t<7, ASYM, LB, BITS>(c, L, coop, st);
    case 8: return launch_tile_t<8, ASYM, LB, BITS>(c, L, coop, st);
    default: break;
  }
  if constexpr (LB != 4) {   // 9-16 tokens: group sizes of 64 and more
    switch (c.T) {
      case 9: return launch_tile_t<9, ASYM, LB, BITS>(c, L, coop, st);
      case 10: return launch_tile_t<10, ASYM, LB, BITS>(c, L, coop, st);
      case 11: return launch_tile_t<11, ASYM, LB, BITS>(c, L, coop, st);
      case 12: return launch_tile_t<12, ASYM, LB, BITS>(c, L, coop, st);
      case 13: return launch_tile_t<13, ASYM, LB, BITS>(c, L, coop, st);
      case 14: return launch_tile_t<14, ASYM, LB, BITS>(c, L, coop, st);
      case 15: return launch_tile_t<15, ASYM, LB, BITS>(c, L, coop, st);
      case 16: return launch_tile_t<16, ASYM, LB, BITS>(c, L, coop, st);
      default: break;
    }
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_tile(const TileConfig& c, const TileLaunch& L, bool coop, cudaStream_t st) {
  if (c.bits == 2) {   // 2-bit weights: group sizes 128 and 256 only
    if (c.LB != 16) return cudaErrorInvalidValue;
    return c.asym ? launch_tile_lb<true, 16, 2>(c, L, coop, st) : launch_tile_lb<false, 16, 2>(c, L, coop, st);
  }
  if (c.asym) {
    if (c.LB == 16) return launch_tile_lb<true, 16, 4>(c, L, coop, st);
    if (c.LB == 8) return launch_tile_lb<true, 8, 4>(c, L, coop, st);
    return launch_tile_lb<true, 4, 4>(c, L, coop, st);
  }
  if (c.LB == 16) return launch_tile_lb<false, 16, 4>(c, L, coop, st);
  if (c.LB == 8) return launch_tile_lb<false, 8, 4>(c, L, coop, st);
  return launch_tile_lb<false, 4, 4>(c, L, coop, st);
}

template <int LB, int BITS>
cudaError_t launch_xblocks_lb(int T, int ntasks, const TileLaunch& L, cudaStream_t st, int ny) {
  const dim3 grid((unsigned)ntasks, (unsigned)(ny < 1 ? 1 : ny));
  switch (T) {
    case 1: q4_xblocks_kernel<1, LB, BITS><<<grid, 256, 0, st>>>(L); break;
    case 2: q4_xblocks_kernel<2, LB, BITS><<<grid, 256, 0, st>>>(L); break;
    case 3: q4_xblocks_kernel<3, LB, BITS><<<grid, 256, 0, st>>>(L); break;
    case 4: q4_xblocks_kernel<4, LB, BITS><<<grid, 256, 0, st>>>(L); break;
    case 5: q4_xblocks_kernel<5, LB, BITS><<<grid, 256, 0, st>>>(L); break;
    case 6: q4_xblocks_kernel<6, LB, BITS><<<grid, 256, 0, st>>>(L); break;
    case 7: q4_xblocks_kernel<7, LB, BITS><<<grid, 256, 0, st>>>(L); break;
    case 8: q4_xblocks_kernel<8, LB, BITS><<<grid, 256, 0, st>>>(L); break;
    default:
      if constexpr (LB != 4) {
        switch (T) {
          case 9: q4_xblocks_kernel<9, LB, BITS><<<grid, 256, 0, st>>>(L); break;
          case 10: q4_xblocks_kernel<10, LB, BITS><<<grid, 256, 0, st>>>(L); break;
          case 11: q4_xblocks_kernel<11, LB, BITS><<<grid, 256, 0, st>>>(L); break;
          case 12: q4_xblocks_kernel<12, LB, BITS><<<grid, 256, 0, st>>>(L); break;
          case 13: q4_xblocks_kernel<13, LB, BITS><<<grid, 256, 0, st>>>(L); break;
          case 14: q4_xblocks_kernel<14, LB, BITS><<<grid, 256, 0, st>>>(L); break;
          case 15: q4_xblocks_kernel<15, LB, BITS><<<grid, 256, 0, st>>>(L); break;
          case 16: q4_xblocks_kernel<16, LB, BITS><<<grid, 256, 0, st>>>(L); break;
          default: return cudaErrorInvalidValue;
        }
      } else {
        return cudaErrorInvalidValue;
      }
  }
  return cudaGetLastError();
}

// ny: CTAs per task (each converts every ny-th run of 8 chunks); chunks per
// task = T*K/256, so ny = ceil(chunks / 8) gives every warp one chunk.
cudaError_t launch_xblocks(int T, int LB, int ntasks, const TileLaunch& L, cudaStream_t st, int ny, int bits = 4) {
  if (ny > 64) ny = 64;
  if (bits == 2) return LB == 16 ? launch_xblocks_lb<16, 2>(T, ntasks, L, st, ny) : cudaErrorInvalidValue;
  if (LB == 16) return launch_xblocks_lb<16, 4>(T, ntasks, L, st, ny);
  if (LB == 8) return launch_xblocks_lb<8, 4>(T, ntasks, L, st, ny);
  return launch_xblocks_lb<4, 4>(T, ntasks, L, st, ny);
}

// Library-owned scratch of the single-GEMV entry, one pair of buffers per
// (device, stream) so that concurrent streams never share one:
//  * per-tile arrival counters, zeroed when allocated and left at zero by the
//    kernel (the last unit of a tile resets its counter), so they must never
//    be reused for anything else;
//  * k-split partial sums and activation blocks.
// Both grow on demand and never shrink.
struct Scratch {
  void* ctr = nullptr;
  size_t ctr_bytes = 0;
  void* data = nullptr;
  size_t data_bytes = 0;
};
std::mutex g_scratch_mu;
std::map<std::pair<int, cudaStream_t>, Scratch> g_scratch;

int grow(cudaStream_t st, void** buf, size_t* have, size_t need, bool zero) {
  if (*have >= need) return SF_OK;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(st, &cs);
  if (cs != cudaStreamCaptureStatusNone)
    return fail(SF_ERR_CAPTURE,
                "GEMV scratch must grow during stream capture: run the same shape once on the capturing "
                "stream before capturing");
  if (*buf) {
    cudaStreamSynchronize(st);
    cudaFree(*buf);
  }
  *buf = nullptr;
  *have = 0;
  const size_t nb = (need + ((size_t)1 << 16) - 1) & ~(((size_t)1 << 16) - 1);
  cudaError_t e = cudaMalloc(buf, nb);
  if (e != cudaSuccess) return cuda_fail(e, "allocating GEMV scratch");
  if (zero) {
    e = cudaMemset(*buf, 0, nb);
    if (e != cudaSuccess) return cuda_fail(e, "clearing GEMV scratch");
  }
  *have = nb;
  return SF_OK;
}

int get_scratch(cudaStream_t st, size_t ctr_bytes, size_t data_bytes, void** ctr, void** data) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  Scratch& s = g_scratch[{dev, st}];
  int rc = grow(st, &s.ctr, &s.ctr_bytes, ctr_bytes, true);
  if (rc != SF_OK) return rc;
  rc = grow(st, &s.data, &s.data_bytes, data_bytes, false);
  if (rc != SF_OK) return rc;
  *ctr = s.ctr;
  *data = s.data;
  return SF_OK;
}

size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

}  // namespace

// One GEMV (T <= 8): activation-block pre-pass, then the tile kernel with a
// k-split sized to give every warp of the GPU about one unit.
// SF_ERR_UNSUPPORTED when the shape is not one this kernel takes.
int run_tile_linear(const uint8_t* W, const float* S, const float* Z, const float* bias,
                    const void* X, int xdt, void* Y, int ydt, int N, int K, int T, int gs,
                    cudaStream_t stream, int epi, int bits) {
  if (T < 1 || T > kMaxGemvT || !shape_ok(N, K, gs, bits)) return SF_ERR_UNSUPPORTED;
  if (epi == kEpiSwiGLU && N % kUnitRows) return SF_ERR_UNSUPPORTED;
  TileConfig c;
  if (!make_config(T, Z != nullptr, gs, c, bits)) return SF_ERR_UNSUPPORTED;
  TileLaunch L{};
  TileTask& q = L.single;
  q.W = W; q.S = S; q.Z = Z; q.bias = bias; q.X = X; q.Y = Y; q.xdt = xdt; q.ydt = ydt;
  q.epi = epi;
  const int ntile = (N + kUnitRows - 1) / kUnitRows;
  const int warps = c.grid * c.wpc;
  int rc = fill_task(q, N, K, gs, T, (warps + ntile - 1) / ntile, bits);
  if (rc != SF_OK) return rc;
  const size_t cbytes = align256((size_t)q.ntile * 4);
  const size_t pbytes = q.ksplit > 1 ? align256((size_t)q.ksplit * T * N * 4) : 0;
  const size_t xbytes = xblocks_bytes(T, K, gs);
  void* cscr = nullptr;
  void* dscr = nullptr;
  rc = get_scratch(stream, cbytes, pbytes + xbytes, &cscr, &dscr);
  if (rc != SF_OK) return rc;
  uint8_t* base = static_cast<uint8_t*>(dscr);
  q.tcnt = static_cast<unsigned int*>(cscr);
  q.part = pbytes ? reinterpret_cast<float*>(base) : nullptr;
  q.xd = base + pbytes;
  q.xpre = 1;
  q.ubase = 0;
  q.phase = 0;
  q.ph_last = 1;
  L.tasks = nullptr; L.ntasks = 1; L.total = (long long)q.ntile * q.ksplit;
  L.phctr = nullptr;
  L.flags = nullptr;
  const int need = (int)((L.total + c.wpc - 1) / c.wpc);
  if (c.grid > need) c.grid = need;
  cudaError_t e = launch_xblocks(T, c.LB, 1, L, stream, (q.nchunk + 7) / 8, bits);
  if (e != cudaSuccess) return cuda_fail(e, "activation pre-pass launch");
  e = launch_tile(c, L, false, stream);
  if (e != cudaSuccess) return cuda_fail(e, "q4_tile_kernel launch");
  g_launches.fetch_add(2, std::memory_order_relaxed);
  return SF_OK;
}

}  // namespace sf

// ===========================================================================
// C ABI: a prepared list of GEMVs run as one persistent launch.
// ===========================================================================
using namespace sf;

namespace {
// Workspace: [per-CTA flag lines | per-phase counters | per-tile arrival
// counters] (cleared before every run) [task table] [k-split partials]
// [activation blocks].
struct StepSizes {
  size_t ctr, tiles, table, part, xblk, cmap;
  size_t total() const { return ctr + tiles + table + part + xblk + cmap; }
};

// k-splits of a task list.  Each phase (a run of tasks that need not wait for
// one another) ends when its busiest warp does.  Warps take the launch's units
// round robin (unit u goes to warp u mod W), so for every candidate split the
// phase's units are dealt out exactly that way and the split whose busiest
// warp has the least work wins; a unit's work is its groups plus kUnitCost
// (its pipeline fill and k-split partials, in groups of streaming time).  This
// keeps a small phase from being cut into slightly more units than the grid
// has warps, which would leave a few warps a second unit and take twice as long.
constexpr int kUnitCost = 4;
std::vector<int> plan_ksplit(const sf_q4_task* tasks, int n, int warps) {
  std::vector<int> ks(n, 1);
  auto stma_of = [&](int k) {
    const int G = tasks[k].K / tasks[k].group_size;
    return G % 4 == 0 &&
           ((reinterpret_cast<uintptr_t>(tasks[k].scales) | reinterpret_cast<uintptr_t>(tasks[k].zeros)) & 15) == 0;
  };
  auto gper_for = [&](int k, int B) {
    const int G = tasks[k].K / tasks[k].group_size;
    return groups_per_unit(G, (G + B - 1) / B, stma_of(k), tasks[k].group_size);
  };
  std::vector<long long> load(warps);
  long long ubase = 0;   // the phase's first unit in the launch
  int i = 0;
  while (i < n) {
    int j = i + 1;
    while (j < n && !tasks[j].wait_before) ++j;
    int gmax = 1;
    for (int k = i; k < j; ++k) gmax = std::max(gmax, tasks[k].K / tasks[k].group_size);
    long long best_cost = -1, best_units = 0;
    int best_b = gmax, last_sig = -1;
    for (int B = gmax; B >= 1; --B) {
      int sig = 0;   // skip a candidate that cuts every task as the previous one did
      for (int k = i; k < j; ++k) sig = sig * 31 + gper_for(k, B);
      if (sig == last_sig) continue;
      last_sig = sig;
      std::fill(load.begin(), load.end(), 0);
      long long u = ubase;
      for (int k = i; k < j; ++k) {
        const int G = tasks[k].K / tasks[k].group_size, gper = gper_for(k, B);
        const int kspl = (G + gper - 1) / gper, ntile = (tasks[k].N + kUnitRows - 1) / kUnitRows;
        for (int s2 = 0; s2 < kspl; ++s2) {   // units of one k-range are consecutive (tile fastest)
          const int len = std::min(gper, G - s2 * gper) + kUnitCost;
          for (int t2 = 0; t2 < ntile; ++t2) load[(size_t)(u++ % warps)] += len;
        }
      }
      const long long units = u - ubase;
      const long long cost = *std::max_element(load.begin(), load.end());
      if (best_cost < 0 || cost < best_cost || (cost == best_cost && units < best_units)) {
        best_cost = cost;
        best_units = units;
        best_b = B;
      }
    }
    for (int k = i; k < j; ++k) {
      const int G = tasks[k].K / tasks[k].group_size, gper = gper_for(k, best_b);
      ks[k] = (G + gper - 1) / gper;
    }
    ubase += best_units;
    i = j;
  }
  return ks;
}

StepSizes step_sizes(const sf_q4_task* tasks, int n, const std::vector<int>& ksplit, int grid) {
  StepSizes z{};
  z.ctr = align256((size_t)128 * grid) + align256((size_t)16 * n + 16);   // flag lines, phase counters, done
  size_t tiles = 0, part = 0, xb = 0, chunks = 0;
  for (int i = 0; i < n; ++i) {
    const sf_q4_task& a = tasks[i];
    const int ntile = (a.N + kUnitRows - 1) / kUnitRows;
    tiles += (size_t)ntile * 4;
    if (ksplit[i] > 1) part += align256((size_t)ksplit[i] * a.T * a.N * 4);
    xb += xblocks_bytes(a.T, a.K, a.group_size);
    chunks += ((size_t)a.T * (a.K / 8) + 31) / 32;
  }
  z.tiles = align256(tiles);
  z.table = align256((size_t)n * sizeof(TileTask));
  z.part = part;
  z.cmap = align256(chunks * 4) + align256((size_t)8 * n);   // chunk map, then the compact unit starts
  z.xblk = xb;
  return z;
}

constexpr size_t kEpochBytes = 256;   // launch epoch of a step with exchange tasks (after the workspace)

struct StepHandle {
  TileConfig cfg;
  TileLaunch L;
  void* workspace;
  bool coop;
  bool tp;                  // has tensor-parallel exchange tasks (epoch at the workspace end)
};

int task_bits(const sf_q4_task& a) { return a.bits == 0 ? 4 : a.bits; }

bool step_config(const sf_q4_task* tasks, TileConfig& c) {
  return make_config(tasks[0].T, tasks[0].zeros != nullptr, tasks[0].group_size, c, task_bits(tasks[0]));
}
}  // namespace

extern "C" {

size_t sf_q4_step_workspace_bytes(const sf_q4_task* tasks, int ntasks) {
  if (!tasks || ntasks < 1) return 0;
  for (int i = 0; i < ntasks; ++i)
    if (tasks[i].T < 1 || tasks[i].T > kMaxGemvT ||
        !shape_ok(tasks[i].N, tasks[i].K, tasks[i].group_size, task_bits(tasks[i])))
      return 0;
  TileConfig c;
  if (!step_config(tasks, c)) return 0;
  return step_sizes(tasks, ntasks, plan_ksplit(tasks, ntasks, c.grid * c.wpc), c.grid).total() + kEpochBytes;
}

}  // extern "C"

namespace {
int step_create_impl(const sf_q4_task* tasks, const int* roles, int ntasks, void* comm, void* workspace,
                     size_t workspace_bytes, void** handle_out) {
  if (!tasks || !workspace || !handle_out) return fail(SF_ERR_NULL, "null pointer argument");
  if (ntasks < 1) return fail(SF_ERR_SHAPE, "ntasks must be >= 1");
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return fail(SF_ERR_ALIGN, "workspace must be 256-byte aligned");
  const int T = tasks[0].T;
  const bool asym = tasks[0].zeros != nullptr;
  if (T < 1 || T > kMaxGemvT) return fail(SF_ERR_UNSUPPORTED, "step tasks need 1 <= T <= %d", kMaxGemvT);
  bool has_tp = false;
  for (int i = 0; i < ntasks; ++i) {
    const sf_q4_task& a = tasks[i];
    const int role = roles ? roles[i] : SF_ROLE_GEMV;
    if (role != SF_ROLE_GEMV) {
      has_tp = true;
      if (!comm) return fail(SF_ERR_NULL, "task %d: an exchange role needs a tensor-parallel communicator", i);
      if (role >= SF_ROLE_REDUCE) {
        const int src = role - SF_ROLE_REDUCE;
        if (src >= i || roles[src] != SF_ROLE_PUSH || tasks[src].N != a.N)
          return fail(SF_ERR_SHAPE, "task %d: reduce role must name an earlier pushed task of the same N", i);
      } else if (role != SF_ROLE_PUSH) {
        return fail(SF_ERR_SHAPE, "task %d: unknown role %d", i, role);
      }
    }
    if (!a.W || !a.scales || !a.X || (!a.Y && role != SF_ROLE_PUSH))
      return fail(SF_ERR_NULL, "task %d: null pointer", i);
    if (a.T != T || (a.zeros != nullptr) != asym || a.group_size <= 0 ||
        lb_for(a.group_size) != lb_for(tasks[0].group_size) || task_bits(a) != task_bits(tasks[0]))
      return fail(SF_ERR_UNSUPPORTED, "task %d: all tasks need the same T, layout, bit width and group class", i);
    if (!shape_ok(a.N, a.K, a.group_size, task_bits(a)))
      return fail(SF_ERR_UNSUPPORTED, "task %d: shape N=%d K=%d gs=%d not supported by the step kernel",
                  i, a.N, a.K, a.group_size);
    if (a.x_dtype < 0 || a.x_dtype > 2 || a.y_dtype < 0 || a.y_dtype > 2)
      return fail(SF_ERR_DTYPE, "task %d: unknown dtype code", i);
    if (a.epilogue != 0 && (a.epilogue != SF_EPI_SWIGLU || a.N % kUnitRows || role != SF_ROLE_GEMV))
      return fail(SF_ERR_UNSUPPORTED,
                  "task %d: epilogue %d needs SF_EPI_SWIGLU, N (gate + up rows) a multiple of 32 and no exchange "
                  "role", i, a.epilogue);
    if ((reinterpret_cast<uintptr_t>(a.W) | reinterpret_cast<uintptr_t>(a.scales) |
         reinterpret_cast<uintptr_t>(a.zeros) | reinterpret_cast<uintptr_t>(a.X)) & 15)
      return fail(SF_ERR_ALIGN, "task %d: W, scales, zeros and X must be 16-byte aligned", i);
  }
  TileConfig c;
  if (!step_config(tasks, c)) return fail(SF_ERR_UNSUPPORTED, "no launch configuration for T=%d", T);
  const std::vector<int> want = plan_ksplit(tasks, ntasks, c.grid * c.wpc);
  const StepSizes z = step_sizes(tasks, ntasks, want, c.grid);
  if (workspace_bytes < z.total() + kEpochBytes)
    return fail(SF_ERR_SHAPE, "workspace too small: need %zu bytes", z.total() + kEpochBytes);

  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint8_t* tiles = ws + z.ctr;
  uint8_t* table = tiles + z.tiles;
  uint8_t* part = table + z.table;
  uint8_t* xblk = part + z.part;
  std::vector<TileTask> h(ntasks);
  unsigned long long* poison = nullptr;
  long long ub = 0;
  int nph = 0;
  for (int i = 0; i < ntasks; ++i) {
    const sf_q4_task& a = tasks[i];
    TileTask& q = h[i];
    q = TileTask{};
    q.W = a.W; q.S = a.scales; q.Z = a.zeros; q.bias = a.bias; q.X = a.X; q.Y = a.Y;
    q.xdt = a.x_dtype; q.ydt = a.y_dtype;
    q.epi = a.epilogue;
    int rc = fill_task(q, a.N, a.K, a.group_size, T, want[i], task_bits(a));
    if (rc != SF_OK) return rc;
    q.tcnt = reinterpret_cast<unsigned int*>(tiles);
    tiles += (size_t)q.ntile * 4;
    q.part = nullptr;
    if (q.ksplit > 1) {
      q.part = reinterpret_cast<float*>(part);
      part += align256((size_t)q.ksplit * T * a.N * 4);
    }
    q.xd = xblk;
    xblk += xblocks_bytes(T, a.K, a.group_size);
    // A task with wait_before opens a phase; every task of a phase reads X only
    // after the whole previous phase has written Y (and, transitively, all
    // earlier ones).  Only phase-0 inputs exist before the launch.
    if (i == 0 || a.wait_before) ++nph;
    q.phase = nph - 1;
    q.xpre = 0;   // every phase converts its inputs inside the launch
    const int role = roles ? roles[i] : SF_ROLE_GEMV;
    if (role != SF_ROLE_GEMV) {
      q.push = role == SF_ROLE_PUSH;
      q.kind = role >= SF_ROLE_REDUCE ? 1 : 0;
      if (q.kind == 1) {   // sums an earlier pushed task: no weights, one unit per kRedTiles tiles
        const TileTask& sq = h[role - SF_ROLE_REDUCE];
        q.ksplit = 1;
        q.ntile = (q.ntile + kRedTiles - 1) / kRedTiles;
        q.xpre = 0;
        q.nchunk = 0;
        q.xpar = sq.xpar;
        for (int r = 0; r < 8; ++r) { q.xdata[r] = sq.xdata[r]; q.xflag[r] = sq.xflag[r]; }
        q.tp_rank = sq.tp_rank;
        q.tp_world = sq.tp_world;
      } else {
        const size_t data = (size_t)T * a.N * 4;   // one source rank's [T][N] fp32
        int rc2 = tp_region(comm, data, (size_t)q.ntile, q.xdata, q.xflag, &q.tp_rank, &q.tp_world, &q.xpar,
                            &poison);
        if (rc2 != SF_OK) return rc2;
      }
    }
    q.ubase = ub;
    ub += (long long)q.ntile * q.ksplit;
  }
  for (int i = 0; i < ntasks;) {
    int j = i;
    long long tiles_ph = 0, chunks = 0, units = 0;
    while (j < ntasks && h[j].phase == h[i].phase) {
      tiles_ph += h[j].ntile;
      chunks += h[j].nchunk;
      units += (long long)h[j].ntile * h[j].ksplit;
      ++j;
    }
    for (int k = i; k < j; ++k) {
      h[k].ph_first = i;
      h[k].ph_tiles = (int)tiles_ph;
      h[k].ph_chunks = (int)chunks;
      h[k].ph_units = units;
      h[k].ph_ubase = h[i].ubase;
      h[k].ph_last = h[k].phase == nph - 1 ? 1 : 0;
    }
    i = j;
  }
  // chunk map: phase by phase, every task's conversion chunks in order
  std::vector<unsigned int> cmap;
  for (int i = 0; i < ntasks; ++i) {
    if (i == 0 || h[i].phase != h[i - 1].phase) {
      for (int k = i; k < ntasks && h[k].phase == h[i].phase; ++k) h[k].ph_cbase = (int)cmap.size();
    }
    if (h[i].nchunk > 0xFFFF || i > 0xFFFF)
      return fail(SF_ERR_UNSUPPORTED, "task %d: too many tasks or conversion chunks for the step's chunk map", i);
    for (int c = 0; c < h[i].nchunk; ++c) cmap.push_back(((unsigned int)i << 16) | (unsigned int)c);
  }
  uint8_t* cmap_d = ws + z.total() - z.cmap;
  long long* ubase_d = reinterpret_cast<long long*>(cmap_d + align256(cmap.size() * 4));
  std::vector<long long> ubase(ntasks);
  for (int i = 0; i < ntasks; ++i) ubase[i] = h[i].ubase;
  StepHandle* hd = new StepHandle{};
  hd->cfg = c;
  hd->workspace = workspace;
  hd->coop = true;   // the input-conversion and exchange waits need every CTA resident
  hd->tp = has_tp;
  TileLaunch& L = hd->L;
  L.tasks = reinterpret_cast<const TileTask*>(table);
  L.ntasks = ntasks;
  L.total = ub;
  L.flags = reinterpret_cast<unsigned int*>(ws);
  L.phctr = reinterpret_cast<unsigned int*>(ws + align256((size_t)128 * c.grid));
  L.done = L.phctr + 4 * ntasks;
  L.cmap = reinterpret_cast<const unsigned int*>(cmap_d);
  L.ubase = ubase_d;
  L.nphase = nph;
  L.epoch = nullptr;
  L.poison = poison;
  cudaError_t e = cudaMemcpy(table, h.data(), (size_t)ntasks * sizeof(TileTask), cudaMemcpyHostToDevice);
  // counters start at zero; every run leaves them so
  if (e == cudaSuccess) e = cudaMemset(ws, 0, z.ctr + z.tiles);
  if (e == cudaSuccess && !cmap.empty())
    e = cudaMemcpy(cmap_d, cmap.data(), cmap.size() * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(ubase_d, ubase.data(), (size_t)ntasks * 8, cudaMemcpyHostToDevice);
  if (e == cudaSuccess && has_tp) {
    L.epoch = reinterpret_cast<unsigned long long*>(ws + z.total());
    e = cudaMemset(L.epoch, 0, kEpochBytes);
  }
  if (e != cudaSuccess) {
    delete hd;
    return cuda_fail(e, "uploading the task table");
  }
  *handle_out = hd;
  return SF_OK;
}
}  // namespace

extern "C" {

int sf_q4_step_create(const sf_q4_task* tasks, int ntasks, void* workspace, size_t workspace_bytes,
                      void** handle_out) {
  return step_create_impl(tasks, nullptr, ntasks, nullptr, workspace, workspace_bytes, handle_out);
}

int sf_q4_step_create_tp(const sf_q4_task* tasks, const int* roles, int ntasks, void* comm, void* workspace,
                         size_t workspace_bytes, void** handle_out) {
  if (!roles) return fail(SF_ERR_NULL, "null pointer argument");
  return step_create_impl(tasks, roles, ntasks, comm, workspace, workspace_bytes, handle_out);
}

int sf_q4_step_run(void* handle, void* stream) {
  if (!handle) return fail(SF_ERR_NULL, "null handle");
  StepHandle* hd = static_cast<StepHandle*>(handle);
  // one launch: the kernel converts each phase's inputs itself and its last
  // CTA leaves the counters cleared for the next run
  cudaError_t e = launch_tile(hd->cfg, hd->L, hd->coop, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "q4 step launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return SF_OK;
}

void sf_q4_step_destroy(void* handle) { delete static_cast<StepHandle*>(handle); }


}  // extern "C"

// ===========================================================================
// SwiGLU on interleaved gate/up weights
// ===========================================================================
namespace sf {
namespace {
__global__ void swiglu_interleaved_kernel(const float* __restrict__ in, void* out, int ydt, int T, int n_out,
                                          const float* __restrict__ bias) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= (long long)T * n_out) return;
  const int t = (int)(i / n_out), o = (int)(i - (long long)t * n_out);
  const int rg = (o >> 4) * 32 + (o & 15), ru = rg + 16;   // interleaved rows of the gate and up halves
  const float* row = in + (size_t)t * 2 * n_out;
  const float g = row[rg] + (bias ? bias[rg] : 0.f), u = row[ru] + (bias ? bias[ru] : 0.f);
  st_y(out, (size_t)i, silu(g) * u, ydt);
}
}  // namespace
}  // namespace sf

extern "C" int sf_q4_linear_swiglu(const uint8_t* W, const float* scales, const float* zeros, const float* bias,
                                   const void* X, int x_dtype, void* Y, int y_dtype, int N, int K, int T,
                                   int group_size, void* stream) {
  if (!W || !scales || !X || !Y) return fail(SF_ERR_NULL, "null pointer argument");
  if (x_dtype < 0 || x_dtype > 2 || y_dtype < 0 || y_dtype > 2) return fail(SF_ERR_DTYPE, "unknown dtype code");
  if (N < 0 || K <= 0 || T < 0) return fail(SF_ERR_SHAPE, "invalid N/K/T");
  if (N % 16) return fail(SF_ERR_SHAPE, "SwiGLU output width N=%d must be a multiple of 16", N);
  if (group_size <= 0 || group_size % 2 || K % group_size)
    return fail(SF_ERR_SHAPE, "in_features must be divisible by an even group_size");
  if (N == 0 || T == 0) return SF_OK;
  if ((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(scales) | reinterpret_cast<uintptr_t>(zeros) |
       reinterpret_cast<uintptr_t>(X)) & 15)
    return fail(SF_ERR_ALIGN, "W, scales, zeros and X must be 16-byte aligned");
  const int rc = run_tile_linear(W, scales, zeros, bias, X, x_dtype, Y, y_dtype, 2 * N, K, T, group_size,
                                 static_cast<cudaStream_t>(stream), kEpiSwiGLU);
  if (rc == SF_ERR_UNSUPPORTED)
    return fail(SF_ERR_UNSUPPORTED,
                "fused SwiGLU runs on the decode kernel: T <= %d (8 at group size 32), K %% 32 == 0 and a "
                "power-of-two group_size in 32..256; use sf_q4_linear on the stacked rows and "
                "sf_swiglu_interleaved", kMaxGemvT);
  return rc;
}

extern "C" int sf_swiglu_interleaved(const float* in, void* out, int out_dtype, int T, int N, const float* bias,
                                     void* stream) {
  if (!in || !out) return fail(SF_ERR_NULL, "null pointer argument");
  if (out_dtype < 0 || out_dtype > 2) return fail(SF_ERR_DTYPE, "unknown dtype code");
  if (T < 0 || N < 0 || N % 16) return fail(SF_ERR_SHAPE, "N=%d must be a multiple of 16", N);
  const long long n = (long long)T * N;
  if (n == 0) return SF_OK;
  swiglu_interleaved_kernel<<<(unsigned)((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      in, out, out_dtype, T, N, bias);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "swiglu_interleaved_kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return SF_OK;
}

// 2-bit weights (siliconfer/quant/primitives.py:383-404 pack_int2: 4 values per
// byte, element i in bits 2i..2i+1; symmetric q in [-2, 1] two's complement,
// asymmetric q in [0, 3] with fp32 zeros).  Decode sizes on the same kernel
// (T <= 16 per launch, larger T in chunks of 16); group size 128 or 256.
extern "C" int sf_q2_linear(const uint8_t* W, const float* scales, const float* zeros, const float* bias,
                            const void* X, int x_dtype, void* Y, int y_dtype, int N, int K, int T, int group_size,
                            void* stream) {
  if (!W || !scales || !X || !Y) return fail(SF_ERR_NULL, "null pointer argument");
  if (x_dtype < 0 || x_dtype > 2 || y_dtype < 0 || y_dtype > 2) return fail(SF_ERR_DTYPE, "unknown dtype code");
  if (N < 0 || K <= 0 || T < 0) return fail(SF_ERR_SHAPE, "invalid N/K/T");
  if (group_size <= 0 || K % group_size) return fail(SF_ERR_SHAPE, "in_features must be divisible by group_size");
  if (K % 4) return fail(SF_ERR_SHAPE, "in_features must be divisible by 4 for int2 packing");
  if (N == 0 || T == 0) return SF_OK;
  if (!shape_ok(N, K, group_size, 2))
    return fail(SF_ERR_UNSUPPORTED, "int2 GEMV takes K %% 64 == 0 and group_size 128 or 256 (got K=%d gs=%d)", K,
                group_size);
  if ((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(scales) | reinterpret_cast<uintptr_t>(zeros) |
       reinterpret_cast<uintptr_t>(X)) & 15)
    return fail(SF_ERR_ALIGN, "W, scales, zeros and X must be 16-byte aligned");
  const size_t xe = x_dtype == SF_F32 ? 4 : 2, ye = y_dtype == SF_F32 ? 4 : 2;
  const int tmax = T <= kMaxGemvT ? kMaxGemvT : 8;   // as sf_q4_linear: chunks of 8 above 16 tokens
  for (int t0 = 0; t0 < T; t0 += tmax) {
    const int tc = T - t0 < tmax ? T - t0 : tmax;
    const int rc = run_tile_linear(W, scales, zeros, bias, static_cast<const uint8_t*>(X) + (size_t)t0 * K * xe,
                                   x_dtype, static_cast<uint8_t*>(Y) + (size_t)t0 * N * ye, y_dtype, N, K, tc,
                                   group_size, static_cast<cudaStream_t>(stream), 0, 2);
    if (rc != SF_OK) return rc == SF_ERR_UNSUPPORTED ? fail(rc, "int2 GEMV: no launch configuration") : rc;
  }
  return SF_OK;
}

// ===========================================================================
// Decode GEMV without any allocation: the single-GEMV launch above, with its
// scratch (arrival counters, k-split partial sums, activation blocks) taken
// from a fixed buffer that lives in this library's own device image.
//
// Why: sf_q4_linear grows a library-owned scratch buffer with cudaMalloc the
// first time it meets a shape.  Some callers cannot let a library allocate at
// all -- a serving process that hands every byte of the GPU to its own pool
// up front, code that runs where an allocation would synchronise the device
// or be refused.  For them this entry point uses only memory that exists from
// the moment the library is loaded.
// ===========================================================================
namespace {
constexpr size_t kStaticCounterBytes = (size_t)64 << 10;               // 16384 tiles: N <= 524288
constexpr size_t kStaticScratchBytes = (size_t)4 << 20;                // 4 MiB in total
constexpr size_t kStaticDataBytes = kStaticScratchBytes - kStaticCounterBytes;

// Part of the module image: created with the library, never allocated or freed.
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_static_mu;
void* g_static_ptr[kMaxDevices] = {nullptr};

// Device address of the buffer on the current device; looked up once per
// device on the first call.
int static_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(SF_ERR_UNSUPPORTED, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_static_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress of the static GEMV scratch");
    g_static_ptr[dev] = p;
  }
  *out = g_static_ptr[dev];
  return SF_OK;
}
}  // namespace

extern "C" int sf_q4_linear_static_scratch(const uint8_t* W, const float* scales, const float* zeros,
                                           const float* bias, const void* X, int x_dtype, void* Y,
                                           int y_dtype, int N, int K, int T, int group_size, void* stream) {
  if (!W || !scales || !X || !Y) return fail(SF_ERR_NULL, "null pointer argument");
  if (x_dtype < 0 || x_dtype > 2 || y_dtype < 0 || y_dtype > 2) return fail(SF_ERR_DTYPE, "unknown dtype code");
  if (N < 0 || K <= 0 || T < 0) return fail(SF_ERR_SHAPE, "invalid N/K/T");
  if (group_size <= 0 || group_size % 2) return fail(SF_ERR_SHAPE, "group_size must be a positive even number");
  if (K % group_size) return fail(SF_ERR_SHAPE, "in_features must be divisible by group_size");
  if (T > kMaxGemvT || !shape_ok(N > 0 ? N : 1, K, group_size))
    return fail(SF_ERR_UNSUPPORTED,
                "static-scratch GEMV takes T <= %d, K %% 32 == 0 and a power-of-two group_size in 32..256",
                kMaxGemvT);
  if ((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(scales) | reinterpret_cast<uintptr_t>(zeros) |
       reinterpret_cast<uintptr_t>(X)) & 15)
    return fail(SF_ERR_ALIGN, "W, scales, zeros and X must be 16-byte aligned");
  const int ntile = (N + kUnitRows - 1) / kUnitRows;
  const size_t cbytes = align256((size_t)ntile * 4);
  const size_t xbytes = xblocks_bytes(T, K, group_size);
  if (cbytes > kStaticCounterBytes || xbytes > kStaticDataBytes)
    return fail(SF_ERR_SHAPE,
                "N=%d K=%d T=%d needs more than the static GEMV scratch holds (%zu KiB of tile counters for "
                "N <= %zu, %zu KiB of activation blocks); use sf_q4_linear",
                N, K, T, kStaticCounterBytes >> 10, (kStaticCounterBytes / 4) * kUnitRows, kStaticDataBytes >> 10);
  if (N == 0 || T == 0) return SF_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* base = nullptr;
  int rc = static_scratch(&base);
  if (rc != SF_OK) return rc;

  TileConfig c;
  if (!make_config(T, zeros != nullptr, group_size, c)) return fail(SF_ERR_UNSUPPORTED, "no launch configuration");
  TileLaunch L{};
  TileTask& q = L.single;
  q.W = W; q.S = scales; q.Z = zeros; q.bias = bias; q.X = X; q.Y = Y; q.xdt = x_dtype; q.ydt = y_dtype;
  // k-split as the allocating entry would choose it, reduced until the
  // partial sums fit next to the activation blocks
  long long want = (c.grid * c.wpc + ntile - 1) / ntile;
  size_t pbytes = 0;
  for (;;) {
    rc = fill_task(q, N, K, group_size, T, want);
    if (rc != SF_OK) return rc;
    pbytes = q.ksplit > 1 ? align256((size_t)q.ksplit * T * N * 4) : 0;
    if (pbytes + xbytes <= kStaticDataBytes || q.ksplit == 1) break;
    want = q.ksplit - 1;
  }
  if (pbytes + xbytes > kStaticDataBytes) return fail(SF_ERR_SHAPE, "static GEMV scratch too small");
  uint8_t* b = static_cast<uint8_t*>(base);
  // The counters must start at zero; a run cut short could have left some set.
  cudaError_t e = cudaMemsetAsync(b, 0, cbytes, st);
  if (e != cudaSuccess) return cuda_fail(e, "clearing the static scratch counters");
  q.tcnt = reinterpret_cast<unsigned int*>(b);
  q.part = pbytes ? reinterpret_cast<float*>(b + kStaticCounterBytes) : nullptr;
  q.xd = b + kStaticCounterBytes + pbytes;
  q.xpre = 1;
  q.ubase = 0;
  q.phase = 0;
  q.ph_last = 1;
  L.tasks = nullptr; L.ntasks = 1; L.total = (long long)q.ntile * q.ksplit;
  L.phctr = nullptr;
  L.flags = nullptr;
  const int need = (int)((L.total + c.wpc - 1) / c.wpc);
  if (c.grid > need) c.grid = need;
  e = launch_xblocks(T, c.LB, 1, L, st, (q.nchunk + 7) / 8);
  if (e != cudaSuccess) return cuda_fail(e, "activation pre-pass launch");
  e = launch_tile(c, L, false, st);
  if (e != cudaSuccess) return cuda_fail(e, "q4_tile_kernel launch");
  g_launches.fetch_add(2, std::memory_order_relaxed);
  return SF_OK;
}
