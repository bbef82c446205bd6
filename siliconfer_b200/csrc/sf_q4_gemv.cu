// sf_q4_gemv.cu -- decode GEMV (T <= 8 tokens) on the sm_100a tensor cores with
// exact integer arithmetic.
//
// Reference semantics (siliconfer/kernels/neon/q4_gemv.cpp:37-140, 145-238;
// siliconfer/kernels/neon/__init__.py:88-124): per output row i and group g,
//   sym : y += s[i,g] * sum_k sext(q[i,k]) * x[k]
//   asym: y += s[i,g] * (sum_k q[i,k] * x[k] - z[i,g] * sum_k x[k])
//
// How it is computed here:
//  * Weights: the nibbles are UNSIGNED int8 A operands.  Symmetric nibbles
//    are flipped (u ^ 8 = q + 8) by the same LOP3 that masks them, so both
//    layouts become  s * (sum u*x - zeff * sum x)  with zeff = 8 (sym) or z
//    (asym).  Unpacking costs 3 integer instructions per 8 weights.
//  * Activations: per (token, group) the values are put on a fixed-point grid
//    x_fix = rint(x * 2^(22-E)), E the binary exponent of the group's max |x|
//    (|x_fix| <= 2^22: every value keeps 22 bits relative to the group max),
//    split into three signed int8 digits x_fix = d0 + 256*d1 + 65536*d2.
//  * mma.sync m16n8k32 u8 x s8 -> s32 accumulates sum u*d EXACTLY; one fp32
//    epilogue per (row, group, token) recombines the digits, subtracts
//    zeff * sum(x_fix) and applies s * 2^(E-22).  The only roundings are the
//    fixed-point rounding of x and the fp32 epilogue and reduction.
//  * Data movement: the producer warp streams W HBM->SMEM with cp.async.bulk
//    into an mbarrier-guarded ring.  When a stage holds whole rows the row
//    block is one contiguous region, copied as >= 4 KB pieces spread over the
//    32 producer lanes (the bulk-copy engine has a per-copy cost, so small
//    copies from one thread cannot keep HBM busy); otherwise each row's slice
//    is one copy into a padded, bank-conflict-free layout.  Each row block's
//    scales and zeros are bulk-copied into a 2-slot ring.
//  * Consumer warps own (K-slice, row-group) pairs; K-slices are whole groups
//    and are reduced through shared memory once per row block.
//  * Programmatic dependent launch: the next kernel may start streaming its
//    own weights while this one finishes; activations are read only after
//    griddepcontrol.wait.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include <cstddef>
#include <cstdint>
#include <cstdlib>
#include <vector>
#include <atomic>

#include "sf_q4.h"
#include "sf_q4_internal.h"

namespace sf {
extern std::atomic<long long> g_launches;
int fail(int code, const char* fmt, ...);

SF_DEFINE_ERROR_READER(take_dev_error_gemv_tc)

namespace {

constexpr int kMT = 2;                 // m16 tiles per warp per row block
constexpr int kImmaMaxThreads = 512;   // consumer warps + weight producer + activation producer
constexpr uint32_t kPiece = 4096;      // contiguous bulk-copy piece (bytes)
constexpr int kSS = 4;                 // scale-ring slots (row blocks of scales in flight)
// shared-memory header: [0,192) mbarriers, [192,256) zero block, then two task slots
constexpr int kZeroOff = 192;
constexpr int kTaskOff = 256;
constexpr int kTaskBytes = (int)sizeof(ImmaParams);
static_assert(sizeof(ImmaParams) % 16 == 0 && alignof(ImmaParams) == 16,
              "descriptors are copied as uint4");
static_assert(offsetof(StepParams, single) % 16 == 0, "embedded descriptor must be 16-byte aligned");

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

// D += A(u8, 16x32) * B(s8, 32x8), s32 accumulate.  Not volatile: it has no
// side effects, so the compiler may interleave independent accumulator chains.
__device__ __forceinline__ void imma(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                     uint32_t a3, uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Low / high nibble of every byte as unsigned bytes; symmetric nibbles are
// flipped to u ^ 8 (= q + 8) in the same instruction.
template <bool ASYM>
__device__ __forceinline__ uint32_t nib_lo(uint32_t w) {
  return (w & 0x0F0F0F0Fu) ^ (ASYM ? 0u : 0x08080808u);
}
template <bool ASYM>
__device__ __forceinline__ uint32_t nib_hi(uint32_t w) {
  return ((w >> 4) & 0x0F0F0F0Fu) ^ (ASYM ? 0u : 0x08080808u);
}

// Low bytes of d[0..7] in B-operand order: word 0 = k offsets {0,2,4,6},
// word 1 = {1,3,5,7} (the A operand's low / high nibbles of one byte run).
__device__ __forceinline__ uint2 pack_digits(const int* d) {
  uint2 r;
  r.x = (uint32_t)(d[0] & 255) | ((uint32_t)(d[2] & 255) << 8) | ((uint32_t)(d[4] & 255) << 16) |
        ((uint32_t)(d[6] & 255) << 24);
  r.y = (uint32_t)(d[1] & 255) | ((uint32_t)(d[3] & 255) << 8) | ((uint32_t)(d[5] & 255) << 16) |
        ((uint32_t)(d[7] & 255) << 24);
  return r;
}

template <int LB>
__device__ __forceinline__ void lds_words(const uint8_t* p, uint32_t* w) {
  if constexpr (LB == 16) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if constexpr (LB == 8) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    w[0] = v.x; w[1] = v.y;
  } else {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
}

// B digits of one segment for one lane: 2*LB bytes.
template <int LB>
__device__ __forceinline__ void lds_digits(const uint8_t* p, uint32_t* b) {
  if constexpr (LB == 16) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint4 v = *reinterpret_cast<const uint4*>(p + 16);
    b[0] = u.x; b[1] = u.y; b[2] = u.z; b[3] = u.w; b[4] = v.x; b[5] = v.y; b[6] = v.z; b[7] = v.w;
  } else if constexpr (LB == 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    b[0] = u.x; b[1] = u.y; b[2] = u.z; b[3] = u.w;
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    b[0] = u.x; b[1] = u.y;
  }
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
__device__ __forceinline__ float ldsf(uint32_t a) { return __uint_as_float(lds32(a)); }

// LB packed bytes of one A row at shared address a.
template <int LB>
__device__ __forceinline__ void lds_words_s(uint32_t a, uint32_t* w) {
  if constexpr (LB == 16) {
    const uint4 v = lds128(a);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if constexpr (LB == 8) {
    const uint2 v = lds64(a);
    w[0] = v.x; w[1] = v.y;
  } else {
    w[0] = lds32(a);
  }
}

// 2*LB digit bytes of one B column at shared address a.
template <int LB>
__device__ __forceinline__ void lds_digits_s(uint32_t a, uint32_t* b) {
  if constexpr (LB == 16) {
    const uint4 u = lds128(a), v = lds128(a + 16);
    b[0] = u.x; b[1] = u.y; b[2] = u.z; b[3] = u.w; b[4] = v.x; b[5] = v.y; b[6] = v.z; b[7] = v.w;
  } else if constexpr (LB == 8) {
    const uint4 u = lds128(a);
    b[0] = u.x; b[1] = u.y; b[2] = u.z; b[3] = u.w;
  } else {
    const uint2 u = lds64(a);
    b[0] = u.x; b[1] = u.y;
  }
}

}  // namespace

// Optional timeline (build with -DSF_GEMV_TRACE): per CTA 16 slots of
// %globaltimer (ns) written to the buffer given to sf_q4_gemv_set_trace.
#ifdef SF_GEMV_TRACE
__device__ unsigned long long* g_gtrace = nullptr;
#define GT(slot)                                                                         \
  do {                                                                                   \
    if (g_gtrace)                                                                        \
      g_gtrace[((size_t)sp.trace_id * gridDim.x + blockIdx.x) * 16 + (slot)] = globaltimer_ns(); \
  } while (0)
// per-task stamps: slot = task * 4 + k, 1024 slots per CTA
#define GTT(ti, k)                                                                       \
  do {                                                                                   \
    if (g_gtrace && (ti) < 128)                                                          \
      g_gtrace[(size_t)blockIdx.x * 1024 + (ti) * 8 + (k)] = globaltimer_ns();           \
  } while (0)
#else
#define GT(slot) do { } while (0)
#define GTT(ti, k) do { } while (0)
#endif

// ---------------------------------------------------------------------------
// Task-list kernel.  A task is one GEMV (ImmaParams); StepParams carries the
// launch-wide shared-memory layout.  The producer warp walks every task's row
// blocks and k-chunks without waiting on anything but ring slots; consumers
// walk the same sequence, so both sides agree on every ring slot and phase.
// ---------------------------------------------------------------------------
__device__ __forceinline__ const ImmaParams& task_at(const StepParams& sp, int i) {
  return sp.tasks ? sp.tasks[i] : sp.single;
}

// Wait until every CTA has finished tasks [from, upto).  done[i] counts the
// CTAs that finished task i, so this stays correct when the two consumer
// groups finish out of order.  Cooperative launch: all CTAs are resident.
// Bounded: on timeout the sticky error word is set and the caller stops waiting.
__device__ __forceinline__ bool wait_tasks(const unsigned int* done, int from, int upto, int gtid,
                                           int bid, int nthr, bool enabled) {
  __shared__ int ok_s[2];
  if (gtid == 0) {
    const long long t0 = clock64();
    int ok = enabled ? 1 : 0;
    for (int i = from; i < upto && ok; ++i) {
      while (true) {
        unsigned int v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(done + i) : "memory");
        if (v >= gridDim.x) break;
        if (clock64() - t0 > kWaitCycles) {
          atomicOr(&g_dev_error, 2u);
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    ok_s[bid - 1] = ok;
  }
  named_barrier_sync(bid, nthr);
  return ok_s[bid - 1] != 0;
}

template <int T, bool ASYM, int LB>
__global__ void __launch_bounds__(kImmaMaxThreads, 1) q4_gemv_imma_kernel(const __grid_constant__ StepParams sp) {
  constexpr int NTG = (T + 3) / 4;    // token groups of 4 (one token per lane t)
  constexpr int NT = 2 * NTG;         // n8 tiles: (d0,d1) and (d2,-) per token group
  constexpr int WPL = LB / 4;         // 32-bit words per lane per row per segment
  constexpr int SEGK = 8 * LB;        // k values per segment (4 lanes x 2*LB)
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  uint64_t* sfull = empty + kMaxStages;
  uint64_t* sempty = sfull + kSS;
  uint64_t* xfull = sempty + kSS;             // per consumer group: its activation buffer
  uint64_t* xempty = xfull + 2;
  float* red;
  float* xgsc;
  uint8_t* xb;
  uint8_t* sring = smem + sp.sring_base;
  uint8_t* stages = smem + sp.stage_base;
  const uint8_t* zblk = smem + kZeroOff;   // 64 zero bytes (B operand of unused columns)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int ncons = sp.ncons;

  if (threadIdx.x == 0) {
    // each stage / scale slot is consumed by exactly one consumer group
    const int gw = ncons / sp.npp;
    for (int i = 0; i < sp.nst; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], gw); }
    for (int i = 0; i < kSS; ++i) { mbar_init(&sfull[i], 1); mbar_init(&sempty[i], gw); }
    for (int i = 0; i < 2; ++i) { mbar_init(&xfull[i], 1); mbar_init(&xempty[i], 1); }
    fence_mbar_init();
  }
  if (threadIdx.x < 16) reinterpret_cast<uint32_t*>(smem + kZeroOff)[threadIdx.x] = 0u;
  // first descriptor of each consumer group -> its slot 0
  for (int gq = 0; gq < sp.npp && gq < sp.ntasks; ++gq)
    if (threadIdx.x < kTaskBytes / 16)
      reinterpret_cast<uint4*>(smem + kTaskOff + gq * 2 * kTaskBytes)[threadIdx.x] =
          reinterpret_cast<const uint4*>(&task_at(sp, gq))[threadIdx.x];
  // Each consumer group owns a slice of the weight ring (nst / npp stages) and
  // of the scale ring (kSS / npp slots), so every ring slice has one in-order
  // consumer and mbarrier parity waits stay unambiguous.  cbase / bbase: the
  // position in its group's slices at which each task starts in this CTA.
  int* cbase = reinterpret_cast<int*>(smem + sp.tb_base);
  int* bbase = cbase + sp.ntasks + 1;
  for (int i = threadIdx.x; i < sp.ntasks; i += blockDim.x) {
    const ImmaParams& q = task_at(sp, i);
    const int rb = (int)((unsigned)q.N * blockIdx.x / gridDim.x);
    const int re = (int)((unsigned)q.N * (blockIdx.x + 1) / gridDim.x);
    const int nrb = (re - rb + q.R - 1) / q.R;
    cbase[i + 1] = nrb * ((q.K + q.KC - 1) / q.KC);
    bbase[i + 1] = nrb;
  }
  __syncthreads();
  if (threadIdx.x == 0) {   // per consumer group: exclusive prefix over that group's tasks
    int rc[2] = {0, 0}, rbk[2] = {0, 0};
    for (int i = 0; i < sp.ntasks; ++i) {
      const int gq = i % sp.npp;
      const int cc = cbase[i + 1], bc = bbase[i + 1];
      cbase[i] = rc[gq];
      bbase[i] = rbk[gq];
      rc[gq] += cc;
      rbk[gq] += bc;
    }
  }
  __syncthreads();
  griddep_launch_dependents();

  if (warp == ncons + 1) {
    // ------------------------- activation producer -------------------------
    // Tasks whose activations were pre-converted (p.xd) get them bulk-copied
    // into their consumer group's buffer once that group has finished its
    // previous task.  A warp of its own, so the weight stream never waits here.
    if (lane == 0) {
      int gown[2] = {0, 0};
      for (int ti = 0; ti < sp.ntasks; ++ti) {
        const ImmaParams& p = task_at(sp, ti);
        const int gq = ti % sp.npp;
        const int k = gown[gq]++;
        // wait for the group's previous task on EVERY task, so that this
        // waiter is never more than one phase ahead of the barrier
        if (k > 0 && !mbar_wait(&xempty[gq], (k - 1) & 1, 0x100u)) return;
        if (!p.xd) continue;
        const uint32_t xsb = (uint32_t)((T * p.G * 8 + 15) & ~15);
        mbar_arrive_expect_tx(&xfull[gq], (uint32_t)(3 * T * p.K) + xsb);
        uint8_t* dst = smem + sp.xb_base + gq * sp.xb_half;
        for (int tok = 0; tok < T; ++tok)
          for (int dg = 0; dg < 3; ++dg)
            bulk_g2s(dst + (size_t)tok * p.TS + (size_t)dg * p.CSB,
                     p.xd + (size_t)(tok * 3 + dg) * p.K, (uint32_t)p.K, &xfull[gq]);
        bulk_g2s(smem + sp.xs_base + gq * sp.xs_half, p.xd + (size_t)3 * T * p.K, xsb, &xfull[gq]);
      }
    }
    return;
  }

  if (warp == ncons) {
    // ------------------------------ producer ------------------------------
    int cg[2] = {0, 0}, bg[2] = {0, 0};
    const int nstg = sp.nst / sp.npp, ssg = kSS / sp.npp;
    for (int ti = 0; ti < sp.ntasks; ++ti) {
      const ImmaParams& p = task_at(sp, ti);
      const int gq = ti % sp.npp;
      int& c = cg[gq];
      int& b = bg[gq];
      const int rb = (int)((unsigned)p.N * blockIdx.x / gridDim.x);
      const int re = (int)((unsigned)p.N * (blockIdx.x + 1) / gridDim.x);
      const int nrb = (re - rb + p.R - 1) / p.R;
      const int nkc = (p.K + p.KC - 1) / p.KC;
      const int KH = p.K >> 1;
      for (int bb = 0; bb < nrb; ++bb, ++b) {
        const int r0 = rb + bb * p.R;
        const int rows = min(p.R, re - r0);
        const int sl = gq * ssg + b % ssg;
        int ok = 1;
        if (lane == 0 && b >= ssg) ok = mbar_wait(&sempty[sl], ((b / ssg) - 1) & 1, 0x40u);
        if (!__shfl_sync(0xffffffffu, ok, 0)) return;
        if (lane == 0 && bb == 0) GTT(ti, 4);
        if (lane == 0) {  // scales (+ zeros) of the row block, from the 16-byte boundary below
          const uintptr_t src = reinterpret_cast<uintptr_t>(p.S + (size_t)r0 * p.G);
          const uint32_t pre = (uint32_t)(src & 15);
          const uint32_t nb = (pre + (uint32_t)rows * p.G * 4) & ~15u;
          uint8_t* dst = sring + (size_t)sl * sp.sring_bytes;
          mbar_arrive_expect_tx(&sfull[sl], ASYM ? 2 * nb : nb);
          if (nb) {
            bulk_g2s(dst, reinterpret_cast<const void*>(src - pre), nb, &sfull[sl]);
            if (ASYM)
              bulk_g2s(dst + sp.sring_bytes / 2,
                       reinterpret_cast<const uint8_t*>(p.Z + (size_t)r0 * p.G) - pre, nb,
                       &sfull[sl]);
          }
        }
        for (int kc = 0; kc < nkc; ++kc, ++c) {
          const int st = gq * nstg + c % nstg, use = c / nstg;
          ok = 1;
          if (lane == 0 && use > 0) ok = mbar_wait(&empty[st], (use - 1) & 1, 0x20u);
          if (!__shfl_sync(0xffffffffu, ok, 0)) return;
          const int k0 = kc * p.KC;
          const uint32_t cb = (uint32_t)(min(p.KC, p.K - k0) >> 1);
          uint8_t* buf = stages + (size_t)st * sp.stage_bytes;
          if (lane == 0 && bb == 0 && kc == 0) GTT(ti, 5);
          if (sp.dbg & 1) {   // development: stage completes without data
            if (lane == 0) mbar_arrive_expect_tx(&full[st], 0);
            continue;
          }
          if (lane == 0) mbar_arrive_expect_tx(&full[st], cb * rows);
          __syncwarp();
          const uint8_t* src = p.W + (size_t)r0 * KH + (k0 >> 1);
          if (p.contiguous) {
            const uint32_t total = cb * rows;   // multiple of 16
            const uint32_t npc = (total + kPiece - 1) / kPiece;
            for (uint32_t j = lane; j < npc; j += 32) {
              const uint32_t off = j * kPiece;
              const uint32_t n = total - off < kPiece ? total - off : kPiece;
              bulk_g2s(buf + off, src + off, n, &full[st]);
            }
          } else {
            for (int r = lane; r < rows; r += 32)
              bulk_g2s(buf + (size_t)r * p.RS, src + (size_t)r * KH, cb, &full[st]);
          }
        }
      }
    }
    return;
  }

  // ------------------------------ consumers -------------------------------
  // npp consumer groups take alternate tasks (ping-pong): while one group does
  // a task's fixed work (dependency wait, activation staging, reduction) the
  // other keeps the tensor cores busy.  Each group owns its activation buffer,
  // reduction buffer, descriptor slots and named barrier.
  const int npp = sp.npp;
  const int GW = ncons / npp;
  const int grp = warp / GW;
  const int cw = warp - grp * GW;               // warp index inside the group
  const int nthr = GW * 32;
  const int gtid = threadIdx.x - grp * nthr;    // thread index inside the group
  const int bid = 1 + grp;                      // named barrier of this group
  xgsc = reinterpret_cast<float*>(smem + sp.xs_base + grp * sp.xs_half);
  xb = smem + sp.xb_base + grp * sp.xb_half;
  red = reinterpret_cast<float*>(smem + sp.red_base) + grp * 2 * sp.red_half;
  uint8_t* tslot = smem + kTaskOff + grp * 2 * kTaskBytes;
  griddep_wait();
  bool ok_wait = true;
  int own = 0, nxpre = 0;

  for (int ti = grp; ti < sp.ntasks; ti += npp, ++own) {
    named_barrier_sync(bid, nthr);   // this group's slot own & 1 is complete and visible
    const ImmaParams& p = *reinterpret_cast<const ImmaParams*>(tslot + (own & 1) * kTaskBytes);
    int c = cbase[ti], b = bbase[ti];   // positions in this group's ring slices
    // prefetch the group's next descriptor; stored into the other slot at the end of this task
    uint4 tnext = make_uint4(0, 0, 0, 0);
    const bool tpre = ti + npp < sp.ntasks && gtid < kTaskBytes / 16;
    if (tpre) tnext = __ldg(reinterpret_cast<const uint4*>(&task_at(sp, ti + npp)) + gtid);
    if (p.wait_before)   // every thread of the group takes part (named barrier inside)
      ok_wait = wait_tasks(sp.done, p.wait_from, ti, gtid, bid, nthr, ok_wait) && ok_wait;
    float* xsum = xgsc + T * p.G;
    if (gtid == 0) GTT(ti, 0);
    const bool xpre = p.xd != nullptr;
    if (xpre) {   // the phase count advances even after an earlier timeout
      const uint32_t par = (uint32_t)(nxpre++) & 1;
      if (ok_wait) ok_wait = mbar_wait(&xfull[grp], par, 0x4u);
    }

    // (1) activations -> per-(token, group) fixed point, three int8 digits.
    //     Token-major; all of a thread's loads for a pass are issued before
    //     any is used; loads go through L2 (an earlier task may have written x).
    const int lg2gs = p.lg2gs, G = p.G;
    if (!(sp.dbg & 2) && !xpre) {
      const int octs = p.K >> 3;
      const int lpg = 1 << (lg2gs - 3);  // octets (lanes) per group: 4, 8, 16 or 32
      const void* X = p.X;
      const int xdt = p.xdt, Kx = p.K;
      const uint32_t TSx = p.TS, CSBx = p.CSB;
      constexpr int NB = 4;
      for (int tok = 0; tok < T; ++tok) {
        for (int base = cw * 32; base < octs; base += nthr * NB) {
          float v[NB][8];
#pragma unroll
          for (int i = 0; i < NB; ++i) {
            const int o = base + i * nthr + lane;
            if (o < octs) ld_x8(X, (size_t)tok * Kx + (size_t)o * 8, xdt, v[i]);
            else {
#pragma unroll
              for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
            }
          }
#pragma unroll
          for (int i = 0; i < NB; ++i) {
            const int ob = base + i * nthr;
            if (ob >= octs) break;                         // uniform across the warp
            const int o = ob + lane;
            float m = 0.f;
            bool bad = false;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              m = fmaxf(m, fabsf(v[i][j]));
              bad |= !(fabsf(v[i][j]) <= 3.402823466e38f);
            }
            int badi = bad;
            for (int off = 1; off < lpg; off <<= 1) {
              m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
              badi |= __shfl_xor_sync(0xffffffffu, badi, off);
            }
            // binary exponent field of the group max; groups below 2^-105 are zero
            const int be = (int)(__float_as_uint(m) >> 23);
            const bool zero = badi || be < 22;
            const float scl = zero ? 0.f : __uint_as_float((uint32_t)(275 - be) << 23);   // 2^(22-E)
            int d[3][8];
            int s = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int xf = __float2int_rn(v[i][j] * scl);
              s += xf;
              const int d0 = (xf << 24) >> 24;
              const int r1 = (xf - d0) >> 8;
              const int d1 = (r1 << 24) >> 24;
              d[0][j] = d0;
              d[1][j] = d1;
              d[2][j] = (r1 - d1) >> 8;
            }
            for (int off = 1; off < lpg; off <<= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
            if (o < octs) {
              uint8_t* col = xb + (size_t)tok * TSx + (size_t)o * 8;
#pragma unroll
              for (int dg = 0; dg < 3; ++dg)
                *reinterpret_cast<uint2*>(col + (size_t)dg * CSBx) = pack_digits(d[dg]);
              if ((lane & (lpg - 1)) == 0) {
                const int gi = (o * 8) >> lg2gs;
                xgsc[tok * G + gi] = badi ? __int_as_float(0x7fc00000)
                                          : (zero ? 0.f : __uint_as_float((uint32_t)(be - 21) << 23));
                xsum[tok * G + gi] = (float)s;
              }
            }
          }
        }
      }
    }
    named_barrier_sync(bid, nthr);
    if (gtid == 0) GTT(ti, 1);

    // (2) stream the row blocks of this task.  Task fields are copied into
    //     registers once; the hot loop uses 32-bit shared-memory addresses.
    const int N = p.N, KS = p.KS, R = p.R, KC = p.KC, GPS = p.GPS;
    const int Kt = p.K;
    const uint32_t RS = p.RS;
    const float* __restrict__ Sg = p.S;
    const float* __restrict__ Zg = p.Z;
    const float* __restrict__ biasg = p.bias;
    void* Yg = p.Y;
    const int ydt = p.ydt;
    const int rb = (int)((unsigned)N * blockIdx.x / gridDim.x);
    const int re = (int)((unsigned)N * (blockIdx.x + 1) / gridDim.x);
    const int nrb = (re - rb + R - 1) / R;
    const int nkc = (Kt + KC - 1) / KC;
    const int ks = cw % KS, rgp = cw / KS;
    const bool active = rgp < p.RG;   // warps beyond KS*RG only keep the barriers moving
    const uint32_t smem_s = smem_u32(smem);
    // B columns this lane supplies, per n8 tile; lanes without a column read a
    // zero block (no divergence, a broadcast read).
    uint32_t bcs[NT], binc[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int tok = (nt >> 1) * 4 + (g >> 1);
      const int dg = (nt & 1) ? ((g & 1) ? -1 : 2) : (g & 1);
      const bool v = tok < T && dg >= 0;
      bcs[nt] = v ? smem_u32(xb) + (uint32_t)tok * p.TS + (uint32_t)dg * p.CSB + t * 2 * LB
                  : smem_s + kZeroOff;
      binc[nt] = v ? 1u : 0u;
    }
    const int row0 = rgp * kMT * 16 + g;   // this lane's first A row inside a row block
    const uint32_t mo1 = 8 * RS, mo2 = 16 * RS, mo3 = 24 * RS;
    const uint32_t gsc_s = smem_u32(xgsc);
    const uint32_t xsum_s = gsc_s + (uint32_t)T * G * 4;

    for (int bb = 0; bb < nrb; ++bb, ++b) {
      const int r0 = rb + bb * R;
      const int rows = min(R, re - r0);
      float acc[kMT][NTG][2];
#pragma unroll
      for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
        for (int tg = 0; tg < NTG; ++tg) acc[mt][tg][0] = acc[mt][tg][1] = 0.f;
      const int sl = grp * (kSS / npp) + b % (kSS / npp);
      if (gtid == 0 && bb == 0) GTT(ti, 6);
      if (ok_wait) ok_wait = mbar_wait(&sfull[sl], (b / (kSS / npp)) & 1, 0x8u);
      if (gtid == 0 && bb == 0) GTT(ti, 7);
      float* ssm = reinterpret_cast<float*>(sring + (size_t)sl * sp.sring_bytes);
      float* zsm = ssm + sp.sring_bytes / 8;
      const int s_pre = (int)(reinterpret_cast<uintptr_t>(Sg + (size_t)r0 * G) & 15) >> 2;
      const int s_end = s_pre + rows * G;
      const int s_cnt = s_end & ~3;
      if (s_cnt < s_end) {   // the last (< 4) values were not bulk-copied: fetch them
        const int i = gtid;
        if (i < s_end - s_cnt) {
          const size_t gi0 = (size_t)r0 * G - s_pre + s_cnt + i;
          ssm[s_cnt + i] = __ldg(Sg + gi0);
          if (ASYM) zsm[s_cnt + i] = __ldg(Zg + gi0);
        }
        named_barrier_sync(bid, nthr);
      }
      // scale / zero addresses of this lane's rows (rows past the block read stale values)
      const uint32_t ss_s = smem_u32(ssm), zs_s = smem_u32(zsm);
      uint32_t so[kMT][2];
#pragma unroll
      for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) so[mt][h] = (uint32_t)(s_pre + min(row0 + mt * 16 + 8 * h, rows - 1) * G) * 4;

      for (int kc = 0; kc < nkc; ++kc, ++c) {
        const int st = grp * (sp.nst / npp) + c % (sp.nst / npp), use = c / (sp.nst / npp);
        const int k0 = kc * KC;
        const int gc0 = k0 >> lg2gs;
        const int gcn = min(KC, Kt - k0) >> lg2gs;
        const int ga = active ? gc0 + min(gcn, ks * GPS) : 0;
        const int gb = active ? gc0 + min(gcn, (ks + 1) * GPS) : 0;
        if (ok_wait) ok_wait = mbar_wait(&full[st], use & 1, 0x10u);
        if (gtid == 0 && bb == 0 && kc == 0) GTT(ti, 2);
        // A address of (row0, k = 0) in this stage
        const uint32_t a_s = smem_s + sp.stage_base + (uint32_t)st * sp.stage_bytes +
                             (uint32_t)row0 * RS + t * LB - (uint32_t)(k0 >> 1);

        for (int gi = ga; gi < gb && ok_wait; ++gi) {
          float sc[kMT][2], zp[kMT][2];
#pragma unroll
          for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              sc[mt][h] = ldsf(ss_s + so[mt][h] + gi * 4);
              zp[mt][h] = ASYM ? ldsf(zs_s + so[mt][h] + gi * 4) : 8.f;
            }
          int C[kMT][NT][4];
#pragma unroll
          for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) C[mt][nt][0] = C[mt][nt][1] = C[mt][nt][2] = C[mt][nt][3] = 0;

          const int kend = (gi + 1) << lg2gs;
          for (int kseg = gi << lg2gs; kseg < kend; kseg += SEGK) {
            uint32_t bq[NT][2 * WPL];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) lds_digits_s<LB>(bcs[nt] + (uint32_t)kseg * binc[nt], bq[nt]);
            const uint32_t ap = a_s + (uint32_t)(kseg >> 1);
            uint32_t w0[kMT][WPL], w1[kMT][WPL];
            lds_words_s<LB>(ap, w0[0]);
            lds_words_s<LB>(ap + mo1, w1[0]);
            lds_words_s<LB>(ap + mo2, w0[1]);
            lds_words_s<LB>(ap + mo3, w1[1]);
#pragma unroll
            for (int q = 0; q < WPL; ++q)
#pragma unroll
              for (int mt = 0; mt < kMT; ++mt) {
                const uint32_t a0 = nib_lo<ASYM>(w0[mt][q]), a2 = nib_hi<ASYM>(w0[mt][q]);
                const uint32_t a1 = nib_lo<ASYM>(w1[mt][q]), a3 = nib_hi<ASYM>(w1[mt][q]);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
                  imma(C[mt][nt], a0, a1, a2, a3, bq[nt][2 * q], bq[nt][2 * q + 1]);
              }
          }
          // epilogue of group gi: recombine digits, remove zeff * sum(x), scale.
          // Lanes whose token does not exist compute on token T-1 and are never stored.
#pragma unroll
          for (int tg = 0; tg < NTG; ++tg) {
            const uint32_t tok = (uint32_t)min(tg * 4 + t, T - 1);
            const float gsc = ldsf(gsc_s + (tok * G + gi) * 4);
            const float xs = ldsf(xsum_s + (tok * G + gi) * 4);
#pragma unroll
            for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int i01 = C[mt][2 * tg][2 * h] + 256 * C[mt][2 * tg][2 * h + 1];
                float f = fmaf(65536.f, (float)C[mt][2 * tg + 1][2 * h], (float)i01);
                f = fmaf(-zp[mt][h], xs, f);
                acc[mt][tg][h] = fmaf(f, sc[mt][h] * gsc, acc[mt][tg][h]);
              }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
      }

      // (3) reduce the K-slices of this row block and write y
      float* rbuf = red + (b & 1) * sp.red_half;
      if (active) {
#pragma unroll
        for (int tg = 0; tg < NTG; ++tg) {
          const int tok = tg * 4 + t;
          if (tok < T) {
#pragma unroll
            for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
              for (int h = 0; h < 2; ++h)
                rbuf[(ks * T + tok) * R + row0 + mt * 16 + 8 * h] = acc[mt][tg][h];
          }
        }
      }
      named_barrier_sync(bid, nthr);
      __syncwarp();
      if (lane == 0) mbar_arrive(&sempty[sl]);
      for (int idx = gtid; idx < rows * T; idx += nthr) {
        const int tok = idx / rows, r = idx - tok * rows;
        float a = 0.f;
        for (int k = 0; k < KS; ++k) a += rbuf[(k * T + tok) * R + r];
        if (biasg) a += __ldg(biasg + r0 + r);
        st_y(Yg, (size_t)tok * N + r0 + r, a, ydt);
      }
    }
    if (tpre) reinterpret_cast<uint4*>(tslot + ((own + 1) & 1) * kTaskBytes)[gtid] = tnext;
    named_barrier_sync(bid, nthr);   // the whole group is done with this task
    if (gtid == 0) {
      mbar_arrive(&xempty[grp]);      // its activation buffer may be refilled
      if (sp.done) {                  // publish completion of task ti by this CTA
        __threadfence();
        atomicAdd(sp.done + ti, 1u);
      }
    }
    if (gtid == 0) GTT(ti, 3);
  }
}

// ---------------------------------------------------------------------------
// Activation pre-pass for tasks whose X does not depend on earlier tasks: the
// same fixed-point digit split as the in-kernel staging, written once to a
// scratch arena ([T][3][K] digit bytes, then [T][G] group scales and [T][G]
// sums), so that the GEMV kernel only bulk-copies it.  One CTA per task.
// ---------------------------------------------------------------------------
template <int T>
__global__ void __launch_bounds__(256) q4_x_digits_kernel(const ImmaParams* __restrict__ tasks) {
  const ImmaParams& p = tasks[blockIdx.x];
  if (!p.xd) return;
  const int lane = threadIdx.x & 31;
  const int octs = p.K >> 3, total = T * octs;
  const int lpg = 1 << (p.lg2gs - 3);
  float* gsc = reinterpret_cast<float*>(p.xd + (size_t)3 * T * p.K);
  float* xsm = gsc + T * p.G;
  for (int ob = (threadIdx.x >> 5) * 32; ob < total; ob += blockDim.x) {
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
    const int be = (int)(__float_as_uint(m) >> 23);
    const bool zero = bad || be < 22;
    const float scl = zero ? 0.f : __uint_as_float((uint32_t)(275 - be) << 23);
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
    if (ok) {
#pragma unroll
      for (int dg = 0; dg < 3; ++dg)
        *reinterpret_cast<uint2*>(p.xd + (size_t)(tok * 3 + dg) * p.K + (size_t)oo * 8) = pack_digits(d[dg]);
      if ((lane & (lpg - 1)) == 0) {
        const int gi = (oo * 8) >> p.lg2gs;
        gsc[tok * p.G + gi] = bad ? __int_as_float(0x7fc00000)
                                  : (zero ? 0.f : __uint_as_float((uint32_t)(be - 21) << 23));
        xsm[tok * p.G + gi] = (float)s;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {

int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return v && *v ? atoi(v) : dflt;
}

// smallest y >= x with y % mod == target
size_t pad_to(size_t x, size_t mod, size_t target) {
  const size_t r = x % mod;
  return x + ((target + mod - r) % mod);
}

int lb_for(int gs) { return (gs % 128 == 0) ? 16 : (gs % 64 == 0 ? 8 : 4); }

struct Need {
  size_t red_half = 0, xs = 0, xb = 0, sring_half = 0;
};

// Per-task plan.  `stage` is the launch-wide stage size in bytes.
bool plan_task(int N, int K, int T, int gs, int ncons, int grid, size_t stage, ImmaParams& q,
               Need& need) {
  if (N < 1 || K % 32 || gs < 32 || gs > 256 || (gs & (gs - 1)) || K % gs) return false;
  const int LB = lb_for(gs);
  const int G = K / gs;
  const int rows_cta = (N + grid - 1) / grid;
  int KS = ncons < G ? ncons : G;
  int RG = ncons / KS;
  const int rg_need = (rows_cta + 16 * kMT - 1) / (16 * kMT);
  if (RG > rg_need) RG = rg_need;
  if (RG > 2) RG = 2;
  if (RG < 1) RG = 1;
  const int R = RG * kMT * 16;
  int KC, contiguous;
  size_t RS;
  if ((size_t)R * (K / 2) <= stage) {
    KC = K; RS = K / 2; contiguous = 1;
  } else {
    long long kc = (long long)(stage / R) * 2;
    kc = (kc / gs) * gs;
    if (kc < gs) return false;
    for (;;) {   // padded rows must still fit the stage
      RS = pad_to((size_t)kc / 2, 128, (size_t)4 * LB);
      if ((size_t)R * RS <= stage || kc <= gs) break;
      kc -= gs;
    }
    if ((size_t)R * RS > stage) return false;
    KC = (int)kc; contiguous = 0;
  }
  const size_t csb_target = LB == 16 ? 16 : (LB == 8 ? 64 : 32);
  const size_t CSB = pad_to((size_t)K, 128, csb_target);
  const size_t TS = pad_to(3 * CSB, 128, LB == 4 ? 64 : 0);
  q.N = N; q.K = K; q.G = G; q.gs = gs; q.lg2gs = __builtin_ctz((unsigned)gs);
  q.KS = KS; q.RG = RG; q.R = R; q.KC = KC; q.GPS = (KC / gs + KS - 1) / KS;
  q.contiguous = contiguous; q.RS = (uint32_t)RS; q.CSB = (uint32_t)CSB; q.TS = (uint32_t)TS;
  const size_t rh = (size_t)KS * T * R * 4;
  const size_t xs = (size_t)2 * T * G * 4;
  const size_t xb = (size_t)T * TS;
  const size_t sh = ((size_t)R * G * 4 + 16 + 127) & ~(size_t)127;
  if (rh > need.red_half) need.red_half = rh;
  if (xs > need.xs) need.xs = xs;
  if (xb > need.xb) need.xb = xb;
  if (sh > need.sring_half) need.sring_half = sh;
  return true;
}

// Lay out shared memory; false when it does not fit.
bool finish_plan(const Need& need, size_t stage, long long nchunks_max, StepPlan& pl) {
  const DeviceInfo& di = device_info();
  StepParams& sp = pl.sp;
  const int npp = sp.npp;
  const size_t red_base = kTaskOff + 4 * kTaskBytes;
  const size_t tb_base = (red_base + (size_t)npp * 2 * need.red_half + 15) & ~(size_t)15;
  const size_t xs_half = (need.xs + 15) & ~(size_t)15;
  const size_t xs_base = (tb_base + (size_t)8 * (sp.ntasks + 1) + 15) & ~(size_t)15;
  const size_t xb_half = (need.xb + 127) & ~(size_t)127;
  const size_t xb_base = (xs_base + npp * xs_half + 127) & ~(size_t)127;
  const size_t sring_bytes = (pl.asym ? 2 : 1) * need.sring_half;   // zeros in the upper half
  const size_t sring_base = (xb_base + npp * xb_half + 127) & ~(size_t)127;
  const size_t stage_base = sring_base + kSS * sring_bytes;
  const size_t budget = (size_t)env_int("SF_GEMV_SMEM_KB", 220) * 1024;
  const size_t cap = budget < (size_t)di.smem_optin ? budget : (size_t)di.smem_optin;
  if (stage_base + (nchunks_max > 1 ? 2 : 1) * stage > cap) return false;
  long long S = (long long)((cap - stage_base) / stage);
  const int want_st = env_int("SF_GEMV_STAGES", 4);
  if (S > want_st) S = want_st;
  if (S > kMaxStages) S = kMaxStages;
  if (S > nchunks_max) S = nchunks_max;
  S -= S % npp;                        // equal ring slices per consumer group
  if (S < npp) S = npp;
  if (stage_base + (size_t)S * stage > cap) return false;
  sp.nst = (int)S;
  sp.stage_bytes = (uint32_t)stage;
  sp.stage_base = (uint32_t)stage_base;
  sp.red_base = (uint32_t)red_base;
  sp.red_half = (uint32_t)(need.red_half / 4);
  sp.tb_base = (uint32_t)tb_base;
  sp.xs_base = (uint32_t)xs_base;
  sp.xs_half = (uint32_t)xs_half;
  sp.xb_base = (uint32_t)xb_base;
  sp.xb_half = (uint32_t)xb_half;
  sp.sring_base = (uint32_t)sring_base;
  sp.sring_bytes = (uint32_t)sring_bytes;
  pl.smem = stage_base + (size_t)S * stage;
  pl.threads = (sp.ncons + 2) * 32;   // + weight producer + activation producer
  return pl.threads <= kImmaMaxThreads;
}

long long task_chunks(const ImmaParams& q, int grid) {
  const int rows_cta = (q.N + grid - 1) / grid;
  return (long long)((rows_cta + q.R - 1) / q.R) * ((q.K + q.KC - 1) / q.KC);
}

template <int T, bool ASYM, int LB>
cudaError_t launch_t(const StepPlan& pl, cudaStream_t st, bool pdl) {
  auto* fn = q4_gemv_imma_kernel<T, ASYM, LB>;
  static int configured[kMaxDevices] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < kMaxDevices && configured[dev] < (int)pl.smem) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
    if (e != cudaSuccess) return e;
    configured[dev] = (int)pl.smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)pl.grid);
  cfg.blockDim = dim3((unsigned)pl.threads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (pl.coop) {
    attr[na].id = cudaLaunchAttributeCooperative;
    attr[na].val.cooperative = 1;
    ++na;
  }
  cfg.attrs = na ? attr : nullptr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, fn, pl.sp);
}

template <bool ASYM, int LB>
cudaError_t launch_lb(const StepPlan& pl, cudaStream_t st, bool pdl) {
  switch (pl.T) {
    case 1: return launch_t<1, ASYM, LB>(pl, st, pdl);
    case 2: return launch_t<2, ASYM, LB>(pl, st, pdl);
    case 3: return launch_t<3, ASYM, LB>(pl, st, pdl);
    case 4: return launch_t<4, ASYM, LB>(pl, st, pdl);
    case 5: return launch_t<5, ASYM, LB>(pl, st, pdl);
    case 6: return launch_t<6, ASYM, LB>(pl, st, pdl);
    case 7: return launch_t<7, ASYM, LB>(pl, st, pdl);
    default: return launch_t<8, ASYM, LB>(pl, st, pdl);
  }
}

#ifdef SF_GEMV_TRACE
int g_trace_counter = 0;
#endif

}  // namespace

#ifdef SF_GEMV_TRACE
extern "C" int sf_q4_gemv_set_trace(unsigned long long* buf) {
  g_trace_counter = 0;
  return cudaMemcpyToSymbol(g_gtrace, &buf, sizeof(buf)) == cudaSuccess ? 0 : 5;
}
#endif

bool plan_gemv_imma(int N, int K, int T, int gs, bool asym, StepPlan& pl) {
  if (T < 1 || T > kMaxGemvT) return false;
  const DeviceInfo& di = device_info();
  int grid = di.sms * env_int("SF_GEMV_CTAS_PER_SM", 1);
  const int max_grid = (N + 15) / 16;                  // at least one 16-row tile per CTA
  if (grid > max_grid) grid = max_grid;
  if (grid < 1) grid = 1;
  pl = StepPlan{};
  pl.T = T; pl.asym = asym; pl.LB = lb_for(gs); pl.grid = grid; pl.coop = false;
  StepParams& sp = pl.sp;
  sp.ncons = env_int("SF_GEMV_WARPS", 14);
  if (sp.ncons > kImmaMaxThreads / 32 - 2) sp.ncons = kImmaMaxThreads / 32 - 2;
  sp.dbg = env_int("SF_GEMV_DBG", 0);
  sp.ntasks = 1; sp.tasks = nullptr; sp.done = nullptr; sp.npp = 1;
  const size_t stage = (size_t)env_int("SF_GEMV_STAGE_KB", 64) * 1024;
  Need need;
  if (!plan_task(N, K, T, gs, sp.ncons, grid, stage, sp.single, need)) return false;
  sp.single.wait_before = 0;
  sp.single.wait_from = 0;
  return finish_plan(need, stage, task_chunks(sp.single, grid), pl);
}

cudaError_t launch_gemv_imma(const StepPlan& pl0, cudaStream_t st, bool pdl) {
  StepPlan pl = pl0;
#ifdef SF_GEMV_TRACE
  pl.sp.trace_id = g_trace_counter++;
#endif
  if (pl.asym) {
    if (pl.LB == 16) return launch_lb<true, 16>(pl, st, pdl);
    if (pl.LB == 8) return launch_lb<true, 8>(pl, st, pdl);
    return launch_lb<true, 4>(pl, st, pdl);
  }
  if (pl.LB == 16) return launch_lb<false, 16>(pl, st, pdl);
  if (pl.LB == 8) return launch_lb<false, 8>(pl, st, pdl);
  return launch_lb<false, 4>(pl, st, pdl);
}

}  // namespace sf

// ===========================================================================
// C ABI: a prepared list of GEMVs run as one persistent launch.
// ===========================================================================
using namespace sf;

namespace {
// workspace: [per-task completion counters, 256-aligned][task table]
size_t step_header(int ntasks) { return ((size_t)4 * (ntasks > 0 ? ntasks : 0) + 255) & ~(size_t)255; }
struct StepHandle {
  StepPlan plan;
  void* workspace;
  int device;
  bool prepass;   // some tasks read pre-converted activations
};

template <int T>
cudaError_t launch_prepass(const StepHandle* hd, cudaStream_t st) {
  q4_x_digits_kernel<T><<<hd->plan.sp.ntasks, 256, 0, st>>>(hd->plan.sp.tasks);
  return cudaGetLastError();
}
}  // namespace

#ifdef SF_LEGACY_STEP
extern "C" {

size_t sf_q4_step_workspace_bytes(int ntasks) {
  return step_header(ntasks) + (size_t)(ntasks > 0 ? ntasks : 0) * sizeof(ImmaParams);
}

// Bytes of the activation arena (digits + group scales/sums) of a task list.
static size_t x_arena_bytes(const sf_q4_task* tasks, int ntasks) {
  size_t n = 0;
  for (int i = 0; i < ntasks; ++i) {
    const sf_q4_task& a = tasks[i];
    const int G = a.group_size > 0 ? a.K / a.group_size : 0;
    n += (((size_t)3 * a.T * a.K + ((size_t)a.T * G * 8 + 15) / 16 * 16) + 127) & ~(size_t)127;
  }
  return n;
}

size_t sf_q4_step_workspace_bytes2(const sf_q4_task* tasks, int ntasks) {
  return sf_q4_step_workspace_bytes(ntasks) + x_arena_bytes(tasks, ntasks);
}

int sf_q4_step_create(const sf_q4_task* tasks, int ntasks, void* workspace, size_t workspace_bytes,
                      void** handle_out) {
  if (!tasks || !workspace || !handle_out) return fail(SF_ERR_NULL, "null pointer argument");
  if (ntasks < 1) return fail(SF_ERR_SHAPE, "ntasks must be >= 1");
  // the activation pre-pass is used when the workspace also has room for its arena
  const bool use_arena = workspace_bytes >= sf_q4_step_workspace_bytes2(tasks, ntasks);
  if (workspace_bytes < sf_q4_step_workspace_bytes(ntasks))
    return fail(SF_ERR_SHAPE, "workspace too small: need %zu bytes",
                sf_q4_step_workspace_bytes(ntasks));
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return fail(SF_ERR_ALIGN, "workspace must be 256-byte aligned");
  const int T = tasks[0].T, gs0 = tasks[0].group_size;
  const bool asym = tasks[0].zeros != nullptr;
  if (T < 1 || T > kMaxGemvT) return fail(SF_ERR_UNSUPPORTED, "step tasks need 1 <= T <= %d", kMaxGemvT);
  const DeviceInfo& di = device_info();
  StepPlan pl{};
  pl.T = T; pl.asym = asym; pl.LB = lb_for(gs0); pl.grid = di.sms;
  StepParams& sp = pl.sp;
  sp.npp = ntasks > 1 ? env_int("SF_GEMV_PINGPONG", 2) : 1;
  if (sp.npp < 1) sp.npp = 1;
  if (sp.npp > 2) sp.npp = 2;
  sp.ncons = env_int("SF_GEMV_WARPS", 14);
  if (sp.ncons > kImmaMaxThreads / 32 - 2) sp.ncons = kImmaMaxThreads / 32 - 2;
  sp.ncons -= sp.ncons % sp.npp;
  sp.ntasks = ntasks;
  sp.dbg = env_int("SF_GEMV_DBG", 0);
  std::vector<ImmaParams> h(ntasks);
  bool any_pre = false;
  // largest stage that fits next to the activations and the scale ring
  bool planned = false;
  for (int stage_kb = env_int("SF_GEMV_STAGE_KB", 64); stage_kb >= 16 && !planned; stage_kb -= 16) {
  const size_t stage = (size_t)stage_kb * 1024;
  Need need;
  long long nch = 1;
  bool any_wait = false;
  int last_wait = 0;
  size_t arena_off = sf_q4_step_workspace_bytes(ntasks);
  any_pre = false;
  for (int i = 0; i < ntasks; ++i) {
    const sf_q4_task& a = tasks[i];
    if (!a.W || !a.scales || !a.X || !a.Y) return fail(SF_ERR_NULL, "task %d: null pointer", i);
    if (a.T != T || (a.zeros != nullptr) != asym || lb_for(a.group_size) != pl.LB)
      return fail(SF_ERR_UNSUPPORTED, "task %d: all tasks need the same T, layout and group class", i);
    if (a.x_dtype < 0 || a.x_dtype > 2 || a.y_dtype < 0 || a.y_dtype > 2)
      return fail(SF_ERR_DTYPE, "task %d: unknown dtype code", i);
    if ((reinterpret_cast<uintptr_t>(a.W) | reinterpret_cast<uintptr_t>(a.scales) |
         reinterpret_cast<uintptr_t>(a.zeros) | reinterpret_cast<uintptr_t>(a.X)) & 15)
      return fail(SF_ERR_ALIGN, "task %d: W, scales, zeros and X must be 16-byte aligned", i);
    ImmaParams& q = h[i];
    q = ImmaParams{};
    if (!plan_task(a.N, a.K, T, a.group_size, sp.ncons / sp.npp, pl.grid, stage, q, need))
      return fail(SF_ERR_UNSUPPORTED, "task %d: shape N=%d K=%d gs=%d not supported by the step kernel",
                  i, a.N, a.K, a.group_size);
    q.W = a.W; q.S = a.scales; q.Z = a.zeros; q.bias = a.bias; q.X = a.X; q.Y = a.Y;
    q.xdt = a.x_dtype; q.ydt = a.y_dtype;
    q.wait_before = i > 0 ? (a.wait_before ? 1 : 0) : 0;
    q.wait_from = last_wait;
    q.xd = nullptr;
    if (use_arena && !q.wait_before) {
      q.xd = static_cast<uint8_t*>(workspace) + arena_off;
      arena_off += (((size_t)3 * T * q.K + ((size_t)T * q.G * 8 + 15) / 16 * 16) + 127) & ~(size_t)127;
      any_pre = true;
    }
    if (q.wait_before) last_wait = i;
    any_wait |= q.wait_before != 0;
    nch += task_chunks(q, pl.grid);
  }
  pl.coop = any_wait;
  planned = finish_plan(need, stage, nch, pl);
  }
  if (!planned) return fail(SF_ERR_UNSUPPORTED, "step does not fit shared memory");
  sp.done = static_cast<unsigned int*>(workspace);
  sp.tasks = reinterpret_cast<const ImmaParams*>(static_cast<uint8_t*>(workspace) + step_header(ntasks));
  cudaError_t e = cudaMemcpy(const_cast<ImmaParams*>(sp.tasks), h.data(), sizeof(ImmaParams) * ntasks,
                             cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(e, "uploading the task table");
  StepHandle* hd = new StepHandle{pl, workspace, 0, any_pre};
  cudaGetDevice(&hd->device);
  *handle_out = hd;
  return SF_OK;
}

int sf_q4_step_run(void* handle, void* stream) {
  if (!handle) return fail(SF_ERR_NULL, "null handle");
  StepHandle* hd = static_cast<StepHandle*>(handle);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(hd->workspace, 0, step_header(hd->plan.sp.ntasks), st);
  if (e != cudaSuccess) return cuda_fail(e, "clearing the barrier counter");
  if (hd->prepass) {
    switch (hd->plan.T) {
      case 1: e = launch_prepass<1>(hd, st); break;
      case 2: e = launch_prepass<2>(hd, st); break;
      case 3: e = launch_prepass<3>(hd, st); break;
      case 4: e = launch_prepass<4>(hd, st); break;
      case 5: e = launch_prepass<5>(hd, st); break;
      case 6: e = launch_prepass<6>(hd, st); break;
      case 7: e = launch_prepass<7>(hd, st); break;
      default: e = launch_prepass<8>(hd, st); break;
    }
    if (e != cudaSuccess) return cuda_fail(e, "activation pre-pass launch");
    g_launches.fetch_add(1, std::memory_order_relaxed);
  }
  e = launch_gemv_imma(hd->plan, st, false);
  if (e != cudaSuccess) return cuda_fail(e, "q4 step launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return SF_OK;
}

void sf_q4_step_destroy(void* handle) { delete static_cast<StepHandle*>(handle); }

}  // extern "C"
#endif  // SF_LEGACY_STEP
