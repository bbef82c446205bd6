// sf_q4_internal.h -- shared host/device helpers of the sm_100a Q4 kernels.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <utility>

namespace sf {

constexpr int kMaxDevices = 16;
constexpr int kMaxGemvT = 16;          // decode GEMV handles up to 16 tokens per launch (one pass over W)
// Bound on every device-side wait, in SM clock cycles (about 2 s at 2 GHz).
// clock64 is read only after a failed poll; it is a cheap per-SM counter
// (%globaltimer is far slower to read and must not sit in a poll loop).
constexpr long long kWaitCycles = 4000000000ll;

struct DeviceInfo {
  bool ready = false;
  int sms = 0;
  int smem_optin = 0;
};
DeviceInfo& device_info();

struct GemvParams {
  const uint8_t* W;
  const float* S;
  const float* Z;
  const float* bias;
  const void* X;
  void* Y;
  int N, K, G, gs, xdt, ydt;
};


int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);

int run_tc_gemm(const uint8_t* W, const float* S, const float* Z, const float* bias,
                const void* X, int xdt, void* Y, int ydt, int N, int K, int T, int gs,
                int flags, cudaStream_t stream);

// Sticky device error word.  Each translation unit (compiled without
// relocatable device code) owns one copy; SF_DEFINE_ERROR_READER gives the
// host a function that reads and clears the copy of that unit.
static __device__ unsigned int g_dev_error = 0;
#define SF_DEFINE_ERROR_READER(fn)                                        \
  unsigned int fn() {                                                     \
    unsigned int v = 0, z = 0;                                            \
    if (cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(v)) != cudaSuccess)  \
      return 0xffffffffu;                                                 \
    if (v) cudaMemcpyToSymbol(g_dev_error, &z, sizeof(z));                \
    return v;                                                             \
  }
// Error-word bit of a kernel that met a poisoned tensor-parallel communicator
// (sf_q4_check_device_error reports SF_ERR_COMM); other bits are expired waits.
constexpr unsigned int kErrPoisoned = 1u << 20;
// Flag value that a rank whose exchange wait expired stores into its peers'
// flag words: a peer that arrives late sees it and fails instead of reading
// a slot that no longer belongs to its call.
constexpr unsigned long long kFlagPoison = ~0ull;
unsigned int take_dev_error_gemv();
unsigned int take_dev_error_tc();
unsigned int take_dev_error_tile();
unsigned int take_dev_error_tp();

// Carves one exchange region for a pushed task from a tensor-parallel
// communicator's arena (same order on every rank, so the same offsets):
// data = 2 parities x world x `src_bytes`, then `tiles` x world u64 flags.
// Fills every rank's mapped data/flag pointers, this rank, the world size and
// the byte size of one parity half.
// Also gives the communicator's sticky poison word (this rank's copy).
int tp_region(void* comm, size_t src_bytes, size_t tiles, uint8_t** data, unsigned long long** flags, int* rank,
              int* world, size_t* par_bytes, unsigned long long** poison);

// Decode GEMV (1 <= T <= kMaxGemvT) on the warp-unit kernel; SF_ERR_UNSUPPORTED
// when the shape is not one it takes.
// epi = 1 (SwiGLU): W holds interleaved gate/up rows (16 of each per 32), N
// counts both, and Y [T, N/2] = silu(gate) * up.
// bits = 2: W holds 2-bit weights, 4 per byte ([N, K/4]).
int run_tile_linear(const uint8_t* W, const float* S, const float* Z, const float* bias,
                    const void* X, int xdt, void* Y, int ydt, int N, int K, int T, int gs,
                    cudaStream_t stream, int epi = 0, int bits = 4);

// ---------------------------------------------------------------------------
// Launch helper: optional programmatic dependent launch (PDL).
// ---------------------------------------------------------------------------
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*fn)(KArgs...), int grid, int threads, size_t smem,
                          cudaStream_t stream, bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((unsigned)threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, fn, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// PTX wrappers (mbarrier, bulk async copy, grid dependency control)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// try_wait with a suspend-time hint: a warp whose phase is not complete
// sleeps (up to ~0.1 ms, woken when the phase completes) instead of spinning
// and stealing issue slots from the warps that are computing.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(100000u)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after kWaitCycles, records the failure in the sticky
// device error word and returns false so that the caller can wind down.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int code = 1u) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) {
      atomicOr(&g_dev_error, code);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void named_barrier_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace sf
