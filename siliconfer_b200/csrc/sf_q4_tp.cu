// sf_q4_tp.cu -- tensor-parallel Q4Linear across the GPUs of one node.
//
// Sharding (siliconfer's Q4Linear has no parallel form; this follows the
// decoder's column/row split): q/k/v/gate/up are column-parallel (each rank
// owns a block of output rows, no exchange), o/down are row-parallel (each
// rank owns a block of whole groups along K and produces a partial Y that
// must be summed across ranks).
//
// The exchange is a one-shot all-reduce over NVLink peer memory, with all of
// its state on the device (so a captured CUDA graph can replay it):
//  * every rank owns one exchange buffer (cudaMalloc, exported as a CUDA IPC
//    handle and opened by every peer): a header (call epoch, finished-block
//    count, poison word), a flag word per (reduce block, source rank), then two fp32 slots
//    used on alternate calls; and a private partial buffer that the
//    row-parallel GEMV writes;
//  * call e (e = device epoch + 1, read by every block at start) splits the
//    result into chunks; block b copies its chunks of this rank's partial into
//    slot e & 1, then stores flag[b][rank] = e into every peer's buffer
//    (system-scope release), waits (bounded) until flag[b][p] >= e for every
//    peer p in its own buffer (acquire), and sums the chunks of ranks
//    0..P-1 in rank order with peer loads -- every rank produces bitwise the
//    same Y; the last block to finish advances the epoch;
//  * slot reuse is safe: a rank writes slot e & 1 again at call e + 2 only
//    after its call e + 1 saw a flag of call e + 1 from every peer, which a
//    peer stores only after its own call e (stream order) has finished
//    reading that slot.
// A wait that expires sets the library's device error word and the kernel
// returns; the host reads SF_ERR_TIMEOUT from sf_q4_check_device_error().
// After an expired wait the ranks' epochs are out of step for good, so the
// communicator is poisoned: the rank that gave up sets its sticky poison word
// and overwrites its flag in every peer with kFlagPoison.  A peer that
// arrives late sees that value instead of a flag it could take for its own
// call, and every later call on either side finds a poison word or a poison
// flag and returns at once with kErrPoisoned (SF_ERR_COMM on the host) until
// the communicator is created again.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include <atomic>
#include <cstdint>
#include <cstring>
#include <vector>

#include "sf_q4.h"
#include "sf_q4_internal.h"

namespace sf {
SF_DEFINE_ERROR_READER(take_dev_error_tp)
extern std::atomic<long long> g_launches;
int run_linear(const uint8_t* W, const float* S, const float* Z, const float* bias, const void* X, int xdt,
               void* Y, int ydt, int N, int K, int T, int gs, int flags, cudaStream_t stream,
               bool force_generic);

namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 1024;                        // reduce blocks per call (chunks beyond: grid stride)
constexpr int kChunk = 1024;                            // floats per chunk (4 per thread, 256 threads)
constexpr size_t kHeader = 256;                         // epoch, finished-block count
constexpr size_t kFlags = (size_t)kMaxBlocks * kMaxRanks * 8;
constexpr size_t kSlot0 = kHeader + kFlags;
constexpr unsigned kErrTpWait = 1u << 16;

struct Comm {
  int rank = 0, world = 1, device = 0;
  size_t slot_bytes = 0;
  size_t arena_bytes = 0, arena_used = 0;   // exchange regions of fused step tasks, after the slots
  uint8_t* local = nullptr;                 // this rank's exchange buffer
  float* partial = nullptr;                 // the row-parallel GEMV's output (private)
  uint8_t* peer[kMaxRanks] = {};            // every rank's buffer as mapped here (peer[rank] = local)
  bool opened[kMaxRanks] = {};
};

struct ReduceArgs {
  uint8_t* peer[kMaxRanks];
  int rank, world;
  size_t slot_bytes;
  const float* partial;                     // this rank's partial [count]
  long long count;                          // T * N
  const float* bias;                        // [ncols] or null
  int ncols;
  void* out;
  int out_dtype;
};

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(256) tp_allreduce_kernel(const ReduceArgs a) {
  __shared__ unsigned long long ep_s;
  __shared__ int ok, poisoned;
  uint8_t* mine = a.peer[a.rank];
  auto* hdr = reinterpret_cast<unsigned long long*>(mine);   // [0] epoch, [1] finished blocks, [2] poison
  if (threadIdx.x == 0) {
    ep_s = *reinterpret_cast<volatile unsigned long long*>(hdr) + 1;
    poisoned = *reinterpret_cast<volatile unsigned long long*>(hdr + 2) != 0;
  }
  __syncthreads();
  if (poisoned) {   // an earlier call gave up: tell the peers and touch nothing else
    if (threadIdx.x < (unsigned)a.world)
      st_release_sys(reinterpret_cast<unsigned long long*>(a.peer[threadIdx.x] + kHeader) +
                         (size_t)blockIdx.x * kMaxRanks + a.rank, kFlagPoison);
    if (threadIdx.x == 0) atomicOr(&g_dev_error, kErrPoisoned);
    return;
  }
  const unsigned long long ep = ep_s;
  const size_t slot = kSlot0 + (size_t)(ep & 1) * a.slot_bytes;
  const long long nchunks = (a.count + kChunk - 1) / kChunk;
  // 1. this rank's chunks of the partial -> own slot
  for (long long c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const long long i = c * kChunk + 4 * threadIdx.x;
    float* dst = reinterpret_cast<float*>(mine + slot);
    if (i + 4 <= a.count) {
      *reinterpret_cast<float4*>(dst + i) = *reinterpret_cast<const float4*>(a.partial + i);
    } else {
      for (long long j = i; j < a.count && j < i + 4; ++j) dst[j] = a.partial[j];
    }
  }
  __syncthreads();
  // 2. publish block b's chunks to every peer, then wait for theirs (bounded)
  if (threadIdx.x < (unsigned)a.world) {
    __threadfence_system();
    auto* f = reinterpret_cast<unsigned long long*>(a.peer[threadIdx.x] + kHeader) +
              (size_t)blockIdx.x * kMaxRanks + a.rank;
    st_release_sys(f, ep);
  }
  if (threadIdx.x == 0) {
    int good = 1;
    const auto* fl = reinterpret_cast<const unsigned long long*>(mine + kHeader) + (size_t)blockIdx.x * kMaxRanks;
    for (int p = 0; p < a.world && good; ++p) {
      unsigned long long v = ld_acquire_sys(fl + p);
      const long long t0 = clock64();
      while (v < ep) {
        if (clock64() - t0 > kWaitCycles) {
          atomicOr(&g_dev_error, kErrTpWait);
          good = 0;
          break;
        }
        __nanosleep(32);
        v = ld_acquire_sys(fl + p);
      }
      if (v == kFlagPoison) {   // that peer gave up on an earlier call
        atomicOr(&g_dev_error, kErrPoisoned);
        good = 0;
      }
    }
    if (!good) *reinterpret_cast<volatile unsigned long long*>(hdr + 2) = 1ull;
    ok = good;
  }
  __syncthreads();
  if (!ok) {
    // poison this block's flag in every peer (it may already hold this call's epoch)
    if (threadIdx.x < (unsigned)a.world) {
      __threadfence_system();
      st_release_sys(reinterpret_cast<unsigned long long*>(a.peer[threadIdx.x] + kHeader) +
                         (size_t)blockIdx.x * kMaxRanks + a.rank, kFlagPoison);
    }
    return;
  }
  // 3. Y = sum over ranks in rank order (+ bias)
  {
    for (long long c = blockIdx.x; c < nchunks; c += gridDim.x) {
      const long long i = c * kChunk + 4 * threadIdx.x;
      if (i >= a.count) continue;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (i + 4 <= a.count) {
        for (int p = 0; p < a.world; ++p) {
          const float4 q = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.peer[p] + slot) + i);
          v[0] += q.x; v[1] += q.y; v[2] += q.z; v[3] += q.w;
        }
      } else {
        for (int p = 0; p < a.world; ++p) {
          const float* q = reinterpret_cast<const float*>(a.peer[p] + slot);
          for (int j = 0; j < 4 && i + j < a.count; ++j) v[j] += q[i + j];
        }
      }
      for (int j = 0; j < 4 && i + j < a.count; ++j) {
        const long long e = i + j;
        const float y = v[j] + (a.bias ? a.bias[e % a.ncols] : 0.f);
        if (a.out_dtype == SF_F32) static_cast<float*>(a.out)[e] = y;
        else if (a.out_dtype == SF_BF16) static_cast<__nv_bfloat16*>(a.out)[e] = __float2bfloat16_rn(y);
        else static_cast<__half*>(a.out)[e] = __float2half_rn(y);
      }
    }
  }
  // 4. the last block to finish advances the epoch for the next call
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(reinterpret_cast<unsigned long long*>(hdr + 1), 1ull) == (unsigned long long)gridDim.x - 1) {
      hdr[1] = 0;
      __threadfence();
      *reinterpret_cast<volatile unsigned long long*>(hdr) = ep;
    }
  }
}

int reduce(Comm* c, const float* partial, long long count, const float* bias, int ncols, void* out, int out_dtype,
           cudaStream_t st) {
  if (count == 0) return SF_OK;
  ReduceArgs a{};
  for (int p = 0; p < c->world; ++p) a.peer[p] = c->peer[p];
  a.rank = c->rank; a.world = c->world; a.slot_bytes = c->slot_bytes;
  a.partial = partial; a.count = count; a.bias = bias; a.ncols = ncols; a.out = out; a.out_dtype = out_dtype;
  long long blocks = (count + kChunk - 1) / kChunk;
  if (blocks > kMaxBlocks) blocks = kMaxBlocks;
  tp_allreduce_kernel<<<(unsigned)blocks, 256, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "tp_allreduce_kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return SF_OK;
}

Comm* as_comm(void* h) { return static_cast<Comm*>(h); }

}  // namespace

int tp_region(void* comm, size_t src_bytes, size_t tiles, uint8_t** data, unsigned long long** flags, int* rank,
              int* world, size_t* par_bytes, unsigned long long** poison) {
  Comm* c = as_comm(comm);
  for (int p = 0; p < c->world; ++p)
    if (!c->peer[p]) return fail(SF_ERR_COMM, "rank %d is not connected (call sf_tp_comm_connect)", p);
  const size_t par = ((size_t)c->world * src_bytes + 255) & ~(size_t)255;
  const size_t fl = (tiles * c->world * 8 + 255) & ~(size_t)255;
  if (c->arena_used + 2 * par + fl > c->arena_bytes)
    return fail(SF_ERR_SHAPE, "tensor-parallel arena too small: %zu of %zu bytes used, %zu more needed",
                c->arena_used, c->arena_bytes, 2 * par + fl);
  const size_t off = kSlot0 + 2 * c->slot_bytes + c->arena_used;
  c->arena_used += 2 * par + fl;
  for (int p = 0; p < 8; ++p) {
    data[p] = p < c->world ? c->peer[p] + off : nullptr;
    flags[p] = p < c->world ? reinterpret_cast<unsigned long long*>(c->peer[p] + off + 2 * par) : nullptr;
  }
  *rank = c->rank;
  *world = c->world;
  *par_bytes = par;
  *poison = reinterpret_cast<unsigned long long*>(c->local) + 2;
  return SF_OK;
}
}  // namespace sf

using namespace sf;

extern "C" {

size_t sf_tp_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int sf_tp_comm_init(int rank, int world, size_t slot_bytes, size_t arena_bytes, void** comm_out,
                    void* handle_out) {
  if (!comm_out || !handle_out) return fail(SF_ERR_NULL, "null pointer argument");
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
    return fail(SF_ERR_SHAPE, "tensor-parallel world size must be 1..%d and 0 <= rank < world", kMaxRanks);
  slot_bytes = (slot_bytes + 255) & ~(size_t)255;
  arena_bytes = (arena_bytes + 255) & ~(size_t)255;
  Comm* c = new Comm();
  c->rank = rank; c->world = world; c->slot_bytes = slot_bytes; c->arena_bytes = arena_bytes;
  cudaGetDevice(&c->device);
  const size_t bytes = kSlot0 + 2 * slot_bytes + arena_bytes;
  cudaError_t e = cudaMalloc(&c->local, bytes);
  if (e != cudaSuccess) { delete c; return cuda_fail(e, "allocating the tensor-parallel exchange buffer"); }
  e = cudaMalloc(&c->partial, slot_bytes);
  if (e != cudaSuccess) {
    cudaFree(c->local);
    delete c;
    return cuda_fail(e, "allocating the tensor-parallel partial buffer");
  }
  e = cudaMemset(c->local, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle_out), c->local);
  if (e != cudaSuccess) {
    cudaFree(c->local);
    cudaFree(c->partial);
    delete c;
    return cuda_fail(e, "exporting the tensor-parallel exchange buffer");
  }
  c->peer[rank] = c->local;
  *comm_out = c;
  return SF_OK;
}

int sf_tp_comm_connect(void* comm, const void* handles) {
  if (!comm || !handles) return fail(SF_ERR_NULL, "null pointer argument");
  Comm* c = as_comm(comm);
  const auto* h = static_cast<const cudaIpcMemHandle_t*>(handles);
  for (int p = 0; p < c->world; ++p) {
    if (p == c->rank || c->opened[p]) continue;
    void* ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&ptr, h[p], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return fail(SF_ERR_COMM, "opening the exchange buffer of rank %d: %s", p, cudaGetErrorString(e));
    c->peer[p] = static_cast<uint8_t*>(ptr);
    c->opened[p] = true;
  }
  return SF_OK;
}

int sf_tp_allreduce(void* comm, const float* partial, void* out, int out_dtype, const float* bias, long long count,
                    int ncols, void* stream) {
  if (!comm || !out || !partial) return fail(SF_ERR_NULL, "null pointer argument");
  Comm* c = as_comm(comm);
  if (out_dtype < 0 || out_dtype > 2) return fail(SF_ERR_DTYPE, "unknown dtype code");
  if (count < 0 || (size_t)count * 4 > c->slot_bytes || ncols <= 0)
    return fail(SF_ERR_SHAPE, "all-reduce of %lld floats exceeds the %zu-byte exchange slot", count, c->slot_bytes);
  for (int p = 0; p < c->world; ++p)
    if (!c->peer[p]) return fail(SF_ERR_COMM, "rank %d is not connected (call sf_tp_comm_connect)", p);
  return reduce(c, partial, count, bias, ncols, out, out_dtype, static_cast<cudaStream_t>(stream));
}

int sf_q4_linear_allreduce(void* comm, const uint8_t* W, const float* scales, const float* zeros, const float* bias,
                           const void* X, int x_dtype, void* Y, int y_dtype, int N, int K, int T, int group_size,
                           void* stream) {
  if (!comm) return fail(SF_ERR_NULL, "null pointer argument");
  Comm* c = as_comm(comm);
  if ((size_t)T * N * 4 > c->slot_bytes)
    return fail(SF_ERR_SHAPE, "row-parallel output [%d, %d] exceeds the %zu-byte exchange slot", T, N, c->slot_bytes);
  for (int p = 0; p < c->world; ++p)
    if (!c->peer[p]) return fail(SF_ERR_COMM, "rank %d is not connected (call sf_tp_comm_connect)", p);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = run_linear(W, scales, zeros, nullptr, X, x_dtype, c->partial, SF_F32, N, K, T, group_size, 0, st, false);
  if (rc != SF_OK) return rc;
  return reduce(c, c->partial, (long long)T * N, bias, N, Y, y_dtype, st);
}

void sf_tp_comm_destroy(void* comm) {
  if (!comm) return;
  Comm* c = as_comm(comm);
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  for (int p = 0; p < c->world; ++p)
    if (c->opened[p]) cudaIpcCloseMemHandle(c->peer[p]);
  cudaFree(c->local);
  cudaFree(c->partial);
  cudaSetDevice(prev);
  delete c;
}

}  // extern "C"
