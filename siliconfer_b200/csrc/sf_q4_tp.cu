// sf_q4_tp.cu -- tensor-parallel Q4Linear across the GPUs of one node.
//
// Sharding (siliconfer's Q4Linear has no parallel form; this follows the
// decoder's column/row split): q/k/v/gate/up are column-parallel (each rank
// owns a block of output rows, no exchange), o/down are row-parallel (each
// rank owns a block of whole groups along K and produces a partial Y that
// must be summed across ranks).
//
// The exchange is a one-shot all-reduce over NVLink peer memory:
//  * every rank owns one exchange buffer (cudaMalloc, exported as a CUDA IPC
//    handle and opened by every peer): a flag line per source rank, then two
//    fp32 partial slots used on alternate calls;
//  * call e writes this rank's partial [T, N] into slot e & 1 (the row-parallel
//    GEMV writes there directly), then the reduce kernel publishes
//    "epoch e ready" into every peer's flag line (system-scope release), waits
//    (bounded) until every peer's flag for epoch e has arrived in its own
//    buffer (acquire), and sums the partials of ranks 0..P-1 in rank order
//    with peer loads -- every rank produces bitwise the same Y;
//  * slot reuse is safe: a rank writes slot e & 1 again at epoch e + 2 only
//    after its reduce of epoch e + 1 saw every peer's e + 1 flag, which each
//    peer stores only after its own reduce of epoch e (stream order) has
//    finished reading that slot.
// A wait that expires sets the library's device error word and the kernel
// returns; the host reads SF_ERR_TIMEOUT from sf_q4_check_device_error().
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
constexpr size_t kFlagLine = 128;                       // one 128-byte line per source rank
constexpr size_t kHeader = kFlagLine * kMaxRanks;       // flags area at the start of the buffer
constexpr unsigned kErrTpWait = 1u << 16;

struct Comm {
  int rank = 0, world = 1, device = 0;
  size_t slot_bytes = 0;
  uint8_t* local = nullptr;                 // this rank's exchange buffer
  uint8_t* peer[kMaxRanks] = {};            // every rank's buffer as mapped here (peer[rank] = local)
  bool opened[kMaxRanks] = {};
  unsigned long long epoch = 0;
};

struct ReduceArgs {
  uint8_t* peer[kMaxRanks];
  int rank, world;
  unsigned long long epoch;
  size_t slot_off;                          // byte offset of this epoch's slot in every buffer
  long long count;                          // T * N
  const float* bias;                        // [N] or null
  int ncols;                                // N (bias index = i % N)
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

__global__ void tp_allreduce_kernel(const ReduceArgs a) {
  __shared__ int ok;
  // 1. publish: this rank's partial (written by the previous kernel on this
  //    stream) is complete; tell every peer.  Block 0 only.
  if (blockIdx.x == 0 && threadIdx.x < (unsigned)a.world) {
    __threadfence_system();
    auto* f = reinterpret_cast<unsigned long long*>(a.peer[threadIdx.x] + kFlagLine * a.rank);
    st_release_sys(f, a.epoch);
  }
  // 2. wait (bounded) until every peer's partial of this epoch is published
  if (threadIdx.x == 0) {
    int good = 1;
    for (int p = 0; p < a.world && good; ++p) {
      const auto* f = reinterpret_cast<const unsigned long long*>(a.peer[a.rank] + kFlagLine * p);
      if (ld_acquire_sys(f) >= a.epoch) continue;
      const long long t0 = clock64();
      while (ld_acquire_sys(f) < a.epoch) {
        if (clock64() - t0 > kWaitCycles) {
          atomicOr(&g_dev_error, kErrTpWait);
          good = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  // 3. Y = sum over ranks in rank order (+ bias), 4 elements per thread
  const long long n4 = a.count / 4;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < (a.count + 3) / 4;
       i += (long long)gridDim.x * blockDim.x) {
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (i < n4) {
      for (int p = 0; p < a.world; ++p) {
        const float4 q = reinterpret_cast<const float4*>(a.peer[p] + a.slot_off)[i];
        v[0] += q.x; v[1] += q.y; v[2] += q.z; v[3] += q.w;
      }
    } else {
      for (int p = 0; p < a.world; ++p) {
        const float* q = reinterpret_cast<const float*>(a.peer[p] + a.slot_off);
        for (int j = 0; j < 4 && 4 * i + j < a.count; ++j) v[j] += q[4 * i + j];
      }
    }
    for (int j = 0; j < 4; ++j) {
      const long long e = 4 * i + j;
      if (e >= a.count) break;
      float y = v[j] + (a.bias ? a.bias[e % a.ncols] : 0.f);
      if (a.out_dtype == SF_F32) static_cast<float*>(a.out)[e] = y;
      else if (a.out_dtype == SF_BF16) static_cast<__nv_bfloat16*>(a.out)[e] = __float2bfloat16_rn(y);
      else static_cast<__half*>(a.out)[e] = __float2half_rn(y);
    }
  }
}

int reduce(Comm* c, long long count, const float* bias, int ncols, void* out, int out_dtype, cudaStream_t st) {
  ReduceArgs a{};
  for (int p = 0; p < c->world; ++p) a.peer[p] = c->peer[p];
  a.rank = c->rank; a.world = c->world; a.epoch = c->epoch;
  a.slot_off = kHeader + (size_t)(c->epoch & 1) * c->slot_bytes;
  a.count = count; a.bias = bias; a.ncols = ncols; a.out = out; a.out_dtype = out_dtype;
  const DeviceInfo& di = device_info();
  long long blocks = ((count + 3) / 4 + 255) / 256;
  if (blocks > 4LL * di.sms) blocks = 4LL * di.sms;
  if (blocks < 1) blocks = 1;
  tp_allreduce_kernel<<<(unsigned)blocks, 256, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "tp_allreduce_kernel launch");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return SF_OK;
}

Comm* as_comm(void* h) { return static_cast<Comm*>(h); }

}  // namespace
}  // namespace sf

using namespace sf;

extern "C" {

size_t sf_tp_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int sf_tp_comm_init(int rank, int world, size_t slot_bytes, void** comm_out, void* handle_out) {
  if (!comm_out || !handle_out) return fail(SF_ERR_NULL, "null pointer argument");
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
    return fail(SF_ERR_SHAPE, "tensor-parallel world size must be 1..%d and 0 <= rank < world", kMaxRanks);
  slot_bytes = (slot_bytes + 255) & ~(size_t)255;
  Comm* c = new Comm();
  c->rank = rank; c->world = world; c->slot_bytes = slot_bytes;
  cudaGetDevice(&c->device);
  const size_t bytes = kHeader + 2 * slot_bytes;
  cudaError_t e = cudaMalloc(&c->local, bytes);
  if (e != cudaSuccess) { delete c; return cuda_fail(e, "allocating the tensor-parallel exchange buffer"); }
  e = cudaMemset(c->local, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle_out), c->local);
  if (e != cudaSuccess) {
    cudaFree(c->local);
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
  if (!comm || !out) return fail(SF_ERR_NULL, "null pointer argument");
  Comm* c = as_comm(comm);
  if (out_dtype < 0 || out_dtype > 2) return fail(SF_ERR_DTYPE, "unknown dtype code");
  if (count < 0 || (size_t)count * 4 > c->slot_bytes || ncols <= 0)
    return fail(SF_ERR_SHAPE, "all-reduce of %lld floats exceeds the %zu-byte exchange slot", count, c->slot_bytes);
  for (int p = 0; p < c->world; ++p)
    if (!c->peer[p]) return fail(SF_ERR_COMM, "rank %d is not connected (call sf_tp_comm_connect)", p);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  c->epoch += 1;
  uint8_t* slot = c->local + kHeader + (size_t)(c->epoch & 1) * c->slot_bytes;
  if (partial && partial != reinterpret_cast<const float*>(slot)) {
    cudaError_t e = cudaMemcpyAsync(slot, partial, (size_t)count * 4, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return cuda_fail(e, "staging the partial sum");
  }
  return reduce(c, count, bias, ncols, out, out_dtype, st);
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
  // the shard's partial goes straight into the next epoch's slot
  float* slot = reinterpret_cast<float*>(c->local + kHeader + (size_t)((c->epoch + 1) & 1) * c->slot_bytes);
  int rc = run_linear(W, scales, zeros, nullptr, X, x_dtype, slot, SF_F32, N, K, T, group_size, 0, st, false);
  if (rc != SF_OK) return rc;
  c->epoch += 1;
  return reduce(c, (long long)T * N, bias, N, Y, y_dtype, st);
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
  cudaSetDevice(prev);
  delete c;
}

}  // extern "C"
