// ref_shim.cpp -- C entry points over the reference's OWN kernel sources
// (siliconfer/kernels/neon/q4_gemv.cpp, q4_gemm.cpp), compiled unmodified
// from the reference tree by oracle/Makefile into oracle/_ref/.  TEST/BASELINE
// INFRASTRUCTURE ONLY.
//
// On x86 the reference's q4_gemv_sym_neon is its scalar C kernel and its
// q4_gemv_asym_neon silently runs the SYMMETRIC scalar kernel
// (q4_gemv.cpp:249-255), so ref_asym_is_correct() reports whether the asym
// entry may be trusted (only when built for aarch64 NEON).
#include <pthread.h>
#include <cstdint>
#include <cstddef>
#include <vector>
#include "q4_gemv.h"

namespace {
struct Job {
  const uint8_t* W; const float* S; const float* Z; const float* X; float* Y;
  int N, K, T, gs, r0, r1;
};
void* run(void* a) {
  const Job* j = static_cast<const Job*>(a);
  const int G = j->K / j->gs, rows = j->r1 - j->r0;
  if (rows <= 0) return nullptr;
  const uint8_t* W = j->W + (size_t)j->r0 * (j->K / 2);
  const float* S = j->S + (size_t)j->r0 * G;
  for (int t = 0; t < j->T; t++) {
    const float* x = j->X + (size_t)t * j->K;
    float* y = j->Y + (size_t)t * j->N + j->r0;
    if (j->Z) q4_gemv_asym_neon(W, S, j->Z + (size_t)j->r0 * G, x, y, rows, j->K, j->gs);
    else      q4_gemv_sym_neon(W, S, x, y, rows, j->K, j->gs);
  }
  return nullptr;
}
}  // namespace

extern "C" {
int ref_neon_available() {
#ifdef __ARM_NEON
  return 1;
#else
  return 0;
#endif
}
int ref_asym_is_correct() { return ref_neon_available(); }

// Rows are split across `nthreads` host threads; each slice is handed to the
// reference's own per-token GEMV exactly as q4_gemm.cpp:19-24 does.
int ref_q4_gemm(const uint8_t* W, const float* S, const float* Z, const float* X,
                float* Y, int N, int K, int T, int gs, int nthreads) {
  if (N <= 0 || K <= 0 || gs <= 0 || K % gs) return -1;
  if (nthreads < 1) nthreads = 1;
  if (nthreads > N) nthreads = N;
  std::vector<pthread_t> th(nthreads);
  std::vector<Job> jobs(nthreads);
  for (int p = 0; p < nthreads; p++) {
    jobs[p] = Job{W, S, Z, X, Y, N, K, T, gs,
                  (int)((long)N * p / nthreads), (int)((long)N * (p + 1) / nthreads)};
    if (p) pthread_create(&th[p], nullptr, run, &jobs[p]);
  }
  run(&jobs[0]);
  for (int p = 1; p < nthreads; p++) pthread_join(th[p], nullptr);
  return 0;
}

// The reference's scalar oracle, q4_gemv.cpp:262-297.
void ref_q4_gemv_scalar(const uint8_t* W, const float* S, const float* x, float* y,
                        int N, int K, int gs) {
  q4_gemv_sym_scalar(W, S, x, y, N, K, gs);
}
}
