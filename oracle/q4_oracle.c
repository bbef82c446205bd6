/*
 * q4_oracle.c -- CPU restatement of siliconfer's int4 GEMV/GEMM.
 * TEST INFRASTRUCTURE ONLY: the product never links this file.  It is the
 * checker used by tests/ and the "port" CPU baseline of bench.py.
 *
 * Algorithm (one fp32 accumulation per (row, group), then scaled):
 *   sym : y[t,i] += s[i,g] * sum_k sext(nib[i,k]) * x[t,k]
 *         (siliconfer/kernels/neon/__init__.py:88-106, q4_gemv.cpp:262-297)
 *   asym: y[t,i] += s[i,g] * (sum_k nib[i,k] * x[t,k] - z[i,g] * sum_k x[t,k])
 *         (siliconfer/kernels/neon/__init__.py:109-124, q4_gemv.cpp:145-238)
 * Packed layout: byte j of row i = w(i,2j) | w(i,2j+1) << 4
 *   (siliconfer/kernels/neon/q4_gemv.h:5-12).
 * Rows are split over pthreads; each row's arithmetic is sequential.
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
  const uint8_t *W; const float *S; const float *Z; const float *X; float *Y;
  int N, K, T, gs, r0, r1;
} job_t;

static void *run_rows(void *arg) {
  const job_t *j = (const job_t *)arg;
  const int G = j->K / j->gs, half = j->gs / 2;
  for (int t = 0; t < j->T; t++) {
    const float *x = j->X + (size_t)t * j->K;
    for (int i = j->r0; i < j->r1; i++) {
      const uint8_t *w = j->W + (size_t)i * (j->K / 2);
      float acc = 0.0f;
      for (int g = 0; g < G; g++) {
        const uint8_t *wg = w + (size_t)g * half;
        const float *xg = x + (size_t)g * j->gs;
        float dot = 0.0f, xs = 0.0f;
        for (int c = 0; c < half; c++) {
          int lo = wg[c] & 15, hi = wg[c] >> 4;
          if (!j->Z) { lo = lo < 8 ? lo : lo - 16; hi = hi < 8 ? hi : hi - 16; }
          dot += (float)lo * xg[2 * c] + (float)hi * xg[2 * c + 1];
          xs += xg[2 * c] + xg[2 * c + 1];
        }
        if (j->Z) dot -= j->Z[(size_t)i * G + g] * xs;
        acc += dot * j->S[(size_t)i * G + g];
      }
      j->Y[(size_t)t * j->N + i] = acc;
    }
  }
  return NULL;
}

/* Y[T,N] = X[T,K] @ dequant(W)^T.  Z == NULL selects the symmetric layout. */
int oracle_q4_gemm(const uint8_t *W, const float *S, const float *Z,
                   const float *X, float *Y, int N, int K, int T, int gs,
                   int nthreads) {
  if (N < 0 || K <= 0 || T < 0 || gs <= 0 || gs % 2 || K % gs) return -1;
  if (nthreads < 1) nthreads = 1;
  if (nthreads > N) nthreads = N > 0 ? N : 1;
  pthread_t *th = (pthread_t *)calloc((size_t)nthreads, sizeof(pthread_t));
  job_t *jobs = (job_t *)calloc((size_t)nthreads, sizeof(job_t));
  for (int p = 0; p < nthreads; p++) {
    job_t j = {W, S, Z, X, Y, N, K, T, gs,
               (int)((long)N * p / nthreads), (int)((long)N * (p + 1) / nthreads)};
    jobs[p] = j;
    if (p) pthread_create(&th[p], NULL, run_rows, &jobs[p]);
  }
  run_rows(&jobs[0]);
  for (int p = 1; p < nthreads; p++) pthread_join(th[p], NULL);
  free(th); free(jobs);
  return 0;
}

/* fp32 dequant, bit-exact target: q*s or (q - z)*s
   (siliconfer/quant/primitives.py:54-75, 117-140). */
void oracle_q4_dequant(const uint8_t *W, const float *S, const float *Z,
                       float *out, int N, int K, int gs) {
  const int G = K / gs;
  for (int i = 0; i < N; i++)
    for (int k = 0; k < K; k++) {
      uint8_t b = W[(size_t)i * (K / 2) + k / 2];
      int q = (k & 1) ? (b >> 4) : (b & 15);
      float s = S[(size_t)i * G + k / gs];
      if (Z) out[(size_t)i * K + k] = ((float)q - Z[(size_t)i * G + k / gs]) * s;
      else   out[(size_t)i * K + k] = (float)(q < 8 ? q : q - 16) * s;
    }
}
