/* ref_matmul.c -- CPU restatement of the reference (cmpext3) matmul kernels.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the
 * sm_100a kernels in cmp_ext_b200/csrc; it is never linked into, loaded by or
 * called from the product path.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg use it.
 *
 * It restates, bit for bit, the arithmetic of the reference's three SIMT
 * kernels on row-major A[M,K], B[K,N] -> C[M,N]:
 *
 *  fp16  gemm_fp16_ampere_optimized_v3 (src/cuda/fp16_matmul.cu:63-283):
 *        accumulator starts at +0 (L91-98); for k = 0..K-1 in ascending order
 *        (tiles L170, inner L190) acc = fma.rn.f16(a, b, acc) -- one rounding
 *        per step (__hfma2, L225-226); the fp16 result is stored (L269-282).
 *  bf16  gemm_bf16_kernel (src/cuda/bf16_matmul.cu:51-226): same with
 *        fma.rn.bf16 (__hfma2 on __nv_bfloat162, L196).
 *  fp32  gemm_fp32_ga100_kernel (src/cuda/fp32_matmul.cu:31-184): acc starts
 *        at 0 (L49); for ascending k, prod = __fmul_rn(a, b),
 *        acc = __fadd_rn(acc, prod) (L20-26, L155-162); compiled with
 *        --use_fast_math (setup.py:79), so inputs and results of both
 *        operations are flushed to zero when subnormal (FTZ).
 *
 * Zero-padded tail iterations of the reference (k >= K inside the last tile)
 * add +0 products and leave the accumulator unchanged, so they are omitted.
 *
 * Exactness argument for the half-precision emulation: a*b of two fp16 (or
 * two bf16) values has at most 22 (16) significant bits and is exact in
 * double.  a*b + acc is then computed in double; when that sum is inexact the
 * discarded part lies below 2^-53 of the sum, while the distance from the exact
 * sum to any fp16/bf16 rounding midpoint is either zero or at least one unit
 * of the product's last place (>= 2^-22 of the sum's half-ulp).  So rounding
 * the double sum once to the target format (round-to-nearest-even, with
 * gradual underflow) gives the same value as the hardware's single-rounding
 * FMA.
 *
 * Build: see oracle/Makefile (gcc -O2 -ffp-contract=off, no fast-math).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_F16 0
#define ORACLE_BF16 1
#define ORACLE_F32 2

static double g_f16_tab[65536];
static double g_bf16_tab[65536];
static pthread_once_t g_once = PTHREAD_ONCE_INIT;

static double f16_bits_to_double(uint16_t h) {
  const int s = h >> 15, e = (h >> 10) & 0x1f, m = h & 0x3ff;
  double v;
  if (e == 0) v = ldexp((double)m, -24);
  else if (e == 31) v = m ? NAN : INFINITY;
  else v = ldexp((double)(m | 0x400), e - 25);
  return s ? -v : v;
}

static double bf16_bits_to_double(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return (double)f;
}

static void init_tables(void) {
  for (int i = 0; i < 65536; ++i) {
    g_f16_tab[i] = f16_bits_to_double((uint16_t)i);
    g_bf16_tab[i] = bf16_bits_to_double((uint16_t)i);
  }
}

/* Round x to a binary format with `mbits` explicit mantissa bits, minimum
 * normal exponent `emin` and maximum exponent `emax`, round-to-nearest-even,
 * gradual underflow.  Returns the rounded value as a double (exact). */
static inline double round_fmt(double x, int mbits, int emin, int emax) {
  if (x == 0.0 || isnan(x) || isinf(x)) return x;
  int e;
  frexp(x, &e); /* |x| = f * 2^e, f in [0.5, 1) -> leading bit exponent e-1 */
  int E = e - 1;
  if (E < emin) E = emin;
  const double q = ldexp(1.0, E - mbits);
  const double r = rint(x / q) * q; /* x/q exact; rint = ties-to-even (default mode) */
  if (fabs(r) >= ldexp(1.0, emax + 1)) return copysign(INFINITY, x);
  return r;
}

static inline double rnd_f16(double x) { return round_fmt(x, 10, -14, 15); }
static inline double rnd_bf16(double x) { return round_fmt(x, 7, -126, 127); }

static uint16_t double_to_f16_bits(double r) { /* r exactly representable */
  uint16_t s = signbit(r) ? 0x8000 : 0;
  double a = fabs(r);
  if (isnan(r)) return 0x7e00;
  if (isinf(a)) return s | 0x7c00;
  if (a == 0.0) return s;
  int e;
  frexp(a, &e);
  const int E = e - 1;
  if (E < -14) return s | (uint16_t)(a * 16777216.0); /* a / 2^-24 */
  const uint16_t m = (uint16_t)(ldexp(a, 10 - E) - 1024.0);
  return s | (uint16_t)((E + 15) << 10) | m;
}

static uint16_t double_to_bf16_bits(double r) { /* r exactly representable as bf16 */
  float f = (float)r;
  uint32_t u;
  memcpy(&u, &f, 4);
  if (isnan(f)) return 0x7fc0;
  return (uint16_t)(u >> 16);
}

static inline float ftz(float x) { return fabsf(x) < 1.17549435e-38f ? copysignf(0.0f, x) : x; }

/* ---------------------------------------------------------------- kernels */
typedef struct {
  int dtype;
  const void* A;
  const void* B;
  void* C;
  int64_t M, N, K, r0, r1;
} job_t;

static void rows_half(const job_t* j, const double* tab, int is_bf16) {
  const uint16_t* A = (const uint16_t*)j->A;
  const uint16_t* B = (const uint16_t*)j->B;
  uint16_t* C = (uint16_t*)j->C;
  const int64_t N = j->N, K = j->K;
  double* acc = (double*)malloc(sizeof(double) * (size_t)(N > 0 ? N : 1));
  double* brow = (double*)malloc(sizeof(double) * (size_t)(N > 0 ? N : 1));
  for (int64_t i = j->r0; i < j->r1; ++i) {
    for (int64_t n = 0; n < N; ++n) acc[n] = 0.0;
    for (int64_t k = 0; k < K; ++k) {
      const double a = tab[A[i * K + k]];
      const uint16_t* bk = B + k * N;
      for (int64_t n = 0; n < N; ++n) brow[n] = tab[bk[n]];
      if (is_bf16) {
        for (int64_t n = 0; n < N; ++n) acc[n] = rnd_bf16(a * brow[n] + acc[n]);
      } else {
        for (int64_t n = 0; n < N; ++n) acc[n] = rnd_f16(a * brow[n] + acc[n]);
      }
    }
    for (int64_t n = 0; n < N; ++n)
      C[i * N + n] = is_bf16 ? double_to_bf16_bits(acc[n]) : double_to_f16_bits(acc[n]);
  }
  free(acc);
  free(brow);
}

static void rows_f32(const job_t* j) {
  const float* A = (const float*)j->A;
  const float* B = (const float*)j->B;
  float* C = (float*)j->C;
  const int64_t N = j->N, K = j->K;
  float* acc = (float*)malloc(sizeof(float) * (size_t)(N > 0 ? N : 1));
  for (int64_t i = j->r0; i < j->r1; ++i) {
    for (int64_t n = 0; n < N; ++n) acc[n] = 0.0f;
    for (int64_t k = 0; k < K; ++k) {
      const float a = ftz(A[i * K + k]);
      const float* bk = B + k * N;
      for (int64_t n = 0; n < N; ++n) {
        const float prod = ftz(a * ftz(bk[n]));
        acc[n] = ftz(acc[n] + prod);
      }
    }
    for (int64_t n = 0; n < N; ++n) C[i * N + n] = acc[n];
  }
  free(acc);
}

static void* run_job(void* p) {
  const job_t* j = (const job_t*)p;
  if (j->dtype == ORACLE_F32) rows_f32(j);
  else rows_half(j, j->dtype == ORACLE_BF16 ? g_bf16_tab : g_f16_tab, j->dtype == ORACLE_BF16);
  return NULL;
}

/* Computes rows [row0, row1) of C = A*B with the reference kernel's
 * arithmetic.  A, B, C are full packed row-major host arrays (fp16/bf16 as
 * raw uint16 bits, fp32 as float).  Returns 0, or -1 on bad arguments. */
int oracle_matmul(int dtype, const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                  int64_t row0, int64_t row1, int nthreads) {
  if (dtype < 0 || dtype > 2 || M < 0 || N < 0 || K < 0) return -1;
  if (row0 < 0 || row1 > M || row0 > row1) return -1;
  pthread_once(&g_once, init_tables);
  const int64_t rows = row1 - row0;
  if (rows == 0 || N == 0) return 0;
  if (nthreads < 1) nthreads = 1;
  if (nthreads > rows) nthreads = (int)rows;
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nthreads);
  job_t* jobs = (job_t*)malloc(sizeof(job_t) * (size_t)nthreads);
  for (int t = 0; t < nthreads; ++t) {
    jobs[t].dtype = dtype;
    jobs[t].A = A;
    jobs[t].B = B;
    jobs[t].C = C;
    jobs[t].M = M;
    jobs[t].N = N;
    jobs[t].K = K;
    jobs[t].r0 = row0 + rows * t / nthreads;
    jobs[t].r1 = row0 + rows * (t + 1) / nthreads;
  }
  for (int t = 1; t < nthreads; ++t) pthread_create(&th[t], NULL, run_job, &jobs[t]);
  run_job(&jobs[0]);
  for (int t = 1; t < nthreads; ++t) pthread_join(th[t], NULL);
  free(th);
  free(jobs);
  return 0;
}

/* Single-rounding conversions exposed for the oracle's own unit tests. */
uint16_t oracle_round_f16(double x) { pthread_once(&g_once, init_tables); return double_to_f16_bits(rnd_f16(x)); }
uint16_t oracle_round_bf16(double x) { pthread_once(&g_once, init_tables); return double_to_bf16_bits(rnd_bf16(x)); }
