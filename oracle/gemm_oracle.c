/*
 * CPU oracle for the bf16 GEMM path.  TEST INFRASTRUCTURE ONLY: the parity
 * tests, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it as
 * the checker / CPU baseline.  The product path never calls it.
 *
 * It restates the arithmetic of the reference kernel
 *   b200_kernels/matmul_1.cuh:329-381 (matmulKernel1):
 *     C[i][j] = bf16_rn( sum_k float(A[i][k]) * float(B[j][k]) )
 *   - A is M x K row-major, B is N x K row-major (both K-major): the TMA maps
 *     at matmul_1.cuh:391-392 walk K fastest for both operands;
 *   - products of bf16 values accumulate in fp32 in TMEM (tcgen05 kind::f16
 *     with D = f32, include/b200_utils.cuh:252-270);
 *   - the epilogue rounds each fp32 sum to bf16 with round-to-nearest-even
 *     (__float22bfloat162_rn, matmul_1.cuh:293-295);
 *   - inputs are produced by float -> bf16 conversion, also RNE
 *     (include/utils.cuh:24-29).
 * The tensor core's fp32 summation order is unspecified, so the oracle sums
 * in fp64 (oracle_gemm_bf16_nt_f64) and tests apply |err| <= 2^-7 (|ref| + 1);
 * when every partial sum is exactly representable (small integers) the
 * result is exact and tests demand bit equality.
 *
 * oracle_gemm_bf16_nt_f32 is the multithreaded fp32 CPU GEMM used as the
 * reported CPU baseline (bf16 inputs widened to fp32, fp32 accumulate).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------ bf16 <-> f32 */
static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f32_to_bf16_rne(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu) != 0) {
    return (uint16_t)((u >> 16) | 0x0040u); /* quiet NaN, keep sign/payload top */
  }
  const uint32_t lsb = (u >> 16) & 1u;
  u += 0x7FFFu + lsb; /* round half to even */
  return (uint16_t)(u >> 16);
}

void oracle_f32_to_bf16(const float* in, uint16_t* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = f32_to_bf16_rne(in[i]);
}

void oracle_bf16_to_f32(const uint16_t* in, float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = bf16_to_f32(in[i]);
}

/* Round doubles to fp32 (RNE, the C default) and then to bf16 (RNE). */
void oracle_f64_to_bf16(const double* in, uint16_t* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = f32_to_bf16_rne((float)in[i]);
}

static int default_threads(int nthreads) {
  if (nthreads > 0) return nthreads;
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

/* --------------------------------------------------- fp64 reference GEMM */
typedef struct {
  int M, N, K, lda, ldb, ldc;
  const uint16_t* A;
  const uint16_t* B;
  double* C;
  int row_begin, row_end;
} f64_job;

static void* f64_worker(void* arg) {
  f64_job* j = (f64_job*)arg;
  float* arow = (float*)malloc(sizeof(float) * (size_t)(j->K > 0 ? j->K : 1));
  for (int i = j->row_begin; i < j->row_end; ++i) {
    for (int k = 0; k < j->K; ++k) arow[k] = bf16_to_f32(j->A[(size_t)i * j->lda + k]);
    for (int n = 0; n < j->N; ++n) {
      const uint16_t* b = j->B + (size_t)n * j->ldb;
      double s = 0.0;
      for (int k = 0; k < j->K; ++k) s += (double)arow[k] * (double)bf16_to_f32(b[k]);
      j->C[(size_t)i * j->ldc + n] = s;
    }
  }
  free(arow);
  return NULL;
}

/* C (fp64, M x N, ldc) = A (bf16 M x K, lda) . B (bf16 N x K, ldb)^T, fp64 sums.
 * Rows [row_begin, row_end) only (pass 0, M for all). */
int oracle_gemm_bf16_nt_f64(int M, int N, int K, const uint16_t* A, int lda, const uint16_t* B,
                            int ldb, double* C, int ldc, int row_begin, int row_end,
                            int nthreads) {
  if (M < 0 || N < 0 || K < 0 || row_begin < 0 || row_end > M || row_begin > row_end) return 1;
  int T = default_threads(nthreads);
  const int rows = row_end - row_begin;
  if (T > rows) T = rows > 0 ? rows : 1;
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)T);
  f64_job* jobs = (f64_job*)malloc(sizeof(f64_job) * (size_t)T);
  for (int t = 0; t < T; ++t) {
    f64_job j = {M, N, K, lda, ldb, ldc, A, B, C,
                 row_begin + (int)((long long)rows * t / T),
                 row_begin + (int)((long long)rows * (t + 1) / T)};
    jobs[t] = j;
    pthread_create(&th[t], NULL, f64_worker, &jobs[t]);
  }
  for (int t = 0; t < T; ++t) pthread_join(th[t], NULL);
  free(th);
  free(jobs);
  return 0;
}

/* Selected elements only: out[s] = sum_k A[rows[s]][k] * B[cols[s]][k] (fp64). */
void oracle_gemm_bf16_nt_f64_sampled(int K, const uint16_t* A, int lda, const uint16_t* B, int ldb,
                                     const int* rows, const int* cols, size_t count, double* out) {
  for (size_t s = 0; s < count; ++s) {
    const uint16_t* a = A + (size_t)rows[s] * lda;
    const uint16_t* b = B + (size_t)cols[s] * ldb;
    double acc = 0.0;
    for (int k = 0; k < K; ++k) acc += (double)bf16_to_f32(a[k]) * (double)bf16_to_f32(b[k]);
    out[s] = acc;
  }
}

/* --------------------------------------------- fp32 CPU baseline GEMM */
/* Inputs are widened to fp32 once; each thread owns a band of C rows and
 * computes 2 x 4 blocks of dot products with 8 independent fp32 lanes per
 * dot product (vectorisable), then rounds to bf16 RNE. */
typedef struct {
  int N, K, ldc;
  const float* A; /* M x K */
  const float* B; /* N x K */
  uint16_t* C;
  int row_begin, row_end;
} f32_job;

#define LANES 8

static inline float hsum8(const float* v) {
  return ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
}

static void* f32_worker(void* arg) {
  f32_job* j = (f32_job*)arg;
  const int K = j->K, K8 = K - (K % LANES);
  for (int i = j->row_begin; i < j->row_end; i += 2) {
    const int i1 = (i + 1 < j->row_end) ? i + 1 : i;
    const float* a0 = j->A + (size_t)i * K;
    const float* a1 = j->A + (size_t)i1 * K;
    for (int n = 0; n < j->N; n += 4) {
      const float* b[4];
      for (int q = 0; q < 4; ++q) b[q] = j->B + (size_t)((n + q < j->N) ? n + q : n) * K;
      float acc[2][4][LANES];
      memset(acc, 0, sizeof(acc));
      for (int k = 0; k < K8; k += LANES) {
        for (int q = 0; q < 4; ++q) {
          for (int l = 0; l < LANES; ++l) {
            acc[0][q][l] += a0[k + l] * b[q][k + l];
            acc[1][q][l] += a1[k + l] * b[q][k + l];
          }
        }
      }
      for (int r = 0; r < 2; ++r) {
        const float* a = r ? a1 : a0;
        const int row = r ? i1 : i;
        if (r == 1 && i1 == i) break;
        for (int q = 0; q < 4 && n + q < j->N; ++q) {
          float s = hsum8(acc[r][q]);
          for (int k = K8; k < K; ++k) s += a[k] * b[q][k];
          j->C[(size_t)row * j->ldc + n + q] = f32_to_bf16_rne(s);
        }
      }
    }
  }
  return NULL;
}

/* C (bf16, rows [row_begin,row_end) of M x N, ldc) = A . B^T with fp32
 * accumulation on `nthreads` threads (0 = all online CPUs).  Returns the
 * thread count used, or -1 on bad arguments / allocation failure. */
int oracle_gemm_bf16_nt_f32(int M, int N, int K, const uint16_t* A, const uint16_t* B, uint16_t* C,
                            int ldc, int row_begin, int row_end, int nthreads) {
  if (M < 0 || N < 0 || K < 0 || row_begin < 0 || row_end > M || row_begin > row_end) return -1;
  const int rows = row_end - row_begin;
  float* Af = (float*)malloc(sizeof(float) * ((size_t)rows * K + 1));
  float* Bf = (float*)malloc(sizeof(float) * ((size_t)N * K + 1));
  if (!Af || !Bf) {
    free(Af);
    free(Bf);
    return -1;
  }
  for (size_t x = 0; x < (size_t)rows * K; ++x) Af[x] = bf16_to_f32(A[(size_t)row_begin * K + x]);
  for (size_t x = 0; x < (size_t)N * K; ++x) Bf[x] = bf16_to_f32(B[x]);
  int T = default_threads(nthreads);
  const int pairs = (rows + 1) / 2;
  if (T > pairs) T = pairs > 0 ? pairs : 1;
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)T);
  f32_job* jobs = (f32_job*)malloc(sizeof(f32_job) * (size_t)T);
  for (int t = 0; t < T; ++t) {
    /* bands of whole row pairs, relative to row_begin */
    const int pb = (int)((long long)pairs * t / T), pe = (int)((long long)pairs * (t + 1) / T);
    f32_job jb = {N, K, ldc, Af, Bf, C + (size_t)row_begin * ldc, 2 * pb,
                  (2 * pe < rows) ? 2 * pe : rows};
    jobs[t] = jb;
    pthread_create(&th[t], NULL, f32_worker, &jobs[t]);
  }
  for (int t = 0; t < T; ++t) pthread_join(th[t], NULL);
  free(th);
  free(jobs);
  free(Af);
  free(Bf);
  return T;
}

int oracle_num_cpus(void) { return default_threads(0); }

/* ------------------------------------------------- fused epilogue (fp64)
 * Restatement of the library's optional fused epilogue, which has no
 * counterpart in the reference (whose epilogue is only the bf16 rounding of
 * matmul_1.cuh:293-295).  On an fp64 GEMM sum s of element (i, j):
 *   d = act(alpha * s + bias[j]) + beta * R[i][j]
 * with act: 0 none, 1 max(x, 0), 2 0.5 x (1 + erf(x / sqrt 2)),
 * 3 0.5 x (1 + tanh(sqrt(2 / pi) (x + 0.044715 x^3))), 4 x / (1 + exp(-x)),
 * evaluated in fp64 with the C library's erf, tanh and exp.  bias (bf16[N])
 * and R (bf16, row pitch ldr) may be NULL. */
static double epi_act(double x, int act) {
  switch (act) {
    case 1: return x > 0.0 ? x : 0.0;
    case 2: return 0.5 * x * (1.0 + erf(x * 0.70710678118654752440));
    case 3: return 0.5 * x * (1.0 + tanh(0.79788456080286535588 * (x + 0.044715 * x * x * x)));
    case 4: return x / (1.0 + exp(-x));
    default: return x;
  }
}

static inline double epi_one(double s, int i, int j, double alpha, const uint16_t* bias, int act,
                             const uint16_t* R, int ldr, double beta) {
  double d = alpha * s;
  if (bias) d += (double)bf16_to_f32(bias[j]);
  d = epi_act(d, act);
  if (R) d += beta * (double)bf16_to_f32(R[(size_t)i * ldr + j]);
  return d;
}

/* In place on D (M x N, row pitch ldd) holding fp64 GEMM sums. */
void oracle_epilogue_f64(double* D, int M, int N, int ldd, double alpha, const uint16_t* bias,
                         int act, const uint16_t* R, int ldr, double beta) {
  for (int i = 0; i < M; ++i)
    for (int j = 0; j < N; ++j) {
      double* x = D + (size_t)i * ldd + j;
      *x = epi_one(*x, i, j, alpha, bias, act, R, ldr, beta);
    }
}

/* In place on sampled sums vals[s] of elements (rows[s], cols[s]). */
void oracle_epilogue_sampled(double* vals, const int* rows, const int* cols, size_t count,
                             double alpha, const uint16_t* bias, int act, const uint16_t* R,
                             int ldr, double beta) {
  for (size_t s = 0; s < count; ++s)
    vals[s] = epi_one(vals[s], rows[s], cols[s], alpha, bias, act, R, ldr, beta);
}

/* ----------------------------------------------------- fp8 e4m3 (OCP FP8)
 * E4M3 "fn": 1 sign, 4 exponent (bias 7), 3 mantissa bits, no infinities,
 * S.1111.111 is NaN, largest finite 448 = 1.75 * 2^8, smallest normal 2^-6,
 * subnormal step 2^-9.  Encoding rounds to nearest, ties to even, and
 * saturates anything at or beyond 448 in magnitude to +-448 (the library's
 * fp8 output uses cvt.rn.satfinite, which does the same); NaN -> 0x7F. */
uint8_t oracle_f64_to_e4m3_one(double x) {
  if (isnan(x)) return 0x7F;
  const uint8_t sign = signbit(x) ? 0x80 : 0x00;
  const double a = fabs(x);
  if (a >= 448.0) return sign | 0x7E;
  if (a == 0.0) return sign;
  int e;
  frexp(a, &e);                 /* a = f * 2^e, f in [0.5, 1) */
  int E = e - 1;                /* exponent of the leading bit */
  if (E < -6) E = -6;           /* subnormal range shares the 2^-9 quantum */
  const double q = ldexp(1.0, E - 3);
  const double v = nearbyint(a / q) * q;   /* a / q is exact (power-of-two scale) */
  if (v >= 448.0) return sign | 0x7E;      /* unreachable for a < 448, kept for safety */
  if (v == 0.0) return sign;
  int ev;
  frexp(v, &ev);
  const int Ev = ev - 1;
  if (Ev < -6) return sign | (uint8_t)(v / ldexp(1.0, -9));            /* subnormal */
  const int mant = (int)(v / ldexp(1.0, Ev - 3)) - 8;
  return sign | (uint8_t)((Ev + 7) << 3) | (uint8_t)mant;
}

double oracle_e4m3_to_f64_one(uint8_t b) {
  const int s = b >> 7, e = (b >> 3) & 15, m = b & 7;
  double v;
  if (e == 15 && m == 7) return NAN;
  if (e == 0) v = ldexp((double)m, -9);
  else v = ldexp(1.0 + m / 8.0, e - 7);
  return s ? -v : v;
}

void oracle_f64_to_e4m3(const double* in, uint8_t* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = oracle_f64_to_e4m3_one(in[i]);
}

void oracle_e4m3_to_f64(const uint8_t* in, double* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = oracle_e4m3_to_f64_one(in[i]);
}
