/*
 * CPU oracle for the math-plus GEMM / attention path — TEST INFRASTRUCTURE ONLY.
 *
 * Restates, in C, the reference's CPU arithmetic so the CUDA kernels can be
 * checked against it. Every function cites the reference file:line it
 * follows (paths inside the math-plus repository). The CUDA library never
 * links this file; only tests/, the smoke check and bench.py's CPU-baseline
 * leg load liboracle (via oracle/oracle.py).
 *
 * Arithmetic contract kept from the reference (packages/tensor-core/src/kernels.ts:8-16):
 * every dot product accumulates in f64 in ascending index order starting from
 * 0, and values are rounded to f32 exactly where the reference stores into a
 * Float32Array or calls Math.fround.  JS `Math.exp/log/sqrt/cos` map to the C
 * library's double functions; those agree with V8 to within an ulp, which is
 * far inside every tolerance used against the GPU.
 */
#include "mp_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ======================================================================== */
/* PCG32 XSH-RR: packages/tensor-core/src/random.ts:14-66                    */
/* ======================================================================== */
#define PCG_MULT 6364136223846793005ULL

static uint64_t rng_step(mp_rng *r) {
  uint64_t old = r->state;
  r->state = old * PCG_MULT + r->inc; /* mod 2^64 by unsigned wrap-around */
  return old;
}

/* random.ts:21-26: inc = (seq<<1)|1; step; state += seed; step. */
void mp_rng_init(mp_rng *r, uint64_t seed, uint64_t seq) {
  r->state = 0;
  r->inc = (seq << 1) | 1u;
  rng_step(r);
  r->state += seed;
  rng_step(r);
}

/* random.ts:35-48 */
uint32_t mp_rng_next_u32(mp_rng *r) {
  uint64_t old = rng_step(r);
  uint32_t xorshifted = (uint32_t)(((old >> 18) ^ old) >> 27);
  uint32_t rot = (uint32_t)(old >> 59);
  return rot == 0 ? xorshifted : ((xorshifted >> rot) | (xorshifted << (32 - rot)));
}

/* random.ts:51-53 */
double mp_rng_next_float(mp_rng *r) { return (double)mp_rng_next_u32(r) / 4294967296.0; }

/* random.ts:56-66: rejection sampling without modulo bias. */
uint32_t mp_rng_next_below(mp_rng *r, uint32_t bound) {
  uint64_t limit = (4294967296ULL / bound) * bound;
  uint32_t x;
  do {
    x = mp_rng_next_u32(r);
  } while ((uint64_t)x >= limit);
  return x % bound;
}

/* random.ts:105-107 */
double mp_uniform_sample(mp_rng *r, double lo, double hi) { return lo + mp_rng_next_float(r) * (hi - lo); }

/* random.ts:109-118: Box-Muller, cosine branch only, two uniforms per call. */
double mp_normal_sample(mp_rng *r, double mean, double std) {
  double u1 = mp_rng_next_float(r);
  if (u1 == 0) u1 = 4.9406564584124654e-324; /* Number.MIN_VALUE */
  double u2 = mp_rng_next_float(r);
  double z0 = sqrt(-2 * log(u1)) * cos(2 * M_PI * u2);
  return mean + z0 * std;
}

/* fillFrom (random.ts:85-103) with `seed(value)` = new Rng(value) (random.ts:69-71). */
void mp_fill_uniform_f32(uint64_t seed, size_t n, double lo, double hi, float *out) {
  mp_rng r;
  mp_rng_init(&r, seed, 1);
  for (size_t i = 0; i < n; i++) out[i] = (float)mp_uniform_sample(&r, lo, hi);
}

void mp_fill_normal_f32(uint64_t seed, size_t n, double mean, double std, float *out) {
  mp_rng r;
  mp_rng_init(&r, seed, 1);
  for (size_t i = 0; i < n; i++) out[i] = (float)mp_normal_sample(&r, mean, std);
}

void mp_fill_normal_half(uint64_t seed, size_t n, double mean, double std, int bf16, uint16_t *out) {
  mp_rng r;
  mp_rng_init(&r, seed, 1);
  for (size_t i = 0; i < n; i++) out[i] = mp_encode_half(bf16, mp_normal_sample(&r, mean, std));
}

/* randintSample(0, bound) (random.ts:120-125) into i32 storage. */
void mp_fill_below_i32(uint64_t seed, size_t n, uint32_t bound, int32_t *out) {
  mp_rng r;
  mp_rng_init(&r, seed, 1);
  for (size_t i = 0; i < n; i++) out[i] = (int32_t)mp_rng_next_below(&r, bound);
}

/* ======================================================================== */
/* Half codec: packages/tensor-core/src/dtype.ts:110-179                     */
/* ======================================================================== */
/* dtype.ts:111-117 */
static double round_half_even(double v) {
  double f = floor(v);
  double d = v - f;
  if (d > 0.5) return f + 1;
  if (d < 0.5) return f;
  return fmod(f, 2.0) == 0 ? f : f + 1;
}

/* dtype.ts:126-149: RNE directly from the double. */
static uint32_t encode_binary_float(double x, int exp_bits, int mant_bits) {
  uint32_t sign_bit = 1u << (exp_bits + mant_bits);
  uint32_t exp_mask = (1u << exp_bits) - 1;
  int bias = (1 << (exp_bits - 1)) - 1;
  if (isnan(x)) return (exp_mask << mant_bits) | (1u << (mant_bits - 1));
  uint32_t sign = signbit(x) ? sign_bit : 0;
  double a = fabs(x);
  if (a == 0) return sign;
  double overflow = (2 - ldexp(1.0, -(mant_bits + 1))) * ldexp(1.0, bias);
  if (a >= overflow) return sign | (exp_mask << mant_bits);
  int emin = 1 - bias;
  if (a < ldexp(1.0, emin)) return sign | (uint32_t)round_half_even(a / ldexp(1.0, emin - mant_bits));
  int e = (int)floor(log2(a));
  if (ldexp(1.0, e) > a) e--;
  else if (ldexp(1.0, e + 1) <= a) e++;
  uint32_t frac = (uint32_t)round_half_even((a / ldexp(1.0, e) - 1) * ldexp(1.0, mant_bits));
  return sign | ((((uint32_t)(e + bias)) << mant_bits) + frac);
}

/* dtype.ts:152-162 */
static double decode_binary_float(uint32_t bits, int exp_bits, int mant_bits) {
  uint32_t exp_mask = (1u << exp_bits) - 1;
  int bias = (1 << (exp_bits - 1)) - 1;
  double sign = ((bits >> (exp_bits + mant_bits)) & 1) ? -1.0 : 1.0;
  uint32_t e = (bits >> mant_bits) & exp_mask;
  uint32_t m = bits & ((1u << mant_bits) - 1);
  if (e == 0) return sign * m * ldexp(1.0, 1 - bias - mant_bits);
  if (e == exp_mask) return m == 0 ? sign * INFINITY : NAN;
  return sign * (1 + m / ldexp(1.0, mant_bits)) * ldexp(1.0, (int)e - bias);
}

/* dtype.ts:172-174 */
uint16_t mp_encode_half(int bf16, double x) {
  return (uint16_t)(bf16 ? encode_binary_float(x, 8, 7) : encode_binary_float(x, 5, 10));
}
/* dtype.ts:177-179 */
double mp_decode_half(int bf16, uint16_t bits) {
  return bf16 ? decode_binary_float(bits, 8, 7) : decode_binary_float(bits, 5, 10);
}

/* ======================================================================== */
/* Test LCGs                                                                 */
/* ======================================================================== */
/* packages/tensor-webgpu/test/gemm.test.ts:85-93: s = s*1664525 + 1013904223 (u32),
 * value (s / 0xffffffff)*2 - 1 stored into a Float32Array. */
void mp_lcg_gemm(size_t n, uint32_t seed, float *out) {
  uint32_t s = seed;
  for (size_t i = 0; i < n; i++) {
    s = s * 1664525u + 1013904223u;
    out[i] = (float)(((double)s / 4294967295.0) * 2 - 1);
  }
}

/* packages/tensor-cpu/test/helpers.ts:115-124: s = seed || 1; value lo + ((s>>>8)/2^24)*(hi-lo). */
void mp_lcg_seeded(size_t n, uint32_t seed, double lo, double hi, double *out) {
  uint32_t s = seed ? seed : 1u;
  for (size_t i = 0; i < n; i++) {
    s = s * 1664525u + 1013904223u;
    out[i] = lo + ((double)(s >> 8) / 16777216.0) * (hi - lo);
  }
}

/* ======================================================================== */
/* erf / erfc / exact GELU: packages/special/src/index.ts:65-193             */
/* ======================================================================== */
static const double TWO_OVER_SQRT_PI = 1.1283791670955126;
static const double INV_SQRT_PI = 0.5641895835477563;
static const double INV_SQRT2 = 0.7071067811865476;
#define ERF_SERIES_CUTOFF 1.0
#define ERFC_UNDERFLOW 27.3

/* index.ts:95-107: Maclaurin series, at most 60 terms after the leading x. */
static double erf_series(double x) {
  if (x == 0) return x;
  double x2 = x * x, term = x, sum = x;
  for (int n = 1; n <= 60; n++) {
    term *= -x2 / n;
    double c = term / (2 * n + 1);
    sum += c;
    if (fabs(c) <= 1e-17 * fabs(sum)) break;
  }
  return TWO_OVER_SQRT_PI * sum;
}

/* index.ts:110-115 */
static int cf_depth_for(double z) {
  if (z < 1.5) return 100;
  if (z < 2) return 60;
  if (z < 3) return 36;
  return 24;
}

/* JS Math.round: floor(v + 0.5) (ties toward +inf). */
static double js_round(double v) { return floor(v + 0.5); }

/* index.ts:118-121 */
static double exp_neg_square(double z) {
  double s = js_round(z * 4096) / 4096;
  return exp(-s * s) * exp(-(z - s) * (z + s));
}

/* index.ts:124-127 */
static double exp_neg_half_square(double x) {
  double s = js_round(x * 4096) / 4096;
  return exp(-0.5 * (s * s)) * exp(-0.5 * (x - s) * (x + s));
}

/* index.ts:130-137: backward evaluation of the even contraction of Laplace's continued fraction. */
static double erfc_tail(double z, double exp_term, int depth) {
  double t = 2 * z * z + 1;
  double f = 0;
  for (int n = depth; n >= 1; n--) f = ((double)(2 * n - 1) * (2 * n)) / (t + 4 * n - f);
  return (exp_term * INV_SQRT_PI * 2 * z) / (t - f);
}

/* index.ts:146-149 */
static double erfc_cf(double z) {
  if (z > ERFC_UNDERFLOW) return 0;
  return erfc_tail(z, exp_neg_square(z), cf_depth_for(z));
}

/* index.ts:169-175 */
double mp_erf(double x) {
  if (x != x) return NAN;
  double ax = fabs(x);
  if (ax < ERF_SERIES_CUTOFF) return erf_series(x);
  double c = erfc_cf(ax);
  return x > 0 ? 1 - c : c - 1;
}

/* index.ts:178-183 */
double mp_erfc(double x) {
  if (x != x) return NAN;
  if (x >= ERF_SERIES_CUTOFF) return erfc_cf(x);
  if (x <= -ERF_SERIES_CUTOFF) return 2 - erfc_cf(-x);
  return 1 - erf_series(x);
}

/* index.ts:157-165: Phi(x) = 0.5*erfc(-x/sqrt2), exponent taken from x in the left tail. */
static double normal_cdf(double x) {
  double z = -x * INV_SQRT2;
  if (z >= ERF_SERIES_CUTOFF) {
    if (z > ERFC_UNDERFLOW) return 0;
    return 0.5 * erfc_tail(z, exp_neg_half_square(x), cf_depth_for(z));
  }
  return 0.5 * mp_erfc(z);
}

/* index.ts:191-193 */
double mp_gelu_erf(double x) { return x * normal_cdf(x); }

/* ======================================================================== */
/* gemmNT / packPanel / softmaxAxis: packages/tensor-core/src/kernels.ts     */
/* ======================================================================== */
/* kernels.ts:299-362: C[i,j] = sum_p A[i*K+p]*B[j*K+p], 4x4 register block, 64-column
 * j-blocks; every output accumulates p = 0..K-1 in order from 0 (so the blocking never
 * changes a result bit). Rows [i0, i1) only, so callers can split rows over threads. */
static void gemm_nt_rows(const double *A, const double *B, double *C, size_t c_off, size_t ldc,
                         int i0, int i1, int N, int K) {
  const int JB = 64;
  for (int j0 = 0; j0 < N; j0 += JB) {
    int j1 = N < j0 + JB ? N : j0 + JB;
    int i = i0;
    for (; i + 4 <= i1; i += 4) {
      const double *a0 = A + (size_t)i * K, *a1 = a0 + K, *a2 = a1 + K, *a3 = a2 + K;
      double *c0 = C + c_off + (size_t)i * ldc, *c1 = c0 + ldc, *c2 = c1 + ldc, *c3 = c2 + ldc;
      int j = j0;
      for (; j + 4 <= j1; j += 4) {
        const double *b0 = B + (size_t)j * K, *b1 = b0 + K, *b2 = b1 + K, *b3 = b2 + K;
        double s00 = 0, s01 = 0, s02 = 0, s03 = 0, s10 = 0, s11 = 0, s12 = 0, s13 = 0;
        double s20 = 0, s21 = 0, s22 = 0, s23 = 0, s30 = 0, s31 = 0, s32 = 0, s33 = 0;
        for (int p = 0; p < K; p++) {
          double x0 = a0[p], x1 = a1[p], x2 = a2[p], x3 = a3[p];
          double y0 = b0[p], y1 = b1[p], y2 = b2[p], y3 = b3[p];
          s00 += x0 * y0; s01 += x0 * y1; s02 += x0 * y2; s03 += x0 * y3;
          s10 += x1 * y0; s11 += x1 * y1; s12 += x1 * y2; s13 += x1 * y3;
          s20 += x2 * y0; s21 += x2 * y1; s22 += x2 * y2; s23 += x2 * y3;
          s30 += x3 * y0; s31 += x3 * y1; s32 += x3 * y2; s33 += x3 * y3;
        }
        c0[j] = s00; c0[j + 1] = s01; c0[j + 2] = s02; c0[j + 3] = s03;
        c1[j] = s10; c1[j + 1] = s11; c1[j + 2] = s12; c1[j + 3] = s13;
        c2[j] = s20; c2[j + 1] = s21; c2[j + 2] = s22; c2[j + 3] = s23;
        c3[j] = s30; c3[j + 1] = s31; c3[j + 2] = s32; c3[j + 3] = s33;
      }
      for (; j < j1; j++) {
        const double *b0 = B + (size_t)j * K;
        double s0 = 0, s1 = 0, s2 = 0, s3 = 0;
        for (int p = 0; p < K; p++) {
          double y = b0[p];
          s0 += a0[p] * y; s1 += a1[p] * y; s2 += a2[p] * y; s3 += a3[p] * y;
        }
        c0[j] = s0; c1[j] = s1; c2[j] = s2; c3[j] = s3;
      }
    }
    for (; i < i1; i++) {
      const double *a0 = A + (size_t)i * K;
      double *c0 = C + c_off + (size_t)i * ldc;
      int j = j0;
      for (; j + 4 <= j1; j += 4) {
        const double *b0 = B + (size_t)j * K, *b1 = b0 + K, *b2 = b1 + K, *b3 = b2 + K;
        double s0 = 0, s1 = 0, s2 = 0, s3 = 0;
        for (int p = 0; p < K; p++) {
          double x = a0[p];
          s0 += x * b0[p]; s1 += x * b1[p]; s2 += x * b2[p]; s3 += x * b3[p];
        }
        c0[j] = s0; c0[j + 1] = s1; c0[j + 2] = s2; c0[j + 3] = s3;
      }
      for (; j < j1; j++) {
        const double *b0 = B + (size_t)j * K;
        double s = 0;
        for (int p = 0; p < K; p++) s += a0[p] * b0[p];
        c0[j] = s;
      }
    }
  }
}

void mp_gemm_nt(const double *A, const double *B, double *C, size_t c_off, size_t ldc, int M, int N,
                int K) {
  gemm_nt_rows(A, B, C, c_off, ldc, 0, M, N, K);
}

/* Row blocks of 4 (the register block height) handed to threads: every output element is
 * still produced by exactly the serial code path, so results are bit-identical to mp_gemm_nt. */
void mp_gemm_nt_par(const double *A, const double *B, double *C, size_t c_off, size_t ldc, int M,
                    int N, int K, int threads) {
#ifdef _OPENMP
  if (threads > 1 && M > 4) {
    int nblk = (M + 15) / 16;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
    for (int blk = 0; blk < nblk; blk++) {
      int i0 = blk * 16, i1 = i0 + 16 < M ? i0 + 16 : M;
      gemm_nt_rows(A, B, C, c_off, ldc, i0, i1, N, K);
    }
    return;
  }
#endif
  (void)threads;
  gemm_nt_rows(A, B, C, c_off, ldc, 0, M, N, K);
}

/* kernels.ts:370-388 */
void mp_pack_panel_f32(const float *src, size_t off, long row_stride, long col_stride, int rows,
                       int cols, double *dst) {
  for (int r = 0; r < rows; r++) {
    const float *s = src + off + (long)r * row_stride;
    double *d = dst + (size_t)r * cols;
    for (int c = 0; c < cols; c++) d[c] = s[(long)c * col_stride];
  }
}

/* kernels.ts:219-247 with f32 = true: x - max and the row sum rounded with Math.fround;
 * exp values stored into the f32 output (rounding them) and re-read for sum and divide. */
void mp_softmax_axis_f32(const float *x, int outer, int dim, int inner, float *o) {
  for (int r = 0; r < outer; r++) {
    size_t base = (size_t)r * dim * inner;
    for (int t = 0; t < inner; t++) {
      size_t lane = base + t;
      double mx = x[lane];
      for (int j = 1; j < dim; j++) {
        double v = x[lane + (size_t)j * inner];
        if (v > mx) mx = v;
      }
      double sum = 0;
      for (int j = 0; j < dim; j++) {
        size_t k = lane + (size_t)j * inner;
        double d = (double)x[k] - mx;
        o[k] = (float)exp((double)(float)d);
        sum += o[k];
      }
      double s = (double)(float)sum;
      for (int j = 0; j < dim; j++) {
        size_t k = lane + (size_t)j * inner;
        o[k] = (float)((double)o[k] / s);
      }
    }
  }
}

/* ======================================================================== */
/* Tensor.matmul: packages/tensor-core/src/index.ts:1584-1730                */
/* ======================================================================== */
int mp_matmul_f32(const float *a, const int64_t *a_shape, int a_rank, const float *b,
                  const int64_t *b_shape, int b_rank, float *out, int threads) {
  if (a_rank < 2 || b_rank < 2) return -1;
  int64_t m = a_shape[a_rank - 2], k = a_shape[a_rank - 1];
  int64_t k2 = b_shape[b_rank - 2], n = b_shape[b_rank - 1];
  if (k != k2) return -2;
  int la = a_rank - 2, lb = b_rank - 2;
  int rank = la > lb ? la : lb;
  if (rank > 16) return -3;
  int64_t shape[16], sa[16], sb[16];
  /* Row-major batch strides of each operand (in matrices), aligned right; 0 on broadcast axes. */
  int64_t stride_a = m * k, stride_b = k * n;
  for (int d = rank - 1; d >= 0; d--) {
    int ia = d - (rank - la), ib = d - (rank - lb);
    int64_t da = ia >= 0 ? a_shape[ia] : 1, db = ib >= 0 ? b_shape[ib] : 1;
    if (da != db && da != 1 && db != 1) return -4;
    shape[d] = da == 1 ? db : da;
    sa[d] = da == 1 ? 0 : stride_a;
    sb[d] = db == 1 ? 0 : stride_b;
    stride_a *= da;
    stride_b *= db;
  }
  int64_t batch = 1;
  for (int d = 0; d < rank; d++) batch *= shape[d];
  double *pa = (double *)malloc(sizeof(double) * (size_t)(m * k > 0 ? m * k : 1));
  double *pb = (double *)malloc(sizeof(double) * (size_t)(n * k > 0 ? n * k : 1));
  double *acc = (double *)malloc(sizeof(double) * (size_t)(m * n > 0 ? m * n : 1));
  int64_t idx[16] = {0};
  int64_t offa = 0, offb = 0, packed_a = -1, packed_b = -1;
  for (int64_t bi = 0; bi < batch; bi++) {
    /* index.ts:1658-1665: a panel is re-packed only when its batch offset changes. */
    if (offa != packed_a) {
      mp_pack_panel_f32(a, (size_t)offa, (long)k, 1, (int)m, (int)k, pa);
      packed_a = offa;
    }
    if (offb != packed_b) {
      /* B transposed: B's column stride as row stride, row stride as column stride. */
      mp_pack_panel_f32(b, (size_t)offb, 1, (long)n, (int)n, (int)k, pb);
      packed_b = offb;
    }
    mp_gemm_nt_par(pa, pb, acc, 0, (size_t)n, (int)m, (int)n, (int)k, threads);
    float *o = out + bi * m * n;
    for (int64_t t = 0; t < m * n; t++) o[t] = (float)acc[t]; /* index.ts:1669-1670 */
    for (int d = rank - 1; d >= 0; d--) {
      idx[d]++;
      offa += sa[d];
      offb += sb[d];
      if (idx[d] < shape[d]) break;
      idx[d] = 0;
      offa -= shape[d] * sa[d];
      offb -= shape[d] * sb[d];
    }
  }
  free(pa);
  free(pb);
  free(acc);
  return 0;
}

/* ======================================================================== */
/* linearNT: packages/tensor-core/src/nn-kernels.ts:70-101                   */
/* ======================================================================== */
void mp_linear_f32(const float *x, int rows, int K, const float *w, int N, const float *bias,
                   float *out, int threads) {
  const int ROW_BLOCK = 256;
  double *pw = (double *)malloc(sizeof(double) * ((size_t)N * K + 1));
  mp_pack_panel_f32(w, 0, K, 1, N, K, pw);
  int rb = rows < ROW_BLOCK ? rows : ROW_BLOCK;
  double *pa = (double *)malloc(sizeof(double) * ((size_t)rb * K + 1));
  double *acc = (double *)malloc(sizeof(double) * ((size_t)rb * N + 1));
  for (int r0 = 0; r0 < rows; r0 += rb) {
    int m = rows - r0 < rb ? rows - r0 : rb;
    mp_pack_panel_f32(x, (size_t)r0 * K, K, 1, m, K, pa);
    mp_gemm_nt_par(pa, pw, acc, 0, (size_t)N, m, N, K, threads);
    float *o = out + (size_t)r0 * N;
    for (int i = 0; i < m; i++)
      for (int j = 0; j < N; j++)
        o[(size_t)i * N + j] = (float)(acc[(size_t)i * N + j] + (bias ? (double)bias[j] : 0.0));
  }
  free(pw);
  free(pa);
  free(acc);
}

/* ======================================================================== */
/* attention: packages/tensor-core/src/nn-kernels.ts:179-239                 */
/* ======================================================================== */
static void attention_head(const float *Q, const float *K, const float *V, int b, int h, int H,
                           int Hk, int Lq, int Lk, int Dh, int Dv, double scale, const void *mask,
                           int mask_kind, const int64_t *ms, float *out, double *pq, double *pk,
                           double *pvt, double *S, double *acc) {
  int rep = H / Hk;
  int kvh = b * Hk + h / rep;
  mp_pack_panel_f32(Q, (size_t)(b * H + h) * Lq * Dh, Dh, 1, Lq, Dh, pq);
  mp_pack_panel_f32(K, (size_t)kvh * Lk * Dh, Dh, 1, Lk, Dh, pk);
  /* V transposed: row d of the panel is column d of this head's V. */
  mp_pack_panel_f32(V, (size_t)kvh * Lk * Dv, 1, Dv, Dv, Lk, pvt);
  mp_gemm_nt(pq, pk, S, 0, (size_t)Lk, Lq, Lk, Dh);
  for (int i = 0; i < Lq; i++) {
    double *row = S + (size_t)i * Lk;
    int64_t mo = (int64_t)b * ms[0] + (int64_t)h * ms[1] + (int64_t)i * ms[2];
    double m = -INFINITY;
    for (int j = 0; j < Lk; j++) {
      double s = row[j] * scale;
      if (mask_kind == 1) {
        if (!((const uint8_t *)mask)[mo + (int64_t)j * ms[3]]) s = -INFINITY;
      } else if (mask_kind == 2) {
        s += (double)((const float *)mask)[mo + (int64_t)j * ms[3]];
      }
      row[j] = s;
      if (s > m) m = s;
    }
    if (m == -INFINITY) { /* nn-kernels.ts:222-225: a fully masked row yields zeros */
      for (int j = 0; j < Lk; j++) row[j] = 0;
      continue;
    }
    double sum = 0;
    for (int j = 0; j < Lk; j++) {
      double e = exp(row[j] - m);
      row[j] = e;
      sum += e;
    }
    double inv = 1 / sum;
    for (int j = 0; j < Lk; j++) row[j] *= inv;
  }
  mp_gemm_nt(S, pvt, acc, 0, (size_t)Dv, Lq, Dv, Lk);
  float *o = out + (size_t)(b * H + h) * Lq * Dv;
  for (size_t t = 0; t < (size_t)Lq * Dv; t++) o[t] = (float)acc[t];
}

void mp_attention_f32(const float *Q, const float *K, const float *V, int B, int H, int Hk, int Lq,
                      int Lk, int Dh, int Dv, double scale, const void *mask, int mask_kind,
                      const int64_t *mask_strides, float *out, int threads) {
  int64_t zero[4] = {0, 0, 0, 0};
  const int64_t *ms = mask_strides ? mask_strides : zero;
  int total = B * H;
#ifdef _OPENMP
#pragma omp parallel num_threads(threads > 1 ? threads : 1)
#endif
  {
    double *pq = (double *)malloc(sizeof(double) * ((size_t)Lq * Dh + 1));
    double *pk = (double *)malloc(sizeof(double) * ((size_t)Lk * Dh + 1));
    double *pvt = (double *)malloc(sizeof(double) * ((size_t)Dv * Lk + 1));
    double *S = (double *)malloc(sizeof(double) * ((size_t)Lq * Lk + 1));
    double *acc = (double *)malloc(sizeof(double) * ((size_t)Lq * Dv + 1));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
    for (int bh = 0; bh < total; bh++)
      attention_head(Q, K, V, bh / H, bh % H, H, Hk, Lq, Lk, Dh, Dv, scale, mask, mask_kind, ms, out,
                     pq, pk, pvt, S, acc);
    free(pq);
    free(pk);
    free(pvt);
    free(S);
    free(acc);
  }
  (void)threads;
}

/* ======================================================================== */
/* layerNormRows / unaryFlat(GELU) / takeRows: nn-kernels.ts                 */
/* ======================================================================== */
/* nn-kernels.ts:108-129: population variance, f64 statistics, two passes. */
void mp_layer_norm_f32(const float *x, int rows, int D, const float *w, const float *b, double eps,
                       float *o) {
  for (int r = 0; r < rows; r++) {
    const float *s = x + (size_t)r * D;
    float *d = o + (size_t)r * D;
    double mean = 0;
    for (int j = 0; j < D; j++) mean += s[j];
    mean /= D;
    double v = 0;
    for (int j = 0; j < D; j++) {
      double c = s[j] - mean;
      v += c * c;
    }
    double inv = 1 / sqrt(v / D + eps);
    for (int j = 0; j < D; j++) {
      double y = (s[j] - mean) * inv;
      if (w) y *= w[j];
      if (b) y += b[j];
      d[j] = (float)y;
    }
  }
}

/* nn-kernels.ts:47 */
void mp_gelu_f32(const float *x, size_t n, float *out) {
  for (size_t i = 0; i < n; i++) out[i] = (float)mp_gelu_erf(x[i]);
}

/* nn-kernels.ts:277-286 */
long mp_take_rows_f32(const float *table, int row_len, int n_rows, const int32_t *idx, size_t n_idx,
                      float *out) {
  for (size_t i = 0; i < n_idx; i++) {
    int32_t r = idx[i];
    if (!(r >= 0 && r < n_rows)) return (long)i;
    memcpy(out + i * (size_t)row_len, table + (size_t)r * row_len, sizeof(float) * (size_t)row_len);
  }
  return -1;
}

/* nn-kernels.ts:138-160 (ropeHalf): split-half rotary embedding over BH contiguous [L, Dh]
 * blocks. inv_freq = f32(2^f32(-f32(i/half) * f32(log2 base))), theta = f32(p * inv_freq), cos and
 * sin in f64, the rotation in f64 (no contraction: -ffp-contract=off), one f32 rounding. */
void mp_rope_half_f32(const float *x, int BH, int L, int Dh, double base, float *o) {
  const int half = Dh / 2;
  const float lb = (float)log2(base);
  double *cs = malloc(sizeof(double) * (size_t)L * half * 2);
  for (int i = 0; i < half; i++) {
    const float fi = (float)((double)i / half);
    const float invf = (float)pow(2.0, (double)(float)(-(double)fi * lb));
    for (int p = 0; p < L; p++) {
      const float th = (float)((double)p * invf);
      cs[((size_t)p * half + i) * 2] = cos(th);
      cs[((size_t)p * half + i) * 2 + 1] = sin(th);
    }
  }
  for (int bh = 0; bh < BH; bh++) {
    for (int p = 0; p < L; p++) {
      const float *s = x + ((size_t)bh * L + p) * Dh;
      float *d = o + ((size_t)bh * L + p) * Dh;
      for (int i = 0; i < half; i++) {
        const double x1 = s[i], x2 = s[half + i];
        const double c = cs[((size_t)p * half + i) * 2], sn = cs[((size_t)p * half + i) * 2 + 1];
        d[i] = (float)(x1 * c - x2 * sn);
        d[half + i] = (float)(x2 * c + x1 * sn);
      }
    }
  }
  free(cs);
}

/* nn-kernels.ts:245-250 (gegluRows): o[r, j] = geluErf(x[r, j]) * x[r, D + j]. */
void mp_geglu_rows_f32(const float *x, int rows, int D, float *o) {
  for (int r = 0; r < rows; r++) {
    const float *s = x + (size_t)r * 2 * D;
    for (int j = 0; j < D; j++) o[(size_t)r * D + j] = (float)(mp_gelu_erf(s[j]) * s[D + j]);
  }
}

/* nn-kernels.ts:256-271 (maskedMeanPool): f64 sums over kept positions (mask nonzero, NaN falsy),
 * times 1 / max(count, 1). */
void mp_masked_mean_pool_f32(const float *x, int B, int L, int D, const float *mask, float *o) {
  double *acc = malloc(sizeof(double) * (size_t)(D > 0 ? D : 1));
  for (int b = 0; b < B; b++) {
    for (int j = 0; j < D; j++) acc[j] = 0;
    int cnt = 0;
    for (int l = 0; l < L; l++) {
      const float m = mask[(size_t)b * L + l];
      if (m == 0 || m != m) continue;
      cnt++;
      const float *s = x + ((size_t)b * L + l) * D;
      for (int j = 0; j < D; j++) acc[j] += s[j];
    }
    const double inv = 1.0 / (cnt > 1 ? cnt : 1);
    for (int j = 0; j < D; j++) o[(size_t)b * D + j] = (float)(acc[j] * inv);
  }
  free(acc);
}
