/*
 * CPU oracle for the math-plus GEMM / attention path — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's own CPU arithmetic (math-plus
 * tensor-core / tensor-cpu / special, TypeScript). Only the tests, the smoke
 * check and the benchmark's CPU-baseline leg load it, as the checker; the
 * CUDA library never links or calls it.
 *
 * Parity pins: tests/golden/ holds vectors produced by the reference's own
 * Python oracles (packages/tensor-cpu/scripts/numpy_oracle.py,
 * packages/tensor-webgpu/scripts/gemm_oracle.py, attention_oracle.py,
 * packages/special/scripts/special_oracle.py) plus the literal known answers
 * of the reference's tests (packages/tensor-core/test/half.test.ts,
 * packages/special/test/special.test.ts, packages/tensor-core/test/tensor.test.ts).
 */
#ifndef MP_ORACLE_H
#define MP_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- seeded inputs: packages/tensor-core/src/random.ts:17-118 ---------- */
typedef struct { uint64_t state; uint64_t inc; } mp_rng;
void mp_rng_init(mp_rng *r, uint64_t seed, uint64_t seq);
uint32_t mp_rng_next_u32(mp_rng *r);
double mp_rng_next_float(mp_rng *r);
uint32_t mp_rng_next_below(mp_rng *r, uint32_t bound);
double mp_uniform_sample(mp_rng *r, double lo, double hi);
double mp_normal_sample(mp_rng *r, double mean, double std);
/* fillFrom (random.ts:85-103) into f32 / half storage. */
void mp_fill_uniform_f32(uint64_t seed, size_t n, double lo, double hi, float *out);
void mp_fill_normal_f32(uint64_t seed, size_t n, double mean, double std, float *out);
void mp_fill_normal_half(uint64_t seed, size_t n, double mean, double std, int bf16, uint16_t *out);
void mp_fill_below_i32(uint64_t seed, size_t n, uint32_t bound, int32_t *out);

/* ---- half codec: packages/tensor-core/src/dtype.ts:130-179 -------------- */
uint16_t mp_encode_half(int bf16, double x);
double mp_decode_half(int bf16, uint16_t bits);

/* ---- the reference tests' LCGs ------------------------------------------ */
/* packages/tensor-webgpu/test/gemm.test.ts:85-93 */
void mp_lcg_gemm(size_t n, uint32_t seed, float *out);
/* packages/tensor-cpu/test/helpers.ts:115-124 (values as f64; f32 storage rounds) */
void mp_lcg_seeded(size_t n, uint32_t seed, double lo, double hi, double *out);

/* ---- special functions: packages/special/src/index.ts:65-193 ------------ */
double mp_erf(double x);
double mp_erfc(double x);
double mp_gelu_erf(double x);

/* ---- flat kernels: packages/tensor-core/src/kernels.ts ------------------ */
void mp_gemm_nt(const double *A, const double *B, double *C, size_t c_off, size_t ldc,
                int M, int N, int K);
/* Same arithmetic, output rows split over `threads` OpenMP threads. */
void mp_gemm_nt_par(const double *A, const double *B, double *C, size_t c_off, size_t ldc,
                    int M, int N, int K, int threads);
void mp_pack_panel_f32(const float *src, size_t off, long row_stride, long col_stride,
                       int rows, int cols, double *dst);
void mp_softmax_axis_f32(const float *x, int outer, int dim, int inner, float *out);

/* ---- op glue: Tensor.matmul (packages/tensor-core/src/index.ts:1584-1730) */
/* Batched, broadcasting f32 matmul, f64 accumulation, one rounding.
 * a: [..batch_a.., m, k] contiguous; b: [..batch_b.., k, n] contiguous.
 * Batch shapes are right-aligned and broadcast; out: [..batch.., m, n]. */
int mp_matmul_f32(const float *a, const int64_t *a_shape, int a_rank,
                  const float *b, const int64_t *b_shape, int b_rank,
                  float *out, int threads);

/* linearNT (packages/tensor-core/src/nn-kernels.ts:74-101). */
void mp_linear_f32(const float *x, int rows, int K, const float *w, int N,
                   const float *bias, float *out, int threads);

/* attention (nn-kernels.ts:179-239). mask_kind: 0 none, 1 bool (u8, nonzero attends),
 * 2 additive f32. mask_strides are element strides aligned to [B,H,Lq,Lk] (0 = broadcast). */
void mp_attention_f32(const float *Q, const float *K, const float *V,
                      int B, int H, int Hk, int Lq, int Lk, int Dh, int Dv, double scale,
                      const void *mask, int mask_kind, const int64_t *mask_strides,
                      float *out, int threads);

/* layerNormRows (nn-kernels.ts:108-129). */
void mp_layer_norm_f32(const float *x, int rows, int D, const float *w, const float *b,
                       double eps, float *out);
/* unaryFlat(UN_GELU) on f32 storage (nn-kernels.ts:47): f64 evaluation, one rounding. */
void mp_gelu_f32(const float *x, size_t n, float *out);
/* takeRows (nn-kernels.ts:277-286); returns the first bad index position or -1. */
long mp_take_rows_f32(const float *table, int row_len, int n_rows, const int32_t *idx, size_t n_idx,
                      float *out);
void mp_rope_half_f32(const float *x, int BH, int L, int Dh, double base, float *o);
void mp_geglu_rows_f32(const float *x, int rows, int D, float *o);
void mp_masked_mean_pool_f32(const float *x, int B, int L, int D, const float *mask, float *o);

#ifdef __cplusplus
}
#endif
#endif
