/* turbo_oracle.h -- CPU restatement of the reference Turbo.cpp tensor-library
 * arithmetic.  TEST INFRASTRUCTURE ONLY: the tests, smoke() and bench.py's
 * CPU-baseline leg use it as the checker; the product never links it.
 *
 * Each function cites the reference file:line it restates (paths inside the
 * reference project).  It is compiled with -ffp-contract=off; every fused
 * multiply-add the reference build performs is written as an explicit fmaf().
 * Which operations GCC fuses in the reference build (-O3 -mavx2 -mfma, gnu++17)
 * was established against the reference library itself (oracle/_ref): the
 * Q8_0 dot product and the RMSNorm sum of squares round each product before
 * the add; the RoPE rotation is fused; the fp32 matmul is an FMA chain.
 *
 * Status codes mirror the reference's exception types:
 *   0 ok, 1 std::invalid_argument, 2 std::out_of_range, 3 std::runtime_error.
 */
#ifndef TURBO_ORACLE_H
#define TURBO_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OR_MAX_RANK 8

/* A strided fp32 view: element (i0..ir) lives at base[offset + sum(i_k * stride_k)]. */
typedef struct {
  const float *base;
  int64_t offset;
  int rank;
  int64_t shape[OR_MAX_RANK];
  int64_t strides[OR_MAX_RANK];
} or_view;

float or_f16_to_f32(uint16_t h);
uint16_t or_f32_to_f16(float f);

void or_dequant_q8_0(const uint8_t *blocks, size_t nblocks, float *y);
void or_dequant_q4_0(const uint8_t *blocks, size_t nblocks, float *y);
void or_quantize_row_q8_0(const float *x, uint8_t *blocks, size_t k);
float or_vec_dot_q8_0_f32(const uint8_t *w, const float *x, size_t k);
float or_vec_dot_q4_0_q8_0(const uint8_t *w, const uint8_t *xq, size_t k);
void or_matmul_q8_0(const float *x, size_t M, size_t K, const uint8_t *w, size_t N, float *y);
void or_matmul_q4_0(const float *x, size_t M, size_t K, const uint8_t *w, size_t N, float *y);

int or_broadcast_shape(const int64_t *s1, int r1, const int64_t *s2, int r2,
                       int64_t *out, int *out_rank);
int or_add(const or_view *a, const or_view *b, float *out, int64_t *out_shape, int *out_rank);
void or_scale(const or_view *x, float s, float *out);
int or_copy(float *dst_base, const or_view *dst, const or_view *src);
void or_contiguous(const or_view *x, float *out);

int or_rmsnorm(const float *x, size_t rows, size_t cols, const float *gamma, float eps,
               float *out);
void or_swiglu(const float *g, const float *u, size_t n, float *out);
void or_softmax(const float *x, size_t rows, size_t cols, float *out);
int64_t or_argmax(const float *x, size_t n);
int or_sample_top_p(const float *logits, size_t n, float temperature, float top_p, double u,
                    int *id, size_t *nucleus, size_t *nucleus_f32, double *slack);
int or_sample_top_p_set(const float *logits, size_t n, float temperature, float top_p, double u, double rel_p,
                        double abs_u, int accurate_sum, int *ids, int *n_ids);

void or_rope_tables(size_t head_dim, size_t max_seq, float theta, float *cos_t, float *sin_t);
int or_rope(float *base, const or_view *x, size_t head_dim, size_t max_seq,
            const float *cos_t, const float *sin_t, size_t pos_offset);

int or_embedding(const uint8_t *w, int dtype, size_t dim, size_t vocab, const float *ids,
                 size_t n, float *out);

int or_matmul_f32(const or_view *a, const or_view *b, float *out);

#ifdef __cplusplus
}
#endif
#endif
