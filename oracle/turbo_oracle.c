/* turbo_oracle.c -- CPU restatement of the reference Turbo.cpp tensor-library
 * arithmetic.  TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * Parity pinned: tests/test_oracle_pin.py compares every function here with the
 * reference library compiled from its own sources (oracle/_ref) and with the
 * known-answer vectors of the reference's gtest suite (tests/golden/).
 *
 * Compiled with -ffp-contract=off.  Operation order and rounding follow the
 * reference build (GCC -O3 -mavx2 -mfma -mf16c, gnu++17) as measured against it:
 * fused multiply-adds are written as fmaf() exactly where the reference build
 * fuses them, and nowhere else.
 */
#include "turbo_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

enum { OK = 0, E_INVAL = 1, E_RANGE = 2, E_RUNTIME = 3 };

/* ---- IEEE binary16 <-> binary32 (F16C semantics) ---------------------------
 * fp16_to_fp32 / convert_f32_to_f16: src/tensor/quant_math.hpp:11-13, 63-65
 * (_cvtsh_ss and _cvtss_sh(f, 0), i.e. round-to-nearest-even). */
float or_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do {
        man <<= 1;
        ++e;
      } while ((man & 0x400u) == 0);
      man &= 0x3FFu;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 0x1F) {
    bits = sign | 0x7F800000u | (man << 13) | (man ? 0x00400000u : 0u);
  } else {
    bits = sign | ((exp + (127 - 15)) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

uint16_t or_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  uint32_t absx = x & 0x7FFFFFFFu;
  if (absx > 0x7F800000u) /* NaN: quiet, keep top payload bits */
    return (uint16_t)(sign | 0x7E00u | ((absx >> 13) & 0x3FFu));
  if (absx >= 0x477FF000u) /* >= 65520 rounds to infinity */
    return (uint16_t)(sign | 0x7C00u);
  if (absx < 0x38800000u) { /* below the smallest normal half: subnormal or zero */
    if (absx < 0x33000000u) /* < 2^-25: rounds to zero (2^-25 itself ties to 0) */
      return sign;
    uint32_t e = absx >> 23;
    uint32_t m = (absx & 0x7FFFFFu) | 0x800000u;
    uint32_t shift = 126u - e; /* 14..24 */
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (q & 1u)))
      ++q;
    return (uint16_t)(sign | q);
  }
  uint32_t e = (absx >> 23) - 112u; /* rebias 127 -> 15 */
  uint32_t m = absx & 0x7FFFFFu;
  uint32_t q = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u)))
    ++q; /* may carry into the exponent, which is correct */
  return (uint16_t)(sign | q);
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static void wr16(uint8_t *p, uint16_t v) {
  p[0] = (uint8_t)(v & 0xFF);
  p[1] = (uint8_t)(v >> 8);
}

/* ---- Q8_0 / Q4_0 blocks (include/turbo/tensor/quant_types.hpp:17-38) -------
 * Q8_0: {u16 d; i8 qs[32]} 34 B.  Q4_0: {u16 d; u8 qs[16]} 18 B; low nibble of
 * qs[j] is element j, high nibble element j + 16. */

/* dequantize_row_q8_0: src/tensor/quant_math.hpp:16-29 (y = q * d). */
void or_dequant_q8_0(const uint8_t *blocks, size_t nblocks, float *y) {
  for (size_t b = 0; b < nblocks; ++b) {
    const uint8_t *blk = blocks + b * 34;
    float d = or_f16_to_f32(rd16(blk));
    for (int j = 0; j < 32; ++j)
      y[b * 32 + j] = (float)(int8_t)blk[2 + j] * d;
  }
}

/* Q4_0 row dequantisation as nn::Embedding does it: src/nn/embedding.cpp:54-63,100-111. */
void or_dequant_q4_0(const uint8_t *blocks, size_t nblocks, float *y) {
  for (size_t b = 0; b < nblocks; ++b) {
    const uint8_t *blk = blocks + b * 18;
    float d = or_f16_to_f32(rd16(blk));
    for (int j = 0; j < 16; ++j) {
      uint8_t packed = blk[2 + j];
      y[b * 32 + j] = (float)((packed & 0x0F) - 8) * d;
      y[b * 32 + j + 16] = (float)((packed >> 4) - 8) * d;
    }
  }
}

/* quantize_row_q8_0: src/tensor/quant_math.hpp:68-90.  amax via std::max (NaN
 * never replaces the running max), d = amax/127 stored as fp16 (RNE), id = 1/d
 * from the fp32 d, q = std::round (half away from zero). */
void or_quantize_row_q8_0(const float *x, uint8_t *blocks, size_t k) {
  size_t nb = k / 32;
  for (size_t b = 0; b < nb; ++b) {
    float max_val = 0.0f;
    for (int j = 0; j < 32; ++j) {
      float a = fabsf(x[b * 32 + j]);
      max_val = (max_val < a) ? a : max_val;
    }
    float d = max_val / 127.0f;
    uint8_t *blk = blocks + b * 34;
    wr16(blk, or_f32_to_f16(d));
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    for (int j = 0; j < 32; ++j)
      blk[2 + j] = (uint8_t)(int8_t)(int)roundf(x[b * 32 + j] * id);
  }
}

/* vec_dot_q8_0_f32: src/tensor/quant_math.hpp:32-60.  Per block, a sequential
 * sum of (q*d)*x with every product rounded (the reference build does not fuse
 * here); block sums are added to the total in block order. */
float or_vec_dot_q8_0_f32(const uint8_t *w, const float *x, size_t k) {
  size_t nb = k / 32;
  float sum = 0.0f;
  for (size_t b = 0; b < nb; ++b) {
    const uint8_t *blk = w + b * 34;
    float d = or_f16_to_f32(rd16(blk));
    float bs = 0.0f;
    for (int j = 0; j < 32; ++j) {
      float wf = (float)(int8_t)blk[2 + j] * d;
      float p = wf * x[b * 32 + j];
      bs = bs + p;
    }
    sum = sum + bs;
  }
  return sum;
}

/* vec_dot_q4_0_q8_0_avx2: src/tensor/quant_math.hpp:184-248.  Eight fp32 lanes:
 * lane l gets the exact int32 pair sums of elements (2l, 2l+1) and then
 * (16+2l, 17+2l) of each block, each added with an FMA by d = d_w*d_x; the eight
 * lanes are summed in order at the end. */
float or_vec_dot_q4_0_q8_0(const uint8_t *w, const uint8_t *xq, size_t k) {
  size_t nb = k / 32;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (size_t b = 0; b < nb; ++b) {
    const uint8_t *wb = w + b * 18;
    const uint8_t *xb = xq + b * 34;
    float d = or_f16_to_f32(rd16(wb)) * or_f16_to_f32(rd16(xb));
    const int8_t *a = (const int8_t *)(xb + 2);
    for (int l = 0; l < 8; ++l) {
      int w00 = (wb[2 + 2 * l] & 0x0F) - 8, w01 = (wb[3 + 2 * l] & 0x0F) - 8;
      int w10 = (wb[2 + 2 * l] >> 4) - 8, w11 = (wb[3 + 2 * l] >> 4) - 8;
      int p0 = w00 * a[2 * l] + w01 * a[2 * l + 1];
      int p1 = w10 * a[16 + 2 * l] + w11 * a[17 + 2 * l];
      acc[l] = fmaf((float)p0, d, acc[l]);
      acc[l] = fmaf((float)p1, d, acc[l]);
    }
  }
  float sum = 0.0f;
  for (int l = 0; l < 8; ++l)
    sum = sum + acc[l];
  return sum;
}

/* Tensor::matmul Q8_0 branch: src/tensor/tensor.cpp:328-382 (X is not quantized;
 * each Y[m,n] is vec_dot_q8_0_f32 of W row n with X row m). */
void or_matmul_q8_0(const float *x, size_t M, size_t K, const uint8_t *w, size_t N, float *y) {
  size_t row_bytes = K / 32 * 34;
  for (size_t m = 0; m < M; ++m)
    for (size_t n = 0; n < N; ++n)
      y[m * N + n] = or_vec_dot_q8_0_f32(w + n * row_bytes, x + m * K, K);
}

/* Tensor::matmul Q4_0 branch: src/tensor/tensor.cpp:383-432 (X rows quantized to
 * Q8_0 first, then vec_dot_q4_0_q8_0_avx2). */
void or_matmul_q4_0(const float *x, size_t M, size_t K, const uint8_t *w, size_t N, float *y) {
  size_t row_bytes = K / 32 * 18;
  size_t xq_row = K / 32 * 34;
  uint8_t *xq = (uint8_t *)malloc(M * xq_row);
  for (size_t m = 0; m < M; ++m)
    or_quantize_row_q8_0(x + m * K, xq + m * xq_row, K);
  for (size_t m = 0; m < M; ++m)
    for (size_t n = 0; n < N; ++n)
      y[m * N + n] = or_vec_dot_q4_0_q8_0(w + n * row_bytes, xq + m * xq_row, K);
  free(xq);
}

/* ---- views, broadcast, elementwise ----------------------------------------- */

static int64_t numel_of(const int64_t *shape, int rank) {
  /* Tensor::numel: src/tensor/tensor.cpp:99-106 (rank 0 counts as 0 elements). */
  if (rank == 0)
    return 0;
  int64_t n = 1;
  for (int i = 0; i < rank; ++i)
    n *= shape[i];
  return n;
}

static int64_t phys(const or_view *v, const int64_t *idx) {
  int64_t off = v->offset;
  for (int i = 0; i < v->rank; ++i)
    off += idx[i] * v->strides[i];
  return off;
}

static void unravel(int64_t flat, const int64_t *shape, int rank, int64_t *idx) {
  /* Tensor::unravel_index: src/tensor/tensor.cpp:49-57. */
  for (int i = rank - 1; i >= 0; --i) {
    idx[i] = flat % shape[i];
    flat /= shape[i];
  }
}

/* Tensor::compute_broadcast_shape: src/tensor/tensor.cpp:29-47. */
int or_broadcast_shape(const int64_t *s1, int r1, const int64_t *s2, int r2, int64_t *out,
                       int *out_rank) {
  int r = r1 > r2 ? r1 : r2;
  for (int k = 0; k < r; ++k) {
    int i = r1 - 1 - k, j = r2 - 1 - k;
    int64_t d1 = i >= 0 ? s1[i] : 1, d2 = j >= 0 ? s2[j] : 1;
    if (d1 != d2 && d1 != 1 && d2 != 1)
      return E_INVAL;
    out[r - 1 - k] = d1 > d2 ? d1 : d2;
  }
  *out_rank = r;
  return OK;
}

/* Tensor::broadcast_to: src/tensor/tensor.cpp:232-256 (stride 0 on broadcast dims). */
static int broadcast_view(const or_view *v, const int64_t *shape, int rank, or_view *out) {
  if (rank < v->rank)
    return E_INVAL;
  int diff = rank - v->rank;
  out->base = v->base;
  out->offset = v->offset;
  out->rank = rank;
  for (int i = 0; i < rank; ++i) {
    int64_t s = i < diff ? 1 : v->shape[i - diff];
    int64_t st = i < diff ? 0 : v->strides[i - diff];
    if (s != shape[i]) {
      if (s != 1)
        return E_INVAL;
      st = 0;
    }
    out->shape[i] = shape[i];
    out->strides[i] = st;
  }
  return OK;
}

/* Tensor::operator+: src/tensor/tensor.cpp:260-282.  Writes the broadcast
 * result contiguously into `out`; `out_shape`/`out_rank` receive its shape. */
int or_add(const or_view *a, const or_view *b, float *out, int64_t *out_shape, int *out_rank) {
  int st = or_broadcast_shape(a->shape, a->rank, b->shape, b->rank, out_shape, out_rank);
  if (st)
    return st;
  or_view ab, bb;
  if ((st = broadcast_view(a, out_shape, *out_rank, &ab)) != OK)
    return st;
  if ((st = broadcast_view(b, out_shape, *out_rank, &bb)) != OK)
    return st;
  int64_t n = numel_of(out_shape, *out_rank);
  int64_t idx[OR_MAX_RANK];
  for (int64_t i = 0; i < n; ++i) {
    unravel(i, out_shape, *out_rank, idx);
    out[i] = ab.base[phys(&ab, idx)] + bb.base[phys(&bb, idx)];
  }
  return OK;
}

/* Tensor::operator*(float): src/tensor/tensor.cpp:284-294. */
void or_scale(const or_view *x, float s, float *out) {
  int64_t n = numel_of(x->shape, x->rank);
  int64_t idx[OR_MAX_RANK];
  for (int64_t i = 0; i < n; ++i) {
    unravel(i, x->shape, x->rank, idx);
    out[i] = x->base[phys(x, idx)] * s;
  }
}

/* Tensor::copy_: src/tensor/tensor.cpp:689-726 (shapes must match exactly). */
int or_copy(float *dst_base, const or_view *dst, const or_view *src) {
  if (dst->rank != src->rank)
    return E_INVAL;
  for (int i = 0; i < dst->rank; ++i)
    if (dst->shape[i] != src->shape[i])
      return E_INVAL;
  int64_t n = numel_of(dst->shape, dst->rank);
  int64_t idx[OR_MAX_RANK];
  for (int64_t i = 0; i < n; ++i) {
    unravel(i, dst->shape, dst->rank, idx);
    dst_base[phys(dst, idx)] = src->base[phys(src, idx)];
  }
  return OK;
}

/* Tensor::contiguous: src/tensor/tensor.cpp:118-132. */
void or_contiguous(const or_view *x, float *out) {
  int64_t n = numel_of(x->shape, x->rank);
  int64_t idx[OR_MAX_RANK];
  for (int64_t i = 0; i < n; ++i) {
    unravel(i, x->shape, x->rank, idx);
    out[i] = x->base[phys(x, idx)];
  }
}

/* ---- row ops ---------------------------------------------------------------- */

/* nn::RMSNorm::forward: src/nn/rmsnorm.cpp:23-68.  Sequential sum of squares
 * with rounded products, mean = sum / cols, rms = sqrtf(mean + eps), and
 * y = (x / rms) * gamma. */
int or_rmsnorm(const float *x, size_t rows, size_t cols, const float *gamma, float eps,
               float *out) {
  if (cols == 0)
    return E_INVAL;
  for (size_t r = 0; r < rows; ++r) {
    const float *xr = x + r * cols;
    float ss = 0.0f;
    for (size_t j = 0; j < cols; ++j) {
      float p = xr[j] * xr[j];
      ss = ss + p;
    }
    float mean = ss / (float)cols;
    float rms = sqrtf(mean + eps);
    for (size_t j = 0; j < cols; ++j)
      out[r * cols + j] = (xr[j] / rms) * gamma[j];
  }
  return OK;
}

/* nn::SwiGLU::forward(gate, up): src/nn/swiglu.cpp:10-40. */
void or_swiglu(const float *g, const float *u, size_t n, float *out) {
  for (size_t i = 0; i < n; ++i) {
    float x1 = g[i];
    float silu = x1 / (1.0f + expf(-x1));
    out[i] = silu * u[i];
  }
}

/* nn::Softmax::forward: src/nn/softmax.cpp:13-54.  Max with a strict '>' from
 * -inf, e = expf(x - max) stored, sequential sum, then e / sum. */
void or_softmax(const float *x, size_t rows, size_t cols, float *out) {
  for (size_t r = 0; r < rows; ++r) {
    const float *xr = x + r * cols;
    float *yr = out + r * cols;
    float mx = -INFINITY;
    for (size_t j = 0; j < cols; ++j)
      if (xr[j] > mx)
        mx = xr[j];
    float sum = 0.0f;
    for (size_t j = 0; j < cols; ++j) {
      float e = expf(xr[j] - mx);
      yr[j] = e;
      sum = sum + e;
    }
    for (size_t j = 0; j < cols; ++j)
      yr[j] = yr[j] / sum;
  }
}

/* greedy_sample: src/core/sampler.cpp:13-26.  First index of the maximum under a
 * strict '>' from -inf: NaN is never chosen; all -inf/NaN gives 0. */
int64_t or_argmax(const float *x, size_t n) {
  float mx = -INFINITY;
  int64_t best = 0;
  for (size_t i = 0; i < n; ++i)
    if (x[i] > mx) {
      mx = x[i];
      best = (int64_t)i;
    }
  return best;
}

/* ---- nucleus sampling ----------------------------------------------------------
 * sample_top_p: src/core/sampler.cpp:28-86.  The probabilities are the
 * reference's bit for bit (temperature divide, strict '>' max, expf, a
 * sequential fp32 sum, divide).  The pairs are ordered by descending
 * probability with ties by ascending token id (std::sort leaves ties in an
 * unspecified order).  Two cut points follow, both over exact prefix sums of
 * the masses q = floor(p * 2^62):
 *   cut:  the first position whose prefix mass reaches ceil(top_p * 2^62)
 *         (capped at the total), the reference's `cumulative_prob >= top_p`;
 *   pick: the first position whose prefix mass reaches ceil(u * C), C the
 *         prefix mass through `cut` -- what std::discrete_distribution's
 *         lower_bound over the normalised partial sums selects for the uniform
 *         number u in [0, 1) (the reference draws u from a random_device-seeded
 *         mt19937; here the caller passes it).
 * Outputs: *id, *nucleus = cut + 1, *nucleus_f32 = the prefix length the
 * reference's own fp32 running sum gives, *slack = the smaller distance, in
 * units of the total / of C, from top_p / u to the nearest prefix boundary
 * (how much rounding either cut can absorb; for a top_p above the total, its
 * distance from the total).  Returns 1 for bad arguments,
 * 3 when no probability is finite and positive (then *id = greedy choice). */
typedef struct {
  uint32_t bits;
  uint32_t id;
} or_pb;

static int or_pb_cmp(const void *a, const void *b) {
  const or_pb *x = (const or_pb *)a, *y = (const or_pb *)b;
  if (x->bits != y->bits) return x->bits > y->bits ? -1 : 1;
  return x->id < y->id ? -1 : (x->id > y->id ? 1 : 0);
}

static uint64_t or_qmass(float p) {
  return (p > 0.f && p <= 1.f) ? (uint64_t)((double)p * 4611686018427387904.0) : 0u;
}

/* Probabilities (the reference's bit for bit), ids ordered by descending
 * probability then id, and the exact prefix masses in that order.  Returns
 * the total mass (0: no positive finite probability); *mi = greedy choice. */
typedef struct {
  float *p;
  or_pb *pb;
  uint64_t *cum;
  uint64_t tot;
  size_t mi;
} or_nucleus;

static void or_nucleus_free(or_nucleus *t) { free(t->p), free(t->pb), free(t->cum); }

static int or_nucleus_build(const float *logits, size_t n, float temperature, int accurate_sum, or_nucleus *t) {
  t->p = (float *)malloc(n * sizeof(float));
  t->pb = (or_pb *)malloc(n * sizeof(or_pb));
  t->cum = (uint64_t *)malloc(n * sizeof(uint64_t));
  t->tot = 0;
  t->mi = 0;
  if (!t->p || !t->pb || !t->cum) return E_RUNTIME;
  float *p = t->p, mx = -INFINITY;
  for (size_t i = 0; i < n; ++i) {
    p[i] = logits[i] / temperature;
    if (p[i] > mx) {
      mx = p[i];
      t->mi = i;
    }
  }
  float sum = 0.f;
  double dsum = 0.0;
  for (size_t i = 0; i < n; ++i) {
    p[i] = expf(p[i] - mx);
    sum += p[i];
    dsum += p[i];
  }
  if (accurate_sum) sum = (float)dsum; /* the exact sum rounded once, not the reference's running sum */
  for (size_t i = 0; i < n; ++i) {
    p[i] /= sum;
    uint32_t b = 0u; /* NaN and 0 order last */
    if (p[i] > 0.f) memcpy(&b, &p[i], sizeof b);
    t->pb[i].bits = b;
    t->pb[i].id = (uint32_t)i;
    t->tot += or_qmass(p[i]);
  }
  if (t->tot == 0) return OK;
  qsort(t->pb, n, sizeof(or_pb), or_pb_cmp);
  uint64_t acc = 0;
  for (size_t i = 0; i < n; ++i) {
    acc += or_qmass(p[t->pb[i].id]);
    t->cum[i] = acc;
  }
  return OK;
}

/* The two cut points for (top_p, u); *slack as described above. */
static void or_nucleus_pick(const or_nucleus *t, float top_p, double u, size_t *cut_out, size_t *pick_out,
                            double *slack) {
  const uint64_t *cum = t->cum, tot = t->tot;
  const double tq = ceil((double)top_p * 4611686018427387904.0);
  const uint64_t t1 = !(tq < (double)tot) ? tot : (tq <= 0.0 ? 0u : (uint64_t)tq);
  size_t cut = 0;
  while (cum[cut] < t1) ++cut;
  const uint64_t C = cum[cut];
  const double uu = u > 0.0 ? u : 0.0, tu = ceil(uu * (double)C);
  const uint64_t t2 = !(tu < (double)C) ? C : (uint64_t)tu;
  size_t pick = 0;
  while (cum[pick] < t2) ++pick;
  /* a target capped at the total keeps the cut at the last positive mass however the total rounds */
  const int capped = t1 == tot && tq > (double)tot;
  double s1 = capped ? tq - (double)tot : (double)(cum[cut] - t1);
  double s2 = (double)(cum[pick] - t2);
  if (!capped && cut > 0 && (double)(t1 - cum[cut - 1]) < s1) s1 = (double)(t1 - cum[cut - 1]);
  if (pick > 0 && (double)(t2 - cum[pick - 1]) < s2) s2 = (double)(t2 - cum[pick - 1]);
  s1 /= (double)tot;
  s2 /= (double)C;
  *cut_out = cut;
  *pick_out = pick;
  if (slack) *slack = s1 < s2 ? s1 : s2;
}

int or_sample_top_p(const float *logits, size_t n, float temperature, float top_p, double u,
                    int *id, size_t *nucleus, size_t *nucleus_f32, double *slack) {
  if (n == 0 || n > 0x7FFFFFFFu || !(temperature > 0.f)) return E_INVAL;
  or_nucleus t;
  int st = or_nucleus_build(logits, n, temperature, 0, &t);
  *id = (int)t.mi;
  *nucleus = *nucleus_f32 = 1;
  *slack = 0.0;
  if (st != OK || t.tot == 0) {
    or_nucleus_free(&t);
    return E_RUNTIME;
  }
  size_t cut, pick, nf = n;
  or_nucleus_pick(&t, top_p, u, &cut, &pick, slack);
  float accf = 0.f; /* the reference's own fp32 running sum (sampler.cpp:62-70) */
  for (size_t i = 0; i < n && nf == n; ++i) {
    accf += t.p[t.pb[i].id];
    if (accf >= top_p) nf = i + 1;
  }
  *id = (int)t.pb[pick].id;
  *nucleus = cut + 1;
  *nucleus_f32 = nf;
  or_nucleus_free(&t);
  return OK;
}

/* Every draw reachable when top_p moves by a factor (1 +- rel_p) and u by
 * +- abs_u: how far rounding of the probabilities (the sum's order, exp within
 * a few ulp) can move the two cut points.  The draw's position in the sorted
 * order never decreases as top_p or u grows, so the reachable draws are the
 * positions between the two corner cases.  With accurate_sum the softmax
 * denominator is the exact sum rounded once instead of the reference's fp32
 * running sum (whose own error reaches 5e-4 over 300k terms), for checking a
 * device sum that is accurate to a few ulp.  ids[n] gets those draws, *n_ids
 * their number.  Same return codes as or_sample_top_p. */
int or_sample_top_p_set(const float *logits, size_t n, float temperature, float top_p, double u, double rel_p,
                        double abs_u, int accurate_sum, int *ids, int *n_ids) {
  if (n == 0 || n > 0x7FFFFFFFu || !(temperature > 0.f)) return E_INVAL;
  or_nucleus t;
  int st = or_nucleus_build(logits, n, temperature, accurate_sum, &t);
  *n_ids = 1;
  ids[0] = (int)t.mi;
  if (st != OK || t.tot == 0) {
    or_nucleus_free(&t);
    return E_RUNTIME;
  }
  const double ulo = u - abs_u, uhi = u + abs_u;
  size_t cut, lo, hi;
  or_nucleus_pick(&t, (float)(top_p * (1.0 - rel_p)), ulo < 0.0 ? 0.0 : ulo, &cut, &lo, NULL);
  or_nucleus_pick(&t, (float)(top_p * (1.0 + rel_p)), uhi >= 1.0 ? 0.9999999999 : uhi, &cut, &hi, NULL);
  *n_ids = 0;
  for (size_t k = lo; k <= hi; ++k) ids[(*n_ids)++] = (int)t.pb[k].id;
  or_nucleus_free(&t);
  return OK;
}

/* ---- RoPE --------------------------------------------------------------------- */

/* RoPE constructor tables: src/nn/rope.cpp:16-32. */
void or_rope_tables(size_t head_dim, size_t max_seq, float theta, float *cos_t, float *sin_t) {
  size_t half = head_dim / 2;
  for (size_t pos = 0; pos < max_seq; ++pos)
    for (size_t i = 0; i < half; ++i) {
      float theta_i = powf(theta, -(float)(2 * i) / (float)head_dim);
      float freq = (float)pos * theta_i;
      cos_t[pos * half + i] = cosf(freq);
      sin_t[pos * half + i] = sinf(freq);
    }
}

/* RoPE::apply_in_place: src/nn/rope.cpp:35-103.  Rotate-half pairs (i, i+half)
 * of a rank-2 [S, D] or rank-4 [B, H, S, D] strided view, in place.  The
 * reference build fuses both rotations:
 *   y0 = fma(x0, c, -(x1*s)),  y1 = fma(x0, s, x1*c).
 * Positions past the table raise out_of_range (checked before any write here). */
int or_rope(float *base, const or_view *x, size_t head_dim, size_t max_seq,
            const float *cos_t, const float *sin_t, size_t pos_offset) {
  if (x->rank == 0 || (size_t)x->shape[x->rank - 1] != head_dim)
    return E_INVAL;
  if (x->rank != 2 && x->rank != 4)
    return E_INVAL;
  size_t half = head_dim / 2;
  int64_t B = x->rank == 4 ? x->shape[0] : 1;
  int64_t H = x->rank == 4 ? x->shape[1] : 1;
  int64_t S = x->shape[x->rank - 2];
  if (S > 0 && B > 0 && pos_offset + (size_t)S - 1 >= max_seq)
    return E_RANGE;
  int64_t sb = x->rank == 4 ? x->strides[0] : 0;
  int64_t sh = x->rank == 4 ? x->strides[1] : 0;
  int64_t ss = x->strides[x->rank - 2];
  int64_t sd = x->strides[x->rank - 1];
  for (int64_t b = 0; b < B; ++b)
    for (int64_t p = 0; p < S; ++p)
      for (int64_t h = 0; h < H; ++h)
        for (size_t i = 0; i < half; ++i) {
          size_t ci = (pos_offset + (size_t)p) * half + i;
          float c = cos_t[ci], s = sin_t[ci];
          int64_t o = x->offset + b * sb + h * sh + p * ss;
          float *p0 = base + o + (int64_t)i * sd;
          float *p1 = base + o + (int64_t)(i + half) * sd;
          float x0 = *p0, x1 = *p1;
          *p0 = fmaf(x0, c, -(x1 * s));
          *p1 = fmaf(x0, s, x1 * c);
        }
  return OK;
}

/* ---- Embedding ------------------------------------------------------------------ */

/* nn::Embedding::forward: src/nn/embedding.cpp:22-118.  Weight of GGUF logical
 * shape {dim, vocab}; dtype 0 FP32 (column gather), 2 Q8_0, 3 Q4_0 (row
 * dequant).  ids are fp32-stored; id >= vocab raises out_of_range. */
int or_embedding(const uint8_t *w, int dtype, size_t dim, size_t vocab, const float *ids,
                 size_t n, float *out) {
  for (size_t t = 0; t < n; ++t) {
    size_t id = (size_t)ids[t];
    if (id >= vocab)
      return E_RANGE;
    float *o = out + t * dim;
    if (dtype == 0) {
      const float *wf = (const float *)w;
      for (size_t d = 0; d < dim; ++d)
        o[d] = wf[d * vocab + id];
    } else if (dtype == 2) {
      or_dequant_q8_0(w + id * (dim / 32 * 34), dim / 32, o);
    } else if (dtype == 3) {
      or_dequant_q4_0(w + id * (dim / 32 * 18), dim / 32, o);
    } else {
      return E_RUNTIME;
    }
  }
  return OK;
}

/* ---- fp32 matmul ------------------------------------------------------------------ */

/* Tensor::matmul fp32 branch: src/tensor/tensor.cpp:434-542.  Batched strided
 * GEMM; every C element is an FMA chain over k in increasing order from 0. */
int or_matmul_f32(const or_view *a, const or_view *b, float *out) {
  int r = a->rank;
  if (r < 2 || b->rank < 2)
    return E_INVAL;
  if (b->rank != r)
    return E_INVAL;
  int64_t batch = 1;
  for (int i = 0; i < r - 2; ++i) {
    if (a->shape[i] != b->shape[i])
      return E_INVAL;
    batch *= a->shape[i];
  }
  int64_t M = a->shape[r - 2], K = a->shape[r - 1], N = b->shape[r - 1];
  if (K != b->shape[r - 2])
    return E_INVAL;
  for (int64_t bi = 0; bi < batch; ++bi) {
    int64_t ao = a->offset, bo = b->offset, t = bi;
    for (int d = r - 3; d >= 0; --d) {
      int64_t idx = t % a->shape[d];
      t /= a->shape[d];
      ao += idx * a->strides[d];
      bo += idx * b->strides[d];
    }
    for (int64_t i = 0; i < M; ++i)
      for (int64_t j = 0; j < N; ++j) {
        float c = 0.0f;
        for (int64_t k = 0; k < K; ++k)
          c = fmaf(a->base[ao + i * a->strides[r - 2] + k * a->strides[r - 1]],
                   b->base[bo + k * b->strides[r - 2] + j * b->strides[r - 1]], c);
        out[(bi * M + i) * N + j] = c;
      }
  }
  return OK;
}
