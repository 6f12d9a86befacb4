// tb_rope.cu -- rotate-half RoPE in place on strided views (A13).
//
// The cos/sin tables are the RoPE constructor's (src/nn/rope.cpp:16-32),
// computed once on the host with the same libm calls and uploaded, so the
// rotation below reproduces the reference bit for bit: the reference build
// fuses both rotations into FMAs,
//   y0 = fma(x0, c, -(x1 * s)),   y1 = fma(x0, s, x1 * c)   (rope.cpp:73-74).
#include <algorithm>

#include "tb_internal.cuh"

namespace tb {
namespace {

struct RopeView {
  int64_t B, H, S, half;
  int64_t sb, sh, ss, sd, off;
};

__global__ void __launch_bounds__(256) rope_kernel(float *__restrict__ x, RopeView v,
                                                   const float *__restrict__ cos_t,
                                                   const float *__restrict__ sin_t,
                                                   int64_t pos_offset, const int32_t *__restrict__ pos_dev,
                                                   int64_t max_seq, uint32_t *__restrict__ err) {
  if (pos_dev) {  // position held in device memory (a captured decode step)
    pos_offset = *pos_dev;
    if (pos_offset < 0 || pos_offset + v.S > max_seq) {
      if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(err, ERR_INDEX);
      return;
    }
  }
  const int64_t total = v.B * v.H * v.S * v.half;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    int64_t i = t % v.half;
    int64_t r = t / v.half;
    int64_t h = r % v.H;
    r /= v.H;
    int64_t p = r % v.S;
    int64_t b = r / v.S;
    int64_t ci = (pos_offset + p) * v.half + i;
    float c = __ldg(cos_t + ci), s = __ldg(sin_t + ci);
    int64_t o = v.off + b * v.sb + h * v.sh + p * v.ss;
    float *p0 = x + o + i * v.sd;
    float *p1 = x + o + (i + v.half) * v.sd;
    float x0 = *p0, x1 = *p1;
    *p0 = __fmaf_rn(x0, c, -__fmul_rn(x1, s));
    *p1 = __fmaf_rn(x0, s, __fmul_rn(x1, c));
  }
}

__global__ void fill_upper_kernel(float *__restrict__ x, int64_t rows, int64_t cols, int64_t ld,
                                  int64_t diag, float value) {
  const int64_t total = rows * cols;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = t / cols, c = t % cols;
    if (c > r + diag) x[r * ld + c] = value;
  }
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" tb_status tb_fill_upper(float *x, int64_t rows, int64_t cols, int64_t ld, int64_t diag,
                                   float value, tb_stream stream) {
  if (rows < 0 || cols < 0 || ld < cols) return fail(TB_EINVAL, "tb_fill_upper: bad extents");
  if (rows == 0 || cols == 0) return TB_OK;
  if (!x) return fail(TB_EINVAL, "tb_fill_upper: null pointer");
  DeviceState *st;
  TB_TRY(device_state(&st));
  const int64_t total = rows * cols;
  const int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)st->sm_count * 8);
  fill_upper_kernel<<<grid, 256, 0, as_stream(stream)>>>(x, rows, cols, ld, diag, value);
  return check_launch("tb_fill_upper");
}

namespace {
tb_status rope_launch(const tb_view *x, const float *cos_t, const float *sin_t, int64_t head_dim,
                      int64_t max_seq, int64_t pos_offset, const int32_t *pos_dev, tb_stream stream) {
  TB_TRY(validate_view(x, "tb_rope x"));
  if (x->dtype != TB_F32) return fail(TB_EINVAL, "tb_rope: fp32 only");
  if (head_dim <= 0 || head_dim % 2 != 0) return fail(TB_EINVAL, "RoPE requires an even head dimension.");
  if (x->rank == 0 || x->shape[x->rank - 1] != head_dim)
    return fail(TB_EINVAL, "Tensor last dimension must match RoPE head_dim.");
  if (x->rank != 2 && x->rank != 4)
    return fail(TB_EINVAL, "RoPE apply_in_place currently supports 2D or 4D tensors.");
  if (pos_offset < 0) return fail(TB_EINVAL, "tb_rope: negative position offset");
  RopeView v;
  v.half = head_dim / 2;
  if (x->rank == 4) {
    v.B = x->shape[0]; v.H = x->shape[1]; v.S = x->shape[2];
    v.sb = x->strides[0]; v.sh = x->strides[1]; v.ss = x->strides[2]; v.sd = x->strides[3];
  } else {
    v.B = 1; v.H = 1; v.S = x->shape[0];
    v.sb = 0; v.sh = 0; v.ss = x->strides[0]; v.sd = x->strides[1];
  }
  v.off = x->offset;
  // rope.cpp:58-61 / 81-84: a position at or past the table raises out_of_range
  // (checked on the device when the position lives there).
  if (!pos_dev && v.B > 0 && v.S > 0 && pos_offset + v.S > max_seq)
    return fail(TB_ERANGE, "Sequence position exceeds RoPE cache size.");
  int64_t total = v.B * v.H * v.S * v.half;
  if (total == 0) return TB_OK;
  if (!cos_t || !sin_t) return fail(TB_EINVAL, "tb_rope: null table");
  DeviceState *st;
  TB_TRY(device_state(&st));
  int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)st->sm_count * 8);
  rope_kernel<<<grid, 256, 0, as_stream(stream)>>>(static_cast<float *>(x->data), v, cos_t, sin_t, pos_offset,
                                                   pos_dev, max_seq, st->err_word);
  return check_launch("tb_rope");
}
}  // namespace

extern "C" tb_status tb_rope(const tb_view *x, const float *cos_t, const float *sin_t,
                             int64_t head_dim, int64_t max_seq, int64_t pos_offset,
                             tb_stream stream) {
  return rope_launch(x, cos_t, sin_t, head_dim, max_seq, pos_offset, nullptr, stream);
}

extern "C" tb_status tb_rope_at(const tb_view *x, const float *cos_t, const float *sin_t, int64_t head_dim,
                                int64_t max_seq, const int32_t *pos_dev, tb_stream stream) {
  if (!pos_dev) return fail(TB_EINVAL, "tb_rope_at: null position");
  return rope_launch(x, cos_t, sin_t, head_dim, max_seq, 0, pos_dev, stream);
}
