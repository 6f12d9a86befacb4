// tb_elementwise.cu -- broadcast binary ops, scalar multiply, strided copy and
// SwiGLU (rows A3, A4, A5, A6, A8 of the hot path).
//
// All of these are HBM-bound.  The kernels read and write 16 bytes per access
// where the views allow it (contiguous and 16-byte aligned), keep several
// accesses in flight per thread, and size grids as a multiple of the SM count.
// Non-contiguous views go through a merged-dimension index walk; a broadcast
// operand whose only varying dims are the innermost ones (a row vector) keeps
// the vectorised path.
#include <algorithm>

#include "tb_internal.cuh"

namespace tb {
namespace {

constexpr int kThreads = 256;

// --------------------------------------------------------------------------
// Index walk over up to TB_MAX_RANK merged dimensions for three operands.
struct Walk3 {
  int rank;
  int64_t shape[TB_MAX_RANK];
  int64_t s0[TB_MAX_RANK];  // output (or dst) strides
  int64_t s1[TB_MAX_RANK];
  int64_t s2[TB_MAX_RANK];
  int64_t o0, o1, o2;  // base offsets (elements)
};

// Drops extent-1 dims and merges neighbours that are contiguous for every
// operand, so that most views collapse to one or two dims.
void merge_dims(Walk3 &w, int nops) {
  int r = 0;
  int64_t sh[TB_MAX_RANK], a[TB_MAX_RANK], b[TB_MAX_RANK], c[TB_MAX_RANK];
  for (int i = 0; i < w.rank; ++i) {
    if (w.shape[i] == 1) continue;
    sh[r] = w.shape[i];
    a[r] = w.s0[i];
    b[r] = w.s1[i];
    c[r] = nops > 2 ? w.s2[i] : 0;
    ++r;
  }
  int m = 0;
  for (int i = 0; i < r; ++i) {
    if (m > 0) {
      int j = m - 1;
      bool ok = a[j] == a[i] * sh[i] && b[j] == b[i] * sh[i] && (nops < 3 || c[j] == c[i] * sh[i]);
      if (ok) {
        sh[j] *= sh[i];
        a[j] = a[i];
        b[j] = b[i];
        c[j] = c[i];
        continue;
      }
    }
    sh[m] = sh[i];
    a[m] = a[i];
    b[m] = b[i];
    c[m] = c[i];
    ++m;
  }
  if (m == 0) {  // a single element
    sh[0] = 1;
    a[0] = b[0] = c[0] = 1;
    m = 1;
  }
  w.rank = m;
  for (int i = 0; i < m; ++i) {
    w.shape[i] = sh[i];
    w.s0[i] = a[i];
    w.s1[i] = b[i];
    w.s2[i] = c[i];
  }
}

template <typename T> struct Vec;
template <> struct Vec<float> {
  static constexpr int N = 4;
};
template <> struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
};

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

template <int OP> __device__ __forceinline__ float apply(float a, float b) {
  if (OP == 0) return __fadd_rn(a, b);
  return __fmul_rn(a, b);
}

// ---- contiguous, 16-byte aligned: out = a OP b -----------------------------
template <typename T, int OP>
__global__ void __launch_bounds__(kThreads) binary_flat_kernel(const T *__restrict__ a,
                                                               const T *__restrict__ b,
                                                               T *__restrict__ out, int64_t n) {
  constexpr int V = Vec<T>::N;
  const int64_t nvec = n / V;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const uint4 *av = reinterpret_cast<const uint4 *>(a);
  const uint4 *bv = reinterpret_cast<const uint4 *>(b);
  uint4 *ov = reinterpret_cast<uint4 *>(out);
  // Two 16-byte loads per operand in flight per iteration.
  for (; i + stride < nvec; i += 2 * stride) {
    uint4 x0 = __ldcs(av + i), y0 = __ldcs(bv + i);
    uint4 x1 = __ldcs(av + i + stride), y1 = __ldcs(bv + i + stride);
    const T *xa = reinterpret_cast<const T *>(&x0), *ya = reinterpret_cast<const T *>(&y0);
    const T *xb = reinterpret_cast<const T *>(&x1), *yb = reinterpret_cast<const T *>(&y1);
    uint4 r0, r1;
    T *ra = reinterpret_cast<T *>(&r0), *rb = reinterpret_cast<T *>(&r1);
#pragma unroll
    for (int k = 0; k < V; ++k) {
      ra[k] = from_f<T>(apply<OP>(to_f(xa[k]), to_f(ya[k])));
      rb[k] = from_f<T>(apply<OP>(to_f(xb[k]), to_f(yb[k])));
    }
    __stcs(ov + i, r0);
    __stcs(ov + i + stride, r1);
  }
  for (; i < nvec; i += stride) {
    uint4 x0 = __ldcs(av + i), y0 = __ldcs(bv + i);
    const T *xa = reinterpret_cast<const T *>(&x0), *ya = reinterpret_cast<const T *>(&y0);
    uint4 r0;
    T *ra = reinterpret_cast<T *>(&r0);
#pragma unroll
    for (int k = 0; k < V; ++k) ra[k] = from_f<T>(apply<OP>(to_f(xa[k]), to_f(ya[k])));
    __stcs(ov + i, r0);
  }
  // tail elements
  int64_t t = nvec * V + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t < n) out[t] = from_f<T>(apply<OP>(to_f(a[t]), to_f(b[t])));
}

// ---- a contiguous [rows, inner], b a row vector [inner] (stride-0 rows) -----
template <typename T, int OP>
__global__ void __launch_bounds__(kThreads) binary_rowvec_kernel(const T *__restrict__ a,
                                                                 const T *__restrict__ b,
                                                                 T *__restrict__ out, int64_t n,
                                                                 int64_t inner, int b_first) {
  constexpr int V = Vec<T>::N;
  const int64_t nvec = n / V;
  const int64_t innerv = inner / V;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const uint4 *av = reinterpret_cast<const uint4 *>(a);
  const uint4 *bv = reinterpret_cast<const uint4 *>(b);
  uint4 *ov = reinterpret_cast<uint4 *>(out);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    uint4 x0 = __ldcs(av + i), y0 = __ldg(bv + (i % innerv));
    const T *xa = reinterpret_cast<const T *>(&x0), *ya = reinterpret_cast<const T *>(&y0);
    uint4 r0;
    T *ra = reinterpret_cast<T *>(&r0);
#pragma unroll
    for (int k = 0; k < V; ++k)
      ra[k] = b_first ? from_f<T>(apply<OP>(to_f(ya[k]), to_f(xa[k])))
                      : from_f<T>(apply<OP>(to_f(xa[k]), to_f(ya[k])));
    __stcs(ov + i, r0);
  }
}

// ---- general strided: out[walk] = a[walk] OP b[walk] --------------------------
template <typename T, int OP>
__global__ void __launch_bounds__(kThreads) binary_strided_kernel(const T *__restrict__ a,
                                                                  const T *__restrict__ b,
                                                                  T *__restrict__ out,
                                                                  int64_t n, Walk3 w) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t rem = i, oo = w.o0, oa = w.o1, ob = w.o2;
    for (int d = w.rank - 1; d >= 0; --d) {
      int64_t idx = rem % w.shape[d];
      rem /= w.shape[d];
      oo += idx * w.s0[d];
      oa += idx * w.s1[d];
      ob += idx * w.s2[d];
    }
    out[oo] = from_f<T>(apply<OP>(to_f(a[oa]), to_f(b[ob])));
  }
}

// ---- scale ----------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) scale_flat_kernel(const float *__restrict__ x,
                                                              float *__restrict__ out, int64_t n,
                                                              float s) {
  const int64_t nvec = n / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const float4 *xv = reinterpret_cast<const float4 *>(x);
  float4 *ov = reinterpret_cast<float4 *>(out);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    float4 v = __ldcs(xv + i);
    v.x = __fmul_rn(v.x, s);
    v.y = __fmul_rn(v.y, s);
    v.z = __fmul_rn(v.z, s);
    v.w = __fmul_rn(v.w, s);
    __stcs(ov + i, v);
  }
  int64_t t = nvec * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t < n) out[t] = __fmul_rn(x[t], s);
}

__global__ void __launch_bounds__(kThreads) scale_strided_kernel(const float *__restrict__ x,
                                                                 float *__restrict__ out,
                                                                 int64_t n, float s, Walk3 w) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t rem = i, oo = w.o0, ox = w.o1;
    for (int d = w.rank - 1; d >= 0; --d) {
      int64_t idx = rem % w.shape[d];
      rem /= w.shape[d];
      oo += idx * w.s0[d];
      ox += idx * w.s1[d];
    }
    out[oo] = __fmul_rn(x[ox], s);
  }
}

// ---- copy -------------------------------------------------------------------
// 16-byte vector copy of a contiguous range.
__global__ void __launch_bounds__(kThreads) copy_flat16_kernel(const uint4 *__restrict__ src,
                                                               uint4 *__restrict__ dst,
                                                               int64_t nvec) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + stride < nvec; i += 2 * stride) {
    uint4 a = __ldcs(src + i), b = __ldcs(src + i + stride);
    __stcs(dst + i, a);
    __stcs(dst + i + stride, b);
  }
  for (; i < nvec; i += stride) __stcs(dst + i, __ldcs(src + i));
}

template <typename T>
__global__ void __launch_bounds__(kThreads) copy_strided_kernel(const T *__restrict__ src,
                                                                T *__restrict__ dst, int64_t n,
                                                                Walk3 w) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t rem = i, od = w.o0, os = w.o1;
    for (int d = w.rank - 1; d >= 0; --d) {
      int64_t idx = rem % w.shape[d];
      rem /= w.shape[d];
      od += idx * w.s0[d];
      os += idx * w.s1[d];
    }
    dst[od] = src[os];
  }
}

// Transposing copy of the innermost two dims through shared memory: a tile of
// 32x32 elements is read along the source's unit-stride dim and written along
// the destination's, so both sides stay coalesced.  Used when the source's
// unit-stride dim is not the destination's (e.g. contiguous() of a transposed
// view, attention.cpp:144-145).
template <typename T, int TILE>
__global__ void __launch_bounds__(256) copy_transpose_kernel(const T *__restrict__ src,
                                                             T *__restrict__ dst, int64_t outer,
                                                             int64_t R, int64_t C, Walk3 w) {
  // Logical element (o, r, c): dst at w.o0 + o..., r*w.s0[R] + c*w.s0[C]; the
  // source has unit stride along r (dim rank-2) and the dst along c (rank-1).
  // TILE x TILE tiles; TILE consecutive threads run along the unit-stride axis
  // of each side, and every thread has TILE*TILE/256 loads in flight before
  // the tile is turned around in shared memory.
  constexpr int TY = 256 / TILE, PER = TILE / TY;
  __shared__ T tile[TILE][TILE + 1];
  const int rd = w.rank - 2, cd = w.rank - 1;
  const int tx = threadIdx.x % TILE, ty = threadIdx.x / TILE;
  const int64_t sc = w.s1[cd], dr = w.s0[rd];
  const int64_t tiles_c = (C + TILE - 1) / TILE, tiles_r = (R + TILE - 1) / TILE;
  const int64_t per_outer = tiles_r * tiles_c, tiles = outer * per_outer;
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int64_t o = t / per_outer, rem = t - o * per_outer;
    const int64_t r0 = (rem / tiles_c) * TILE, c0 = (rem % tiles_c) * TILE;
    int64_t od = w.o0, os = w.o1, ro = o;
    for (int d = w.rank - 3; d >= 0; --d) {
      const int64_t idx = ro % w.shape[d];
      ro /= w.shape[d];
      od += idx * w.s0[d];
      os += idx * w.s1[d];
    }
    T v[PER];
    {
      const int64_t r = r0 + tx;
      const T *sp = src + os + r;  // src unit stride along r
#pragma unroll
      for (int k = 0; k < PER; ++k) {
        const int64_t c = c0 + ty + k * TY;
        v[k] = (r < R && c < C) ? sp[c * sc] : T(0);
      }
    }
#pragma unroll
    for (int k = 0; k < PER; ++k) tile[ty + k * TY][tx] = v[k];
    __syncthreads();
    {
      const int64_t c = c0 + tx;
      T *dp = dst + od + c;  // dst unit stride along c
#pragma unroll
      for (int k = 0; k < PER; ++k) {
        const int64_t r = r0 + ty + k * TY;
        if (r < R && c < C) dp[r * dr] = tile[tx][ty + k * TY];
      }
    }
    __syncthreads();
  }
}

// 16-bit elements, TR x 64 tiles (TR rows along the source's unit stride)
// moved as 32-bit pairs on both sides: a thread loads pairs (r, r+1) of one
// column, the tile is turned around in shared memory, and a thread stores the
// pair (c, c+1) of one row (unit stride along c in the destination).  With
// TR = 128 each thread has 64 bytes of loads in flight, as the fp32 tile does.
// Needs even extents, strides and offsets and 4-byte aligned bases (checked
// by the host).
template <int TR>
__global__ void __launch_bounds__(256) copy_transpose16_kernel(const uint16_t *__restrict__ src,
                                                               uint16_t *__restrict__ dst, int64_t outer,
                                                               int64_t R, int64_t C, Walk3 w) {
  constexpr int TC = 64, TY = 8, PC = TC / TY, PR = TR / 64;  // PR pairs-of-32-threads along r
  __shared__ __align__(4) uint16_t tile[TR][TC + 2];  // [r][c]; a 33-word pitch
  const int rd = w.rank - 2, cd = w.rank - 1;
  const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;
  const int64_t sc = w.s1[cd], dr = w.s0[rd];
  const int64_t tiles_c = (C + TC - 1) / TC, tiles_r = (R + TR - 1) / TR;
  const int64_t per_outer = tiles_r * tiles_c, tiles = outer * per_outer;
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int64_t o = t / per_outer, rem = t - o * per_outer;
    const int64_t r0 = (rem / tiles_c) * TR, c0 = (rem % tiles_c) * TC;
    int64_t od = w.o0, os = w.o1, ro = o;
    for (int d = w.rank - 3; d >= 0; --d) {
      const int64_t idx = ro % w.shape[d];
      ro /= w.shape[d];
      od += idx * w.s0[d];
      os += idx * w.s1[d];
    }
    uint32_t v[PR][PC];
#pragma unroll
    for (int p = 0; p < PR; ++p) {
      const int64_t r = r0 + 64 * p + 2 * tx;
      const uint16_t *sp = src + os + r;
#pragma unroll
      for (int k = 0; k < PC; ++k) {
        const int64_t c = c0 + ty + k * TY;
        v[p][k] = (r < R && c < C) ? *reinterpret_cast<const uint32_t *>(sp + c * sc) : 0u;
      }
    }
#pragma unroll
    for (int p = 0; p < PR; ++p)
#pragma unroll
      for (int k = 0; k < PC; ++k) {
        tile[64 * p + 2 * tx][ty + k * TY] = (uint16_t)(v[p][k] & 0xFFFFu);
        tile[64 * p + 2 * tx + 1][ty + k * TY] = (uint16_t)(v[p][k] >> 16);
      }
    __syncthreads();
    {
      const int64_t c = c0 + 2 * tx;
      uint16_t *dp = dst + od + c;
#pragma unroll
      for (int k = 0; k < TR / TY; ++k) {
        const int rl = ty + k * TY;
        const int64_t r = r0 + rl;
        if (r < R && c < C) *reinterpret_cast<uint32_t *>(dp + r * dr) = *reinterpret_cast<const uint32_t *>(&tile[rl][2 * tx]);
      }
    }
    __syncthreads();
  }
}

// ---- SwiGLU -----------------------------------------------------------------
// silu(g) * u with silu(g) = g / (1 + exp(-g)) (src/nn/swiglu.cpp:25-31): the
// division and products are IEEE-rounded as in the reference; exp is the
// correctly rounding exp_cr (the reference's glibc expf is too, but on ~0.03%
// of inputs).
__device__ __forceinline__ float swiglu1(float g, float u, const double *tab) { return swiglu_f32(g, u, tab); }
__device__ __forceinline__ float swiglu1_bf16(float g, float u) {
  float e = __expf(-g);  // bf16 results: fp32 exp is far below the output rounding
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, e)), u);
}

template <typename T>
__device__ __forceinline__ uint4 swiglu_vec(const uint4 a, const uint4 b, const double *tab) {
  constexpr int V = Vec<T>::N;
  const T *ga = reinterpret_cast<const T *>(&a), *ub = reinterpret_cast<const T *>(&b);
  uint4 r;
  T *rr = reinterpret_cast<T *>(&r);
#pragma unroll
  for (int k = 0; k < V; ++k) {
    const float gf = to_f(ga[k]), uf = to_f(ub[k]);
    rr[k] = from_f<T>(sizeof(T) == 4 ? swiglu1(gf, uf, tab) : swiglu1_bf16(gf, uf));
  }
  return r;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) swiglu_kernel(const T *__restrict__ g,
                                                          const T *__restrict__ u,
                                                          T *__restrict__ y, int64_t n,
                                                          int vec_ok) {
  constexpr int V = Vec<T>::N;
  __shared__ double tab[64];
  exp_cr_table_init(tab);
  __syncthreads();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t base = 0;
  if (vec_ok) {
    const int64_t nvec = n / V;
    const uint4 *gv = reinterpret_cast<const uint4 *>(g);
    const uint4 *uv = reinterpret_cast<const uint4 *>(u);
    uint4 *yv = reinterpret_cast<uint4 *>(y);
    // two vectors per thread per step: four 16-byte loads in flight
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + stride < nvec; i += 2 * stride) {
      const uint4 a0 = __ldcs(gv + i), b0 = __ldcs(uv + i);
      const uint4 a1 = __ldcs(gv + i + stride), b1 = __ldcs(uv + i + stride);
      __stcs(yv + i, swiglu_vec<T>(a0, b0, tab));
      __stcs(yv + i + stride, swiglu_vec<T>(a1, b1, tab));
    }
    if (i < nvec) __stcs(yv + i, swiglu_vec<T>(__ldcs(gv + i), __ldcs(uv + i), tab));
    base = nvec * V;
  }
  for (int64_t i = base + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float gf = to_f(g[i]), uf = to_f(u[i]);
    y[i] = from_f<T>(sizeof(T) == 4 ? swiglu1(gf, uf, tab) : swiglu1_bf16(gf, uf));
  }
}

// ---- host helpers --------------------------------------------------------------

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Broadcast shape per Tensor::compute_broadcast_shape (src/tensor/tensor.cpp:29-47).
tb_status broadcast_shape(const tb_view *a, const tb_view *b, int64_t *out, int *rank) {
  int r = std::max(a->rank, b->rank);
  for (int k = 0; k < r; ++k) {
    int i = a->rank - 1 - k, j = b->rank - 1 - k;
    int64_t d1 = i >= 0 ? a->shape[i] : 1, d2 = j >= 0 ? b->shape[j] : 1;
    if (d1 != d2 && d1 != 1 && d2 != 1) return fail(TB_EINVAL, "Shapes are not broadcastable.");
    out[r - 1 - k] = std::max(d1, d2);
  }
  *rank = r;
  return TB_OK;
}

// Strides of `v` broadcast to `shape` (Tensor::broadcast_to, tensor.cpp:232-256).
void broadcast_strides(const tb_view *v, const int64_t *shape, int rank, int64_t *st) {
  int diff = rank - v->rank;
  for (int i = 0; i < rank; ++i) {
    if (i < diff) {
      st[i] = 0;
    } else {
      int64_t s = v->shape[i - diff];
      st[i] = (s == shape[i]) ? v->strides[i - diff] : 0;
    }
  }
}

template <typename T, int OP>
tb_status launch_binary(const tb_view *a, const tb_view *b, const tb_view *out, const int64_t *shape,
                        int rank, cudaStream_t s, const DeviceState *st) {
  const int64_t n = numel(out);
  if (n == 0) return TB_OK;
  const T *pa = static_cast<const T *>(a->data) + a->offset;
  const T *pb = static_cast<const T *>(b->data) + b->offset;
  T *po = static_cast<T *>(out->data) + out->offset;
  constexpr int V = Vec<T>::N;
  Walk3 w;
  w.rank = rank;
  for (int i = 0; i < rank; ++i) w.shape[i] = shape[i];
  broadcast_strides(out, shape, rank, w.s0);
  broadcast_strides(a, shape, rank, w.s1);
  broadcast_strides(b, shape, rank, w.s2);
  w.o0 = w.o1 = w.o2 = 0;
  merge_dims(w, 3);
  bool out_c = w.rank == 1 && w.s0[0] == 1;
  if (out_c && w.s1[0] == 1 && w.s2[0] == 1 && aligned16(pa) && aligned16(pb) && aligned16(po)) {
    binary_flat_kernel<T, OP><<<wave_grid(binary_flat_kernel<T, OP>, kThreads, n / V / 2 + 1, st->sm_count), kThreads, 0, s>>>(pa, pb, po, n);
    return check_launch("tb_binary");
  }
  // row-vector broadcast: [rows, inner] with one side stride-0 over rows
  if (w.rank == 2 && w.s0[0] == w.shape[1] && w.s0[1] == 1 && w.shape[1] % V == 0 &&
      aligned16(pa) && aligned16(pb) && aligned16(po)) {
    bool a_full = w.s1[0] == w.shape[1] && w.s1[1] == 1;
    bool b_full = w.s2[0] == w.shape[1] && w.s2[1] == 1;
    bool a_row = w.s1[0] == 0 && w.s1[1] == 1;
    bool b_row = w.s2[0] == 0 && w.s2[1] == 1;
    if (a_full && b_row) {
      binary_rowvec_kernel<T, OP><<<wave_grid(binary_rowvec_kernel<T, OP>, kThreads, n / V, st->sm_count), kThreads, 0, s>>>(pa, pb, po, n, w.shape[1], 0);
      return check_launch("tb_binary");
    }
    if (b_full && a_row) {
      binary_rowvec_kernel<T, OP><<<wave_grid(binary_rowvec_kernel<T, OP>, kThreads, n / V, st->sm_count), kThreads, 0, s>>>(pb, pa, po, n, w.shape[1], 1);
      return check_launch("tb_binary");
    }
  }
  binary_strided_kernel<T, OP><<<wave_grid(binary_strided_kernel<T, OP>, kThreads, n, st->sm_count), kThreads, 0, s>>>(pa, pb, po, n, w);
  return check_launch("tb_binary");
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" {

tb_status tb_binary(int op, const tb_view *a, const tb_view *b, const tb_view *out, tb_stream stream) {
  TB_TRY(validate_view(a, "tb_binary a"));
  TB_TRY(validate_view(b, "tb_binary b"));
  TB_TRY(validate_view(out, "tb_binary out"));
  if (op != 0 && op != 1) return fail(TB_EINVAL, "tb_binary: op %d (0 add, 1 mul)", op);
  int dt = a->dtype;
  if (b->dtype != dt || out->dtype != dt || (dt != TB_F32 && dt != TB_BF16))
    return fail(TB_EINVAL, "tb_binary: dtypes must all be TB_F32 or all TB_BF16");
  int64_t shape[TB_MAX_RANK];
  int rank = 0;
  TB_TRY(broadcast_shape(a, b, shape, &rank));
  if (out->rank != rank) return fail(TB_EINVAL, "tb_binary: out rank %d, broadcast rank %d", out->rank, rank);
  for (int i = 0; i < rank; ++i)
    if (out->shape[i] != shape[i]) return fail(TB_EINVAL, "tb_binary: out shape is not the broadcast shape");
  if (!is_contiguous(out)) return fail(TB_EINVAL, "tb_binary: out must be contiguous");
  DeviceState *st;
  TB_TRY(device_state(&st));
  cudaStream_t s = as_stream(stream);
  if (dt == TB_F32)
    return op == 0 ? launch_binary<float, 0>(a, b, out, shape, rank, s, st)
                   : launch_binary<float, 1>(a, b, out, shape, rank, s, st);
  return op == 0 ? launch_binary<__nv_bfloat16, 0>(a, b, out, shape, rank, s, st)
                 : launch_binary<__nv_bfloat16, 1>(a, b, out, shape, rank, s, st);
}

tb_status tb_scale(const tb_view *x, float sc, const tb_view *out, tb_stream stream) {
  TB_TRY(validate_view(x, "tb_scale x"));
  TB_TRY(validate_view(out, "tb_scale out"));
  if (x->dtype != TB_F32 || out->dtype != TB_F32) return fail(TB_EINVAL, "tb_scale: fp32 only");
  if (out->rank != x->rank) return fail(TB_EINVAL, "tb_scale: rank mismatch");
  for (int i = 0; i < x->rank; ++i)
    if (out->shape[i] != x->shape[i]) return fail(TB_EINVAL, "tb_scale: shape mismatch");
  if (!is_contiguous(out)) return fail(TB_EINVAL, "tb_scale: out must be contiguous");
  int64_t n = numel(x);
  if (n == 0) return TB_OK;
  DeviceState *st;
  TB_TRY(device_state(&st));
  cudaStream_t s = as_stream(stream);
  const float *px = static_cast<const float *>(x->data) + x->offset;
  float *po = static_cast<float *>(out->data) + out->offset;
  if (is_contiguous(x) && aligned16(px) && aligned16(po)) {
    scale_flat_kernel<<<wave_grid(scale_flat_kernel, kThreads, n / 4 + 1, st->sm_count), kThreads, 0, s>>>(px, po, n, sc);
    return check_launch("tb_scale");
  }
  Walk3 w;
  w.rank = x->rank;
  for (int i = 0; i < x->rank; ++i) {
    w.shape[i] = x->shape[i];
    w.s0[i] = out->strides[i];
    w.s1[i] = x->strides[i];
    w.s2[i] = 0;
  }
  w.o0 = w.o1 = w.o2 = 0;
  merge_dims(w, 2);
  scale_strided_kernel<<<wave_grid(scale_strided_kernel, kThreads, n, st->sm_count), kThreads, 0, s>>>(px, po, n, sc, w);
  return check_launch("tb_scale");
}

tb_status tb_copy(const tb_view *dst, const tb_view *src, tb_stream stream) {
  TB_TRY(validate_view(dst, "tb_copy dst"));
  TB_TRY(validate_view(src, "tb_copy src"));
  // Tensor::copy_ (src/tensor/tensor.cpp:691-698): shapes and dtypes must match.
  if (dst->rank != src->rank) return fail(TB_EINVAL, "Tensor::copy_ failed: Target and source shapes must match exactly.");
  for (int i = 0; i < dst->rank; ++i)
    if (dst->shape[i] != src->shape[i])
      return fail(TB_EINVAL, "Tensor::copy_ failed: Target and source shapes must match exactly.");
  if (dst->dtype != src->dtype)
    return fail(TB_EINVAL, "Tensor::copy_ failed: Target and source data types must match.");
  int es = dtype_size(dst->dtype);
  if (es == 0) return fail(TB_EINVAL, "tb_copy: block-quantized views are copied as raw bytes (use a byte view)");
  int64_t n = numel(dst);
  if (n == 0) return TB_OK;
  DeviceState *st;
  TB_TRY(device_state(&st));
  cudaStream_t s = as_stream(stream);
  const char *ps = static_cast<const char *>(src->data) + src->offset * es;
  char *pd = static_cast<char *>(dst->data) + dst->offset * es;
  Walk3 w;
  w.rank = dst->rank;
  for (int i = 0; i < dst->rank; ++i) {
    w.shape[i] = dst->shape[i];
    w.s0[i] = dst->strides[i];
    w.s1[i] = src->strides[i];
    w.s2[i] = 0;
  }
  w.o0 = w.o1 = w.o2 = 0;
  merge_dims(w, 2);
  if (w.rank == 1 && w.s0[0] == 1 && w.s1[0] == 1) {
    int64_t bytes = n * es;
    if (aligned16(ps) && aligned16(pd) && bytes % 16 == 0) {
      copy_flat16_kernel<<<wave_grid(copy_flat16_kernel, kThreads, bytes / 32 + 1, st->sm_count), kThreads, 0, s>>>(
          reinterpret_cast<const uint4 *>(ps), reinterpret_cast<uint4 *>(pd), bytes / 16);
      return check_launch("tb_copy");
    }
    cudaError_t e = cudaMemcpyAsync(pd, ps, bytes, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return fail(TB_ECUDA, "tb_copy: %s", cudaGetErrorString(e));
    return TB_OK;
  }
  // Transposed innermost pair: dst unit stride on the last merged dim, src on
  // the one before it.
  if (w.rank >= 2 && w.s0[w.rank - 1] == 1 && w.s1[w.rank - 2] == 1 && w.s1[w.rank - 1] != 1) {
    int64_t R = w.shape[w.rank - 2], C = w.shape[w.rank - 1];
    int64_t outer = n / (R * C);
    const bool big = R >= 64 && C >= 64;
    const int T_ = big ? 64 : 32;
    int64_t tiles = outer * ((R + T_ - 1) / T_) * ((C + T_ - 1) / T_);
    int grid = (int)std::min<int64_t>(tiles, (int64_t)st->sm_count * 8);
    if (es == 4) {
      if (big) copy_transpose_kernel<float, 64><<<grid, 256, 0, s>>>((const float *)ps, (float *)pd, outer, R, C, w);
      else copy_transpose_kernel<float, 32><<<grid, 256, 0, s>>>((const float *)ps, (float *)pd, outer, R, C, w);
    } else {
      // pairs of 16-bit elements as 32-bit words when every offset stays even
      bool pairs = big && R % 2 == 0 && C % 2 == 0 && w.s1[w.rank - 1] % 2 == 0 && w.s0[w.rank - 2] % 2 == 0 &&
                   w.o0 % 2 == 0 && w.o1 % 2 == 0 && (reinterpret_cast<uintptr_t>(ps) & 3) == 0 &&
                   (reinterpret_cast<uintptr_t>(pd) & 3) == 0;
      for (int d = 0; d < w.rank - 2; ++d) pairs = pairs && w.s0[d] % 2 == 0 && w.s1[d] % 2 == 0;
      if (pairs) {
        const int64_t tiles16 = outer * ((R + 127) / 128) * ((C + 63) / 64);
        const int g16 = (int)std::min<int64_t>(
            tiles16, (int64_t)st->sm_count * resident_ctas((const void *)copy_transpose16_kernel<128>, 256, 0));
        copy_transpose16_kernel<128><<<g16, 256, 0, s>>>((const uint16_t *)ps, (uint16_t *)pd, outer, R, C, w);
      }
      else if (big)
        copy_transpose_kernel<uint16_t, 64><<<grid, 256, 0, s>>>((const uint16_t *)ps, (uint16_t *)pd, outer, R, C, w);
      else
        copy_transpose_kernel<uint16_t, 32><<<grid, 256, 0, s>>>((const uint16_t *)ps, (uint16_t *)pd, outer, R, C, w);
    }
    return check_launch("tb_copy");
  }
  if (es == 4)
    copy_strided_kernel<float><<<wave_grid(copy_strided_kernel<float>, kThreads, n, st->sm_count), kThreads, 0, s>>>((const float *)ps, (float *)pd, n, w);
  else
    copy_strided_kernel<uint16_t><<<wave_grid(copy_strided_kernel<uint16_t>, kThreads, n, st->sm_count), kThreads, 0, s>>>((const uint16_t *)ps, (uint16_t *)pd, n, w);
  return check_launch("tb_copy");
}

tb_status tb_swiglu(int dtype, const void *g, const void *u, void *y, int64_t n, tb_stream stream) {
  if (n < 0) return fail(TB_EINVAL, "tb_swiglu: negative n");
  if (n == 0) return TB_OK;
  if (!g || !u || !y) return fail(TB_EINVAL, "tb_swiglu: null pointer");
  DeviceState *st;
  TB_TRY(device_state(&st));
  cudaStream_t s = as_stream(stream);
  int vec_ok = aligned16(g) && aligned16(u) && aligned16(y);
  if (dtype == TB_F32) {
    swiglu_kernel<float><<<wave_grid(swiglu_kernel<float>, kThreads, n / 4 + 1, st->sm_count), kThreads, 0, s>>>(
        (const float *)g, (const float *)u, (float *)y, n, vec_ok);
  } else if (dtype == TB_BF16) {
    swiglu_kernel<__nv_bfloat16><<<wave_grid(swiglu_kernel<__nv_bfloat16>, kThreads, n / 8 + 1, st->sm_count), kThreads, 0, s>>>(
        (const __nv_bfloat16 *)g, (const __nv_bfloat16 *)u, (__nv_bfloat16 *)y, n, vec_ok);
  } else {
    return fail(TB_EINVAL, "tb_swiglu: dtype must be TB_F32 or TB_BF16");
  }
  return check_launch("tb_swiglu");
}

}  // extern "C"
