// tb_rows.cu -- row reductions: RMSNorm (A7), softmax (A9), argmax (A15) and
// the per-shard halves of the vocab-sharded softmax/argmax.
//
// Long rows (a 128256-entry logits row is 501 KiB) are split over a thread
// block cluster: each CTA stages its slice of the row in shared memory, the
// CTAs exchange their partial maxima/sums through distributed shared memory,
// and the row is read from HBM once and written once, in one launch.
#include <cooperative_groups.h>

#include <algorithm>
#include <map>
#include <mutex>

#include "tb_internal.cuh"

namespace cg = cooperative_groups;

namespace tb {
namespace {

constexpr int kRowThreads = 256;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    uint64_t w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  return v;
}

// Block-wide reductions (blockDim.x a multiple of 32, <= 1024); result in all threads.
__device__ float block_sum(float v, float *scratch) {
  v = warp_sum(v);
  int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) scratch[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += scratch[i];  // fixed order: deterministic
  return t;
}
__device__ float block_max(float v, float *scratch) {
  v = warp_max(v);
  int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) scratch[w] = v;
  __syncthreads();
  float t = -INFINITY;
  for (int i = 0; i < nw; ++i) t = fmaxf(t, scratch[i]);
  return t;
}
__device__ uint64_t block_max_u64(uint64_t v, uint64_t *scratch) {
  v = warp_max_u64(v);
  int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) scratch[w] = v;
  __syncthreads();
  uint64_t t = 0;
  for (int i = 0; i < nw; ++i) t = scratch[i] > t ? scratch[i] : t;
  return t;
}

// ---------------------------------------------------------------- RMSNorm ----
// One CTA per row (grid-stride over rows); the row stays in registers between
// the sum of squares and the normalisation, so x is read once.
// y = (x / rms) * gamma with rms = sqrtf(sum(x*x) / cols + eps)
// (src/nn/rmsnorm.cpp:38-47); the sum is a tree, the rest IEEE as the reference.
template <typename T> struct RV;
template <> struct RV<float> { static constexpr int N = 4; };
template <> struct RV<__nv_bfloat16> { static constexpr int N = 8; };
__device__ __forceinline__ float tf(float v) { return v; }
__device__ __forceinline__ float tf(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T ft(float v);
template <> __device__ __forceinline__ float ft<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 ft<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <typename T, int VPT>
__global__ void __launch_bounds__(kRowThreads) rmsnorm_vec_kernel(const T *__restrict__ x,
                                                                  const float *__restrict__ gamma,
                                                                  T *__restrict__ y, int64_t rows,
                                                                  int cols, float eps) {
  constexpr int V = RV<T>::N;
  __shared__ float scratch[32];
  const int nvec = cols / V;
  // the next row of this CTA is loaded while the current one is reduced and
  // written (two rows in flight per CTA)
  uint4 nx[VPT];
  auto load = [&](int64_t r) {
    const uint4 *xr = reinterpret_cast<const uint4 *>(x + r * cols);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int i = threadIdx.x + k * kRowThreads;
      if (i < nvec) nx[k] = __ldcs(xr + i);
    }
  };
  if (blockIdx.x < rows) load(blockIdx.x);
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    uint4 v[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) v[k] = nx[k];
    if (r + gridDim.x < rows) load(r + gridDim.x);
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      int i = threadIdx.x + k * kRowThreads;
      if (i < nvec) {
        const T *e = reinterpret_cast<const T *>(&v[k]);
#pragma unroll
        for (int j = 0; j < V; ++j) {
          float f = tf(e[j]);
          ss = __fadd_rn(ss, __fmul_rn(f, f));
        }
      }
    }
    ss = block_sum(ss, scratch);
    float mean = __fdiv_rn(ss, (float)cols);
    float rms = __fsqrt_rn(__fadd_rn(mean, eps));
    // fp32 divides by rms as the reference does (bit-exact); bf16 output
    // (tolerance 1e-2) multiplies by 1/rms: the per-element IEEE division
    // made the bf16 form compute-bound (0.55 of HBM against 0.92 for fp32)
    const float inv = __frcp_rn(rms);
    auto nrm = [&](float v) { return sizeof(T) == 2 ? __fmul_rn(v, inv) : __fdiv_rn(v, rms); };
    uint4 *yr = reinterpret_cast<uint4 *>(y + r * cols);
    const float4 *g4 = reinterpret_cast<const float4 *>(gamma);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      int i = threadIdx.x + k * kRowThreads;
      if (i < nvec) {
        const T *e = reinterpret_cast<const T *>(&v[k]);
        uint4 o;
        T *oe = reinterpret_cast<T *>(&o);
#pragma unroll
        for (int j = 0; j < V; j += 4) {
          float4 g = __ldg(g4 + (i * V + j) / 4);
          oe[j + 0] = ft<T>(__fmul_rn(nrm(tf(e[j + 0])), g.x));
          oe[j + 1] = ft<T>(__fmul_rn(nrm(tf(e[j + 1])), g.y));
          oe[j + 2] = ft<T>(__fmul_rn(nrm(tf(e[j + 2])), g.z));
          oe[j + 3] = ft<T>(__fmul_rn(nrm(tf(e[j + 3])), g.w));
        }
        __stcs(yr + i, o);
      }
    }
  }
}

// Any cols / alignment: two reads of the row.
template <typename T>
__global__ void __launch_bounds__(kRowThreads) rmsnorm_any_kernel(const T *__restrict__ x,
                                                                  const float *__restrict__ gamma,
                                                                  T *__restrict__ y, int64_t rows,
                                                                  int64_t cols, float eps) {
  __shared__ float scratch[32];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const T *xr = x + r * cols;
    float ss = 0.f;
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
      float f = tf(xr[i]);
      ss = __fadd_rn(ss, __fmul_rn(f, f));
    }
    ss = block_sum(ss, scratch);
    float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)cols), eps));
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x)
      y[r * cols + i] = ft<T>(__fmul_rn(__fdiv_rn(tf(xr[i]), rms), gamma[i]));
  }
}

// ---------------------------------------------------------------- softmax ----
// MODE 0: softmax of each row (src/nn/softmax.cpp:30-50): M = max (strict '>',
//   so NaN never becomes the maximum), e = exp(x - M) stored, S = sum of e,
//   y = e / S, here e * (1/S) (within 1.5 ulp of the quotient; the reference's
//   own S is a sequential fp32 sum, which a parallel sum matches only within a
//   tolerance anyway).
// MODE 1: shard statistics only: row max and sum of exp(x - max) of this slice.
// The cluster's CTAs split the row's columns: CTA c owns [c*span, (c+1)*span),
// span a multiple of 4 so a slice is 16-byte aligned whenever its row is.  Each
// CTA stages its slice in shared memory, so the row is read once and written
// once; the CTAs exchange their maxima, then their sums, through distributed
// shared memory.
template <int MODE, int NT>
__global__ void __launch_bounds__(NT) softmax_cluster_kernel(
    const float *__restrict__ x, float *__restrict__ y, int64_t rows, int64_t cols, int64_t ldx,
    int64_t ldy, int span, float *__restrict__ out_max, float *__restrict__ out_sum,
    uint32_t *__restrict__ err) {
  extern __shared__ float4 slice4[];  // span floats
  float *slice = reinterpret_cast<float *>(slice4);
  __shared__ float scratch[32];
  __shared__ float part[2];  // this CTA's [max, sum] for the cluster exchange
  __shared__ __align__(8) uint64_t bar;
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  const int csize = (int)cluster.num_blocks();
  const int64_t row = blockIdx.x / csize;
  if (row >= rows) return;  // whole clusters share a row, so this is uniform
  const int64_t c0 = (int64_t)crank * span;
  const int64_t c1 = (c0 + span < cols) ? c0 + span : cols;
  const int n = c1 > c0 ? (int)(c1 - c0) : 0;
  const int n4 = n >> 2;
  const float *xr = x + row * ldx + c0;

  // Stage the slice: one bulk copy of its 16-byte part when the slice is
  // aligned (plain loads for the last n % 4 floats), else plain loads.
  const bool bulk = n4 > 0 && (reinterpret_cast<uintptr_t>(xr) & 15) == 0;
  if (bulk) {
    if (threadIdx.x == 0) {
      mbar_init(&bar, 1);
      fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(&bar, (uint32_t)n4 * 16u);
      bulk_g2s(slice4, xr, (uint32_t)n4 * 16u, &bar);
    }
    for (int i = 4 * n4 + threadIdx.x; i < n; i += NT) slice[i] = xr[i];
    if (!mbar_wait_bounded(&bar, 0, err)) mbar_wait_bounded(&bar, 0, err);  // second, bounded wait for the copy
  } else {
    for (int i = threadIdx.x; i < n; i += NT) slice[i] = xr[i];
  }
  __syncthreads();
  float m = -INFINITY;
  for (int i = threadIdx.x; i < n4; i += NT) {
    const float4 v = slice4[i];
    m = v.x > m ? v.x : m;
    m = v.y > m ? v.y : m;
    m = v.z > m ? v.z : m;
    m = v.w > m ? v.w : m;
  }
  for (int i = 4 * n4 + threadIdx.x; i < n; i += NT) m = slice[i] > m ? slice[i] : m;
  m = block_max(m, scratch);
  if (threadIdx.x == 0) part[0] = m;
  cluster.sync();
  float M = -INFINITY;
  for (int c = 0; c < csize; ++c) {
    const float pm = *cluster.map_shared_rank(&part[0], c);
    M = pm > M ? pm : M;
  }
  float s = 0.f;
  for (int i = threadIdx.x; i < n4; i += NT) {
    float4 v = slice4[i];
    v.x = __expf(__fsub_rn(v.x, M));
    v.y = __expf(__fsub_rn(v.y, M));
    v.z = __expf(__fsub_rn(v.z, M));
    v.w = __expf(__fsub_rn(v.w, M));
    if (MODE == 0) slice4[i] = v;
    s = __fadd_rn(s, __fadd_rn(__fadd_rn(v.x, v.y), __fadd_rn(v.z, v.w)));
  }
  for (int i = 4 * n4 + threadIdx.x; i < n; i += NT) {
    const float e = __expf(__fsub_rn(slice[i], M));
    if (MODE == 0) slice[i] = e;
    s = __fadd_rn(s, e);
  }
  s = block_sum(s, scratch);
  if (threadIdx.x == 0) part[1] = s;
  cluster.sync();
  float S = 0.f;
  for (int c = 0; c < csize; ++c) S = __fadd_rn(S, *cluster.map_shared_rank(&part[1], c));
  if (MODE == 1) {
    if (crank == 0 && threadIdx.x == 0) {
      out_max[row] = M;
      out_sum[row] = S;
    }
  } else {
    const float inv = __frcp_rn(S);
    float *yr = y + row * ldy + c0;
    if ((reinterpret_cast<uintptr_t>(yr) & 15) == 0) {
      for (int i = threadIdx.x; i < n4; i += NT) {
        float4 v = slice4[i];
        v.x = __fmul_rn(v.x, inv);
        v.y = __fmul_rn(v.y, inv);
        v.z = __fmul_rn(v.z, inv);
        v.w = __fmul_rn(v.w, inv);
        __stcs(reinterpret_cast<float4 *>(yr) + i, v);
      }
      for (int i = 4 * n4 + threadIdx.x; i < n; i += NT) yr[i] = __fmul_rn(slice[i], inv);
    } else {
      for (int i = threadIdx.x; i < n; i += NT) yr[i] = __fmul_rn(slice[i], inv);
    }
  }
  cluster.sync();  // keep this CTA's shared memory alive until every peer has read it
}

// One or a few rows of whole float4s (the 128256-wide logits of a decode
// step): a cluster of up to 16 CTAs per row, each thread holding up to VPT
// float4s of its CTA's slice in registers, all loaded at once -- no
// shared-memory staging.  Same arithmetic as softmax_cluster_kernel: max under
// '>' (NaN never wins), e = exp(x - M), S = block sums added in cluster-rank
// order, y = e * (1/S).  Slices are multiples of 4 columns and row strides
// multiples of 4, so every load and store is a float4.
template <int MODE, int NT, int VPT>
__global__ void __launch_bounds__(NT) softmax_cluster_reg_kernel(
    const float *__restrict__ x, float *__restrict__ y, int64_t rows, int64_t cols, int64_t ldx, int64_t ldy,
    int span, float *__restrict__ out_max, float *__restrict__ out_sum) {
  __shared__ float scratch[32];
  __shared__ float part[2];
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  const int csize = (int)cluster.num_blocks();
  const int64_t row = blockIdx.x / csize;
  if (row >= rows) return;  // whole clusters share a row
  const int64_t c0 = (int64_t)crank * span;
  const int64_t c1 = (c0 + span < cols) ? c0 + span : cols;
  const int n4 = c1 > c0 ? (int)((c1 - c0) >> 2) : 0;
  const float4 *xr = reinterpret_cast<const float4 *>(x + row * ldx + c0);
  float4 v[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = threadIdx.x + j * NT;
    if (i < n4) v[j] = MODE == 0 ? __ldcs(xr + i) : __ldg(xr + i);
  }
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    if (threadIdx.x + j * NT < n4) {
      m = v[j].x > m ? v[j].x : m;
      m = v[j].y > m ? v[j].y : m;
      m = v[j].z > m ? v[j].z : m;
      m = v[j].w > m ? v[j].w : m;
    }
  }
  m = block_max(m, scratch);
  if (threadIdx.x == 0) part[0] = m;
  cluster.sync();
  float M = -INFINITY;
  for (int c = 0; c < csize; ++c) {
    const float pm = *cluster.map_shared_rank(&part[0], c);
    M = pm > M ? pm : M;
  }
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    if (threadIdx.x + j * NT < n4) {
      v[j].x = __expf(__fsub_rn(v[j].x, M));
      v[j].y = __expf(__fsub_rn(v[j].y, M));
      v[j].z = __expf(__fsub_rn(v[j].z, M));
      v[j].w = __expf(__fsub_rn(v[j].w, M));
      s = __fadd_rn(s, __fadd_rn(__fadd_rn(v[j].x, v[j].y), __fadd_rn(v[j].z, v[j].w)));
    }
  }
  s = block_sum(s, scratch);
  if (threadIdx.x == 0) part[1] = s;
  cluster.sync();
  float S = 0.f;
  for (int c = 0; c < csize; ++c) S = __fadd_rn(S, *cluster.map_shared_rank(&part[1], c));
  if (MODE == 1) {
    if (crank == 0 && threadIdx.x == 0) {
      out_max[row] = M;
      out_sum[row] = S;
    }
  } else {
    const float inv = __frcp_rn(S);
    float4 *yr = reinterpret_cast<float4 *>(y + row * ldy + c0);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int i = threadIdx.x + j * NT;
      if (i < n4)
        __stcs(yr + i, make_float4(__fmul_rn(v[j].x, inv), __fmul_rn(v[j].y, inv), __fmul_rn(v[j].z, inv),
                                   __fmul_rn(v[j].w, inv)));
    }
  }
  cluster.sync();  // keep this CTA's shared memory alive until every peer has read it
}

// Tens of rows of whole float4s (a batch of logits): two launches with no
// cluster barriers.  Chunk stats: CTA (row, chunk) writes its chunk's max m_c
// and sum of exp(x - m_c) (x read once from HBM, kept in registers).  Finish
// (programmatic dependent launch): M = max_c m_c, S = sum over chunks in order
// of s_c exp(m_c - M), then y = exp(x - M) * (1/S) for the chunk, x read again
// (from L2 when the batch fits there).
template <int NT, int VPT>
__global__ void __launch_bounds__(NT) softmax_chunk_stats_kernel(const float *__restrict__ x, int64_t cols,
                                                                  int64_t ldx, int span, int chunks,
                                                                  float2 *__restrict__ part) {
  __shared__ float scratch[32];
  pdl_launch_dependents();
  const int64_t row = blockIdx.x / chunks;
  const int c = blockIdx.x % chunks;
  const int64_t c0 = (int64_t)c * span, c1 = (c0 + span < cols) ? c0 + span : cols;
  const int n4 = c1 > c0 ? (int)((c1 - c0) >> 2) : 0;
  const float4 *xr = reinterpret_cast<const float4 *>(x + row * ldx + c0);
  float4 v[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = threadIdx.x + j * NT;
    if (i < n4) v[j] = __ldg(xr + i);
  }
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    if (threadIdx.x + j * NT < n4) {
      m = v[j].x > m ? v[j].x : m;
      m = v[j].y > m ? v[j].y : m;
      m = v[j].z > m ? v[j].z : m;
      m = v[j].w > m ? v[j].w : m;
    }
  }
  m = block_max(m, scratch);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    if (threadIdx.x + j * NT < n4) {
      s = __fadd_rn(s, __fadd_rn(__fadd_rn(__expf(__fsub_rn(v[j].x, m)), __expf(__fsub_rn(v[j].y, m))),
                                 __fadd_rn(__expf(__fsub_rn(v[j].z, m)), __expf(__fsub_rn(v[j].w, m)))));
    }
  }
  s = block_sum(s, scratch);
  if (threadIdx.x == 0) part[blockIdx.x] = make_float2(m, s);
}

template <int NT, int VPT>
__global__ void __launch_bounds__(NT) softmax_chunk_finish_kernel(const float *__restrict__ x, float *__restrict__ y,
                                                                   int64_t cols, int64_t ldx, int64_t ldy, int span,
                                                                   int chunks, const float2 *__restrict__ part) {
  const int64_t row = blockIdx.x / chunks;
  const int c = blockIdx.x % chunks;
  const int64_t c0 = (int64_t)c * span, c1 = (c0 + span < cols) ? c0 + span : cols;
  const int n4 = c1 > c0 ? (int)((c1 - c0) >> 2) : 0;
  const float4 *xr = reinterpret_cast<const float4 *>(x + row * ldx + c0);
  float4 v[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {  // x does not depend on the stats kernel: load before the wait
    const int i = threadIdx.x + j * NT;
    if (i < n4) v[j] = __ldcs(xr + i);
  }
  pdl_wait();
  const float2 *pr = part + row * chunks;
  float M = -INFINITY;
  for (int k = 0; k < chunks; ++k) {
    const float pm = pr[k].x;
    M = pm > M ? pm : M;
  }
  float S = 0.f;
  for (int k = 0; k < chunks; ++k) {
    const float2 p = pr[k];
    S = __fadd_rn(S, p.x == -INFINITY ? 0.f : __fmul_rn(p.y, __expf(__fsub_rn(p.x, M))));
  }
  const float inv = __frcp_rn(S);
  float4 *yr = reinterpret_cast<float4 *>(y + row * ldy + c0);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = threadIdx.x + j * NT;
    if (i < n4)
      __stcs(yr + i, make_float4(__fmul_rn(__expf(__fsub_rn(v[j].x, M)), inv), __fmul_rn(__expf(__fsub_rn(v[j].y, M)), inv),
                                 __fmul_rn(__expf(__fsub_rn(v[j].z, M)), inv), __fmul_rn(__expf(__fsub_rn(v[j].w, M)), inv)));
  }
}

// Many rows: one CTA per row, persistent over rows (grid = one CTA per SM).
// Pass 1 reads the row once from HBM keeping a running (max, sum of exp) per
// thread (the sum rescaled whenever the max grows), combined over the block;
// pass 2 writes exp(x - M) * (1/S).  Between the passes the row stays on chip
// as far as it fits: each thread keeps its first kRowRegF4 float4s in
// registers (96 KB per CTA; eight would spill) and the next ones in shared memory (up
// to the opt-in limit, ~226 KB; each thread stores and later reads only its
// own float4s, so no barrier guards them); only the rest is read again, from
// L2 (for a 513 KB logits row ~190 KB, ~28 MB for 148 rows in flight).  With
// the whole row re-read from L2 (76 MB in flight) half of it came from HBM
// again (ncu, [1024, 128256]: 771 MB read for 525 MB of logits; now 530 MB).
// The register and shared-memory tiers are loaded evict-first (they are not
// read again from memory), the L2 tier normally.  Filling the shared-memory
// tier by one bulk copy per row instead, single- or double-buffered across
// rows, measured 2-6 % slower.  Every thread walks its
// float4s i = t, t + T, t + 2T, ... in order in both passes, whichever tier
// holds them.  Rows must be 16-byte aligned (cols % 4 == 0).
__device__ __forceinline__ void online_add(float v, float &m, float &s) {
  if (v > m) {  // NaN never raises the maximum
    s = __fadd_rn(__fmul_rn(s, __expf(__fsub_rn(m, v))), 1.0f);
    m = v;
  } else if (v != -INFINITY) {  // -inf adds exp(-inf) = 0; NaN makes the sum NaN
    s = __fadd_rn(s, __expf(__fsub_rn(v, m)));
  }
}
__device__ __forceinline__ void online_add4(const float4 &v, float &m, float &s) {
  online_add(v.x, m, s);
  online_add(v.y, m, s);
  online_add(v.z, m, s);
  online_add(v.w, m, s);
}

constexpr int kRowRegF4 = 6;  // float4s per thread kept in registers between the passes

__global__ void __launch_bounds__(1024, 1) softmax_rows_kernel(const float *__restrict__ x, float *__restrict__ y,
                                                               int64_t rows, int64_t cols, int stash_f4) {
  extern __shared__ float4 stash[];  // [stash_f4], each thread's own elements only
  __shared__ float sm[32], ss[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int T = blockDim.x;
  const int64_t n4 = cols >> 2;
  const int64_t RG = min(n4, (int64_t)kRowRegF4 * T);  // [0, RG): registers
  const int64_t SG = RG + min(n4 - RG, (int64_t)stash_f4);  // [RG, SG): shared memory; [SG, n4): L2
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float4 *x4 = reinterpret_cast<const float4 *>(x + r * cols);
    float m = -INFINITY, s = 0.f;
    float4 reg[kRowRegF4];
#pragma unroll
    for (int u = 0; u < kRowRegF4; ++u) {
      const int64_t i = threadIdx.x + (int64_t)u * T;
      if (i < RG) reg[u] = __ldcs(x4 + i);
    }
#pragma unroll
    for (int u = 0; u < kRowRegF4; ++u)
      if (threadIdx.x + (int64_t)u * T < RG) online_add4(reg[u], m, s);
    int64_t i = RG + threadIdx.x;
    for (; i + 3 * (int64_t)T < SG; i += 4 * (int64_t)T) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldcs(x4 + i + u * (int64_t)T);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        stash[i - RG + u * (int64_t)T] = v[u];
        online_add4(v[u], m, s);
      }
    }
    for (; i < SG; i += T) {
      const float4 v = __ldcs(x4 + i);
      stash[i - RG] = v;
      online_add4(v, m, s);
    }
    for (; i + 3 * (int64_t)T < n4; i += 4 * (int64_t)T) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldcg(x4 + i + u * (int64_t)T);
#pragma unroll
      for (int u = 0; u < 4; ++u) online_add4(v[u], m, s);
    }
    for (; i < n4; i += T) online_add4(__ldcg(x4 + i), m, s);
    // combine (m, s) over the warp, then over the block, in a fixed order
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const float mm = fmaxf(m, m2);
      s = (mm == -INFINITY) ? 0.f
                            : __fadd_rn(__fmul_rn(s, __expf(__fsub_rn(m, mm))), __fmul_rn(s2, __expf(__fsub_rn(m2, mm))));
      m = mm;
    }
    __syncthreads();  // the previous row's sm/ss reads are done
    if (lane == 0) {
      sm[warp] = m;
      ss[warp] = s;
    }
    __syncthreads();
    float M = -INFINITY;
    for (int w = 0; w < nw; ++w) M = fmaxf(M, sm[w]);
    float S = 0.f;
    if (M != -INFINITY)
      for (int w = 0; w < nw; ++w) S = __fadd_rn(S, __fmul_rn(ss[w], __expf(__fsub_rn(sm[w], M))));
    // NaN anywhere in the row makes the reference's sum NaN
    const float inv = __frcp_rn(S);
    float4 *y4 = reinterpret_cast<float4 *>(y + r * cols);
    auto out = [&](float4 v) {
      v.x = __fmul_rn(__expf(__fsub_rn(v.x, M)), inv);
      v.y = __fmul_rn(__expf(__fsub_rn(v.y, M)), inv);
      v.z = __fmul_rn(__expf(__fsub_rn(v.z, M)), inv);
      v.w = __fmul_rn(__expf(__fsub_rn(v.w, M)), inv);
      return v;
    };
#pragma unroll
    for (int u = 0; u < kRowRegF4; ++u) {
      const int64_t j = threadIdx.x + (int64_t)u * T;
      if (j < RG) __stcs(y4 + j, out(reg[u]));
    }
    for (int64_t j = RG + threadIdx.x; j < SG; j += T) __stcs(y4 + j, out(stash[j - RG]));
    int64_t j = SG + threadIdx.x;
    for (; j + 3 * (int64_t)T < n4; j += 4 * (int64_t)T) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldcg(x4 + j + u * (int64_t)T);
#pragma unroll
      for (int u = 0; u < 4; ++u) __stcs(y4 + j + u * (int64_t)T, out(v[u]));
    }
    for (; j < n4; j += T) __stcs(y4 + j, out(__ldcg(x4 + j)));
  }
}

// Rows too long for the cluster's shared memory: max, then sum, then the
// output, each a pass over the row (the later passes mostly hit L2).
__global__ void __launch_bounds__(kRowThreads) softmax_long_kernel(const float *__restrict__ x,
                                                                   float *__restrict__ y,
                                                                   int64_t rows, int64_t cols) {
  __shared__ float scratch[32];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float *xr = x + r * cols;
    float m = -INFINITY;
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) m = xr[i] > m ? xr[i] : m;
    m = block_max(m, scratch);
    float s = 0.f;
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) s = __fadd_rn(s, __expf(__fsub_rn(xr[i], m)));
    s = block_sum(s, scratch);
    const float inv = __frcp_rn(s);
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x)
      y[r * cols + i] = __fmul_rn(__expf(__fsub_rn(xr[i], m)), inv);
  }
}

// Shard finish: y = exp(x - M) * (1/S) for this shard's columns.
__global__ void __launch_bounds__(kRowThreads) softmax_finish_kernel(
    const float *__restrict__ x, int64_t rows, int64_t cols, int64_t ldx,
    const float *__restrict__ gmax, const float *__restrict__ gsum, float *__restrict__ y,
    int64_t ldy) {
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const float M = gmax[r], inv = __frcp_rn(gsum[r]);
    const float *xr = x + r * ldx;
    float *yr = y + r * ldy;
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < cols;
         c += (int64_t)gridDim.x * blockDim.x)
      yr[c] = __fmul_rn(__expf(__fsub_rn(xr[c], M)), inv);
  }
}

__global__ void softmax_rescale_kernel(const float *__restrict__ lmax, const float *__restrict__ gmax,
                                       float *__restrict__ sum, int64_t rows) {
  int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r < rows) sum[r] = __fmul_rn(sum[r], __expf(__fsub_rn(lmax[r], gmax[r])));
}

// ----------------------------------------------------------------- argmax ----
// Key of a candidate: order-preserving bits of the value in the high word and
// 0xFFFFFFFF - column in the low word, so the largest key is the largest value
// and, among equal values, the first column.  Only values > -inf that are not
// NaN are candidates (greedy_sample, src/core/sampler.cpp:17-24, takes x only
// when x > running max, which starts at -inf); key 0 = no candidate -> index 0.
__device__ __forceinline__ uint64_t argmax_key(float v, int64_t col) {
  if (!(v > -INFINITY)) return 0ull;
  // -0.0 and +0.0 compare equal under '>', so they must get the same key.
  uint32_t b = v == 0.0f ? 0u : __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((uint64_t)b << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)col);
}

// Shard keys leave the kernel with the top bit flipped, so that their order as
// signed 64-bit integers is the unsigned key order (no candidate = INT64_MIN):
// a plain int64 MAX all-reduce then combines the shards.
constexpr uint64_t kKeySignFlip = 0x8000000000000000ull;

// KEYS = 0: writes the row's index; KEYS = 1: writes the row's key (shards).
template <int KEYS>
__global__ void __launch_bounds__(kRowThreads) argmax_cluster_kernel(
    const float *__restrict__ x, int64_t rows, int64_t cols, int64_t ldx, int64_t col_base,
    int span, int64_t *__restrict__ idx_out, int64_t *__restrict__ key_out) {
  __shared__ uint64_t scratch[32];
  __shared__ uint64_t part;
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  const int csize = (int)cluster.num_blocks();
  const int64_t row = blockIdx.x / csize;
  if (row >= rows) return;
  const int64_t c0 = (int64_t)crank * span;
  const int64_t c1 = (c0 + span < cols) ? c0 + span : cols;
  const float *xr = x + row * ldx;
  // Each thread scans its columns in increasing order keeping the first
  // strict maximum (greedy_sample's rule: NaN and -inf never win, a tie keeps
  // the earlier column); the key is formed once, for the block reduction.
  float bv = -INFINITY;
  int64_t bi = -1;
  const bool vec = ((reinterpret_cast<uintptr_t>(xr + c0) & 15) == 0);
  int64_t tail = c0;
  if (vec) {
    const int64_t nv = (c1 - c0) / 4;
    const float4 *x4 = reinterpret_cast<const float4 *>(xr + c0);
    int64_t j = threadIdx.x;
    for (; j + 3 * (int64_t)blockDim.x < nv; j += 4 * (int64_t)blockDim.x) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldcs(x4 + j + u * (int64_t)blockDim.x);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t col = c0 + 4 * (j + u * (int64_t)blockDim.x);
        if (v[u].x > bv) { bv = v[u].x; bi = col; }
        if (v[u].y > bv) { bv = v[u].y; bi = col + 1; }
        if (v[u].z > bv) { bv = v[u].z; bi = col + 2; }
        if (v[u].w > bv) { bv = v[u].w; bi = col + 3; }
      }
    }
    for (; j < nv; j += blockDim.x) {
      const float4 v = __ldcs(x4 + j);
      const int64_t col = c0 + 4 * j;
      if (v.x > bv) { bv = v.x; bi = col; }
      if (v.y > bv) { bv = v.y; bi = col + 1; }
      if (v.z > bv) { bv = v.z; bi = col + 2; }
      if (v.w > bv) { bv = v.w; bi = col + 3; }
    }
    tail = c0 + 4 * nv;
  }
  for (int64_t k = tail + threadIdx.x; k < c1; k += blockDim.x) {
    const float v = xr[k];
    if (v > bv) { bv = v; bi = k; }
  }
  uint64_t best = bi >= 0 ? argmax_key(bv, col_base + bi) : 0ull;
  best = block_max_u64(best, scratch);
  if (threadIdx.x == 0) part = best;
  cluster.sync();
  if (crank == 0 && threadIdx.x == 0) {
    uint64_t k = 0;
    for (int c = 0; c < csize; ++c) {
      uint64_t p = *cluster.map_shared_rank(&part, c);
      k = p > k ? p : k;
    }
    if (KEYS) key_out[row] = (int64_t)(k ^ kKeySignFlip);
    else idx_out[row] = k ? (int64_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFu)) : 0;
  }
  cluster.sync();
}

__global__ void key_index_kernel(const int64_t *__restrict__ keys, int64_t rows,
                                 int64_t *__restrict__ idx) {
  int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r < rows) {
    const uint64_t k = (uint64_t)keys[r] ^ kKeySignFlip;
    idx[r] = k ? (int64_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFu)) : 0;
  }
}

// Cluster size for a row of `cols` columns: enough CTAs that each slice fits
// the shared memory budget, at most 8 (the portable cluster size); 0 when the
// row needs more than that.
int cluster_for(int64_t cols, int64_t smem_budget_floats) {
  int c = 1;
  while (c < 8 && (cols + c - 1) / c > smem_budget_floats) c *= 2;
  if ((cols + c - 1) / c > smem_budget_floats) return 0;
  // Spread long rows for latency even when one CTA could hold them.
  while (c < 8 && (cols + c - 1) / c > 8192) c *= 2;
  return c;
}

template <int NT, typename Kern, typename... Args>
tb_status launch_cluster_nt(Kern k, int64_t rows, int csize, size_t smem, cudaStream_t s,
                            Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(rows * csize), 1, 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (csize > 8) {
    static bool nonportable = false;  // one attribute call per process
    if (!nonportable) {
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess) return fail(TB_ECUDA, "cluster attribute: %s", cudaGetErrorString(e));
      nonportable = true;
    }
  }
  TB_TRY(ensure_smem_for(k, smem));
  cudaError_t e = cudaLaunchKernelEx(&cfg, k, args...);
  if (e != cudaSuccess) return fail(TB_ECUDA, "cluster launch: %s", cudaGetErrorString(e));
  return TB_OK;
}

template <typename Kern, typename... Args>
tb_status launch_cluster(Kern k, int64_t rows, int csize, size_t smem, cudaStream_t s, Args... args) {
  return launch_cluster_nt<kRowThreads>(k, rows, csize, smem, s, args...);
}

constexpr int64_t kSliceFloats = (96 * 1024) / 4;  // dynamic smem per CTA for a slice

// Columns per CTA of a cluster of `cs`: a multiple of 4, so that each slice
// starts 16-byte aligned when its row does.
int softmax_span(int64_t cols, int cs) {
  int64_t span = (cols + cs - 1) / cs;
  return (int)((span + 3) / 4 * 4);
}

constexpr int kRegNT = 256, kRegVPT = 8;  // softmax_cluster_reg_kernel: 8192 floats per CTA

// Launches softmax_cluster_reg_kernel when the rows are few, whole float4s
// and at most 16 x 8192 wide; returns false (nothing launched) otherwise.
template <int MODE>
bool softmax_reg_launch(const float *x, float *y, int64_t rows, int64_t cols, int64_t ldx, int64_t ldy, float *mx,
                        float *sm, cudaStream_t s, const DeviceState *st, tb_status *status) {
  if (rows >= st->sm_count || cols % 4 != 0 || ldx % 4 != 0 || (MODE == 0 && ldy % 4 != 0) ||
      (reinterpret_cast<uintptr_t>(x) & 15) || (MODE == 0 && (reinterpret_cast<uintptr_t>(y) & 15)))
    return false;
  constexpr int64_t per_cta = (int64_t)kRegNT * kRegVPT * 4;
  int cl = 1;
  while (cl < 16 && (cols + cl - 1) / cl > per_cta) cl *= 2;
  if ((cols + cl - 1) / cl > per_cta) return false;
  auto kern = softmax_cluster_reg_kernel<MODE, kRegNT, kRegVPT>;
  if (cl > 8) {
    // a 16-CTA cluster is a non-portable size: check once that one fits
    static int fits[64] = {0};
    if (fits[st->device] == 0) {
      int n = 0;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(16, 1, 1);
      cfg.blockDim = dim3(kRegNT, 1, 1);
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 16;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e == cudaSuccess) e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
      fits[st->device] = (e == cudaSuccess && n > 0) ? 1 : -1;
    }
    if (fits[st->device] < 0) return false;
  }
  *status = launch_cluster_nt<kRegNT>(kern, rows, cl, 0, s, x, y, rows, cols, ldx, ldy, softmax_span(cols, cl), mx, sm);
  return true;
}

// Launches the two-kernel chunked softmax (8 to sm_count rows of whole
// float4s, at most 16 x 8192 wide); false (nothing launched) otherwise.  The
// chunk statistics live in stream-ordered scratch.
bool softmax_chunks_launch(const float *x, float *y, int64_t rows, int64_t cols, cudaStream_t s, const DeviceState *st,
                           tb_status *status) {
  if (rows < 8 || rows >= st->sm_count || cols % 4 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(y) & 15))
    return false;
  constexpr int64_t per_cta = (int64_t)kRegNT * kRegVPT * 4;
  int chunks = 1;
  while (chunks < 16 && (cols + chunks - 1) / chunks > per_cta) chunks *= 2;
  if ((cols + chunks - 1) / chunks > per_cta) return false;
  const int span = softmax_span(cols, chunks);
  const int64_t grid = rows * chunks;
  float2 *part = nullptr;
  cudaError_t e = cudaMallocAsync(reinterpret_cast<void **>(&part), (size_t)grid * sizeof(float2), s);
  if (e != cudaSuccess) {
    *status = fail(TB_ENOMEM, "tb_softmax: scratch: %s", cudaGetErrorString(e));
    return true;
  }
  softmax_chunk_stats_kernel<kRegNT, kRegVPT><<<(unsigned)grid, kRegNT, 0, s>>>(x, cols, cols, span, chunks, part);
  *status = check_launch("tb_softmax (chunk stats)");
  if (*status == TB_OK) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid, 1, 1);
    cfg.blockDim = dim3(kRegNT, 1, 1);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, softmax_chunk_finish_kernel<kRegNT, kRegVPT>, x, y, cols, cols, cols, span, chunks,
                           (const float2 *)part);
    if (e != cudaSuccess) *status = fail(TB_ECUDA, "tb_softmax (chunk finish): %s", cudaGetErrorString(e));
  }
  e = cudaFreeAsync(part, s);
  if (*status == TB_OK && e != cudaSuccess) *status = fail(TB_ECUDA, "tb_softmax: scratch: %s", cudaGetErrorString(e));
  return true;
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" {

tb_status tb_rmsnorm(int dtype, const void *x, const float *gamma, void *y, int64_t rows,
                     int64_t cols, float eps, tb_stream stream) {
  if (rows < 0 || cols <= 0) return fail(TB_EINVAL, "Input last dimension must match hidden_size.");
  if (rows == 0) return TB_OK;
  if (!x || !gamma || !y) return fail(TB_EINVAL, "tb_rmsnorm: null pointer");
  if (dtype != TB_F32 && dtype != TB_BF16) return fail(TB_EINVAL, "tb_rmsnorm: dtype must be TB_F32 or TB_BF16");
  DeviceState *st;
  TB_TRY(device_state(&st));
  cudaStream_t s = as_stream(stream);
  int64_t grid = std::min<int64_t>(rows, (int64_t)st->sm_count * 8);
  const int V = dtype == TB_F32 ? 4 : 8;
  bool al = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) |
              reinterpret_cast<uintptr_t>(gamma)) & 15) == 0;
  int64_t nvec = cols / V;
  int vpt = (int)((nvec + kRowThreads - 1) / kRowThreads);
  if (al && cols % V == 0 && vpt <= 8) {
    int pick = vpt <= 1 ? 1 : vpt <= 2 ? 2 : vpt <= 4 ? 4 : 8;
#define TB_RMS(T, P)                                                                                \
  rmsnorm_vec_kernel<T, P><<<(int)std::min<int64_t>(rows, (int64_t)st->sm_count *                     \
                                                              resident_ctas((const void *)rmsnorm_vec_kernel<T, P>, \
                                                                            kRowThreads, 0)),        \
                             kRowThreads, 0, s>>>((const T *)x, gamma, (T *)y, rows, (int)cols, eps)
    if (dtype == TB_F32) {
      if (pick == 1) TB_RMS(float, 1); else if (pick == 2) TB_RMS(float, 2);
      else if (pick == 4) TB_RMS(float, 4); else TB_RMS(float, 8);
    } else {
      if (pick == 1) TB_RMS(__nv_bfloat16, 1); else if (pick == 2) TB_RMS(__nv_bfloat16, 2);
      else if (pick == 4) TB_RMS(__nv_bfloat16, 4); else TB_RMS(__nv_bfloat16, 8);
    }
#undef TB_RMS
  } else if (dtype == TB_F32) {
    rmsnorm_any_kernel<float><<<(int)grid, kRowThreads, 0, s>>>((const float *)x, gamma, (float *)y, rows, cols, eps);
  } else {
    rmsnorm_any_kernel<__nv_bfloat16><<<(int)grid, kRowThreads, 0, s>>>(
        (const __nv_bfloat16 *)x, gamma, (__nv_bfloat16 *)y, rows, cols, eps);
  }
  return check_launch("tb_rmsnorm");
}

tb_status tb_softmax(const float *x, float *y, int64_t rows, int64_t cols, tb_stream stream) {
  if (rows < 0 || cols < 0) return fail(TB_EINVAL, "tb_softmax: negative extent");
  if (rows == 0 || cols == 0) return TB_OK;
  if (!x || !y) return fail(TB_EINVAL, "tb_softmax: null pointer");
  DeviceState *st;
  TB_TRY(device_state(&st));
  cudaStream_t s = as_stream(stream);
  int cs = cluster_for(cols, kSliceFloats);
  if (cs == 0) {
    int64_t grid = std::min<int64_t>(rows, (int64_t)st->sm_count * 4);
    softmax_long_kernel<<<(int)grid, kRowThreads, 0, s>>>(x, y, rows, cols);
    return check_launch("tb_softmax");
  }
  const int span = softmax_span(cols, cs);
  // many rows of whole float4s: a persistent CTA per row (two passes, the
  // second from L2)
  if (cols % 4 == 0 && rows >= st->sm_count && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(y) & 15) == 0) {
    // shared memory for as much of a row as the SM allows, beyond the registers
    const int64_t beyond = std::max<int64_t>(0, cols / 4 - (int64_t)kRowRegF4 * 1024);
    const int stash_f4 = (int)std::min<int64_t>(beyond, (st->smem_optin - 1024) / 16);
    const size_t smem = (size_t)stash_f4 * 16;
    TB_TRY(ensure_smem_for(softmax_rows_kernel, smem));
    softmax_rows_kernel<<<st->sm_count, 1024, smem, s>>>(x, y, rows, cols, stash_f4);
    return check_launch("tb_softmax");
  }
  tb_status rs = TB_OK;
  if (softmax_chunks_launch(x, y, rows, cols, s, st, &rs)) return rs;
  if (rows < 8 && softmax_reg_launch<0>(x, y, rows, cols, cols, cols, nullptr, nullptr, s, st, &rs)) return rs;
  if (rows * cs <= st->sm_count)  // few rows: wide CTAs shorten each row's critical path
    return launch_cluster_nt<1024>(softmax_cluster_kernel<0, 1024>, rows, cs, (size_t)span * 4, s, x, y,
                                   rows, cols, cols, cols, span, (float *)nullptr, (float *)nullptr,
                                   st->err_word);
  return launch_cluster_nt<512>(softmax_cluster_kernel<0, 512>, rows, cs, (size_t)span * 4, s, x, y, rows,
                                cols, cols, cols, span, (float *)nullptr, (float *)nullptr, st->err_word);
}

tb_status tb_argmax(const float *x, int64_t rows, int64_t cols, int64_t *idx, tb_stream stream) {
  if (rows < 0 || cols < 0) return fail(TB_EINVAL, "tb_argmax: negative extent");
  if (rows == 0) return TB_OK;
  if (!x || !idx) return fail(TB_EINVAL, "tb_argmax: null pointer");
  if (cols > 0xFFFFFFFFll) return fail(TB_EINVAL, "tb_argmax: more than 2^32 columns");
  DeviceState *st;
  TB_TRY(device_state(&st));
  cudaStream_t s = as_stream(stream);
  int cs = 1;
  while (cs < 8 && (cols + cs - 1) / cs > 8192) cs *= 2;
  int span = (int)((cols + cs - 1) / cs);
  span = (span + 3) / 4 * 4;
  return launch_cluster(argmax_cluster_kernel<0>, rows, cs, 0, s, x, rows, cols, cols, (int64_t)0,
                        span, idx, (int64_t *)nullptr);
}

tb_status tb_softmax_shard_stats(const float *x, int64_t rows, int64_t cols, int64_t ld,
                                 float *row_max, float *row_sum, tb_stream stream) {
  if (rows < 0 || cols <= 0 || ld < cols) return fail(TB_EINVAL, "tb_softmax_shard_stats: bad extents");
  if (rows == 0) return TB_OK;
  if (!x || !row_max || !row_sum) return fail(TB_EINVAL, "tb_softmax_shard_stats: null pointer");
  DeviceState *st;
  TB_TRY(device_state(&st));
  int cs = cluster_for(cols, kSliceFloats);
  if (cs == 0) return fail(TB_EINVAL, "tb_softmax_shard_stats: shard too wide (%lld columns)", (long long)cols);
  const int span = softmax_span(cols, cs);
  tb_status rs = TB_OK;
  if (rows < 8 && softmax_reg_launch<1>(x, nullptr, rows, cols, ld, 0, row_max, row_sum, as_stream(stream), st, &rs))
    return rs;
  if (rows * cs <= st->sm_count)
    return launch_cluster_nt<1024>(softmax_cluster_kernel<1, 1024>, rows, cs, (size_t)span * 4, as_stream(stream),
                                   x, (float *)nullptr, rows, cols, ld, (int64_t)0, span, row_max, row_sum,
                                   st->err_word);
  return launch_cluster_nt<512>(softmax_cluster_kernel<1, 512>, rows, cs, (size_t)span * 4, as_stream(stream), x,
                                (float *)nullptr, rows, cols, ld, (int64_t)0, span, row_max, row_sum,
                                st->err_word);
}

tb_status tb_softmax_shard_rescale(const float *lmax, const float *gmax, float *sum, int64_t rows,
                                   tb_stream stream) {
  if (rows < 0) return fail(TB_EINVAL, "tb_softmax_shard_rescale: negative rows");
  if (rows == 0) return TB_OK;
  if (!lmax || !gmax || !sum) return fail(TB_EINVAL, "tb_softmax_shard_rescale: null pointer");
  softmax_rescale_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, as_stream(stream)>>>(lmax, gmax, sum, rows);
  return check_launch("tb_softmax_shard_rescale");
}

tb_status tb_softmax_shard_finish(const float *x, int64_t rows, int64_t cols, int64_t ld,
                                  const float *gmax, const float *gsum, float *y, int64_t ld_y,
                                  tb_stream stream) {
  if (rows < 0 || cols < 0 || ld < cols || ld_y < cols) return fail(TB_EINVAL, "tb_softmax_shard_finish: bad extents");
  if (rows == 0 || cols == 0) return TB_OK;
  if (!x || !gmax || !gsum || !y) return fail(TB_EINVAL, "tb_softmax_shard_finish: null pointer");
  DeviceState *st;
  TB_TRY(device_state(&st));
  // columns across blockIdx.x, rows across blockIdx.y: about 8 CTAs per SM in all
  const int64_t per_row = (cols + kRowThreads - 1) / kRowThreads;
  const int64_t gy = std::min<int64_t>(rows, 65535);
  const int64_t gx = std::max<int64_t>(1, std::min<int64_t>(per_row, ((int64_t)st->sm_count * 8 + gy - 1) / gy));
  softmax_finish_kernel<<<dim3((unsigned)gx, (unsigned)gy), kRowThreads, 0, as_stream(stream)>>>(
      x, rows, cols, ld, gmax, gsum, y, ld_y);
  return check_launch("tb_softmax_shard_finish");
}

tb_status tb_argmax_shard_keys(const float *x, int64_t rows, int64_t cols, int64_t ld,
                               int64_t col_base, int64_t *keys, tb_stream stream) {
  if (rows < 0 || cols < 0 || ld < cols || col_base < 0) return fail(TB_EINVAL, "tb_argmax_shard_keys: bad extents");
  if (col_base + cols > 0xFFFFFFFFll) return fail(TB_EINVAL, "tb_argmax_shard_keys: more than 2^32 columns");
  if (rows == 0) return TB_OK;
  if (!x || !keys) return fail(TB_EINVAL, "tb_argmax_shard_keys: null pointer");
  int cs = 1;
  while (cs < 8 && (cols + cs - 1) / cs > 8192) cs *= 2;
  int span = (int)((cols + cs - 1) / cs);
  span = (span + 3) / 4 * 4;
  return launch_cluster(argmax_cluster_kernel<1>, rows, cs, 0, as_stream(stream), x, rows, cols, ld,
                        col_base, span, (int64_t *)nullptr, keys);
}

tb_status tb_argmax_key_index(const int64_t *keys, int64_t rows, int64_t *idx, tb_stream stream) {
  if (rows < 0) return fail(TB_EINVAL, "tb_argmax_key_index: negative rows");
  if (rows == 0) return TB_OK;
  if (!keys || !idx) return fail(TB_EINVAL, "tb_argmax_key_index: null pointer");
  key_index_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, as_stream(stream)>>>(keys, rows, idx);
  return check_launch("tb_argmax_key_index");
}

}  // extern "C"
