// tb_gemv.cu -- quantized matmul on CUDA cores with the reference's exact
// operation order (A10 decode GEMV, A11 Q4_0 rows).
//
// Q8_0 (src/tensor/quant_math.hpp:32-60): for every output,
//   per block b:  bs_b = sum_j round(round(q_j * d_b) * x_j)   (sequential in j)
//   y = sum_b bs_b                                            (sequential in b)
// q*d is exact in fp32 (8-bit q times an 11-bit half scale), so the kernel may
// form it any exact way; it builds it from a magic-number float (no int->float
// conversion instruction).  Each lane runs two blocks' chains side by side:
// the exact dequantisation and the rounded products use the sm_100a packed
// f32x2 fma/add/mul (each half an IEEE op), the accumulation is scalar so the
// product rounding is kept.  The block sums land in shared memory and one lane
// per row adds them in block order.
//
// Data movement: a CTA owns ROWS consecutive weight rows (one contiguous byte
// range) and fetches all of it with one bulk TMA copy at kernel start, so the
// whole matrix is in flight at once across the grid.  x is staged in shared
// memory transposed ([j][block], padded) so that each lane pulls its two
// blocks' 64 activations into registers without bank conflicts.
#include <algorithm>

#include "tb_internal.cuh"
#include "tb_q8_row.cuh"

namespace tb {
namespace {


// Stages the CTA's weight byte range [B0, B1) (relative to W) into smem.
// Returns the shift of byte B0 inside the staged buffer.  Thread 0 issues the
// bulk copy of the 16-byte-aligned body; all threads load the ragged tail.
// The caller __syncthreads() afterwards and waits on `bar` before reading.
__device__ __forceinline__ int stage_rows(const uint8_t *__restrict__ W, int64_t B0, int64_t B1,
                                          uint8_t *wsm, uint64_t *bar, bool use_tma) {
  int64_t t0 = B0 & ~int64_t(15);
  int shift = (int)(B0 - t0);
  if (use_tma) {
    int64_t t1 = B1 & ~int64_t(15);
    uint32_t body = t1 > t0 ? (uint32_t)(t1 - t0) : 0u;
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(bar, body);
      if (body) bulk_g2s(wsm, W + t0, body, bar);
    }
    int64_t tail0 = t1 > t0 ? t1 : B0;
    for (int64_t i = tail0 + threadIdx.x; i < B1; i += blockDim.x) wsm[i - t0] = W[i];
  } else {
    if (threadIdx.x == 0) mbar_arrive(bar);
    for (int64_t i = B0 + threadIdx.x; i < B1; i += blockDim.x) wsm[i - t0] = W[i];
  }
  return shift;
}

template <int NW>
__global__ void __launch_bounds__(NW * 32) gemv_q8_0_kernel(
    const uint8_t *__restrict__ W, const float *__restrict__ X, float *__restrict__ Y, int N,
    int K, int M, int rows_per_cta, int use_tma, uint32_t *__restrict__ err) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int nb = K / 32;
  const int rb = nb * 34;
  const int XS = (nb & 1) ? nb + 2 : nb + 1;  // odd row pitch: conflict-free
  const int rpw = rows_per_cta / NW;
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem);
  float *xs = reinterpret_cast<float *>(smem + 128);
  const int BP = (nb + 4) & ~3;  // block-sum row pitch, a multiple of 4 floats (16-byte rows)
  float *bsum = xs + 32 * XS;                       // [NW][rpw][BP]
  uint8_t *wsm = reinterpret_cast<uint8_t *>(bsum + NW * rpw * BP);
  wsm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(wsm) + 127) & ~uintptr_t(127));

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n0 = blockIdx.x * rows_per_cta;
  const int n1 = min(N, n0 + rows_per_cta);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  const int shift = stage_rows(W, (int64_t)n0 * rb, (int64_t)n1 * rb, wsm, bar, use_tma != 0);

  float *mysum = bsum + warp * rpw * BP;
  bool ready = false;
  for (int m = 0; m < M; ++m) {
    const float *xrow = X + (int64_t)m * K;
    if (m > 0) __syncthreads();  // previous x no longer read
    // All loads of this thread's share of x are issued before any store, so
    // the L2 round trips overlap instead of queueing behind each other.
    if ((K & 3) == 0 && (reinterpret_cast<uintptr_t>(xrow) & 15) == 0) {
      const float4 *x4 = reinterpret_cast<const float4 *>(xrow);
      const int nv = K >> 2;
      for (int base = 0; base < nv; base += 4 * NW * 32) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int iv = base + u * NW * 32 + threadIdx.x;
          v[u] = iv < nv ? __ldg(x4 + iv) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int iv = base + u * NW * 32 + threadIdx.x;
          if (iv < nv) {
            const int i = iv * 4;
            xs[((i + 0) & 31) * XS + ((i + 0) >> 5)] = v[u].x;
            xs[((i + 1) & 31) * XS + ((i + 1) >> 5)] = v[u].y;
            xs[((i + 2) & 31) * XS + ((i + 2) >> 5)] = v[u].z;
            xs[((i + 3) & 31) * XS + ((i + 3) >> 5)] = v[u].w;
          }
        }
      }
    } else {
      for (int i = threadIdx.x; i < K; i += blockDim.x) xs[(i & 31) * XS + (i >> 5)] = __ldg(xrow + i);
    }
    __syncthreads();
    if (!ready) {
      // Every thread waits; if any gave up, all leave together (no thread may
      // be left behind at a later __syncthreads).
      const bool ok = mbar_wait_bounded(bar, 0, err);
      if (__syncthreads_or(!ok)) return;
      ready = true;
    }
    for (int p = 0; p * 64 < nb; ++p) {
      const int b1 = p * 64 + lane, b2 = b1 + 32;
      const bool v1 = b1 < nb, v2 = b2 < nb;
      uint64_t xp[32];
#pragma unroll
      for (int j = 0; j < 32; ++j)
        xp[j] = pack2(v1 ? xs[j * XS + b1] : 0.f, v2 ? xs[j * XS + b2] : 0.f);
      for (int rr = 0; rr < rpw; ++rr) {
        const int r = warp * rpw + rr;
        if (n0 + r >= n1) break;
        const int rowoff = shift + r * rb;
        float d1 = 0.f, d2 = 0.f;
        uint32_t q1[8], q2[8];
        load_q8_block(wsm, rowoff + 34 * (v1 ? b1 : 0), d1, q1);
        load_q8_block(wsm, rowoff + 34 * (v2 ? b2 : 0), d2, q2);
        float s1, s2;
        if (isfinite(d1) && isfinite(d2)) {
          const uint64_t dd = pack2(d1, d2);
          const uint64_t c1 = pack2(-kMagic * d1, -kMagic * d2);  // exact: 3*2^22*d
          const uint64_t c2 = pack2(-128.0f * d1, -128.0f * d2);
          s1 = 0.f;
          s2 = 0.f;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t u1 = q1[k] ^ 0x80808080u, u2 = q2[k] ^ 0x80808080u;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              // float(0x4B4000uu) = 12582912 + (q + 128)
              const uint32_t sel = 0x7650u | (uint32_t)e;
              const float m1 = __uint_as_float(__byte_perm(u1, kMagicHi, sel));
              const float m2 = __uint_as_float(__byte_perm(u2, kMagicHi, sel));
              uint64_t t = fma2(pack2(m1, m2), dd, c1);  // (q+128)*d, exact
              t = add2(t, c2);                           // q*d, exact
              float p1, p2;
              unpack2(mul2(t, xp[4 * k + e]), p1, p2);   // round(w * x)
              // The accumulation stays scalar: ptxas contracts a packed
              // mul + packed add into a packed FMA, which would skip the
              // rounding of the product that the reference performs.
              s1 = __fadd_rn(s1, p1);
              s2 = __fadd_rn(s2, p2);
            }
          }
        } else {  // non-finite scale: the plain expression, as the reference
          s1 = 0.f;
          s2 = 0.f;
#pragma unroll
          for (int k = 0; k < 8; ++k)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float x1, x2;
              unpack2(xp[4 * k + e], x1, x2);
              s1 = __fadd_rn(s1, __fmul_rn(__fmul_rn((float)(int8_t)(q1[k] >> (8 * e)), d1), x1));
              s2 = __fadd_rn(s2, __fmul_rn(__fmul_rn((float)(int8_t)(q2[k] >> (8 * e)), d2), x2));
            }
        }
        if (v1) mysum[rr * BP + b1] = s1;
        if (v2) mysum[rr * BP + b2] = s2;
      }
    }
    __syncwarp();
    if (lane < rpw && n0 + warp * rpw + lane < n1) {
      // y = sum of the block sums in block order (quant_math.hpp:56).
      const float4 *bs4 = reinterpret_cast<const float4 *>(mysum + lane * BP);
      float s = 0.f;
      int b = 0;
      for (; b + 8 <= nb; b += 8) {
        const float4 a = bs4[b / 4], c = bs4[b / 4 + 1];
        s = __fadd_rn(s, a.x); s = __fadd_rn(s, a.y); s = __fadd_rn(s, a.z); s = __fadd_rn(s, a.w);
        s = __fadd_rn(s, c.x); s = __fadd_rn(s, c.y); s = __fadd_rn(s, c.z); s = __fadd_rn(s, c.w);
      }
      for (; b < nb; ++b) s = __fadd_rn(s, mysum[lane * BP + b]);
      Y[(int64_t)m * N + n0 + warp * rpw + lane] = s;
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Span GEMV (M == 1), tb_matmul_quant_exact's path: the reference's order bit
// for bit.
//
// One CTA per SM owns a contiguous range of rows.  The range is cut into spans
// that fit in shared memory; two span buffers are in flight, and each span is
// fetched as four large bulk TMA copies (row-aligned quarters) with one
// mbarrier each, so warps start on the first quarter while the rest streams.
// Few large copies per SM stream at the same rate as plain 16-byte loads from
// every thread; many small copies do not.
//
// Programmatic dependent launch: the first span's copies are issued before
// griddepcontrol.wait (weights never depend on the previous kernel), x is
// read and y written only after it, and the kernel lets its dependents launch
// at once.  A GEMV that follows another kernel in the stream therefore starts
// streaming its weights while the predecessor drains.  The second span's
// copies go out right after the first loads of x, so that x does not queue
// behind them (8192 x 2048: 8.77 against 9.46 us with both spans issued before
// the wait).

struct SpanCfg {
  int span_rows;  // rows per span buffer
};

template <int NWARP>
__global__ void __launch_bounds__(NWARP * 32, 1) gemv_q8_0_span_kernel(
    const uint8_t *__restrict__ W, const float *__restrict__ X, float *__restrict__ Y, int N,
    int K, int span_rows, uint32_t *__restrict__ err) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int abort_flag;
  const int nb = K / 32;
  const int rb = nb * 34;
  const int XS = (nb & 1) ? nb + 2 : nb + 1;
  const int BP = (nb + 4) & ~3;
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem);  // [2 buffers][4 quarters]
  float *xs = reinterpret_cast<float *>(smem + 256);
  float *bsum = xs + 32 * XS;  // [span_rows][BP] block sums
  uint8_t *buf0 = reinterpret_cast<uint8_t *>(bsum + span_rows * BP);
  buf0 = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(buf0) + 127) & ~uintptr_t(127));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  // this CTA's rows: [n0, n0 + cnt), balanced over the grid
  const int G = gridDim.x, base = N / G, rem = N % G;
  const int n0 = blockIdx.x * base + min((int)blockIdx.x, rem);
  const int cnt = base + ((int)blockIdx.x < rem ? 1 : 0);
  const int nspans = (cnt + span_rows - 1) / span_rows;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 8; ++i) mbar_init(bar + i, 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  __syncthreads();

  // thread q < 4 issues quarter q of span k into buffer (k & 1)
  auto issue = [&](int k) {
    const int q = threadIdx.x;
    const int r0 = k * span_rows;
    const int nr = min(span_rows, cnt - r0);
    const int qr = (nr + 3) / 4;
    const int a = min(nr, q * qr), b = min(nr, (q + 1) * qr);
    const uint32_t bytes = (uint32_t)((b - a) * rb);
    uint64_t *bq = bar + (k & 1) * 4 + q;
    mbar_arrive_expect_tx(bq, bytes);
    if (bytes)
      bulk_g2s(buf0 + (size_t)(k & 1) * span_rows * rb + (size_t)a * rb,
               W + ((int64_t)n0 + r0 + a) * rb, bytes, bq);
  };
  if (threadIdx.x < 4 && nspans > 0) issue(0);  // span 1 once x's first loads are out (below)
  pdl_launch_dependents();
  pdl_wait();  // x (and the order of our y writes) depend on the previous kernel

  // x -> shared memory, transposed [j][block] with an odd pitch
  {
    const float4 *x4 = reinterpret_cast<const float4 *>(X);
    const int nv = K >> 2;
    for (int base4 = 0; base4 < nv; base4 += 4 * NWARP * 32) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int iv = base4 + u * NWARP * 32 + threadIdx.x;
        v[u] = iv < nv ? __ldg(x4 + iv) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      if (base4 == 0 && threadIdx.x < 4 && nspans > 1) issue(1);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int iv = base4 + u * NWARP * 32 + threadIdx.x;
        if (iv < nv) {
          const int i = iv * 4;
          xs[((i + 0) & 31) * XS + ((i + 0) >> 5)] = v[u].x;
          xs[((i + 1) & 31) * XS + ((i + 1) >> 5)] = v[u].y;
          xs[((i + 2) & 31) * XS + ((i + 2) >> 5)] = v[u].z;
          xs[((i + 3) & 31) * XS + ((i + 3) >> 5)] = v[u].w;
        }
      }
    }
  }
  __syncthreads();
  const bool onepass = nb <= 64;
  uint64_t xp[32];
  if (onepass) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      xp[j] = pack2(lane < nb ? xs[j * XS + lane] : 0.f, lane + 32 < nb ? xs[j * XS + lane + 32] : 0.f);
  }

  for (int k = 0; k < nspans; ++k) {
    const int r0 = k * span_rows;
    const int nr = min(span_rows, cnt - r0);
    const int qr = (nr + 3) / 4;
    const uint8_t *sbuf = buf0 + (size_t)(k & 1) * span_rows * rb;
    const uint32_t phase = (uint32_t)((k >> 1) & 1);
    int waited = -1;
    for (int r = warp; r < nr; r += NWARP) {
      const int q = r / qr;
      if (q != waited) {
        if (!mbar_wait_bounded(bar + (k & 1) * 4 + q, phase, err)) {
          abort_flag = 1;
          break;
        }
        waited = q;
      }
      const uint8_t *wrow = sbuf + (size_t)r * rb;
      for (int p = 0; p * 64 < nb; ++p) {
        const int b1 = p * 64 + lane, b2 = b1 + 32;
        const bool v1 = b1 < nb, v2 = b2 < nb;
        if (!onepass) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            xp[j] = pack2(v1 ? xs[j * XS + b1] : 0.f, v2 ? xs[j * XS + b2] : 0.f);
        }
        float d1, d2;
        uint32_t q1[8], q2[8];
        load_q8_block(wrow, 34 * (v1 ? b1 : 0), d1, q1);
        load_q8_block(wrow, 34 * (v2 ? b2 : 0), d2, q2);
        {
          float s1 = 0.f, s2 = 0.f;
          if (isfinite(d1) && isfinite(d2)) {
            const uint64_t dd = pack2(d1, d2);
            const uint64_t c1 = pack2(-kMagic * d1, -kMagic * d2);
            const uint64_t c2 = pack2(-128.0f * d1, -128.0f * d2);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint32_t u1 = q1[kk] ^ 0x80808080u, u2 = q2[kk] ^ 0x80808080u;
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const uint32_t sel = 0x7650u | (uint32_t)e;
                const float m1 = __uint_as_float(__byte_perm(u1, kMagicHi, sel));
                const float m2 = __uint_as_float(__byte_perm(u2, kMagicHi, sel));
                uint64_t t = fma2(pack2(m1, m2), dd, c1);
                t = add2(t, c2);
                float p1, p2;
                unpack2(mul2(t, xp[4 * kk + e]), p1, p2);
                s1 = __fadd_rn(s1, p1);
                s2 = __fadd_rn(s2, p2);
              }
            }
          } else {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float x1, x2;
                unpack2(xp[4 * kk + e], x1, x2);
                s1 = __fadd_rn(s1, __fmul_rn(__fmul_rn((float)(int8_t)(q1[kk] >> (8 * e)), d1), x1));
                s2 = __fadd_rn(s2, __fmul_rn(__fmul_rn((float)(int8_t)(q2[kk] >> (8 * e)), d2), x2));
              }
          }
          if (v1) bsum[r * BP + b1] = s1;
          if (v2) bsum[r * BP + b2] = s2;
        }
      }
    }
    __syncthreads();  // span buffer and block sums complete
    if (abort_flag) return;
    {
      // thread t adds the block sums of row t in block order (quant_math.hpp:56)
      for (int t = threadIdx.x; t < nr; t += NWARP * 32) {
        const float4 *b4 = reinterpret_cast<const float4 *>(bsum + t * BP);
        float s = 0.f;
        int b = 0;
        for (; b + 8 <= nb; b += 8) {
          const float4 a = b4[b / 4], c = b4[b / 4 + 1];
          s = __fadd_rn(s, a.x); s = __fadd_rn(s, a.y); s = __fadd_rn(s, a.z); s = __fadd_rn(s, a.w);
          s = __fadd_rn(s, c.x); s = __fadd_rn(s, c.y); s = __fadd_rn(s, c.z); s = __fadd_rn(s, c.w);
        }
        for (; b < nb; ++b) s = __fadd_rn(s, bsum[t * BP + b]);
        Y[n0 + r0 + t] = s;
      }
      __syncthreads();  // block sums consumed
    }
    if (k + 2 < nspans && threadIdx.x < 4) issue(k + 2);
  }
}

size_t span_smem_bytes(int K, int span_rows) {
  const int nb = K / 32;
  const int XS = (nb & 1) ? nb + 2 : nb + 1;
  const int BP = (nb + 4) & ~3;
  size_t s = 256 + (size_t)32 * XS * 4 + (size_t)span_rows * BP * 4;
  s = (s + 127) & ~size_t(127);
  // + slack: up to 127 bytes of alignment of the buffers, and the last block's
  // 9-word read may run 2 bytes past them
  return s + (size_t)2 * span_rows * nb * 34 + 256;
}

tb_status launch_span(const float *x, int64_t K, const void *w, int64_t N, float *y, cudaStream_t s,
                      const DeviceState *st) {
  constexpr int NWARP = 16;
  const int grid = (int)std::min<int64_t>(N, st->sm_count);
  const int64_t rows_per_cta = (N + grid - 1) / grid;
  int sr = (int)((rows_per_cta + 1) / 2);
  while (sr > 1 && span_smem_bytes((int)K, sr) > (size_t)st->smem_optin) --sr;
  const size_t smem = span_smem_bytes((int)K, sr);
  if (smem > (size_t)st->smem_optin) return fail(TB_EINVAL, "tb_matmul_quant: K=%lld too large", (long long)K);
  auto kern = gemv_q8_0_span_kernel<NWARP>;
  TB_TRY(ensure_smem_for(kern, smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(NWARP * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, (const uint8_t *)w, x, y, (int)N, (int)K, sr, st->err_word);
  if (e != cudaSuccess) return fail(TB_ECUDA, "tb_matmul_quant(Q8_0 span): %s", cudaGetErrorString(e));
  return TB_OK;
}

// ---------------------------------------------------------------------------
// Q4_0 weights times Q8_0-quantized activations, in the order of
// vec_dot_q4_0_q8_0_avx2 (quant_math.hpp:184-248): eight fp32 lanes, lane l
// accumulating, block after block, fma(p0, d, acc) then fma(p1, d, acc) where
// p0/p1 are the exact int pair sums of elements (2l, 2l+1) and (16+2l, 17+2l)
// and d = d_w * d_x; the eight lanes are then added in order.  Here the eight
// accumulators of one output are eight threads of a warp (4 outputs per warp).
template <int NW>
__global__ void __launch_bounds__(NW * 32) matmul_q4_0_kernel(
    const uint8_t *__restrict__ W, const uint8_t *__restrict__ XQ, float *__restrict__ Y, int N,
    int K, int M, int rows_per_cta, int use_tma, uint32_t *__restrict__ err, uint64_t wait_ns) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int nb = K / 32;
  const int rb = nb * 18;
  const int xb = nb * 34;
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem);
  uint8_t *xsm = smem + 128;
  uint8_t *wsm = xsm + ((xb + 127) & ~127);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int l = lane & 7, sub = lane >> 3;
  const int n0 = blockIdx.x * rows_per_cta;
  const int n1 = min(N, n0 + rows_per_cta);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  const int shift = stage_rows(W, (int64_t)n0 * rb, (int64_t)n1 * rb, wsm, bar, use_tma != 0);
  bool ready = false;
  for (int m = 0; m < M; ++m) {
    if (m > 0) __syncthreads();
    const uint8_t *xq = XQ + (int64_t)m * xb;
    for (int i = threadIdx.x; i < xb / 2; i += blockDim.x)
      reinterpret_cast<uint16_t *>(xsm)[i] = reinterpret_cast<const uint16_t *>(xq)[i];
    __syncthreads();
    if (!ready) {
      const bool ok = mbar_wait_limit(bar, 0, err, wait_ns);
      if (__syncthreads_or(!ok)) {
        // ERR_TIMEOUT is set; the weight copy may still be in flight into this
        // CTA's shared memory, so one thread waits for it (bounded) before the
        // CTA leaves.
        if (threadIdx.x == 0) mbar_wait_bounded(bar, 0, err);
        return;
      }
      ready = true;
    }
    for (int r0 = warp * 4; r0 < n1 - n0; r0 += NW * 4) {
      const int r = r0 + sub;
      const bool valid = r < n1 - n0;
      const uint8_t *wrow = wsm + shift + (valid ? r : 0) * rb;
      float acc = 0.f;
      for (int b = 0; b < nb; ++b) {
        const uint8_t *wbk = wrow + 18 * b;
        const uint8_t *xbk = xsm + 34 * b;
        const uint16_t wd = *reinterpret_cast<const uint16_t *>(wbk);
        const uint16_t w2 = *reinterpret_cast<const uint16_t *>(wbk + 2 + 2 * l);
        const uint16_t xd = *reinterpret_cast<const uint16_t *>(xbk);
        const uint16_t a01 = *reinterpret_cast<const uint16_t *>(xbk + 2 + 2 * l);
        const uint16_t a23 = *reinterpret_cast<const uint16_t *>(xbk + 18 + 2 * l);
        const float d = __fmul_rn(half_bits_to_float(wd), half_bits_to_float(xd));
        const int w00 = (int)(w2 & 0x0F) - 8, w01 = (int)((w2 >> 8) & 0x0F) - 8;
        const int w10 = (int)((w2 >> 4) & 0x0F) - 8, w11 = (int)(w2 >> 12) - 8;
        const int p0 = w00 * (int)(int8_t)(a01 & 0xFF) + w01 * (int)(int8_t)(a01 >> 8);
        const int p1 = w10 * (int)(int8_t)(a23 & 0xFF) + w11 * (int)(int8_t)(a23 >> 8);
        // |p| <= 2032: exact as 12582912 + p, then subtract the magic
        const float f0 = __fsub_rn(__int_as_float((int)kMagicHi + p0), kMagic);
        const float f1 = __fsub_rn(__int_as_float((int)kMagicHi + p1), kMagic);
        acc = __fmaf_rn(f0, d, acc);
        acc = __fmaf_rn(f1, d, acc);
      }
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) s = __fadd_rn(s, __shfl_sync(0xffffffffu, acc, (lane & ~7) + k));
      if (valid && l == 0) Y[(int64_t)m * N + n0 + r] = s;
    }
  }
}

size_t q8_smem_bytes(int K, int rows, int nw) {
  int nb = K / 32;
  int XS = (nb & 1) ? nb + 2 : nb + 1;
  size_t s = 128 + (size_t)32 * XS * 4 + (size_t)rows * ((nb + 4) & ~3) * 4;
  s = (s + 127) & ~size_t(127);
  s += (size_t)rows * nb * 34 + 32;
  (void)nw;
  return s;
}

size_t q4_smem_bytes(int K, int rows) {
  int nb = K / 32;
  return 128 + (size_t)((nb * 34 + 127) & ~127) + (size_t)rows * nb * 18 + 32;
}

}  // namespace

// Q8_0 matmul on CUDA cores.  M == 1 with aligned operands runs the
// pipelined GEMV (exact or fast arithmetic); everything else the one-shot
// kernel, which always follows the reference's order.
bool gemv_tc_eligible(int64_t K, int64_t N, const void *w, const float *x);
bool stream_gemv_fits(int64_t K, const DeviceState *st);

// The default M = 1 GEMV with a second copy of its outputs (PeerOut): the
// tensor-core GEMV for vocabulary-sized N, else the streaming GEMV.  TB_EINVAL
// when neither takes the operands.
tb_status launch_q8_0_gemv_peer(const float *x, int64_t K, const void *w, int64_t N, float *y, const PeerOut &peer,
                                cudaStream_t s, const DeviceState *st) {
  const int64_t rbytes = K / 32 * 34;
  if ((reinterpret_cast<uintptr_t>(w) & 15) != 0 || rbytes % 16 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0)
    return fail(TB_EINVAL, "row-sharded GEMV: W and x must be 16-byte aligned and K a multiple of 256");
  if (gemv_tc_eligible(K, N, w, x)) return launch_gemv_tc(x, K, w, N, y, s, st, &peer);
  if (stream_gemv_fits(K, st)) return launch_stream_gemv(x, K, w, N, y, s, st, &peer);
  return fail(TB_EINVAL, "row-sharded GEMV: K=%lld too large", (long long)K);
}

tb_status launch_q8_0(const float *x, int64_t M, int64_t K, const void *w, int64_t N, float *y,
                      bool exact, cudaStream_t s, const DeviceState *st) {
  const int64_t rbytes = K / 32 * 34;
  if (M == 1 && (reinterpret_cast<uintptr_t>(w) & 15) == 0 && rbytes % 16 == 0 &&
      (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    if (exact) return launch_span(x, K, w, N, y, s, st);
    if (gemv_tc_eligible(K, N, w, x)) return launch_gemv_tc(x, K, w, N, y, s, st);
    if (stream_gemv_fits(K, st)) return launch_stream_gemv(x, K, w, N, y, s, st);
  }
  constexpr int NW = 4;
  // ~36 KB of weights per CTA (a multiple of NW rows), several CTAs per SM.
  int rb = (int)(K / 32 * 34);
  int rows = std::max(NW, (36 * 1024 / rb) / NW * NW);
  rows = std::min(rows, 64);
  size_t smem = q8_smem_bytes((int)K, rows, NW);
  while (smem > (size_t)st->smem_optin && rows > NW) {
    rows -= NW;
    smem = q8_smem_bytes((int)K, rows, NW);
  }
  if (smem > (size_t)st->smem_optin) return fail(TB_EINVAL, "tb_matmul_quant: K=%lld too large", (long long)K);
  int use_tma = (reinterpret_cast<uintptr_t>(w) & 15) == 0;
  TB_TRY(ensure_smem_for(gemv_q8_0_kernel<NW>, smem));
  unsigned grid = (unsigned)((N + rows - 1) / rows);
  gemv_q8_0_kernel<NW><<<grid, NW * 32, smem, s>>>((const uint8_t *)w, x, y, (int)N, (int)K, (int)M,
                                                   rows, use_tma, st->err_word);
  return check_launch("tb_matmul_quant(Q8_0)");
}

tb_status launch_q4_0_exact(const uint8_t *xq, int64_t M, int64_t K, const void *w, int64_t N,
                            float *y, cudaStream_t s, const DeviceState *st) {
  constexpr int NW = 8;
  int rb = (int)(K / 32 * 18);
  int rows = std::max(NW * 4, (32 * 1024 / rb) / (NW * 4) * (NW * 4));
  size_t smem = q4_smem_bytes((int)K, rows);
  while (smem > (size_t)st->smem_optin && rows > 4) {
    rows -= 4;
    smem = q4_smem_bytes((int)K, rows);
  }
  if (smem > (size_t)st->smem_optin) return fail(TB_EINVAL, "tb_matmul_quant: K=%lld too large", (long long)K);
  int use_tma = (reinterpret_cast<uintptr_t>(w) & 15) == 0;
  TB_TRY(ensure_smem_for(matmul_q4_0_kernel<NW>, smem));
  unsigned grid = (unsigned)((N + rows - 1) / rows);
  matmul_q4_0_kernel<NW><<<grid, NW * 32, smem, s>>>((const uint8_t *)w, xq, y, (int)N, (int)K, (int)M,
                                                     rows, use_tma, st->err_word, wait_limit_ns());
  return check_launch("tb_matmul_quant(Q4_0)");
}

}  // namespace tb
