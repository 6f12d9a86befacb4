// tb_matmul_f32.cu -- batched strided fp32 matmul (A12): the attention score
// and context products of src/nn/attention.cpp:115-132 and fp32 Linear layers.
//
// Each output is the FMA chain over k = 0..K-1 in increasing order starting
// from 0, which is what the reference's packed AVX2 kernel computes per output
// element (src/tensor/tensor.cpp:503-538), so results are bit-identical.  The
// products are small in the decode path (K = head_dim = 64): there a CTA
// computes a 32x8 tile of outputs, one per thread, walking k in order.  From
// 32 rows and 32 columns on (prefill attention, fp32 Linear layers) a CTA
// computes a 64x64 tile with 4x4 outputs per thread (128x128 with 8x8 when
// there are at least as many such tiles as SMs): k-tiles of A and B
// are staged in shared memory (loaded along whichever of the view's strides is
// 1), the next k-tile is fetched into registers while the current one is
// used, and every output is still one fma chain over k in increasing order.
#include <algorithm>

#include "tb_internal.cuh"

namespace tb {
namespace {

struct MMView {
  int rank;
  int64_t batch, M, K, N;
  int64_t bshape[TB_MAX_RANK];
  int64_t sa_b[TB_MAX_RANK], sb_b[TB_MAX_RANK];
  int64_t sam, sak, sbk, sbn;
  int64_t oa, ob;
};

constexpr int TN = 32, TM = 8;

__global__ void __launch_bounds__(TN * TM) matmul_f32_kernel(const float *__restrict__ a,
                                                             const float *__restrict__ b,
                                                             float *__restrict__ out, MMView v) {
  const int64_t tiles_n = (v.N + TN - 1) / TN, tiles_m = (v.M + TM - 1) / TM;
  const int64_t tiles = v.batch * tiles_m * tiles_n;
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    int64_t bi = t / (tiles_m * tiles_n);
    int64_t rem = t % (tiles_m * tiles_n);
    int64_t m = (rem / tiles_n) * TM + threadIdx.y;
    int64_t n = (rem % tiles_n) * TN + threadIdx.x;
    int64_t ao = v.oa, bo = v.ob, tb_ = bi;
    for (int d = v.rank - 3; d >= 0; --d) {
      int64_t idx = tb_ % v.bshape[d];
      tb_ /= v.bshape[d];
      ao += idx * v.sa_b[d];
      bo += idx * v.sb_b[d];
    }
    if (m < v.M && n < v.N) {
      const float *ar = a + ao + m * v.sam;
      const float *bc = b + bo + n * v.sbn;
      float c = 0.f;
      int64_t k = 0;
      for (; k + 4 <= v.K; k += 4) {
        float a0 = __ldg(ar + k * v.sak), a1 = __ldg(ar + (k + 1) * v.sak);
        float a2 = __ldg(ar + (k + 2) * v.sak), a3 = __ldg(ar + (k + 3) * v.sak);
        float b0 = __ldg(bc + k * v.sbk), b1 = __ldg(bc + (k + 1) * v.sbk);
        float b2 = __ldg(bc + (k + 2) * v.sbk), b3 = __ldg(bc + (k + 3) * v.sbk);
        c = __fmaf_rn(a0, b0, c);
        c = __fmaf_rn(a1, b1, c);
        c = __fmaf_rn(a2, b2, c);
        c = __fmaf_rn(a3, b3, c);
      }
      for (; k < v.K; ++k) c = __fmaf_rn(__ldg(ar + k * v.sak), __ldg(bc + k * v.sbk), c);
      out[(bi * v.M + m) * v.N + n] = c;
    }
  }
}

// BT x BT output tile per CTA (BT = 64 or 128), 256 threads as 16 x 16:
// thread (ty, tx) owns R = BT / 16 rows and R columns, taken as R / 4 groups
// of four, BT / 2 apart (rows h BT/2 + 4 ty + 0..3, likewise columns), so that
// its shared-memory reads are float4s that a warp serves without bank
// conflicts.  A k-tile of A (BT x BK) and of B (BK x BT) is staged per step
// (BK = 16 for 64-wide tiles, 8 for 128-wide ones, to stay within 128 registers):
// thread i loads elements i + 256 j, mapped so that consecutive threads walk
// the view's unit-stride dimension (a_kfast: A's k stride is 1, else its m
// stride; b_nfast likewise), and the next k-tile is fetched into registers
// while the current one is used.
template <int BT, int BK>
__global__ void __launch_bounds__(256, BT == 128 ? 2 : 1) matmul_f32_tiled_kernel(const float *__restrict__ a,
                                                               const float *__restrict__ b,
                                                               float *__restrict__ out, MMView v, bool a_kfast,
                                                               bool b_nfast) {
  constexpr int R = BT / 16, H = R / 4, L = BT * BK / 256;  // outputs per side, groups, loads per operand
  __shared__ __align__(16) float As[BK][BT + 4];  // [k][m]
  __shared__ __align__(16) float Bs[BK][BT + 4];  // [k][n]
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t tiles_n = (v.N + BT - 1) / BT, tiles_m = (v.M + BT - 1) / BT;
  const int64_t tiles = v.batch * tiles_m * tiles_n;
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int64_t bi = t / (tiles_m * tiles_n), rem = t % (tiles_m * tiles_n);
    const int64_t m0 = (rem / tiles_n) * BT, n0 = (rem % tiles_n) * BT;
    int64_t ao = v.oa, bo = v.ob, tb_ = bi;
    for (int d = v.rank - 3; d >= 0; --d) {
      const int64_t idx = tb_ % v.bshape[d];
      tb_ /= v.bshape[d];
      ao += idx * v.sa_b[d];
      bo += idx * v.sb_b[d];
    }
    // this thread's L elements of A and of B in a k-tile: (m, k) and (k, n),
    // element i = tid + 256 j (recomputed where used, to save registers)
    auto am = [&](int j) { const int i = tid + 256 * j; return a_kfast ? i / BK : i % BT; };
    auto ak = [&](int j) { const int i = tid + 256 * j; return a_kfast ? i % BK : i / BT; };
    auto bn = [&](int j) { const int i = tid + 256 * j; return b_nfast ? i % BT : i / BK; };
    auto bk = [&](int j) { const int i = tid + 256 * j; return b_nfast ? i / BT : i % BK; };
    float ra[L], rb[L];
    auto fetch = [&](int64_t k0) {
#pragma unroll
      for (int j = 0; j < L; ++j) {
        const int64_t m = m0 + am(j), k = k0 + ak(j);
        ra[j] = (m < v.M && k < v.K) ? __ldg(a + ao + m * v.sam + k * v.sak) : 0.f;
        const int64_t kk = k0 + bk(j), n = n0 + bn(j);
        rb[j] = (kk < v.K && n < v.N) ? __ldg(b + bo + kk * v.sbk + n * v.sbn) : 0.f;
      }
    };
    float c[R][R];
#pragma unroll
    for (int i = 0; i < R; ++i)
#pragma unroll
      for (int j = 0; j < R; ++j) c[i][j] = 0.f;
    fetch(0);
    for (int64_t k0 = 0; k0 < v.K; k0 += BK) {
      __syncthreads();  // the previous k-tile's reads are done
#pragma unroll
      for (int j = 0; j < L; ++j) {
        As[ak(j)][am(j)] = ra[j];
        Bs[bk(j)][bn(j)] = rb[j];
      }
      __syncthreads();
      if (k0 + BK < v.K) fetch(k0 + BK);  // in flight while this k-tile is used
      const int kmax = (int)min((int64_t)BK, v.K - k0);
#pragma unroll 4
      for (int kk = 0; kk < kmax; ++kk) {
        float ar[R], br[R];
#pragma unroll
        for (int h = 0; h < H; ++h) {
          const float4 av = *reinterpret_cast<const float4 *>(&As[kk][h * (BT / 2) + 4 * ty]);
          const float4 bv = *reinterpret_cast<const float4 *>(&Bs[kk][h * (BT / 2) + 4 * tx]);
          ar[4 * h + 0] = av.x; ar[4 * h + 1] = av.y; ar[4 * h + 2] = av.z; ar[4 * h + 3] = av.w;
          br[4 * h + 0] = bv.x; br[4 * h + 1] = bv.y; br[4 * h + 2] = bv.z; br[4 * h + 3] = bv.w;
        }
#pragma unroll
        for (int i = 0; i < R; ++i)
#pragma unroll
          for (int j = 0; j < R; ++j) c[i][j] = __fmaf_rn(ar[i], br[j], c[i][j]);
      }
    }
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int64_t m = m0 + (i / 4) * (BT / 2) + 4 * ty + (i % 4);
      if (m >= v.M) continue;
      float *orow = out + (bi * v.M + m) * v.N;
#pragma unroll
      for (int j = 0; j < R; ++j) {
        const int64_t n = n0 + (j / 4) * (BT / 2) + 4 * tx + (j % 4);
        if (n < v.N) orow[n] = c[i][j];
      }
    }
    __syncthreads();  // shared tiles are reused by the CTA's next output tile
  }
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" tb_status tb_matmul_f32(const tb_view *a, const tb_view *b, const tb_view *out,
                                   tb_stream stream) {
  TB_TRY(validate_view(a, "tb_matmul_f32 a"));
  TB_TRY(validate_view(b, "tb_matmul_f32 b"));
  TB_TRY(validate_view(out, "tb_matmul_f32 out"));
  if (a->dtype != TB_F32 || b->dtype != TB_F32 || out->dtype != TB_F32)
    return fail(TB_EINVAL, "tb_matmul_f32: fp32 only");
  // Tensor::matmul checks (src/tensor/tensor.cpp:321-323, 434-455).
  if (a->rank < 2 || b->rank < 2) return fail(TB_EINVAL, "matmul requires at least 2D tensors");
  if (a->rank != b->rank) return fail(TB_EINVAL, "matmul requires both tensors to have the same rank");
  int r = a->rank;
  MMView v;
  v.rank = r;
  v.batch = 1;
  for (int i = 0; i < r - 2; ++i) {
    if (a->shape[i] != b->shape[i]) return fail(TB_EINVAL, "Batch dimensions must match");
    v.bshape[i] = a->shape[i];
    v.sa_b[i] = a->strides[i];
    v.sb_b[i] = b->strides[i];
    v.batch *= a->shape[i];
  }
  v.M = a->shape[r - 2];
  v.K = a->shape[r - 1];
  v.N = b->shape[r - 1];
  if (v.K != b->shape[r - 2]) return fail(TB_EINVAL, "Inner dimensions must match");
  if (out->rank != r || !is_contiguous(out)) return fail(TB_EINVAL, "tb_matmul_f32: out must be contiguous [batch..., M, N]");
  for (int i = 0; i < r - 2; ++i)
    if (out->shape[i] != a->shape[i]) return fail(TB_EINVAL, "tb_matmul_f32: out batch shape");
  if (out->shape[r - 2] != v.M || out->shape[r - 1] != v.N) return fail(TB_EINVAL, "tb_matmul_f32: out shape");
  v.sam = a->strides[r - 2];
  v.sak = a->strides[r - 1];
  v.sbk = b->strides[r - 2];
  v.sbn = b->strides[r - 1];
  v.oa = a->offset;
  v.ob = b->offset;
  if (v.batch * v.M * v.N == 0) return TB_OK;
  DeviceState *st;
  TB_TRY(device_state(&st));
  if (v.M >= 32 && v.N >= 32) {
    // 128x128 tiles where there is at least one per SM, else 64x64 ones
    const int64_t t128 = v.batch * ((v.M + 127) / 128) * ((v.N + 127) / 128);
    const float *pa = static_cast<const float *>(a->data), *pb = static_cast<const float *>(b->data);
    float *po = static_cast<float *>(out->data) + out->offset;
    if (t128 >= (int64_t)st->sm_count) {
      const int g = (int)std::min<int64_t>(t128, (int64_t)st->sm_count * 2);
      matmul_f32_tiled_kernel<128, 8><<<g, 256, 0, as_stream(stream)>>>(pa, pb, po, v, v.sak == 1, v.sbn == 1);
    } else {
      const int64_t t64 = v.batch * ((v.M + 63) / 64) * ((v.N + 63) / 64);
      const int g = (int)std::min<int64_t>(t64, (int64_t)st->sm_count * 8);
      matmul_f32_tiled_kernel<64, 16><<<g, 256, 0, as_stream(stream)>>>(pa, pb, po, v, v.sak == 1, v.sbn == 1);
    }
    return check_launch("tb_matmul_f32");
  }
  int64_t tiles = v.batch * ((v.M + TM - 1) / TM) * ((v.N + TN - 1) / TN);
  int grid = (int)std::min<int64_t>(tiles, (int64_t)st->sm_count * 16);
  matmul_f32_kernel<<<grid, dim3(TN, TM), 0, as_stream(stream)>>>(
      static_cast<const float *>(a->data), static_cast<const float *>(b->data),
      static_cast<float *>(out->data) + out->offset, v);
  return check_launch("tb_matmul_f32");
}
