// tb_decode_gemv.cu -- the decode step's matrix-vector products with their
// neighbours fused in, so that one 1B-shaped layer is six launches instead of
// sixteen:
//   tb_gemv_q8_0_multi    RMSNorm(x) * gamma (optional), then up to three
//                         weight matrices over the same input (Q, K, V) with an
//                         optional residual add per output (O + h, down + h)
//   tb_gemv_q8_0_swiglu   RMSNorm(x) * gamma (optional), then silu(G x) * (U x)
//   tb_rope_kv_append     RoPE of q and k at the device-held position and the
//                         key/value cache append, in one launch
// The GEMVs stream weights exactly as the ring GEMV does (spans of 8 rows per
// CTA through two shared-memory slots, two CTAs per SM, programmatic dependent
// launch) and compute each row with the same q8_row_dot; the fused prologue and
// epilogue use the formulas of tb_rmsnorm, tb_binary(add) and tb_swiglu, so a
// fused step differs from the op-by-op step only in the RMSNorm's sum order.
#include <algorithm>

#include "tb_internal.cuh"
#include "tb_q8_row.cuh"

namespace tb {
namespace {

constexpr int kFusedWarps = 8;
constexpr int kFusedSlots = 2;

struct FusedArgs {
  const uint8_t *w[3];
  float *y[3];
  const float *res[3];
  int n[3];
  int nseg;
  const float *x;
  const float *gamma;  // RMSNorm weight, or null
  float eps;
  int K;
};

// SWIGLU: segment 0 = gate, segment 1 = up (same rows), y[0] = silu(g) * u.
template <int NW, bool NORM, bool SWIGLU>
__global__ void __launch_bounds__(NW * 32) gemv_fused_kernel(const FusedArgs a, uint32_t *__restrict__ err) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int done[kFusedSlots];
  __shared__ int abort_flag;
  __shared__ float red[NW];
  __shared__ double tab[64];  // exp_cr table (SWIGLU epilogue)
  const int K = a.K, nb = K / 32, rb = nb * 34;
  const int XS = (nb & 1) ? nb + 2 : nb + 1;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  float *xs = reinterpret_cast<float *>(smem + 128);
  uint8_t *ring = reinterpret_cast<uint8_t *>(xs + 32 * XS);
  ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(ring) + 127) & ~uintptr_t(127));
  constexpr int kRowsPerSlot = SWIGLU ? 2 * NW : NW;
  const size_t slot_bytes = (size_t)kRowsPerSlot * rb;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  // logical rows: SWIGLU -> the gate/up row index; else segments back to back
  const int total = SWIGLU ? a.n[0] : a.n[0] + (a.nseg > 1 ? a.n[1] : 0) + (a.nseg > 2 ? a.n[2] : 0);
  const int G = gridDim.x, base = total / G, rem = total % G;
  const int n0 = blockIdx.x * base + min((int)blockIdx.x, rem);
  const int cnt = base + ((int)blockIdx.x < rem ? 1 : 0);
  const int nspans = (cnt + NW - 1) / NW;

  auto issue = [&](int k) {  // span k -> slot k % slots (one thread)
    const int slot = k % kFusedSlots;
    const int r0 = n0 + k * NW;
    const int nr = min(NW, cnt - k * NW);
    uint8_t *dst = ring + slot * slot_bytes;
    if (SWIGLU) {
      mbar_arrive_expect_tx(full + slot, (uint32_t)(2 * nr * rb));
      bulk_g2s(dst, a.w[0] + (int64_t)r0 * rb, (uint32_t)(nr * rb), full + slot);
      bulk_g2s(dst + (size_t)NW * rb, a.w[1] + (int64_t)r0 * rb, (uint32_t)(nr * rb), full + slot);
    } else {
      mbar_arrive_expect_tx(full + slot, (uint32_t)(nr * rb));
      int start = 0;
      for (int s = 0; s < a.nseg; ++s) {  // the span may cross segment boundaries
        const int lo = max(r0, start), hi = min(r0 + nr, start + a.n[s]);
        if (lo < hi)
          bulk_g2s(dst + (size_t)(lo - r0) * rb, a.w[s] + (int64_t)(lo - start) * rb, (uint32_t)((hi - lo) * rb),
                   full + slot);
        start += a.n[s];
      }
    }
  };
  if (threadIdx.x == 0) {
    for (int i = 0; i < kFusedSlots; ++i) {
      mbar_init(full + i, 1);
      done[i] = 0;
    }
    abort_flag = 0;
    fence_mbar_init();
    for (int k = 0; k < kFusedSlots && k < nspans; ++k) issue(k);
  }
  pdl_launch_dependents();
  if (SWIGLU) exp_cr_table_init(tab);  // visible after the barrier below
  pdl_wait();  // x and the residuals come from the previous kernel

  // x (RMS-normalised as tb_rmsnorm does when gamma is given) -> smem, transposed
  const float4 *x4 = reinterpret_cast<const float4 *>(a.x);
  const int nv = K >> 2;
  float rms = 1.f;
  if (NORM) {
    float ss = 0.f;
    for (int b4 = threadIdx.x; b4 < nv; b4 += NW * 32) {
      const float4 v = __ldg(x4 + b4);
      ss = __fadd_rn(ss, __fmul_rn(v.x, v.x));
      ss = __fadd_rn(ss, __fmul_rn(v.y, v.y));
      ss = __fadd_rn(ss, __fmul_rn(v.z, v.z));
      ss = __fadd_rn(ss, __fmul_rn(v.w, v.w));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float t = 0.f;
    for (int w = 0; w < NW; ++w) t = __fadd_rn(t, red[w]);
    rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)K), a.eps));
  }
  for (int b4 = threadIdx.x; b4 < nv; b4 += NW * 32) {
    float4 v = __ldg(x4 + b4);
    if (NORM) {
      const float4 g = __ldg(reinterpret_cast<const float4 *>(a.gamma) + b4);
      v.x = __fmul_rn(__fdiv_rn(v.x, rms), g.x);
      v.y = __fmul_rn(__fdiv_rn(v.y, rms), g.y);
      v.z = __fmul_rn(__fdiv_rn(v.z, rms), g.z);
      v.w = __fmul_rn(__fdiv_rn(v.w, rms), g.w);
    }
    const int i = b4 * 4;
    xs[((i + 0) & 31) * XS + ((i + 0) >> 5)] = v.x;
    xs[((i + 1) & 31) * XS + ((i + 1) >> 5)] = v.y;
    xs[((i + 2) & 31) * XS + ((i + 2) >> 5)] = v.z;
    xs[((i + 3) & 31) * XS + ((i + 3) >> 5)] = v.w;
  }
  __syncthreads();
  uint64_t xp[32];
  if (nb <= 64) q8_load_xp(xp, xs, XS, nb, 0, lane);

  for (int k = 0; k < nspans; ++k) {
    const int slot = k % kFusedSlots;
    const int nr = min(NW, cnt - k * NW);
    if (warp < nr) {
      const bool ok =
          !*(volatile int *)&abort_flag && mbar_wait_bounded(full + slot, (uint32_t)((k / kFusedSlots) & 1), err);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) abort_flag = 1;
        return;
      }
      const uint8_t *wrow = ring + slot * slot_bytes + (size_t)warp * rb;
      const int r = n0 + k * NW + warp;
      if (SWIGLU) {
        const float g = q8_row_dot(wrow, nb, xp, xs, XS, lane);
        const float u = q8_row_dot(wrow + (size_t)NW * rb, nb, xp, xs, XS, lane);
        if (lane == 0) a.y[0][r] = swiglu_f32(g, u, tab);
      } else {
        const float v = q8_row_dot(wrow, nb, xp, xs, XS, lane);
        if (lane == 0) {
          int s = 0, start = 0;
          while (s + 1 < a.nseg && r >= start + a.n[s]) start += a.n[s++];
          const int i = r - start;
          a.y[s][i] = a.res[s] ? __fadd_rn(a.res[s][i], v) : v;
        }
      }
      // the last of the span's nr warps refills the slot (only warps that
      // waited for the span count; see gemv_q8_0_ring_kernel)
      if (lane == 0) {
        __threadfence_block();
        if (atomicAdd(&done[slot], 1) == nr - 1) {
          done[slot] = 0;
          if (k + kFusedSlots < nspans) {
            fence_proxy_async_smem();
            issue(k + kFusedSlots);
          }
        }
      }
      __syncwarp();
    }
  }
}

size_t fused_smem_bytes(int K, bool swiglu) {
  const int nb = K / 32;
  const int XS = (nb & 1) ? nb + 2 : nb + 1;
  size_t s = 128 + (size_t)32 * XS * 4;
  s = (s + 127) & ~size_t(127);
  return s + (size_t)kFusedSlots * (swiglu ? 2 : 1) * kFusedWarps * nb * 34 + 128;
}

template <bool NORM, bool SWIGLU>
tb_status launch_fused(const FusedArgs &a, int total_rows, cudaStream_t s, const DeviceState *st) {
  const size_t smem = fused_smem_bytes(a.K, SWIGLU);
  if (smem > (size_t)st->smem_optin) return fail(TB_EINVAL, "fused GEMV: K=%d too large", a.K);
  const int cps = 2 * smem <= (size_t)st->smem_optin ? 2 : 1;
  const int grid = std::max(1, std::min(total_rows, st->sm_count * cps));
  auto kern = gemv_fused_kernel<kFusedWarps, NORM, SWIGLU>;
  TB_TRY(ensure_smem_for(kern, smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(kFusedWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a, st->err_word);
  if (e != cudaSuccess) return fail(TB_ECUDA, "fused GEMV launch: %s", cudaGetErrorString(e));
  return TB_OK;
}

tb_status check_gemv_input(const float *x, int64_t K, const float *gamma, const void *w, const char *who) {
  if (K <= 0 || K % 32 != 0 || K > 65536) return fail(TB_EINVAL, "%s: K=%lld must be a positive multiple of 32", who, (long long)K);
  if ((K / 32 * 34) % 16 != 0) return fail(TB_EINVAL, "%s: rows of K=%lld are not 16-byte multiples", who, (long long)K);
  if (!x || ((reinterpret_cast<uintptr_t>(x) & 15) != 0)) return fail(TB_EINVAL, "%s: x must be 16-byte aligned", who);
  if (gamma && (reinterpret_cast<uintptr_t>(gamma) & 15) != 0) return fail(TB_EINVAL, "%s: gamma must be 16-byte aligned", who);
  if (!w || (reinterpret_cast<uintptr_t>(w) & 15) != 0) return fail(TB_EINVAL, "%s: weights must be 16-byte aligned", who);
  return TB_OK;
}

// RoPE (rope_kernel's arithmetic) of q [H, D] and k [KVH, D] at position
// *pos, then k and v into the caches' row pos.  One thread per rotated pair of
// q or k, plus the value copy.
__global__ void rope_kv_kernel(float *__restrict__ q, float *__restrict__ k, const float *__restrict__ v, int H,
                               int KVH, int D, const float *__restrict__ cos_t, const float *__restrict__ sin_t,
                               int rope_max_seq, float *__restrict__ kc, float *__restrict__ vc, int max_seq,
                               const int32_t *__restrict__ pos_dev, uint32_t *__restrict__ err) {
  const int pos = *pos_dev;
  if (pos < 0 || pos >= max_seq || pos >= rope_max_seq) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(err, ERR_INDEX);
    return;
  }
  const int half = D / 2;
  const int nq = H * half, nk = KVH * half, row = KVH * D;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t < nq + nk) {
    const bool isq = t < nq;
    const int u = isq ? t : t - nq;
    const int h = u / half, i = u % half;
    float *base = (isq ? q : k) + h * D;
    const float c = __ldg(cos_t + (int64_t)pos * half + i), s = __ldg(sin_t + (int64_t)pos * half + i);
    const float x0 = base[i], x1 = base[i + half];
    const float y0 = __fmaf_rn(x0, c, -__fmul_rn(x1, s));
    const float y1 = __fmaf_rn(x0, s, __fmul_rn(x1, c));
    base[i] = y0;
    base[i + half] = y1;
    if (!isq) {
      kc[(int64_t)pos * row + h * D + i] = y0;
      kc[(int64_t)pos * row + h * D + i + half] = y1;
    }
  } else if (t < nq + nk + row) {
    const int j = t - nq - nk;
    vc[(int64_t)pos * row + j] = v[j];
  }
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" {

tb_status tb_gemv_q8_0_multi(const float *x, int64_t K, const float *gamma, float eps, const tb_gemv_segment *segs,
                             int nseg, tb_stream stream) {
  if (nseg < 1 || nseg > 3 || !segs) return fail(TB_EINVAL, "tb_gemv_q8_0_multi: 1 to 3 segments");
  FusedArgs a = {};
  int64_t total = 0;
  for (int s = 0; s < nseg; ++s) {
    TB_TRY(check_gemv_input(x, K, gamma, segs[s].w, "tb_gemv_q8_0_multi"));
    if (segs[s].n <= 0 || !segs[s].y) return fail(TB_EINVAL, "tb_gemv_q8_0_multi: segment %d has no rows or output", s);
    a.w[s] = static_cast<const uint8_t *>(segs[s].w);
    a.y[s] = segs[s].y;
    a.res[s] = segs[s].residual;
    a.n[s] = (int)segs[s].n;
    total += segs[s].n;
  }
  if (total > 0x7FFFFFFF) return fail(TB_EINVAL, "tb_gemv_q8_0_multi: too many rows");
  a.nseg = nseg;
  a.x = x;
  a.gamma = gamma;
  a.eps = eps;
  a.K = (int)K;
  DeviceState *st;
  TB_TRY(device_state(&st));
  cudaStream_t s = as_stream(stream);
  return gamma ? launch_fused<true, false>(a, (int)total, s, st) : launch_fused<false, false>(a, (int)total, s, st);
}

tb_status tb_gemv_q8_0_swiglu(const float *x, int64_t K, const float *gamma, float eps, const void *w_gate,
                              const void *w_up, int64_t n, float *y, tb_stream stream) {
  TB_TRY(check_gemv_input(x, K, gamma, w_gate, "tb_gemv_q8_0_swiglu"));
  TB_TRY(check_gemv_input(x, K, gamma, w_up, "tb_gemv_q8_0_swiglu"));
  if (n <= 0 || n > 0x7FFFFFFF || !y) return fail(TB_EINVAL, "tb_gemv_q8_0_swiglu: bad rows or output");
  FusedArgs a = {};
  a.w[0] = static_cast<const uint8_t *>(w_gate);
  a.w[1] = static_cast<const uint8_t *>(w_up);
  a.n[0] = a.n[1] = (int)n;
  a.y[0] = y;
  a.nseg = 2;
  a.x = x;
  a.gamma = gamma;
  a.eps = eps;
  a.K = (int)K;
  DeviceState *st;
  TB_TRY(device_state(&st));
  cudaStream_t s = as_stream(stream);
  return gamma ? launch_fused<true, true>(a, (int)n, s, st) : launch_fused<false, true>(a, (int)n, s, st);
}

tb_status tb_rope_kv_append(float *q, float *k, const float *v, int64_t heads, int64_t kv_heads, int64_t head_dim,
                            const float *cos_dev, const float *sin_dev, int64_t rope_max_seq, float *k_cache,
                            float *v_cache, int64_t max_seq, const int32_t *pos_dev, tb_stream stream) {
  if (heads <= 0 || kv_heads <= 0 || head_dim <= 0 || head_dim % 2 != 0 || max_seq <= 0 || rope_max_seq <= 0)
    return fail(TB_EINVAL, "tb_rope_kv_append: bad extents");
  if (heads * head_dim > (1 << 24)) return fail(TB_EINVAL, "tb_rope_kv_append: too many heads");
  if (!q || !k || !v || !cos_dev || !sin_dev || !k_cache || !v_cache || !pos_dev)
    return fail(TB_EINVAL, "tb_rope_kv_append: null pointer");
  DeviceState *st;
  TB_TRY(device_state(&st));
  const int threads = (int)((heads + kv_heads) * head_dim / 2 + kv_heads * head_dim);
  rope_kv_kernel<<<(threads + 255) / 256, 256, 0, as_stream(stream)>>>(
      q, k, v, (int)heads, (int)kv_heads, (int)head_dim, cos_dev, sin_dev, (int)rope_max_seq, k_cache, v_cache,
      (int)max_seq, pos_dev, st->err_word);
  return check_launch("tb_rope_kv_append");
}

}  // extern "C"
