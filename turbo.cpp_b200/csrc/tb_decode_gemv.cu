// tb_decode_gemv.cu -- the decode step's matrix-vector products with their
// neighbours fused in, so that one 1B-shaped layer is six launches instead of
// sixteen:
//   tb_gemv_q8_0_multi    RMSNorm(x) * gamma (optional), then up to three
//                         weight matrices over the same input (Q, K, V) with an
//                         optional residual add per output (O + h, down + h)
//   tb_gemv_q8_0_swiglu   RMSNorm(x) * gamma (optional), then silu(G x) * (U x)
//   tb_rope_kv_append     RoPE of q and k at the device-held position and the
//                         key/value cache append, in one launch
//   tb_prefetch_l2        background L2 fills of weights a later kernel reads
// All of them, and tb_matmul_quant's default M = 1 Q8_0 path below the LM-head
// size, run gemv_stream_kernel (below); the fused prologue and epilogue use the
// formulas of tb_rmsnorm, tb_binary(add) and tb_swiglu, so a fused step differs
// from the op-by-op step only in the RMSNorm's sum order.
#include <algorithm>

#include "tb_internal.cuh"
#include "tb_q8_row.cuh"

namespace tb {
namespace {

constexpr int kStreamWarps = 4;     // rows per span (one per warp); 4 CTAs per SM
constexpr int kWideWarps = 16;      // the plain GEMV: one CTA of 16 warps per SM
constexpr int kStreamMaxSlots = 16;

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
  int slots;  // span buffers per CTA (kStreamMaxSlots at most)
  PeerOut peer;  // single segment, no residual: a second copy of the outputs (peer.dst)
};

// Streaming Q8_0 GEMV (M = 1), default tolerance.  Each CTA owns a contiguous
// range of logical rows, cut into spans of kStreamWarps rows (one per warp;
// SWIGLU: the gate rows and the up rows of the same indices).  Spans stream
// through `slots` shared-memory buffers, one bulk copy per span and segment and
// one mbarrier per buffer; when every span of the CTA fits (the common decode
// case) all copies are in flight once x is staged, otherwise the last warp to
// finish a span refills its buffer with the span `slots` ahead.
// Small CTAs, four per SM, so that rows are spread finely over the GPU and the
// warps' issue slots, not one CTA's latency chain, bound the compute.
// Programmatic dependent launch: the first span's copy (and the RMSNorm
// weight) is issued before griddepcontrol.wait, since weights never depend on
// the previous kernel; after the wait every thread issues its loads of x and
// only then do the other spans' copies go out (8192 x 2048: 5.35 against
// 5.71 us per launch with the copies issued after x had landed).
// SWIGLU: segment 0 = gate, segment 1 = up (same rows), y[0] = silu(g) * u.
template <int NW, bool NORM, bool SWIGLU, bool DIG>
__global__ void __launch_bounds__(NW * 32, 16 / NW) gemv_stream_kernel(const FusedArgs a,
                                                                      uint32_t *__restrict__ err) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int done[kStreamMaxSlots];
  __shared__ int abort_flag;
  __shared__ int dig_special;  // DIG: a block of x needs the fp32 dot
  __shared__ float red[NW];
  __shared__ double tab[SWIGLU ? 64 : 1];  // exp_cr table (SWIGLU epilogue)
  const int K = a.K, nb = K / 32, rb = nb * 34;
  const int XS = nb + 2;  // even: a lane's x pair is one 8-byte load
  const int slots = a.slots;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);  // [kStreamMaxSlots]
  float *xs = reinterpret_cast<float *>(smem + 8 * kStreamMaxSlots);
  uint8_t *ring = reinterpret_cast<uint8_t *>(xs + 32 * XS + (DIG ? 3 * 16 * 32 + 64 : 0));
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
    const int slot = k % slots;
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
#pragma unroll
      for (int s = 0; s < 3; ++s) {  // the span may cross segment boundaries
        if (s < a.nseg) {
          const int lo = max(r0, start), hi = min(r0 + nr, start + a.n[s]);
          if (lo < hi)
            bulk_g2s(dst + (size_t)(lo - r0) * rb, a.w[s] + (int64_t)(lo - start) * rb,
                     (uint32_t)((hi - lo) * rb), full + slot);
          start += a.n[s];
        }
      }
    }
  };
  int64_t pbuf = 0;  // the exchange buffer of this call (set after griddepcontrol.wait)
  // logical row r's output: y[r] of its segment, plus the segment's residual
  auto store = [&](int r, float v) {
    int i = r;
    float *y = a.y[0];
    const float *res = a.res[0];
    if (a.nseg > 1 && i >= a.n[0]) {
      i -= a.n[0];
      y = a.y[1];
      res = a.res[1];
      if (a.nseg > 2 && i >= a.n[1]) {
        i -= a.n[1];
        y = a.y[2];
        res = a.res[2];
      }
    }
    const float o = res ? __fadd_rn(res[i], v) : v;
    y[i] = o;
    peer_store(a.peer, pbuf, i, o);
  };
  if (threadIdx.x == 0) {
    for (int i = 0; i < slots; ++i) {
      mbar_init(full + i, 1);
      done[i] = 0;
    }
    abort_flag = 0;
    dig_special = 0;
    fence_mbar_init();
    if (nspans > 0) issue(0);  // the rest once x's loads are issued (below)
  }
  pdl_launch_dependents();
  if (SWIGLU) exp_cr_table_init(tab);  // visible after the barrier below
  // A thread's first kXReg float4s of x (and of gamma) are held in registers:
  // gamma is a weight and is loaded before the wait; x's loads are issued right
  // after it, ahead of the CTA's remaining weight copies, so that they do not
  // queue behind them, and neither RMSNorm pass reloads them.
  constexpr int kXReg = 4;
  const float4 *x4 = reinterpret_cast<const float4 *>(a.x);
  const int nv = K >> 2;
  float4 gv[NORM ? kXReg : 1];
  if (NORM) {
#pragma unroll
    for (int i = 0; i < kXReg; ++i) {
      const int b4 = (int)threadIdx.x + i * NW * 32;
      gv[i] = b4 < nv ? __ldg(reinterpret_cast<const float4 *>(a.gamma) + b4) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  pdl_wait();  // x and the residuals come from the previous kernel
  float4 xv[kXReg];
#pragma unroll
  for (int i = 0; i < kXReg; ++i) {
    const int b4 = (int)threadIdx.x + i * NW * 32;
    xv[i] = b4 < nv ? __ldg(x4 + b4) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (threadIdx.x == 0)
    for (int k = 1; k < slots && k < nspans; ++k) issue(k);
  pbuf = peer_buffer(a.peer);

  // x (RMS-normalised as tb_rmsnorm does when gamma is given) -> smem, transposed
  float rms = 1.f;
  if (NORM) {
    float ss = 0.f;
    auto sq = [&](const float4 v) {
      ss = __fadd_rn(ss, __fmul_rn(v.x, v.x));
      ss = __fadd_rn(ss, __fmul_rn(v.y, v.y));
      ss = __fadd_rn(ss, __fmul_rn(v.z, v.z));
      ss = __fadd_rn(ss, __fmul_rn(v.w, v.w));
    };
#pragma unroll
    for (int i = 0; i < kXReg; ++i)
      if ((int)threadIdx.x + i * NW * 32 < nv) sq(xv[i]);
    for (int b4 = threadIdx.x + kXReg * NW * 32; b4 < nv; b4 += NW * 32) sq(__ldg(x4 + b4));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float t = 0.f;
    for (int w = 0; w < NW; ++w) t = __fadd_rn(t, red[w]);
    rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)K), a.eps));
  }
  auto put = [&](int b4, float4 v, float4 g) {
    if (NORM) {
      v.x = __fmul_rn(__fdiv_rn(v.x, rms), g.x);
      v.y = __fmul_rn(__fdiv_rn(v.y, rms), g.y);
      v.z = __fmul_rn(__fdiv_rn(v.z, rms), g.z);
      v.w = __fmul_rn(__fdiv_rn(v.w, rms), g.w);
    }
    const int j = b4 * 4;
    xs[((j + 0) & 31) * XS + ((j + 0) >> 5)] = v.x;
    xs[((j + 1) & 31) * XS + ((j + 1) >> 5)] = v.y;
    xs[((j + 2) & 31) * XS + ((j + 2) >> 5)] = v.z;
    xs[((j + 3) & 31) * XS + ((j + 3) >> 5)] = v.w;
  };
#pragma unroll
  for (int i = 0; i < kXReg; ++i) {
    const int b4 = (int)threadIdx.x + i * NW * 32;
    if (b4 < nv) put(b4, xv[i], gv[NORM ? i : 0]);
  }
  for (int b4 = threadIdx.x + kXReg * NW * 32; b4 < nv; b4 += NW * 32)
    put(b4, __ldg(x4 + b4), NORM ? __ldg(reinterpret_cast<const float4 *>(a.gamma) + b4) : make_float4(0.f, 0.f, 0.f, 0.f));
  __syncthreads();
  // DIG (K = 2048, one block pair per lane): x as int8 digits and dp4a row
  // dots, unless a block of x cannot be written so (then the whole CTA takes
  // the fp32 dot)
  bool use_dig = false;
  uint32_t *dgs = reinterpret_cast<uint32_t *>(xs + 32 * XS);  // DIG: [3][16][32] digits, then sx[64]
  float *sxs = reinterpret_cast<float *>(dgs + 3 * 16 * 32);
  if (DIG) {
    const int t = threadIdx.x;  // threads 0-127 (whole warps): half a block each
    if (t < 128 && q8_make_digits(xs, XS, t >> 1, t & 1, dgs, sxs)) atomicOr(&dig_special, 1);
    __syncthreads();
    use_dig = *(volatile int *)&dig_special == 0;
  }

  // Runs the CTA's spans with row dot `dot(wrow)` (every lane returns it).
  auto spans = [&](auto &&dot) {
  for (int k = 0; k < nspans; ++k) {
    const int slot = k % slots;
    const int nr = min(NW, cnt - k * NW);
    if (warp < nr) {
      const bool ok =
          !*(volatile int *)&abort_flag && mbar_wait_bounded(full + slot, (uint32_t)((k / slots) & 1), err);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) abort_flag = 1;
        return;
      }
      const uint8_t *wrow = ring + slot * slot_bytes + (size_t)warp * rb;
      const int r = n0 + k * NW + warp;
      if (SWIGLU) {
        const float g = dot(wrow);
        const float u = dot(wrow + (size_t)NW * rb);
        if (lane == 0) a.y[0][r] = swiglu_f32(g, u, tab);
      } else {
        const float v = dot(wrow);
        if (lane == 0) store(r, v);
      }
      // With a ring (nspans > slots), the last of the span's nr warps refills
      // the slot with span k + slots.  Only warps that waited for this span
      // count: a warp without a row (only in the last, partial span) must not
      // touch a counter, or it could run ahead and count toward a span that is
      // still being read.
      if (nspans > slots && lane == 0) {
        __threadfence_block();
        if (atomicAdd(&done[slot], 1) == nr - 1) {
          done[slot] = 0;
          if (k + slots < nspans) {
            fence_proxy_async_smem();
            issue(k + slots);
          }
        }
      }
      __syncwarp();
    }
  }
  };
  if (use_dig) {
    uint32_t dgr[3][16];
    float sxr[2];
#pragma unroll
    for (int j = 0; j < 3; ++j)
#pragma unroll
      for (int i = 0; i < 16; ++i) dgr[j][i] = dgs[(j * 16 + i) * 32 + lane];
    sxr[0] = sxs[2 * lane];
    sxr[1] = sxs[2 * lane + 1];
    spans([&](const uint8_t *wrow) { return q8_row_dot_digits(wrow, dgr, sxr, lane); });
  } else {
    float2 xp[32];
    if (nb <= 64) q8_pair_x(xp, xs, XS, 2 * lane, 2 * lane < nb);
    spans([&](const uint8_t *wrow) { return q8_row_dot_pairs(wrow, nb, xp, xs, XS, lane); });
  }
}

size_t stream_fixed_smem(int K, bool dig = false) {
  const int nb = K / 32;
  const size_t s = 8 * kStreamMaxSlots + (size_t)32 * (nb + 2) * 4 + (dig ? (3 * 16 * 32 + 64) * 4 : 0);
  return (s + 127) & ~size_t(127);
}

template <int NW, bool NORM, bool SWIGLU, bool DIG>
tb_status launch_stream_as(FusedArgs a, int grid, size_t smem, cudaStream_t s, const DeviceState *st) {
  auto kern = gemv_stream_kernel<NW, NORM, SWIGLU, DIG>;
  TB_TRY(ensure_smem_for(kern, smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(NW * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a, st->err_word);
  if (e != cudaSuccess) return fail(TB_ECUDA, "streaming GEMV launch: %s", cudaGetErrorString(e));
  return TB_OK;
}

// Grid and span buffers: four CTAs per SM when at least two buffers (or all
// the CTA's spans) fit in a quarter of the SM's shared memory, else fewer CTAs
// per SM; then as many buffers as the CTA has spans, up to what fits.  At
// K = 2048 with at least kDigitRows rows per CTA the row dots take x as int8
// digits (dp4a); below that the per-CTA digit preparation costs more than it
// saves (2048 x 2048: 3.6 against 3.1 us; 8192 x 2048: 5.1 against 6.2 us,
// lab copies timed back to back).
constexpr int kDigitRows = 8;

template <int NW, bool NORM, bool SWIGLU>
tb_status launch_stream(FusedArgs a, int total_rows, cudaStream_t s, const DeviceState *st) {
  const int nb = a.K / 32;
  const size_t slot_bytes = (size_t)(SWIGLU ? 2 : 1) * NW * nb * 34;
  for (int dig = nb == 64 ? 1 : 0; dig >= 0; --dig) {
    const size_t fixed = stream_fixed_smem(a.K, dig != 0);
    int cps = 16 / NW, slots = 0, grid = 1, maxcnt = 0;
    for (; cps >= 1; --cps) {
      grid = std::max(1, std::min(total_rows, st->sm_count * cps));
      maxcnt = (total_rows + grid - 1) / grid;
      const int nspans = (maxcnt + NW - 1) / NW;
      const int64_t budget = std::min<int64_t>((int64_t)st->smem_per_sm / cps - st->smem_reserved - 2048,
                                               (int64_t)st->smem_optin) - (int64_t)fixed;
      const int fit = budget > 0 ? (int)std::min<int64_t>(budget / (int64_t)slot_bytes, kStreamMaxSlots) : 0;
      slots = std::min(nspans, fit);
      if (slots >= std::min(nspans, 2)) break;
    }
    if (cps < 1 || slots < 1) {
      if (dig) continue;
      return fail(TB_EINVAL, "streaming GEMV: K=%d too large", a.K);
    }
    if (dig && maxcnt < kDigitRows) continue;
    a.slots = slots;
    const size_t smem = fixed + (size_t)slots * slot_bytes;
    return dig ? launch_stream_as<NW, NORM, SWIGLU, true>(a, grid, smem, s, st)
               : launch_stream_as<NW, NORM, SWIGLU, false>(a, grid, smem, s, st);
  }
  return fail(TB_EINVAL, "streaming GEMV: K=%d too large", a.K);
}

// One 16-warp CTA per SM when every warp has a row and two span buffers fit
// (x is then staged, and turned into digits, once per SM instead of four
// times: 8192 x 2048, 5.7 against 5.9 us), else four 4-warp CTAs per SM.
template <bool NORM, bool SWIGLU>
tb_status launch_stream_auto(const FusedArgs &a, int total_rows, cudaStream_t s, const DeviceState *st) {
  const int grid = std::min(total_rows, st->sm_count);
  const int64_t per = (total_rows + grid - 1) / grid, nspans = (per + kWideWarps - 1) / kWideWarps;
  const size_t need = stream_fixed_smem(a.K, a.K == 2048) +
                      (size_t)std::min<int64_t>(nspans, 2) * (SWIGLU ? 2 : 1) * kWideWarps * (a.K / 32) * 34;
  if (2 * per >= kWideWarps && need <= (size_t)st->smem_optin)
    return launch_stream<kWideWarps, NORM, SWIGLU>(a, total_rows, s, st);
  return launch_stream<kStreamWarps, NORM, SWIGLU>(a, total_rows, s, st);
}

}  // namespace

// Whether one span buffer and x fit in a CTA's shared memory at this K.
bool stream_gemv_fits(int64_t K, const DeviceState *st) {
  if (K <= 0 || K % 256 != 0 || K > 65536) return false;
  return stream_fixed_smem((int)K) + (size_t)2 * kStreamWarps * (K / 32) * 34 <= (size_t)st->smem_optin;
}

// tb_matmul_quant(Q8_0), M = 1, default tolerance: one weight matrix, no norm,
// no residual.  Operands as check_gemv_input requires (the caller checks).
tb_status launch_stream_gemv(const float *x, int64_t K, const void *w, int64_t N, float *y, cudaStream_t s,
                             const DeviceState *st, const PeerOut *peer) {
  if (N <= 0 || N > 0x7FFFFFFF) return fail(TB_EINVAL, "tb_matmul_quant: N=%lld out of range", (long long)N);
  FusedArgs a = {};
  if (peer) a.peer = *peer;
  a.w[0] = static_cast<const uint8_t *>(w);
  a.y[0] = y;
  a.n[0] = (int)N;
  a.nseg = 1;
  a.x = x;
  a.K = (int)K;
  return launch_stream_auto<false, false>(a, (int)N, s, st);
}

namespace {

struct PrefetchRanges {
  const uint8_t *p[8];
  int64_t n[8];  // bytes, multiples of 16
  int count;
};

// One warp: lane i issues the 1 MiB chunks i, i + 32, ... of the ranges in
// turn; the L2 fills continue after the kernel exits.  griddepcontrol.wait at
// the end makes this kernel's completion imply its predecessor's, so the next
// kernel's own wait still orders it after every earlier kernel.
__global__ void __launch_bounds__(32) prefetch_l2_kernel(const PrefetchRanges r) {
  pdl_launch_dependents();
  constexpr int64_t kChunk = 1 << 20;
  for (int i = 0; i < r.count; ++i) {
    const int64_t chunks = (r.n[i] + kChunk - 1) / kChunk;
    for (int64_t c = threadIdx.x; c < chunks; c += 32) {
      const int64_t off = c * kChunk;
      const uint32_t len = (uint32_t)(r.n[i] - off < kChunk ? r.n[i] - off : kChunk);
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(r.p[i] + off), "r"(len) : "memory");
    }
  }
  pdl_wait();
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
  return gamma ? launch_stream_auto<true, false>(a, (int)total, s, st)
               : launch_stream_auto<false, false>(a, (int)total, s, st);
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
  return gamma ? launch_stream_auto<true, true>(a, (int)n, s, st)
               : launch_stream_auto<false, true>(a, (int)n, s, st);
}

tb_status tb_prefetch_l2(const void *const *ptrs, const int64_t *bytes, int n, tb_stream stream) {
  if (n < 0 || n > 8 || (n > 0 && (!ptrs || !bytes))) return fail(TB_EINVAL, "tb_prefetch_l2: 0 to 8 ranges");
  PrefetchRanges r = {};
  for (int i = 0; i < n; ++i) {
    if (bytes[i] < 0) return fail(TB_EINVAL, "tb_prefetch_l2: negative size");
    const uintptr_t a = reinterpret_cast<uintptr_t>(ptrs[i]);
    const uintptr_t lo = (a + 15) & ~uintptr_t(15), hi = (a + (uintptr_t)bytes[i]) & ~uintptr_t(15);
    if (!ptrs[i] || hi <= lo) continue;
    r.p[r.count] = reinterpret_cast<const uint8_t *>(lo);
    r.n[r.count] = (int64_t)(hi - lo);
    ++r.count;
  }
  if (r.count == 0) return TB_OK;
  DeviceState *st;
  TB_TRY(device_state(&st));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, 1);
  cfg.blockDim = dim3(32, 1, 1);
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, prefetch_l2_kernel, r);
  if (e != cudaSuccess) return fail(TB_ECUDA, "tb_prefetch_l2: %s", cudaGetErrorString(e));
  return TB_OK;
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
