// tb_gemm_f16.cu -- the quantized prefill matmul (M >= 32) on the tensor cores,
// kind::f16 with fp32 accumulation in tensor memory.
//
// Arithmetic.  Y[m, n] = sum over 32-wide blocks b of d_w[n, b] * s[m, b] *
// T[n, m, b], with T the block's dot product of small exact numbers:
//   weights  the block's quants as fp16, exact: q (Q8_0) or q - 8 (Q4_0);
//   Q8_0     X kept to 22 bits: per (token, block) a power of two 2^e puts
//            max|x| in [2^14, 2^15), and x * 2^e = hi + lo with hi, lo fp16
//            (s = 2^-e); T = q . hi + q . lo, both products exact in fp32;
//   Q4_0     X quantised to Q8_0 exactly as the reference does
//            (quantize_row_q8_0, src/tensor/quant_math.hpp:68-90; s = its
//            fp16 scale), T = (q_w - 8) . q_x, an exact integer below 2^24.
// T accumulates in a fresh fp32 TMEM accumulator per block (one or two
// planes x two K halves of kind::f16 MMAs, M = 128 weight rows, N = 128
// tokens, K = 16); the epilogue adds fma(T, d_w * s, y) block after block.
// Against the reference: Q4_0 products and block sums are the reference's
// exactly, only the fp32 order of the block sums differs; Q8_0 differs by the
// 22-bit representation of x (~2^-23 of each block's max|x|).
//
// Operands are packed once per call into the MMA's K-major layout (8-row x
// 16-byte core matrices: 16-byte K chunks 128 B apart, 8-row groups 512 B
// apart; one 8 KiB tile per 128 rows x 32 K), so every pipeline stage is a
// handful of contiguous bulk copies.  Kernel roles (576 threads, one CTA per
// SM, all 512 TMEM columns):
//   warp 0     bulk copies of a stage (2 blocks: weight tiles, x planes, scales)
//   warp 1     tensor memory, and one lane issuing the MMAs into four
//              rotating 128-column accumulators
//   warps 2-17 epilogue: TMEM lane = weight row, four warps per lane quarter,
//              32 tokens each; fp32 accumulators in registers
// No TMA multicast anywhere.
#include <algorithm>

#include <cuda_fp16.h>

#include "tb_internal.cuh"

namespace tb {
namespace {

constexpr int kRowsT = 128;                 // weight rows per tile (MMA M)
constexpr int kToksT = 128;                 // tokens per tile (MMA N)
constexpr int kOpTile = 128 * 32 * 2;       // one block's 128 x 32 fp16 operand tile: 8 KiB
constexpr int kSB = 2;                      // blocks per stage
constexpr int kAccBufs = 4;                 // 4 x 128 TMEM columns
constexpr int kEpiWarps = 16;
constexpr int kF16Threads = (2 + kEpiWarps) * 32;

__host__ __device__ constexpr int op_off(int r, int c) { return (r >> 3) * 512 + c * 128 + (r & 7) * 16; }

template <int P>
__host__ __device__ constexpr int stage_bytes() {
  return kSB * kOpTile * (1 + P) + kSB * 2 * kRowsT * 4;
}
template <int P>
__host__ __device__ constexpr int num_stages() {
  return P == 2 ? 4 : 6;
}
template <int P>
constexpr size_t f16_smem() {
  return (size_t)num_stages<P>() * stage_bytes<P>() + 1024;
}

__device__ __forceinline__ uint64_t desc_k(uint32_t saddr) {  // K-major, no swizzle, LBO 128 B, SBO 512 B
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(512 >> 4) << 32) |
         (1ull << 46);
}

// kind::f16: D fp32 (bits 4-5 = 1), A and B fp16 (formats 0), both K-major,
// N = 128 (N >> 3 at bit 17), M = 128 (M >> 4 at bit 24).
constexpr uint32_t kIdescF16 = (1u << 4) | ((uint32_t)(kToksT >> 3) << 17) | ((uint32_t)(kRowsT >> 4) << 24);

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdescF16), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void commit_to(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}


// ---- operand packing ------------------------------------------------------------

// eight fp16 values as one 16-byte word (element 0 in the low half of .x)
__device__ __forceinline__ uint4 pack8(const __half *h) {
  uint32_t w[4];
#pragma unroll
  for (int k = 0; k < 4; ++k)
    w[k] = (uint32_t)__half_as_ushort(h[2 * k]) | ((uint32_t)__half_as_ushort(h[2 * k + 1]) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Weights: thread per (row n < N_pad, 8 consecutive blocks), rows fastest:
// the 8 blocks are one 16-byte aligned run (144 or 272 bytes, nb % 8 == 0),
// and consecutive threads' 16-byte tile stores fill whole 128-byte lines.
// Tile (row tile, b) at Ap + (rt * nb + b) * 8 KiB; the block scale at
// dW[(rt * nb + b) * 128 + j].
template <bool Q4>
__global__ void __launch_bounds__(256) pack_w_kernel(const uint8_t *__restrict__ w, int N, int N_pad, int nb,
                                                     uint8_t *__restrict__ Ap, float *__restrict__ dW) {
  constexpr int BB = Q4 ? 18 : 34;     // bytes per block
  constexpr int NV = 8 * BB / 16;      // 16-byte words per 8 blocks: 9 or 17
  const int64_t total = (int64_t)N_pad * (nb / 8);
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int n = (int)(idx % N_pad), b8 = (int)(idx / N_pad) * 8;
    const int rt = n >> 7, j = n & 127;
    uint32_t wv[NV * 4];
    if (n < N) {
      const uint4 *src = reinterpret_cast<const uint4 *>(w + ((int64_t)n * nb + b8) * BB);
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const uint4 v = __ldg(src + k);
        wv[4 * k] = v.x;
        wv[4 * k + 1] = v.y;
        wv[4 * k + 2] = v.z;
        wv[4 * k + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int k = 0; k < NV * 4; ++k) wv[k] = 0u;
    }
    auto byte_at = [&](int o) { return (int)((wv[o >> 2] >> (8 * (o & 3))) & 0xFFu); };
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int o = u * BB;
      __half h[32];
      if (Q4) {
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const int byte = byte_at(o + 2 + k);
          h[k] = __int2half_rn((byte & 0x0F) - 8);
          h[k + 16] = __int2half_rn((byte >> 4) - 8);
        }
      } else {
#pragma unroll
        for (int k = 0; k < 32; ++k) h[k] = __int2half_rn((int)(int8_t)byte_at(o + 2 + k));
      }
      const float d = __half2float(__ushort_as_half((uint16_t)(byte_at(o) | (byte_at(o + 1) << 8))));
      const int b = b8 + u;
      uint8_t *dst = Ap + ((int64_t)rt * nb + b) * kOpTile;
#pragma unroll
      for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4 *>(dst + op_off(j, c)) = pack8(h + 8 * c);
      dW[((int64_t)rt * nb + b) * kRowsT + j] = d;
    }
  }
}

// Activations: thread per (token m < M_pad, block b), tokens fastest.  Planes of (tile, b) at
// Bp + ((tt * nb + b) * P + p) * 8 KiB; the block's scale at Sx[(tt * nb + b) * 128 + i].
template <bool Q4>
__global__ void __launch_bounds__(256) pack_x_kernel(const float *__restrict__ x, int M, int M_pad, int K,
                                                     uint8_t *__restrict__ Bp, float *__restrict__ Sx) {
  constexpr int P = Q4 ? 1 : 2;
  const int nb = K / 32;
  const int64_t total = (int64_t)M_pad * nb;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int m = (int)(idx % M_pad), b = (int)(idx / M_pad);  // consecutive tokens: whole-line tile stores
    const int tt = m >> 7, i = m & 127;
    float v[32];
    if (m < M) {
      const float4 *x4 = reinterpret_cast<const float4 *>(x + (int64_t)m * K + 32 * b);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float4 f = __ldg(x4 + u);
        v[4 * u] = f.x;
        v[4 * u + 1] = f.y;
        v[4 * u + 2] = f.z;
        v[4 * u + 3] = f.w;
      }
    } else {
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = 0.f;
    }
    float am = 0.f;
#pragma unroll
    for (int k = 0; k < 32; ++k) am = fmaxf(am, fabsf(v[k]));  // fmaxf skips NaN
    __half hp[P][32];
    float s;
    if (Q4) {
      // quantize_row_q8_0: d = amax / 127, id = 1 / d (the fp32 d), q = round(x * id); the dot uses fp16(d)
      const float d = __fdiv_rn(am, 127.0f);
      const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
#pragma unroll
      for (int k = 0; k < 32; ++k) hp[0][k] = __int2half_rn((int)roundf(__fmul_rn(v[k], id)));
      s = __half2float(__float2half_rn(d));
    } else {
      int e = 0;
      if (am > 0.f && am <= 3.0e38f) {
        int ex;
        frexpf(am, &ex);  // am in [2^(ex-1), 2^ex)
        e = min(15 - ex, 126);
      }
      const float up = ldexpf(1.0f, e);
      s = ldexpf(1.0f, -e);
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const float t = __fmul_rn(v[k], up);  // exact: a power of two
        const __half hi = __float2half_rn(t);
        hp[0][k] = hi;
        hp[P - 1][k] = __float2half_rn(__fsub_rn(t, __half2float(hi)));
      }
    }
#pragma unroll
    for (int p = 0; p < P; ++p) {
      uint8_t *dst = Bp + (((int64_t)tt * nb + b) * P + p) * kOpTile;
#pragma unroll
      for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4 *>(dst + op_off(i, c)) = pack8(hp[p] + 8 * c);
    }
    Sx[((int64_t)tt * nb + b) * kToksT + i] = m < M ? s : 0.f;
  }
}

struct F16Args {
  const uint8_t *Ap;
  const float *dW;
  const uint8_t *Bp;
  const float *Sx;
  float *out;            // Y [M, N], or this split's slice of the partial sums
  int64_t split_stride;  // elements between splits' partial sums
  int M, N, nb, kb_per;
};

template <int P>
__global__ void __launch_bounds__(kF16Threads, 1) gemm_f16_kernel(const F16Args a, uint32_t *__restrict__ err) {
  constexpr int NS = num_stages<P>();
  constexpr int SBYTES = stage_bytes<P>();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[NS], empty[NS], acc_full[kAccBufs], acc_empty[kAccBufs], mma_done;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rt = blockIdx.x, tt = blockIdx.y, ks = blockIdx.z;
  const int b0 = ks * a.kb_per, b1 = min(a.nb, b0 + a.kb_per);
  const int nstage = (b1 - b0) / kSB;  // kb_per and nb are multiples of kSB
  uint8_t *base = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
  auto sA = [&](int s) { return base + (size_t)s * SBYTES; };
  auto sB = [&](int s) { return base + (size_t)s * SBYTES + kSB * kOpTile; };
  auto sD = [&](int s) { return reinterpret_cast<const float *>(base + (size_t)s * SBYTES + kSB * kOpTile * (1 + P)); };
  auto sS = [&](int s) { return sD(s) + kSB * kRowsT; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1 + kEpiWarps);  // the MMAs' commit and every epilogue warp
    }
    for (int i = 0; i < kAccBufs; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpiWarps);
    }
    mbar_init(&mma_done, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                 "r"(kAccBufs * 128));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    // ---- producer ------------------------------------------------------------------
    if (lane == 0) {
      for (int i = 0; i < nstage; ++i) {
        const int s = i % NS, b = b0 + i * kSB;
        if (i >= NS && !mbar_wait_bounded(&empty[s], (uint32_t)(((i / NS) + 1) & 1), err)) {
          abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[s], (uint32_t)SBYTES);
        bulk_g2s(sA(s), a.Ap + ((int64_t)rt * a.nb + b) * kOpTile, kSB * kOpTile, &full[s]);
        bulk_g2s(sB(s), a.Bp + ((int64_t)tt * a.nb + b) * P * kOpTile, kSB * P * kOpTile, &full[s]);
        bulk_g2s(const_cast<float *>(sD(s)), a.dW + ((int64_t)rt * a.nb + b) * kRowsT, kSB * kRowsT * 4, &full[s]);
        bulk_g2s(const_cast<float *>(sS(s)), a.Sx + ((int64_t)tt * a.nb + b) * kToksT, kSB * kToksT * 4, &full[s]);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issue -----------------------------------------------------------------
    if (lane == 0) {
      for (int i = 0; i < nstage && !*(volatile int *)&abort_flag; ++i) {
        const int s = i % NS;
        if (!mbar_wait_bounded(&full[s], (uint32_t)((i / NS) & 1), err)) {
          abort_flag = 1;
          break;
        }
        fence_after();
        bool ok = true;
        for (int u = 0; u < kSB && ok; ++u) {
          const int blk = i * kSB + u, ab = blk % kAccBufs;
          if (blk >= kAccBufs) ok = mbar_wait_bounded(&acc_empty[ab], (uint32_t)(((blk / kAccBufs) + 1) & 1), err);
          if (!ok) break;
          fence_after();
          const uint32_t aaddr = smem_addr(sA(s)) + u * kOpTile;
#pragma unroll
          for (int p = 0; p < P; ++p) {
            const uint32_t baddr = smem_addr(sB(s)) + (u * P + p) * kOpTile;
#pragma unroll
            for (int h = 0; h < 2; ++h)  // K halves: chunks 2h, 2h+1
              mma_f16(tmem + (uint32_t)(ab * 128), desc_k(aaddr + h * 256), desc_k(baddr + h * 256),
                      (p | h) != 0 ? 1u : 0u);
          }
          commit_to(&acc_full[ab]);
        }
        if (!ok) {
          abort_flag = 1;
          break;
        }
        commit_to(&empty[s]);  // this stage's operand tiles are consumed
      }
      commit_to(&mma_done);  // completes once every MMA above has
      mbar_wait_bounded(&mma_done, 0, err);
    }
  } else {
    // ---- epilogue: warps 2-17; lane quarter q = warp % 4, token quarter tq ------------
    const int q = warp & 3, tq = (warp - 2) >> 2;
    const int r = 32 * q + lane;  // weight row in the tile = TMEM lane
    const uint32_t taddr0 = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(tq * 32);
    float2 y2[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) y2[k] = make_float2(0.f, 0.f);
    bool ok = true;
    for (int i = 0; i < nstage && ok; ++i) {
      const int s = i % NS;
      ok = mbar_wait_bounded(&full[s], (uint32_t)((i / NS) & 1), err);
      for (int u = 0; u < kSB && ok; ++u) {
        const int blk = i * kSB + u, ab = blk % kAccBufs;
        ok = mbar_wait_bounded(&acc_full[ab], (uint32_t)((blk / kAccBufs) & 1), err);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        fence_after();
        uint32_t t[32];
        tmem_ld32(taddr0 + (uint32_t)(ab * 128), t);
        const float dw = sD(s)[u * kRowsT + r];
        const float2 dw2 = make_float2(dw, dw);
        const float4 *sx4 = reinterpret_cast<const float4 *>(sS(s) + u * kToksT + tq * 32);
#pragma unroll
        for (int m4 = 0; m4 < 8; ++m4) {  // packed pairs: c = d_w * s, y = fma(T, c, y)
          const float4 sv = sx4[m4];
          const float2 c0 = __fmul2_rn(dw2, make_float2(sv.x, sv.y)), c1 = __fmul2_rn(dw2, make_float2(sv.z, sv.w));
          y2[2 * m4] = __ffma2_rn(make_float2(__uint_as_float(t[4 * m4]), __uint_as_float(t[4 * m4 + 1])), c0,
                                  y2[2 * m4]);
          y2[2 * m4 + 1] = __ffma2_rn(make_float2(__uint_as_float(t[4 * m4 + 2]), __uint_as_float(t[4 * m4 + 3])),
                                      c1, y2[2 * m4 + 1]);
        }
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[ab]);
      }
      ok = __all_sync(0xffffffffu, ok);
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(&empty[s]);  // done with this stage's scales
    }
    if (!ok) {
      if (lane == 0) abort_flag = 1;
    } else {
      const int n = rt * kRowsT + r;
      if (n < a.N) {
        float *o = a.out + (int64_t)ks * a.split_stride + n;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const int tok = tt * kToksT + tq * 32 + 2 * k;
          if (tok < a.M) o[(int64_t)tok * a.N] = y2[k].x;
          if (tok + 1 < a.M) o[(int64_t)(tok + 1) * a.N] = y2[k].y;
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kAccBufs * 128));
  }
}

__global__ void __launch_bounds__(256) sum_parts_kernel(const float *__restrict__ part, int splits, int64_t n,
                                                        float *__restrict__ y) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float s = part[i];
    for (int z = 1; z < splits; ++z) s = __fadd_rn(s, part[(int64_t)z * n + i]);
    y[i] = s;
  }
}

}  // namespace

bool gemm_f16_eligible(int64_t M, int64_t K, const float *x, const void *w) {
  return M >= 32 && K >= 256 && K % 256 == 0 && K <= (1 << 20) && (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(x) & 15) == 0;
}

tb_status launch_gemm_f16(int dtype, const float *x, int64_t M, int64_t K, const void *w, int64_t N, float *y,
                          cudaStream_t s, const DeviceState *st) {
  const bool q4 = dtype == TB_Q4_0;
  const int P = q4 ? 1 : 2;
  const int nb = (int)(K / 32);
  const int64_t M_pad = (M + kToksT - 1) / kToksT * kToksT, N_pad = (N + kRowsT - 1) / kRowsT * kRowsT;
  const int tiles_n = (int)(N_pad / kRowsT), tiles_m = (int)(M_pad / kToksT);
  if ((int64_t)tiles_n * tiles_m > 65535LL * 65535LL || M > 0x7FFFFFFF || N > 0x7FFFFFFF)
    return fail(TB_EINVAL, "tb_matmul_quant: shape too large");
  // split the K loop until the grid covers the SMs (each split >= 16 blocks)
  int splits = 1;
  while ((int64_t)tiles_n * tiles_m * splits * 2 <= st->sm_count && nb / (splits * 2) >= 16) splits *= 2;
  int kb_per = (nb + splits - 1) / splits;
  kb_per = (kb_per + kSB - 1) / kSB * kSB;
  splits = (nb + kb_per - 1) / kb_per;

  auto al = [](size_t v) { return (v + 1023) & ~size_t(1023); };
  const size_t a_bytes = al((size_t)N_pad * K * 2), dw_bytes = al((size_t)N_pad * nb * 4);
  const size_t b_bytes = al((size_t)M_pad * K * 2 * P), sx_bytes = al((size_t)M_pad * nb * 4);
  const size_t p_bytes = splits > 1 ? (size_t)splits * M * N * 4 : 0;
  uint8_t *ws = nullptr;
  cudaError_t e = cudaMallocAsync(reinterpret_cast<void **>(&ws), a_bytes + dw_bytes + b_bytes + sx_bytes + p_bytes, s);
  if (e != cudaSuccess) return fail(TB_ENOMEM, "tb_matmul_quant: tensor-core workspace: %s", cudaGetErrorString(e));
  uint8_t *Ap = ws, *Bp = ws + a_bytes + dw_bytes;
  float *dW = reinterpret_cast<float *>(ws + a_bytes);
  float *Sx = reinterpret_cast<float *>(ws + a_bytes + dw_bytes + b_bytes);
  float *part = splits > 1 ? reinterpret_cast<float *>(ws + a_bytes + dw_bytes + b_bytes + sx_bytes) : y;

  tb_status rs = TB_OK;
  {
    const int64_t nw = N_pad * (nb / 8), nx = M_pad * nb;
    const int gw = (int)std::min<int64_t>((nw + 255) / 256, (int64_t)st->sm_count * 8);
    const int gx = (int)std::min<int64_t>((nx + 255) / 256, (int64_t)st->sm_count * 8);
    if (q4) {
      pack_w_kernel<true><<<gw, 256, 0, s>>>((const uint8_t *)w, (int)N, (int)N_pad, nb, Ap, dW);
      pack_x_kernel<true><<<gx, 256, 0, s>>>(x, (int)M, (int)M_pad, (int)K, Bp, Sx);
    } else {
      pack_w_kernel<false><<<gw, 256, 0, s>>>((const uint8_t *)w, (int)N, (int)N_pad, nb, Ap, dW);
      pack_x_kernel<false><<<gx, 256, 0, s>>>(x, (int)M, (int)M_pad, (int)K, Bp, Sx);
    }
    rs = check_launch("tb_matmul_quant (operand packing)");
  }
  if (rs == TB_OK) {
    F16Args a;
    a.Ap = Ap;
    a.dW = dW;
    a.Bp = Bp;
    a.Sx = Sx;
    a.out = part;
    a.split_stride = (int64_t)M * N;
    a.M = (int)M;
    a.N = (int)N;
    a.nb = nb;
    a.kb_per = kb_per;
    const dim3 grid((unsigned)tiles_n, (unsigned)tiles_m, (unsigned)splits);
    if (q4) {
      rs = ensure_smem_for(gemm_f16_kernel<1>, f16_smem<1>());
      if (rs == TB_OK) gemm_f16_kernel<1><<<grid, kF16Threads, f16_smem<1>(), s>>>(a, st->err_word);
    } else {
      rs = ensure_smem_for(gemm_f16_kernel<2>, f16_smem<2>());
      if (rs == TB_OK) gemm_f16_kernel<2><<<grid, kF16Threads, f16_smem<2>(), s>>>(a, st->err_word);
    }
    if (rs == TB_OK) rs = check_launch("tb_matmul_quant (tensor cores)");
  }
  if (rs == TB_OK && splits > 1) {
    const int64_t n = M * N;
    const int grid = (int)std::min<int64_t>((n + 255) / 256, (int64_t)st->sm_count * 8);
    sum_parts_kernel<<<grid, 256, 0, s>>>(part, splits, n, y);
    rs = check_launch("tb_matmul_quant (split sum)");
  }
  e = cudaFreeAsync(ws, s);
  if (rs == TB_OK && e != cudaSuccess) return fail(TB_ECUDA, "tb_matmul_quant: free workspace: %s", cudaGetErrorString(e));
  return rs;
}

}  // namespace tb
