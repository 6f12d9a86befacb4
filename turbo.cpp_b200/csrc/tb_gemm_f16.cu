// tb_gemm_f16.cu -- the quantized prefill matmul (M >= 32) on the tensor cores,
// kind::f16 with fp32 accumulation in tensor memory.
//
// Arithmetic.  K is cut into chunks of 256 (eight 32-wide blocks).  Within a
// chunk every operand carries its block scale, and a power of two per
// (row, chunk) or (token, chunk) keeps it in fp16's range:
//   weights  a = q d_w 2^e (Q8_0: q; Q4_0: q - 8), the block scale d_w as
//            fp32; q d_w has at most 19 significant bits, so a = hi + lo
//            with hi, lo fp16 holds it exactly;
//   Q4_0 x   quantised to Q8_0 exactly as the reference does
//            (quantize_row_q8_0, src/tensor/quant_math.hpp:68-90): b =
//            q_x d_x 2^f, also exact as hi + lo;
//   Q8_0 x   b = x 2^f = hi + lo, 22 bits (error below 2^-23 of the chunk's
//            largest |x|).
// The chunk's dot product T = sum over its 256 k of a b accumulates in one
// fp32 TMEM accumulator from three kind::f16 MMAs per 16-wide K step (hi.hi,
// hi.lo, lo.hi; lo.lo is below 2^-22 of the product and left out); the
// epilogue adds y = fma(T, 2^-(e + f), y) once per chunk.  The block products
// are exact; only fp32 rounding inside the tensor core and of the chunk sums
// differs from the reference's order.
//
// Operands are packed once per call into the MMA's K-major layout (8-row x
// 16-byte core matrices: 16-byte K chunks 128 B apart, 8-row groups 512 B
// apart; one 8 KiB tile per 128 rows x 32 K and plane), so every pipeline
// stage is two contiguous bulk copies.  Kernel roles (320 threads, one CTA per
// SM, all 512 TMEM columns):
//   warp 0     bulk copies of a stage (2 blocks: both planes of weights and x)
//   warp 1     tensor memory, and one lane issuing the MMAs into four
//              rotating 128-column accumulators, one per chunk
//   warps 2-9  epilogue: TMEM lane = weight row, two warps per lane quarter,
//              half the tile's tokens each; fp32 sums in registers
// When K is split over CTAs, the splits of a tile form one thread-block
// cluster: each CTA leaves its partial tile in its shared memory and CTA z sums
// its share of the rows over the cluster (distributed shared memory) in split
// order, so there is no partial-sum buffer and no extra launch.  No TMA
// multicast anywhere.
#include <algorithm>

#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include "tb_internal.cuh"

namespace tb {
namespace {

namespace cg = cooperative_groups;

constexpr int kRowsT = 128;                 // weight rows per tile (MMA M)
constexpr int kOpTile = 128 * 32 * 2;       // a weight plane of one block: 128 rows x 32 K fp16, 8 KiB
constexpr int kCB = 8;                      // blocks per chunk (one accumulator)
constexpr int kEpiWarps = 8;
constexpr int kF16Threads = (2 + kEpiWarps) * 32;
constexpr int kStageRoom = 192 * 1024;      // shared memory of the operand ring

__host__ __device__ constexpr int op_off(int r, int c) { return (r >> 3) * 512 + c * 128 + (r & 7) * 16; }

// TN tokens per tile (MMA N, 128 or 256); a stage is one block: both weight
// planes and both x planes.
template <int TN>
__host__ __device__ constexpr int x_tile() {
  return TN * 32 * 2;
}
template <int TN>
__host__ __device__ constexpr int stage_bytes() {
  return 2 * kOpTile + 2 * x_tile<TN>();
}
template <int TN>
__host__ __device__ constexpr int num_stages() {
  return kStageRoom / stage_bytes<TN>();  // 6 (TN 128) or 4 (TN 256)
}
template <int TN>
__host__ __device__ constexpr int acc_bufs() {
  return 512 / TN;  // TN-column accumulators in the 512 TMEM columns
}
template <int TN>
constexpr size_t f16_smem() {
  return (size_t)num_stages<TN>() * stage_bytes<TN>() + 1024;
}

__device__ __forceinline__ uint64_t desc_k(uint32_t saddr) {  // K-major, no swizzle, LBO 128 B, SBO 512 B
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(512 >> 4) << 32) |
         (1ull << 46);
}

// kind::f16: D fp32 (bits 4-5 = 1), A and B fp16 (formats 0), both K-major,
// N = TN (N >> 3 at bit 17), M = 128 (M >> 4 at bit 24).
template <int TN>
__host__ __device__ constexpr uint32_t idesc_f16() {
  return (1u << 4) | ((uint32_t)(TN >> 3) << 17) | ((uint32_t)(kRowsT >> 4) << 24);
}

template <int TN>
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc_f16<TN>()), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void commit_to(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
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

// Weights: thread per (row n < N_pad, chunk of 8 blocks), rows fastest: the
// 8 blocks are one 16-byte aligned run (144 or 272 bytes) read with 16-byte
// loads, and consecutive threads' 16-byte tile stores fill whole 128-byte
// lines.  Planes of (row tile rt, block b) at Ap + ((rt * nb + b) * 2 + p) *
// 8 KiB; the chunk's scale 2^-e at sW[(rt * (nb / 8) + chunk) * 128 + j].
// The exponent comes from the bound max |d| * max |q| (8 for Q4_0, 128 for
// Q8_0), so the quants are decoded once.
__device__ __forceinline__ float pow2f(int e) { return __uint_as_float((uint32_t)(127 + e) << 23); }

// The power of two e with max * 2^e in [2^14, 2^15) (0 for a zero or
// non-finite maximum), clamped so that 2^e and 2^-e stay normal.  Every
// operand of the chunk is then below 2^15, inside fp16's range.
__device__ __forceinline__ int chunk_exp(float mx) {
  const int E = (int)((__float_as_uint(mx) >> 23) & 0xFFu);
  if (mx == 0.f || E == 255) return 0;
  const int e = 141 - E;  // mx in [2^(E-127), 2^(E-126))
  return min(max(e, -126), 126);
}

template <bool Q4>
__global__ void __launch_bounds__(256) pack_w_kernel(const uint8_t *__restrict__ w, int N, int N_pad, int nb,
                                                     uint8_t *__restrict__ Ap, float *__restrict__ sW) {
  constexpr int BB = Q4 ? 18 : 34;  // bytes per block
  constexpr int NV = 8 * BB / 16;    // 16-byte words per 8 blocks: 9 or 17
  const int nc = nb / kCB;
  const int64_t total = (int64_t)N_pad * nc;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int n = (int)(idx % N_pad), c = (int)(idx / N_pad), b8 = c * kCB;
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
      for (int k = 0; k < NV * 4; ++k) wv[k] = Q4 ? 0x88888888u : 0u;  // zero quants
#pragma unroll
      for (int u = 0; u < kCB; ++u) wv[(u * BB) >> 2] &= ~(0xFFFFu << (8 * ((u * BB) & 3)));  // zero scales
    }
    auto byte_at = [&](int o) { return (wv[o >> 2] >> (8 * (o & 3))) & 0xFFu; };
    auto scale = [&](int u) {
      const int o = u * BB;  // even: the scale never straddles two words
      return __half2float(__ushort_as_half((uint16_t)((wv[o >> 2] >> (8 * (o & 3))) & 0xFFFFu)));
    };
    float mx = 0.f;
#pragma unroll
    for (int u = 0; u < kCB; ++u) mx = fmaxf(mx, fabsf(scale(u)));
    const int e = chunk_exp(__fmul_rn(mx, Q4 ? 8.0f : 128.0f));
    const float up = pow2f(e);
#pragma unroll
    for (int u = 0; u < kCB; ++u) {
      const float d = __fmul_rn(scale(u), up);  // exact: a power of two
      uint8_t *dst = Ap + ((int64_t)rt * nb + b8 + u) * 2 * kOpTile;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        __half hi[8], lo[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int kk = 8 * cc + k;
          int qv;
          if (Q4) {
            const uint32_t byte = byte_at(u * BB + 2 + (kk & 15));
            qv = (int)(kk < 16 ? (byte & 0x0Fu) : (byte >> 4)) - 8;
          } else {
            qv = (int)(int8_t)byte_at(u * BB + 2 + kk);
          }
          const float t = __fmul_rn((float)qv, d);  // exact: 19 significant bits at most
          hi[k] = __float2half_rn(t);
          lo[k] = __float2half_rn(__fsub_rn(t, __half2float(hi[k])));
        }
        *reinterpret_cast<uint4 *>(dst + op_off(j, cc)) = pack8(hi);
        *reinterpret_cast<uint4 *>(dst + kOpTile + op_off(j, cc)) = pack8(lo);
      }
    }
    sW[((int64_t)rt * nc + c) * kRowsT + j] = pow2f(-e);
  }
}

// Activations: warp per (8 tokens m0 .. m0 + 7, chunk of 8 blocks); lane
// (t, g) = (lane / 4, lane % 4) holds elements 8g .. 8g + 7 of each block of
// token m0 + t, so every 8 lanes of a store fill one 128-byte line of a tile.
// Planes of (token tile tt of TN, block b) at Bp + ((tt * nb + b) * 2 + p) *
// TN * 64; the chunk's scale 2^-f at sX[(tt * (nb / 8) + chunk) * TN + i] (0
// for padding tokens).  Q4: each block quantised as quantize_row_q8_0 does,
// b = q_x d_x 2^f.
template <bool Q4, int TN>
__global__ void __launch_bounds__(256) pack_x_kernel(const float *__restrict__ x, int M, int M_pad, int K,
                                                     uint8_t *__restrict__ Bp, float *__restrict__ sX) {
  pdl_launch_dependents();  // the tensor-core kernel may set up meanwhile
  const int nb = K / 32, nc = nb / kCB, lane = threadIdx.x & 31;
  const int t = lane >> 2, g = lane & 3;
  const int64_t total = (int64_t)(M_pad / 8) * nc;
  const int64_t stride = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t idx = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; idx < total; idx += stride) {
    const int m = (int)(idx % (M_pad / 8)) * 8 + t, c = (int)(idx / (M_pad / 8));
    const int tt = m / TN, i = m % TN;
    float v[kCB][8];
    if (m < M) {
      const float4 *x4 = reinterpret_cast<const float4 *>(x + (int64_t)m * K + 32 * kCB * c + 8 * g);
#pragma unroll
      for (int u = 0; u < kCB; ++u) {
        const float4 f0 = __ldg(x4 + 8 * u), f1 = __ldg(x4 + 8 * u + 1);
        v[u][0] = f0.x, v[u][1] = f0.y, v[u][2] = f0.z, v[u][3] = f0.w;
        v[u][4] = f1.x, v[u][5] = f1.y, v[u][6] = f1.z, v[u][7] = f1.w;
      }
    } else {
#pragma unroll
      for (int u = 0; u < kCB; ++u)
#pragma unroll
        for (int k = 0; k < 8; ++k) v[u][k] = 0.f;
    }
    float mx = 0.f, d16[kCB];
#pragma unroll
    for (int u = 0; u < kCB; ++u) {
      float am = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) am = fmaxf(am, fabsf(v[u][k]));  // fmaxf skips NaN
      if (Q4) {
        // quantize_row_q8_0 of block u: amax over the token's four lanes,
        // d = amax / 127, id = 1 / d (the fp32 d), q = round(x * id); the dot
        // uses the fp16 d
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
        const float d = __fdiv_rn(am, 127.0f);
        const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
        float qa = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          v[u][k] = roundf(__fmul_rn(v[u][k], id));
          qa = fmaxf(qa, fabsf(v[u][k]));
        }
        d16[u] = __half2float(__float2half_rn(d));
        mx = fmaxf(mx, __fmul_rn(qa, d16[u]));
      } else {
        mx = fmaxf(mx, am);
      }
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));  // the token's chunk maximum
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const int f = chunk_exp(mx);
    const float up = pow2f(f);
#pragma unroll
    for (int u = 0; u < kCB; ++u) {
      const float gs = Q4 ? __fmul_rn(d16[u], up) : up;  // exact: a power of two
      __half hi[8], lo[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float tv = __fmul_rn(v[u][k], gs);  // exact (Q4: 18 significant bits at most)
        hi[k] = __float2half_rn(tv);
        lo[k] = __float2half_rn(__fsub_rn(tv, __half2float(hi[k])));
      }
      uint8_t *dst = Bp + ((int64_t)tt * nb + c * kCB + u) * 2 * x_tile<TN>() + op_off(i, g);
      *reinterpret_cast<uint4 *>(dst) = pack8(hi);
      *reinterpret_cast<uint4 *>(dst + x_tile<TN>()) = pack8(lo);
    }
    if (g == 0) sX[((int64_t)tt * nc + c) * TN + i] = m < M ? pow2f(-f) : 0.f;
  }
}

struct F16Args {
  const uint8_t *Ap;
  const float *sW;
  const uint8_t *Bp;
  const float *sX;
  float *out;            // Y [M, N], or this split's slice of the partial sums
  int64_t split_stride;  // elements between splits' partial sums
  int M, N, nb, kb_per;
  int cl;                // 1: the splits of a tile are one cluster and sum there into out = Y
};

// Y rows [z * 128 / NZ, (z + 1) * 128 / NZ) of the tile = the sum over the
// cluster's NZ partial tiles ([128][TN + 4] in each CTA's shared memory), in
// split order.  Items are (row, four tokens), consecutive threads on
// consecutive rows; each thread loads 16 / NZ items from every CTA before it
// adds, so the remote loads overlap.
template <int NZ, int TN>
__device__ __forceinline__ void cluster_sum(const cg::cluster_group &cluster, const float *pt, int z, const F16Args &a,
                                            int rt, int tt) {
  constexpr int ROWS = kRowsT / NZ, ITEMS = ROWS * (TN / 4), B = 16 / NZ;
  for (int it0 = threadIdx.x; it0 < ITEMS; it0 += B * kF16Threads) {
    float4 v[B][NZ];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const int it = it0 + b * kF16Threads;
      if (it < ITEMS) {
        const int r = z * ROWS + it % ROWS, k = 4 * (it / ROWS);
        const float *src = pt + r * (TN + 4) + k;
#pragma unroll
        for (int zz = 0; zz < NZ; ++zz) v[b][zz] = *reinterpret_cast<const float4 *>(cluster.map_shared_rank(src, zz));
      }
    }
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const int it = it0 + b * kF16Threads;
      if (it < ITEMS) {
        const int r = z * ROWS + it % ROWS, k = 4 * (it / ROWS);
        const int n = rt * kRowsT + r, tok = tt * TN + k;
        float4 acc = v[b][0];
#pragma unroll
        for (int zz = 1; zz < NZ; ++zz) {
          acc.x = __fadd_rn(acc.x, v[b][zz].x);
          acc.y = __fadd_rn(acc.y, v[b][zz].y);
          acc.z = __fadd_rn(acc.z, v[b][zz].z);
          acc.w = __fadd_rn(acc.w, v[b][zz].w);
        }
        if (n < a.N) {
          float *o = a.out + (int64_t)tok * a.N + n;
          if (tok < a.M) o[0] = acc.x;
          if (tok + 1 < a.M) o[a.N] = acc.y;
          if (tok + 2 < a.M) o[2 * (int64_t)a.N] = acc.z;
          if (tok + 3 < a.M) o[3 * (int64_t)a.N] = acc.w;
        }
      }
    }
  }
}

template <int TN>
__global__ void __launch_bounds__(kF16Threads, 1) gemm_f16_kernel(const F16Args a, uint32_t *__restrict__ err) {
  constexpr int NS = num_stages<TN>();
  constexpr int SBYTES = stage_bytes<TN>();
  constexpr int NACC = acc_bufs<TN>();
  constexpr int TPW = TN / 2;  // tokens per epilogue warp
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[NS], empty[NS], acc_full[NACC], acc_empty[NACC], mma_done;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rt = blockIdx.x, tt = blockIdx.y, ks = blockIdx.z;
  const int b0 = ks * a.kb_per, b1 = min(a.nb, b0 + a.kb_per);
  const int nblk = b1 - b0;  // kb_per and nb are multiples of kCB
  const int nc = a.nb / kCB, c0 = b0 / kCB;
  uint8_t *base = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
  auto sA = [&](int s) { return base + (size_t)s * SBYTES; };
  auto sB = [&](int s) { return base + (size_t)s * SBYTES + 2 * kOpTile; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);  // the MMAs' commit
    }
    for (int i = 0; i < NACC; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpiWarps);
    }
    mbar_init(&mma_done, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = tmem_base;
  pdl_wait();  // the packed operands are written by the kernels before this one

  if (warp == 0) {
    // ---- producer: one block (both planes of weights and x) per stage ---------------
    if (lane == 0) {
      for (int i = 0; i < nblk; ++i) {
        const int s = i % NS, b = b0 + i;
        if (i >= NS && !mbar_wait_bounded(&empty[s], (uint32_t)(((i / NS) + 1) & 1), err)) {
          abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[s], (uint32_t)SBYTES);
        bulk_g2s(sA(s), a.Ap + ((int64_t)rt * a.nb + b) * 2 * kOpTile, 2 * kOpTile, &full[s]);
        bulk_g2s(sB(s), a.Bp + ((int64_t)tt * a.nb + b) * 2 * x_tile<TN>(), 2 * x_tile<TN>(), &full[s]);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issue: hi.hi, hi.lo, lo.hi per 16-wide K step into the chunk's accumulator
    if (lane == 0) {
      for (int i = 0; i < nblk && !*(volatile int *)&abort_flag; ++i) {
        const int s = i % NS, ch = i / kCB, u = i % kCB, ab = ch % NACC;
        if (!mbar_wait_bounded(&full[s], (uint32_t)((i / NS) & 1), err)) {
          abort_flag = 1;
          break;
        }
        if (u == 0 && ch >= NACC && !mbar_wait_bounded(&acc_empty[ab], (uint32_t)(((ch / NACC) + 1) & 1), err)) {
          abort_flag = 1;
          break;
        }
        fence_after();
        const uint32_t d = tmem + (uint32_t)(ab * TN);
        const uint32_t ahi = smem_addr(sA(s)), alo = ahi + kOpTile;
        const uint32_t bhi = smem_addr(sB(s)), blo = bhi + x_tile<TN>();
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // K halves: 16-byte K groups 2h, 2h+1
          mma_f16<TN>(d, desc_k(ahi + h * 256), desc_k(bhi + h * 256), (u | h) != 0 ? 1u : 0u);
          mma_f16<TN>(d, desc_k(ahi + h * 256), desc_k(blo + h * 256), 1u);
          mma_f16<TN>(d, desc_k(alo + h * 256), desc_k(bhi + h * 256), 1u);
        }
        commit_to(&empty[s]);  // this stage's operand tiles are consumed
        if (u == kCB - 1) commit_to(&acc_full[ab]);
      }
      commit_to(&mma_done);  // completes once every MMA above has
      mbar_wait_bounded(&mma_done, 0, err);
    }
  } else {
    // ---- epilogue: warps 2-9; lane quarter q = warp % 4, token half tq ----------------
    const int q = warp & 3, tq = (warp - 2) >> 2;
    const int r = 32 * q + lane;  // weight row in the tile = TMEM lane
    const uint32_t taddr0 = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(tq * TPW);
    const float *sw = a.sW + ((int64_t)rt * nc + c0) * kRowsT + r;
    const float *sx = a.sX + ((int64_t)tt * nc + c0) * TN + tq * TPW;
    float2 y2[TPW / 2];
#pragma unroll
    for (int k = 0; k < TPW / 2; ++k) y2[k] = make_float2(0.f, 0.f);
    bool ok = true;
    for (int ch = 0; ch < nblk / kCB && ok; ++ch) {
      const int ab = ch % NACC;
      const float w2 = __ldg(sw + (int64_t)ch * kRowsT);
      const float2 ww = make_float2(w2, w2);
      ok = mbar_wait_bounded(&acc_full[ab], (uint32_t)((ch / NACC) & 1), err);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      fence_after();
#pragma unroll
      for (int part = 0; part < TPW / 16; ++part) {
        uint32_t t[16];
        tmem_ld16(taddr0 + (uint32_t)(ab * TN + part * 16), t);
        const float4 *sx4 = reinterpret_cast<const float4 *>(sx + (int64_t)ch * TN + part * 16);
#pragma unroll
        for (int m4 = 0; m4 < 4; ++m4) {  // packed pairs: c = 2^-e 2^-f, y = fma(T, c, y)
          const float4 sv = __ldg(sx4 + m4);
          const float2 c0v = __fmul2_rn(ww, make_float2(sv.x, sv.y)), c1v = __fmul2_rn(ww, make_float2(sv.z, sv.w));
          float2 &ya = y2[part * 8 + 2 * m4], &yb = y2[part * 8 + 2 * m4 + 1];
          ya = __ffma2_rn(make_float2(__uint_as_float(t[4 * m4]), __uint_as_float(t[4 * m4 + 1])), c0v, ya);
          yb = __ffma2_rn(make_float2(__uint_as_float(t[4 * m4 + 2]), __uint_as_float(t[4 * m4 + 3])), c1v, yb);
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
    }
    if (!ok) {
      if (lane == 0) abort_flag = 1;
    } else if (a.cl) {
      // the partial tile into this CTA's shared memory, [128 rows][TN + 4]
      // (16-byte units of consecutive rows 65 or 33 apart: no bank conflicts;
      // the MMAs have read every stage, as each chunk's accumulator was full)
      float4 *pt = reinterpret_cast<float4 *>(reinterpret_cast<float *>(base) + r * (TN + 4) + tq * TPW);
#pragma unroll
      for (int k = 0; k < TPW / 4; ++k) pt[k] = make_float4(y2[2 * k].x, y2[2 * k].y, y2[2 * k + 1].x, y2[2 * k + 1].y);
    } else {
      const int n = rt * kRowsT + r;
      if (n < a.N) {
        float *o = a.out + (int64_t)ks * a.split_stride + n;
#pragma unroll
        for (int k = 0; k < TPW / 2; ++k) {
          const int tok = tt * TN + tq * TPW + 2 * k;
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
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
  if (a.cl) {
    // every thread of every CTA of the cluster comes here (each wait above is
    // bounded), so the cluster barriers complete
    cg::cluster_group cluster = cg::this_cluster();
    const int nz = (int)cluster.num_blocks(), z = (int)cluster.block_rank();
    cluster.sync();
    const float *pt = reinterpret_cast<const float *>(base);
    if (nz == 2) cluster_sum<2, TN>(cluster, pt, z, a, rt, tt);
    else if (nz == 4) cluster_sum<4, TN>(cluster, pt, z, a, rt, tt);
    else if (nz == 8) cluster_sum<8, TN>(cluster, pt, z, a, rt, tt);
    cluster.sync();  // the peers' shared memory stays alive until every CTA has read it
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

// Whether clusters of `splits` CTAs of the kernel can be resident (each CTA
// takes a whole SM); checked once per size.
template <int TN>
bool cluster_fits(int splits) {
  static int fits[9] = {-1, -1, -1, -1, -1, -1, -1, -1, -1};
  if (fits[splits] < 0) {
    int n = 0;
    if (ensure_smem_for(gemm_f16_kernel<TN>, f16_smem<TN>()) == TB_OK) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1, 1, (unsigned)splits);
      cfg.blockDim = dim3(kF16Threads, 1, 1);
      cfg.dynamicSmemBytes = f16_smem<TN>();
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 1;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = (unsigned)splits;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, gemm_f16_kernel<TN>, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        n = 0;
      }
    }
    fits[splits] = n >= 1 ? 1 : 0;
  }
  return fits[splits] == 1;
}

size_t al1k(size_t v) { return (v + 1023) & ~size_t(1023); }

// The packed weights: both fp16 planes of every (row tile, block), then the
// chunk scales 2^-e, [N_pad / 128][K / 256][128].
void packed_layout(int64_t N, int64_t K, size_t *planes, size_t *total) {
  const int64_t N_pad = (N + kRowsT - 1) / kRowsT * kRowsT;
  *planes = al1k((size_t)N_pad * (size_t)K * 4);
  *total = *planes + al1k((size_t)N_pad * (size_t)(K / 256) * 4);
}

tb_status pack_weights(bool q4, const void *w, int64_t N, int64_t K, uint8_t *packed, cudaStream_t s,
                       const DeviceState *st) {
  size_t planes, total;
  packed_layout(N, K, &planes, &total);
  const int nb = (int)(K / 32), nc = nb / kCB;
  const int64_t N_pad = (N + kRowsT - 1) / kRowsT * kRowsT;
  const int64_t nw = N_pad * nc;
  const int gw = (int)std::min<int64_t>((nw + 255) / 256, (int64_t)st->sm_count * 8);
  float *sW = reinterpret_cast<float *>(packed + planes);
  if (q4)
    pack_w_kernel<true><<<gw, 256, 0, s>>>((const uint8_t *)w, (int)N, (int)N_pad, nb, packed, sW);
  else
    pack_w_kernel<false><<<gw, 256, 0, s>>>((const uint8_t *)w, (int)N, (int)N_pad, nb, packed, sW);
  return check_launch("tb_matmul_quant (weight packing)");
}

// X packing, the tensor-core kernel and, when the K splits are not summed in
// their cluster, the split sum.  Ap / sW: the packed weights.
template <int TN>
tb_status run_gemm_f16(bool q4, const float *x, int64_t M, int64_t K, const uint8_t *Ap, const float *sW,
                       int64_t N, float *y, cudaStream_t s, const DeviceState *st) {
  const int nb = (int)(K / 32), nc = nb / kCB;
  const int64_t M_pad = (M + TN - 1) / TN * TN, N_pad = (N + kRowsT - 1) / kRowsT * kRowsT;
  const int tiles_n = (int)(N_pad / kRowsT), tiles_m = (int)(M_pad / TN);
  if (tiles_n > 0x7FFFFFFF / 2 || tiles_m > 65535 || M > 0x7FFFFFFF || N > 0x7FFFFFFF)
    return fail(TB_EINVAL, "tb_matmul_quant: shape too large");
  // split the K loop (in whole chunks) until the grid covers the SMs
  int splits = 1;
  while ((int64_t)tiles_n * tiles_m * splits * 2 <= st->sm_count && nc / (splits * 2) >= 2 && splits < 8) splits *= 2;
  const int kc_per = (nc + splits - 1) / splits;
  splits = (nc + kc_per - 1) / kc_per;

  const size_t b_bytes = al1k((size_t)M_pad * K * 4), sx_bytes = al1k((size_t)M_pad * nc * 4);
  // the splits of a tile as one cluster (at most 8 CTAs, all co-resident)
  const bool cl = splits > 1 && splits <= 8 && cluster_fits<TN>(splits);
  const size_t p_bytes = splits > 1 && !cl ? (size_t)splits * M * N * 4 : 0;
  uint8_t *ws = nullptr;
  cudaError_t e = cudaMallocAsync(reinterpret_cast<void **>(&ws), b_bytes + sx_bytes + p_bytes, s);
  if (e != cudaSuccess) return fail(TB_ENOMEM, "tb_matmul_quant: tensor-core workspace: %s", cudaGetErrorString(e));
  uint8_t *Bp = ws;
  float *sX = reinterpret_cast<float *>(ws + b_bytes);
  float *part = splits > 1 && !cl ? reinterpret_cast<float *>(ws + b_bytes + sx_bytes) : y;

  tb_status rs = TB_OK;
  {
    const int64_t nx = M_pad / 8 * nc * 32;
    const int gx = (int)std::min<int64_t>((nx + 255) / 256, (int64_t)st->sm_count * 16);
    if (q4)
      pack_x_kernel<true, TN><<<gx, 256, 0, s>>>(x, (int)M, (int)M_pad, (int)K, Bp, sX);
    else
      pack_x_kernel<false, TN><<<gx, 256, 0, s>>>(x, (int)M, (int)M_pad, (int)K, Bp, sX);
    rs = check_launch("tb_matmul_quant (activation packing)");
  }
  if (rs == TB_OK) {
    F16Args a;
    a.Ap = Ap;
    a.sW = sW;
    a.Bp = Bp;
    a.sX = sX;
    a.out = part;
    a.split_stride = (int64_t)M * N;
    a.M = (int)M;
    a.N = (int)N;
    a.nb = nb;
    a.kb_per = kc_per * kCB;
    a.cl = cl ? 1 : 0;
    rs = ensure_smem_for(gemm_f16_kernel<TN>, f16_smem<TN>());
    if (rs == TB_OK) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)tiles_n, (unsigned)tiles_m, (unsigned)splits);
      cfg.blockDim = dim3(kF16Threads, 1, 1);
      cfg.dynamicSmemBytes = f16_smem<TN>();
      cfg.stream = s;
      cudaLaunchAttribute attr[2];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 1;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = cl ? (unsigned)splits : 1u;
      attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[1].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 2;
      e = cudaLaunchKernelEx(&cfg, gemm_f16_kernel<TN>, a, st->err_word);
      if (e != cudaSuccess) rs = fail(TB_ECUDA, "tb_matmul_quant (tensor cores): %s", cudaGetErrorString(e));
    }
    if (rs == TB_OK) rs = check_launch("tb_matmul_quant (tensor cores)");
  }
  if (rs == TB_OK && splits > 1 && !cl) {
    const int64_t n = M * N;
    const int grid = (int)std::min<int64_t>((n + 255) / 256, (int64_t)st->sm_count * 8);
    sum_parts_kernel<<<grid, 256, 0, s>>>(part, splits, n, y);
    rs = check_launch("tb_matmul_quant (split sum)");
  }
  e = cudaFreeAsync(ws, s);
  if (rs == TB_OK && e != cudaSuccess) return fail(TB_ECUDA, "tb_matmul_quant: free workspace: %s", cudaGetErrorString(e));
  return rs;
}

tb_status run_packed(bool q4, const float *x, int64_t M, int64_t K, const uint8_t *packed, int64_t N, float *y,
                     cudaStream_t s, const DeviceState *st) {
  size_t planes, total;
  packed_layout(N, K, &planes, &total);
  const float *sW = reinterpret_cast<const float *>(packed + planes);
  // 256-token tiles (MMA N = 256) once there are that many tokens
  if (M >= 256) return run_gemm_f16<256>(q4, x, M, K, packed, sW, N, y, s, st);
  return run_gemm_f16<128>(q4, x, M, K, packed, sW, N, y, s, st);
}

tb_status launch_gemm_f16(int dtype, const float *x, int64_t M, int64_t K, const void *w, int64_t N, float *y,
                          cudaStream_t s, const DeviceState *st) {
  const bool q4 = dtype == TB_Q4_0;
  size_t planes, total;
  packed_layout(N, K, &planes, &total);
  uint8_t *packed = nullptr;
  cudaError_t e = cudaMallocAsync(reinterpret_cast<void **>(&packed), total, s);
  if (e != cudaSuccess) return fail(TB_ENOMEM, "tb_matmul_quant: packed weights: %s", cudaGetErrorString(e));
  tb_status rs = pack_weights(q4, w, N, K, packed, s, st);
  if (rs == TB_OK) rs = run_packed(q4, x, M, K, packed, N, y, s, st);
  e = cudaFreeAsync(packed, s);
  if (rs == TB_OK && e != cudaSuccess) return fail(TB_ECUDA, "tb_matmul_quant: free workspace: %s", cudaGetErrorString(e));
  return rs;
}

}  // namespace tb

using namespace tb;

namespace {
tb_status check_packed_args(const char *who, int dtype, int64_t N, int64_t K) {
  if (dtype != TB_Q8_0 && dtype != TB_Q4_0) return fail(TB_EINVAL, "%s: dtype must be TB_Q8_0 or TB_Q4_0", who);
  if (N <= 0 || N > 0x7FFFFFFF) return fail(TB_EINVAL, "%s: N=%lld out of range", who, (long long)N);
  if (K < 256 || K % 256 != 0 || K > (1 << 20))
    return fail(TB_EINVAL, "%s: K=%lld must be a positive multiple of 256, at most 2^20", who, (long long)K);
  return TB_OK;
}
}  // namespace

extern "C" tb_status tb_packed_quant_weights_bytes(int dtype, int64_t N, int64_t K, size_t *bytes) {
  if (!bytes) return fail(TB_EINVAL, "tb_packed_quant_weights_bytes: null pointer");
  TB_TRY(check_packed_args("tb_packed_quant_weights_bytes", dtype, N, K));
  size_t planes;
  packed_layout(N, K, &planes, bytes);
  return TB_OK;
}

extern "C" tb_status tb_pack_quant_weights(int dtype, const void *w_dev, int64_t N, int64_t K, void *packed_dev,
                                           size_t packed_bytes, tb_stream stream) {
  TB_TRY(check_packed_args("tb_pack_quant_weights", dtype, N, K));
  if (!w_dev || !packed_dev) return fail(TB_EINVAL, "tb_pack_quant_weights: null pointer");
  if ((reinterpret_cast<uintptr_t>(w_dev) & 15) != 0 || (reinterpret_cast<uintptr_t>(packed_dev) & 15) != 0)
    return fail(TB_EINVAL, "tb_pack_quant_weights: pointers must be 16-byte aligned");
  size_t planes, total;
  packed_layout(N, K, &planes, &total);
  if (packed_bytes < total)
    return fail(TB_EINVAL, "tb_pack_quant_weights: %zu bytes given, %zu needed", packed_bytes, total);
  DeviceState *st;
  TB_TRY(device_state(&st));
  return pack_weights(dtype == TB_Q4_0, w_dev, N, K, static_cast<uint8_t *>(packed_dev), as_stream(stream), st);
}

extern "C" tb_status tb_matmul_quant_packed(int dtype, const float *x_dev, int64_t M, int64_t K,
                                            const void *packed_dev, int64_t N, float *y_dev, tb_stream stream) {
  TB_TRY(check_packed_args("tb_matmul_quant_packed", dtype, N, K));
  if (M < 32 || M > 0x7FFFFFFF)
    return fail(TB_EINVAL, "tb_matmul_quant_packed: M=%lld (32 or more; tb_matmul_quant takes smaller M)",
                (long long)M);
  if (!x_dev || !packed_dev || !y_dev) return fail(TB_EINVAL, "tb_matmul_quant_packed: null pointer");
  if ((reinterpret_cast<uintptr_t>(x_dev) & 15) != 0 || (reinterpret_cast<uintptr_t>(packed_dev) & 15) != 0)
    return fail(TB_EINVAL, "tb_matmul_quant_packed: X and the packed weights must be 16-byte aligned");
  DeviceState *st;
  TB_TRY(device_state(&st));
  return run_packed(dtype == TB_Q4_0, x_dev, M, K, static_cast<const uint8_t *>(packed_dev), N, y_dev,
                    as_stream(stream), st);
}
