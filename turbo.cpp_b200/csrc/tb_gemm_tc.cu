// tb_gemm_tc.cu -- prefill matmul on the 5th-generation tensor cores (tcgen05):
// Y[M, N] = X[M, K] . W for Q8_0 / Q4_0 weights W stored as N rows of K/32
// blocks (Tensor::matmul, src/tensor/tensor.cpp:328-432), M >= 32 rows.
//
// Arithmetic (3xTF32).  Both operands are dequantised exactly to fp32 and split
// as v = hi + lo, hi = v with the low 13 mantissa bits cleared (a tf32 value)
// and lo = tf32(v - hi).  A tf32 x tf32 product is exact in the fp32
// accumulator, and hi*hi + hi*lo + lo*hi leaves out only lo*lo, below 2^-21 of
// each product.
//   * Q8_0 weights: w = q * d has at most 19 significant bits, so w = hi + lo
//     exactly.  X is the fp32 activation (the reference does not quantise it
//     on this branch), so its lo part is rounded to tf32: relative error per
//     product <= 2^-21.
//   * Q4_0 weights: the reference quantises each X row to Q8_0 and takes an
//     integer dot product per block scaled by d_w * d_x.  Here X is quantised
//     the same way and dequantised (q_x * d_x, exact in fp32), so every product
//     equals the reference's up to fp32 rounding of the sums.
// Results agree with the reference within 1e-5 of sum |w x| per output (the
// summation order differs); tb_matmul_quant_exact keeps the CUDA-core path
// with the reference's order.
//
// Kernel.  One CTA per 128 weight rows x 128 tokens (x a K range when the K
// loop is split), 256 threads:
//   warp 0      bulk copies of the activation operand tiles (hi, lo) per stage
//   warp 1      TMEM allocation; one lane issues the tcgen05.mma instructions
//   warps 4-7   converters: thread t dequantises weight row t of the tile for
//               each stage into the hi/lo operand tiles; afterwards the same
//               threads are the epilogue (TMEM lane t = weight row t)
// Operand tiles are K-major without swizzle: 128 rows x 32 tf32 (one quant
// block), byte(r, k) = (r/8)*1024 + (k/4)*128 + (r%8)*16 + (k%4)*4, i.e. 8x16-byte
// core matrices, 128 B apart along K (leading byte offset) and 1024 B apart
// along rows (stride byte offset).  The activations are written in exactly
// this layout by split_x_kernel, block-column by block-column, so a stage's
// 128 x 32 tile is one contiguous 16 KiB bulk copy.  The accumulators
// (128 lanes x 128 fp32 columns each) live in tensor memory.
// No TMA multicast anywhere: every load reads this GPU's own memory.
#include <algorithm>

#include "tb_internal.cuh"

namespace tb {
namespace {

constexpr int kTileRows = 128;  // weight rows per CTA (UMMA M)
constexpr int kTileTok = 128;   // tokens per CTA (UMMA N)
constexpr int kStages = 3;
// Tensor-memory accumulators: the tensor core's fp32 accumulation truncates
// each MMA's sum, so the error grows with the number of MMAs folded into one
// accumulator and with its magnitude.  The hi*hi products rotate over three
// accumulators (k-block i into i % 3) and the two small correction products
// (hi*lo, lo*hi, ~2^-11 of the main term) go to a fourth; the epilogue adds
// the four with round-to-nearest.  4 x 128 columns = all 512 of tensor memory.
constexpr int kMainAcc = 3;
constexpr int kTmemCols = 512;
constexpr int kOpBytes = 128 * 32 * 4;    // one 128 x 32 tf32 operand tile
constexpr int kStageBytes = 4 * kOpBytes;  // A hi, A lo, B hi, B lo
constexpr int kGemmThreads = 256;
constexpr size_t kGemmSmem = (size_t)kStages * kStageBytes + 1024;

// ---- tcgen05 / descriptor helpers ----------------------------------------------

// Shared-memory matrix descriptor: K-major, no swizzle, LBO 128 B, SBO 1024 B,
// descriptor version 1 (bits 46-47), layout type 0 (bits 61-63).
__device__ __forceinline__ uint64_t op_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
         (1ull << 46);
}

// Instruction descriptor of kind::tf32: D fp32 (bits 4-5 = 1), A and B tf32
// (bits 7-9, 10-12 = 2), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(kTileTok >> 3) << 17) |
                            ((uint32_t)(kTileRows >> 4) << 24);

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// v = hi + lo: hi keeps the top 11 significant bits (a tf32 value), lo is the
// remainder rounded to tf32 (exact when v has at most 22 significant bits).
__device__ __forceinline__ void split_tf32(float v, float &hi, float &lo) {
  hi = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(__fsub_rn(v, hi)));
  lo = __uint_as_float(r);
}

// int8 (two's complement) byte `sel` of w (already xor-ed with 0x80808080) as
// float: byte into the mantissa of 1.5 * 2^23 (0x4B400000 | byte), minus
// 1.5 * 2^23 + 128.
__device__ __forceinline__ float s8_to_f(uint32_t wx, int sel) {
  return __fsub_rn(__uint_as_float(__byte_perm(wx, 0x4B400000u, 0x7650u | (uint32_t)sel)), 12583040.0f);
}
// unsigned byte (a nibble, 0..15) minus 8, as float
__device__ __forceinline__ float nib_to_f(uint32_t w, int sel) {
  return __fsub_rn(__uint_as_float(__byte_perm(w, 0x4B400000u, 0x7650u | (uint32_t)sel)), 12582920.0f);
}

// ---- activations -> canonical hi/lo operand layout --------------------------------
// Thread per (row m, 16-byte chunk c of quant block kb); eight consecutive
// threads hold one block.  Rows M..M_pad-1 are zero.
template <bool Q4>
__global__ void __launch_bounds__(256) split_x_kernel(const float *__restrict__ x, int M, int K, int M_pad,
                                                      float *__restrict__ xh, float *__restrict__ xl) {
  const int nkb = K / 32;
  const int64_t total = (int64_t)M_pad * nkb * 8;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // all 32 lanes stay in the loop together (the Q4 amax shuffles use the warp)
  const int64_t span = (total + 31) / 32 * 32;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < span; g += stride) {
    const bool live = g < total;
    const int c = (int)(g & 7);
    const int64_t rest = g >> 3;
    const int kb = (int)(rest % nkb);
    const int m = (int)(rest / nkb);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (live && m < M) v = __ldg(reinterpret_cast<const float4 *>(x + (int64_t)m * K + kb * 32 + c * 4));
    if (Q4) {
      // quantize_row_q8_0 (src/tensor/quant_math.hpp:68-90), then q * half(d)
      float a = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
      a = (a == a) ? a : 0.f;
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 4));
      const float d = __fdiv_rn(a, 127.0f);
      const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
      const float dh = __half2float(__float2half_rn(d));
      v.x = __fmul_rn((float)(int8_t)(int)roundf(__fmul_rn(v.x, id)), dh);
      v.y = __fmul_rn((float)(int8_t)(int)roundf(__fmul_rn(v.y, id)), dh);
      v.z = __fmul_rn((float)(int8_t)(int)roundf(__fmul_rn(v.z, id)), dh);
      v.w = __fmul_rn((float)(int8_t)(int)roundf(__fmul_rn(v.w, id)), dh);
    }
    if (!live) continue;
    float4 h, l;
    split_tf32(v.x, h.x, l.x);
    split_tf32(v.y, h.y, l.y);
    split_tf32(v.z, h.z, l.z);
    split_tf32(v.w, h.w, l.w);
    const int64_t off = ((int64_t)kb * (M_pad / 8) + m / 8) * 256 + c * 32 + (m % 8) * 4;  // floats
    *reinterpret_cast<float4 *>(xh + off) = h;
    *reinterpret_cast<float4 *>(xl + off) = l;
  }
}

// ---- the GEMM ----------------------------------------------------------------------
// grid (ceil(N/128), M_pad/128, splits); split z covers quant blocks
// [z*kb_per, min((z+1)*kb_per, nkb)), kb_per a multiple of 8.
template <bool Q4>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_tc_kernel(
    const uint8_t *__restrict__ w, const float *__restrict__ xh, const float *__restrict__ xl, int M,
    int M_pad, int N, int K, int kb_per, float *__restrict__ out, int64_t split_stride,
    uint32_t *__restrict__ err) {
  constexpr int BB = Q4 ? 18 : 34;  // bytes per quant block
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ __align__(8) uint64_t b_full[kStages], a_full[kStages], s_empty[kStages], acc_full;
  __shared__ uint32_t tmem_base;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = K / 32;
  const int n0 = blockIdx.x * kTileRows;
  const int m0 = blockIdx.y * kTileTok;
  const int kb0 = blockIdx.z * kb_per;
  const int kb1 = min(kb0 + kb_per, nkb);
  const int iters = kb1 - kb0;
  // 1 KiB-aligned stage base (the descriptors address 16-byte units)
  uint8_t *base = smem + ((1024 - (smem_addr(smem) & 1023)) & 1023);
  const uint32_t sbase = smem_addr(base);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&a_full[s], 4);
      mbar_init(&s_empty[s], 1);
    }
    mbar_init(&acc_full, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    // ---- activation tiles: two 16 KiB bulk copies per stage --------------------
    if (lane == 0) {
      for (int i = 0; i < iters; ++i) {
        const int s = i % kStages;
        if (i >= kStages && !mbar_wait_bounded(&s_empty[s], ((i / kStages) + 1) & 1, err)) break;
        const int64_t off = ((int64_t)(kb0 + i) * (M_pad / 8) + m0 / 8) * 256;  // floats
        uint8_t *st = base + (size_t)s * kStageBytes;
        mbar_arrive_expect_tx(&b_full[s], 2u * kOpBytes);
        bulk_g2s(st + 2 * kOpBytes, xh + off, kOpBytes, &b_full[s]);
        bulk_g2s(st + 3 * kOpBytes, xl + off, kOpBytes, &b_full[s]);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issue ----------------------------------------------------------------
    if (lane == 0) {
      for (int i = 0; i < iters; ++i) {
        const int s = i % kStages;
        const uint32_t ph = (i / kStages) & 1;
        if (!mbar_wait_bounded(&b_full[s], ph, err) || !mbar_wait_bounded(&a_full[s], ph, err)) break;
        tc_fence_after();
        const uint32_t st = sbase + (uint32_t)(s * kStageBytes);
#pragma unroll
        const uint32_t dmain = tmem + (uint32_t)((i % kMainAcc) * kTileTok);
        const uint32_t dcorr = tmem + (uint32_t)(kMainAcc * kTileTok);
        for (int j = 0; j < 4; ++j) {  // four k-steps of 8 tf32 (32 bytes) per block
          const uint64_t ah = op_desc(st + j * 256), al = op_desc(st + kOpBytes + j * 256);
          const uint64_t bh = op_desc(st + 2 * kOpBytes + j * 256), bl = op_desc(st + 3 * kOpBytes + j * 256);
          mma_tf32(dmain, ah, bh, (i >= kMainAcc || j != 0) ? 1u : 0u);
          mma_tf32(dcorr, ah, bl, (i | j) != 0);
          mma_tf32(dcorr, al, bh, 1);
        }
        mma_commit(&s_empty[s]);
      }
      mma_commit(&acc_full);  // completes when every MMA above has
    }
  } else if (warp >= 4) {
    // ---- converters: weight row t of the tile, one quant block per stage ---------
    // Eight consecutive blocks of a row (272 B for Q8_0, 144 B for Q4_0) start
    // 16-byte aligned (the K range of a CTA starts at a multiple of 8 blocks and
    // a row holds a multiple of 8), so they are loaded as whole 16-byte words and
    // every block's position inside them is a compile-time constant.
    constexpr int GW = 2 * BB;  // 32-bit words per group of eight blocks (68 or 36)
    const int t = threadIdx.x - 128;
    const int n = n0 + t;
    const bool live = n < N;
    const uint4 *wrow = reinterpret_cast<const uint4 *>(w + (int64_t)(live ? n : 0) * nkb * BB);
    bool ok = true;
    for (int g = 0; g < iters && ok; g += 8) {
      uint32_t W[GW];
      const uint4 *src = wrow + (int64_t)(kb0 + g) * BB / 16;
      if (live) {
#pragma unroll
        for (int q = 0; q < GW / 4; ++q) {
          const uint4 u = __ldg(src + q);
          W[4 * q] = u.x; W[4 * q + 1] = u.y; W[4 * q + 2] = u.z; W[4 * q + 3] = u.w;
        }
        if (g + 8 < iters) {  // the next group into L2 while this one is converted
          const char *nx = reinterpret_cast<const char *>(src + GW / 4);
          for (int q = 0; q < 8 * BB; q += 128)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(nx + q));
        }
      } else {
#pragma unroll
        for (int q = 0; q < GW; ++q) W[q] = 0;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = g + u;
        const int s = i % kStages;
        // scale: half at byte BB*u; quants from byte BB*u + 2
        const int sb = BB * u, qb = BB * u + 2;
        const uint32_t dbits = (sb & 2) ? (W[sb >> 2] >> 16) : (W[sb >> 2] & 0xFFFFu);
        const float d = half_bits_to_float((uint16_t)dbits);
        constexpr int NQ = Q4 ? 4 : 8;  // 32-bit words of quants
        uint32_t qw[NQ];
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
          const int wi = (qb >> 2) + q;
          qw[q] = (qb & 2) ? __funnelshift_r(W[wi], W[wi + 1 < GW ? wi + 1 : wi], 16) : W[wi];
        }
        float v[32];
        if (!Q4) {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const uint32_t wx = qw[q] ^ 0x80808080u;
#pragma unroll
            for (int b = 0; b < 4; ++b) v[4 * q + b] = __fmul_rn(s8_to_f(wx, b), d);
          }
        } else {
          // byte j: low nibble = element j, high nibble = element j + 16
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t lo = qw[q] & 0x0F0F0F0Fu, hi = (qw[q] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              v[4 * q + b] = __fmul_rn(nib_to_f(lo, b), d);
              v[16 + 4 * q + b] = __fmul_rn(nib_to_f(hi, b), d);
            }
          }
        }
        if (i >= kStages) {  // every lane waits; the warp leaves together if any gave up
          const bool got = mbar_wait_bounded(&s_empty[s], ((i / kStages) + 1) & 1, err);
          if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            break;
          }
        }
        uint8_t *ah = base + (size_t)s * kStageBytes;
        uint8_t *al = ah + kOpBytes;
        const int rb = (t >> 3) * 1024 + (t & 7) * 16;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          float4 h, l;
          split_tf32(v[4 * c + 0], h.x, l.x);
          split_tf32(v[4 * c + 1], h.y, l.y);
          split_tf32(v[4 * c + 2], h.z, l.z);
          split_tf32(v[4 * c + 3], h.w, l.w);
          *reinterpret_cast<float4 *>(ah + rb + c * 128) = h;
          *reinterpret_cast<float4 *>(al + rb + c * 128) = l;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[s]);
      }
    }
    // ---- epilogue: TMEM lane t holds output column n for the tile's 128 tokens -----
    if (__all_sync(0xffffffffu, mbar_wait_bounded(&acc_full, 0, err))) {
      tc_fence_after();
      const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
      float *o = out + (int64_t)blockIdx.z * split_stride;
      const int nmain = iters < kMainAcc ? iters : kMainAcc;
#pragma unroll 1
      for (int cb = 0; cb < kTileTok / 32; ++cb) {
        // (main 0 + main 1 + main 2) + corrections, each add rounded to nearest
        float acc[32];
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + (uint32_t)(kMainAcc * kTileTok + cb * 32), r);
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = __uint_as_float(r[j]);
        float sum[32];
        tmem_ld32(tmem + lane_base + (uint32_t)(cb * 32), r);
#pragma unroll
        for (int j = 0; j < 32; ++j) sum[j] = __uint_as_float(r[j]);
#pragma unroll 1
        for (int p = 1; p < nmain; ++p) {
          tmem_ld32(tmem + lane_base + (uint32_t)(p * kTileTok + cb * 32), r);
#pragma unroll
          for (int j = 0; j < 32; ++j) sum[j] = __fadd_rn(sum[j], __uint_as_float(r[j]));
        }
        if (live) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int m = m0 + cb * 32 + j;
            if (m < M) o[(int64_t)m * N + n] = __fadd_rn(sum[j], acc[j]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (lane == 0) mbar_wait_bounded(&acc_full, 0, err);  // no MMA may still write the accumulator
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// y[i] = sum over splits, in split order
__global__ void __launch_bounds__(256) sum_splits_kernel(const float *__restrict__ part, int splits, int64_t n,
                                                         float *__restrict__ y) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float s = part[i];
    for (int z = 1; z < splits; ++z) s = __fadd_rn(s, part[(int64_t)z * n + i]);
    y[i] = s;
  }
}

}  // namespace

// Whether the tensor-core path takes this shape: K a multiple of 256 (rows and
// eight-block groups 16-byte aligned), 16-byte aligned weight and activation bases.
bool gemm_tc_eligible(int64_t M, int64_t K, const float *x, const void *w) {
  return M >= 32 && K >= 256 && K % 256 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(x) & 15) == 0;
}

tb_status launch_gemm_tc(int dtype, const float *x, int64_t M, int64_t K, const void *w, int64_t N, float *y,
                         cudaStream_t s, const DeviceState *st) {
  const bool q4 = dtype == TB_Q4_0;
  const int64_t M_pad = (M + kTileTok - 1) / kTileTok * kTileTok;
  const int nkb = (int)(K / 32);
  const int tiles_n = (int)((N + kTileRows - 1) / kTileRows);
  const int tiles_m = (int)(M_pad / kTileTok);
  // split the K loop until the grid covers the SMs (each split >= 32 blocks)
  int splits = 1;
  while ((int64_t)tiles_n * tiles_m * splits * 2 <= st->sm_count && nkb / (splits * 2) >= 32) splits *= 2;
  int kb_per = (nkb + splits - 1) / splits;
  kb_per = (kb_per + 7) / 8 * 8;
  splits = (nkb + kb_per - 1) / kb_per;

  const size_t xbytes = (size_t)M_pad * (size_t)K * sizeof(float);
  const size_t pbytes = splits > 1 ? (size_t)splits * (size_t)M * (size_t)N * sizeof(float) : 0;
  uint8_t *ws = nullptr;
  cudaError_t e = cudaMallocAsync(reinterpret_cast<void **>(&ws), 2 * xbytes + pbytes, s);
  if (e != cudaSuccess) return fail(TB_ENOMEM, "tb_matmul_quant: tensor-core workspace: %s", cudaGetErrorString(e));
  float *xh = reinterpret_cast<float *>(ws);
  float *xl = reinterpret_cast<float *>(ws + xbytes);
  float *part = splits > 1 ? reinterpret_cast<float *>(ws + 2 * xbytes) : y;

  tb_status rs = TB_OK;
  {
    const int64_t chunks = M_pad * nkb * 8;
    const int grid = (int)std::min<int64_t>((chunks + 255) / 256, (int64_t)st->sm_count * 8);
    if (q4)
      split_x_kernel<true><<<grid, 256, 0, s>>>(x, (int)M, (int)K, (int)M_pad, xh, xl);
    else
      split_x_kernel<false><<<grid, 256, 0, s>>>(x, (int)M, (int)K, (int)M_pad, xh, xl);
    rs = check_launch("tb_matmul_quant (activation split)");
  }
  if (rs == TB_OK) {
    const dim3 grid((unsigned)tiles_n, (unsigned)tiles_m, (unsigned)splits);
    const int64_t sstride = (int64_t)M * N;
    if (q4) {
      rs = ensure_smem_for(gemm_tc_kernel<true>, kGemmSmem);
      if (rs == TB_OK)
        gemm_tc_kernel<true><<<grid, kGemmThreads, kGemmSmem, s>>>((const uint8_t *)w, xh, xl, (int)M, (int)M_pad,
                                                                     (int)N, (int)K, kb_per, part, sstride,
                                                                     st->err_word);
    } else {
      rs = ensure_smem_for(gemm_tc_kernel<false>, kGemmSmem);
      if (rs == TB_OK)
        gemm_tc_kernel<false><<<grid, kGemmThreads, kGemmSmem, s>>>((const uint8_t *)w, xh, xl, (int)M,
                                                                      (int)M_pad, (int)N, (int)K, kb_per, part,
                                                                      sstride, st->err_word);
    }
    if (rs == TB_OK) rs = check_launch("tb_matmul_quant (tensor cores)");
  }
  if (rs == TB_OK && splits > 1) {
    const int64_t n = M * N;
    const int grid = (int)std::min<int64_t>((n + 255) / 256, (int64_t)st->sm_count * 8);
    sum_splits_kernel<<<grid, 256, 0, s>>>(part, splits, n, y);
    rs = check_launch("tb_matmul_quant (split sum)");
  }
  e = cudaFreeAsync(ws, s);
  if (rs == TB_OK && e != cudaSuccess) return fail(TB_ECUDA, "tb_matmul_quant: free workspace: %s", cudaGetErrorString(e));
  return rs;
}

}  // namespace tb
