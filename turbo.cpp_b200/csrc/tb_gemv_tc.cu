// tb_gemv_tc.cu -- the Q8_0 decode GEMV (M = 1) on the tensor cores.
//
// Arithmetic.  x is cut into 32-wide blocks (the weight blocks' K ranges); each
// block is written as x ~ sx * (X0 * 2^16 + X1 * 2^8 + X2) * 2^-16 with three
// balanced int8 digits per element and sx = max|x_block| / 126 (24 bits below
// the block maximum).  For weight row n and block b the integer dot products
// T_c = sum_j q[n,b,j] * X_c[j] are exact (tcgen05.mma kind::i8, int32
// accumulate), and the block contributes d[n,b] * sx[b] * 2^-16 *
// (T0 * 2^16 + T1 * 2^8 + T2) to y[n], accumulated in fp32 in block order.
// The only rounding besides that fp32 accumulation is the 24-bit
// representation of x: results agree with the float path within ~2e-8 of
// sum |w x| (the tolerance is 1e-5).
//
// Kernel.  One CTA per contiguous range of rows (tiles of <= 128 rows), 320
// threads:
//   warp 8     a 2-D TMA load per stage: the tile's rows x 8 blocks (272 B per
//              row) of raw Q8_0 bytes into a ring of staging buffers
//   warps 4-7  converters: thread = row; the raw row's quants are rearranged
//              into the MMA's K-major layout (8-row x 16-byte core matrices,
//              leading byte offset 128 B, stride byte offset 256 B) and the
//              block scales kept aside -- no per-element arithmetic
//   warp 9     owns tensor memory; one lane issues one M=128, N=8, K=32 MMA per
//              block (the three digit rows of x are the N columns)
//   warps 0-3  epilogue: thread = row = TMEM lane; reads each stage's 8 x 8
//              int32 columns, scales and accumulates
// Tensor-core work is tiny; the point is that the CUDA cores no longer turn
// every weight into a float: ~0.8 instructions per weight instead of ~2.9.
// No TMA multicast anywhere.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "tb_internal.cuh"

namespace tb {
namespace {

constexpr int kStageBlocks = 8;          // 8 blocks x 34 B = 272 B per row per stage
constexpr int kRowStageBytes = 272;
constexpr int kTileRowsMax = 128;        // UMMA M
constexpr int kAStages = 2;
constexpr int kAStageBytes = kTileRowsMax * kStageBlocks * 32;  // 32 KiB
constexpr int kMaxRawStages = 8;
constexpr int kThreads = 320;

__device__ __forceinline__ uint64_t desc_kmajor(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// kind::i8: D s32 (bits 4-5 = 2), A and B signed 8-bit (bits 7-9, 10-12 = 1),
// K-major, N = 8 (N >> 3 at bit 17), M = 128 (M >> 4 at bit 24).
constexpr uint32_t kIdescI8 = (2u << 4) | (1u << 7) | (1u << 10) | (1u << 17) | (8u << 24);

// D = A . B (enable-input-d false: each block's product starts a fresh accumulator)
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdescI8), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void mma_commit_to(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tcf_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tcf_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 2-D tiled TMA load (no multicast) completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, "
      "%36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, "
      "%57, %58, %59, %60, %61, %62, %63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct GemvTcArgs {
  const float *x;
  float *y;
  int N, K;
  int rows_per_cta;  // rows owned by each CTA (the last may own fewer)
  int tile_rows;     // TMA box rows (<= 128)
  int raw_stages;
  int raw_stride;    // bytes per raw stage: tile_rows * 272 rounded up to 128
  PeerOut peer;      // a second copy of the outputs (peer.dst)
};

// Shared memory (dynamic, from a 1 KiB-aligned base):
//   A stages [kAStages][8 blocks][128 rows x 32 B]   canonical MMA layout
//   B tiles  [nb][8 rows x 32 B]                     x digits, rows 3-7 zero
//   raw      [raw_stages][tile_rows x 272 B]         TMA destination
//   sxs      [nb] floats                             x block scale * 2^-16
//   dsc      [kAStages][8 blocks][128 rows] floats   weight block scales
__global__ void __launch_bounds__(kThreads, 1) gemv_tc_kernel(const __grid_constant__ CUtensorMap wmap,
                                                              const GemvTcArgs a, uint32_t *__restrict__ err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t raw_full[kMaxRawStages], raw_empty[kMaxRawStages];
  __shared__ __align__(8) uint64_t a_full[kAStages], acc_full[kAStages], stage_free[kAStages], d_full[kAStages];
  __shared__ __align__(8) uint64_t mma_done;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = a.K / 32, nchunks = nb / kStageBlocks;
  const int n0 = blockIdx.x * a.rows_per_cta;
  const int cnt = min(a.rows_per_cta, a.N - n0);
  const int TR = a.tile_rows;
  const int ntiles = (cnt + TR - 1) / TR;
  const int total = ntiles * nchunks;
  const int RS = a.raw_stages;
  const int RSTR = a.raw_stride;

  uint8_t *base = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
  uint8_t *A = base;
  uint8_t *B = A + kAStages * kAStageBytes;
  uint8_t *raw = B + (size_t)nb * 256;
  float *sxs = reinterpret_cast<float *>(raw + (size_t)RS * RSTR);
  float *dsc = sxs + nb;
  const uint32_t sA = smem_addr(A), sB = smem_addr(B);

  if (threadIdx.x == 0) {
    for (int i = 0; i < RS; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], 4);
    }
    for (int i = 0; i < kAStages; ++i) {
      mbar_init(&a_full[i], 4);
      mbar_init(&acc_full[i], 1);
      mbar_init(&stage_free[i], 4);
      mbar_init(&d_full[i], 4);
    }
    mbar_init(&mma_done, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                 "r"(kAStages * 64));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tcf_before();
  __syncthreads();
  tcf_after();
  const uint32_t tmem = tmem_base;

  // the first weight stages do not depend on the previous kernel
  auto produce = [&](int i) {
    const int t = i / nchunks, kc = i % nchunks, rs = i % RS;
    mbar_arrive_expect_tx(&raw_full[rs], (uint32_t)(TR * kRowStageBytes));
    tma_load_2d(raw + (size_t)rs * RSTR, &wmap, kc * (kRowStageBytes / 4), n0 + t * TR, &raw_full[rs]);
  };
  if (warp == 8 && lane == 0)
    for (int i = 0; i < RS && i < total; ++i) produce(i);
  pdl_launch_dependents();
  pdl_wait();  // x comes from the previous kernel
  const int64_t pbuf = peer_buffer(a.peer);

  // ---- x -> three int8 digits per element in the B tiles (warps 0-7) ----------
  if (warp < 8) {
    for (int i = threadIdx.x; i < nb * 64; i += 256) reinterpret_cast<uint32_t *>(B)[i] = 0u;
  }
  __syncthreads();
  if (warp < 8) {
    for (int g = threadIdx.x; g < nb * 8; g += 256) {  // 8 threads per block, 4 elements each
      const int b = g >> 3, w = g & 7;
      const float4 v = __ldg(reinterpret_cast<const float4 *>(a.x + b * 32 + w * 4));
      float am = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
      am = (am == am) ? am : 0.f;
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 4));
      const float sx = am * (1.0f / 126.0f);
      const float inv = sx > 0.f ? __fdiv_rn(65536.0f, sx) : 0.f;
      const float e[4] = {v.x, v.y, v.z, v.w};
      uint32_t l0 = 0, l1 = 0, l2 = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        int vv = __float2int_rn(__fmul_rn(e[j], inv));
        const int d2 = (int)(int8_t)(vv & 0xFF);
        vv = (vv - d2) >> 8;
        const int d1 = (int)(int8_t)(vv & 0xFF);
        const int d0 = (vv - d1) >> 8;
        l0 |= (uint32_t)(d0 & 0xFF) << (8 * j);
        l1 |= (uint32_t)(d1 & 0xFF) << (8 * j);
        l2 |= (uint32_t)(d2 & 0xFF) << (8 * j);
      }
      // block b, K bytes 4w..4w+3: chunk w/4, digit row c, byte 4(w%4)
      uint32_t *bt = reinterpret_cast<uint32_t *>(B + b * 256 + (w >> 2) * 128 + (w & 3) * 4);
      bt[0] = l0;
      bt[4] = l1;  // + 16 B: row 1
      bt[8] = l2;  // + 32 B: row 2
      if (w == 0) sxs[b] = sx * (1.0f / 65536.0f);
    }
    fence_proxy_async_smem();
  }
  __syncthreads();

  if (warp == 8) {
    // ---- producer ----------------------------------------------------------------
    if (lane == 0) {
      for (int i = RS; i < total; ++i) {
        const int rs = i % RS;
        if (!mbar_wait_bounded(&raw_empty[rs], (uint32_t)(((i / RS) + 1) & 1), err)) {
          abort_flag = 1;
          break;
        }
        produce(i);
      }
    }
  } else if (warp == 9) {
    // ---- MMA issue ---------------------------------------------------------------
    if (lane == 0) {
      for (int i = 0; i < total; ++i) {
        const int kc = i % nchunks, as = i % kAStages;
        if (!mbar_wait_bounded(&a_full[as], (uint32_t)((i / kAStages) & 1), err)) {
          abort_flag = 1;
          break;
        }
        tcf_after();
#pragma unroll
        for (int u = 0; u < kStageBlocks; ++u) {
          const uint64_t ad = desc_kmajor(sA + as * kAStageBytes + u * 4096, 128, 256);
          const uint64_t bd = desc_kmajor(sB + (kc * kStageBlocks + u) * 256, 128, 256);
          mma_i8(tmem + (uint32_t)(as * 64 + u * 8), ad, bd);
        }
        mma_commit_to(&acc_full[as]);
      }
      mma_commit_to(&mma_done);  // completes once every MMA above has
      mbar_wait_bounded(&mma_done, 0, err);
    }
  } else if (warp >= 4) {  // warps 4-7
    // ---- converters: thread j = row j of the tile --------------------------------
    const int j = threadIdx.x - 128;
    for (int i = 0; i < total; ++i) {
      const int t = i / nchunks, rs = i % RS, as = i % kAStages;
      const int tr = min(TR, cnt - t * TR);
      bool ok = mbar_wait_bounded(&raw_full[rs], (uint32_t)((i / RS) & 1), err);
      if (ok && i >= kAStages) ok = mbar_wait_bounded(&stage_free[as], (uint32_t)(((i / kAStages) + 1) & 1), err);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) abort_flag = 1;
        break;
      }
      uint32_t W[68];
      if (j < tr) {
        const uint4 *src = reinterpret_cast<const uint4 *>(raw + (size_t)rs * RSTR + j * kRowStageBytes);
#pragma unroll
        for (int q = 0; q < 17; ++q) {
          const uint4 u = src[q];
          W[4 * q] = u.x;
          W[4 * q + 1] = u.y;
          W[4 * q + 2] = u.z;
          W[4 * q + 3] = u.w;
        }
      } else {
#pragma unroll
        for (int q = 0; q < 68; ++q) W[q] = 0u;
      }
      uint8_t *As = A + as * kAStageBytes;
      float *ds = dsc + as * (kStageBlocks * kTileRowsMax);
#pragma unroll
      for (int u = 0; u < kStageBlocks; ++u) {
        const int sb = 34 * u, qb = 34 * u + 2;  // scale and quants of block u
        const uint32_t dbits = (sb & 2) ? (W[sb >> 2] >> 16) : (W[sb >> 2] & 0xFFFFu);
        ds[u * kTileRowsMax + j] = j < tr ? half_bits_to_float((uint16_t)dbits) : 0.f;
        uint32_t qw[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int wi = (qb >> 2) + q;
          qw[q] = (qb & 2) ? __funnelshift_r(W[wi], W[wi + 1 < 68 ? wi + 1 : wi], 16) : W[wi];
        }
        uint8_t *dst = As + u * 4096 + (j >> 3) * 256 + (j & 7) * 16;
        *reinterpret_cast<uint4 *>(dst) = make_uint4(qw[0], qw[1], qw[2], qw[3]);
        *reinterpret_cast<uint4 *>(dst + 128) = make_uint4(qw[4], qw[5], qw[6], qw[7]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&a_full[as]);
        mbar_arrive(&d_full[as]);  // the block scales, for the epilogue
        mbar_arrive(&raw_empty[rs]);
      }
    }
  } else {
    // ---- epilogue (warps 0-3): thread j = row j = TMEM lane j ---------------------
    const int j = threadIdx.x;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    float acc = 0.f;
    for (int i = 0; i < total; ++i) {
      const int t = i / nchunks, kc = i % nchunks, as = i % kAStages;
      const uint32_t ph = (uint32_t)((i / kAStages) & 1);
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&acc_full[as], ph, err) && mbar_wait_bounded(&d_full[as], ph, err))) {
        if (lane == 0) abort_flag = 1;
        break;
      }
      tcf_after();
      uint32_t r[64];
      tmem_ld64(tmem + lane_base + (uint32_t)(as * 64), r);
      const float *ds = dsc + as * (kStageBlocks * kTileRowsMax);
#pragma unroll
      for (int u = 0; u < kStageBlocks; ++u) {
        const float f = fmaf((float)(int)r[u * 8], 65536.0f, fmaf((float)(int)r[u * 8 + 1], 256.0f, (float)(int)r[u * 8 + 2]));
        acc = fmaf(f, __fmul_rn(ds[u * kTileRowsMax + j], sxs[kc * kStageBlocks + u]), acc);
      }
      tcf_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&stage_free[as]);
      if (kc == nchunks - 1) {
        const int row = t * TR + j;
        if (j < TR && row < cnt) {
          a.y[n0 + row] = acc;
          peer_store(a.peer, pbuf, n0 + row, acc);
        }
        acc = 0.f;
      }
    }
  }
  tcf_before();
  __syncthreads();
  if (warp == 9) {
    tcf_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kAStages * 64));
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

}  // namespace

// Whether the tensor-core GEMV takes this shape: K a multiple of 256, 16-byte
// aligned weights and x, and at least 32768 rows.  Each CTA then owns hundreds
// of rows, enough stages to fill the load -> rearrange -> MMA -> epilogue
// pipeline; with a few dozen rows per CTA that pipeline's per-stage latency
// dominates and the ring GEMV is faster (measured: 128256 x 2048 49.5 us
// against 69.5 us; 8192 x 2048 10.2 us against 7.2 us; 2048 x 8192 26.8 us
// against 9.3 us).
bool gemv_tc_eligible(int64_t K, int64_t N, const void *w, const float *x) {
  return K >= 256 && K % 256 == 0 && K <= 16384 && N >= 32768 && N <= 0x7FFFFFFF &&
         (reinterpret_cast<uintptr_t>(w) & 15) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
         encode_fn() != nullptr;
}

tb_status launch_gemv_tc(const float *x, int64_t K, const void *w, int64_t N, float *y, cudaStream_t s,
                         const DeviceState *st, const PeerOut *peer) {
  const int nb = (int)(K / 32);
  const int rb = nb * 34;
  const int G0 = st->sm_count;
  const int rows_per_cta = (int)((N + G0 - 1) / G0);
  const int grid = (int)((N + rows_per_cta - 1) / rows_per_cta);
  const int TR = std::min(rows_per_cta, kTileRowsMax);
  const size_t fixed = 1024 + (size_t)kAStages * kAStageBytes + (size_t)nb * 256 + (size_t)nb * 4 +
                       (size_t)kAStages * kStageBlocks * kTileRowsMax * 4;
  const size_t per_raw = ((size_t)TR * kRowStageBytes + 127) / 128 * 128;
  int RS = (int)std::min<size_t>(kMaxRawStages, ((size_t)st->smem_optin - fixed) / per_raw);
  if (RS < 2) return fail(TB_EINVAL, "tensor-core GEMV: K=%lld does not fit", (long long)K);
  const size_t smem = fixed + (size_t)RS * per_raw;

  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)(rb / 4), (cuuint64_t)N};
  const cuuint64_t strides[1] = {(cuuint64_t)rb};
  const cuuint32_t box[2] = {(cuuint32_t)(kRowStageBytes / 4), (cuuint32_t)TR};
  const cuuint32_t estr[2] = {1, 1};
  CUresult cr = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void *>(w), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(TB_ECUDA, "tensor-core GEMV: tensor map (error %d)", (int)cr);

  GemvTcArgs a;
  a.x = x;
  a.y = y;
  a.N = (int)N;
  a.K = (int)K;
  a.rows_per_cta = rows_per_cta;
  a.tile_rows = TR;
  a.raw_stages = RS;
  a.raw_stride = (int)per_raw;
  a.peer = peer ? *peer : PeerOut{};
  TB_TRY(ensure_smem_for(gemv_tc_kernel, smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_tc_kernel, map, a, st->err_word);
  if (e != cudaSuccess) return fail(TB_ECUDA, "tensor-core GEMV launch: %s", cudaGetErrorString(e));
  return TB_OK;
}

}  // namespace tb
