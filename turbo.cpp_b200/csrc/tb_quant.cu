// tb_quant.cu -- GGUF block formats: exact dequantisation (A14/A17), Q8_0
// quantisation of activations (A11, first half) and the embedding gather (A14).
//
// Blocks are 34 B (Q8_0) or 18 B (Q4_0), so a block never starts on a 16-byte
// boundary.  A warp therefore moves a run of 32 consecutive blocks (1088 B or
// 576 B, contiguous) into shared memory with coalesced 32-bit loads and then
// unpacks it so that each output row of 32 floats is written by 8 lanes with
// 16-byte stores: reads and writes are both fully coalesced.
#include <algorithm>

#include "tb_internal.cuh"

namespace tb {
namespace {

constexpr int kWarps = 8;

template <int BB>  // block bytes: 34 (Q8_0) or 18 (Q4_0)
__device__ __forceinline__ void unpack_block4(const uint8_t *blk, int e0, float out[4]) {
  float d = half_bits_to_float((uint16_t)(blk[0] | (blk[1] << 8)));
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    int e = e0 + k;
    if (BB == 34) {
      out[k] = __fmul_rn((float)(int8_t)blk[2 + e], d);  // q * d (quant_math.hpp:26)
    } else {
      uint8_t p = blk[2 + (e & 15)];
      int q = (e < 16 ? (p & 0x0F) : (p >> 4)) - 8;  // embedding.cpp:58-59
      out[k] = __fmul_rn((float)q, d);
    }
  }
}

// Copies `nbytes` (<= 32*BB) starting at `src` into warp-private smem `dst`
// with 32-bit loads when aligned, byte loads otherwise.
__device__ __forceinline__ void warp_stage(uint8_t *dst, const uint8_t *src, int nbytes, int lane) {
  if ((reinterpret_cast<uintptr_t>(src) & 3) == 0) {
    const uint32_t *s32 = reinterpret_cast<const uint32_t *>(src);
    uint32_t *d32 = reinterpret_cast<uint32_t *>(dst);
    int nw = nbytes / 4;
    for (int i = lane; i < nw; i += 32) d32[i] = __ldcs(s32 + i);
    for (int i = nw * 4 + lane; i < nbytes; i += 32) dst[i] = src[i];
  } else {
    for (int i = lane; i < nbytes; i += 32) dst[i] = src[i];
  }
}

// Dequantise `nblocks` consecutive blocks (each warp takes runs of 32).
template <int BB>
__global__ void __launch_bounds__(kWarps * 32) dequant_kernel(const uint8_t *__restrict__ w,
                                                             int64_t nblocks,
                                                             float *__restrict__ y) {
  __shared__ __align__(16) uint8_t stage[kWarps][32 * BB + 4];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int64_t nruns = (nblocks + 31) / 32;
  for (int64_t run = (int64_t)blockIdx.x * kWarps + wid; run < nruns;
       run += (int64_t)gridDim.x * kWarps) {
    int64_t b0 = run * 32;
    int nb = (int)(nblocks - b0 < 32 ? nblocks - b0 : 32);
    warp_stage(stage[wid], w + b0 * BB, nb * BB, lane);
    __syncwarp();
    // 4 blocks per step: lane l -> block l/8, elements 4*(l%8)..+3
    for (int b = lane >> 3; b < nb; b += 4) {
      float v[4];
      unpack_block4<BB>(stage[wid] + b * BB, (lane & 7) * 4, v);
      float4 o = make_float4(v[0], v[1], v[2], v[3]);
      __stcs(reinterpret_cast<float4 *>(y + (b0 + b) * 32) + (lane & 7), o);
    }
    __syncwarp();
  }
}

// Embedding: rows of `dim/32` blocks gathered by id.  grid.x covers
// (token, run-of-32-blocks) pairs.
template <int BB>
__global__ void __launch_bounds__(kWarps * 32) embedding_q_kernel(
    const uint8_t *__restrict__ w, int64_t dim, int64_t vocab, const int32_t *__restrict__ ids,
    int64_t n, float *__restrict__ out, uint32_t *__restrict__ err) {
  __shared__ __align__(16) uint8_t stage[kWarps][32 * BB + 4];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int64_t nb_row = dim / 32;
  const int64_t runs_row = (nb_row + 31) / 32;
  const int64_t total = n * runs_row;
  for (int64_t job = (int64_t)blockIdx.x * kWarps + wid; job < total;
       job += (int64_t)gridDim.x * kWarps) {
    int64_t t = job / runs_row, run = job % runs_row;
    int64_t id = ids[t];
    int64_t b0 = run * 32;
    int nb = (int)(nb_row - b0 < 32 ? nb_row - b0 : 32);
    float *orow = out + t * dim + b0 * 32;
    if (id < 0 || id >= vocab) {  // out of range: zeros + error bit
      if (lane == 0 && run == 0) atomicOr(err, ERR_INDEX);
      for (int i = lane; i < nb * 32; i += 32) orow[i] = 0.f;
      continue;
    }
    warp_stage(stage[wid], w + (id * nb_row + b0) * BB, nb * BB, lane);
    __syncwarp();
    for (int b = lane >> 3; b < nb; b += 4) {
      float v[4];
      unpack_block4<BB>(stage[wid] + b * BB, (lane & 7) * 4, v);
      reinterpret_cast<float4 *>(orow + b * 32)[lane & 7] = make_float4(v[0], v[1], v[2], v[3]);
    }
    __syncwarp();
  }
}

// FP32 weight of logical shape {dim, vocab}: element d of token id is at
// d * vocab + id (embedding.cpp:46-49, 91-94).
__global__ void embedding_f32_kernel(const float *__restrict__ w, int64_t dim, int64_t vocab,
                                     const int32_t *__restrict__ ids, int64_t n,
                                     float *__restrict__ out, uint32_t *__restrict__ err) {
  int64_t total = n * dim;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t t = i / dim, d = i % dim;
    int64_t id = ids[t];
    if (id < 0 || id >= vocab) {
      if (d == 0) atomicOr(err, ERR_INDEX);
      out[i] = 0.f;
    } else {
      out[i] = w[d * vocab + id];
    }
  }
}

// Q8_0 quantisation (quant_math.hpp:68-90): amax with NaN ignored (std::max
// keeps the running max), d = amax / 127, stored as half (round to nearest
// even), id = 1/d from the fp32 d, q = roundf(x * id) (half away from zero).
// With k a multiple of 32 the blocks of consecutive rows are consecutive, so
// block i reads x[32 i, 32 i + 32).  One warp takes 32 consecutive blocks:
// 8 coalesced 16-byte loads per lane (8 lanes per block), the amax over each
// group of 8 lanes, the 1088 output bytes assembled in shared memory and
// written as 68 16-byte stores.
constexpr int kQuantWarps = 8;

__device__ __forceinline__ void st_shared_u16(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

__global__ void __launch_bounds__(kQuantWarps * 32) quantize_q8_0_kernel(const float *__restrict__ x,
                                                                         int64_t nblocks,
                                                                         uint8_t *__restrict__ out) {
  __shared__ __align__(16) uint8_t stage[kQuantWarps][32 * 34];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane & 7;  // this lane's 4 values of its block
  const bool vin = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  const bool vout = (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(&stage[warp][0]);
  const int64_t nwarps = (int64_t)gridDim.x * kQuantWarps;
  for (int64_t g = (int64_t)blockIdx.x * kQuantWarps + warp; g * 32 < nblocks; g += nwarps) {
    const int64_t b0 = g * 32;
    const int nb = (nblocks - b0 < 32) ? (int)(nblocks - b0) : 32;
    float4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int bl = j * 4 + (lane >> 3);
      v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (bl < nb) {
        const float *p = x + (b0 + bl) * 32 + sub * 4;
        v[j] = vin ? __ldcs(reinterpret_cast<const float4 *>(p)) : make_float4(p[0], p[1], p[2], p[3]);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int bl = j * 4 + (lane >> 3);
      float a = fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w)));
      a = (a == a) ? a : 0.f;  // fmaxf already skips a NaN operand; all four NaN gives 0
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 4));
      const float d = __fdiv_rn(a, 127.0f);
      const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
      const uint32_t q0 = (uint32_t)(uint8_t)(int8_t)(int)roundf(__fmul_rn(v[j].x, id));
      const uint32_t q1 = (uint32_t)(uint8_t)(int8_t)(int)roundf(__fmul_rn(v[j].y, id));
      const uint32_t q2 = (uint32_t)(uint8_t)(int8_t)(int)roundf(__fmul_rn(v[j].z, id));
      const uint32_t q3 = (uint32_t)(uint8_t)(int8_t)(int)roundf(__fmul_rn(v[j].w, id));
      // block bl occupies stage bytes [34 bl, 34 bl + 34): half d, then 32 quants
      const uint32_t at = sbase + (uint32_t)(bl * 34);
      st_shared_u16(at + 2 + sub * 4, q0 | (q1 << 8));
      st_shared_u16(at + 4 + sub * 4, q2 | (q3 << 8));
      if (sub == 0) st_shared_u16(at, __half_as_ushort(__float2half_rn(d)));
    }
    __syncwarp();
    uint8_t *ob = out + b0 * 34;
    if (nb == 32 && vout) {
      const uint4 *src = reinterpret_cast<const uint4 *>(&stage[warp][0]);
      for (int i = lane; i < 68; i += 32) reinterpret_cast<uint4 *>(ob)[i] = src[i];
    } else {
      for (int i = lane; i < nb * 34; i += 32) ob[i] = stage[warp][i];
    }
    __syncwarp();
  }
}

}  // namespace

// Launches the Q8_0 quantisation with the caller's SM count (no device-state
// lookup), for entry points that must not allocate.
tb_status launch_quantize_q8_0(const float *x, int64_t rows, int64_t k, void *blocks, cudaStream_t s,
                               int sm_count) {
  const int64_t total = rows * (k / 32);
  const int64_t groups = (total + 31) / 32;
  int grid = (int)std::min<int64_t>((groups + kQuantWarps - 1) / kQuantWarps, (int64_t)sm_count * 8);
  if (grid < 1) grid = 1;
  quantize_q8_0_kernel<<<grid, kQuantWarps * 32, 0, s>>>(x, total, (uint8_t *)blocks);
  return check_launch("quantize_q8_0");
}

}  // namespace tb

using namespace tb;

extern "C" {

tb_status tb_dequant(int dtype, const void *blocks, int64_t nblocks, float *y, tb_stream stream) {
  if (nblocks < 0) return fail(TB_EINVAL, "tb_dequant: negative block count");
  if (nblocks == 0) return TB_OK;
  if (!blocks || !y) return fail(TB_EINVAL, "tb_dequant: null pointer");
  if ((reinterpret_cast<uintptr_t>(y) & 15) != 0) return fail(TB_EINVAL, "tb_dequant: output must be 16-byte aligned");
  DeviceState *st;
  TB_TRY(device_state(&st));
  int64_t runs = (nblocks + 31) / 32;
  int grid = (int)std::min<int64_t>((runs + kWarps - 1) / kWarps, (int64_t)st->sm_count * 8);
  if (dtype == TB_Q8_0)
    dequant_kernel<34><<<grid, kWarps * 32, 0, as_stream(stream)>>>((const uint8_t *)blocks, nblocks, y);
  else if (dtype == TB_Q4_0)
    dequant_kernel<18><<<grid, kWarps * 32, 0, as_stream(stream)>>>((const uint8_t *)blocks, nblocks, y);
  else
    return fail(TB_EINVAL, "tb_dequant: dtype must be TB_Q8_0 or TB_Q4_0");
  return check_launch("tb_dequant");
}

tb_status tb_quantize_q8_0(const float *x, int64_t rows, int64_t k, void *blocks, tb_stream stream) {
  if (rows < 0 || k < 0 || k % 32 != 0) return fail(TB_EINVAL, "tb_quantize_q8_0: k must be a multiple of 32");
  if (rows == 0 || k == 0) return TB_OK;
  if (!x || !blocks) return fail(TB_EINVAL, "tb_quantize_q8_0: null pointer");
  DeviceState *st;
  TB_TRY(device_state(&st));
  return launch_quantize_q8_0(x, rows, k, blocks, as_stream(stream), st->sm_count);
}

tb_status tb_embedding(int dtype, const void *w, int64_t dim, int64_t vocab, const int32_t *ids,
                       int64_t n, float *out, tb_stream stream) {
  if (dim < 0 || vocab < 0 || n < 0) return fail(TB_EINVAL, "tb_embedding: negative extent");
  if (n == 0 || dim == 0) return TB_OK;
  if (!w || !ids || !out) return fail(TB_EINVAL, "tb_embedding: null pointer");
  DeviceState *st;
  TB_TRY(device_state(&st));
  cudaStream_t s = as_stream(stream);
  if (dtype == TB_F32) {
    int64_t total = n * dim;
    int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)st->sm_count * 8);
    embedding_f32_kernel<<<grid, 256, 0, s>>>((const float *)w, dim, vocab, ids, n, out, st->err_word);
    return check_launch("tb_embedding");
  }
  if (dtype != TB_Q8_0 && dtype != TB_Q4_0)
    return fail(TB_ERUNTIME, "Unsupported embedding dtype");
  if (dim % 32 != 0) return fail(TB_EINVAL, "tb_embedding: dim must be a multiple of 32 for block formats");
  if ((reinterpret_cast<uintptr_t>(out) & 15) != 0) return fail(TB_EINVAL, "tb_embedding: output must be 16-byte aligned");
  int64_t jobs = n * ((dim / 32 + 31) / 32);
  int grid = (int)std::min<int64_t>((jobs + kWarps - 1) / kWarps, (int64_t)st->sm_count * 8);
  if (dtype == TB_Q8_0)
    embedding_q_kernel<34><<<grid, kWarps * 32, 0, s>>>((const uint8_t *)w, dim, vocab, ids, n, out, st->err_word);
  else
    embedding_q_kernel<18><<<grid, kWarps * 32, 0, s>>>((const uint8_t *)w, dim, vocab, ids, n, out, st->err_word);
  return check_launch("tb_embedding");
}

}  // extern "C"
