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

// Q8_0 quantisation, one warp per block of 32 (quant_math.hpp:68-90):
// amax with NaN ignored (std::max keeps the running max), d = amax / 127,
// stored as half (round to nearest even), id = 1/d from the fp32 d,
// q = roundf(x * id) (half away from zero).
__global__ void __launch_bounds__(256) quantize_q8_0_kernel(const float *__restrict__ x,
                                                            int64_t rows, int64_t k,
                                                            uint8_t *__restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t nb_row = k / 32;
  const int64_t total = rows * nb_row;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t blk = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); blk < total;
       blk += warps) {
    int64_t r = blk / nb_row, b = blk % nb_row;
    float v = x[r * k + b * 32 + lane];
    float a = fabsf(v);
    a = (a == a) ? a : 0.f;  // a NaN never replaces the running max
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    float d = __fdiv_rn(a, 127.0f);
    float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
    uint8_t *ob = out + blk * 34;
    int q = (int)roundf(__fmul_rn(v, id));
    ob[2 + lane] = (uint8_t)(int8_t)q;
    if (lane == 0) {
      // Explicit byte stores: nvcc 12.9 was seen to drop the low byte when the
      // two halves of a 16-bit value were stored as `h & 0xFF` / `h >> 8`.
      const uint32_t h = __half_as_ushort(__float2half_rn(d));
      asm volatile("st.u8 [%0], %1;" ::"l"(ob), "r"(h & 0xFFu) : "memory");
      asm volatile("st.u8 [%0], %1;" ::"l"(ob + 1), "r"(h >> 8) : "memory");
    }
  }
}

}  // namespace

// Launches the Q8_0 quantisation with the caller's SM count (no device-state
// lookup), for entry points that must not allocate.
tb_status launch_quantize_q8_0(const float *x, int64_t rows, int64_t k, void *blocks, cudaStream_t s,
                               int sm_count) {
  int64_t total = rows * (k / 32);
  int grid = (int)std::min<int64_t>((total + 7) / 8, (int64_t)sm_count * 16);
  if (grid < 1) grid = 1;
  quantize_q8_0_kernel<<<grid, 256, 0, s>>>(x, rows, k, (uint8_t *)blocks);
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
  int64_t total = rows * (k / 32);
  int grid = (int)std::min<int64_t>((total + 7) / 8, (int64_t)st->sm_count * 16);
  quantize_q8_0_kernel<<<grid, 256, 0, as_stream(stream)>>>(x, rows, k, (uint8_t *)blocks);
  return check_launch("tb_quantize_q8_0");
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
