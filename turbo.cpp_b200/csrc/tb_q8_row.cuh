// tb_q8_row.cuh -- reading Q8_0 blocks from shared memory and the default
// (tolerance) dot product of one weight row with x used by the streaming GEMVs.
#pragma once
#include "tb_internal.cuh"

namespace tb {

constexpr uint32_t kMagicHi = 0x4B400000u;  // float 12582912 = 3 * 2^22
constexpr float kMagic = 12582912.0f;

// Reads the 34-byte Q8_0 block at smem byte offset `off` (even): the scale as
// float and the 32 quants as 8 little-endian words.
__device__ __forceinline__ void load_q8_block(const uint8_t *wsm, int off, float &d, uint32_t qw[8]) {
  const uint32_t *w32 = reinterpret_cast<const uint32_t *>(wsm + (off & ~3));
  uint32_t w[9];
#pragma unroll
  for (int k = 0; k < 9; ++k) w[k] = w32[k];
  const uint32_t sh = (uint32_t)(off & 3) * 8u;  // 0 or 16
  d = half_bits_to_float((uint16_t)(__funnelshift_rc(w[0], w[1], sh) & 0xFFFFu));
#pragma unroll
  for (int k = 0; k < 8; ++k) qw[k] = __funnelshift_rc(w[k], w[k + 1], 16u + sh);
}

// ---- block pairs: the streaming GEMVs' row dot --------------------------------
//
// Lane l of a warp owns the consecutive blocks (2l, 2l + 1) of each 64-block
// pass: 68 bytes that start on a 4-byte boundary whenever the row length is a
// multiple of 4 (nb even), read as 17 words with no bank conflicts (the lanes'
// word offsets 17 l are distinct modulo 32).  Quants are taken straight from
// those words by prmt into the mantissa of 1.5 * 2^23 (after flipping every
// quant byte's sign bit once per word), so no funnel shifts are needed.
// x is staged as xs[j * XS + b] = x[32 b + j] with an even pitch XS, and a
// lane's pair of x columns, xp[j] = (x[32 b + j], x[32 (b + 1) + j]), is one
// 8-byte load per j.

__device__ __forceinline__ void q8_pair_x(float2 (&xp)[32], const float *xs, int XS, int b, bool valid) {
#pragma unroll
  for (int j = 0; j < 32; ++j)
    xp[j] = valid ? *reinterpret_cast<const float2 *>(xs + j * XS + b) : make_float2(0.f, 0.f);
}

// acc + d1 * (q1 . x1) + d2 * (q2 . x2) for the two blocks at `wp` (4-byte
// aligned): per block two packed fma chains (elements 0-15 and 16-31) over
// exact quants, added, times the block scale.
__device__ __forceinline__ float q8_pair_dot(const uint8_t *wp, const float2 (&xp)[32], float acc) {
  const uint32_t *w32 = reinterpret_cast<const uint32_t *>(wp);
  uint32_t w[17];
#pragma unroll
  for (int k = 0; k < 17; ++k) w[k] = w32[k];
  const float d1 = half_bits_to_float((uint16_t)(w[0] & 0xFFFFu));
  const float d2 = half_bits_to_float((uint16_t)(w[8] >> 16));
  // quant bytes: 2..33 (first block) and 36..67 (second); bytes 0-1 and 34-35 are the scales
  w[0] ^= 0x80800000u;
#pragma unroll
  for (int k = 1; k < 8; ++k) w[k] ^= 0x80808080u;
  w[8] ^= 0x00008080u;
#pragma unroll
  for (int k = 9; k < 17; ++k) w[k] ^= 0x80808080u;
  const float2 off2 = make_float2(-(kMagic + 128.0f), -(kMagic + 128.0f));
  float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int a = 2 + j, b = 36 + j, c = 18 + j, e = 52 + j;  // byte offsets of elements j, j + 16
    const float2 m = make_float2(__uint_as_float(__byte_perm(w[a >> 2], kMagicHi, 0x7650u | (a & 3))),
                                 __uint_as_float(__byte_perm(w[b >> 2], kMagicHi, 0x7650u | (b & 3))));
    const float2 n = make_float2(__uint_as_float(__byte_perm(w[c >> 2], kMagicHi, 0x7650u | (c & 3))),
                                 __uint_as_float(__byte_perm(w[e >> 2], kMagicHi, 0x7650u | (e & 3))));
    acc0 = __ffma2_rn(__fadd2_rn(m, off2), xp[j], acc0);
    acc1 = __ffma2_rn(__fadd2_rn(n, off2), xp[16 + j], acc1);
  }
  const float2 s = __fadd2_rn(acc0, acc1);
  return fmaf(s.y, d2, fmaf(s.x, d1, acc));
}

// Dot product of the Q8_0 row at `wrow` (nb blocks, nb even, 4-byte aligned)
// with x, reduced over the warp (every lane returns it).  With nb <= 64, xp
// must hold pass 0 (q8_pair_x at b = 2 lane); otherwise each pass reloads it.
__device__ __forceinline__ float q8_row_dot_pairs(const uint8_t *wrow, int nb, float2 (&xp)[32], const float *xs,
                                                  int XS, int lane) {
  float acc = 0.f;
  if (nb <= 64) {
    if (2 * lane < nb) acc = q8_pair_dot(wrow + 68 * lane, xp, 0.f);
  } else {
    for (int b = 2 * lane; b < nb; b += 64) {
      q8_pair_x(xp, xs, XS, b, true);
      acc = q8_pair_dot(wrow + 34 * b, xp, acc);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  return acc;
}

}  // namespace tb
