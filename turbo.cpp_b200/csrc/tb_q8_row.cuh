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

// ---- x as three int8 digits per block: the dp4a row dot (K = 2048) -------------
//
// Block b of x (32 values) is scaled by the power of two 2^sh that puts its
// largest magnitude in [2^21, 2^22) and rounded to an integer v (22 bits, an
// error below 2^-22 of the block's largest |x|), written as three signed
// digits v = d2 65536 + d1 256 + d0, each in [-128, 127].  A block's dot with
// the weight quants is then three exact integer dp4a chains; the float result
// (s2 65536 + s1 256 + s0) * (d_w 2^-sh) carries the same rounding as the fp32
// path's.  Blocks with a NaN or an infinity, or whose largest magnitude is
// nonzero but below 2^-104, cannot be written so: the caller falls back to the
// fp32 row dot for them.
//
// Digits are stored lane-interleaved: word q (0..15) of lane L's block pair
// (2L, 2L + 1), digit plane j, at dg[(j * 16 + q) * 32 + L], so that a lane's
// 48 words load without bank conflicts.

__device__ __forceinline__ int q8_sdigit(int v) { return ((v + 128) & 255) - 128; }

// One half block (16 values at xs[(16 h + j) * XS + b]) per thread; both
// halves of a block in adjacent lanes.  Returns true when the block needs the
// fp32 fallback.  sx[b] = 2^-sh.
__device__ __forceinline__ bool q8_make_digits(const float *xs, int XS, int b, int h, uint32_t *dg, float *sx) {
  float v[16];
  float m = 0.f;
  bool nan = false;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    v[j] = xs[(16 * h + j) * XS + b];
    nan |= v[j] != v[j];
    m = fmaxf(m, fabsf(v[j]));
  }
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
  const int E = (int)((__float_as_uint(m) >> 23) & 0xFFu);
  const bool special = nan || (m != 0.f && (E < 24 || E == 255));
  const int sh = 148 - E;  // m 2^sh in [2^21, 2^22)
  const float up = (m != 0.f && !special) ? __uint_as_float((uint32_t)(127 + sh) << 23) : 0.f;
  if (h == 0) sx[b] = (m != 0.f && !special) ? __uint_as_float((uint32_t)(127 - sh) << 23) : 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int iv = __float2int_rn(__fmul_rn(v[4 * i + c], up));  // exact scaling, then one rounding
      const int a0 = q8_sdigit(iv), r1 = (iv - a0) >> 8, a1 = q8_sdigit(r1), a2 = (r1 - a1) >> 8;
      w0 |= (uint32_t)(a0 & 255) << (8 * c);
      w1 |= (uint32_t)(a1 & 255) << (8 * c);
      w2 |= (uint32_t)(a2 & 255) << (8 * c);
    }
    const int q = 8 * (b & 1) + 4 * h + i, L = b >> 1;
    dg[(0 * 16 + q) * 32 + L] = w0;
    dg[(1 * 16 + q) * 32 + L] = w1;
    dg[(2 * 16 + q) * 32 + L] = w2;
  }
  return special;
}

// acc + the two blocks at `wp` (lane's pair) against the digits dgr[3][16] and
// the pair's scales sxr[2]
__device__ __forceinline__ float q8_pair_dot_digits(const uint8_t *wp, const uint32_t (&dgr)[3][16],
                                                    const float (&sxr)[2], float acc) {
  const uint32_t *w32 = reinterpret_cast<const uint32_t *>(wp);
  uint32_t w[17];
#pragma unroll
  for (int k = 0; k < 17; ++k) w[k] = w32[k];
  const float d1 = half_bits_to_float((uint16_t)(w[0] & 0xFFFFu));
  const float d2 = half_bits_to_float((uint16_t)(w[8] >> 16));
  int s[2][3];
#pragma unroll
  for (int j = 0; j < 3; ++j) s[0][j] = s[1][j] = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t qa = __funnelshift_r(w[i], w[i + 1], 16);  // quants 4i..4i+3 of the first block
    const uint32_t qb = w[9 + i];                             // of the second block (4-byte aligned)
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      s[0][j] = __dp4a((int)qa, (int)dgr[j][i], s[0][j]);
      s[1][j] = __dp4a((int)qb, (int)dgr[j][8 + i], s[1][j]);
    }
  }
  const float v0 = fmaf((float)s[0][2], 65536.f, fmaf((float)s[0][1], 256.f, (float)s[0][0]));
  const float v1 = fmaf((float)s[1][2], 65536.f, fmaf((float)s[1][1], 256.f, (float)s[1][0]));
  return fmaf(v1, d2 * sxr[1], fmaf(v0, d1 * sxr[0], acc));
}

__device__ __forceinline__ float q8_row_dot_digits(const uint8_t *wrow, const uint32_t (&dgr)[3][16],
                                                   const float (&sxr)[2], int lane) {
  float acc = q8_pair_dot_digits(wrow + 68 * lane, dgr, sxr, 0.f);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  return acc;
}

}  // namespace tb
