// tb_q8_row.cuh -- reading Q8_0 blocks from shared memory and the default
// (tolerance) dot product of one weight row with x, shared by the decode GEMVs.
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

// x staged in shared memory transposed, xs[j * XS + b] = x[32 b + j], with an
// odd pitch XS; lane l works on blocks l and l + 32 of each 64-block pass and
// keeps those blocks' x in xp[j] = (x[32 b1 + j], x[32 b2 + j]).
__device__ __forceinline__ void q8_load_xp(uint64_t (&xp)[32], const float *xs, int XS, int nb, int pass,
                                           int lane) {
  const int b1 = pass * 64 + lane, b2 = b1 + 32;
#pragma unroll
  for (int j = 0; j < 32; ++j) xp[j] = pack2(b1 < nb ? xs[j * XS + b1] : 0.f, b2 < nb ? xs[j * XS + b2] : 0.f);
}

// Dot product of the Q8_0 row at `wrow` (nb blocks) with x, reduced over the
// warp (every lane returns it).  Each block: quants to float through the
// mantissa of 1.5 * 2^23 (prmt, packed subtraction), two packed fma chains
// (elements 0-15 and 16-31), times the block scale, accumulated per lane in
// block order, then a butterfly sum over the lanes.  With nb <= 64, xp must
// hold pass 0 on entry; otherwise it is reloaded from xs per pass.
__device__ __forceinline__ float q8_row_dot(const uint8_t *wrow, int nb, uint64_t (&xp)[32], const float *xs,
                                            int XS, int lane) {
  const bool onepass = nb <= 64;
  const uint64_t off2 = pack2(-(kMagic + 128.0f), -(kMagic + 128.0f));
  float racc = 0.f;
  for (int p = 0; p * 64 < nb; ++p) {
    const int b1 = p * 64 + lane, b2 = b1 + 32;
    const bool v1 = b1 < nb, v2 = b2 < nb;
    if (!onepass) q8_load_xp(xp, xs, XS, nb, p, lane);
    float d1, d2;
    uint32_t q1[8], q2[8];
    load_q8_block(wrow, 34 * (v1 ? b1 : 0), d1, q1);
    load_q8_block(wrow, 34 * (v2 ? b2 : 0), d2, q2);
    uint64_t acc0 = pack2(0.f, 0.f), acc1 = pack2(0.f, 0.f);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t u1 = q1[kk] ^ 0x80808080u, u2 = q2[kk] ^ 0x80808080u;
      const uint32_t w1 = q1[kk + 4] ^ 0x80808080u, w2 = q2[kk + 4] ^ 0x80808080u;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t sel = 0x7650u | (uint32_t)e;
        const uint64_t m = pack2(__uint_as_float(__byte_perm(u1, kMagicHi, sel)),
                                 __uint_as_float(__byte_perm(u2, kMagicHi, sel)));
        const uint64_t n = pack2(__uint_as_float(__byte_perm(w1, kMagicHi, sel)),
                                 __uint_as_float(__byte_perm(w2, kMagicHi, sel)));
        acc0 = fma2(add2(m, off2), xp[4 * kk + e], acc0);
        acc1 = fma2(add2(n, off2), xp[4 * kk + 16 + e], acc1);
      }
    }
    float s1, s2;
    unpack2(add2(acc0, acc1), s1, s2);
    if (v1) racc = fmaf(s1, d1, racc);
    if (v2) racc = fmaf(s2, d2, racc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) racc += __shfl_xor_sync(0xffffffffu, racc, o);
  return racc;
}

}  // namespace tb
