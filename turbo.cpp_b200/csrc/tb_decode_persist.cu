// tb_decode_persist.cu -- one whole decode step of a Llama-shaped MiniGPT (all
// layers, the final norm and the LM head) as ONE persistent cooperative
// kernel: tb_decode_step_persistent.
//
// The op-by-op and fused decode paths launch a kernel per op; every launch
// waits for its predecessor to finish before its own input is ready, and that
// chain, not HBM, bounds the step.  Here one CTA per SM runs the whole step:
//
//   * a producer warp streams every weight row the CTA owns, in the order the
//     step consumes them (layer by layer: Q/K/V, O, gate/up, down; then the LM
//     head), through a ring of shared-memory spans with one bulk copy per span
//     (full/empty mbarriers).  Weights never depend on activations, so the
//     stream never waits for a phase: it runs ahead as far as the ring allows;
//   * twelve consumer warps (three groups of four; span i goes to group i % 3,
//     chunk j of a span to warp j of the group) compute the row dot products of
//     each phase once its input vector is ready, and write that phase's
//     outputs; phases are separated by grid barriers (a monotonic 64-bit
//     arrival counter, bounded spins that give up, flag the device error word
//     and end the kernel).
//
// Per layer (reference op sequence, src/nn/transformer_block.cpp,
// attention.cpp:41-148, ffn.cpp:17-27, one token):
//   A  xn = RMSNorm(h) * attn_norm; q, k, v = Wq xn, Wk xn, Wv xn
//   B  RoPE of q and k at pos; k, v into the caches' row pos; attention of the
//      query heads of each key/value head over key chunks (flash-decoding
//      partials: max, sum of exp, unnormalised output per chunk); the CTA that
//      finishes a key/value head's last chunk combines its partials into ctx
//   C  h2 = h + Wo ctx
//   D  xn = RMSNorm(h2) * ffn_norm; act = silu(Wg xn) * (Wu xn)
//   E  h = h2 + Wd act
// then xn = RMSNorm(h) * final_norm and logits = W_lm xn.
//
// Arithmetic per dot product is the streaming GEMV's (tb_q8_row.cuh: exact
// block products, fp32 accumulation), RMSNorm divides by the rms as
// src/nn/rmsnorm.cpp does, SwiGLU is swiglu_f32, attention scores are the fp32
// matmul's fma chain over d times the scale; only summation orders differ from
// the op-by-op path (within the GEMV and softmax tolerances).
//
// Shapes: hidden 2048 (one 64-block chunk per row), head_dim 64, ffn a
// multiple of 2048 with ffn / 2048 in {1, 2, 4}, at most 4 query heads per
// key/value head, max_seq <= 2048; Q8_0 weights with 16-byte-aligned rows.
#include <algorithm>

#include "tb_internal.cuh"
#include "tb_q8_row.cuh"

namespace tb {
namespace {

constexpr int kCW = 12;                         // consumer warps (3 groups of 4)
constexpr int kNG = kCW / 4;                    // consumer groups
constexpr int kCT = kCW * 32;                   // consumer threads
constexpr int kThreads = kCT + 32;              // + the producer warp
constexpr int kE = 2048;                        // hidden size this kernel is built for
constexpr int kNB = kE / 32;                    // blocks per 2048-wide chunk
constexpr int kChunk = kNB * 34;                // 2176 bytes: 2048 weights of one row
constexpr int kSpanChunks = 4;
constexpr int kSpan = kSpanChunks * kChunk;     // 8704 bytes
constexpr int kSlots = 21;                      // ring spans (a multiple of kNG)
constexpr int kXS = kNB + 2;                    // transposed x pitch (even)
constexpr int kMaxFC = 4;                       // ffn / 2048
constexpr int kNCH = 8;                         // attention key chunks per key/value head
constexpr int kMaxG = 4;                        // query heads per key/value head
constexpr int kMaxSeq = 2048;
constexpr int kMaxKeys = kMaxSeq / kNCH;        // keys per chunk
constexpr int kD = 64;                          // head_dim
constexpr int kPart = 4 + kD;                   // partial: max, sum, 2 pad, out[64] (16-byte aligned)
constexpr int kSlices = 2 * kCW;                // key slices of the probability x V sums
constexpr uint64_t kWaitNs = 2000000000ull;

static_assert(kSlots % kNG == 0, "span i and span i + kSlots belong to the same group");

typedef tb_decode_layer PLayer;
__device__ __forceinline__ const uint8_t *u8(const void *p) { return static_cast<const uint8_t *>(p); }

struct PArgs {
  const PLayer *layers;
  int L, F, H, KVH, V, max_seq, rope_max_seq;
  float eps_attn, eps_ffn, eps_final, scale;
  const uint8_t *emb, *lm;
  const float *final_norm, *cos_t, *sin_t;
  const int32_t *token, *pos;
  float *logits;
  // workspace
  float *hA, *hB, *q, *k, *v, *part, *ctx, *act;
  unsigned long long *ctr;
  int *abort_flag;
  int *head_done;  // per key/value head: key chunks finished in this layer
  uint32_t *err;
};

// contiguous share [lo, hi) of n rows for CTA b of G
__device__ __forceinline__ void share(int n, int G, int b, int &lo, int &hi) {
  const int base = n / G, rem = n % G;
  lo = b * base + min(b, rem);
  hi = lo + base + (b < rem ? 1 : 0);
}

__device__ __forceinline__ uint64_t ld_acquire_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_volatile_i32(const int *p) {
  int v;
  asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void cons_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kCT) : "memory"); }
__device__ __forceinline__ void group_sync(int g) { asm volatile("bar.sync %0, 128;" ::"r"(2 + g) : "memory"); }
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t *bar) { mbar_arrive(bar); }

struct Smem {
  uint64_t full[kSlots];
  uint64_t empty[kSlots];
  double tab[64];                   // exp_cr table (SwiGLU)
  float red[kCW];
  float gsum[kNG][2][4];            // per group, double-buffered chunk partials
  float gate[64], up[64];           // this CTA's gate/up results (<= 64 rows)
  int4 meta[kSlots];                // per slot: phase, first row, rows, chunks per row (written by the producer)
  int abort_local;
  int pad[3];
};

// Span walk shared by the producer and the consumers: every weight span the
// CTA streams, in consumption order.  A span is up to four 2176-byte chunks,
// contiguous in global memory except where it crosses from one of Wq/Wk/Wv
// into the next (two pieces then).
struct SpanInfo {
  const uint8_t *src0, *src1;
  uint32_t bytes0, bytes1;
  int rows;       // rows in the span
  int row0;       // first row (phase-relative, or within the concatenated Q/K/V rows)
  int cpr;        // chunks per row (1, 2 or 4)
};

__device__ __forceinline__ SpanInfo span_rows(const uint8_t *w, int row0, int rows, int cpr) {
  SpanInfo s;
  s.src0 = w + (int64_t)row0 * cpr * kChunk;
  s.bytes0 = (uint32_t)(rows * cpr * kChunk);
  s.src1 = nullptr;
  s.bytes1 = 0;
  s.rows = rows;
  s.row0 = row0;
  s.cpr = cpr;
  return s;
}

// rows [r, r + n) of the concatenation Wq (E rows) | Wk (kv rows) | Wv (kv rows)
__device__ __forceinline__ SpanInfo span_qkv(const PLayer &ly, int r, int n, int kv) {
  SpanInfo s;
  s.rows = n;
  s.row0 = r;
  s.cpr = 1;
  // segment of row r and the segment after it (selects, not indexed arrays)
  const bool inq = r < kE, ink = !inq && r < kE + kv;
  const uint8_t *b0 = inq ? u8(ly.wq) : (ink ? u8(ly.wk) : u8(ly.wv));
  const uint8_t *b1 = inq ? u8(ly.wk) : u8(ly.wv);
  const int start = inq ? 0 : (ink ? kE : kE + kv);
  const int lim = inq ? kE : (ink ? kE + kv : kE + 2 * kv);
  const int n0 = min(n, lim - r);
  s.src0 = b0 + (int64_t)(r - start) * kChunk;
  s.bytes0 = (uint32_t)(n0 * kChunk);
  s.src1 = n0 < n ? b1 : nullptr;
  s.bytes1 = n0 < n ? (uint32_t)((n - n0) * kChunk) : 0u;
  return s;
}

// The CTA's weight spans in consumption order, as a resumable cursor (the
// producer and every consumer warp keep one each).  Phases: 0 = Q/K/V rows,
// 2 = O, 3 = gate, 4 = up (gate and up spans of the same rows alternate),
// 5 = down, 6 = LM head, 7 = end.
struct Cursor {
  int l, ph, r, lo, hi;
};

__device__ __forceinline__ void cur_phase(Cursor &c, const PArgs &a, int G, int b, int ph) {
  c.ph = ph;
  const int n = ph == 0 ? kE + 2 * a.KVH * kD : (ph == 2 || ph == 5) ? kE : (ph == 3 ? a.F : (ph == 6 ? a.V : 0));
  if (ph != 4) {
    share(n, G, b, c.lo, c.hi);
    c.r = c.lo;
  }
}

__device__ __forceinline__ void cur_init(Cursor &c, const PArgs &a, int G, int b) {
  c.l = 0;
  cur_phase(c, a, G, b, 0);
}

// Skips phases with no rows left; afterwards c.ph is the next span's phase.
__device__ __forceinline__ void cur_norm(Cursor &c, const PArgs &a, int G, int b) {
  while (c.ph != 7 && c.r >= c.hi) {
    if (c.ph == 0) cur_phase(c, a, G, b, 2);
    else if (c.ph == 2) cur_phase(c, a, G, b, 3);
    else if (c.ph == 3 || c.ph == 4) cur_phase(c, a, G, b, 5);
    else if (c.ph == 5) {
      if (++c.l < a.L) cur_phase(c, a, G, b, 0);
      else cur_phase(c, a, G, b, 6);
    } else c.ph = 7;
  }
}

// The next span and its phase; false at the end.
__device__ __forceinline__ bool cur_next(Cursor &c, const PArgs &a, int G, int b, SpanInfo &s, int &ph) {
  cur_norm(c, a, G, b);
  ph = c.ph;
  if (ph == 7) return false;
  const int kv = a.KVH * kD, fc = a.F / kE;
  if (ph == 0) {
    const int n = min(4, c.hi - c.r);
    s = span_qkv(a.layers[c.l], c.r, n, kv);
    c.r += n;
  } else if (ph == 2) {
    const int n = min(4, c.hi - c.r);
    s = span_rows(u8(a.layers[c.l].wo), c.r, n, 1);
    c.r += n;
  } else if (ph == 3) {
    s = span_rows(u8(a.layers[c.l].w_gate), c.r, min(4, c.hi - c.r), 1);
    c.ph = 4;  // the up rows of the same indices come next
  } else if (ph == 4) {
    const int n = min(4, c.hi - c.r);
    s = span_rows(u8(a.layers[c.l].w_up), c.r, n, 1);
    c.r += n;
    c.ph = 3;
  } else if (ph == 5) {
    const int n = min(kSpanChunks / fc, c.hi - c.r);
    s = span_rows(u8(a.layers[c.l].w_down), c.r, n, fc);
    c.r += n;
  } else {
    const int n = min(4, c.hi - c.r);
    s = span_rows(a.lm, c.r, n, 1);
    c.r += n;
  }
  return true;
}

// ---- grid barrier --------------------------------------------------------------
// All consumer threads call it.  Returns false when the kernel is aborting.
__device__ __forceinline__ bool grid_barrier(const PArgs &a, Smem &sm, uint64_t target) {
  cons_sync();
  if (threadIdx.x == 0 && !*(volatile int *)&sm.abort_local) {
    __threadfence();
    atomicAdd(a.ctr, 1ull);
    const uint64_t t0 = globaltimer_ns();
    uint32_t it = 0;
    while (ld_acquire_u64(a.ctr) < target) {
      if ((++it & 63u) == 0) {
        if (ld_volatile_i32(a.abort_flag) || globaltimer_ns() - t0 > kWaitNs) {
          atomicOr(a.err, ERR_TIMEOUT);
          atomicExch(a.abort_flag, 1);
          sm.abort_local = 1;
          break;
        }
      }
    }
    __threadfence();
  }
  cons_sync();
  return *(volatile int *)&sm.abort_local == 0;
}

__device__ __forceinline__ void cons_abort(const PArgs &a, Smem &sm) {
  atomicOr(a.err, ERR_TIMEOUT);
  atomicExch(a.abort_flag, 1);
  *(volatile int *)&sm.abort_local = 1;
}

// ---- input staging ----------------------------------------------------------------
// xs[c][j * kXS + b] = x[2048 c + 32 b + j] for the chunks c < nc of a vector.
__device__ __forceinline__ void put_x(float *xs, int i, float v) {
  const int c = i >> 11, w = i & 2047;
  xs[c * 32 * kXS + (w & 31) * kXS + (w >> 5)] = v;
}

// RMSNorm(src) * gamma (src: kE floats, written by other CTAs: read through L2)
// into xs chunk 0; tid < kCT.  sum of squares per thread (4 values), warp
// shuffles, then the warps' sums in order.
__device__ __forceinline__ void stage_norm(Smem &sm, float *xs, const float *src, const float *gamma, float eps,
                                           bool from_l2) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float ss = 0.f;
  for (int i4 = tid; i4 < kE / 4; i4 += kCT) {
    const float4 v = from_l2 ? __ldcg(reinterpret_cast<const float4 *>(src) + i4)
                             : reinterpret_cast<const float4 *>(src)[i4];
    ss = __fadd_rn(ss, __fmul_rn(v.x, v.x));
    ss = __fadd_rn(ss, __fmul_rn(v.y, v.y));
    ss = __fadd_rn(ss, __fmul_rn(v.z, v.z));
    ss = __fadd_rn(ss, __fmul_rn(v.w, v.w));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) sm.red[warp] = ss;
  cons_sync();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kCW; ++w) t = __fadd_rn(t, sm.red[w]);
  const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)kE), eps));
  for (int i4 = tid; i4 < kE / 4; i4 += kCT) {
    const float4 v = from_l2 ? __ldcg(reinterpret_cast<const float4 *>(src) + i4)
                             : reinterpret_cast<const float4 *>(src)[i4];
    const float4 g = __ldg(reinterpret_cast<const float4 *>(gamma) + i4);
    put_x(xs, 4 * i4 + 0, __fmul_rn(__fdiv_rn(v.x, rms), g.x));
    put_x(xs, 4 * i4 + 1, __fmul_rn(__fdiv_rn(v.y, rms), g.y));
    put_x(xs, 4 * i4 + 2, __fmul_rn(__fdiv_rn(v.z, rms), g.z));
    put_x(xs, 4 * i4 + 3, __fmul_rn(__fdiv_rn(v.w, rms), g.w));
  }
}

// the token's embedding row (Q8_0, exact dequantisation) into dst (kE floats)
__device__ __forceinline__ void embed_row(const uint8_t *emb, int id, float *dst) {
  const uint8_t *row = emb + (int64_t)id * kChunk;
  for (int i = threadIdx.x; i < kE; i += kCT) {
    const uint8_t *blk = row + (i >> 5) * 34;
    const uint16_t d = (uint16_t)blk[0] | ((uint16_t)blk[1] << 8);
    dst[i] = __fmul_rn((float)(int8_t)blk[2 + (i & 31)], half_bits_to_float(d));
  }
}

// ---- attention (phase B) ------------------------------------------------------------
// Item = (key/value head kvh, key chunk c): the G query heads of kvh against
// keys [c cs, min(T, (c + 1) cs)), T = pos + 1, cs = ceil(T / kNCH).  Writes
// per query head the chunk's max score, sum of exp and sum of exp * v; the
// CTA that finishes the last chunk of kvh combines the kNCH partials into the
// context rows of kvh's query heads.
__device__ void attention_item(const PArgs &a, const PLayer &ly, int item, int pos, float *scr, int &s_last) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = a.H / a.KVH, kvh = item / kNCH, c = item % kNCH;
  const int T = pos + 1, cs = (T + kNCH - 1) / kNCH;
  const int t0 = c * cs, t1 = min(T, t0 + cs), nk = max(0, t1 - t0);
  const int row = a.KVH * kD, half = kD / 2;
  float *qs = scr;                       // [kMaxG][64]
  float *kn = qs + kMaxG * kD;           // [64] rotated new key
  float *vn = kn + kD;                   // [64] new value
  float *sc = vn + kD;                   // [kMaxG][kMaxKeys] scores, then exp
  float *mx = sc + kMaxG * kMaxKeys;     // [kMaxG] max, [kMaxG] sum
  float *red = mx + 2 * kMaxG;           // [kCW][kMaxG][64] per-warp output partials
  const float *ct = a.cos_t + (int64_t)pos * half, *st = a.sin_t + (int64_t)pos * half;
  const float *kbase = ly.k_cache + kvh * kD, *vbase = ly.v_cache + kvh * kD;
  // RoPE of q (the item's G heads) and of the new key; the new value
  for (int u = tid; u < G * half + half + kD; u += kCT) {
    if (u < G * half) {
      const int h = u / half, i = u % half;
      const float *qh = a.q + (int64_t)(kvh * G + h) * kD;
      const float x0 = __ldcg(qh + i), x1 = __ldcg(qh + i + half);
      const float cc = __ldg(ct + i), ss = __ldg(st + i);
      qs[h * kD + i] = __fmaf_rn(x0, cc, -__fmul_rn(x1, ss));
      qs[h * kD + i + half] = __fmaf_rn(x0, ss, __fmul_rn(x1, cc));
    } else if (u < G * half + half) {
      const int i = u - G * half;
      const float *kh = a.k + (int64_t)kvh * kD;
      const float x0 = __ldcg(kh + i), x1 = __ldcg(kh + i + half);
      const float cc = __ldg(ct + i), ss = __ldg(st + i);
      kn[i] = __fmaf_rn(x0, cc, -__fmul_rn(x1, ss));
      kn[i + half] = __fmaf_rn(x0, ss, __fmul_rn(x1, cc));
    } else {
      const int d = u - G * half - half;
      vn[d] = __ldcg(a.v + (int64_t)kvh * kD + d);
    }
  }
  cons_sync();
  // the item holding key pos writes this token's key and value into the caches
  if (t0 <= pos && pos < t1 && tid < kD) {
    ly.k_cache[(int64_t)pos * row + kvh * kD + tid] = kn[tid];
    ly.v_cache[(int64_t)pos * row + kvh * kD + tid] = vn[tid];
  }
  // scores (q . k) * scale: four threads per key, each an fma chain over 16 of
  // the 64 dimensions, the quarters added pairwise
  for (int base = 0; base < nk; base += kCT / 4) {
    const int kk = base + (tid >> 2), qq = tid & 3;
    float acc[kMaxG];
#pragma unroll
    for (int h = 0; h < kMaxG; ++h) acc[h] = 0.f;
    if (kk < nk) {
      const int t = t0 + kk;
      float4 k4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        k4[i] = t == pos ? reinterpret_cast<const float4 *>(kn + 16 * qq)[i]
                         : __ldcg(reinterpret_cast<const float4 *>(kbase + (int64_t)t * row + 16 * qq) + i);
#pragma unroll
      for (int h = 0; h < kMaxG; ++h) {
        if (h < G) {
          const float *qh = qs + h * kD + 16 * qq;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            acc[h] = __fmaf_rn(qh[4 * i + 0], k4[i].x, acc[h]);
            acc[h] = __fmaf_rn(qh[4 * i + 1], k4[i].y, acc[h]);
            acc[h] = __fmaf_rn(qh[4 * i + 2], k4[i].z, acc[h]);
            acc[h] = __fmaf_rn(qh[4 * i + 3], k4[i].w, acc[h]);
          }
        }
      }
    }
#pragma unroll
    for (int h = 0; h < kMaxG; ++h) {
      acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 1);
      acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 2);
    }
    if (kk < nk && qq == 0)
#pragma unroll
      for (int h = 0; h < kMaxG; ++h)
        if (h < G) sc[h * kMaxKeys + kk] = __fmul_rn(acc[h], a.scale);
  }
  cons_sync();
  // per head: max, exp(s - max), sum (warp h)
  if (warp < G) {
    float m = -INFINITY;
    for (int t = lane; t < nk; t += 32) m = fmaxf(m, sc[warp * kMaxKeys + t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
    for (int t = lane; t < nk; t += 32) {
      const float e = __expf(sc[warp * kMaxKeys + t] - m);
      sc[warp * kMaxKeys + t] = e;
      s += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) {
      mx[warp] = nk > 0 ? m : -INFINITY;
      mx[kMaxG + warp] = s;
    }
  }
  cons_sync();
  // sum of exp * v: lane (half-warp sub, d quad) over keys kk = slice, slice + kSlices, ...
  {
    const int sub = lane >> 4, d4 = lane & 15, slice = 2 * warp + sub;
    float4 o[kMaxG];
#pragma unroll
    for (int h = 0; h < kMaxG; ++h) o[h] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int kk = slice; kk < nk; kk += kSlices) {
      const int t = t0 + kk;
      const float4 v4 = t == pos ? reinterpret_cast<const float4 *>(vn)[d4]
                                 : __ldcg(reinterpret_cast<const float4 *>(vbase + (int64_t)t * row) + d4);
#pragma unroll
      for (int h = 0; h < kMaxG; ++h) {
        if (h < G) {
          const float p = sc[h * kMaxKeys + kk];
          o[h].x = __fmaf_rn(p, v4.x, o[h].x);
          o[h].y = __fmaf_rn(p, v4.y, o[h].y);
          o[h].z = __fmaf_rn(p, v4.z, o[h].z);
          o[h].w = __fmaf_rn(p, v4.w, o[h].w);
        }
      }
    }
#pragma unroll
    for (int h = 0; h < kMaxG; ++h) {
      o[h].x += __shfl_xor_sync(0xffffffffu, o[h].x, 16);
      o[h].y += __shfl_xor_sync(0xffffffffu, o[h].y, 16);
      o[h].z += __shfl_xor_sync(0xffffffffu, o[h].z, 16);
      o[h].w += __shfl_xor_sync(0xffffffffu, o[h].w, 16);
      if (sub == 0 && h < G) reinterpret_cast<float4 *>(red + (warp * kMaxG + h) * kD)[d4] = o[h];
    }
  }
  cons_sync();
  for (int u = tid; u < G * kD; u += kCT) {
    const int h = u / kD, d = u % kD;
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kCW; ++w) acc = __fadd_rn(acc, red[(w * kMaxG + h) * kD + d]);
    float *p = a.part + ((int64_t)(kvh * G + h) * kNCH + c) * kPart;
    p[4 + d] = acc;
    if (d == 0) {
      p[0] = mx[h];
      p[1] = mx[kMaxG + h];
    }
  }
  // the last chunk of kvh to finish combines: ctx[h * 64 + d] =
  // sum_c w_c o_c[d] / sum_c w_c s_c, w_c = exp(m_c - max_c m_c)
  __threadfence();
  cons_sync();
  if (tid == 0) s_last = atomicAdd(a.head_done + kvh, 1) == kNCH - 1;
  cons_sync();
  if (s_last) {
    __threadfence();
    for (int u = tid; u < G * kD; u += kCT) {
      const int h = u / kD, d = u % kD;
      const float *p = a.part + (int64_t)(kvh * G + h) * kNCH * kPart;
      float m = -INFINITY;
#pragma unroll
      for (int cc = 0; cc < kNCH; ++cc) m = fmaxf(m, __ldcg(p + cc * kPart));
      float sden = 0.f, onum = 0.f;
#pragma unroll
      for (int cc = 0; cc < kNCH; ++cc) {
        const float mc = __ldcg(p + cc * kPart);
        const float w = mc == -INFINITY ? 0.f : __expf(mc - m);
        sden = __fmaf_rn(w, __ldcg(p + cc * kPart + 1), sden);
        onum = __fmaf_rn(w, __ldcg(p + cc * kPart + 4 + d), onum);
      }
      a.ctx[(int64_t)(kvh * G + h) * kD + d] = __fdiv_rn(onum, sden);
    }
    if (tid == 0) a.head_done[kvh] = 0;  // for the next layer (after grid barriers)
  }
}

// the context vector (written in phase B) into xs chunk 0
__device__ __forceinline__ void stage_ctx(const PArgs &a, float *xs) {
  for (int i4 = threadIdx.x; i4 < kE / 4; i4 += kCT) {
    const float4 v = __ldcg(reinterpret_cast<const float4 *>(a.ctx) + i4);
    put_x(xs, 4 * i4 + 0, v.x);
    put_x(xs, 4 * i4 + 1, v.y);
    put_x(xs, 4 * i4 + 2, v.z);
    put_x(xs, 4 * i4 + 3, v.w);
  }
}

// ---- the kernel ------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1) decode_persist_kernel(const PArgs a) {
  extern __shared__ __align__(128) uint8_t dsm[];
  Smem &sm = *reinterpret_cast<Smem *>(dsm);
  uint8_t *ring = dsm + ((sizeof(Smem) + 127) & ~size_t(127));
  float *xs = reinterpret_cast<float *>(ring + (size_t)kSlots * kSpan);  // [kMaxFC][32][kXS]
  const int G = gridDim.x, b = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nbar = 5 * a.L;  // grid barriers per step

  const int pos = *a.pos;
  const int token = *a.token;
  if (pos < 0 || pos >= a.max_seq || pos >= a.rope_max_seq || token < 0 || token >= a.V) {
    if (b == 0 && tid == 0) atomicOr(a.err, ERR_INDEX);
    return;  // every CTA takes this branch: no barrier is entered
  }
  if (tid == 0) {
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 4);
    }
    sm.abort_local = 0;
    fence_mbar_init();
  }
  exp_cr_table_init(sm.tab);
  __syncthreads();

  if (warp == kCW) {
    // ---------------- producer ----------------
    if (lane != 0) return;
    int i = 0;
    bool ok = true;
    Cursor cur;
    cur_init(cur, a, G, b);
    SpanInfo sp;
    int ph;
    while (ok && cur_next(cur, a, G, b, sp, ph)) {
      const int slot = i % kSlots;
      if (i >= kSlots) {
        const uint32_t par = (uint32_t)(((i / kSlots) - 1) & 1);
        if (!mbar_try_wait(&sm.empty[slot], par)) {
          const uint64_t t0 = globaltimer_ns();
          uint32_t it = 0;
          while (!mbar_try_wait(&sm.empty[slot], par)) {
            if ((++it & 63u) == 0 &&
                (*(volatile int *)&sm.abort_local || globaltimer_ns() - t0 > kWaitNs)) {
              ok = false;
              break;
            }
          }
          if (!ok) break;
        }
        fence_proxy_async_smem();  // the consumers' reads of the slot before the copy overwrites it
      }
      uint8_t *dst = ring + (size_t)slot * kSpan;
      sm.meta[slot] = make_int4(ph, sp.row0, sp.rows, sp.cpr);  // published by the barrier's completion
      mbar_arrive_expect_tx(&sm.full[slot], sp.bytes0 + sp.bytes1);
      bulk_g2s(dst, sp.src0, sp.bytes0, &sm.full[slot]);
      if (sp.bytes1) bulk_g2s(dst + sp.bytes0, sp.src1, sp.bytes1, &sm.full[slot]);
      ++i;
    }
    if (!ok) {
      // drain: every span issued may still be landing in this CTA's ring
      for (int j = max(0, i - kSlots); j < i; ++j) mbar_wait_bounded(&sm.full[j % kSlots], (uint32_t)((j / kSlots) & 1), nullptr);
    }
    return;
  }

  // ---------------- consumers ----------------
  uint64_t ctr0 = 0;
  if (tid == 0) {
    const unsigned long long per = (unsigned long long)G * (unsigned long long)nbar;
    ctr0 = (ld_acquire_u64(a.ctr) / per) * per;
  }
  // every consumer needs the barrier base: broadcast through shared memory
  __shared__ unsigned long long s_ctr0;
  __shared__ int s_last;
  if (tid == 0) s_ctr0 = ctr0;
  cons_sync();
  ctr0 = s_ctr0;
  int nb_done = 0;
  auto barrier = [&]() -> bool {
    ++nb_done;
    return grid_barrier(a, sm, ctr0 + (uint64_t)nb_done * (uint64_t)G);
  };

  const int grp = warp >> 2, wj = warp & 3;
  const int kv = a.KVH * kD, fc = a.F / kE;
  int span_i = 0;       // spans walked so far (all groups)
  int grp_spans = 0;    // spans this warp's group consumed (partial-sum buffer parity)
  float2 xp[32];
  int lo = 0, hi = 0;
  // spans per phase of this CTA (the producer's walk, counted): Q/K/V, O,
  // gate + up, down, LM head
  int nsp[5];
  {
    int l0, h0;
    share(kE + 2 * kv, G, b, l0, h0);
    nsp[0] = (h0 - l0 + 3) / 4;
    share(kE, G, b, l0, h0);
    nsp[1] = (h0 - l0 + 3) / 4;
    share(a.F, G, b, l0, h0);
    nsp[2] = 2 * ((h0 - l0 + 3) / 4);
    share(kE, G, b, l0, h0);
    const int rps = kSpanChunks / fc;
    nsp[3] = (h0 - l0 + rps - 1) / rps;
    share(a.V, G, b, l0, h0);
    nsp[4] = (h0 - l0 + 3) / 4;
  }

  // Consumes the next `count` spans (one phase): the warp waits for each span
  // of its group, reads the span's rows from the producer's table, computes
  // its chunk's dot product, releases the slot and hands finished rows to
  // out(phase, row, value).  After an abort (a wait that gave up, here or in
  // another CTA) the warp still goes through the spans and meets every group
  // barrier, without waiting or computing, so that all consumer warps reach
  // the same named barriers.
  auto consume = [&](int count, bool multi_chunk, auto &&out) {
    for (int k = 0; k < count; ++k) {
      const int my = span_i++;
      if (my % kNG != grp) continue;
      const int slot = my % kSlots;
      bool live = *(volatile int *)&sm.abort_local == 0;
      if (live && !mbar_wait_bounded(&sm.full[slot], (uint32_t)((my / kSlots) & 1), a.err)) {
        if (lane == 0) cons_abort(a, sm);
        live = false;
      }
      live = __all_sync(0xffffffffu, live);
      int4 mt = make_int4(0, 0, 0, 1);
      if (live) mt = sm.meta[slot];
      const int ph = mt.x, row0 = mt.y, rows = mt.z, cpr = mt.w;
      const int nchunks = rows * cpr;
      float v = 0.f;
      if (live && wj < nchunks) {
        const uint8_t *w = ring + (size_t)slot * kSpan + (size_t)wj * kChunk;
        v = q8_row_dot_pairs(w, kNB, xp, nullptr, kXS, lane);
      }
      __syncwarp();
      if (live && lane == 0) mbar_arrive_cnt(&sm.empty[slot]);
      if (!multi_chunk) {
        if (live && wj < rows && lane == 0) out(ph, row0 + wj, v);
      } else {
        // rows of several chunks: chunk partials summed in chunk order
        const int p = grp_spans & 1;
        if (lane == 0) sm.gsum[grp][p][wj] = v;
        group_sync(grp);
        if (live && lane == 0 && wj % cpr == 0 && wj < nchunks) {
          float t = 0.f;
          for (int q = 0; q < cpr; ++q) t = __fadd_rn(t, sm.gsum[grp][p][wj + q]);
          out(ph, row0 + wj / cpr, t);
        }
      }
      ++grp_spans;
    }
  };

  // layer 0 input: the token's embedding; CTA 0 also stores it as h
  float *emb_s = xs + (kMaxFC - 1) * 32 * kXS;  // scratch in the last x chunk (free in phase A)
  embed_row(a.emb, token, emb_s);
  cons_sync();
  if (b == 0)
    for (int i = tid; i < kE; i += kCT) a.hA[i] = emb_s[i];

  for (int l = 0; l < a.L; ++l) {
    const PLayer ly = a.layers[l];
    // ---- A: Q/K/V ----
    stage_norm(sm, xs, l == 0 ? emb_s : a.hA, ly.attn_norm, a.eps_attn, l != 0);
    cons_sync();
    q8_pair_x(xp, xs, kXS, 2 * lane, true);
    consume(nsp[0], false, [&](int, int r, float v) {
      float *dst = r < kE ? a.q + r : (r < kE + kv ? a.k + (r - kE) : a.v + (r - kE - kv));
      *dst = v;
    });
    if (!barrier()) return;
    // ---- B: attention items ----
    for (int item = b; item < a.KVH * kNCH; item += G) {
      attention_item(a, ly, item, pos, xs, s_last);
      cons_sync();
    }
    if (!barrier()) return;
    // ---- C: O projection + residual ----
    stage_ctx(a, xs);
    cons_sync();
    q8_pair_x(xp, xs, kXS, 2 * lane, true);
    consume(nsp[1], false, [&](int, int r, float v) { a.hB[r] = __fadd_rn(__ldcg(a.hA + r), v); });
    if (!barrier()) return;
    // ---- D: gate/up + SwiGLU ----
    stage_norm(sm, xs, a.hB, ly.ffn_norm, a.eps_ffn, true);
    cons_sync();
    q8_pair_x(xp, xs, kXS, 2 * lane, true);
    share(a.F, G, b, lo, hi);
    consume(nsp[2], false, [&](int ph, int r, float v) {
      if (ph == 3) sm.gate[r - lo] = v;
      else sm.up[r - lo] = v;
    });
    cons_sync();
    for (int r = lo + tid; r < hi; r += kCT) a.act[r] = swiglu_f32(sm.gate[r - lo], sm.up[r - lo], sm.tab);
    if (!barrier()) return;
    // ---- E: down projection + residual ----
    for (int i = tid; i < a.F / 4; i += kCT) {
      const float4 v4 = __ldcg(reinterpret_cast<const float4 *>(a.act) + i);
      put_x(xs, 4 * i + 0, v4.x);
      put_x(xs, 4 * i + 1, v4.y);
      put_x(xs, 4 * i + 2, v4.z);
      put_x(xs, 4 * i + 3, v4.w);
    }
    cons_sync();
    q8_pair_x(xp, xs + (wj % fc) * 32 * kXS, kXS, 2 * lane, true);
    consume(nsp[3], fc > 1, [&](int, int r, float v) { a.hA[r] = __fadd_rn(__ldcg(a.hB + r), v); });
    if (!barrier()) return;
  }
  // ---- final norm + LM head ----
  stage_norm(sm, xs, a.hA, a.final_norm, a.eps_final, true);
  cons_sync();
  q8_pair_x(xp, xs, kXS, 2 * lane, true);
  consume(nsp[4], false, [&](int, int r, float v) { a.logits[r] = v; });
}

size_t persist_smem() {
  return ((sizeof(Smem) + 127) & ~size_t(127)) + (size_t)kSlots * kSpan + (size_t)kMaxFC * 32 * kXS * 4;
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" {

tb_status tb_decode_workspace_bytes(const tb_decode_model *m, size_t *bytes) {
  if (!m || !bytes) return fail(TB_EINVAL, "tb_decode_workspace_bytes: null pointer");
  const size_t f = sizeof(float);
  size_t n = 256;  // barrier counter, abort flag, per key/value head chunk counters
  n += 3 * kE * f;                                                  // hA, hB, ctx
  n += (size_t)(kE + 2 * m->kv_heads * kD) * f;                     // q, k, v
  n += (size_t)m->heads * kNCH * kPart * f;                          // attention partials
  n += (size_t)m->ffn * f;                                          // act
  *bytes = (n + 255) & ~size_t(255);
  return TB_OK;
}

tb_status tb_decode_step_persistent(const tb_decode_model *m, tb_stream stream) {
  if (!m) return fail(TB_EINVAL, "tb_decode_step_persistent: null model");
  if (m->hidden != kE || m->head_dim != kD || m->heads * kD != kE || m->kv_heads <= 0 || m->heads % m->kv_heads != 0 ||
      m->heads / m->kv_heads > kMaxG || m->kv_heads > 56)
    return fail(TB_EINVAL, "tb_decode_step_persistent: needs hidden %d, head_dim %d, heads * head_dim = hidden, "
                           "<= %d query heads per key/value head, <= 56 key/value heads", kE, kD, kMaxG);
  if (m->ffn <= 0 || m->ffn % kE != 0 || !(m->ffn / kE == 1 || m->ffn / kE == 2 || m->ffn / kE == 4))
    return fail(TB_EINVAL, "tb_decode_step_persistent: ffn must be 2048, 4096 or 8192");
  if (m->n_layers <= 0 || m->vocab <= 0 || m->vocab > 0x7FFFFFFF || m->max_seq <= 0 || m->max_seq > kMaxSeq ||
      m->rope_max_seq <= 0)
    return fail(TB_EINVAL, "tb_decode_step_persistent: bad layer count, vocab or sequence length (max %d)", kMaxSeq);
  if (!m->layers_dev || !m->tok_emb || !m->lm_head || !m->final_norm || !m->rope_cos || !m->rope_sin ||
      !m->token_dev || !m->pos_dev || !m->logits || !m->workspace)
    return fail(TB_EINVAL, "tb_decode_step_persistent: null pointer");
  if ((reinterpret_cast<uintptr_t>(m->lm_head) & 15) || (reinterpret_cast<uintptr_t>(m->workspace) & 255))
    return fail(TB_EINVAL, "tb_decode_step_persistent: lm_head must be 16-byte and workspace 256-byte aligned");
  size_t need = 0;
  TB_TRY(tb_decode_workspace_bytes(m, &need));
  if (m->workspace_bytes < need)
    return fail(TB_EINVAL, "tb_decode_step_persistent: workspace of %zu bytes, %zu needed", m->workspace_bytes, need);
  DeviceState *st;
  TB_TRY(device_state(&st));
  if ((m->ffn + st->sm_count - 1) / st->sm_count > 64)
    return fail(TB_EINVAL, "tb_decode_step_persistent: more than 64 gate/up rows per SM");
  const size_t smem = persist_smem();
  if (smem > (size_t)st->smem_optin)
    return fail(TB_EINVAL, "tb_decode_step_persistent: %zu bytes of shared memory per CTA exceed the device's", smem);
  TB_TRY(ensure_smem_for(decode_persist_kernel, smem));
  static int blocks_per_sm[64] = {0};
  const int dev = st->device;
  if (blocks_per_sm[dev] == 0) {
    int n = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_persist_kernel, kThreads, smem);
    if (e != cudaSuccess) return fail(TB_ECUDA, "tb_decode_step_persistent: %s", cudaGetErrorString(e));
    if (n < 1) return fail(TB_EINVAL, "tb_decode_step_persistent: the kernel does not fit on an SM");
    blocks_per_sm[dev] = n;
  }
  PArgs a = {};
  a.layers = m->layers_dev;
  a.L = m->n_layers;
  a.F = (int)m->ffn;
  a.H = (int)m->heads;
  a.KVH = (int)m->kv_heads;
  a.V = (int)m->vocab;
  a.max_seq = (int)m->max_seq;
  a.rope_max_seq = (int)m->rope_max_seq;
  a.eps_attn = m->eps_attn;
  a.eps_ffn = m->eps_ffn;
  a.eps_final = m->eps_final;
  a.scale = m->attn_scale;
  a.emb = static_cast<const uint8_t *>(m->tok_emb);
  a.lm = static_cast<const uint8_t *>(m->lm_head);
  a.final_norm = m->final_norm;
  a.cos_t = m->rope_cos;
  a.sin_t = m->rope_sin;
  a.token = m->token_dev;
  a.pos = m->pos_dev;
  a.logits = m->logits;
  uint8_t *w = static_cast<uint8_t *>(m->workspace);
  a.ctr = reinterpret_cast<unsigned long long *>(w);
  a.abort_flag = reinterpret_cast<int *>(w + 8);
  a.head_done = reinterpret_cast<int *>(w + 16);
  float *f = reinterpret_cast<float *>(w + 256);
  a.hA = f;
  f += kE;
  a.hB = f;
  f += kE;
  a.q = f;
  f += kE;
  a.k = f;
  f += m->kv_heads * kD;
  a.v = f;
  f += m->kv_heads * kD;
  a.part = f;
  f += m->heads * kNCH * kPart;
  a.ctx = f;
  f += kE;
  a.act = f;
  a.err = st->err_word;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)st->sm_count, 1, 1);  // one CTA per SM, all resident (cooperative)
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, decode_persist_kernel, a);
  if (e != cudaSuccess) return fail(TB_ECUDA, "tb_decode_step_persistent: %s", cudaGetErrorString(e));
  return TB_OK;
}

}  // extern "C"
