// tb_decode.cu -- the pieces of a one-token decode step whose arguments depend
// on the position, with the position held in device memory so that one step
// can be captured once in a CUDA graph and replayed for every token:
//   tb_kv_append         cache rows [pos] <- this token's K and V
//                        (attention.cpp:66-84 with S = 1: Kc.slice(pos).copy_(K))
//   tb_attention_decode  all query heads of one token against the cache
//                        (attention.cpp:104-141 with S = 1, fused per head)
//   tb_rope_attention_decode  the same with RoPE of q and k and the cache
//                        append of k and v fused in (one launch for
//                        attention.cpp:50-141 at S = 1)
//   tb_decode_margin     top-1 minus top-2 logit (a diagnostic for callers)
//   tb_decode_advance    next token id, history, pos += 1
// plus stream and graph handles for callers without the CUDA runtime.
// Every kernel checks pos against the cache length: a position outside it
// sets bit 1 of the device error word and writes nothing.
#include <cooperative_groups.h>

#include <algorithm>

#include "tb_internal.cuh"

namespace cg = cooperative_groups;

namespace tb {
namespace {

__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void kv_append_kernel(float *__restrict__ kc, float *__restrict__ vc, const float *__restrict__ k,
                                 const float *__restrict__ v, int row, int max_seq,
                                 const int32_t *__restrict__ pos_dev, uint32_t *__restrict__ err) {
  const int pos = *pos_dev;
  if (pos < 0 || pos >= max_seq) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(err, ERR_INDEX);
    return;
  }
  const int64_t base = (int64_t)pos * row;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < row; i += gridDim.x * blockDim.x) {
    kc[base + i] = k[i];
    vc[base + i] = v[i];
  }
}

// One thread-block cluster of NC CTAs per query head h (key/value head
// h / (H / KVH)); ctx = pos + 1 keys, CTA r of the cluster owns keys
// [r * chunk, (r + 1) * chunk):
//   score[c] = (fma chain over d of q[d] * K[c][d]) * scale   -- the fp32
//              matmul's order (tb_matmul_f32), then Tensor::operator*(float)
//   per CTA: m_r = max of its scores, e[c] = exp(score[c] - m_r),
//              s_r = sum of e, o_r[d] = sum over its keys of e[c] * V[c][d]
//              (four consecutive key ranges, each an fma chain, added in order)
//   out[d]   = (sum over r of o_r[d] exp(m_r - M)) * (1 / S), with M = max m_r
//              and S = sum over r of s_r exp(m_r - M), both in rank order,
//              combined by rank 0 after every CTA has stored its (m_r, s_r, o_r)
//              into rank 0's shared memory (distributed shared memory)
// That is softmax(score) . V with the normalisation applied once per output
// instead of once per key (within 1e-5 of sum p |v| of the exact result).
// Latency is what bounds one token's attention, so the kernel makes one pass:
// as soon as the position is known every thread loads the key row it scores
// (16 float4s) and the first kVPre values it multiplies, before q is staged,
// and the cluster meets once to combine.
// fma chain over d of q[d] * k[d], k held in registers
template <int D>
__device__ __forceinline__ float qk_dot_reg(const float *qs, const float4 (&kv)[D / 4]) {
  float acc = 0.f;
#pragma unroll
  for (int d4 = 0; d4 < D / 4; ++d4) {
    acc = __fmaf_rn(qs[4 * d4 + 0], kv[d4].x, acc);
    acc = __fmaf_rn(qs[4 * d4 + 1], kv[d4].y, acc);
    acc = __fmaf_rn(qs[4 * d4 + 2], kv[d4].z, acc);
    acc = __fmaf_rn(qs[4 * d4 + 3], kv[d4].w, acc);
  }
  return acc;
}

struct AttnArgs {
  const float *q;      // [H, D]
  const float *kc;     // key cache [max_seq, KVH, D]
  const float *vc;     // value cache
  float *kc_w, *vc_w;  // ROPE: the caches again, for the append
  const float *k_new;  // ROPE: this token's keys [KVH, D] before RoPE
  const float *v_new;  // ROPE: this token's values [KVH, D]
  const float *cos_t, *sin_t;  // ROPE: [rope_max_seq, D / 2]
  int rope_max_seq;
  int H, KVH, max_seq;
  float scale;
  const int32_t *pos_dev;
  float *out;  // [H, D]
};

constexpr int kVPre = 8;  // values per thread loaded ahead of the scores

// ROPE: RoPE of q and of the new key at pos (tb_rope_at's arithmetic) and the
// cache append of this token's key and value, fused in: each cluster rotates
// its query head and its key/value head's new key itself, uses the new key and
// value from shared memory for position pos, and the first cluster of each
// key/value group (rank 0) writes them into the caches.  No cluster reads the
// cache row pos, so the writes race with nothing.
template <int D, int NC, bool ROPE>
__global__ void __launch_bounds__(256) attention_decode_kernel(const AttnArgs a, uint32_t *__restrict__ err) {
  extern __shared__ float sc[];  // this CTA's scores, then exp(score - m_r); ceil(max_seq / NC) floats
  __shared__ float qs[D];
  __shared__ __align__(16) float kn[ROPE ? D : 4];
  __shared__ float vn[ROPE ? D : 1];  // the new key (rotated) and value
  __shared__ float red[8];
  __shared__ float pv[256 / D][D];    // partial outputs of the four key ranges
  __shared__ float gpart[NC][2];      // rank 0: every CTA's [m_r, s_r], written by that CTA
  __shared__ float gocta[NC][D];      // rank 0: every CTA's o_r, written by that CTA
  cg::cluster_group cluster = cg::this_cluster();
  const int cr = (int)cluster.block_rank();
  const int H = a.H, KVH = a.KVH;
  const int h = blockIdx.x / NC;
  const int kvh = h / (H / KVH);
  pdl_launch_dependents();
  const int pos = *a.pos_dev;
  if (pos < 0 || pos >= a.max_seq || (ROPE && pos >= a.rope_max_seq)) {  // the cluster leaves together
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(err, ERR_INDEX);
    return;
  }
  const int ctx = pos + 1;
  const int chunk = (ctx + NC - 1) / NC;
  const int c0 = min(ctx, cr * chunk), c1 = min(ctx, c0 + chunk);
  const int rs = KVH * D;  // cache row stride (floats)
  const int t = threadIdx.x;
  // loads that depend only on pos: this thread's first key row and its first
  // kVPre values (the key and value of row pos come from shared memory with ROPE)
  const int ck = c0 + t;
  const bool own_k = ck < c1 && !(ROPE && ck == pos);
  float4 kreg[D / 4];
  if (own_k) {
    const float4 *kr = reinterpret_cast<const float4 *>(a.kc + (int64_t)ck * rs + kvh * D);
#pragma unroll
    for (int d4 = 0; d4 < D / 4; ++d4) kreg[d4] = __ldg(kr + d4);
  }
  constexpr int NCH = 256 / D;
  const int d = t % D, ch = t / D;
  const int n = c1 - c0, len = (n + NCH - 1) / NCH;
  const int a0 = c0 + ch * len, a1 = min(c1, a0 + len);
  const float *vcol = a.vc + kvh * D + d;
  float vreg[kVPre];
#pragma unroll
  for (int j = 0; j < kVPre; ++j) {
    const int c = a0 + j;
    vreg[j] = (c < a1 && !(ROPE && c == pos)) ? __ldg(vcol + (int64_t)c * rs) : 0.f;
  }
  if (ROPE) {
    constexpr int half = D / 2;
    if (t < 2 * half) {
      const bool isq = t < half;
      const int i = isq ? t : t - half;
      const float *src = isq ? a.q + h * D : a.k_new + kvh * D;
      float *dst = isq ? qs : kn;
      const float c = __ldg(a.cos_t + (int64_t)pos * half + i), s = __ldg(a.sin_t + (int64_t)pos * half + i);
      const float x0 = src[i], x1 = src[i + half];
      dst[i] = __fmaf_rn(x0, c, -__fmul_rn(x1, s));
      dst[i + half] = __fmaf_rn(x0, s, __fmul_rn(x1, c));
    } else if (t < 2 * half + D) {
      vn[t - 2 * half] = a.v_new[kvh * D + t - 2 * half];
    }
    __syncthreads();
    if (h % (H / KVH) == 0 && cr == 0 && t < D) {
      a.kc_w[(int64_t)pos * rs + kvh * D + t] = kn[t];
      a.vc_w[(int64_t)pos * rs + kvh * D + t] = vn[t];
    }
  } else {
    if (t < D) qs[t] = a.q[h * D + t];
    __syncthreads();
  }
  const int warp = t >> 5, lane = t & 31;

  // scores and this CTA's maximum
  float m = -INFINITY;
  for (int c = ck; c < c1; c += 256) {
    if (c != ck || !own_k) {  // a later key row (more than 256 keys per CTA), or the new key
      const float4 *kr = (ROPE && c == pos) ? reinterpret_cast<const float4 *>(kn)
                                            : reinterpret_cast<const float4 *>(a.kc + (int64_t)c * rs + kvh * D);
#pragma unroll
      for (int d4 = 0; d4 < D / 4; ++d4) kreg[d4] = (ROPE && c == pos) ? kr[d4] : __ldg(kr + d4);
    }
    const float sv = __fmul_rn(qk_dot_reg<D>(qs, kreg), a.scale);
    sc[c - c0] = sv;
    m = sv > m ? sv : m;
  }
  m = warp_max_f(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = red[0];
  for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
  // exp(score - m_r) and their sum
  float s = 0.f;
  for (int c = ck; c < c1; c += 256) {
    const float e = __expf(__fsub_rn(sc[c - c0], m));
    sc[c - c0] = e;
    s = __fadd_rn(s, e);
  }
  s = warp_sum_f(s);
  __syncthreads();  // red[] reads above are done; sc[] is complete
  if (lane == 0) red[warp] = s;
  // o_r: four consecutive key ranges, each an fma chain over its keys
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < kVPre; ++j) {
    const int c = a0 + j;
    if (c < a1) acc = __fmaf_rn(sc[c - c0], (ROPE && c == pos) ? vn[d] : vreg[j], acc);
  }
  for (int c = a0 + kVPre; c < a1; ++c) {
    const float v = (ROPE && c == pos) ? vn[d] : __ldg(vcol + (int64_t)c * rs);
    acc = __fmaf_rn(sc[c - c0], v, acc);
  }
  pv[ch][d] = acc;
  __syncthreads();
  // Every CTA stores its (m_r, s_r) and o_r into rank 0's shared memory; after
  // the cluster barrier rank 0 combines them from its own memory, and no CTA
  // reads another's, so the others may exit at once (one cluster barrier).
  if (t < D) {
    float o = pv[0][t];
    for (int k = 1; k < NCH; ++k) o = __fadd_rn(o, pv[k][t]);
    *cluster.map_shared_rank(&gocta[cr][t], 0) = o;
  }
  if (t == 0) {
    float tot = 0.f;
    for (int w = 0; w < 8; ++w) tot = __fadd_rn(tot, red[w]);
    *cluster.map_shared_rank(&gpart[cr][0], 0) = m;
    *cluster.map_shared_rank(&gpart[cr][1], 0) = tot;
  }
  cluster.sync();
  if (cr == 0 && t < D) {
    float M = -INFINITY;
    for (int r = 0; r < NC; ++r) M = fmaxf(M, gpart[r][0]);
    float S = 0.f, o = 0.f;
    for (int r = 0; r < NC; ++r) {
      const float mr = gpart[r][0];
      if (mr == -INFINITY) continue;  // a CTA without keys
      const float w = __expf(__fsub_rn(mr, M));
      S = __fadd_rn(S, __fmul_rn(gpart[r][1], w));
      o = __fmaf_rn(gocta[r][t], w, o);
    }
    a.out[h * D + t] = __fmul_rn(o, __frcp_rn(S));
  }
}

template <bool ROPE>
tb_status launch_attention(const AttnArgs &a, const char *who, cudaStream_t s) {
  constexpr int NC = 8;  // CTAs per head (a portable cluster)
  const size_t smem = (size_t)((a.max_seq + NC - 1) / NC) * sizeof(float);
  if (smem > 200 * 1024) return fail(TB_EINVAL, "%s: cache of %d rows too long", who, a.max_seq);
  DeviceState *st;
  TB_TRY(device_state(&st));
  auto kern = attention_decode_kernel<64, NC, ROPE>;
  TB_TRY(ensure_smem_for(kern, smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.H * NC), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  // No programmatic serialization for this launch: the clusters would then be
  // launched while the preceding GEMV's CTAs still hold the SMs, and waiting
  // for eight co-resident CTAs per GPC cost more than it saved (measured on
  // the 1B decode: 1282 against 1377 tokens/s).  The kernel still lets the
  // next kernel launch early (griddepcontrol.launch_dependents).
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = NC;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a, st->err_word);
  if (e != cudaSuccess) return fail(TB_ECUDA, "%s: %s", who, cudaGetErrorString(e));
  return check_launch(who);
}

// margins[pos] = logits[idx] - (largest other logit; NaN never counts)
__global__ void __launch_bounds__(1024) margin_kernel(const float *__restrict__ logits, int64_t V,
                                                      const int64_t *__restrict__ idx,
                                                      const int32_t *__restrict__ pos_dev, int max_seq,
                                                      float *__restrict__ margins) {
  __shared__ float red[32];
  const int64_t id = *idx;
  float t = -INFINITY;
  for (int64_t i = threadIdx.x; i < V; i += blockDim.x)
    if (i != id) t = fmaxf(t, logits[i]);
  t = warp_max_f(t);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = t;
  __syncthreads();
  if (threadIdx.x == 0) {
    float top2 = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) top2 = fmaxf(top2, red[w]);
    const int pos = *pos_dev;
    if (pos >= 0 && pos < max_seq) margins[pos] = logits[id] - top2;
  }
}

__global__ void advance_kernel(const int64_t *__restrict__ idx, int32_t *__restrict__ ids,
                               int32_t *__restrict__ pos_dev, int32_t *__restrict__ history, int max_seq) {
  const int pos = *pos_dev;
  const int tok = (int)*idx;
  ids[0] = tok;
  if (pos >= 0 && pos < max_seq) history[pos] = tok;
  *pos_dev = pos + 1;
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" {

tb_status tb_kv_append(float *k_cache, float *v_cache, const float *k, const float *v, int64_t row_elems,
                       int64_t max_seq, const int32_t *pos_dev, tb_stream stream) {
  if (row_elems <= 0 || max_seq <= 0 || row_elems > 0x7FFFFFFF || max_seq > 0x7FFFFFFF)
    return fail(TB_EINVAL, "tb_kv_append: bad extents");
  if (!k_cache || !v_cache || !k || !v || !pos_dev) return fail(TB_EINVAL, "tb_kv_append: null pointer");
  DeviceState *st;
  TB_TRY(device_state(&st));
  const int grid = (int)std::min<int64_t>((row_elems + 255) / 256, 64);
  kv_append_kernel<<<grid, 256, 0, as_stream(stream)>>>(k_cache, v_cache, k, v, (int)row_elems, (int)max_seq,
                                                         pos_dev, st->err_word);
  return check_launch("tb_kv_append");
}

tb_status tb_attention_decode(const float *q, const float *k_cache, const float *v_cache, int64_t heads,
                              int64_t kv_heads, int64_t head_dim, int64_t max_seq, float scale,
                              const int32_t *pos_dev, float *out, tb_stream stream) {
  if (heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0 || max_seq <= 0)
    return fail(TB_EINVAL, "tb_attention_decode: heads must be a positive multiple of kv_heads");
  if (head_dim != 64) return fail(TB_EINVAL, "tb_attention_decode: head_dim %lld (64 supported)", (long long)head_dim);
  if (!q || !k_cache || !v_cache || !pos_dev || !out) return fail(TB_EINVAL, "tb_attention_decode: null pointer");
  if ((reinterpret_cast<uintptr_t>(k_cache) & 15) != 0)
    return fail(TB_EINVAL, "tb_attention_decode: the key cache must be 16-byte aligned");
  if (max_seq > 0x7FFFFFFF || heads > 4096) return fail(TB_EINVAL, "tb_attention_decode: extents too large");
  AttnArgs a = {};
  a.q = q;
  a.kc = k_cache;
  a.vc = v_cache;
  a.H = (int)heads;
  a.KVH = (int)kv_heads;
  a.max_seq = (int)max_seq;
  a.scale = scale;
  a.pos_dev = pos_dev;
  a.out = out;
  return launch_attention<false>(a, "tb_attention_decode", as_stream(stream));
}

tb_status tb_rope_attention_decode(const float *q, const float *k, const float *v, int64_t heads, int64_t kv_heads,
                                   int64_t head_dim, const float *cos_dev, const float *sin_dev,
                                   int64_t rope_max_seq, float *k_cache, float *v_cache, int64_t max_seq,
                                   float scale, const int32_t *pos_dev, float *out, tb_stream stream) {
  if (heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0 || max_seq <= 0 || rope_max_seq <= 0)
    return fail(TB_EINVAL, "tb_rope_attention_decode: heads must be a positive multiple of kv_heads");
  if (head_dim != 64)
    return fail(TB_EINVAL, "tb_rope_attention_decode: head_dim %lld (64 supported)", (long long)head_dim);
  if (!q || !k || !v || !cos_dev || !sin_dev || !k_cache || !v_cache || !pos_dev || !out)
    return fail(TB_EINVAL, "tb_rope_attention_decode: null pointer");
  if ((reinterpret_cast<uintptr_t>(k_cache) & 15) != 0)
    return fail(TB_EINVAL, "tb_rope_attention_decode: the key cache must be 16-byte aligned");
  if (max_seq > 0x7FFFFFFF || rope_max_seq > 0x7FFFFFFF || heads > 4096)
    return fail(TB_EINVAL, "tb_rope_attention_decode: extents too large");
  AttnArgs a = {};
  a.q = q;
  a.kc = k_cache;
  a.vc = v_cache;
  a.kc_w = k_cache;
  a.vc_w = v_cache;
  a.k_new = k;
  a.v_new = v;
  a.cos_t = cos_dev;
  a.sin_t = sin_dev;
  a.rope_max_seq = (int)rope_max_seq;
  a.H = (int)heads;
  a.KVH = (int)kv_heads;
  a.max_seq = (int)max_seq;
  a.scale = scale;
  a.pos_dev = pos_dev;
  a.out = out;
  return launch_attention<true>(a, "tb_rope_attention_decode", as_stream(stream));
}

tb_status tb_decode_margin(const float *logits, int64_t vocab, const int64_t *idx_dev, const int32_t *pos_dev,
                           int64_t max_seq, float *margins_dev, tb_stream stream) {
  if (vocab <= 0 || max_seq <= 0) return fail(TB_EINVAL, "tb_decode_margin: bad extents");
  if (!logits || !idx_dev || !pos_dev || !margins_dev) return fail(TB_EINVAL, "tb_decode_margin: null pointer");
  margin_kernel<<<1, 1024, 0, as_stream(stream)>>>(logits, vocab, idx_dev, pos_dev, (int)max_seq, margins_dev);
  return check_launch("tb_decode_margin");
}

tb_status tb_decode_advance(const int64_t *idx_dev, int32_t *ids_dev, int32_t *pos_dev, int32_t *history_dev,
                            int64_t max_seq, tb_stream stream) {
  if (max_seq <= 0) return fail(TB_EINVAL, "tb_decode_advance: bad extents");
  if (!idx_dev || !ids_dev || !pos_dev || !history_dev) return fail(TB_EINVAL, "tb_decode_advance: null pointer");
  advance_kernel<<<1, 1, 0, as_stream(stream)>>>(idx_dev, ids_dev, pos_dev, history_dev, (int)max_seq);
  return check_launch("tb_decode_advance");
}

// ---- streams and graphs ------------------------------------------------------------

tb_status tb_stream_create(tb_stream *out) {
  if (!out) return fail(TB_EINVAL, "tb_stream_create: null pointer");
  DeviceState *st;
  TB_TRY(device_state(&st));
  cudaStream_t s = nullptr;
  cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (e != cudaSuccess) return fail(TB_ECUDA, "tb_stream_create: %s", cudaGetErrorString(e));
  *out = reinterpret_cast<tb_stream>(s);
  return TB_OK;
}

tb_status tb_stream_destroy(tb_stream s) {
  if (!s) return TB_OK;
  cudaError_t e = cudaStreamDestroy(as_stream(s));
  if (e != cudaSuccess) return fail(TB_ECUDA, "tb_stream_destroy: %s", cudaGetErrorString(e));
  return TB_OK;
}

tb_status tb_capture_begin(tb_stream s) {
  if (!s) return fail(TB_EINVAL, "tb_capture_begin: capture needs a created stream, not the default stream");
  cudaError_t e = cudaStreamBeginCapture(as_stream(s), cudaStreamCaptureModeRelaxed);
  if (e != cudaSuccess) return fail(TB_ECUDA, "tb_capture_begin: %s", cudaGetErrorString(e));
  return TB_OK;
}

tb_status tb_capture_end(tb_stream s, tb_graph *out) {
  if (!s || !out) return fail(TB_EINVAL, "tb_capture_end: null argument");
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(as_stream(s), &g);
  if (e != cudaSuccess) return fail(TB_ECUDA, "tb_capture_end: %s", cudaGetErrorString(e));
  cudaGraphExec_t x = nullptr;
  e = cudaGraphInstantiate(&x, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return fail(TB_ECUDA, "tb_capture_end: instantiate: %s", cudaGetErrorString(e));
  *out = reinterpret_cast<tb_graph>(x);
  return TB_OK;
}

tb_status tb_graph_launch(tb_graph g, tb_stream s) {
  if (!g) return fail(TB_EINVAL, "tb_graph_launch: null graph");
  cudaError_t e = cudaGraphLaunch(reinterpret_cast<cudaGraphExec_t>(g), as_stream(s));
  if (e != cudaSuccess) return fail(TB_ECUDA, "tb_graph_launch: %s", cudaGetErrorString(e));
  return TB_OK;
}

tb_status tb_graph_destroy(tb_graph g) {
  if (!g) return TB_OK;
  cudaError_t e = cudaGraphExecDestroy(reinterpret_cast<cudaGraphExec_t>(g));
  if (e != cudaSuccess) return fail(TB_ECUDA, "tb_graph_destroy: %s", cudaGetErrorString(e));
  return TB_OK;
}

}  // extern "C"
