// tb_attention.cu -- causal grouped-query attention of a prompt (prefill) in
// one launch: tb_attention_prefill.
//
// The reference computes it head by head (src/nn/attention.cpp:104-141): for
// query head h with key/value head h / (H / KVH), scores = Q_h K_h^T (the fp32
// matmul: an fma chain over d in increasing order), scores * scale, the causal
// mask (key t > query position: -1e9), Softmax::forward (max, exp(x - max),
// sum, divide), then probs V_h (an fma chain over the keys in increasing
// order) copied into the context.  Here one CTA takes one key/value head and a
// block of queries for every query head of the group, so each key and value row
// is read once per CTA for all of them:
//   1. the group's query rows into shared memory;
//   2. scores for key tiles of 64 (the tile transposed in shared memory so
//      that consecutive threads read consecutive keys), the same fma chain
//      over d, then * scale; keys past a query's position are left out;
//   3. per row: max, e = exp(s - max), sum, p = e / sum (a warp per row; exp
//      is the __expf intrinsic and the sum a warp tree, as in tb_softmax);
//      left-out keys have p = 0, exactly what exp(-1e9 - max) gives;
//   4. out = sum over keys in increasing order of p * v, an fma chain, value
//      tiles of 64 rows in shared memory.
// Only exp and the order of the softmax sum differ from the reference.
#include <algorithm>

#include "tb_internal.cuh"

namespace tb {
namespace {

constexpr int kAD = 64;        // head_dim
constexpr int kAT = 256;       // threads
constexpr int kKT = 64;        // keys per tile

// CTA (query block qb, key/value head kvh): rows r = g * QB + i for query head
// g of the group (G heads) and query i of the block.
template <int QB>
__global__ void __launch_bounds__(kAT) attention_prefill_kernel(
    const float *__restrict__ q, int64_t ldq, const float *__restrict__ kc, const float *__restrict__ vc, int S,
    int pos0, int H, int KVH, float scale, float *__restrict__ out, int64_t ldo, int ld_scores) {
  extern __shared__ __align__(16) float sm[];
  const int G = H / KVH, R = G * QB;
  const int kvh = blockIdx.y, q0 = blockIdx.x * QB;
  const int nq = min(QB, S - q0);
  const int nkeys = pos0 + q0 + nq;  // keys 0 .. position of the block's last query
  const int row = KVH * kAD;
  float *qs = sm;                          // [R][64]
  float *kt = qs + R * kAD;                // [64][kKT + 1] keys transposed
  float *vt = kt + kAD * (kKT + 1);        // [kKT][64]
  float *sc = vt + kKT * kAD;              // [R][ld_scores]
  const int tid = threadIdx.x;
  for (int u = tid; u < R * kAD; u += kAT) {
    const int r = u / kAD, d = u % kAD, g = r / QB, i = r % QB;
    qs[u] = i < nq ? q[(int64_t)(q0 + i) * ldq + (kvh * G + g) * kAD + d] : 0.f;
  }
  // 2. scores
  const int tk = tid % kKT, rg = tid / kKT;  // key of the tile; rows rg, rg + 4, ...
  for (int t0 = 0; t0 < nkeys; t0 += kKT) {
    __syncthreads();  // the previous tile is no longer read (and qs is complete)
    for (int u = tid; u < kKT * kAD; u += kAT) {
      const int j = u / kAD, d = u % kAD;
      kt[d * (kKT + 1) + j] = t0 + j < nkeys ? kc[(int64_t)(t0 + j) * row + kvh * kAD + d] : 0.f;
    }
    __syncthreads();
    const int t = t0 + tk;
    for (int r = rg; r < R; r += kAT / kKT) {
      const float *qr = qs + r * kAD;
      float acc = 0.f;
#pragma unroll 16
      for (int d = 0; d < kAD; ++d) acc = __fmaf_rn(qr[d], kt[d * (kKT + 1) + tk], acc);
      if (t < nkeys) sc[r * ld_scores + t] = __fmul_rn(acc, scale);
    }
  }
  __syncthreads();
  // 3. softmax per row over its keys 0 .. pos0 + q0 + i
  const int warp = tid >> 5, lane = tid & 31;
  for (int r = warp; r < R; r += kAT / 32) {
    const int i = r % QB;
    if (i >= nq) continue;
    const int n = pos0 + q0 + i + 1;
    float *sr = sc + r * ld_scores;
    float m = -INFINITY;
    for (int t = lane; t < n; t += 32) m = fmaxf(m, sr[t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
    for (int t = lane; t < n; t += 32) {
      const float e = __expf(__fsub_rn(sr[t], m));
      sr[t] = e;
      s = __fadd_rn(s, e);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    for (int t = lane; t < nkeys; t += 32) sr[t] = t < n ? __fdiv_rn(sr[t], s) : 0.f;
  }
  // 4. out = p . V, keys in increasing order
  const int d = tid % kAD;
  float acc[QB * 4 / (kAT / kAD)];  // rows rg, rg + 4, ... (R <= 4 QB rows)
  constexpr int NR = QB * 4 / (kAT / kAD);
#pragma unroll
  for (int j = 0; j < NR; ++j) acc[j] = 0.f;
  for (int t0 = 0; t0 < nkeys; t0 += kKT) {
    __syncthreads();
    for (int u = tid; u < kKT * kAD; u += kAT) {
      const int j = u / kAD, dd = u % kAD;
      vt[u] = t0 + j < nkeys ? vc[(int64_t)(t0 + j) * row + kvh * kAD + dd] : 0.f;
    }
    __syncthreads();
    const int tn = min(kKT, nkeys - t0);
    for (int j = 0; j < tn; ++j) {
      const float vv = vt[j * kAD + d];
#pragma unroll
      for (int k = 0; k < NR; ++k) {
        const int r = rg + k * (kAT / kAD);
        if (r < R) acc[k] = __fmaf_rn(sc[r * ld_scores + t0 + j], vv, acc[k]);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < NR; ++k) {
    const int r = rg + k * (kAT / kAD);
    if (r < R) {
      const int g = r / QB, i = r % QB;
      if (i < nq) out[(int64_t)(q0 + i) * ldo + (kvh * G + g) * kAD + d] = acc[k];
    }
  }
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" tb_status tb_attention_prefill(const float *q_dev, int64_t ldq, const float *k_cache_dev,
                                          const float *v_cache_dev, int64_t S, int64_t pos0, int64_t heads,
                                          int64_t kv_heads, int64_t head_dim, float scale, float *out_dev,
                                          int64_t ldo, tb_stream stream) {
  if (head_dim != kAD) return fail(TB_EINVAL, "tb_attention_prefill: head_dim %lld (64 supported)", (long long)head_dim);
  if (S < 0 || pos0 < 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0 || heads / kv_heads > 4)
    return fail(TB_EINVAL, "tb_attention_prefill: bad extents (at most 4 query heads per key/value head)");
  if (S == 0) return TB_OK;
  if (!q_dev || !k_cache_dev || !v_cache_dev || !out_dev) return fail(TB_EINVAL, "tb_attention_prefill: null pointer");
  if (ldq < heads * kAD || ldo < heads * kAD) return fail(TB_EINVAL, "tb_attention_prefill: row strides too small");
  if (pos0 + S > (1 << 20)) return fail(TB_EINVAL, "tb_attention_prefill: sequence too long");
  DeviceState *st;
  TB_TRY(device_state(&st));
  const int G = (int)(heads / kv_heads);
  const int ctx = (int)(pos0 + S);
  // the scores of a CTA's rows stay in shared memory: R rows x ctx keys
  auto smem_for = [&](int qb) {
    const int ld = (ctx + 3) / 4 * 4;
    return (size_t)(G * qb * kAD + kAD * (kKT + 1) + kKT * kAD + (size_t)G * qb * ld) * 4;
  };
  const size_t room = (size_t)st->smem_optin;
  cudaStream_t s = as_stream(stream);
  const int ld = (ctx + 3) / 4 * 4;
#define TB_ATTN(QB)                                                                                                 \
  do {                                                                                                              \
    const size_t smem = smem_for(QB);                                                                               \
    TB_TRY(ensure_smem_for(attention_prefill_kernel<QB>, smem));                                                    \
    const dim3 grid((unsigned)((S + QB - 1) / QB), (unsigned)kv_heads);                                            \
    attention_prefill_kernel<QB><<<grid, kAT, smem, s>>>(q_dev, ldq, k_cache_dev, v_cache_dev, (int)S, (int)pos0,   \
                                                         (int)heads, (int)kv_heads, scale, out_dev, ldo, ld);       \
    return check_launch("tb_attention_prefill");                                                                    \
  } while (0)
  if (smem_for(8) <= room) TB_ATTN(8);
  if (smem_for(4) <= room) TB_ATTN(4);
  if (smem_for(1) <= room) TB_ATTN(1);
#undef TB_ATTN
  return fail(TB_EINVAL, "tb_attention_prefill: %d keys exceed the shared memory of one CTA", ctx);
}
