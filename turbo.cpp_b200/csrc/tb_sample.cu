// tb_sample.cu -- nucleus (top-p) sampling of one row of logits on the device
// (sample_top_p, src/core/sampler.cpp:28-86).
//
// The reference: probabilities softmax(logits / temperature) with a
// sequential fp32 sum, (probability, id) pairs sorted by descending
// probability (std::sort), the shortest prefix whose fp32 running sum reaches
// top_p, then a draw from std::discrete_distribution over that prefix with a
// random_device-seeded mt19937.  Here the caller supplies the uniform number
// u in [0, 1); the draw is the first prefix position whose cumulative mass
// reaches u times the prefix's mass (discrete_distribution's lower_bound over
// its normalised partial sums).
//
// No sort.  Both cut points -- the end of the top_p prefix and the drawn
// token -- are found by a radix select over the probabilities' bit patterns
// (non-negative floats order as their bits) with each bucket's probability
// mass summed exactly as an integer, q(p) = floor(p * 2^62), so a prefix mass
// is exact.  Digits are bits 29..19, 18..7 and 6..0 (bits 31 and 30 are 0
// for 0 <= p <= 1); equal probabilities are ordered by token id (std::sort
// leaves them in an unspecified order).  The result can differ from the reference's only where
// top_p or u lies within fp32 rounding of a prefix boundary: the device's exp
// is CUDA's expf (within 2 ulp), its sum is taken in another order, and the
// reference's prefix sums are fp32 running sums.  A NaN logit makes the sum
// NaN (in the reference too); no probability is then positive and finite and
// the result is greedy_sample's choice, the first maximum.
//
// Layout: one thread-block cluster of CL CTAs x 1024 threads.  CTA r keeps
// the contiguous slice [r*n_loc, (r+1)*n_loc) of the row in shared memory for
// the whole kernel (read from HBM once), turned in place into scaled logits,
// exp values and probabilities.  Per digit level each CTA histograms its slice
// (count and exact mass per bucket, 32-bit shared atomics); CTA r then owns
// 1/CL of the buckets, sums them over the cluster through distributed shared
// memory, scans them, and the cluster agrees on the bucket where the running
// mass reaches the target.  Waits are the hardware cluster barrier only.
#include <cooperative_groups.h>

#include <climits>

#include "tb_internal.cuh"

namespace tb {
namespace {

namespace cg = cooperative_groups;

constexpr int kSampThreads = 1024;
constexpr int kL0Buckets = 2048;  // level 0: bits 29..19 (p <= 1 keeps bit 30 clear)
constexpr int kL1Buckets = 4096;  // levels 1 and 2: bits 18..7, then 6..0
constexpr int kCacheBuckets = kL0Buckets / 8;  // one CTA's level-0 bucket range (8-CTA cluster)
// per bucket four 32-bit counters: mass bits 63..32, 31..16, 15..0 and the count
constexpr int kFixedSmem = (kL0Buckets + kL1Buckets) * 16 + kCacheBuckets * 12;
constexpr double kQ62 = 4611686018427387904.0;  // 2^62
constexpr size_t kStaticReserve = 2048;  // bytes kept for the kernel's static shared memory

__device__ __forceinline__ uint32_t pbits(float p) { return p > 0.f ? __float_as_uint(p) : 0u; }
// floor(p * 2^62) from p's bits (bit 31 clear): the 24-bit significand times
// 2^(exponent - 88), exactly; 0 for zero, subnormals (below 2^-126, whose
// product is below 1) and anything above 1.
__device__ __forceinline__ uint64_t qmass_bits(uint32_t b) {
  const int e = (int)(b >> 23);
  if (e == 0 || b > 0x3F800000u) return 0ull;
  const uint64_t m = (uint64_t)((b & 0x7FFFFFu) | 0x800000u);
  const int sh = e - 88;
  return sh >= 0 ? m << sh : (sh > -64 ? m >> -sh : 0ull);
}
__device__ __forceinline__ uint64_t qmass(float p) { return qmass_bits(pbits(p)); }
__device__ __forceinline__ int level_shift(int l) { return l == 0 ? 19 : (l == 1 ? 7 : 0); }
__device__ __forceinline__ int level_width(int l) { return l == 0 ? 11 : (l == 1 ? 12 : 7); }

// A histogram of nbk buckets in shared memory.  Each bucket's exact mass is
// kept in three 32-bit sums (a 64-bit shared atomic costs about ten 32-bit
// ones): bits 63..32 of the element masses, whose sum is bounded by the total
// mass (< 2^32 * 1.1), and bits 31..16 and 15..0, whose sums are bounded by
// 2^16 times the slice length (< 2^31).
struct Hist {
  uint32_t *hi, *mid, *lo, *cnt;
};
__device__ __forceinline__ Hist hist_at(uint32_t *base, int nbk) {
  return Hist{base, base + nbk, base + 2 * nbk, base + 3 * nbk};
}
__device__ __forceinline__ void hist_clear(const Hist &h, int nbk) {
  for (int d = threadIdx.x; d < nbk; d += blockDim.x) h.hi[d] = h.mid[d] = h.lo[d] = h.cnt[d] = 0u;
}
__device__ __forceinline__ void hist_add(const Hist &h, uint32_t d, uint64_t q) {
  atomicAdd(&h.cnt[d], 1u);
  const uint32_t hi = (uint32_t)(q >> 32), mid = (uint32_t)(q >> 16) & 0xFFFFu, lo = (uint32_t)q & 0xFFFFu;
  if (hi) atomicAdd(&h.hi[d], hi);
  if (mid) atomicAdd(&h.mid[d], mid);
  if (lo) atomicAdd(&h.lo[d], lo);
}

// What each CTA publishes to the others (read through distributed shared memory).
struct SamplePub {
  float maxv;        // slice maximum of the scaled logits
  int32_t maxi;      // its first global index
  float esum;        // slice sum of exp(scaled - M)
  uint64_t mass;     // slice total of q(p)
  uint64_t seg;      // per level: total mass of this CTA's bucket range
  int32_t cand_q;    // per level: first bucket (descending) of this range where the target is reached, or INT_MAX
  uint32_t cand_digit, cand_count;
  uint64_t cand_above;  // mass before that bucket
  int32_t last_q;       // per level: last non-empty bucket of this range, or -1
  uint32_t last_digit, last_count;
  uint64_t last_above;
};

// Cluster-uniform selection state (every CTA holds the same values).
struct SelState {
  uint32_t prefix, mask;  // bits fixed so far
  uint64_t above;         // mass of every element ordered before the group
  uint32_t count;         // elements in the group
  uint32_t reached;       // 0 when the target exceeded the mass (fallback taken)
};

struct SampleScratch {
  float redf[32];
  int32_t redi[32];
  uint64_t red64[32];
  float M, S;
  int32_t Mi;
  uint64_t off;
  int32_t qmin, qlast, owner, jl;
};

// Histogram of the slice elements in the current group by the digit of level l.
__device__ void build_hist(const float *sl, int len, int l, const SelState &st, const Hist &h) {
  const int shift = level_shift(l), nbk = 1 << level_width(l);
  hist_clear(h, nbk);
  __syncthreads();
  const uint32_t prefix = st.prefix, mask = st.mask;
  for (int k0 = threadIdx.x; k0 < len; k0 += 4 * kSampThreads) {
    uint32_t b[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int k = k0 + u * kSampThreads;
      b[u] = k < len ? pbits(sl[k]) : 0u;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (k0 + u * kSampThreads < len && (b[u] & mask) == prefix)
        hist_add(h, (b[u] >> shift) & (uint32_t)(nbk - 1), qmass_bits(b[u]));
  }
  __syncthreads();
}

// One digit level across the cluster: finds the bucket where the running mass
// (descending order, from st.above) first reaches `target` and narrows st to it.
// cm/cc (this CTA's range of cluster-summed buckets) are filled when `cache`
// is 1 and read instead of the remote histograms when it is 2.
template <int CL>
__device__ void cluster_level(cg::cluster_group &cluster, int l, const Hist &h, uint64_t target, SelState &st,
                              SamplePub &pub, SampleScratch &scr, uint64_t *cm, uint32_t *cc, int cache) {
  const int r = (int)cluster.block_rank(), tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nbk = 1 << level_width(l), per = nbk / CL;
  // bucket q of this CTA's range (descending digit order), summed over the cluster
  const int q = r * per + tid;
  const uint32_t d = (uint32_t)(nbk - 1 - q);
  uint64_t gm = 0;
  uint32_t gc = 0;
  if (tid < per) {
    if (cache == 2) {
      gm = cm[tid];
      gc = cc[tid];
    } else {
#pragma unroll 8
      for (int rr = 0; rr < CL; ++rr) {
        gm += ((uint64_t)*cluster.map_shared_rank(&h.hi[d], rr) << 32) +
              ((uint64_t)*cluster.map_shared_rank(&h.mid[d], rr) << 16) + *cluster.map_shared_rank(&h.lo[d], rr);
        gc += *cluster.map_shared_rank(&h.cnt[d], rr);
      }
      if (cache == 1) {
        cm[tid] = gm;
        cc[tid] = gc;
      }
    }
  }
  // inclusive scan of gm over the range (threads >= per hold 0)
  uint64_t incl = gm;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) scr.red64[warp] = incl;
  if (tid == 0) {
    scr.qmin = INT_MAX;
    scr.qlast = -1;
  }
  __syncthreads();
  for (int w = 0; w < warp; ++w) incl += scr.red64[w];
  if (tid == per - 1) pub.seg = incl;
  cluster.sync();  // every range total published; the level's histograms are no longer read
  if (warp == 0) {
    uint64_t v = lane < r ? cluster.map_shared_rank(&pub, lane)->seg : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) scr.off = st.above + v;
  }
  __syncthreads();
  const uint64_t acc = scr.off + incl;  // mass through bucket q
  if (tid < per && gc > 0) {
    if (acc >= target) atomicMin(&scr.qmin, q);
    atomicMax(&scr.qlast, q);
  }
  __syncthreads();
  if (tid == 0) {
    pub.cand_q = scr.qmin;
    pub.last_q = scr.qlast;
  }
  if (tid < per && q == scr.qmin) {
    pub.cand_digit = d;
    pub.cand_count = gc;
    pub.cand_above = acc - gm;
  }
  if (tid < per && q == scr.qlast) {
    pub.last_digit = d;
    pub.last_count = gc;
    pub.last_above = acc - gm;
  }
  cluster.sync();  // candidates published
  if (warp == 0) {
    const SamplePub *rp = cluster.map_shared_rank(&pub, lane < CL ? lane : 0);
    const bool has = lane < CL && rp->cand_q != INT_MAX;
    const bool nonempty = lane < CL && rp->last_q >= 0;
    const uint32_t hb = __ballot_sync(0xffffffffu, has), nb = __ballot_sync(0xffffffffu, nonempty);
    // the first range holding a candidate; if none, the last non-empty bucket
    const int src = hb ? __ffs(hb) - 1 : (nb ? 31 - __clz(nb) : 0);
    if (lane == src) {
      const uint32_t dig = hb ? rp->cand_digit : rp->last_digit;
      st.prefix |= dig << level_shift(l);
      st.mask |= (uint32_t)(nbk - 1) << level_shift(l);
      st.above = hb ? rp->cand_above : rp->last_above;
      st.count = hb ? rp->cand_count : rp->last_count;
      if (!hb) st.reached = 0u;
    }
  }
  __syncthreads();
}

// Position j (1-based, among elements of equal bits ordered by id) of the
// element where the running mass reaches `target` inside the final group.
__device__ __forceinline__ uint32_t tie_rank(const SelState &st, uint64_t target) {
  if (!st.reached) return st.count > 0 ? st.count : 1u;
  const uint64_t qs = qmass(__uint_as_float(st.prefix));
  if (qs == 0 || target <= st.above) return 1u;
  const uint64_t j = (target - st.above + qs - 1) / qs;
  return (uint32_t)max((uint64_t)1, min(j, (uint64_t)max(st.count, 1u)));
}

// `first`: the level-0 cluster sums are read remotely and kept (cm, cc); the
// second selection reuses them.
template <int CL>
__device__ void select_desc(cg::cluster_group &cluster, uint64_t target, const float *sl, int len, const Hist &h0,
                            const Hist &h1, uint64_t *cm, uint32_t *cc, bool first, SelState &st, SamplePub &pub,
                            SampleScratch &scr) {
  __syncthreads();  // every thread is done with the previous selection's state
  if (threadIdx.x == 0) st = SelState{0u, 0u, 0ull, 0u, 1u};
  __syncthreads();
  cluster_level<CL>(cluster, 0, h0, target, st, pub, scr, cm, cc, first ? 1 : 2);
  for (int l = 1; l < 3; ++l) {
    build_hist(sl, len, l, st, h1);
    cluster.sync();  // every CTA's histogram of this level is complete before any is read
    cluster_level<CL>(cluster, l, h1, target, st, pub, scr, cm, cc, 0);
  }
}

// Where the uniform number comes from and where the drawn id goes: u, or
// u_dev[*pos_dev] (position clamped into [0, max_seq)) when u_dev is set; the
// id to out32 and/or out64.
struct SampleIO {
  double u;
  const double *u_dev;
  const int32_t *pos_dev;
  int max_seq;
  int32_t *out32;
  int64_t *out64;
};

__device__ __forceinline__ void emit(const SampleIO &io, int64_t id) {
  if (io.out32) *io.out32 = (int32_t)id;
  if (io.out64) *io.out64 = id;
}

template <int CL>
__global__ void __launch_bounds__(kSampThreads, 1)
    sample_top_p_kernel(const float *__restrict__ logits, int V, int n_loc, float temperature, float top_p,
                        SampleIO io) {
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) uint8_t smem[];
  uint32_t *hbase = reinterpret_cast<uint32_t *>(smem);
  const Hist h0 = hist_at(hbase, kL0Buckets), h1 = hist_at(hbase + 4 * kL0Buckets, kL1Buckets);
  uint64_t *cm = reinterpret_cast<uint64_t *>(hbase + 4 * (kL0Buckets + kL1Buckets));
  uint32_t *cc = reinterpret_cast<uint32_t *>(cm + kCacheBuckets);
  float *sl = reinterpret_cast<float *>(cc + kCacheBuckets);
  __shared__ SamplePub pub;
  __shared__ SampleScratch scr;
  __shared__ SelState st;
  const int r = (int)cluster.block_rank(), tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int start = r * n_loc, len = max(0, min(n_loc, V - start));

  // 1. the slice, scaled by 1/temperature (a division, as the reference), and its first maximum
  hist_clear(h0, kL0Buckets);
  float m = -INFINITY;
  int mi = INT_MAX;
  const float *src = logits + start;
  if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    const int nq = len >> 2;
    for (int k = tid; k < nq; k += kSampThreads) {
      float4 v = __ldg(reinterpret_cast<const float4 *>(src) + k);
      v.x = __fdiv_rn(v.x, temperature);
      v.y = __fdiv_rn(v.y, temperature);
      v.z = __fdiv_rn(v.z, temperature);
      v.w = __fdiv_rn(v.w, temperature);
      reinterpret_cast<float4 *>(sl)[k] = v;
      if (v.x > m) m = v.x, mi = start + 4 * k;
      if (v.y > m) m = v.y, mi = start + 4 * k + 1;
      if (v.z > m) m = v.z, mi = start + 4 * k + 2;
      if (v.w > m) m = v.w, mi = start + 4 * k + 3;
    }
    for (int k = 4 * nq + tid; k < len; k += kSampThreads) {
      const float v = __fdiv_rn(__ldg(src + k), temperature);
      sl[k] = v;
      if (v > m) m = v, mi = start + k;
    }
  } else {
    for (int k = tid; k < len; k += kSampThreads) {
      const float v = __fdiv_rn(__ldg(src + k), temperature);
      sl[k] = v;
      if (v > m) m = v, mi = start + k;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, mi, o);
    if (m2 > m || (m2 == m && i2 < mi)) m = m2, mi = i2;
  }
  if (lane == 0) scr.redf[warp] = m, scr.redi[warp] = mi;
  __syncthreads();
  if (tid == 0) {
    float bm = -INFINITY;
    int bi = INT_MAX;
    for (int w = 0; w < kSampThreads / 32; ++w)
      if (scr.redf[w] > bm || (scr.redf[w] == bm && scr.redi[w] < bi)) bm = scr.redf[w], bi = scr.redi[w];
    pub.maxv = bm;
    pub.maxi = bi;
  }
  cluster.sync();

  // 2. M = the row maximum; e = exp(scaled - M) in place and the slice sum
  if (warp == 0) {
    const SamplePub *rp = cluster.map_shared_rank(&pub, lane < CL ? lane : 0);
    float bm = lane < CL ? rp->maxv : -INFINITY;
    int bi = lane < CL ? rp->maxi : INT_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, bm, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      if (m2 > bm || (m2 == bm && i2 < bi)) bm = m2, bi = i2;
    }
    if (lane == 0) scr.M = bm, scr.Mi = bi == INT_MAX ? 0 : bi;
  }
  __syncthreads();
  const float M = scr.M;
  float s = 0.f;
  for (int k = tid; k < len; k += kSampThreads) {
    const float e = expf(__fsub_rn(sl[k], M));
    sl[k] = e;
    s = __fadd_rn(s, e);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
  if (lane == 0) scr.redf[warp] = s;
  __syncthreads();
  if (tid == 0) {
    float t = 0.f;
    for (int w = 0; w < kSampThreads / 32; ++w) t = __fadd_rn(t, scr.redf[w]);
    pub.esum = t;
  }
  cluster.sync();

  // 3. S = the row sum (slices in order); p = e / S in place, the level-0 histogram, the slice mass
  if (warp == 0) {
    const float v = lane < CL ? cluster.map_shared_rank(&pub, lane)->esum : 0.f;
    float t = 0.f;
    for (int rr = 0; rr < CL; ++rr) t = __fadd_rn(t, __shfl_sync(0xffffffffu, v, rr));
    if (lane == 0) scr.S = t;
  }
  __syncthreads();
  const float S = scr.S;
  uint64_t mass = 0;
  for (int k0 = tid; k0 < len; k0 += 4 * kSampThreads) {
    float e[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int k = k0 + u * kSampThreads;
      e[u] = k < len ? sl[k] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int k = k0 + u * kSampThreads;
      if (k < len) {
        const float p = __fdiv_rn(e[u], S);
        sl[k] = p;
        const uint32_t b = pbits(p);
        const uint64_t qm = qmass_bits(b);
        mass += qm;
        hist_add(h0, min(b >> 19, (uint32_t)(kL0Buckets - 1)), qm);  // p <= 1: b >> 19 <= 2032
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mass += __shfl_xor_sync(0xffffffffu, mass, o);
  if (lane == 0) scr.red64[warp] = mass;
  __syncthreads();
  if (tid == 0) {
    uint64_t t = 0;
    for (int w = 0; w < kSampThreads / 32; ++w) t += scr.red64[w];
    pub.mass = t;
  }
  cluster.sync();
  uint64_t tot = 0;
  if (warp == 0) {
    uint64_t v = lane < CL ? cluster.map_shared_rank(&pub, lane)->mass : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) scr.off = v;
  }
  __syncthreads();
  tot = scr.off;
  if (r == 0 && tid == 0) emit(io, scr.Mi);  // greedy choice unless a draw replaces it
  if (tot == 0) {  // no positive finite probability (a NaN or infinite logit)
    cluster.sync();
    return;
  }

  // 4. end of the top_p prefix: first position whose prefix mass reaches ceil(top_p * 2^62)
  const double tq = ceil((double)top_p * kQ62);
  const uint64_t t1 = !(tq < (double)tot) ? tot : (tq <= 0.0 ? 0ull : (uint64_t)tq);
  select_desc<CL>(cluster, t1, sl, len, h0, h1, cm, cc, true, st, pub, scr);
  const uint64_t C = st.above + (uint64_t)tie_rank(st, t1) * qmass(__uint_as_float(st.prefix));

  // 5. the draw: first position whose prefix mass reaches ceil(u * C)
  const double u = io.u_dev ? io.u_dev[min(max(*io.pos_dev, 0), io.max_seq - 1)] : io.u;
  const double uu = u > 0.0 ? u : 0.0;
  const double tu = ceil(uu * (double)C);
  const uint64_t t2 = !(tu < (double)C) ? C : (uint64_t)tu;
  select_desc<CL>(cluster, t2, sl, len, h0, h1, cm, cc, false, st, pub, scr);
  const uint32_t j = tie_rank(st, t2);
  const uint32_t bstar = st.prefix, dlast = bstar & 0x7Fu;
  // the j-th element (by id) of the final group: find the CTA that holds it
  if (warp == 0) {
    const uint32_t c = lane < CL ? *cluster.map_shared_rank(&h1.cnt[dlast], lane) : 0u;
    uint32_t incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    const uint32_t hit = __ballot_sync(0xffffffffu, lane < CL && c > 0 && incl - c < j && j <= incl);
    const int own = hit ? __ffs(hit) - 1 : -1;
    const uint32_t before = __shfl_sync(0xffffffffu, incl - c, own < 0 ? 0 : own);
    if (lane == 0) {
      scr.owner = own;
      scr.jl = (int)(j - before);
    }
  }
  __syncthreads();
  if (r == scr.owner) {
    const int jl = scr.jl;
    int running = 0;
    const int rounds = (len + kSampThreads - 1) / kSampThreads;
    for (int it = 0; it < rounds; ++it) {
      const int k = it * kSampThreads + tid;
      const bool match = k < len && pbits(sl[k]) == bstar;
      const int cnt = __syncthreads_count(match);
      if (running + cnt >= jl) {
        const uint32_t bal = __ballot_sync(0xffffffffu, match);
        if (lane == 0) scr.redi[warp] = __popc(bal);
        __syncthreads();
        if (match) {
          int rank = running + __popc(bal & ((1u << lane) - 1u)) + 1;
          for (int w = 0; w < warp; ++w) rank += scr.redi[w];
          if (rank == jl) emit(io, start + k);
        }
        break;
      }
      running += cnt;
    }
  }
  cluster.sync();  // no CTA leaves while another may still read its shared memory
}

template <int CL>
tb_status launch_sample(const float *logits, int V, float temperature, float top_p, const SampleIO &io, size_t smem,
                        int n_loc, cudaStream_t s) {
  auto kern = sample_top_p_kernel<CL>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess && CL > 8) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return fail(TB_ECUDA, "tb_sample_top_p: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CL, 1, 1);
  cfg.blockDim = dim3(kSampThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // The mid-bit mass sums of a bucket (16-bit parts of up to n_loc elements)
  // stay below 2^32 only while n_loc < 2^16.
  if (n_loc >= 65536) return fail(TB_EINVAL, "tb_sample_top_p: slice of %d elements per CTA", n_loc);
  if (CL > 8) {
    // A 16-CTA cluster of 1024-thread CTAs with nearly all of each SM's shared
    // memory is a non-portable size: check that the GPU can place one.
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
    if (e != cudaSuccess) return fail(TB_ECUDA, "tb_sample_top_p: %s", cudaGetErrorString(e));
    if (clusters < 1) return fail(TB_EINVAL, "tb_sample_top_p: a %d-CTA cluster does not fit this GPU", CL);
  }
  e = cudaLaunchKernelEx(&cfg, kern, logits, V, n_loc, temperature, top_p, io);
  if (e != cudaSuccess) return fail(TB_ECUDA, "tb_sample_top_p: %s", cudaGetErrorString(e));
  return check_launch("tb_sample_top_p");
}

// Checks the arguments, picks the cluster size and launches.
tb_status sample_launch(const char *who, const float *logits, int64_t vocab, float temperature, float top_p,
                        const SampleIO &io, tb_stream stream) {
  if (!logits || !(io.out32 || io.out64)) return fail(TB_EINVAL, "%s: null pointer", who);
  if (vocab <= 0 || vocab > INT_MAX) return fail(TB_EINVAL, "%s: vocab %lld out of range", who, (long long)vocab);
  if (!(temperature > 0.f)) return fail(TB_EINVAL, "%s: temperature must be positive", who);
  DeviceState *st;
  TB_TRY(device_state(&st));
  // slices of a multiple of 4 elements, so that each starts 16-byte aligned when the row does
  auto slice = [&](int cl) { return (int)((((vocab + cl - 1) / cl) + 3) / 4 * 4); };
  const int n8 = slice(8), n16 = slice(16);
  const size_t fixed = kFixedSmem;
  const size_t smem8 = fixed + (size_t)n8 * 4, smem16 = fixed + (size_t)n16 * 4;
  const size_t room = (size_t)st->smem_optin - kStaticReserve;  // the kernel's static shared memory is below this
  cudaStream_t s = as_stream(stream);
  if (smem8 <= room) return launch_sample<8>(logits, (int)vocab, temperature, top_p, io, smem8, n8, s);
  if (smem16 <= room) return launch_sample<16>(logits, (int)vocab, temperature, top_p, io, smem16, n16, s);
  return fail(TB_EINVAL, "%s: vocab %lld exceeds the %lld a 16-CTA cluster holds in shared memory", who,
              (long long)vocab, (long long)((room - fixed) / 4 * 16));
}
}  // namespace
}  // namespace tb

using namespace tb;

extern "C" {

tb_status tb_sample_top_p(const float *logits, int64_t vocab, float temperature, float top_p, double u,
                          int32_t *out, tb_stream stream) {
  return sample_launch("tb_sample_top_p", logits, vocab, temperature, top_p,
                       SampleIO{u, nullptr, nullptr, 0, out, nullptr}, stream);
}

tb_status tb_sample_top_p_at(const float *logits, int64_t vocab, float temperature, float top_p, const double *u_dev,
                             const int32_t *pos_dev, int64_t max_seq, int64_t *idx_dev, tb_stream stream) {
  if (!u_dev || !pos_dev || max_seq <= 0 || max_seq > INT_MAX)
    return fail(TB_EINVAL, "tb_sample_top_p_at: uniform numbers, position or max_seq missing");
  return sample_launch("tb_sample_top_p_at", logits, vocab, temperature, top_p,
                       SampleIO{0.0, u_dev, pos_dev, (int)max_seq, nullptr, idx_dev}, stream);
}

}  // extern "C"
