// tb_internal.cuh -- shared host/device helpers of the sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "turbo_b200.h"

namespace tb {

// ------------------------------------------------------------------ host side

struct DeviceState {
  int device = -1;
  int sm_count = 0;
  int smem_optin = 0;     // max dynamic shared memory per block (opt-in)
  int smem_per_sm = 0;    // shared memory per SM, all resident blocks together
  int smem_reserved = 0;  // shared memory the system reserves per block
  uint32_t *err_word = nullptr;  // device error word (bit 0 timeout, bit 1 index)
};

// Per-device state of the current device; creates it on first use.
tb_status device_state(DeviceState **out);

// Records `msg` as the calling thread's last error and returns `s`.
tb_status fail(tb_status s, const char *fmt, ...);

// Limit of the bounded waits that take it from the host (tb_set_wait_limit_ns;
// default 2 s).
uint64_t wait_limit_ns();

// Reads and clears the error word of tb_matmul_q4_0_static_scratch on the
// current device (0 when that entry point was never called there).
tb_status static_scratch_take_errors(uint32_t *flags);

// Maps a pending launch error to TB_ECUDA.
tb_status check_launch(const char *what);

inline cudaStream_t as_stream(tb_stream s) { return reinterpret_cast<cudaStream_t>(s); }

#define TB_TRY(expr)                                                                            \
  do {                                                                                          \
    tb_status _tb_s = (expr);                                                                   \
    if (_tb_s != TB_OK) return _tb_s;                                                           \
  } while (0)

// Element size of the plain (non-block) dtypes; 0 for block formats.
inline int dtype_size(int dt) {
  switch (dt) {
    case TB_F32: return 4;
    case TB_F16: return 2;
    case TB_I32: return 4;
    case TB_BF16: return 2;
    default: return 0;
  }
}

// A view with its dimensions merged where memory allows (fewer index steps).
struct Shape {
  int rank = 0;
  int64_t shape[TB_MAX_RANK];
  int64_t stride[TB_MAX_RANK];
};

inline int64_t numel(const tb_view *v) {
  // Tensor::numel (src/tensor/tensor.cpp:99-106): rank 0 counts as empty.
  if (v->rank <= 0) return 0;
  int64_t n = 1;
  for (int i = 0; i < v->rank; ++i) n *= v->shape[i];
  return n;
}

inline bool is_contiguous(const tb_view *v) {
  // Tensor::is_contiguous (src/tensor/tensor.cpp:108-116).
  int64_t expect = 1;
  for (int i = v->rank - 1; i >= 0; --i) {
    if (v->strides[i] != expect) return false;
    expect *= v->shape[i];
  }
  return true;
}

tb_status validate_view(const tb_view *v, const char *name);

// Raises the dynamic shared memory limit of `func` on the current device to at
// least `bytes`, once per (function, device): later launches make no runtime
// call besides the launch itself, so they can be captured in CUDA graphs.
tb_status ensure_smem(const void *func, size_t bytes);
template <typename F> inline tb_status ensure_smem_for(F *func, size_t bytes) {
  return ensure_smem(reinterpret_cast<const void *>(func), bytes);
}

// CTAs of `func` (launched with `threads` threads and `smem` dynamic shared
// memory) that fit on one SM at once, cached per (function, device, shape).
// Grid-stride kernels launch SMs x this many CTAs: one full wave, no tail.
int resident_ctas(const void *func, int threads, size_t smem);
template <typename F> inline int wave_grid(F *func, int threads, int64_t work_items, int sm_count,
                                           size_t smem = 0) {
  const int64_t cap = (int64_t)sm_count * resident_ctas(reinterpret_cast<const void *>(func), threads, smem);
  int64_t want = (work_items + threads - 1) / threads;
  if (want > cap) want = cap;
  return (int)(want < 1 ? 1 : want);
}

// ----------------------------------------------------------------- device side

constexpr uint32_t ERR_TIMEOUT = 1u;
constexpr uint32_t ERR_INDEX = 2u;

__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier + bulk-copy (TMA, non-tensor) helpers -------------------------

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

// Waits for `phase` of `bar` for at most `limit_ns`; on timeout sets
// ERR_TIMEOUT in *err and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t phase, uint32_t *err,
                                                  uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, phase)) return true;
  uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, phase)) return true;
    if ((it & 255u) == 255u && globaltimer_ns() - t0 > limit_ns) {
      if (err) atomicOr(err, ERR_TIMEOUT);
      return false;
    }
  }
}

// A bounded wait with a caller-given limit (tb_set_wait_limit_ns).  Limit 0
// allows no waiting at all: the wait gives up before testing the barrier, so a
// caller can exercise a kernel's timeout path without any stalled copy.
__device__ __forceinline__ bool mbar_wait_limit(uint64_t *bar, uint32_t phase, uint32_t *err,
                                                uint64_t limit_ns) {
  if (limit_ns == 0) {
    if (err) atomicOr(err, ERR_TIMEOUT);
    return false;
  }
  return mbar_wait_bounded(bar, phase, err, limit_ns);
}

// Bulk global->shared copy completing on `bar` (16-byte aligned addresses,
// size a multiple of 16).  No multicast.
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src_gmem, uint32_t bytes,
                                         uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// L2 prefetch of [src, src + bytes) (16-byte aligned address, size a multiple
// of 16); nothing is returned to the SM.
__device__ __forceinline__ void prefetch_l2(const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ---- packed fp32 pairs (sm_100a f32x2 arithmetic; each lane op is IEEE rn) ---

__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// ---- exp for the SiLU path ------------------------------------------------------
// The reference calls glibc expf, whose documented error bound is 0.502 ulp: it
// is correctly rounded except on ~0.03% of inputs.  exp_cr is written from the
// textbook table method (Tang): x = (64 m + j) ln2/64 + r, |r| <= ln2/128,
// exp(x) = 2^m * 2^(j/64) * exp(r), exp(r) from its Taylor series to degree 5
// (truncation below 2^-54 on that interval), all in double precision, rounded
// once to float.  Correctly rounded unless exp(x) lies within ~2^-47
// (relative) of a float rounding boundary.  The 64 table entries 2^(j/64) are
// computed once per CTA into the caller's shared memory (exp_cr_table_init,
// followed by a barrier).  exp_ref, double-precision libdevice exp rounded to
// float, is the self-check's yardstick, not used on a product path.
// The softmax kernels use the __expf intrinsic (2 + 1.17|x| ulp, documented),
// which is far inside their tolerance and cheaper than any of these.
__device__ __forceinline__ float exp_ref(float x) { return __double2float_rn(exp((double)x)); }

__device__ __forceinline__ void exp_cr_table_init(double *tab) {
  for (int j = threadIdx.x; j < 64; j += blockDim.x) tab[j] = exp2((double)j * (1.0 / 64.0));
}

__device__ __forceinline__ float exp_cr(float xf, const double *tab) {
  if (xf != xf) return xf;
  // exp(-110) rounds to +0 and exp(100) to +inf, so clamping changes no result
  const double x = (double)fminf(fmaxf(xf, -110.0f), 100.0f);
  const double kRound = 6755399441055744.0;  // 1.5 * 2^52: t's low word holds rint(64 x / ln2)
  const double t = fma(x, 92.33248261689366, kRound);  // 64 / ln2
  const int k = __double2loint(t);
  const double kd = t - kRound;
  const double r = fma(kd, -0.010830424696249145, x);  // ln2 / 64
  double p = 1.0 / 120.0;
  p = fma(p, r, 1.0 / 24.0);
  p = fma(p, r, 1.0 / 6.0);
  p = fma(p, r, 0.5);
  p = fma(p, r, 1.0);
  p = fma(p, r, 1.0);
  const double y = tab[k & 63] * p;  // in [0.99, 2.0): 2^m keeps it a normal double
  const int m = k >> 6;              // arithmetic shift: floor(k / 64)
  return __double2float_rn(__hiloint2double(__double2hiint(y) + (int)((unsigned)m << 20), __double2loint(y)));
}

// silu(g) * u as src/nn/swiglu.cpp:25-31 rounds it: g / (1 + exp(-g)), then * u
// (tab: the exp_cr table in shared memory)
__device__ __forceinline__ float swiglu_f32(float g, float u, const double *tab) {
  const float e = exp_cr(-g, tab);
  const float s = __fdiv_rn(g, __fadd_rn(1.0f, e));
  return __fmul_rn(s, u);
}

// programmatic dependent launch
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- a second copy of a GEMV's outputs, for other GPUs to read (NVLink) ---------

// The GEMV also stores y[i] at dst[(e & 1) * par_stride + i], where the call
// number e = *ctr + 1 (ctr: this rank's count of finished exchanges, advanced
// by the kernel that follows; read after griddepcontrol.wait).  dst is this
// GPU's exchange buffer 0 at this rank's rows; other GPUs read it once that
// kernel has published e.  Plain local stores: the launch boundary makes them
// visible.
struct PeerOut {
  float *dst;  // null: no second copy
  const unsigned long long *ctr;
  int64_t par_stride;  // floats between the two buffers
};

// The offset of this call's buffer: read once per thread, after
// griddepcontrol.wait, and passed to peer_store.
__device__ __forceinline__ int64_t peer_buffer(const PeerOut &p) {
  return p.dst ? (int64_t)((*reinterpret_cast<const volatile unsigned long long *>(p.ctr) + 1) & 1) * p.par_stride
               : 0;
}

__device__ __forceinline__ void peer_store(const PeerOut &p, int64_t buf, int64_t i, float v) {
  if (p.dst) p.dst[buf + i] = v;
}

// Q8_0 GEMV launchers (M = 1); `peer` adds the peer stores.
tb_status launch_stream_gemv(const float *x, int64_t K, const void *w, int64_t N, float *y, cudaStream_t s,
                             const DeviceState *st, const PeerOut *peer = nullptr);
tb_status launch_gemv_tc(const float *x, int64_t K, const void *w, int64_t N, float *y, cudaStream_t s,
                         const DeviceState *st, const PeerOut *peer = nullptr);
tb_status launch_q8_0_gemv_peer(const float *x, int64_t K, const void *w, int64_t N, float *y, const PeerOut &peer,
                                cudaStream_t s, const DeviceState *st);

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

}  // namespace tb
