// tb_noalloc.cu -- a Q4_0 matmul entry point that allocates no device memory.
//
// tb_matmul_quant(TB_Q4_0, ...) first quantizes X to Q8_0 into scratch memory
// taken from the stream-ordered allocator.  Some callers cannot allocate at
// that point: a serving process that reserves its whole device-memory budget
// at start-up and must not grow it per request, or a latency-critical loop in
// which an allocator call may synchronize or fail.  For them,
// tb_matmul_q4_0_static_scratch runs the same two kernels with the scratch in
// a fixed array compiled into this library instead.
//
// The array (kScratchBytes, 8 MiB) lives in every GPU that loads the library,
// for as long as the process runs.  Its host-side name is only a stand-in for
// the symbol, never a device address; the device address is looked up once
// per device with cudaGetSymbolAddress and cached.  A second file-scope word
// is this entry point's device error word (a bounded wait that gave up sets
// bit 0), found the same way; tb_take_device_errors reads and clears it
// together with the library's regular error word.
#include <atomic>
#include <mutex>

#include "tb_internal.cuh"

namespace tb {
tb_status launch_quantize_q8_0(const float *x, int64_t rows, int64_t k, void *blocks, cudaStream_t s,
                               int sm_count);
tb_status launch_q4_0_exact(const uint8_t *xq, int64_t M, int64_t K, const void *w, int64_t N,
                            float *y, cudaStream_t s, const DeviceState *st);
}  // namespace tb

namespace {

constexpr size_t kScratchBytes = size_t(8) << 20;  // 8 MiB: X[512, 8192] as Q8_0 is 4.25 MiB

// Holds the Q8_0 copy of X between the two kernels of a call.
static __device__ __align__(256) uint8_t g_q4_scratch[kScratchBytes];
// The kernels' error word for calls through this entry point.
static __device__ uint32_t g_q4_scratch_err;

struct ScratchSlot {
  std::atomic<void *> addr{nullptr};
  uint32_t *err = nullptr;  // device address of g_q4_scratch_err
  int sm_count = 0;
  int smem_optin = 0;
};
ScratchSlot g_slots[64];
std::mutex g_slot_mu;

// Per-device set-up on the first call made with that device current.
tb_status scratch_for_device(ScratchSlot **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return tb::fail(TB_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return tb::fail(TB_ECUDA, "device %d out of range", dev);
  ScratchSlot &slot = g_slots[dev];
  if (slot.addr.load(std::memory_order_acquire) == nullptr) {
    std::lock_guard<std::mutex> lk(g_slot_mu);
    if (slot.addr.load(std::memory_order_relaxed) == nullptr) {
      int sms = 0, optin = 0, major = 0;
      e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
      if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
      if (e != cudaSuccess) return tb::fail(TB_ECUDA, "device attributes: %s", cudaGetErrorString(e));
      if (major != 10) return tb::fail(TB_ECUDA, "device %d is not an sm_100 part", dev);
      void *p = nullptr, *pe = nullptr;
      e = cudaGetSymbolAddress(&p, g_q4_scratch);
      if (e != cudaSuccess || p == nullptr)
        return tb::fail(TB_ECUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
      e = cudaGetSymbolAddress(&pe, g_q4_scratch_err);
      if (e != cudaSuccess || pe == nullptr)
        return tb::fail(TB_ECUDA, "cudaGetSymbolAddress(error word): %s", cudaGetErrorString(e));
      slot.err = static_cast<uint32_t *>(pe);
      slot.sm_count = sms;
      slot.smem_optin = optin;
      slot.addr.store(p, std::memory_order_release);
    }
  }
  *out = &slot;
  return TB_OK;
}

}  // namespace

namespace tb {
// Reads and clears this entry point's error word on the current device; a
// device where the entry point never ran has none and reports 0.
tb_status static_scratch_take_errors(uint32_t *flags) {
  *flags = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(TB_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64 || g_slots[dev].addr.load(std::memory_order_acquire) == nullptr) return TB_OK;
  uint32_t *w = g_slots[dev].err;
  uint32_t v = 0;
  e = cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && v) e = cudaMemset(w, 0, sizeof(uint32_t));
  if (e != cudaSuccess) return fail(TB_ECUDA, "tb_take_device_errors(static scratch): %s", cudaGetErrorString(e));
  *flags = v;
  return TB_OK;
}
}  // namespace tb

using namespace tb;

extern "C" tb_status tb_matmul_q4_0_static_scratch(const float *x, int64_t M, int64_t K,
                                                   const void *w, int64_t N, float *y,
                                                   tb_stream stream) {
  if (M < 0 || K < 0 || N < 0) return fail(TB_EINVAL, "tb_matmul_q4_0_static_scratch: negative extent");
  if (K % 32 != 0) return fail(TB_EINVAL, "tb_matmul_q4_0_static_scratch: K=%lld is not a multiple of 32", (long long)K);
  if (M == 0 || N == 0 || K == 0) {
    if (M > 0 && N > 0 && y) {
      cudaError_t e = cudaMemsetAsync(y, 0, (size_t)(M * N) * sizeof(float), as_stream(stream));
      if (e != cudaSuccess) return fail(TB_ECUDA, "tb_matmul_q4_0_static_scratch: %s", cudaGetErrorString(e));
    }
    return TB_OK;
  }
  if (!x || !w || !y) return fail(TB_EINVAL, "tb_matmul_q4_0_static_scratch: null pointer");
  if (N > 0x7FFFFFFF || K > 0x7FFFFFFF || M > 0x7FFFFFFF)
    return fail(TB_EINVAL, "tb_matmul_q4_0_static_scratch: extent too large");
  const size_t need = (size_t)M * (size_t)(K / 32) * 34;
  if (need > kScratchBytes)
    return fail(TB_EINVAL,
                "tb_matmul_q4_0_static_scratch: X[%lld, %lld] needs %zu bytes of Q8_0 scratch, above the "
                "fixed %zu-byte buffer; use tb_matmul_quant",
                (long long)M, (long long)K, need, kScratchBytes);
  ScratchSlot *slot;
  TB_TRY(scratch_for_device(&slot));
  void *scratch = slot->addr.load(std::memory_order_acquire);
  cudaStream_t s = as_stream(stream);
  // Every byte of the scratch that the matmul reads is written by the
  // quantisation first, so nothing needs clearing between calls.
  TB_TRY(launch_quantize_q8_0(x, M, K, scratch, s, slot->sm_count));
  DeviceState st;  // launch parameters only; nothing allocated
  st.device = -1;
  st.sm_count = slot->sm_count;
  st.smem_optin = slot->smem_optin;
  st.err_word = slot->err;
  return launch_q4_0_exact(static_cast<const uint8_t *>(scratch), M, K, w, N, y, s, &st);
}
