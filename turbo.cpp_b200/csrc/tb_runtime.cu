// tb_runtime.cu -- per-device state, error reporting, the HBM arena and the
// host<->device copies of the C ABI.
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <tuple>
#include <mutex>
#include <vector>

#include "tb_internal.cuh"

namespace tb {

namespace {
thread_local char g_msg[512] = "";
std::mutex g_mu;
DeviceState g_dev[64];

// ---- arena -----------------------------------------------------------------
// Segments are cudaMalloc'ed on demand (at least 256 MiB each) and carved by a
// first-fit free list with coalescing.  Every block is 256-byte aligned.
struct Segment {
  int device;
  char *base;
  size_t size;
  std::map<size_t, size_t> free_blocks;  // offset -> size
};
std::vector<Segment *> g_segments;
std::map<void *, std::pair<Segment *, size_t>> g_live;  // ptr -> (segment, size)
constexpr size_t kAlign = 256;
constexpr size_t kMinSegment = size_t(256) << 20;

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
}  // namespace

namespace {
std::atomic<uint64_t> g_wait_limit{2000000000ull};
}

uint64_t wait_limit_ns() { return g_wait_limit.load(std::memory_order_relaxed); }

tb_status fail(tb_status s, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return s;
}

tb_status check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(TB_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return TB_OK;
}

tb_status device_state(DeviceState **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(TB_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(TB_ECUDA, "device %d out of range", dev);
  DeviceState &st = g_dev[dev];
  if (st.device < 0) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (st.device < 0) {
      cudaDeviceProp p;
      e = cudaGetDeviceProperties(&p, dev);
      if (e != cudaSuccess) return fail(TB_ECUDA, "cudaGetDeviceProperties: %s", cudaGetErrorString(e));
      if (p.major != 10) return fail(TB_ECUDA, "device %d is sm_%d%d; this library is built for sm_100a", dev, p.major, p.minor);
      uint32_t *w = nullptr;
      e = cudaMalloc(&w, 256);
      if (e != cudaSuccess) return fail(TB_ECUDA, "cudaMalloc(error word): %s", cudaGetErrorString(e));
      e = cudaMemset(w, 0, 256);
      if (e != cudaSuccess) return fail(TB_ECUDA, "cudaMemset: %s", cudaGetErrorString(e));
      st.sm_count = p.multiProcessorCount;
      st.smem_optin = (int)p.sharedMemPerBlockOptin;
      st.smem_per_sm = (int)p.sharedMemPerMultiprocessor;
      st.smem_reserved = (int)p.reservedSharedMemPerBlock;
      st.err_word = w;
      st.device = dev;
    }
  }
  *out = &st;
  return TB_OK;
}

tb_status ensure_smem(const void *func, size_t bytes) {
  if (bytes <= 48 * 1024) return TB_OK;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(TB_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  static std::map<std::pair<const void *, int>, size_t> done;
  std::lock_guard<std::mutex> lk(g_mu);
  size_t &cur = done[{func, dev}];
  if (cur >= bytes) return TB_OK;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return fail(TB_ECUDA, "dynamic smem of %zu bytes: %s", bytes, cudaGetErrorString(e));
  // Prefer the largest shared-memory carveout so that several such CTAs fit
  // on an SM at once (the default split can leave room for only one).
  e = cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout,
                           (int)cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return fail(TB_ECUDA, "smem carveout: %s", cudaGetErrorString(e));
  cur = bytes;
  return TB_OK;
}

int resident_ctas(const void *func, int threads, size_t smem) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 1;
  static std::map<std::tuple<const void *, int, int, size_t>, int> cache;
  std::lock_guard<std::mutex> lk(g_mu);
  auto key = std::make_tuple(func, dev, threads, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, func, threads, smem) != cudaSuccess || n < 1) n = 1;
  cache[key] = n;
  return n;
}

tb_status validate_view(const tb_view *v, const char *name) {
  if (!v) return fail(TB_EINVAL, "%s: null view", name);
  if (v->rank < 0 || v->rank > TB_MAX_RANK) return fail(TB_EINVAL, "%s: rank %d unsupported", name, v->rank);
  for (int i = 0; i < v->rank; ++i) {
    if (v->shape[i] < 0) return fail(TB_EINVAL, "%s: negative extent", name);
    if (v->strides[i] < 0) return fail(TB_EINVAL, "%s: negative stride", name);
  }
  if (v->offset < 0) return fail(TB_EINVAL, "%s: negative offset", name);
  if (numel(v) > 0 && !v->data) return fail(TB_EINVAL, "%s: null data", name);
  return TB_OK;
}

}  // namespace tb

namespace tb {
namespace {
// Small copies between page-locked host memory and the device run as a kernel
// that reads or writes the host buffer through its device mapping instead of
// on a copy engine: a transfer of a few KB (a decode step's token, one row of
// activations) then costs one kernel's latency instead of a DMA round trip
// and its hand-offs with the compute engine, and, being a kernel launched with
// programmatic dependent launch, the next kernel's weight prefetch overlaps it.
// Uploads read the host buffer before griddepcontrol.wait (the host data does
// not depend on the previous kernel; the device buffer may still be read by
// it), downloads read the device buffer after it.  Pageable host memory, sizes
// above kSmallCopyMax and addresses or sizes not in 16-byte units keep the
// DMA copy.
constexpr size_t kSmallCopyMax = size_t(256) << 10;

template <bool UP>
__global__ void __launch_bounds__(256) small_copy_kernel(uint4 *__restrict__ dst, const uint4 *__restrict__ src,
                                                         int64_t n16) {
  pdl_launch_dependents();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (UP) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (i + u * stride < n16) v[u] = src[i + u * stride];
    pdl_wait();
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (i + u * stride < n16) dst[i + u * stride] = v[u];
  } else {
    pdl_wait();
    for (; i < n16; i += stride) dst[i] = src[i];
  }
}

// The device address of `host` when it is page-locked memory mapped into the
// device's address space, `dev` is device memory and the copy qualifies for
// small_copy_kernel; else null (the DMA copy then runs, and reports a pointer
// of the wrong kind as an error instead of a kernel touching it).
const void *small_pinned_alias(const void *host, const void *dev, size_t bytes) {
  if (bytes > kSmallCopyMax || bytes % 16 != 0 || ((reinterpret_cast<uintptr_t>(host) |
                                                     reinterpret_cast<uintptr_t>(dev)) & 15) != 0)
    return nullptr;
  cudaPointerAttributes at, ad;
  if (cudaPointerGetAttributes(&at, host) != cudaSuccess || cudaPointerGetAttributes(&ad, dev) != cudaSuccess) {
    cudaGetLastError();  // not a pointer the runtime knows: pageable memory
    return nullptr;
  }
  if (at.type != cudaMemoryTypeHost || !at.devicePointer) return nullptr;
  if (ad.type != cudaMemoryTypeDevice && ad.type != cudaMemoryTypeManaged) return nullptr;
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || ad.device != cur) return nullptr;  // another GPU's memory: DMA
  return at.devicePointer;
}

tb_status launch_small_copy(void *dst, const void *src, size_t bytes, bool up, cudaStream_t s, const char *who) {
  const int64_t n16 = (int64_t)(bytes / 16);
  // four 16-byte elements per thread (kSmallCopyMax / 16 / 4 / 256 = 16 CTAs at most)
  const int grid = (int)std::max<int64_t>(1, (n16 + 4 * 256 - 1) / (4 * 256));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = up ? cudaLaunchKernelEx(&cfg, small_copy_kernel<true>, static_cast<uint4 *>(dst),
                                          static_cast<const uint4 *>(src), n16)
                     : cudaLaunchKernelEx(&cfg, small_copy_kernel<false>, static_cast<uint4 *>(dst),
                                          static_cast<const uint4 *>(src), n16);
  if (e != cudaSuccess) return fail(TB_ECUDA, "%s: %s", who, cudaGetErrorString(e));
  return TB_OK;
}
}  // namespace
}  // namespace tb

using namespace tb;

extern "C" {

tb_status tb_init(int device) {
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return fail(TB_ECUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
  DeviceState *st;
  return device_state(&st);
}

const char *tb_last_error(void) { return g_msg; }

const char *tb_status_name(tb_status s) {
  switch (s) {
    case TB_OK: return "TB_OK";
    case TB_EINVAL: return "TB_EINVAL";
    case TB_ERANGE: return "TB_ERANGE";
    case TB_ERUNTIME: return "TB_ERUNTIME";
    case TB_ECUDA: return "TB_ECUDA";
    case TB_ETIMEOUT: return "TB_ETIMEOUT";
    case TB_ENOMEM: return "TB_ENOMEM";
  }
  return "TB_UNKNOWN";
}

const char *tb_version(void) { return "turbo_b200 sm_100a " __DATE__; }

tb_status tb_alloc(void **ptr, size_t bytes) {
  if (!ptr) return fail(TB_EINVAL, "tb_alloc: null out pointer");
  DeviceState *st;
  TB_TRY(device_state(&st));
  size_t need = round_up(bytes ? bytes : 1, kAlign);
  std::lock_guard<std::mutex> lk(g_mu);
  for (Segment *seg : g_segments) {
    if (seg->device != st->device) continue;
    for (auto it = seg->free_blocks.begin(); it != seg->free_blocks.end(); ++it) {
      if (it->second < need) continue;
      size_t off = it->first, sz = it->second;
      seg->free_blocks.erase(it);
      if (sz > need) seg->free_blocks[off + need] = sz - need;
      void *p = seg->base + off;
      g_live[p] = {seg, need};
      *ptr = p;
      return TB_OK;
    }
  }
  size_t segsz = need > kMinSegment ? need : kMinSegment;
  char *base = nullptr;
  cudaError_t e = cudaMalloc(&base, segsz);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(TB_ENOMEM, "tb_alloc(%zu): cudaMalloc of a %zu-byte segment failed: %s", bytes, segsz, cudaGetErrorString(e));
  }
  Segment *seg = new Segment{st->device, base, segsz, {}};
  if (segsz > need) seg->free_blocks[need] = segsz - need;
  g_segments.push_back(seg);
  g_live[base] = {seg, need};
  *ptr = base;
  return TB_OK;
}

tb_status tb_free(void *p) {
  if (!p) return TB_OK;
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_live.find(p);
  if (it == g_live.end()) return fail(TB_EINVAL, "tb_free: %p was not allocated by tb_alloc", p);
  Segment *seg = it->second.first;
  size_t off = (char *)p - seg->base, sz = it->second.second;
  g_live.erase(it);
  auto nx = seg->free_blocks.lower_bound(off);
  if (nx != seg->free_blocks.end() && nx->first == off + sz) {  // merge with next
    sz += nx->second;
    nx = seg->free_blocks.erase(nx);
  }
  if (nx != seg->free_blocks.begin()) {  // merge with previous
    auto pv = std::prev(nx);
    if (pv->first + pv->second == off) {
      pv->second += sz;
      return TB_OK;
    }
  }
  seg->free_blocks[off] = sz;
  return TB_OK;
}

tb_status tb_upload(void *dst, const void *src, size_t bytes, tb_stream s) {
  if (bytes == 0) return TB_OK;
  if (!dst || !src) return fail(TB_EINVAL, "tb_upload: null pointer");
  const void *src_dev = small_pinned_alias(src, dst, bytes);
  if (src_dev) return launch_small_copy(dst, src_dev, bytes, true, as_stream(s), "tb_upload");
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, as_stream(s));
  if (e != cudaSuccess) return fail(TB_ECUDA, "tb_upload: %s", cudaGetErrorString(e));
  return TB_OK;
}

tb_status tb_download(void *dst, const void *src, size_t bytes, tb_stream s) {
  if (bytes == 0) return TB_OK;
  if (!dst || !src) return fail(TB_EINVAL, "tb_download: null pointer");
  const void *dst_dev = small_pinned_alias(dst, src, bytes);
  if (dst_dev) return launch_small_copy(const_cast<void *>(dst_dev), src, bytes, false, as_stream(s), "tb_download");
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, as_stream(s));
  if (e != cudaSuccess) return fail(TB_ECUDA, "tb_download: %s", cudaGetErrorString(e));
  return TB_OK;
}

tb_status tb_memset(void *dst, int value, size_t bytes, tb_stream s) {
  if (bytes == 0) return TB_OK;
  if (!dst) return fail(TB_EINVAL, "tb_memset: null pointer");
  cudaError_t e = cudaMemsetAsync(dst, value, bytes, as_stream(s));
  if (e != cudaSuccess) return fail(TB_ECUDA, "tb_memset: %s", cudaGetErrorString(e));
  return TB_OK;
}

tb_status tb_sync(tb_stream s) {
  cudaError_t e = cudaStreamSynchronize(as_stream(s));
  if (e != cudaSuccess) return fail(TB_ECUDA, "tb_sync: %s", cudaGetErrorString(e));
  return TB_OK;
}

tb_status tb_take_device_errors(uint32_t *flags) {
  if (!flags) return fail(TB_EINVAL, "tb_take_device_errors: null out pointer");
  DeviceState *st;
  TB_TRY(device_state(&st));
  uint32_t v = 0;
  cudaError_t e = cudaMemcpy(&v, st->err_word, sizeof(v), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(TB_ECUDA, "tb_take_device_errors: %s", cudaGetErrorString(e));
  if (v) {
    e = cudaMemset(st->err_word, 0, sizeof(uint32_t));
    if (e != cudaSuccess) return fail(TB_ECUDA, "tb_take_device_errors: %s", cudaGetErrorString(e));
  }
  uint32_t vs = 0;
  TB_TRY(static_scratch_take_errors(&vs));
  *flags = v | vs;
  return TB_OK;
}

tb_status tb_set_wait_limit_ns(uint64_t ns) {
  g_wait_limit.store(ns, std::memory_order_relaxed);
  return TB_OK;
}

}  // extern "C"
