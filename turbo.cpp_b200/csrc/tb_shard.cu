// tb_shard.cu -- vocab-sharded softmax and argmax, and the row-sharded Q8_0
// GEMV, for a group of GPUs, each held by one process (or thread) that owns
// one shard, exchanging over NCCL.
//
// The reference runs these ops whole on one CPU (src/nn/softmax.cpp:13-54,
// src/core/sampler.cpp:13-26, src/tensor/tensor.cpp:328-382); here each rank
// holds a contiguous slice of the columns (logits) or rows (weights):
//   softmax  per-shard row statistics (max m, sum of exp(x - m)) from
//            tb_softmax_shard_stats, ONE all-gather of the (m, s) pairs (over
//            NVLink peer memory after tb_shard_group_enable_peer), a
//            combine in rank order (M = max m_r, S = sum_r s_r exp(m_r - M)),
//            then tb_softmax_shard_finish writes exp(x - M) / S;
//   argmax   per-shard 64-bit keys (tb_argmax_shard_keys), one int64 MAX
//            all-reduce (or, with peer memory, a gather of the keys and a
//            max over the ranks), then tb_argmax_key_index;
//   GEMV     the rank's rows into its slot of y, one in-place all-gather; or,
//            after tb_shard_group_enable_peer, the GEMV also writes its rows
//            into this GPU's exchange buffer, and a small kernel on each rank
//            publishes the call's number in the other ranks' flags, waits for
//            theirs and reads their rows from their buffers over NVLink.
// NCCL is loaded at run time (dlopen of libnccl.so.2, preferring a copy the
// process already has loaded), so the library has no link-time dependency on
// it.  The communicator is created non-blocking with a host-side time limit,
// and aborted when the limit passes; tb_shard_group_wait bounds the wait for
// a stream's collectives the same way.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "tb_internal.cuh"

namespace tb {
namespace {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId *);
  ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *);
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *);
  ncclResult_t (*CommAbort)(ncclComm_t);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
  const char *(*GetErrorString)(ncclResult_t);
  bool ok = false;
};

NcclApi g_nccl;
std::mutex g_nccl_mu;

tb_status nccl_api(NcclApi **out) {
  std::lock_guard<std::mutex> lk(g_nccl_mu);
  if (!g_nccl.ok) {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return fail(TB_ERUNTIME, "tb_shard_group: cannot load libnccl.so.2: %s", dlerror());
#define TB_NCCL_SYM(field, name)                                                                        \
  *reinterpret_cast<void **>(&g_nccl.field) = dlsym(h, name);                                           \
  if (!g_nccl.field) return fail(TB_ERUNTIME, "tb_shard_group: libnccl.so.2 lacks %s", name);
    TB_NCCL_SYM(GetUniqueId, "ncclGetUniqueId")
    TB_NCCL_SYM(CommInitRankConfig, "ncclCommInitRankConfig")
    TB_NCCL_SYM(CommGetAsyncError, "ncclCommGetAsyncError")
    TB_NCCL_SYM(CommAbort, "ncclCommAbort")
    TB_NCCL_SYM(CommDestroy, "ncclCommDestroy")
    TB_NCCL_SYM(AllGather, "ncclAllGather")
    TB_NCCL_SYM(AllReduce, "ncclAllReduce")
    TB_NCCL_SYM(GetErrorString, "ncclGetErrorString")
#undef TB_NCCL_SYM
    g_nccl.ok = true;
  }
  *out = &g_nccl;
  return TB_OK;
}

// M[r] = max_k m_k[r], S[r] = sum over k in rank order of s_k[r] exp(m_k[r] - M[r]),
// from the gathered stats [n_ranks][2][rows] (m then s per rank).  The rescale
// is tb_softmax_shard_rescale's (__expf of the difference).
__global__ void combine_stats_kernel(const float *__restrict__ g, int n, int rows, float *__restrict__ M,
                                     float *__restrict__ S) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float m = -INFINITY;
  for (int k = 0; k < n; ++k) m = fmaxf(m, g[(size_t)k * 2 * rows + r]);
  float s = 0.f;
  for (int k = 0; k < n; ++k) {
    const float mk = g[(size_t)k * 2 * rows + r], sk = g[(size_t)k * 2 * rows + rows + r];
    const float w = mk == -INFINITY ? 0.f : __expf(__fsub_rn(mk, m));
    s = __fadd_rn(s, __fmul_rn(sk, w));
  }
  M[r] = m;
  S[r] = s;
}

struct PeerRegions {
  const uint8_t *r[8];  // rank j's exchange region (this rank's own at [rank])
};

// The row-sharded GEMV's exchange, launched right after the GEMV.
// griddepcontrol.wait: the local GEMV has finished, so this rank's rows are in
// its slot of y and of its exchange buffer e & 1 (e = *ctr + 1, the call
// number).  Thread 0 of CTA 0 publishes e in every other rank's flag for this
// rank (release, system scope: the rows are in this GPU's memory, where the
// other GPUs read them); thread 0 of each CTA waits (bounded) until every
// other rank has published e here, then the CTA reads those ranks' slots of
// their buffer e & 1 over NVLink into y.  A rank does not start call e + 2's
// GEMV (which rewrites buffer e & 1) before its exchange of call e + 1, which
// waits for this rank's flag of e + 1, published only after this kernel has
// finished.  The last CTA to finish (a ticket counter in this GPU's memory)
// sets *ctr = e.
__global__ void peer_gather_kernel(PeerRegions pr, int n, int rank, int64_t cap, int64_t n_local, float *y,
                                   uint64_t wait_ns, uint32_t *err) {
  pdl_launch_dependents();  // the next kernel may set up meanwhile; it waits for this one's end
  pdl_wait();
  unsigned long long *region = reinterpret_cast<unsigned long long *>(const_cast<uint8_t *>(pr.r[rank]));
  const unsigned long long *flags = region;
  unsigned long long *ctr = region + 9, *ticket = region + 10;
  const unsigned long long e = *reinterpret_cast<volatile unsigned long long *>(ctr) + 1;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    for (int j = 0; j < n; ++j)  // st.release orders the rows (visible here since griddepcontrol.wait) first
      if (j != rank) {
        unsigned long long *f = reinterpret_cast<unsigned long long *>(const_cast<uint8_t *>(pr.r[j])) + rank;
        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(f), "l"(e) : "memory");
      }
  }
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const uint64_t t0 = globaltimer_ns();
    for (int j = 0; j < n && ok; ++j) {
      if (j == rank) continue;
      for (uint32_t it = 1; ld_acquire_sys(flags + j) < e; ++it)
        if ((it & 63u) == 0 && globaltimer_ns() - t0 > wait_ns) {
          atomicOr(err, ERR_TIMEOUT);
          ok = 0;
          break;
        }
    }
  }
  __syncthreads();
  if (ok) {
    // remote reads cost a round trip over NVLink each: every thread issues
    // four 16-byte loads before it stores any (n_local % 4 == 0, y 16-byte
    // aligned and cap % 4 == 0; else one float at a time)
    const int64_t buf = (int64_t)(e & 1) * cap;
    const int64_t total = (int64_t)n * n_local, nth = (int64_t)gridDim.x * blockDim.x;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (n_local % 4 == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0) {
      const int64_t nv = total / 4;
      for (int64_t v0 = tid; v0 < nv; v0 += 4 * nth) {
        float4 r[4];
        bool use[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t v = v0 + u * nth;
          const int j = v < nv ? (int)(4 * v / n_local) : rank;
          use[u] = j != rank;
          if (use[u]) {
            const float *src = reinterpret_cast<const float *>(pr.r[j] + 256) + buf + 4 * v;
            asm volatile("ld.relaxed.sys.global.v4.f32 {%0, %1, %2, %3}, [%4];"
                         : "=f"(r[u].x), "=f"(r[u].y), "=f"(r[u].z), "=f"(r[u].w)
                         : "l"(src)
                         : "memory");
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (use[u]) reinterpret_cast<float4 *>(y)[v0 + u * nth] = r[u];
      }
    } else {
      for (int64_t i = tid; i < total; i += nth) {
        const int j = (int)(i / n_local);
        if (j != rank) {
          const float *src = reinterpret_cast<const float *>(pr.r[j] + 256) + buf + i;
          float v;
          asm volatile("ld.relaxed.sys.global.f32 %0, [%1];" : "=f"(v) : "l"(src) : "memory");
          y[i] = v;
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(ticket, 1ull) + 1 == gridDim.x) {  // every CTA has read ctr
      *ticket = 0;
      __threadfence();
      *ctr = e;
    }
  }
}

// This rank's n_local floats (the previous kernel's output) into its slot of
// y and of its exchange buffer for the coming exchange call (e = count of
// finished calls + 1, read after griddepcontrol.wait: the previous exchange
// kernel set it), ahead of peer_gather_kernel.  The vocab-sharded softmax and
// argmax send their per-row statistics and keys this way.
__global__ void peer_stage_kernel(const float *__restrict__ src, int64_t n_local, uint8_t *xbase, int64_t cap,
                                  int rank, float *__restrict__ y) {
  pdl_launch_dependents();
  pdl_wait();
  const unsigned long long e = *reinterpret_cast<volatile unsigned long long *>(xbase + 9 * 8) + 1;
  float *dst = reinterpret_cast<float *>(xbase + 256) + (int64_t)(e & 1) * cap + (int64_t)rank * n_local;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_local; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = src[i];
    dst[i] = v;
    y[(int64_t)rank * n_local + i] = v;
  }
}

// out[r] = the largest of the ranks' keys for row r (signed 64-bit order,
// as the all-reduce's ncclMax over ncclInt64)
__global__ void combine_keys_kernel(const int64_t *__restrict__ g, int n, int rows, int64_t *__restrict__ out) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  int64_t k = g[r];
  for (int j = 1; j < n; ++j) k = max(k, g[(int64_t)j * rows + r]);
  out[r] = k;
}

}  // namespace
}  // namespace tb

struct tb_shard_group_s {
  ncclComm_t comm = nullptr;
  int rank = 0, n = 1, device = 0;
  int64_t max_rows = 0;
  float *stats = nullptr;   // [2][max_rows]: this rank's m then s
  float *gathered = nullptr;  // [n][2][max_rows]
  float *gm = nullptr, *gs = nullptr;  // [max_rows] combined
  int64_t *keys = nullptr;  // [max_rows]
  double timeout_s = 30.0;
  // peer exchange (tb_shard_group_enable_peer): this rank's region holds, as
  // 64-bit words, the flags [0, 8) (per rank, the last call number it
  // published), this rank's count of finished calls [9] and the exchange
  // kernel's ticket counter [10]; from byte 256 two buffers of xcap floats
  // (calls alternate between them).  peer[j] maps rank j's region.
  uint8_t *xbase = nullptr;
  uint8_t *peer[8] = {};
  int64_t xcap = 0;
};

using namespace tb;

namespace {

// Waits (bounded) until a non-blocking communicator's last call has finished.
tb_status nccl_settle(NcclApi *api, ncclComm_t comm, ncclResult_t r, double timeout_s, const char *what) {
  const auto t0 = std::chrono::steady_clock::now();
  while (r == ncclInProgress) {
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s) {
      api->CommAbort(comm);
      return fail(TB_ETIMEOUT, "%s: no progress within %.1f s; communicator aborted", what, timeout_s);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(100));
    if (api->CommGetAsyncError(comm, &r) != ncclSuccess) break;
  }
  if (r != ncclSuccess) return fail(TB_ERUNTIME, "%s: %s", what, api->GetErrorString(r));
  return TB_OK;
}

// Stages n_local floats of this rank (src) and gathers every rank's into
// y[n][n_local] over NVLink peer memory (tb_shard_group_enable_peer).
tb_status peer_exchange(tb_shard_group g, const float *src, int64_t n_local, float *y, cudaStream_t s,
                        const char *who) {
  DeviceState *st;
  TB_TRY(device_state(&st));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, peer_stage_kernel, src, n_local, g->xbase, (int64_t)g->xcap, g->rank, y);
  if (e != cudaSuccess) return fail(TB_ECUDA, "%s (stage): %s", who, cudaGetErrorString(e));
  PeerRegions pr = {};
  for (int j = 0; j < g->n; ++j) pr.r[j] = j == g->rank ? g->xbase : g->peer[j];
  e = cudaLaunchKernelEx(&cfg, peer_gather_kernel, pr, g->n, g->rank, (int64_t)g->xcap, n_local, y,
                         (uint64_t)wait_limit_ns(), st->err_word);
  if (e != cudaSuccess) return fail(TB_ECUDA, "%s (exchange): %s", who, cudaGetErrorString(e));
  return check_launch(who);
}

tb_status check_group(tb_shard_group g, const char *who) {
  if (!g || !g->comm) return fail(TB_EINVAL, "%s: no shard group", who);
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != g->device)
    return fail(TB_EINVAL, "%s: the group's device %d is not the current device %d", who, g->device, dev);
  return TB_OK;
}

}  // namespace

extern "C" {

tb_status tb_shard_group_unique_id(void *id_out) {
  if (!id_out) return fail(TB_EINVAL, "tb_shard_group_unique_id: null pointer");
  NcclApi *api;
  TB_TRY(nccl_api(&api));
  ncclUniqueId id;
  ncclResult_t r = api->GetUniqueId(&id);
  if (r != ncclSuccess) return fail(TB_ERUNTIME, "ncclGetUniqueId: %s", api->GetErrorString(r));
  static_assert(sizeof(ncclUniqueId) == TB_SHARD_ID_BYTES, "NCCL unique id size");
  std::memcpy(id_out, &id, sizeof(id));
  return TB_OK;
}

tb_status tb_shard_group_create(int n_ranks, int rank, const void *id, int64_t max_rows, double timeout_s,
                                tb_shard_group *out) {
  if (!out || !id) return fail(TB_EINVAL, "tb_shard_group_create: null pointer");
  *out = nullptr;
  if (n_ranks < 1 || rank < 0 || rank >= n_ranks || max_rows < 1 || max_rows > (1 << 24) || !(timeout_s > 0))
    return fail(TB_EINVAL, "tb_shard_group_create: bad rank %d of %d, max_rows %lld or timeout", rank, n_ranks,
                (long long)max_rows);
  NcclApi *api;
  TB_TRY(nccl_api(&api));
  DeviceState *st;
  TB_TRY(device_state(&st));
  tb_shard_group g = new tb_shard_group_s();
  g->rank = rank;
  g->n = n_ranks;
  g->device = st->device;
  g->max_rows = max_rows;
  g->timeout_s = timeout_s;
  const size_t R = (size_t)max_rows;
  void *p = nullptr;
  tb_status s = tb_alloc(&p, sizeof(float) * R * (2 + 2 * (size_t)n_ranks + 2) + sizeof(int64_t) * R + 256);
  if (s != TB_OK) {
    delete g;
    return s;
  }
  g->stats = static_cast<float *>(p);
  g->gathered = g->stats + 2 * R;
  g->gm = g->gathered + 2 * R * (size_t)n_ranks;
  g->gs = g->gm + R;
  g->keys = reinterpret_cast<int64_t *>((reinterpret_cast<uintptr_t>(g->gs + R) + 255) & ~uintptr_t(255));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclResult_t r = api->CommInitRankConfig(&g->comm, n_ranks, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    tb_free(p);
    delete g;
    return fail(TB_ERUNTIME, "ncclCommInitRankConfig: %s", api->GetErrorString(r));
  }
  s = nccl_settle(api, g->comm, r, timeout_s, "tb_shard_group_create");
  if (s != TB_OK) {
    tb_free(p);
    delete g;
    return s;
  }
  *out = g;
  return TB_OK;
}

tb_status tb_shard_group_destroy(tb_shard_group g) {
  if (!g) return TB_OK;
  NcclApi *api;
  TB_TRY(nccl_api(&api));
  if (g->comm) {
    int dev = -1;
    cudaGetDevice(&dev);
    cudaSetDevice(g->device);
    api->CommDestroy(g->comm);
    cudaSetDevice(dev);
  }
  if (g->stats) tb_free(g->stats);
  if (g->xbase) {
    int dev = -1;
    cudaGetDevice(&dev);
    cudaSetDevice(g->device);
    cudaDeviceSynchronize();  // this rank's stores into the peers have landed
    for (int j = 0; j < g->n; ++j)
      if (g->peer[j]) cudaIpcCloseMemHandle(g->peer[j]);
    cudaFree(g->xbase);
    cudaSetDevice(dev);
  }
  delete g;
  return TB_OK;
}

tb_status tb_shard_group_enable_peer(tb_shard_group g, int64_t max_elems) {
  TB_TRY(check_group(g, "tb_shard_group_enable_peer"));
  if (max_elems < 1 || max_elems > (int64_t(1) << 28))
    return fail(TB_EINVAL, "tb_shard_group_enable_peer: max_elems %lld out of range", (long long)max_elems);
  if (g->n > 8) return fail(TB_EINVAL, "tb_shard_group_enable_peer: %d ranks (at most 8)", g->n);
  if (g->xbase) return fail(TB_EINVAL, "tb_shard_group_enable_peer: already enabled");
  if (g->n == 1) return TB_OK;  // nothing to exchange
  NcclApi *api;
  TB_TRY(nccl_api(&api));
  const int64_t cap = (max_elems + 3) / 4 * 4;  // 16-byte aligned buffers
  const size_t bytes = 256 + 2 * (size_t)cap * sizeof(float);
  uint8_t *base = nullptr;
  cudaError_t e = cudaMalloc(reinterpret_cast<void **>(&base), bytes);
  if (e != cudaSuccess) return fail(TB_ENOMEM, "tb_shard_group_enable_peer: %s", cudaGetErrorString(e));
  uint8_t *hb = nullptr;  // the ranks' IPC handles, gathered
  tb_status rs = TB_OK;
  uint8_t *opened[8] = {};
  cudaIpcMemHandle_t h;
  std::vector<uint8_t> all((size_t)g->n * sizeof(h));
  e = cudaMemset(base, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, base);
  if (e != cudaSuccess) rs = fail(TB_ECUDA, "tb_shard_group_enable_peer: %s", cudaGetErrorString(e));
  if (rs == TB_OK) rs = tb_alloc(reinterpret_cast<void **>(&hb), all.size());
  if (rs == TB_OK) rs = tb_upload(hb + (size_t)g->rank * sizeof(h), &h, sizeof(h), nullptr);
  if (rs == TB_OK) {
    ncclResult_t r = api->AllGather(hb + (size_t)g->rank * sizeof(h), hb, sizeof(h), ncclUint8, g->comm, nullptr);
    rs = nccl_settle(api, g->comm, r, g->timeout_s, "tb_shard_group_enable_peer(all-gather)");
  }
  if (rs == TB_OK) rs = tb_download(all.data(), hb, all.size(), nullptr);
  if (rs == TB_OK) rs = tb_sync(nullptr);
  for (int j = 0; j < g->n && rs == TB_OK; ++j) {
    if (j == g->rank) continue;
    cudaIpcMemHandle_t hj;
    std::memcpy(&hj, all.data() + (size_t)j * sizeof(h), sizeof(h));
    e = cudaIpcOpenMemHandle(reinterpret_cast<void **>(&opened[j]), hj, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess)
      rs = fail(TB_ECUDA, "tb_shard_group_enable_peer: mapping rank %d's buffer: %s (one process per GPU, peer "
                "access between the GPUs)", j, cudaGetErrorString(e));
  }
  if (hb) tb_free(hb);
  if (rs != TB_OK) {
    for (int j = 0; j < g->n; ++j)
      if (opened[j]) cudaIpcCloseMemHandle(opened[j]);
    cudaFree(base);
    return rs;
  }
  g->xbase = base;
  for (int j = 0; j < g->n; ++j) g->peer[j] = opened[j];
  g->xcap = cap;
  return TB_OK;
}

tb_status tb_shard_group_abort(tb_shard_group g) {
  if (!g || !g->comm) return fail(TB_EINVAL, "tb_shard_group_abort: no shard group");
  NcclApi *api;
  TB_TRY(nccl_api(&api));
  api->CommAbort(g->comm);
  g->comm = nullptr;
  return TB_OK;
}

tb_status tb_shard_group_wait(tb_shard_group g, tb_stream stream, double timeout_s) {
  TB_TRY(check_group(g, "tb_shard_group_wait"));
  NcclApi *api;
  TB_TRY(nccl_api(&api));
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaStreamQuery(as_stream(stream));
    if (e == cudaSuccess) return TB_OK;
    if (e != cudaErrorNotReady) return fail(TB_ECUDA, "tb_shard_group_wait: %s", cudaGetErrorString(e));
    ncclResult_t ar = ncclSuccess;
    api->CommGetAsyncError(g->comm, &ar);
    if (ar != ncclSuccess && ar != ncclInProgress) {
      api->CommAbort(g->comm);
      g->comm = nullptr;
      return fail(TB_ERUNTIME, "tb_shard_group_wait: %s; communicator aborted", api->GetErrorString(ar));
    }
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s) {
      api->CommAbort(g->comm);
      g->comm = nullptr;
      return fail(TB_ETIMEOUT, "tb_shard_group_wait: the stream did not finish within %.1f s; communicator aborted",
                  timeout_s);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

tb_status tb_softmax_vocab_sharded(tb_shard_group g, const float *x_dev, int64_t rows, int64_t cols, int64_t ld,
                                   float *y_dev, int64_t ld_y, tb_stream stream) {
  TB_TRY(check_group(g, "tb_softmax_vocab_sharded"));
  if (rows < 0 || rows > g->max_rows) return fail(TB_EINVAL, "tb_softmax_vocab_sharded: rows %lld above the group's %lld",
                                                  (long long)rows, (long long)g->max_rows);
  if (rows == 0) return TB_OK;
  NcclApi *api;
  TB_TRY(nccl_api(&api));
  cudaStream_t s = as_stream(stream);
  TB_TRY(tb_softmax_shard_stats(x_dev, rows, cols, ld, g->stats, g->stats + rows, stream));
  const float *gm = g->stats, *gs = g->stats + rows;
  if (g->n > 1) {
    if (g->xbase && (int64_t)g->n * 2 * rows <= g->xcap) {  // the (m, s) pairs over NVLink peer memory
      TB_TRY(peer_exchange(g, g->stats, 2 * rows, g->gathered, s, "tb_softmax_vocab_sharded"));
    } else {
      ncclResult_t r = api->AllGather(g->stats, g->gathered, (size_t)(2 * rows), ncclFloat32, g->comm, s);
      TB_TRY(nccl_settle(api, g->comm, r, g->timeout_s, "tb_softmax_vocab_sharded(all-gather)"));
    }
    combine_stats_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, s>>>(g->gathered, g->n, (int)rows, g->gm, g->gs);
    TB_TRY(check_launch("tb_softmax_vocab_sharded"));
    gm = g->gm;
    gs = g->gs;
  }
  return tb_softmax_shard_finish(x_dev, rows, cols, ld, gm, gs, y_dev, ld_y, stream);
}

tb_status tb_argmax_vocab_sharded(tb_shard_group g, const float *x_dev, int64_t rows, int64_t cols, int64_t ld,
                                  int64_t col_base, int64_t *idx_dev, tb_stream stream) {
  TB_TRY(check_group(g, "tb_argmax_vocab_sharded"));
  if (rows < 0 || rows > g->max_rows) return fail(TB_EINVAL, "tb_argmax_vocab_sharded: rows %lld above the group's %lld",
                                                  (long long)rows, (long long)g->max_rows);
  if (rows == 0) return TB_OK;
  NcclApi *api;
  TB_TRY(nccl_api(&api));
  TB_TRY(tb_argmax_shard_keys(x_dev, rows, cols, ld, col_base, g->keys, stream));
  if (g->n > 1) {
    if (g->xbase && (int64_t)g->n * 2 * rows <= g->xcap) {  // the keys over NVLink peer memory
      int64_t *all = reinterpret_cast<int64_t *>(g->gathered);  // [n][rows] keys
      TB_TRY(peer_exchange(g, reinterpret_cast<const float *>(g->keys), 2 * rows, g->gathered, as_stream(stream),
                           "tb_argmax_vocab_sharded"));
      combine_keys_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, as_stream(stream)>>>(all, g->n, (int)rows,
                                                                                          g->keys);
      TB_TRY(check_launch("tb_argmax_vocab_sharded"));
    } else {
      ncclResult_t r = api->AllReduce(g->keys, g->keys, (size_t)rows, ncclInt64, ncclMax, g->comm, as_stream(stream));
      TB_TRY(nccl_settle(api, g->comm, r, g->timeout_s, "tb_argmax_vocab_sharded(all-reduce)"));
    }
  }
  return tb_argmax_key_index(g->keys, rows, idx_dev, stream);
}

tb_status tb_gemv_q8_0_row_sharded(tb_shard_group g, const float *x_dev, int64_t K, const void *w_local_dev,
                                   int64_t n_local, float *y_dev, tb_stream stream) {
  TB_TRY(check_group(g, "tb_gemv_q8_0_row_sharded"));
  if (n_local <= 0 || K <= 0) return fail(TB_EINVAL, "tb_gemv_q8_0_row_sharded: bad extents");
  float *slot = y_dev + (int64_t)g->rank * n_local;
  if (g->n > 1 && g->xbase && (int64_t)g->n * n_local <= g->xcap) {
    DeviceState *st;
    TB_TRY(device_state(&st));
    cudaStream_t s = as_stream(stream);
    PeerOut po = {};
    po.dst = reinterpret_cast<float *>(g->xbase + 256) + (int64_t)g->rank * n_local;
    po.ctr = reinterpret_cast<const unsigned long long *>(g->xbase) + 9;
    po.par_stride = g->xcap;
    TB_TRY(launch_q8_0_gemv_peer(x_dev, K, w_local_dev, n_local, slot, po, s, st));
    PeerRegions pr = {};
    for (int j = 0; j < g->n; ++j) pr.r[j] = j == g->rank ? g->xbase : g->peer[j];
    const int64_t total = (int64_t)g->n * n_local;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::min<int64_t>(64, std::max<int64_t>(1, total / 4096)), 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, peer_gather_kernel, pr, g->n, g->rank, (int64_t)g->xcap,
                                       (int64_t)n_local, y_dev, (uint64_t)wait_limit_ns(), st->err_word);
    if (e != cudaSuccess) return fail(TB_ECUDA, "tb_gemv_q8_0_row_sharded (exchange): %s", cudaGetErrorString(e));
    return check_launch("tb_gemv_q8_0_row_sharded (exchange)");
  }
  NcclApi *api;
  TB_TRY(nccl_api(&api));
  TB_TRY(tb_matmul_quant(TB_Q8_0, x_dev, 1, K, w_local_dev, n_local, slot, stream));
  if (g->n > 1) {
    ncclResult_t r = api->AllGather(slot, y_dev, (size_t)n_local, ncclFloat32, g->comm, as_stream(stream));
    TB_TRY(nccl_settle(api, g->comm, r, g->timeout_s, "tb_gemv_q8_0_row_sharded(all-gather)"));
  }
  return TB_OK;
}

}  // extern "C"
