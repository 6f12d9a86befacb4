/* turbo_b200.h -- C ABI of the B200 (sm_100a) tensor-library hot path.
 *
 * This is the drop-in boundary under the Turbo.cpp `Tensor`/`Storage` API
 * (include/turbo/tensor/tensor.hpp) and the `nn` layers' forward call sites
 * (the files under src/nn).  Every entry point replaces one reference interface, cited
 * beside it as file:line inside the reference project.
 *
 * Conventions
 *  - Plain pointers and sizes only.  Pointers named `*_dev` or held in a
 *    tb_view are device (HBM) addresses; everything else is host memory.
 *  - Offsets and strides are in ELEMENTS, as in the reference `Tensor`
 *    (tensor.hpp:98-101).  Strides may be 0 (broadcast views).
 *  - Every op is asynchronous on `stream` (a cudaStream_t; NULL = legacy
 *    default stream) and returns a status.  TB_EINVAL / TB_ERANGE /
 *    TB_ERUNTIME correspond to the reference's std::invalid_argument /
 *    std::out_of_range / std::runtime_error; the host C++ layer rethrows them
 *    as those types.  tb_last_error() gives the message of the calling
 *    thread's last failure.
 *  - Calls act on the current CUDA device of the calling thread.
 *  - No entry point falls back to the CPU: when the CUDA library cannot run,
 *    the call fails with TB_ECUDA.
 */
#ifndef TURBO_B200_H
#define TURBO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden visibility; only this header's entry
 * points are exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef enum {
  TB_OK = 0,
  TB_EINVAL = 1,   /* std::invalid_argument in the reference */
  TB_ERANGE = 2,   /* std::out_of_range */
  TB_ERUNTIME = 3, /* std::runtime_error */
  TB_ECUDA = 4,    /* CUDA launch or runtime failure */
  TB_ETIMEOUT = 5, /* a bounded device-side wait gave up */
  TB_ENOMEM = 6    /* device arena exhausted */
} tb_status;

/* Element types.  Values 0..4 are the reference DataType enum in order
 * (include/turbo/tensor/tensor.hpp:10-16); BF16 is added for the sweep. */
typedef enum {
  TB_F32 = 0,
  TB_F16 = 1,
  TB_Q8_0 = 2, /* 34-byte blocks of 32: {u16 half d; i8 q[32]} (quant_types.hpp:17-20) */
  TB_Q4_0 = 3, /* 18-byte blocks of 32: {u16 half d; u8 q[16]} (quant_types.hpp:32-35) */
  TB_I32 = 4,
  TB_BF16 = 5
} tb_dtype;

#define TB_MAX_RANK 8

/* A strided view over device memory: element (i0, .., ir-1) is at
 * data + (offset + sum_k i_k * strides[k]) * sizeof(element).
 * Mirrors Tensor{storage, offset, shape, strides} (tensor.hpp:96-104). */
typedef struct {
  void *data;
  int32_t dtype;
  int32_t rank;
  int64_t offset;
  int64_t shape[TB_MAX_RANK];
  int64_t strides[TB_MAX_RANK];
} tb_view;

typedef void *tb_stream; /* cudaStream_t */

/* ---------------------------------------------------------------- runtime -- */

/* Binds the calling thread to `device` and creates its per-device state
 * (error word, arena).  Replaces nothing in the reference (CPU only); called
 * implicitly by every entry point for the current device. */
tb_status tb_init(int device);
const char *tb_last_error(void);
const char *tb_status_name(tb_status s);
/* Version string of this library (build date and arch). */
const char *tb_version(void);

/* Device arena: Storage(size_t) (tensor.hpp:59-64) gains HBM backing.
 * 256-byte aligned; tb_free returns the block to the arena. */
tb_status tb_alloc(void **ptr_dev, size_t bytes);
tb_status tb_free(void *ptr_dev);
/* Host <-> device copies: the mmap constructor Storage(void*, size_t)
 * (tensor.hpp:76-77) uploads weights once; data_ptr() reads back.
 * Asynchronous on `stream`.  Page-locked host buffers of up to 256 KB whose
 * address and size are multiples of 16 bytes are copied by a kernel through
 * the buffer's device mapping (a few microseconds less per call than a DMA
 * copy, and the next kernel may start behind it); the host buffer must stay
 * valid until the stream reaches the copy.  Other buffers use DMA. */
tb_status tb_upload(void *dst_dev, const void *src_host, size_t bytes, tb_stream stream);
tb_status tb_download(void *dst_host, const void *src_dev, size_t bytes, tb_stream stream);
tb_status tb_memset(void *dst_dev, int value, size_t bytes, tb_stream stream);
tb_status tb_sync(tb_stream stream);
/* Reads and clears the device error word set by bounded waits and by
 * device-side index checks (bit 0: timeout, bit 1: index out of range). */
tb_status tb_take_device_errors(uint32_t *flags_out);
/* Limit, in nanoseconds, of the bounded waits of the Q4_0 matmul kernels
 * (tb_matmul_quant / tb_matmul_quant_exact with TB_Q4_0 on the CUDA cores, and
 * tb_matmul_q4_0_static_scratch); default 2e9.  A wait that gives up sets bit 0
 * of the device error word and the kernel leaves its rows unwritten, after
 * waiting for its own copies in flight.  0 lets no wait wait at all, a
 * host-side way to exercise that path.  Read at launch (a captured graph keeps
 * the value it was captured with).  No reference counterpart. */
tb_status tb_set_wait_limit_ns(uint64_t ns);

/* ------------------------------------------------------ elementwise (A3-A8) -- */

/* out = broadcast(a) OP broadcast(b), written contiguously in the broadcast
 * shape.  op 0 = add: Tensor::operator+ (src/tensor/tensor.cpp:260-282) with
 * compute_broadcast_shape (:29-47) and broadcast_to (:232-256); op 1 = mul
 * (the row-broadcast multiply of the sharded sweep).  fp32, or bf16 when all
 * three views are bf16.  `out` must be contiguous with the broadcast shape. */
tb_status tb_binary(int op, const tb_view *a, const tb_view *b, const tb_view *out,
                    tb_stream stream);

/* out = x * s: Tensor::operator*(float) (src/tensor/tensor.cpp:284-294);
 * `out` contiguous of x's shape. */
tb_status tb_scale(const tb_view *x, float s, const tb_view *out, tb_stream stream);

/* dst <- src elementwise, shapes equal: Tensor::copy_ (src/tensor/tensor.cpp:689-726)
 * and, with a contiguous dst, Tensor::contiguous (:118-132). */
tb_status tb_copy(const tb_view *dst, const tb_view *src, tb_stream stream);

/* y = x / sqrt(mean(x^2) + eps) * gamma over rows of `cols` contiguous
 * elements: nn::RMSNorm::forward (src/nn/rmsnorm.cpp:23-68).  dtype TB_F32 or
 * TB_BF16 for x/y (gamma is fp32, as the reference requires). */
tb_status tb_rmsnorm(int dtype, const void *x_dev, const float *gamma_dev, void *y_dev,
                     int64_t rows, int64_t cols, float eps, tb_stream stream);

/* y = g / (1 + exp(-g)) * u: nn::SwiGLU::forward(gate, up) (src/nn/swiglu.cpp:10-40).
 * dtype TB_F32 or TB_BF16. */
tb_status tb_swiglu(int dtype, const void *g_dev, const void *u_dev, void *y_dev, int64_t n,
                    tb_stream stream);

/* ------------------------------------------------------- rows (A9, A15) -- */

/* Last-dim softmax of x[rows, cols] (contiguous): nn::Softmax::forward
 * (src/nn/softmax.cpp:13-54). */
tb_status tb_softmax(const float *x_dev, float *y_dev, int64_t rows, int64_t cols,
                     tb_stream stream);

/* Per row, index of the first maximum under a strict '>' from -inf (NaN never
 * wins; a row of only -inf/NaN gives 0): greedy_sample (src/core/sampler.cpp:13-26). */
tb_status tb_argmax(const float *x_dev, int64_t rows, int64_t cols, int64_t *idx_dev,
                    tb_stream stream);

/* Nucleus (top-p) sampling of one row of logits: sample_top_p
 * (src/core/sampler.cpp:28-86).  Probabilities softmax(logits / temperature),
 * ordered by descending probability (equal ones by ascending id); the prefix
 * ends at the first position whose cumulative probability reaches top_p; the
 * result is the first prefix position whose cumulative mass reaches u times
 * the prefix mass, i.e. std::discrete_distribution's draw for the uniform
 * number u in [0, 1), which the caller supplies (the reference draws it from a
 * random_device-seeded mt19937).  Prefix sums are exact (integer masses
 * floor(p * 2^62)); the result differs from a reference draw with the same u
 * only where top_p or u lies within fp32 rounding of a prefix boundary.  With
 * no positive finite probability (a NaN or +inf logit) *out_dev is the first
 * maximum, as greedy_sample.  temperature must be > 0; vocab at most what a
 * 16-CTA cluster holds in shared memory (about 500k).  One cluster launch, no
 * allocation; *out_dev is written on the device. */
tb_status tb_sample_top_p(const float *logits_dev, int64_t vocab, float temperature, float top_p,
                          double u, int32_t *out_dev, tb_stream stream);
/* The same draw with the uniform number read on the device, u_dev[*pos_dev]
 * (the position clamped into [0, max_seq)), and the id written as int64 to
 * *idx_dev -- the slot tb_argmax fills -- so that a decode step recorded in a
 * CUDA graph samples each token with the uniform number of its position. */
tb_status tb_sample_top_p_at(const float *logits_dev, int64_t vocab, float temperature, float top_p,
                             const double *u_dev, const int32_t *pos_dev, int64_t max_seq, int64_t *idx_dev,
                             tb_stream stream);

/* Causal mask of the prefill attention scores (src/nn/attention.cpp:120-129):
 * x[r, c] = value wherever c > r + diag_offset, for x[rows, cols] with row
 * stride ld (elements). */
tb_status tb_fill_upper(float *x_dev, int64_t rows, int64_t cols, int64_t ld, int64_t diag_offset,
                        float value, tb_stream stream);

/* ------------------------------------------------------------- RoPE (A13) -- */

/* Rotate-half RoPE in place on a rank-2 [S, D] or rank-4 [B, H, S, D] fp32
 * view, positions pos_offset..pos_offset+S-1, using the constructor's tables
 * cos/sin[max_seq, D/2] (uploaded once): RoPE::apply_in_place
 * (src/nn/rope.cpp:35-103).  TB_ERANGE if a position reaches max_seq. */
tb_status tb_rope(const tb_view *x, const float *cos_dev, const float *sin_dev,
                  int64_t head_dim, int64_t max_seq, int64_t pos_offset, tb_stream stream);

/* --------------------------------------------------- quant formats (A14, A17) -- */

/* Exact dequantisation of `nblocks` consecutive blocks to fp32 (q*d, or
 * (nibble-8)*d): dequantize_row_q8_0 (src/tensor/quant_math.hpp:16-29) and the
 * Q4_0 unpacking of src/nn/embedding.cpp:54-63. */
tb_status tb_dequant(int dtype, const void *blocks_dev, int64_t nblocks, float *y_dev,
                     tb_stream stream);

/* Rows of fp32 x[rows, k] to Q8_0 blocks: quantize_row_q8_0
 * (src/tensor/quant_math.hpp:68-90), bit for bit. */
tb_status tb_quantize_q8_0(const float *x_dev, int64_t rows, int64_t k, void *blocks_dev,
                           tb_stream stream);

/* Token-row gather with exact dequantisation: nn::Embedding::forward
 * (src/nn/embedding.cpp:22-118).  The weight has GGUF logical shape
 * {dim, vocab} (dtype TB_F32, TB_Q8_0 or TB_Q4_0); ids are device int32.
 * ids are checked on the device: a row with id outside [0, vocab) is written
 * as zeros and sets bit 1 of the device error word (tb_take_device_errors);
 * callers holding host ids check them first (TB_ERANGE), as the host layer does. */
tb_status tb_embedding(int dtype, const void *w_dev, int64_t dim, int64_t vocab,
                       const int32_t *ids_dev, int64_t n, float *out_dev, tb_stream stream);

/* ------------------------------------------------------------- matmul (A10-A12) -- */

/* Y[M, N] = X[M, K] . W for a quantized W of GGUF logical shape {K, N}, stored
 * as N rows of K/32 blocks (Tensor::matmul, src/tensor/tensor.cpp:328-432).
 *  - dtype TB_Q8_0: X is fp32 and is not quantized (tensor.cpp:370-381).  The
 *    decode GEMV (M == 1) accumulates each block as an FMA chain and applies
 *    the block scale once: within 1e-5 relative of vec_dot_q8_0_f32
 *    (quant_math.hpp:32-60), typically ~1e-7.
 *  - dtype TB_Q4_0: X rows are first quantized to Q8_0 (tensor.cpp:413-421),
 *    bit for bit, then multiplied with the Q4_0 rows in the order of
 *    vec_dot_q4_0_q8_0_avx2 (quant_math.hpp:184-248).
 *  - M >= 32 with K a multiple of 256 and 16-byte aligned X and W runs on the
 *    tensor cores (both dtypes): per 256-wide K chunk, w = q d (with X as
 *    Q8_0, q_x d_x, for TB_Q4_0) held exactly as two fp16 values, three fp16
 *    products per pair accumulated in fp32 tensor memory, chunk sums added
 *    in fp32 -- within 1e-5 of sum |w x| per output, typically 1e-7 to 6e-7;
 *    it allocates stream-ordered scratch for the packed operands.
 * K must be a multiple of 32. */
tb_status tb_matmul_quant(int dtype, const float *x_dev, int64_t M, int64_t K,
                          const void *w_dev, int64_t N, float *y_dev, tb_stream stream);

/* As tb_matmul_quant, but every output is computed in the reference's exact
 * operation order, so results are bit-identical to Tensor::matmul
 * (src/tensor/tensor.cpp:328-432, quant_math.hpp:32-60 and 184-248). */
tb_status tb_matmul_quant_exact(int dtype, const float *x_dev, int64_t M, int64_t K,
                                const void *w_dev, int64_t N, float *y_dev, tb_stream stream);

/* tb_matmul_quant(TB_Q4_0, ...) for callers that cannot allocate device memory
 * during the call (a process that reserves its whole device-memory budget at
 * start-up, or a latency-critical loop where an allocator call may synchronize
 * or fail).  No counterpart in the reference, which runs on the CPU.
 * The quantized copy of X goes to a fixed 8 MiB buffer compiled into the
 * library (held on every GPU that loads it until the process exits) instead
 * of allocated scratch; results are identical to tb_matmul_quant_exact(TB_Q4_0)
 * (the reference's summation order), and so to tb_matmul_quant(TB_Q4_0) on
 * every shape that entry does not send to the tensor cores (M < 32). 
 * Requires M * (K/32) * 34 <= 8 MiB (e.g. M = 512 at K = 8192), else TB_EINVAL.
 * Calls no cudaMalloc/cudaFree.  The first call on a device looks up the
 * buffer's address (cudaGetSymbolAddress); make it before any stream capture.
 * All calls share the one buffer: calls that may overlap on the GPU (other
 * streams, other host threads) race and must be serialized by the caller.
 * A bounded wait that gives up inside the kernel sets bit 0 of this entry
 * point's own device error word (also a file-scope device variable), which
 * tb_take_device_errors reads and clears with the regular one. */
tb_status tb_matmul_q4_0_static_scratch(const float *x_dev, int64_t M, int64_t K,
                                        const void *w_dev, int64_t N, float *y_dev,
                                        tb_stream stream);

/* Weights packed once for the tensor-core matmul (M >= 32), so a prefill
 * that multiplies by the same W many times does not convert it on every
 * call.  No counterpart in the reference (its matmul reads the GGUF blocks
 * directly, src/tensor/tensor.cpp:328-432); tb_matmul_quant packs W into
 * scratch on every call and is otherwise the same computation.
 * The packed form holds, per 128 rows x 256 K, the products q * d as two
 * fp16 planes scaled by a power of two (4 bytes per weight), plus the scales:
 * about 7x the Q4_0 bytes, 3.8x the Q8_0 bytes.
 *  - tb_packed_quant_weights_bytes: the size for N rows of K (K a positive
 *    multiple of 256, at most 2^20; dtype TB_Q8_0 or TB_Q4_0), else TB_EINVAL.
 *  - tb_pack_quant_weights: W (N rows of K/32 blocks, 16-byte aligned) into
 *    `packed_dev` (16-byte aligned, at least that many bytes), on `stream`.
 *    The packed copy does not follow later changes of W.
 *  - tb_matmul_quant_packed: Y[M, N] = X[M, K] . W from the packed copy, M >=
 *    32 (TB_EINVAL below: those shapes belong to tb_matmul_quant), the same
 *    dtype as packed (it decides how X is treated: TB_Q4_0 quantizes X rows
 *    to Q8_0 first).  Results are identical to tb_matmul_quant on the same
 *    arguments. */
tb_status tb_packed_quant_weights_bytes(int dtype, int64_t N, int64_t K, size_t *bytes);
tb_status tb_pack_quant_weights(int dtype, const void *w_dev, int64_t N, int64_t K, void *packed_dev,
                                size_t packed_bytes, tb_stream stream);
tb_status tb_matmul_quant_packed(int dtype, const float *x_dev, int64_t M, int64_t K,
                                 const void *packed_dev, int64_t N, float *y_dev, tb_stream stream);

/* Batched strided fp32 matmul, out = a @ b over matching leading (batch) dims,
 * `out` contiguous [batch..., M, N]: Tensor::matmul fp32 branch
 * (src/tensor/tensor.cpp:434-542) and matmul_threaded_packed_avx2 (:591-650).
 * Each output is the FMA chain over k in increasing order, as the reference. */
tb_status tb_matmul_f32(const tb_view *a, const tb_view *b, const tb_view *out,
                        tb_stream stream);

/* --------------------------------------- vocab-sharded softmax / argmax (8e) -- */

/* Local half of a softmax whose columns are split across GPUs: per row of this
 * shard's x[rows, cols] (row stride ld), the shard maximum and the sum of
 * exp(x - shard maximum).  Combined across shards by a max and a sum
 * all-reduce, then tb_softmax_shard_finish writes exp(x - M) / S. */
tb_status tb_softmax_shard_stats(const float *x_dev, int64_t rows, int64_t cols, int64_t ld,
                                 float *row_max_dev, float *row_sum_dev, tb_stream stream);
/* Given the local stats and the global row maxima, rescales the local sums in
 * place: sum_dev[r] *= exp(local_max[r] - global_max[r]). */
tb_status tb_softmax_shard_rescale(const float *local_max_dev, const float *global_max_dev,
                                   float *row_sum_dev, int64_t rows, tb_stream stream);
tb_status tb_softmax_shard_finish(const float *x_dev, int64_t rows, int64_t cols, int64_t ld,
                                  const float *global_max_dev, const float *global_sum_dev,
                                  float *y_dev, int64_t ld_y, tb_stream stream);
/* Per row of this shard, a 64-bit key that orders candidates the way
 * greedy_sample (src/core/sampler.cpp:13-26) does: (order-preserving bits of the
 * value) << 32 | (0xFFFFFFFF - global column), with the top bit flipped so that
 * the keys compare as signed int64.  A signed int64 MAX all-reduce of the keys
 * across shards (ncclInt64/ncclMax) gives the global first maximum;
 * tb_argmax_key_index decodes it.  A row with no candidate (all NaN or -inf)
 * gets INT64_MIN, which decodes to index 0. */
tb_status tb_argmax_shard_keys(const float *x_dev, int64_t rows, int64_t cols, int64_t ld,
                               int64_t col_base, int64_t *keys_dev, tb_stream stream);
tb_status tb_argmax_key_index(const int64_t *keys_dev, int64_t rows, int64_t *idx_dev,
                              tb_stream stream);

/* A group of n_ranks GPUs, one per process or thread, for the shard-level ops
 * below (the reference runs them whole on one CPU: src/nn/softmax.cpp:13-54,
 * src/core/sampler.cpp:13-26, src/tensor/tensor.cpp:328-382).  Rank 0 makes
 * an id (tb_shard_group_unique_id), the caller passes it to every rank, and
 * each rank calls tb_shard_group_create with its device current.  The
 * exchange is NCCL over NVLink, loaded at run time (libnccl.so.2).  Creation
 * is bounded by timeout_s (TB_ETIMEOUT, communicator aborted);  max_rows
 * bounds the rows of later calls.  Every rank issues the same calls in the
 * same order; they are asynchronous on `stream`.  tb_shard_group_wait waits
 * at most timeout_s for a stream's work and aborts the group otherwise (a
 * rank that never joins a collective cannot hang the others past it). */
#define TB_SHARD_ID_BYTES 128
typedef struct tb_shard_group_s *tb_shard_group;
tb_status tb_shard_group_unique_id(void *id_out);
tb_status tb_shard_group_create(int n_ranks, int rank, const void *id, int64_t max_rows, double timeout_s,
                                tb_shard_group *out);
tb_status tb_shard_group_wait(tb_shard_group group, tb_stream stream, double timeout_s);
tb_status tb_shard_group_abort(tb_shard_group group);
tb_status tb_shard_group_destroy(tb_shard_group group);
/* Lets the group's ranks store into one another's memory over NVLink (no
 * counterpart in the reference): every rank allocates an exchange buffer for
 * up to max_elems floats (twice, plus 256 bytes of flags) and maps the other
 * ranks' buffers through CUDA IPC handles, exchanged with one all-gather.
 * Collective (every rank calls it); needs one process per GPU and peer access
 * between the GPUs, else an error and the group keeps using NCCL.  A group of
 * one rank needs nothing (TB_OK).  Afterwards tb_gemv_q8_0_row_sharded with
 * n_ranks * n_local <= max_elems exchanges through these buffers. */
tb_status tb_shard_group_enable_peer(tb_shard_group group, int64_t max_elems);
/* Softmax over rows split by columns: this rank holds x[rows, cols] (row
 * stride ld), its slice of the full rows; y (row stride ld_y) gets the same
 * slice of the full rows' softmax.  One all-gather of each rank's per-row
 * (max, sum of exp) and a combine in rank order; then exp(x - M) / S. */
tb_status tb_softmax_vocab_sharded(tb_shard_group group, const float *x_dev, int64_t rows, int64_t cols,
                                   int64_t ld, float *y_dev, int64_t ld_y, tb_stream stream);
/* greedy_sample over rows split by columns: this rank's columns start at
 * global column col_base; idx_dev[rows] gets the global first-maximum column
 * on every rank (one int64 MAX all-reduce of tb_argmax_shard_keys). */
tb_status tb_argmax_vocab_sharded(tb_shard_group group, const float *x_dev, int64_t rows, int64_t cols,
                                  int64_t ld, int64_t col_base, int64_t *idx_dev, tb_stream stream);
/* Tensor-parallel Q8_0 GEMV (Tensor::matmul, src/tensor/tensor.cpp:328-382,
 * rows split): this rank holds rows [rank n_local, (rank + 1) n_local) of W
 * (their Q8_0 blocks) and the full x[K]; y_dev[n_ranks * n_local] gets the
 * full product on every rank.  Every rank passes the same n_local.  With NCCL:
 * the rank's rows, then one in-place all-gather.  After
 * tb_shard_group_enable_peer (and n_ranks * n_local within its max_elems):
 * the GEMV kernel also writes its rows into this GPU's exchange buffer; then a
 * kernel on each rank publishes the call's number to the other ranks, waits
 * for theirs (bounded by tb_set_wait_limit_ns: on expiry bit 0 of the device
 * error word is set and y keeps the old values of those rows) and reads their
 * rows from their exchange buffers over NVLink into y.  No host work per call,
 * so the calls can be captured in a CUDA graph.  Calls of one group go in
 * order on one stream per rank.  W and x 16-byte aligned, K a multiple of 256
 * on that path. */
tb_status tb_gemv_q8_0_row_sharded(tb_shard_group group, const float *x_dev, int64_t K, const void *w_local_dev,
                                   int64_t n_local, float *y_dev, tb_stream stream);

/* ------------------------------------------- decode step with a device position -- */

/* tb_rope with the position offset read from device memory (*pos_dev) when
 * the kernel runs, so a decode step can be captured once and replayed.  A
 * position outside the table sets bit 1 of the device error word and leaves x
 * unchanged (tb_rope itself returns TB_ERANGE, rope.cpp:58-61). */
tb_status tb_rope_at(const tb_view *x, const float *cos_dev, const float *sin_dev, int64_t head_dim,
                     int64_t max_seq, const int32_t *pos_dev, tb_stream stream);
/* One token's K and V rows into the layer caches [max_seq, row_elems] at row
 * *pos_dev: the cache writes of src/nn/attention.cpp:66-84 for S = 1. */
tb_status tb_kv_append(float *k_cache_dev, float *v_cache_dev, const float *k_dev, const float *v_dev,
                       int64_t row_elems, int64_t max_seq, const int32_t *pos_dev, tb_stream stream);
/* All query heads of one token against the caches' first *pos_dev + 1 rows
 * (src/nn/attention.cpp:104-141 with S = 1; no mask applies): per head, scores
 * as the fp32 matmul computes them (fma chain over head_dim) times scale,
 * softmax as tb_softmax, then probabilities x V.  q [heads, head_dim], caches
 * [max_seq, kv_heads, head_dim], out [heads, head_dim]; head_dim 64. */
tb_status tb_attention_decode(const float *q_dev, const float *k_cache_dev, const float *v_cache_dev,
                              int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t max_seq, float scale,
                              const int32_t *pos_dev, float *out_dev, tb_stream stream);
/* tb_rope_kv_append followed by tb_attention_decode, in one launch: q [heads,
 * head_dim] and k [kv_heads, head_dim] are rotated at position *pos_dev
 * inside the attention kernel (q_dev and k_dev are not modified), the rotated
 * k and v are appended to the caches' row *pos_dev, and out holds the
 * attention output.  Results equal the two-call sequence bit for bit. */
tb_status tb_rope_attention_decode(const float *q_dev, const float *k_dev, const float *v_dev, int64_t heads,
                                   int64_t kv_heads, int64_t head_dim, const float *cos_dev, const float *sin_dev,
                                   int64_t rope_max_seq, float *k_cache_dev, float *v_cache_dev, int64_t max_seq,
                                   float scale, const int32_t *pos_dev, float *out_dev, tb_stream stream);
/* margins[*pos_dev] = logits[*idx_dev] - the largest other logit. */
tb_status tb_decode_margin(const float *logits_dev, int64_t vocab, const int64_t *idx_dev,
                           const int32_t *pos_dev, int64_t max_seq, float *margins_dev, tb_stream stream);
/* End of a decode step: ids[0] = *idx (the next step's input token),
 * history[*pos] = *idx, *pos += 1. */
tb_status tb_decode_advance(const int64_t *idx_dev, int32_t *ids_dev, int32_t *pos_dev, int32_t *history_dev,
                            int64_t max_seq, tb_stream stream);

/* Causal grouped-query attention of a prompt in one launch: the 32-head loop
 * of MultiHeadAttention::forward (src/nn/attention.cpp:104-141) for S query
 * tokens at positions pos0 .. pos0 + S - 1 whose keys and values are already
 * in the caches (rows 0 .. pos0 + S - 1, [max_seq, kv_heads * head_dim]).
 * q: [S, heads * head_dim] rows (row stride ldq, RoPE applied); out: the
 * context [S, heads * head_dim] (row stride ldo).  Scores are the fp32
 * matmul's fma chain over d times `scale`; a query's later keys are masked;
 * softmax divides by the sum; p . V is the fma chain over keys in increasing
 * order.  Only exp and the order of the softmax sum differ from the reference
 * (the softmax tolerance).  head_dim 64, at most 4 query heads per key/value
 * head. */
tb_status tb_attention_prefill(const float *q_dev, int64_t ldq, const float *k_cache_dev, const float *v_cache_dev,
                               int64_t S, int64_t pos0, int64_t heads, int64_t kv_heads, int64_t head_dim,
                               float scale, float *out_dev, int64_t ldo, tb_stream stream);

/* One whole decode step of a Llama-shaped MiniGPT in a single persistent
 * kernel: MiniGPT::forward({token}, &kv) at S = 1 (src/model/minigpt.cpp:55-74,
 * the per-layer sequence of src/nn/transformer_block.cpp, attention.cpp:41-148,
 * ffn.cpp:17-27), from the token's embedding to the logits, with RoPE and the
 * KV-cache append of the new key/value at *pos_dev.  The choice of the next
 * token (tb_argmax / tb_sample_top_p_at, tb_decode_advance) follows it.
 * Layout and arithmetic are those of the fused decode kernels above (Q8_0
 * projections, fp32 activations, caches [max_seq, kv_heads * head_dim]); only
 * summation orders differ, within the GEMV and softmax tolerances.
 * Shapes: hidden 2048, head_dim 64, heads * head_dim = hidden, at most 4 query
 * heads per key/value head, ffn 2048, 4096 or 8192, max_seq <= 2048; every
 * weight Q8_0 and 16-byte aligned.  Runs one cooperative CTA per SM; a grid
 * barrier that waits 2 s without progress gives up, sets bit 0 of the device
 * error word and ends the kernel (the workspace must then be zeroed again).
 * The workspace (tb_decode_workspace_bytes, 256-byte aligned) holds the
 * step's activations and its barrier counter: zero it once before the first
 * step and keep it for the following steps. */
typedef struct tb_decode_layer {
  const void *wq, *wk, *wv, *wo, *w_gate, *w_up, *w_down; /* Q8_0, GGUF rows */
  const float *attn_norm, *ffn_norm;                      /* RMSNorm weights */
  float *k_cache, *v_cache;                               /* [max_seq, kv_heads * head_dim] */
} tb_decode_layer;
typedef struct tb_decode_model {
  int32_t n_layers;
  int64_t hidden, ffn, heads, kv_heads, head_dim, vocab, max_seq, rope_max_seq;
  float eps_attn, eps_ffn, eps_final, attn_scale;
  const tb_decode_layer *layers_dev;        /* device array of n_layers entries */
  const void *tok_emb, *lm_head;            /* Q8_0 [vocab rows of hidden] */
  const float *final_norm, *rope_cos, *rope_sin; /* RoPE tables [rope_max_seq, head_dim / 2] */
  const int32_t *token_dev, *pos_dev;       /* the step's input token and position */
  float *logits;                            /* out: [vocab] */
  void *workspace;
  size_t workspace_bytes;
} tb_decode_model;
tb_status tb_decode_workspace_bytes(const tb_decode_model *model, size_t *bytes_out);
tb_status tb_decode_step_persistent(const tb_decode_model *model, tb_stream stream);

/* Fused decode-step GEMVs (Q8_0 weights, one input row x[K], K a multiple of
 * 256; x, gamma and weights 16-byte aligned).  When gamma is non-NULL the input
 * is first RMS-normalised as tb_rmsnorm does (x / sqrt(mean(x^2) + eps) *
 * gamma; the sum of squares is taken in a different order, so results agree
 * with the unfused pair within 1e-5).  The dot products are those of
 * tb_matmul_quant for M = 1. */
typedef struct {
  const void *w;          /* n rows of K/32 Q8_0 blocks (GGUF logical {K, n}) */
  int64_t n;              /* rows */
  float *y;               /* out [n] */
  const float *residual;  /* optional [n]: y = residual + W.x, added as tb_binary(add) */
} tb_gemv_segment;
/* Up to three matrices over the same input in one launch (e.g. the Q, K and V
 * projections of attention.cpp:44-46, or the O projection plus the residual
 * of transformer_block.cpp). */
tb_status tb_gemv_q8_0_multi(const float *x_dev, int64_t K, const float *gamma_dev, float eps,
                             const tb_gemv_segment *segs, int nseg, tb_stream stream);
/* y[i] = silu(G x)[i] * (U x)[i] for gate and up weights of n rows each: the
 * FeedForward's gate_proj, up_proj and SwiGLU (src/nn/ffn.cpp,
 * src/nn/swiglu.cpp:25-31) in one launch, with tb_swiglu's rounding. */
tb_status tb_gemv_q8_0_swiglu(const float *x_dev, int64_t K, const float *gamma_dev, float eps,
                              const void *w_gate_dev, const void *w_up_dev, int64_t n, float *y_dev,
                              tb_stream stream);
/* RoPE of q [heads, head_dim] and k [kv_heads, head_dim] at position *pos_dev
 * (tb_rope_at's arithmetic) and the cache append of k and v at row *pos_dev
 * (tb_kv_append), in one launch.  A position outside the table or the cache
 * sets bit 1 of the device error word and writes nothing. */
tb_status tb_rope_kv_append(float *q_dev, float *k_dev, const float *v_dev, int64_t heads, int64_t kv_heads,
                            int64_t head_dim, const float *cos_dev, const float *sin_dev, int64_t rope_max_seq,
                            float *k_cache_dev, float *v_cache_dev, int64_t max_seq, const int32_t *pos_dev,
                            tb_stream stream);

/* Asks L2 to fetch up to 8 device byte ranges (each trimmed inward to 16-byte
 * boundaries) in the background, for weights that a later kernel of the same
 * step will read: the copies overlap the kernels in between.  A hint: results
 * never depend on it.  The launch completes only after the preceding kernel of
 * the stream has (programmatic dependent launch), so it may sit anywhere in a
 * dependent chain.  Measured NEGATIVE where this library could use it: in the
 * 1B-shaped decode step (each layer's O/gate/up/down and the next layer's
 * Q/K/V prefetched at the layer's start) 1359 against 1396 tokens/s, since
 * those GEMVs are latency-bound, not HBM-bound; the decode does not call it.
 * Kept for callers whose kernels between two weight reads leave HBM idle.  No
 * reference counterpart (the reference's weights are host memory). */
tb_status tb_prefetch_l2(const void *const *ptrs_dev, const int64_t *bytes, int n, tb_stream stream);

/* Streams and CUDA graphs for callers without the CUDA runtime: capture a
 * sequence of calls on a created stream once, replay it many times. */
typedef struct tb_graph_s *tb_graph;
tb_status tb_stream_create(tb_stream *out);
tb_status tb_stream_destroy(tb_stream stream);
tb_status tb_capture_begin(tb_stream stream);
tb_status tb_capture_end(tb_stream stream, tb_graph *out);
tb_status tb_graph_launch(tb_graph graph, tb_stream stream);
tb_status tb_graph_destroy(tb_graph graph);

/* ---------------------------------------------------------------- diagnostics -- */


#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* TURBO_B200_H */
