// ref_shim.cpp -- test infrastructure, NOT product code.
//
// A flat extern "C" surface over the reference Turbo.cpp tensor library, compiled
// from the reference's own sources (see oracle/Makefile) into oracle/_ref/libturbo_ref.so.
// It lets the tests and the CPU-baseline leg of bench.py call the reference ops
// from Python through ctypes, so that the CUDA path can be compared with the
// reference's own arithmetic on identical bytes.
//
// Every function builds reference `Tensor` objects around the caller's host buffers
// and calls the reference entry point named in its comment; the result is copied
// out into the caller's buffer.  C++ exceptions are mapped to status codes:
//   0 ok, 1 std::invalid_argument, 2 std::out_of_range, 3 std::runtime_error, 4 other.
//
// All C++ symbols of the reference are compiled with hidden visibility, so this
// library can be loaded next to the product library (which has its own `Tensor`)
// without symbol interposition.

#include "turbo/core/kv_cache.hpp"
#include "turbo/core/sampler.hpp"
#include "turbo/loader/gguf_loader.hpp"
#include "turbo/model/minigpt.hpp"
#include "turbo/nn/embedding.hpp"
#include "turbo/nn/linear.hpp"
#include "turbo/nn/rmsnorm.hpp"
#include "turbo/nn/rope.hpp"
#include "turbo/nn/softmax.hpp"
#include "turbo/nn/swiglu.hpp"
#include "turbo/tensor/tensor.hpp"
#include "../src/tensor/quant_math.hpp"

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <limits>
#include <memory>
#include <stdexcept>
#include <vector>

#define REF_API extern "C" __attribute__((visibility("default")))

namespace {

template <class F> int guarded(F &&f) {
  try {
    f();
    return 0;
  } catch (const std::invalid_argument &) {
    return 1;
  } catch (const std::out_of_range &) {
    return 2;
  } catch (const std::runtime_error &) {
    return 3;
  } catch (...) {
    return 4;
  }
}

std::vector<size_t> to_vec(const size_t *p, int n) {
  return std::vector<size_t>(p, p + n);
}

// Non-owning view over a caller buffer of `len` floats.
Tensor view_of(float *base, size_t len, size_t off, const size_t *shape,
               const size_t *strides, int rank) {
  auto st = std::make_shared<Storage>(static_cast<void *>(base), len * sizeof(float));
  return Tensor(st, off, to_vec(shape, rank), to_vec(strides, rank));
}

void copy_out(const Tensor &t, float *out) {
  // Results of the reference ops are fresh contiguous tensors.
  std::memcpy(out, t.data_ptr(), t.numel() * sizeof(float));
}

} // namespace

// Tensor::operator+ (src/tensor/tensor.cpp:260-282), broadcasting.
// `out` must hold the broadcast shape's element count.
REF_API int ref_add(const float *a, const size_t *a_shape, int a_rank,
                    const float *b, const size_t *b_shape, int b_rank,
                    float *out) {
  return guarded([&] {
    size_t na = 1, nb = 1;
    for (int i = 0; i < a_rank; ++i) na *= a_shape[i];
    for (int i = 0; i < b_rank; ++i) nb *= b_shape[i];
    Tensor ta(std::vector<float>(a, a + na), to_vec(a_shape, a_rank));
    Tensor tb(std::vector<float>(b, b + nb), to_vec(b_shape, b_rank));
    Tensor r = ta + tb;
    copy_out(r, out);
  });
}

// Tensor::operator+ on two strided views (src/tensor/tensor.cpp:260-282).
REF_API int ref_add_views(float *a, size_t a_len, size_t a_off,
                          const size_t *a_shape, const size_t *a_strides, int a_rank,
                          float *b, size_t b_len, size_t b_off,
                          const size_t *b_shape, const size_t *b_strides, int b_rank,
                          float *out) {
  return guarded([&] {
    Tensor ta = view_of(a, a_len, a_off, a_shape, a_strides, a_rank);
    Tensor tb = view_of(b, b_len, b_off, b_shape, b_strides, b_rank);
    Tensor r = ta + tb;
    copy_out(r, out);
  });
}

// Tensor::operator*(float) (src/tensor/tensor.cpp:284-294) on a strided view.
REF_API int ref_scale(float *x, size_t len, size_t off, const size_t *shape,
                      const size_t *strides, int rank, float s, float *out) {
  return guarded([&] {
    Tensor t = view_of(x, len, off, shape, strides, rank);
    Tensor r = t * s;
    copy_out(r, out);
  });
}

// Tensor::copy_ (src/tensor/tensor.cpp:689-726): dst view <- src view.
REF_API int ref_copy(float *dst, size_t dst_len, size_t dst_off,
                     const size_t *dst_shape, const size_t *dst_strides, int dst_rank,
                     float *src, size_t src_len, size_t src_off,
                     const size_t *src_shape, const size_t *src_strides, int src_rank) {
  return guarded([&] {
    Tensor d = view_of(dst, dst_len, dst_off, dst_shape, dst_strides, dst_rank);
    Tensor s = view_of(src, src_len, src_off, src_shape, src_strides, src_rank);
    d.copy_(s);
  });
}

// Tensor::contiguous (src/tensor/tensor.cpp:118-132).
REF_API int ref_contiguous(float *x, size_t len, size_t off, const size_t *shape,
                           const size_t *strides, int rank, float *out) {
  return guarded([&] {
    Tensor t = view_of(x, len, off, shape, strides, rank);
    Tensor r = t.contiguous();
    size_t n = r.numel();
    std::memcpy(out, r.data_ptr(), n * sizeof(float));
  });
}

// nn::RMSNorm::forward (src/nn/rmsnorm.cpp:23-68) on x[rows, cols].
REF_API int ref_rmsnorm(const float *x, size_t rows, size_t cols,
                        const float *gamma, float eps, float *out) {
  return guarded([&] {
    Tensor w(std::vector<float>(gamma, gamma + cols), {cols});
    turbo::nn::RMSNorm layer(w, eps);
    Tensor in(std::vector<float>(x, x + rows * cols), {rows, cols});
    copy_out(layer.forward(in), out);
  });
}

// nn::SwiGLU::forward(gate, up) (src/nn/swiglu.cpp:10-40) on n elements.
REF_API int ref_swiglu(const float *g, const float *u, size_t n, float *out) {
  return guarded([&] {
    Tensor tg(std::vector<float>(g, g + n), {n});
    Tensor tu(std::vector<float>(u, u + n), {n});
    turbo::nn::SwiGLU layer;
    copy_out(layer.forward(tg, tu), out);
  });
}

// nn::Softmax::forward (src/nn/softmax.cpp:13-54) over the last dim of x[rows, cols].
REF_API int ref_softmax(const float *x, size_t rows, size_t cols, float *out) {
  return guarded([&] {
    Tensor in(std::vector<float>(x, x + rows * cols), {rows, cols});
    turbo::nn::Softmax layer(-1);
    copy_out(layer.forward(in), out);
  });
}

// greedy_sample (src/core/sampler.cpp:13-26).
REF_API int ref_greedy_sample(const float *logits, size_t n) {
  return turbo::greedy_sample(logits, n);
}

// sample_top_p (src/core/sampler.cpp:28-86): `draws` calls, each drawing from the
// reference's own random_device-seeded generator.
REF_API void ref_sample_top_p(const float *logits, size_t n, float temperature, float top_p, int draws,
                              int *out) {
  for (int i = 0; i < draws; ++i) out[i] = turbo::sample_top_p(logits, n, temperature, top_p);
}

// nn::RoPE ctor + apply_in_place (src/nn/rope.cpp:9-103) on a rank-2 or rank-4
// strided view over `x`, modified in place.
REF_API int ref_rope(float *x, size_t len, size_t off, const size_t *shape,
                     const size_t *strides, int rank, size_t head_dim,
                     size_t max_seq_len, float theta, size_t pos_offset) {
  return guarded([&] {
    turbo::nn::RoPE rope(head_dim, max_seq_len, theta);
    Tensor t = view_of(x, len, off, shape, strides, rank);
    rope.apply_in_place(t, pos_offset);
  });
}

// The cos/sin tables built by the RoPE constructor (src/nn/rope.cpp:16-32),
// recomputed with the same expressions; each table is [max_seq_len, head_dim/2].
REF_API void ref_rope_tables(size_t head_dim, size_t max_seq_len, float theta,
                             float *cos_out, float *sin_out) {
  size_t half = head_dim / 2;
  for (size_t pos = 0; pos < max_seq_len; ++pos)
    for (size_t i = 0; i < half; ++i) {
      float theta_i = std::pow(theta, -static_cast<float>(2 * i) / head_dim);
      float freq = pos * theta_i;
      cos_out[pos * half + i] = std::cos(freq);
      sin_out[pos * half + i] = std::sin(freq);
    }
}

// nn::Embedding::forward (src/nn/embedding.cpp:22-118).  `dtype` follows the
// reference DataType enum (0 FP32, 2 Q8_0, 3 Q4_0).  The weight has GGUF logical
// shape {dim, vocab}.  ids are fp32-stored token ids, as the reference takes them.
REF_API int ref_embedding(void *w, int dtype, size_t dim, size_t vocab,
                          const float *ids, size_t n, float *out) {
  return guarded([&] {
    Tensor wt({dim, vocab}, static_cast<DataType>(dtype), w);
    turbo::nn::Embedding emb(wt);
    Tensor tid(std::vector<float>(ids, ids + n), {n});
    copy_out(emb.forward(tid), out);
  });
}

// Tensor::matmul Q8_0 / Q4_0 branches (src/tensor/tensor.cpp:328-432):
// Y[M, N] = X[M, K] . W, W of logical shape {K, N} stored as N rows of K/32 blocks.
REF_API int ref_matmul_quant(const float *x, size_t M, size_t K, void *w,
                             int dtype, size_t N, float *y) {
  return guarded([&] {
    Tensor tx(std::vector<float>(x, x + M * K), {M, K});
    Tensor tw({K, N}, static_cast<DataType>(dtype), w);
    copy_out(tx.matmul(tw), y);
  });
}

// Same, timed variant: the X tensor is built once, the matmul is run `iters`
// times and the result of the last run is kept.  Used for the CPU baseline.
REF_API int ref_matmul_quant_repeat(const float *x, size_t M, size_t K, void *w,
                                    int dtype, size_t N, float *y, int iters) {
  return guarded([&] {
    Tensor tx(std::vector<float>(x, x + M * K), {M, K});
    Tensor tw({K, N}, static_cast<DataType>(dtype), w);
    Tensor r;
    for (int i = 0; i < iters; ++i) r = tx.matmul(tw);
    copy_out(r, y);
  });
}

// Tensor::matmul fp32 branch (src/tensor/tensor.cpp:434-542) on strided views.
// Result is [batch..., M, N] contiguous.
REF_API int ref_matmul_f32(float *a, size_t a_len, size_t a_off,
                           const size_t *a_shape, const size_t *a_strides,
                           float *b, size_t b_len, size_t b_off,
                           const size_t *b_shape, const size_t *b_strides, int rank,
                           float *out) {
  return guarded([&] {
    Tensor ta = view_of(a, a_len, a_off, a_shape, a_strides, rank);
    Tensor tb = view_of(b, b_len, b_off, b_shape, b_strides, rank);
    copy_out(ta.matmul(tb), out);
  });
}

// nn::Linear::forward (src/nn/linear.cpp:26-55) with an fp32 weight {K, N} and
// optional bias {N} (nullptr for none).
REF_API int ref_linear_f32(const float *x, size_t M, size_t K, const float *w,
                           size_t N, const float *bias, float *y) {
  return guarded([&] {
    Tensor tw(std::vector<float>(w, w + K * N), {K, N});
    Tensor tb = bias ? Tensor(std::vector<float>(bias, bias + N), {N}) : Tensor();
    turbo::nn::Linear lin(tw, tb);
    Tensor tx(std::vector<float>(x, x + M * K), {M, K});
    copy_out(lin.forward(tx), y);
  });
}

// Quant helpers from src/tensor/quant_math.hpp.
REF_API void ref_dequantize_row_q8_0(const void *blocks, float *y, int k) {
  turbo::dequantize_row_q8_0(blocks, y, k); // quant_math.hpp:16-29
}
REF_API void ref_quantize_row_q8_0(const float *x, void *blocks, int k) {
  turbo::quantize_row_q8_0(x, blocks, k); // quant_math.hpp:68-90
}
REF_API float ref_vec_dot_q8_0_f32(int n, const void *w, const float *x) {
  return turbo::vec_dot_q8_0_f32(n, w, x); // quant_math.hpp:32-60
}
REF_API float ref_vec_dot_q4_0_q8_0(int n, const void *w, const void *xq) {
  return turbo::vec_dot_q4_0_q8_0(n, w, xq); // quant_math.hpp:139-181
}
REF_API float ref_vec_dot_q4_0_q8_0_avx2(int n, const void *w, const void *xq) {
  return turbo::vec_dot_q4_0_q8_0_avx2(n, w, xq); // quant_math.hpp:184-248
}
REF_API unsigned short ref_f32_to_f16(float f) { return turbo::convert_f32_to_f16(f); }
REF_API float ref_f16_to_f32(unsigned short h) { return turbo::fp16_to_fp32(h); }

// ---------------------------------------------------------------------------
// Whole model: GGUFLoader + MiniGPT + KVCache + greedy_sample, driven the way
// src/core/generate.cpp:9-70 drives them (prefill the prompt, then one token per
// step), but with a fixed number of greedy steps and no tokenizer.
// ---------------------------------------------------------------------------
struct RefModel {
  std::unique_ptr<turbo::GGUFLoader> loader;
  std::unique_ptr<turbo::MiniGPT> model;
};

REF_API void *ref_model_load(const char *path) {
  try {
    auto m = new RefModel();
    m->loader = std::make_unique<turbo::GGUFLoader>(path);
    m->loader->parse();
    m->model = std::make_unique<turbo::MiniGPT>(*m->loader);
    return m;
  } catch (...) {
    return nullptr;
  }
}

REF_API void ref_model_free(void *h) { delete static_cast<RefModel *>(h); }

// Runs prefill over `prompt` then `steps` greedy steps.  out_ids[steps+1] gets the
// token chosen after the prefill and after each decode step; margins[steps+1]
// the top-1 minus top-2 logit of that choice.  Optional prefill_ms/decode_ms.
REF_API int ref_model_generate(void *h, const int *prompt, size_t n_prompt,
                               size_t steps, size_t max_seq, int *out_ids,
                               float *margins, float *last_logits,
                               double *prefill_ms, double *decode_ms) {
  auto *m = static_cast<RefModel *>(h);
  return guarded([&] {
    turbo::KVCache kv((int)max_seq, (int)m->model->get_num_layers(),
                      (int)m->model->get_num_kv_heads(), (int)m->model->get_head_dim());
    auto pick = [&](const Tensor &logits, size_t slot) {
      size_t seq = logits.get_shape()[1];
      size_t V = logits.get_shape()[2];
      const float *row = logits.data_ptr() + (seq - 1) * V;
      int id = turbo::greedy_sample(row, V);
      float top1 = row[id], top2 = -std::numeric_limits<float>::infinity();
      for (size_t i = 0; i < V; ++i)
        if ((int)i != id && row[i] > top2) top2 = row[i];
      out_ids[slot] = id;
      if (margins) margins[slot] = top1 - top2;
      if (last_logits) std::memcpy(last_logits, row, V * sizeof(float));
      return id;
    };
    auto t0 = std::chrono::steady_clock::now();
    std::vector<int> ids(prompt, prompt + n_prompt);
    Tensor logits = m->model->forward(ids, &kv);
    kv.increment_seq_len((int)n_prompt);
    int next = pick(logits, 0);
    auto t1 = std::chrono::steady_clock::now();
    for (size_t s = 0; s < steps; ++s) {
      logits = m->model->forward(std::vector<int>{next}, &kv);
      kv.increment_seq_len(1);
      next = pick(logits, s + 1);
    }
    auto t2 = std::chrono::steady_clock::now();
    if (prefill_ms)
      *prefill_ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
    if (decode_ms)
      *decode_ms = std::chrono::duration<double, std::milli>(t2 - t1).count();
  });
}
