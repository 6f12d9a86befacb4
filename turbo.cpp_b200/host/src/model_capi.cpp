// model_capi.cpp -- a flat C interface over the host layer's MiniGPT for
// callers outside C++ (the tests and bench.py drive the 1B-shaped decode
// through it).  It runs what src/core/generate.cpp:9-70 runs: prefill the
// prompt, then one greedy token per step with the KV cache.
#include <chrono>
#include <cmath>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "host_util.hpp"
#include "turbo/core/decode_graph.hpp"
#include "turbo/core/kv_cache.hpp"
#include "turbo/core/sampler.hpp"
#include "turbo/loader/gguf_loader.hpp"
#include "turbo/model/minigpt.hpp"

#define TBM_API extern "C" __attribute__((visibility("default")))

namespace {
thread_local std::string g_err;

struct Model {
  std::unique_ptr<turbo::GGUFLoader> loader;
  std::unique_ptr<turbo::MiniGPT> model;
  bool exact = false;
};

template <class F> int guarded(F &&f) {
  try {
    f();
    return 0;
  } catch (const std::invalid_argument &e) {
    g_err = e.what();
    return 1;
  } catch (const std::out_of_range &e) {
    g_err = e.what();
    return 2;
  } catch (const std::exception &e) {
    g_err = e.what();
    return 3;
  }
}
}  // namespace

TBM_API const char *tbm_last_error() { return g_err.c_str(); }

// Loads a GGUF model onto the current device.  exact != 0 selects the
// bit-identical quantized matmul kernels for this process and the reference's
// op-by-op decode; otherwise decode steps replay one CUDA graph per token
// (turbo::DecodeGraph).
TBM_API void *tbm_model_load(const char *path, int exact) {
  Model *m = nullptr;
  int st = guarded([&] {
    turbo::set_exact_matmul(exact != 0);
    auto mm = std::make_unique<Model>();
    mm->loader = std::make_unique<turbo::GGUFLoader>(path);
    mm->loader->parse();
    mm->model = std::make_unique<turbo::MiniGPT>(*mm->loader);
    mm->exact = exact != 0;
    turbo::device_synchronize();
    m = mm.release();
  });
  return st == 0 ? m : nullptr;
}

TBM_API void tbm_model_free(void *h) { delete static_cast<Model *>(h); }

// persistent != 0: decode steps run as one persistent kernel per token where
// the model's shapes allow it (turbo::set_persistent_decode); 0 (the default)
// keeps the fused per-op CUDA graph.  Applies to later generate calls.
TBM_API void tbm_set_persistent_decode(int persistent) { turbo::set_persistent_decode(persistent != 0); }

// Prefill `prompt`, then `steps` decode steps.  out_ids[steps + 1] receives
// the token chosen after the prefill and after each step: greedy, or with
// temperature > 0 sample_top_p(logits, temperature, top_p) drawn with
// uniforms[steps + 1] (src/core/generate.cpp:42-47).  margins (optional)
// receives each choice's logit minus the largest other logit, last_logits
// (optional) the final step's logits -- diagnostics read back from the device.
static int generate_impl(Model *m, const int *prompt, size_t n_prompt, size_t steps, size_t max_seq, float temperature,
                         float top_p, const double *uniforms, int *out_ids, float *margins, float *last_logits,
                         double *prefill_ms, double *decode_ms) {
  return guarded([&] {
    if (temperature > 0.f && !uniforms) throw std::invalid_argument("sampling needs a uniform number per token");
    turbo::MiniGPT &model = *m->model;
    turbo::KVCache kv((int)max_seq, (int)model.get_num_layers(), (int)model.get_num_kv_heads(),
                      (int)model.get_head_dim());
    auto pick = [&](const Tensor &logits, size_t slot) {
      const int id = temperature > 0.f ? turbo::sample_top_p(logits, temperature, top_p, uniforms[slot])
                                       : turbo::greedy_sample(logits);
      out_ids[slot] = id;
      if (margins || last_logits) {
        const size_t V = logits.get_shape().back();
        const float *row = logits.data_ptr() + (logits.numel() - V);
        if (margins) {
          float top2 = -INFINITY;
          for (size_t i = 0; i < V; ++i)
            if ((int)i != id && row[i] > top2) top2 = row[i];
          margins[slot] = row[id] - top2;
        }
        if (last_logits) std::memcpy(last_logits, row, V * sizeof(float));
      }
      return id;
    };
    turbo::device_synchronize();
    auto t0 = std::chrono::steady_clock::now();
    std::vector<int> ids(prompt, prompt + n_prompt);
    Tensor logits = model.forward(ids, &kv);
    kv.increment_seq_len((int)n_prompt);
    int next = pick(logits, 0);
    auto t1 = std::chrono::steady_clock::now();
    if (!m->exact && steps > 0 && !last_logits) {
      turbo::device_synchronize();  // the prefill's cache writes, before the decode stream starts
      turbo::DecodeGraph dg(model, kv, margins != nullptr, temperature, top_p);
      dg.generate(next, steps, out_ids + 1, margins ? margins + 1 : nullptr,
                  temperature > 0.f ? uniforms + 1 : nullptr);
    } else {
      for (size_t s = 0; s < steps; ++s) {
        logits = model.forward(std::vector<int>{next}, &kv);
        kv.increment_seq_len(1);
        next = pick(logits, s + 1);
      }
    }
    turbo::device_synchronize();
    auto t2 = std::chrono::steady_clock::now();
    if (prefill_ms) *prefill_ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
    if (decode_ms) *decode_ms = std::chrono::duration<double, std::milli>(t2 - t1).count();
  });
}

TBM_API int tbm_model_generate(void *h, const int *prompt, size_t n_prompt, size_t steps, size_t max_seq,
                               int *out_ids, float *margins, float *last_logits, double *prefill_ms,
                               double *decode_ms) {
  return generate_impl(static_cast<Model *>(h), prompt, n_prompt, steps, max_seq, 0.f, 0.f, nullptr, out_ids,
                       margins, last_logits, prefill_ms, decode_ms);
}

// generate_text with temperature > 0 (src/core/generate.cpp:42-47; top_p is
// 0.9 there): uniforms[steps + 1] are the uniform numbers of the draws.
TBM_API int tbm_model_generate_sampled(void *h, const int *prompt, size_t n_prompt, size_t steps, size_t max_seq,
                                       float temperature, float top_p, const double *uniforms, int *out_ids,
                                       float *margins, double *prefill_ms, double *decode_ms) {
  return generate_impl(static_cast<Model *>(h), prompt, n_prompt, steps, max_seq, temperature, top_p, uniforms,
                       out_ids, margins, nullptr, prefill_ms, decode_ms);
}
