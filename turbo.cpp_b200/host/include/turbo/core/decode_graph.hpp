// decode_graph.hpp -- decode of MiniGPT as one CUDA graph per token, greedy or
// nucleus-sampled.
// No reference counterpart: the reference loop (src/core/generate.cpp:30-63)
// calls MiniGPT::forward once per token.
#pragma once
#include <cstddef>
#include <cstdint>

#include "turbo_b200.h"

namespace turbo {
class MiniGPT;
class KVCache;

// Selects the single-kernel decode step where the model's shapes allow it
// (default off: the fused per-op graph).  Read when a DecodeGraph is created.
void set_persistent_decode(bool on);
bool persistent_decode();

// One decode step -- embedding, the transformer blocks, final norm, LM head,
// argmax or nucleus sample -- recorded once as a CUDA graph.  The position, the input token and
// the chosen tokens live in device memory, so the same graph is replayed for
// every token with no host work in between.  The step runs the kernels
// MiniGPT::forward runs for one token, except that each layer's attention is a
// single fused kernel (tb_attention_decode) instead of the per-head loop of
// attention.cpp:104-141; its softmax sum and probability-times-V order differ
// within the fp32 tolerance.  Unless the bit-identical matmul kernels are
// selected (set_exact_matmul), a layer with Q8_0 projections runs as five
// launches: RMSNorm + Q/K/V GEMVs, RoPE + cache append + attention, O GEMV +
// residual, RMSNorm + gate/up GEMVs + SwiGLU, down GEMV + residual.
// When the shapes allow it (hidden 2048, head_dim 64, Q8_0 weights; see
// tb_decode_step_persistent) and persistent decode is switched on
// (set_persistent_decode; off by default: on the 1B-shaped model it measures
// 1226 against 1367 tokens/s for the fused kernels), the whole step up to the
// logits is instead ONE persistent kernel, followed by the argmax or sample
// and the advance.
class DecodeGraph {
 public:
  // `kv` holds the prompt's keys/values (kv.get_current_seq_len() rows).
  // temperature > 0 samples each token as sample_top_p(logits, temperature,
  // top_p) does (src/core/generate.cpp:42-47), with the uniform numbers that
  // generate() is given; otherwise the choice is greedy.
  DecodeGraph(MiniGPT &model, KVCache &kv, bool want_margins, float temperature = 0.f, float top_p = 0.9f);
  ~DecodeGraph();
  DecodeGraph(const DecodeGraph &) = delete;
  DecodeGraph &operator=(const DecodeGraph &) = delete;

  // Feeds `first` at the cache's current position and the chosen token after
  // it, `steps` times: out_ids[s] is the token chosen at step s; margins[s]
  // (optional) its logit minus the largest other logit.  When sampling,
  // uniforms[s] in [0, 1) draws step s's token.  Advances the cache by `steps`.
  void generate(int first, size_t steps, int *out_ids, float *margins, const double *uniforms = nullptr);

 private:
  void enqueue_step();
  void enqueue_step_fused();
  void setup_persistent();  // tables and workspace of the single-kernel step
  void enqueue_step_persistent();
  bool persistent_ = false;
  tb_decode_model pm_{};
  void enqueue_pick(tb_stream s);  // argmax or sample, margin, advance
  void *buf(size_t bytes);
  bool fused_ = false;

  MiniGPT &m_;
  KVCache &kv_;
  bool margins_on_;
  float temperature_, top_p_;
  tb_stream stream_ = nullptr;
  tb_graph graph_ = nullptr;
  size_t E_, H_, KVH_, D_, F_, V_;
  int max_seq_;
  float scale_;
  // device buffers
  void *arena_[40] = {};
  int n_arena_ = 0;
  int32_t *ids_, *pos_, *hist_;
  int64_t *idx_;
  double *uniform_ = nullptr;  // [max_seq]: the uniform number of each position's draw
  float *margins_, *x_, *xn_, *h_, *q_, *k_, *v_, *ctx_, *ao_, *g_, *u_, *sw_, *fo_, *logits_;
};

}  // namespace turbo
