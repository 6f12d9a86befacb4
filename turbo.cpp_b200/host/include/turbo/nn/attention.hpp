#pragma once
#include "layer.hpp"
#include "linear.hpp"
#include "rope.hpp"
#include "softmax.hpp"

namespace turbo {
class DecodeGraph;
class KVCache;
namespace nn {
// nn::MultiHeadAttention with grouped KV heads (reference include/turbo/nn/attention.hpp).
class MultiHeadAttention : public Layer {
 private:
  friend class ::turbo::DecodeGraph;
  size_t embed_dim;
  size_t num_heads;
  size_t num_kv_heads;
  size_t head_dim;
  Linear q_proj, k_proj, v_proj, o_proj;
  RoPE rope;
  Softmax softmax;

 public:
  MultiHeadAttention(Tensor q, Tensor k, Tensor v, Tensor o, size_t embed_dim, size_t num_heads,
                     size_t num_kv_heads, size_t max_seq_len = 4096, float theta_base = 10000.0f);
  MultiHeadAttention(size_t embed_dim, size_t num_heads, size_t num_kv_heads, size_t max_seq_len = 4096,
                     float theta_base = 10000.0f);
  Tensor forward(const Tensor &input) override;
  Tensor forward(const Tensor &input, size_t position_offset, KVCache *kv_cache = nullptr,
                 int layer_idx = -1);
};
}  // namespace nn
}  // namespace turbo
