#pragma once
#include "attention.hpp"
#include "ffn.hpp"
#include "layer.hpp"
#include "rmsnorm.hpp"

namespace turbo {
class DecodeGraph;
class KVCache;
class GGUFLoader;
namespace nn {
// nn::TransformerBlock (reference include/turbo/nn/transformer_block.hpp).
class TransformerBlock : public Layer {
 private:
  friend class ::turbo::DecodeGraph;
  RMSNorm attention_norm;
  MultiHeadAttention attention;
  RMSNorm ffn_norm;
  FeedForward ffn;

 public:
  TransformerBlock(GGUFLoader &loader, int layer_idx, size_t embed_dim, size_t num_heads, size_t num_kv_heads,
                   size_t max_seq_len = 4096, float theta_base = 10000.0f);
  TransformerBlock(size_t embed_dim, size_t num_heads, size_t num_kv_heads, size_t intermediate_size,
                   size_t max_seq_len = 4096, float theta_base = 10000.0f);
  Tensor forward(const Tensor &input, size_t position_offset, KVCache *kv_cache = nullptr, int layer_idx = -1);
  Tensor forward(const Tensor &input) override;
};
}  // namespace nn
}  // namespace turbo
