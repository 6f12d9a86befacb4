#pragma once
#include <memory>
#include <vector>

#include "../nn/embedding.hpp"
#include "../nn/linear.hpp"
#include "../nn/rmsnorm.hpp"
#include "../nn/transformer_block.hpp"
#include "../tensor/tensor.hpp"

namespace turbo {
class DecodeGraph;
class KVCache;
class GGUFLoader;

// MiniGPT (reference include/turbo/model/minigpt.hpp): embedding -> blocks ->
// output norm -> LM head on the last token (tied to token_embd if no output.weight).
class MiniGPT {
 private:
  friend class ::turbo::DecodeGraph;
  nn::Embedding tok_emb;
  std::vector<nn::TransformerBlock> blocks;
  nn::RMSNorm norm;
  nn::Linear lm_head;
  size_t num_heads_ = 0;
  size_t num_kv_heads_ = 0;
  size_t head_dim_ = 0;

 public:
  MiniGPT(size_t vocab_size, size_t hidden_dim, size_t num_layers, size_t num_heads);
  explicit MiniGPT(GGUFLoader &loader);
  size_t get_num_layers() const { return blocks.size(); }
  size_t get_num_heads() const { return num_heads_; }
  size_t get_num_kv_heads() const { return num_kv_heads_; }
  size_t get_head_dim() const { return head_dim_; }
  Tensor forward(const Tensor &token_ids, KVCache *kv_cache = nullptr);
  Tensor forward(const std::vector<int> &ids, KVCache *kv_cache = nullptr);
};
}  // namespace turbo
