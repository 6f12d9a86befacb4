#pragma once
#include "layer.hpp"

namespace turbo {
namespace nn {
// nn::Embedding (reference include/turbo/nn/embedding.hpp): weight {dim, vocab}.
class Embedding : public Layer {
 private:
  Tensor weight;
  size_t num_embeddings = 0;
  size_t embedding_dim = 0;

 public:
  Embedding() = default;
  Embedding(Tensor w);
  Embedding(size_t num_embeddings, size_t embedding_dim);
  Tensor forward(const Tensor &input_ids) override;
  Tensor &get_weight() { return weight; }
};
}  // namespace nn
}  // namespace turbo
