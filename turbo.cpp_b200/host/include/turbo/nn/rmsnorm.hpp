#pragma once
#include "layer.hpp"

namespace turbo {
class DecodeGraph;
namespace nn {
// nn::RMSNorm (reference include/turbo/nn/rmsnorm.hpp).
class RMSNorm : public Layer {
 private:
  friend class ::turbo::DecodeGraph;
  Tensor weight;
  float epsilon = 1e-5f;
  size_t hidden_size = 0;

 public:
  RMSNorm() = default;
  RMSNorm(Tensor w, float epsilon = 1e-5f);
  RMSNorm(size_t hidden_size, float epsilon = 1e-5f);
  Tensor forward(const Tensor &input) override;
  Tensor &get_weight() { return weight; }
};
}  // namespace nn
}  // namespace turbo
