#pragma once
#include "layer.hpp"

namespace turbo {
namespace nn {
// nn::Linear (reference include/turbo/nn/linear.hpp): weight {in, out}, optional bias {out}.
class Linear : public Layer {
 private:
  Tensor weight;
  Tensor bias;
  size_t in_features = 0;
  size_t out_features = 0;

 public:
  Linear() = default;
  Linear(Tensor w, Tensor b = Tensor());
  Linear(size_t in_features, size_t out_features);
  Tensor forward(const Tensor &input) override;
  Tensor &get_weight() { return weight; }
  Tensor &get_bias() { return bias; }
};
}  // namespace nn
}  // namespace turbo
