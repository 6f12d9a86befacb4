#pragma once
#include "../tensor/tensor.hpp"

namespace turbo {
namespace nn {
// Interface of include/turbo/nn/layer.hpp in the reference.
class Layer {
 public:
  virtual ~Layer() = default;
  virtual Tensor forward(const Tensor &input) = 0;
};
}  // namespace nn
}  // namespace turbo
