#pragma once
#include "layer.hpp"

namespace turbo {
namespace nn {
// nn::SwiGLU (reference include/turbo/nn/swiglu.hpp).
class SwiGLU : public Layer {
 public:
  SwiGLU() = default;
  Tensor forward(const Tensor &gate, const Tensor &up);
  Tensor forward(const Tensor &input) override;  // deprecated in the reference: throws
};
}  // namespace nn
}  // namespace turbo
