#pragma once
#include "layer.hpp"
#include "linear.hpp"
#include "swiglu.hpp"

namespace turbo {
class DecodeGraph;
namespace nn {
// nn::FeedForward (reference include/turbo/nn/ffn.hpp).
class FeedForward : public Layer {
 private:
  friend class ::turbo::DecodeGraph;
  Linear gate_proj;
  Linear up_proj;
  SwiGLU swiglu;
  Linear down_proj;

 public:
  FeedForward(Tensor gate, Tensor down, Tensor up);
  FeedForward(size_t embed_dim, size_t intermediate_size);
  Tensor forward(const Tensor &input) override;
};
}  // namespace nn
}  // namespace turbo
