#pragma once
#include <memory>
#include <vector>

#include "../tensor/tensor.hpp"

namespace turbo {
class DecodeGraph;
namespace nn {
// nn::RoPE (reference include/turbo/nn/rope.hpp).  The cos/sin tables are
// computed on the host as the reference constructor does and uploaded once.
class RoPE {
 private:
  friend class ::turbo::DecodeGraph;
  size_t head_dim;
  size_t max_seq_len;
  float theta_base;
  std::vector<float> cos_cache;
  std::vector<float> sin_cache;
  std::shared_ptr<Tensor> dev_cos, dev_sin;

 public:
  RoPE(size_t head_dim, size_t max_seq_len = 4096, float theta_base = 10000.0f);
  void apply_in_place(Tensor &x, size_t position_offset = 0);
};
}  // namespace nn
}  // namespace turbo
