#pragma once
#include "../tensor/tensor.hpp"

namespace turbo {
// greedy_sample (reference include/turbo/core/sampler.hpp:6): index of the
// first maximum.  The pointer form takes host logits (uploaded and reduced on
// the GPU); the Tensor form reduces the last row of device-resident logits.
int greedy_sample(const float *last_token_logits, size_t vocab_size);
int greedy_sample(const Tensor &logits);
}  // namespace turbo
