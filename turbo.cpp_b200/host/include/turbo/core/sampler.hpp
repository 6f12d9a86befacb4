#pragma once
#include "../tensor/tensor.hpp"

namespace turbo {
// greedy_sample (reference include/turbo/core/sampler.hpp:6): index of the
// first maximum.  The pointer form takes host logits (uploaded and reduced on
// the GPU); the Tensor form reduces the last row of device-resident logits.
int greedy_sample(const float *last_token_logits, size_t vocab_size);
int greedy_sample(const Tensor &logits);

// sample_top_p (reference include/turbo/core/sampler.hpp:8): nucleus sampling
// on the GPU (tb_sample_top_p).  The reference's form takes host logits and
// draws its uniform number from a random_device-seeded mt19937, as the
// reference does; the Tensor form samples the last row of device-resident
// logits with the uniform number u in [0, 1) given (reproducible draws).
int sample_top_p(const float *last_token_logits, size_t vocab_size, float temperature, float top_p);
int sample_top_p(const Tensor &logits, float temperature, float top_p, double u);
}  // namespace turbo
