// quant_types.hpp -- the GGUF Q8_0 / Q4_0 block formats (a file format, so the
// layout is the reference's: include/turbo/tensor/quant_types.hpp:17-38).
#pragma once
#include <cstdint>

#define QK8_0 32
#define QK4_0 32

namespace turbo {

// 34 bytes: IEEE half scale d, then 32 signed quants; value j = q[j] * d.
struct block_q8_0 {
  uint16_t d;
  int8_t qs[QK8_0];
};
static_assert(sizeof(block_q8_0) == 34, "block_q8_0 must be 34 bytes");

// 18 bytes: half scale d, then 16 bytes of nibbles; byte j holds value j in its
// low nibble and value j + 16 in its high nibble; value = (nibble - 8) * d.
struct block_q4_0 {
  uint16_t d;
  uint8_t qs[QK4_0 / 2];
};
static_assert(sizeof(block_q4_0) == 18, "block_q4_0 must be 18 bytes");

}  // namespace turbo
