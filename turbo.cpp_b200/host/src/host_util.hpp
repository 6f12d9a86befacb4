// host_util.hpp -- status-to-exception mapping and Tensor -> tb_view.
#pragma once
#include <stdexcept>
#include <string>

#include "turbo/tensor/tensor.hpp"
#include "turbo_b200.h"

namespace turbo {
namespace detail {

// Rethrows a C ABI status as the exception type the reference throws.
inline void tb_check(tb_status st) {
  switch (st) {
    case TB_OK: return;
    case TB_EINVAL: throw std::invalid_argument(tb_last_error());
    case TB_ERANGE: throw std::out_of_range(tb_last_error());
    case TB_ERUNTIME: throw std::runtime_error(tb_last_error());
    default: throw std::runtime_error(std::string(tb_status_name(st)) + ": " + tb_last_error());
  }
}

inline int tb_dtype_of(DataType d) {
  switch (d) {
    case DataType::FP32: return TB_F32;
    case DataType::FP16: return TB_F16;
    case DataType::Q8_0: return TB_Q8_0;
    case DataType::Q4_0: return TB_Q4_0;
    case DataType::INT32: return TB_I32;
  }
  return TB_F32;
}

// The reference's Tensor metadata as a C ABI view over the device storage.
inline tb_view view_of(const Tensor &t) {
  tb_view v{};
  v.data = t.get_storage()->size_bytes() ? t.get_storage()->device_data() : nullptr;
  v.dtype = tb_dtype_of(t.dtype());
  v.rank = (int32_t)t.rank();
  v.offset = (int64_t)t.get_offset();
  for (size_t i = 0; i < t.rank(); ++i) {
    v.shape[i] = (int64_t)t.get_shape()[i];
    v.strides[i] = (int64_t)t.get_strides()[i];
  }
  return v;
}

}  // namespace detail
}  // namespace turbo
