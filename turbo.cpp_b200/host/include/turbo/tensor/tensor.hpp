// tensor.hpp -- the Turbo.cpp Tensor/Storage API (include/turbo/tensor/tensor.hpp
// of the reference) with device-resident storage on the B200.
//
// Same class names, constructors, methods and exceptions as the reference, so
// src/nn-style call sites compile unchanged.  Differences that a caller sees:
//  - Storage bytes live in HBM (tb_alloc arena).  The zero-copy mmap
//    constructor uploads the bytes once instead of aliasing the file.
//  - Host access (at(), data_ptr(), Storage::data()) goes through a host shadow
//    that is filled from the device on first access and written back before
//    the next device op.  It is for inspection and tests; every op runs on the
//    GPU.
//  - Quantized matmuls use the library's default GEMV/GEMM (within 1e-5 of the
//    reference); set_exact_matmul(true) selects the bit-identical kernels.
//  - A quantized weight multiplied by 32 or more rows keeps a packed copy for
//    the tensor cores (tb_pack_quant_weights, 4 bytes per weight) beside its
//    blocks, made on first use; set_weight_packing(false) turns this off.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <memory>
#include <vector>

#include "turbo/tensor/quant_types.hpp"

enum class DataType { FP32, FP16, Q8_0, Q4_0, INT32 };

inline size_t get_block_size(DataType type) {
  return (type == DataType::Q8_0 || type == DataType::Q4_0) ? 32 : 1;
}

inline size_t get_type_size(DataType type) {
  switch (type) {
    case DataType::FP32: return 4;
    case DataType::FP16: return 2;
    case DataType::INT32: return 4;
    case DataType::Q8_0: return sizeof(turbo::block_q8_0);
    case DataType::Q4_0: return sizeof(turbo::block_q4_0);
  }
  return 0;
}

enum class Device { CPU, CUDA, MPS };

namespace turbo {
// Selects the bit-identical quantized matmul kernels for every Tensor::matmul.
void set_exact_matmul(bool exact);
bool exact_matmul();
// Lets quantized weights keep a packed copy for prefill-sized matmuls
// (default on).  Turning it off frees nothing already packed.
void set_weight_packing(bool on);
bool weight_packing();
// Blocks until every queued device op has finished.
void device_synchronize();
}  // namespace turbo

class Storage {
 public:
  Storage();
  explicit Storage(size_t size_bytes);
  explicit Storage(const std::vector<float> &d);
  // Binds an external host buffer (e.g. an mmap'd GGUF tensor): the bytes are
  // uploaded to HBM once; the external buffer is not kept.
  Storage(void *external_ptr, size_t size_bytes);
  Storage(const Storage &) = delete;
  Storage &operator=(const Storage &) = delete;
  ~Storage();

  // Host view of the bytes (synchronised from the device; marks the host copy
  // as the newer one, so device ops upload it first).
  uint8_t *data() const;
  size_t size_bytes() const { return size_bytes_; }
  bool owns_memory() const { return owns_memory_; }

  // Device address of the bytes, after writing back any host-side changes.
  void *device_data() const;
  // Device address for an op that overwrites the bytes (no write-back).
  void *device_data_discard() const;

  // The bytes, as N rows of K quantized values of `dtype` (TB_Q8_0 or
  // TB_Q4_0), packed for the tensor-core matmul: made on first use and kept
  // until data() or device_data_discard() hands out the bytes for writing.
  // A caller that writes the bytes through device_data() must call
  // drop_packed() itself.
  const void *packed_quant(int dtype, int64_t N, int64_t K) const;
  void drop_packed() const;

 private:
  void *dev_ = nullptr;
  size_t size_bytes_ = 0;
  bool owns_memory_ = true;
  mutable std::vector<uint8_t> host_;
  mutable int state_ = 0;  // 0: device newer, 1: host newer, 2: both equal
  mutable void *packed_ = nullptr;
  mutable int packed_dtype_ = 0;
  mutable int64_t packed_N_ = 0, packed_K_ = 0;
};

class Tensor {
 private:
  std::shared_ptr<Storage> storage;
  size_t offset;
  std::vector<size_t> shape;
  std::vector<size_t> strides;

  DataType dtype_ = DataType::FP32;
  Device device_ = Device::CUDA;

  static std::vector<size_t> compute_strides(const std::vector<size_t> &shape);
  static std::vector<size_t> compute_broadcast_shape(const std::vector<size_t> &s1,
                                                     const std::vector<size_t> &s2);
  static std::vector<size_t> unravel_index(size_t flat_index, const std::vector<size_t> &shape);

 public:
  Tensor();
  Tensor(std::vector<float> d, std::vector<size_t> s);
  Tensor(std::shared_ptr<Storage> st, size_t off, std::vector<size_t> s, std::vector<size_t> str);
  Tensor(const std::vector<size_t> &shape, DataType dtype, void *external_ptr);

  // New device tensor with uninitialised contents (contiguous).
  static Tensor empty(const std::vector<size_t> &shape, DataType dtype = DataType::FP32);
  static Tensor zeros(const std::vector<size_t> &shape);

  bool is_empty() const { return storage == nullptr || storage->size_bytes() == 0; }
  size_t rank() const { return shape.size(); }
  size_t numel() const;
  const std::vector<size_t> &get_shape() const { return shape; }
  const std::vector<size_t> &get_strides() const { return strides; }
  size_t get_offset() const { return offset; }
  DataType dtype() const { return dtype_; }
  Device device() const { return device_; }
  bool is_contiguous() const;
  Tensor contiguous() const;

  Tensor transpose() const;
  Tensor transpose(size_t dim0, size_t dim1) const;
  Tensor slice(size_t dim, size_t index) const;
  Tensor slice(size_t dim, size_t start, size_t end) const;
  Tensor reshape(const std::vector<size_t> &new_shape) const;
  Tensor flatten() const;
  Tensor unsqueeze(size_t dim) const;
  Tensor squeeze(size_t dim) const;
  Tensor broadcast_to(const std::vector<size_t> &target_shape) const;
  void copy_(const Tensor &src);

  Tensor operator+(const Tensor &other) const;
  Tensor operator*(float scalar) const;
  Tensor matmul(const Tensor &other) const;

  float &at(const std::vector<size_t> &indices);
  const float &at(const std::vector<size_t> &indices) const;

  float *data_ptr();
  const float *data_ptr() const;
  void *data_ptr_raw() const;

  // Device address of element 0 of this view (offset applied).
  void *device_ptr() const;
  std::shared_ptr<Storage> get_storage() const { return storage; }

  void print() const;
};

// The reference's raw packed fp32 GEMM (host pointers, C += A.B over an
// M x K x N block).  Runs on the GPU: the operands are uploaded, multiplied
// with the k-ordered FMA kernel and the result written back.
void matmul_threaded_packed_avx2(const float *A, const float *B, float *C, size_t M, size_t K,
                                 size_t N, size_t stride_A, size_t stride_B, size_t stride_C);
