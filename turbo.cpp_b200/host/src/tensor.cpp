// tensor.cpp -- Tensor/Storage over the B200 C ABI.  View manipulation is host
// metadata (as in the reference, src/tensor/tensor.cpp:99-256); every op that
// touches element values is a kernel of libturbo_b200.
#include "turbo/tensor/tensor.hpp"

#include <algorithm>
#include <iostream>
#include <stdexcept>
#include <string>

#include "host_util.hpp"

namespace turbo {
namespace {
bool g_exact = false;
bool g_packing = true;
}
void set_exact_matmul(bool exact) { g_exact = exact; }
bool exact_matmul() { return g_exact; }
void set_weight_packing(bool on) { g_packing = on; }
bool weight_packing() { return g_packing; }
void device_synchronize() { detail::tb_check(tb_sync(nullptr)); }
}  // namespace turbo

using turbo::detail::tb_check;

// ------------------------------------------------------------------ Storage --

Storage::Storage() : dev_(nullptr), size_bytes_(0), owns_memory_(false) {}

Storage::Storage(size_t size_bytes) : size_bytes_(size_bytes), owns_memory_(true) {
  if (size_bytes_ > 0) tb_check(tb_alloc(&dev_, size_bytes_));
  state_ = 0;
}

Storage::Storage(const std::vector<float> &d) : size_bytes_(d.size() * sizeof(float)), owns_memory_(true) {
  if (size_bytes_ > 0) {
    tb_check(tb_alloc(&dev_, size_bytes_));
    tb_check(tb_upload(dev_, d.data(), size_bytes_, nullptr));
  }
  state_ = 0;
}

Storage::Storage(void *external_ptr, size_t size_bytes) : size_bytes_(size_bytes), owns_memory_(false) {
  // The reference aliases the mmap'd bytes (tensor.hpp:76-77); here they are
  // uploaded once.  The device copy is owned by this Storage.
  if (size_bytes_ > 0) {
    tb_check(tb_alloc(&dev_, size_bytes_));
    tb_check(tb_upload(dev_, external_ptr, size_bytes_, nullptr));
    tb_check(tb_sync(nullptr));  // the caller may unmap the file afterwards
  }
  state_ = 0;
}

Storage::~Storage() {
  // All host-layer ops run on the default stream, so a later kernel that gets
  // this block from the arena is ordered after every kernel that used it.
  drop_packed();
  if (dev_) tb_free(dev_);
}

void Storage::drop_packed() const {
  if (packed_) tb_free(packed_);
  packed_ = nullptr;
}

const void *Storage::packed_quant(int dtype, int64_t N, int64_t K) const {
  if (packed_ && packed_dtype_ == dtype && packed_N_ == N && packed_K_ == K) return packed_;
  drop_packed();
  size_t bytes = 0;
  tb_check(tb_packed_quant_weights_bytes(dtype, N, K, &bytes));
  void *p = nullptr;
  tb_check(tb_alloc(&p, bytes));
  const tb_status rs = tb_pack_quant_weights(dtype, device_data(), N, K, p, bytes, nullptr);
  if (rs != TB_OK) {
    tb_free(p);
    tb_check(rs);
  }
  packed_ = p;
  packed_dtype_ = dtype;
  packed_N_ = N;
  packed_K_ = K;
  return packed_;
}

uint8_t *Storage::data() const {
  drop_packed();  // the caller may write through the pointer
  if (size_bytes_ == 0) return nullptr;
  if (state_ == 0) {
    host_.resize(size_bytes_);
    tb_check(tb_download(host_.data(), dev_, size_bytes_, nullptr));
    tb_check(tb_sync(nullptr));
  }
  state_ = 1;  // the caller may write through the pointer
  return host_.data();
}

void *Storage::device_data() const {
  if (state_ == 1) {
    tb_check(tb_upload(dev_, host_.data(), size_bytes_, nullptr));
    state_ = 0;
  } else if (state_ == 2) {
    state_ = 0;
  }
  return dev_;
}

void *Storage::device_data_discard() const {
  drop_packed();
  state_ = 0;
  return dev_;
}

// ------------------------------------------------------------------- Tensor --

std::vector<size_t> Tensor::compute_strides(const std::vector<size_t> &shape) {
  std::vector<size_t> st(shape.size());
  size_t acc = 1;
  for (size_t i = shape.size(); i-- > 0;) {
    st[i] = acc;
    acc *= shape[i];
  }
  return st;
}

std::vector<size_t> Tensor::compute_broadcast_shape(const std::vector<size_t> &s1,
                                                    const std::vector<size_t> &s2) {
  const size_t r = std::max(s1.size(), s2.size());
  std::vector<size_t> out(r);
  for (size_t k = 0; k < r; ++k) {
    size_t d1 = k < s1.size() ? s1[s1.size() - 1 - k] : 1;
    size_t d2 = k < s2.size() ? s2[s2.size() - 1 - k] : 1;
    if (d1 != d2 && d1 != 1 && d2 != 1) throw std::invalid_argument("Shapes are not broadcastable.");
    out[r - 1 - k] = std::max(d1, d2);
  }
  return out;
}

std::vector<size_t> Tensor::unravel_index(size_t flat, const std::vector<size_t> &shape) {
  std::vector<size_t> idx(shape.size());
  for (size_t i = shape.size(); i-- > 0;) {
    idx[i] = flat % shape[i];
    flat /= shape[i];
  }
  return idx;
}

Tensor::Tensor() : storage(std::make_shared<Storage>()), offset(0) {}

Tensor::Tensor(std::vector<float> d, std::vector<size_t> s)
    : storage(std::make_shared<Storage>(d)), offset(0), shape(std::move(s)) {
  strides = compute_strides(shape);
}

Tensor::Tensor(std::shared_ptr<Storage> st, size_t off, std::vector<size_t> s, std::vector<size_t> str)
    : storage(std::move(st)), offset(off), shape(std::move(s)), strides(std::move(str)) {}

Tensor::Tensor(const std::vector<size_t> &s, DataType dtype, void *external_ptr)
    : offset(0), shape(s), dtype_(dtype) {
  strides = compute_strides(shape);
  size_t n = 1;
  for (size_t d : shape) n *= d;
  const size_t bs = get_block_size(dtype);
  if (n % bs != 0) throw std::invalid_argument("Tensor shape is not divisible by block size.");
  storage = std::make_shared<Storage>(external_ptr, n / bs * get_type_size(dtype));
}

Tensor Tensor::empty(const std::vector<size_t> &shape, DataType dtype) {
  size_t n = 1;
  for (size_t d : shape) n *= d;
  auto st = std::make_shared<Storage>(n / get_block_size(dtype) * get_type_size(dtype));
  Tensor t(st, 0, shape, compute_strides(shape));
  t.dtype_ = dtype;
  return t;
}

Tensor Tensor::zeros(const std::vector<size_t> &shape) {
  Tensor t = empty(shape);
  if (t.storage->size_bytes())
    tb_check(tb_memset(t.storage->device_data_discard(), 0, t.storage->size_bytes(), nullptr));
  return t;
}

size_t Tensor::numel() const {
  if (shape.empty()) return 0;  // as the reference (tensor.cpp:99-106)
  size_t n = 1;
  for (size_t d : shape) n *= d;
  return n;
}

bool Tensor::is_contiguous() const {
  size_t expect = 1;
  for (size_t i = shape.size(); i-- > 0;) {
    if (strides[i] != expect) return false;
    expect *= shape[i];
  }
  return true;
}

Tensor Tensor::contiguous() const {
  if (is_contiguous()) return *this;  // shares storage, as the reference
  Tensor out = empty(shape, dtype_);
  tb_view d = turbo::detail::view_of(out), s = turbo::detail::view_of(*this);
  tb_check(tb_copy(&d, &s, nullptr));
  return out;
}

Tensor Tensor::transpose() const {
  if (rank() != 2) throw std::invalid_argument("transpose() without args requires a 2D tensor.");
  return transpose(0, 1);
}

Tensor Tensor::transpose(size_t d0, size_t d1) const {
  if (d0 >= rank() || d1 >= rank()) throw std::out_of_range("Transpose dimensions out of bounds");
  std::vector<size_t> sh = shape, st = strides;
  std::swap(sh[d0], sh[d1]);
  std::swap(st[d0], st[d1]);
  Tensor t(storage, offset, sh, st);
  t.dtype_ = dtype_;
  return t;
}

Tensor Tensor::slice(size_t dim, size_t index) const {
  if (dim >= shape.size()) throw std::invalid_argument("Dimension out of range.");
  if (index >= shape[dim]) throw std::out_of_range("Slice index out of bounds.");
  std::vector<size_t> sh = shape, st = strides;
  sh.erase(sh.begin() + dim);
  st.erase(st.begin() + dim);
  Tensor t(storage, offset + index * strides[dim], sh, st);
  t.dtype_ = dtype_;
  return t;
}

Tensor Tensor::slice(size_t dim, size_t start, size_t end) const {
  if (dim >= shape.size()) throw std::invalid_argument("Dimension out of range.");
  if (start > end || end > shape[dim]) throw std::out_of_range("Slice range out of bounds.");
  std::vector<size_t> sh = shape;
  sh[dim] = end - start;
  Tensor t(storage, offset + start * strides[dim], sh, strides);
  t.dtype_ = dtype_;
  return t;
}

Tensor Tensor::reshape(const std::vector<size_t> &new_shape) const {
  if (!is_contiguous()) throw std::runtime_error("Cannot reshape a non-contiguous tensor.");
  size_t n = 1;
  for (size_t d : new_shape) n *= d;
  if (n != numel()) {
    std::string err = "Reshape changes total elements. Old shape: [";
    for (size_t d : shape) err += std::to_string(d) + ", ";
    err += "] (numel=" + std::to_string(numel()) + ") -> New shape: [";
    for (size_t d : new_shape) err += std::to_string(d) + ", ";
    err += "] (new_numel=" + std::to_string(n) + ")";
    throw std::invalid_argument(err);
  }
  Tensor t(storage, offset, new_shape, compute_strides(new_shape));
  t.dtype_ = dtype_;
  return t;
}

Tensor Tensor::flatten() const { return reshape({numel()}); }

Tensor Tensor::unsqueeze(size_t dim) const {
  if (dim > shape.size()) throw std::out_of_range("Unsqueeze dimension out of bounds.");
  std::vector<size_t> sh = shape, st = strides;
  sh.insert(sh.begin() + dim, 1);
  st.insert(st.begin() + dim, dim < strides.size() ? strides[dim] : 1);
  Tensor t(storage, offset, sh, st);
  t.dtype_ = dtype_;
  return t;
}

Tensor Tensor::squeeze(size_t dim) const {
  if (dim >= shape.size()) throw std::out_of_range("Squeeze dimension out of bounds.");
  if (shape[dim] != 1) throw std::invalid_argument("Can only squeeze dimensions of size 1.");
  std::vector<size_t> sh = shape, st = strides;
  sh.erase(sh.begin() + dim);
  st.erase(st.begin() + dim);
  Tensor t(storage, offset, sh, st);
  t.dtype_ = dtype_;
  return t;
}

Tensor Tensor::broadcast_to(const std::vector<size_t> &target) const {
  if (target.size() < shape.size()) throw std::invalid_argument("Target rank too small.");
  const size_t diff = target.size() - shape.size();
  std::vector<size_t> sh(diff, 1), st(diff, 0);
  sh.insert(sh.end(), shape.begin(), shape.end());
  st.insert(st.end(), strides.begin(), strides.end());
  for (size_t i = 0; i < target.size(); ++i) {
    if (sh[i] != target[i]) {
      if (sh[i] != 1) throw std::invalid_argument("Shapes are not broadcastable.");
      sh[i] = target[i];
      st[i] = 0;
    }
  }
  Tensor t(storage, offset, sh, st);
  t.dtype_ = dtype_;
  return t;
}

void Tensor::copy_(const Tensor &src) {
  if (shape != src.shape)
    throw std::invalid_argument("Tensor::copy_ failed: Target and source shapes must match exactly.");
  if (dtype_ != src.dtype_)
    throw std::invalid_argument("Tensor::copy_ failed: Target and source data types must match.");
  if (numel() == 0) return;
  tb_view d = turbo::detail::view_of(*this), s = turbo::detail::view_of(src);
  tb_check(tb_copy(&d, &s, nullptr));
}

Tensor Tensor::operator+(const Tensor &other) const {
  if (is_empty()) return other;  // tensor.cpp:261-264
  if (other.is_empty()) return *this;
  Tensor out = empty(compute_broadcast_shape(shape, other.shape));
  tb_view a = turbo::detail::view_of(*this), b = turbo::detail::view_of(other);
  tb_view o = turbo::detail::view_of(out);
  tb_check(tb_binary(0, &a, &b, &o, nullptr));
  return out;
}

Tensor Tensor::operator*(float scalar) const {
  Tensor out = empty(shape);
  if (numel() == 0) return out;
  tb_view x = turbo::detail::view_of(*this), o = turbo::detail::view_of(out);
  tb_check(tb_scale(&x, scalar, &o, nullptr));
  return out;
}

Tensor Tensor::matmul(const Tensor &other) const {
  if (rank() < 2 || other.rank() < 2) throw std::invalid_argument("matmul requires at least 2D tensors");
  if (dtype_ == DataType::FP32 && (other.dtype_ == DataType::Q8_0 || other.dtype_ == DataType::Q4_0)) {
    // tensor.cpp:328-432: X flattened to [M, K] from its data pointer; W has
    // logical shape {K, N} and is read from its storage base.
    size_t M = 1;
    for (size_t i = 0; i + 1 < rank(); ++i) M *= shape[i];
    const size_t K = shape.back();
    if (K != other.shape[0]) throw std::invalid_argument("Inner dimensions must match for quantized matmul");
    const size_t N = other.shape[1];
    std::vector<size_t> rs = shape;
    rs.back() = N;
    Tensor out = empty(rs);
    const int dt = other.dtype_ == DataType::Q8_0 ? TB_Q8_0 : TB_Q4_0;
    const float *x = static_cast<const float *>(device_ptr());
    const void *w = other.storage->device_data();
    float *y = static_cast<float *>(out.storage->device_data_discard());
    if (turbo::exact_matmul()) {
      tb_check(tb_matmul_quant_exact(dt, x, (int64_t)M, (int64_t)K, w, (int64_t)N, y, nullptr));
    } else if (turbo::weight_packing() && M >= 32 && K >= 256 && K % 256 == 0 && K <= (1u << 20) &&
               (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0) {
      // prefill: the tensor cores with W packed once (identical results)
      const void *pk = other.storage->packed_quant(dt, (int64_t)N, (int64_t)K);
      tb_check(tb_matmul_quant_packed(dt, x, (int64_t)M, (int64_t)K, pk, (int64_t)N, y, nullptr));
    } else {
      tb_check(tb_matmul_quant(dt, x, (int64_t)M, (int64_t)K, w, (int64_t)N, y, nullptr));
    }
    return out;
  }
  if (rank() != other.rank()) throw std::invalid_argument("matmul requires both tensors to have the same rank");
  std::vector<size_t> rs;
  for (size_t i = 0; i + 2 < rank(); ++i) {
    if (shape[i] != other.shape[i]) throw std::invalid_argument("Batch dimensions must match");
    rs.push_back(shape[i]);
  }
  if (shape[rank() - 1] != other.shape[rank() - 2]) throw std::invalid_argument("Inner dimensions must match");
  rs.push_back(shape[rank() - 2]);
  rs.push_back(other.shape[rank() - 1]);
  Tensor out = empty(rs);
  tb_view a = turbo::detail::view_of(*this), b = turbo::detail::view_of(other), o = turbo::detail::view_of(out);
  tb_check(tb_matmul_f32(&a, &b, &o, nullptr));
  return out;
}

float *Tensor::data_ptr() { return reinterpret_cast<float *>(storage->data()) + offset; }
const float *Tensor::data_ptr() const { return reinterpret_cast<const float *>(storage->data()) + offset; }

void *Tensor::data_ptr_raw() const {
  if (dtype_ == DataType::FP32) return reinterpret_cast<float *>(storage->data()) + offset;
  return storage->data();  // quantized: offset assumed 0 (tensor.cpp:559-563)
}

void *Tensor::device_ptr() const {
  char *base = static_cast<char *>(storage->device_data());
  if (dtype_ == DataType::Q8_0 || dtype_ == DataType::Q4_0) return base;
  return base + offset * get_type_size(dtype_);
}

float &Tensor::at(const std::vector<size_t> &idx) {
  if (idx.size() != shape.size()) throw std::invalid_argument("Rank mismatch.");
  size_t flat = offset;
  for (size_t i = 0; i < idx.size(); ++i) {
    if (idx[i] >= shape[i]) throw std::out_of_range("Index out of bounds.");
    flat += idx[i] * strides[i];
  }
  return reinterpret_cast<float *>(storage->data())[flat];
}

const float &Tensor::at(const std::vector<size_t> &idx) const {
  if (idx.size() != shape.size()) throw std::invalid_argument("Rank mismatch.");
  size_t flat = offset;
  for (size_t i = 0; i < idx.size(); ++i) {
    if (idx[i] >= shape[i]) throw std::out_of_range("Index out of bounds.");
    flat += idx[i] * strides[i];
  }
  return reinterpret_cast<const float *>(storage->data())[flat];
}

void Tensor::print() const {
  if (shape.size() != 2) {
    std::cout << "Print currently supports 2D tensors.\n";
    return;
  }
  for (size_t i = 0; i < shape[0]; ++i) {
    for (size_t j = 0; j < shape[1]; ++j) std::cout << at({i, j}) << " ";
    std::cout << "\n";
  }
}

void matmul_threaded_packed_avx2(const float *A, const float *B, float *C, size_t M, size_t K, size_t N,
                                 size_t stride_A, size_t stride_B, size_t stride_C) {
  // C += A . B with row strides; host buffers in, host buffer out.
  Tensor a(std::vector<float>(A, A + (M ? (M - 1) * stride_A + K : 0)), {M ? (M - 1) * stride_A + K : 0});
  Tensor b(std::vector<float>(B, B + (K ? (K - 1) * stride_B + N : 0)), {K ? (K - 1) * stride_B + N : 0});
  Tensor av(a.get_storage(), 0, {M, K}, {stride_A, 1});
  Tensor bv(b.get_storage(), 0, {K, N}, {stride_B, 1});
  Tensor p = av.matmul(bv);
  std::vector<float> c((M ? (M - 1) * stride_C + N : 0));
  for (size_t i = 0; i < M; ++i) std::memcpy(&c[i * stride_C], C + i * stride_C, N * sizeof(float));
  Tensor ct(c, {c.size()});
  Tensor cv(ct.get_storage(), 0, {M, N}, {stride_C, 1});
  Tensor sum = cv + p;  // contiguous [M, N]
  const float *h = sum.data_ptr();
  for (size_t i = 0; i < M; ++i) std::memcpy(C + i * stride_C, h + i * N, N * sizeof(float));
}
