#pragma once
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

#include "turbo/tensor/tensor.hpp"

namespace turbo {
// A GGUF (v2/v3) reader with the query methods of the reference
// GGUFLoader (include/turbo/loader/gguf_loader.hpp) that MiniGPT uses.
// get_tensor() uploads the tensor's bytes to the device once.
class GGUFLoader {
 public:
  explicit GGUFLoader(const std::string &filepath);
  ~GGUFLoader();
  GGUFLoader(const GGUFLoader &) = delete;
  GGUFLoader &operator=(const GGUFLoader &) = delete;

  void parse();
  uint32_t get_num_layers() const { return num_layers_; }
  uint32_t get_hidden_dim() const { return hidden_dim_; }
  uint32_t get_ffn_intermediate_size() const { return ffn_; }
  uint32_t get_num_heads() const { return num_heads_; }
  uint32_t get_num_kv_heads() const { return num_kv_heads_; }
  uint32_t get_context_length() const { return context_length_; }
  float get_rope_freq_base() const { return rope_freq_base_; }
  uint32_t get_rope_dim_count() const { return rope_dim_count_; }
  Tensor get_tensor(const std::string &name);
  bool has_tensor(const std::string &name) const;

 private:
  struct Info {
    std::vector<uint64_t> shape;
    uint32_t type;
    uint64_t offset;
  };
  std::string path_;
  const uint8_t *map_ = nullptr;
  size_t size_ = 0;
  uint64_t data_offset_ = 0;
  uint32_t alignment_ = 32;
  uint32_t num_layers_ = 32, hidden_dim_ = 4096, ffn_ = 0, num_heads_ = 32, num_kv_heads_ = 32;
  uint32_t context_length_ = 4096, rope_dim_count_ = 0;
  float rope_freq_base_ = 10000.0f;
  std::unordered_map<std::string, Info> tensors_;
};
}  // namespace turbo
