// model.cpp -- KVCache, greedy_sample, the GGUF reader and MiniGPT over the
// device Tensor (reference src/core/kv_cache.cpp, src/core/sampler.cpp,
// src/loader/gguf_loader.cpp, src/model/minigpt.cpp).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <random>
#include <stdexcept>
#include <string>

#include "host_util.hpp"
#include "turbo/core/kv_cache.hpp"
#include "turbo/core/sampler.hpp"
#include "turbo/loader/gguf_loader.hpp"
#include "turbo/model/minigpt.hpp"

using turbo::detail::tb_check;

namespace turbo {

// ----------------------------------------------------------------- KVCache --
KVCache::KVCache(int max_seq_len, int num_layers, int num_kv_heads, int head_dim)
    : max_seq_len_(max_seq_len), num_layers_(num_layers), num_kv_heads_(num_kv_heads), head_dim_(head_dim) {
  const std::vector<size_t> shape = {(size_t)max_seq_len, (size_t)num_kv_heads, (size_t)head_dim};
  for (int i = 0; i < num_layers; ++i) {
    k_caches_.push_back(Tensor::zeros(shape));
    v_caches_.push_back(Tensor::zeros(shape));
  }
}

// ----------------------------------------------------------------- sampler --
static int argmax_device(const float *x_dev, size_t n) {
  Tensor idx64 = Tensor::empty({2}, DataType::INT32);  // 8 bytes: one int64 index
  tb_check(tb_argmax(x_dev, 1, (int64_t)n, static_cast<int64_t *>(idx64.get_storage()->device_data_discard()),
                     nullptr));
  int64_t out = 0;
  tb_check(tb_download(&out, idx64.get_storage()->device_data(), sizeof(out), nullptr));
  tb_check(tb_sync(nullptr));
  return (int)out;
}

int greedy_sample(const float *last_token_logits, size_t vocab_size) {
  // Host logits (the reference signature): uploaded, reduced by tb_argmax.
  Tensor t(std::vector<float>(last_token_logits, last_token_logits + vocab_size), {vocab_size});
  return argmax_device(static_cast<const float *>(t.device_ptr()), vocab_size);
}

int greedy_sample(const Tensor &logits) {
  const size_t V = logits.get_shape().back();
  const size_t rows = logits.numel() / V;
  const Tensor c = logits.contiguous();  // kept alive while its memory is read
  const float *last = static_cast<const float *>(c.device_ptr()) + (rows - 1) * V;
  return argmax_device(last, V);
}

static int sample_device(const float *x_dev, size_t n, float temperature, float top_p, double u) {
  Tensor id = Tensor::empty({1}, DataType::INT32);
  tb_check(tb_sample_top_p(x_dev, (int64_t)n, temperature, top_p, u,
                           static_cast<int32_t *>(id.get_storage()->device_data_discard()), nullptr));
  int32_t out = 0;
  tb_check(tb_download(&out, id.get_storage()->device_data(), sizeof(out), nullptr));
  tb_check(tb_sync(nullptr));
  return (int)out;
}

int sample_top_p(const float *last_token_logits, size_t vocab_size, float temperature, float top_p) {
  // The reference's generator (src/core/sampler.cpp:80-81): one random_device-seeded
  // mt19937 for the process; the uniform number is what discrete_distribution draws.
  static std::random_device rd;
  static std::mt19937 gen(rd());
  const double u = std::generate_canonical<double, 53>(gen);
  Tensor t(std::vector<float>(last_token_logits, last_token_logits + vocab_size), {vocab_size});
  return sample_device(static_cast<const float *>(t.device_ptr()), vocab_size, temperature, top_p, u);
}

int sample_top_p(const Tensor &logits, float temperature, float top_p, double u) {
  const size_t V = logits.get_shape().back();
  const size_t rows = logits.numel() / V;
  const Tensor c = logits.contiguous();  // kept alive while its memory is read
  const float *last = static_cast<const float *>(c.device_ptr()) + (rows - 1) * V;
  return sample_device(last, V, temperature, top_p, u);
}

// -------------------------------------------------------------- GGUFLoader --
namespace {
struct Reader {
  const uint8_t *p, *end;
  template <typename T> T get() {
    if (p + sizeof(T) > end) throw std::runtime_error("GGUF file is truncated.");
    T v;
    std::memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string str() {
    uint64_t n = get<uint64_t>();
    if (p + n > end) throw std::runtime_error("GGUF file is truncated.");
    std::string s(reinterpret_cast<const char *>(p), n);
    p += n;
    return s;
  }
  void skip(uint32_t type) {
    static const int sz[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (type == 8) {
      str();
    } else if (type == 9) {
      uint32_t at = get<uint32_t>();
      uint64_t n = get<uint64_t>();
      for (uint64_t i = 0; i < n; ++i) skip(at);
    } else if (type < 13) {
      p += sz[type];
    } else {
      throw std::runtime_error("Unknown GGUF metadata type");
    }
  }
};
}  // namespace

GGUFLoader::GGUFLoader(const std::string &filepath) : path_(filepath) {
  int fd = ::open(filepath.c_str(), O_RDONLY);
  if (fd < 0) throw std::runtime_error("Cannot open GGUF file: " + filepath);
  struct stat st;
  if (fstat(fd, &st) != 0) {
    ::close(fd);
    throw std::runtime_error("Cannot stat GGUF file: " + filepath);
  }
  size_ = (size_t)st.st_size;
  void *m = mmap(nullptr, size_, PROT_READ, MAP_SHARED, fd, 0);
  ::close(fd);
  if (m == MAP_FAILED) throw std::runtime_error("mmap failed: " + filepath);
  map_ = static_cast<const uint8_t *>(m);
}

GGUFLoader::~GGUFLoader() {
  if (map_) munmap(const_cast<uint8_t *>(map_), size_);
}

void GGUFLoader::parse() {
  Reader r{map_, map_ + size_};
  if (r.get<uint32_t>() != 0x46554747u) throw std::runtime_error("Invalid GGUF magic bytes. Not a GGUF file.");
  r.get<uint32_t>();  // version
  const uint64_t n_tensors = r.get<uint64_t>();
  const uint64_t n_kv = r.get<uint64_t>();
  for (uint64_t i = 0; i < n_kv; ++i) {
    const std::string key = r.str();
    const uint32_t type = r.get<uint32_t>();
    auto u32 = [&](uint32_t &dst) {
      if (type == 4) dst = r.get<uint32_t>();
      else r.skip(type);
    };
    if (key == "general.alignment") u32(alignment_);
    else if (key == "llama.block_count") u32(num_layers_);
    else if (key == "llama.embedding_length") u32(hidden_dim_);
    else if (key == "llama.feed_forward_length") u32(ffn_);
    else if (key == "llama.attention.head_count") u32(num_heads_);
    else if (key == "llama.attention.head_count_kv") u32(num_kv_heads_);
    else if (key == "llama.context_length") u32(context_length_);
    else if (key == "llama.rope.dimension_count") u32(rope_dim_count_);
    else if (key == "llama.rope.freq_base" && type == 6) rope_freq_base_ = r.get<float>();
    else r.skip(type);
  }
  for (uint64_t i = 0; i < n_tensors; ++i) {
    Info info;
    const std::string name = r.str();
    const uint32_t nd = r.get<uint32_t>();
    for (uint32_t d = 0; d < nd; ++d) info.shape.push_back(r.get<uint64_t>());
    info.type = r.get<uint32_t>();
    info.offset = r.get<uint64_t>();
    tensors_[name] = info;
  }
  const uint64_t meta = (uint64_t)(r.p - map_);
  data_offset_ = meta + (alignment_ - meta % alignment_) % alignment_;
}

bool GGUFLoader::has_tensor(const std::string &name) const { return tensors_.count(name) != 0; }

Tensor GGUFLoader::get_tensor(const std::string &name) {
  auto it = tensors_.find(name);
  if (it == tensors_.end())
    throw std::runtime_error("Tensor weight matching name '" + name + "' not found in GGUF file architecture.");
  const Info &info = it->second;
  DataType dt;
  switch (info.type) {
    case 0: dt = DataType::FP32; break;
    case 1: dt = DataType::FP16; break;
    case 2: dt = DataType::Q4_0; break;
    case 8: dt = DataType::Q8_0; break;
    default: throw std::runtime_error("Unsupported GGUF tensor type encountered: " + std::to_string(info.type));
  }
  size_t n = 1;
  std::vector<size_t> shape;
  for (uint64_t d : info.shape) {
    n *= d;
    shape.push_back((size_t)d);
  }
  const size_t bytes = n / get_block_size(dt) * get_type_size(dt);
  if (data_offset_ + info.offset + bytes > size_)
    throw std::runtime_error("Tensor '" + name + "' is beyond the end of the file. The GGUF file is truncated or corrupted!");
  return Tensor(shape, dt, const_cast<uint8_t *>(map_ + data_offset_ + info.offset));
}

// ----------------------------------------------------------------- MiniGPT --
MiniGPT::MiniGPT(size_t vocab, size_t hidden, size_t layers, size_t heads)
    : tok_emb(vocab, hidden), norm(hidden), lm_head(hidden, vocab), num_heads_(heads), num_kv_heads_(heads),
      head_dim_(hidden / heads) {
  for (size_t i = 0; i < layers; ++i) blocks.emplace_back(hidden, heads, heads, 4 * hidden);
}

MiniGPT::MiniGPT(GGUFLoader &L)
    : tok_emb(L.get_tensor("token_embd.weight")), norm(L.get_tensor("output_norm.weight")),
      num_heads_(L.get_num_heads()), num_kv_heads_(L.get_num_kv_heads()),
      head_dim_(L.get_hidden_dim() / L.get_num_heads()) {
  // The LM head is tied to token_embd when the file has no output.weight
  // (minigpt.cpp:21); the embedding's device copy is shared, not uploaded twice.
  lm_head = L.has_tensor("output.weight") ? nn::Linear(L.get_tensor("output.weight"))
                                          : nn::Linear(tok_emb.get_weight());
  for (uint32_t i = 0; i < L.get_num_layers(); ++i)
    blocks.emplace_back(L, (int)i, L.get_hidden_dim(), num_heads_, num_kv_heads_, L.get_context_length(),
                        L.get_rope_freq_base());
}

Tensor MiniGPT::forward(const Tensor &token_ids, KVCache *kv_cache) {
  Tensor x = tok_emb.forward(token_ids).unsqueeze(0);
  const size_t S = x.get_shape()[1];
  const size_t pos = kv_cache ? (size_t)kv_cache->get_current_seq_len() : 0;
  for (size_t i = 0; i < blocks.size(); ++i) x = blocks[i].forward(x, pos, kv_cache, (int)i);
  x = norm.forward(x);
  Tensor last = x.slice(1, S - 1, S);  // the LM head runs on the last token only
  return lm_head.forward(last.contiguous());
}

Tensor MiniGPT::forward(const std::vector<int> &ids, KVCache *kv_cache) {
  std::vector<float> f(ids.begin(), ids.end());
  Tensor t(f, {ids.size()});
  return forward(t, kv_cache);
}

}  // namespace turbo
