// nn.cpp -- the nn layers over the device Tensor.  Each forward follows the
// reference's sequence of tensor ops (src/nn/*.cpp); the element math is done
// by the C ABI kernels.
#include <cmath>
#include <stdexcept>
#include <string>

#include "host_util.hpp"
#include "turbo/core/kv_cache.hpp"
#include "turbo/loader/gguf_loader.hpp"
#include "turbo/nn/attention.hpp"
#include "turbo/nn/embedding.hpp"
#include "turbo/nn/ffn.hpp"
#include "turbo/nn/linear.hpp"
#include "turbo/nn/rmsnorm.hpp"
#include "turbo/nn/rope.hpp"
#include "turbo/nn/softmax.hpp"
#include "turbo/nn/swiglu.hpp"
#include "turbo/nn/transformer_block.hpp"

using turbo::detail::tb_check;

namespace turbo {
namespace nn {

// ------------------------------------------------------------------ Linear --
// src/nn/linear.cpp:26-55
Linear::Linear(Tensor w, Tensor b)
    : weight(std::move(w)), bias(std::move(b)),
      in_features(weight.rank() > 0 ? weight.get_shape()[0] : 0),
      out_features(weight.rank() > 1 ? weight.get_shape()[1] : 0) {}

Linear::Linear(size_t in, size_t out)
    : weight(Tensor::zeros({in, out})), bias(Tensor::zeros({out})), in_features(in), out_features(out) {}

Tensor Linear::forward(const Tensor &input) {
  const std::vector<size_t> in_shape = input.get_shape();
  Tensor x = input;
  if (in_shape.size() > 2) {
    size_t rows = 1;
    for (size_t i = 0; i + 1 < in_shape.size(); ++i) rows *= in_shape[i];
    x = input.reshape({rows, in_shape.back()});
  }
  Tensor out = x.matmul(weight);
  if (!bias.is_empty()) out = out + bias;
  if (in_shape.size() > 2) {
    std::vector<size_t> os = in_shape;
    os.back() = out_features;
    out = out.reshape(os);
  }
  return out;
}

// ----------------------------------------------------------------- RMSNorm --
// src/nn/rmsnorm.cpp:23-68
RMSNorm::RMSNorm(Tensor w, float eps)
    : weight(std::move(w)), epsilon(eps), hidden_size(weight.rank() > 0 ? weight.get_shape()[0] : 0) {}

RMSNorm::RMSNorm(size_t hidden, float eps)
    : weight(std::vector<float>(hidden, 1.0f), {hidden}), epsilon(eps), hidden_size(hidden) {}

Tensor RMSNorm::forward(const Tensor &input) {
  const auto &sh = input.get_shape();
  if (sh.empty() || sh.back() != hidden_size)
    throw std::invalid_argument("Input last dimension must match hidden_size.");
  if (weight.dtype() != DataType::FP32)
    throw std::runtime_error("RMSNorm weight must be FP32! Found dtype: " +
                             std::to_string(static_cast<int>(weight.dtype())));
  Tensor out = Tensor::empty(sh);
  size_t rows = 1;
  for (size_t i = 0; i + 1 < sh.size(); ++i) rows *= sh[i];
  tb_check(tb_rmsnorm(TB_F32, input.device_ptr(), static_cast<const float *>(weight.device_ptr()),
                      out.device_ptr(), (int64_t)rows, (int64_t)hidden_size, epsilon, nullptr));
  return out;
}

// ------------------------------------------------------------------ SwiGLU --
// src/nn/swiglu.cpp:10-44
Tensor SwiGLU::forward(const Tensor &gate, const Tensor &up) {
  if (gate.get_shape() != up.get_shape())
    throw std::invalid_argument("SwiGLU requires gate and up tensors to have the same shape.");
  Tensor out = Tensor::empty(gate.get_shape());
  tb_check(tb_swiglu(TB_F32, gate.device_ptr(), up.device_ptr(), out.device_ptr(), (int64_t)gate.numel(), nullptr));
  return out;
}

Tensor SwiGLU::forward(const Tensor &) {
  throw std::runtime_error("SwiGLU::forward(const Tensor &input) is deprecated. Use forward(gate, up).");
}

// ----------------------------------------------------------------- Softmax --
// src/nn/softmax.cpp:13-54 (last dimension)
Tensor Softmax::forward(const Tensor &input) {
  if (input.get_shape().empty()) throw std::invalid_argument("Cannot softmax an empty tensor.");
  Tensor x = input.contiguous();
  Tensor out = Tensor::empty(x.get_shape());
  const size_t cols = x.get_shape().back();
  const size_t rows = cols ? x.numel() / cols : 0;
  tb_check(tb_softmax(static_cast<const float *>(x.device_ptr()), static_cast<float *>(out.device_ptr()),
                      (int64_t)rows, (int64_t)cols, nullptr));
  return out;
}

// -------------------------------------------------------------------- RoPE --
// src/nn/rope.cpp:9-103.  The tables use the same float expressions and libm
// calls as the reference constructor, so they are bit-identical.
RoPE::RoPE(size_t hd, size_t max_seq, float theta) : head_dim(hd), max_seq_len(max_seq), theta_base(theta) {
  if (head_dim % 2 != 0) throw std::invalid_argument("RoPE requires an even head dimension.");
  const size_t half = head_dim / 2;
  cos_cache.resize(max_seq_len * half);
  sin_cache.resize(max_seq_len * half);
  for (size_t pos = 0; pos < max_seq_len; ++pos)
    for (size_t i = 0; i < half; ++i) {
      const float theta_i = std::pow(theta_base, -static_cast<float>(2 * i) / head_dim);
      const float freq = pos * theta_i;
      cos_cache[pos * half + i] = std::cos(freq);
      sin_cache[pos * half + i] = std::sin(freq);
    }
  dev_cos = std::make_shared<Tensor>(cos_cache, std::vector<size_t>{max_seq_len, half});
  dev_sin = std::make_shared<Tensor>(sin_cache, std::vector<size_t>{max_seq_len, half});
}

void RoPE::apply_in_place(Tensor &x, size_t position_offset) {
  tb_view v = turbo::detail::view_of(x);
  tb_check(tb_rope(&v, static_cast<const float *>(dev_cos->device_ptr()),
                   static_cast<const float *>(dev_sin->device_ptr()), (int64_t)head_dim, (int64_t)max_seq_len,
                   (int64_t)position_offset, nullptr));
}

// --------------------------------------------------------------- Embedding --
// src/nn/embedding.cpp:22-118
Embedding::Embedding(Tensor w)
    : weight(std::move(w)),
      num_embeddings(weight.rank() > 1 ? weight.get_shape()[1] : (weight.rank() > 0 ? weight.get_shape()[0] : 0)),
      embedding_dim(weight.rank() > 0 ? weight.get_shape()[0] : 0) {}

Embedding::Embedding(size_t n, size_t dim)
    : weight(Tensor::zeros({dim, n})), num_embeddings(n), embedding_dim(dim) {}

Tensor Embedding::forward(const Tensor &input_ids) {
  if (input_ids.rank() != 1) throw std::invalid_argument("Embedding layer expects a 1D tensor of Token IDs.");
  const size_t S = input_ids.get_shape()[0];
  std::vector<int32_t> ids(S);
  for (size_t i = 0; i < S; ++i) {
    const size_t id = static_cast<size_t>(input_ids.at({i}));
    if (id >= num_embeddings)
      throw std::out_of_range("Token ID " + std::to_string(id) + " exceeds vocabulary size " +
                              std::to_string(num_embeddings));
    ids[i] = (int32_t)id;
  }
  int dt;
  switch (weight.dtype()) {
    case DataType::FP32: dt = TB_F32; break;
    case DataType::Q8_0: dt = TB_Q8_0; break;
    case DataType::Q4_0: dt = TB_Q4_0; break;
    default: throw std::runtime_error("Unsupported embedding dtype");
  }
  Tensor dev_ids = Tensor::empty({S}, DataType::INT32);
  tb_check(tb_upload(dev_ids.get_storage()->device_data_discard(), ids.data(), S * sizeof(int32_t), nullptr));
  Tensor out = Tensor::empty({S == 1 ? 1 : S, embedding_dim});
  const void *w = dt == TB_F32 ? weight.device_ptr() : weight.get_storage()->device_data();
  tb_check(tb_embedding(dt, w, (int64_t)embedding_dim, (int64_t)num_embeddings,
                        static_cast<const int32_t *>(dev_ids.device_ptr()), (int64_t)S,
                        static_cast<float *>(out.device_ptr()), nullptr));
  return out;
}

// ------------------------------------------------------------- FeedForward --
// src/nn/ffn.cpp:17-27
FeedForward::FeedForward(Tensor gate, Tensor down, Tensor up)
    : gate_proj(std::move(gate)), up_proj(std::move(up)), down_proj(std::move(down)) {}

FeedForward::FeedForward(size_t embed_dim, size_t inter)
    : gate_proj(embed_dim, inter), up_proj(embed_dim, inter), down_proj(inter, embed_dim) {}

Tensor FeedForward::forward(const Tensor &input) {
  Tensor gate = gate_proj.forward(input);
  Tensor up = up_proj.forward(input);
  Tensor hidden = swiglu.forward(gate, up);
  return down_proj.forward(hidden);
}

// ------------------------------------------------------- MultiHeadAttention --
// src/nn/attention.cpp:41-148
MultiHeadAttention::MultiHeadAttention(Tensor q, Tensor k, Tensor v, Tensor o, size_t E, size_t H, size_t KVH,
                                       size_t max_seq, float theta)
    : embed_dim(E), num_heads(H), num_kv_heads(KVH), head_dim(E / H), q_proj(std::move(q)),
      k_proj(std::move(k)), v_proj(std::move(v)), o_proj(std::move(o)), rope(E / H, max_seq, theta), softmax(-1) {
  if (E % H != 0) throw std::invalid_argument("Embedding dimension must be divisible by number of heads.");
}

MultiHeadAttention::MultiHeadAttention(size_t E, size_t H, size_t KVH, size_t max_seq, float theta)
    : embed_dim(E), num_heads(H), num_kv_heads(KVH), head_dim(E / H), q_proj(E, E), k_proj(E, E), v_proj(E, E),
      o_proj(E, E), rope(E / H, max_seq, theta), softmax(-1) {
  if (E % H != 0) throw std::invalid_argument("Embedding dimension must be divisible by number of heads.");
}

Tensor MultiHeadAttention::forward(const Tensor &input, size_t position_offset, KVCache *kv_cache, int layer_idx) {
  const size_t B = input.get_shape()[0];
  const size_t S = input.get_shape()[1];
  Tensor Q = q_proj.forward(input).reshape({B, S, num_heads, head_dim}).transpose(1, 2);
  Tensor K = k_proj.forward(input).reshape({B, S, num_kv_heads, head_dim}).transpose(1, 2);
  Tensor V = v_proj.forward(input).reshape({B, S, num_kv_heads, head_dim}).transpose(1, 2);
  rope.apply_in_place(Q, position_offset);
  rope.apply_in_place(K, position_offset);

  const size_t n_rep = num_heads / num_kv_heads;
  const float scale = 1.0f / std::sqrt(static_cast<float>(head_dim));
  if (kv_cache != nullptr && layer_idx >= 0) {
    const size_t start = (size_t)kv_cache->get_current_seq_len();
    Tensor &Kc = kv_cache->get_k_cache(layer_idx);
    Tensor &Vc = kv_cache->get_v_cache(layer_idx);
    Kc.slice(0, start, start + S).copy_(K.squeeze(0).transpose(0, 1));
    Vc.slice(0, start, start + S).copy_(V.squeeze(0).transpose(0, 1));
    if (B == 1 && head_dim == 64 && n_rep <= 4 && !exact_matmul()) {
      // every head of the prompt in one launch: Q rows [S, H * D] as the
      // projection wrote them (RoPE applied in place), keys/values from the
      // cache rows 0 .. start + S; the context comes out as [S, H * D], the
      // layout the per-head loop's transpose + contiguous would give
      Tensor context = Tensor::empty({B, S, embed_dim});
      tb_check(tb_attention_prefill(static_cast<const float *>(Q.device_ptr()), (int64_t)(num_heads * head_dim),
                                    static_cast<const float *>(Kc.device_ptr()),
                                    static_cast<const float *>(Vc.device_ptr()), (int64_t)S, (int64_t)start,
                                    (int64_t)num_heads, (int64_t)num_kv_heads, (int64_t)head_dim, scale,
                                    static_cast<float *>(context.get_storage()->device_data_discard()),
                                    (int64_t)embed_dim, nullptr));
      return o_proj.forward(context);
    }
    K = Kc.slice(0, 0, start + S).transpose(0, 1).unsqueeze(0);
    V = Vc.slice(0, 0, start + S).transpose(0, 1).unsqueeze(0);
  }

  Tensor context = Tensor::zeros({B, num_heads, S, head_dim});
  for (size_t b = 0; b < B; ++b) {
    for (size_t h = 0; h < num_heads; ++h) {
      const size_t kvh = h / n_rep;
      Tensor Qh = Q.slice(0, b).slice(0, h);
      Tensor Kh = K.slice(0, b).slice(0, kvh);
      Tensor Vh = V.slice(0, b).slice(0, kvh);
      Tensor scores = Qh.matmul(Kh.transpose(0, 1)) * scale;
      const size_t ctx = scores.get_shape().back();
      if (ctx > 1 && S > 1)  // causal mask: k_pos > q_pos + offset -> -1e9
        tb_check(tb_fill_upper(static_cast<float *>(scores.device_ptr()), (int64_t)S, (int64_t)ctx, (int64_t)ctx,
                               (int64_t)position_offset, -1e9f, nullptr));
      Tensor probs = softmax.forward(scores);
      Tensor ch = probs.matmul(Vh);
      context.slice(0, b).slice(0, h).copy_(ch);
    }
  }
  context = context.transpose(1, 2).contiguous().reshape({B, S, embed_dim});
  return o_proj.forward(context);
}

Tensor MultiHeadAttention::forward(const Tensor &input) { return forward(input, 0, nullptr, -1); }

// --------------------------------------------------------- TransformerBlock --
// src/nn/transforrmer_block.cpp:9-58
static std::string blk(int i, const char *name) { return "blk." + std::to_string(i) + "." + name; }

TransformerBlock::TransformerBlock(GGUFLoader &L, int i, size_t E, size_t H, size_t KVH, size_t max_seq, float theta)
    : attention_norm(L.get_tensor(blk(i, "attn_norm.weight"))),
      attention(L.get_tensor(blk(i, "attn_q.weight")), L.get_tensor(blk(i, "attn_k.weight")),
                L.get_tensor(blk(i, "attn_v.weight")), L.get_tensor(blk(i, "attn_output.weight")), E, H, KVH,
                max_seq, theta),
      ffn_norm(L.get_tensor(blk(i, "ffn_norm.weight"))),
      ffn(L.get_tensor(blk(i, "ffn_gate.weight")), L.get_tensor(blk(i, "ffn_down.weight")),
          L.get_tensor(blk(i, "ffn_up.weight"))) {}

TransformerBlock::TransformerBlock(size_t E, size_t H, size_t KVH, size_t inter, size_t max_seq, float theta)
    : attention_norm(E), attention(E, H, KVH, max_seq, theta), ffn_norm(E), ffn(E, inter) {}

Tensor TransformerBlock::forward(const Tensor &input, size_t position_offset, KVCache *kv_cache, int layer_idx) {
  Tensor norm_x = attention_norm.forward(input);
  Tensor attn_out = attention.forward(norm_x, position_offset, kv_cache, layer_idx);
  Tensor h = input + attn_out;
  Tensor norm_h = ffn_norm.forward(h);
  Tensor ffn_out = ffn.forward(norm_h);
  return h + ffn_out;
}

Tensor TransformerBlock::forward(const Tensor &input) { return forward(input, 0); }

}  // namespace nn
}  // namespace turbo
