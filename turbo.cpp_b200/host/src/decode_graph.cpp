// decode_graph.cpp -- DecodeGraph: one greedy decode step of MiniGPT captured
// as a CUDA graph (see turbo/core/decode_graph.hpp).
#include "turbo/core/decode_graph.hpp"

#include <cmath>
#include <stdexcept>
#include <string>
#include <vector>

#include "host_util.hpp"
#include "turbo/core/kv_cache.hpp"
#include "turbo/model/minigpt.hpp"

using turbo::detail::tb_check;
using turbo::detail::tb_dtype_of;

namespace turbo {

namespace {
bool g_persistent = false;
}
void set_persistent_decode(bool on) { g_persistent = on; }
bool persistent_decode() { return g_persistent; }

void *DecodeGraph::buf(size_t bytes) {
  if (n_arena_ >= (int)(sizeof(arena_) / sizeof(arena_[0])))
    throw std::runtime_error("DecodeGraph: too many device buffers");
  void *p = nullptr;
  tb_check(tb_alloc(&p, bytes));
  arena_[n_arena_++] = p;
  return p;
}

DecodeGraph::DecodeGraph(MiniGPT &model, KVCache &kv, bool want_margins, float temperature, float top_p)
    : m_(model), kv_(kv), margins_on_(want_margins), temperature_(temperature), top_p_(top_p) {
  if (m_.blocks.empty()) throw std::invalid_argument("DecodeGraph: the model has no blocks");
  const Tensor &emb = m_.tok_emb.get_weight();
  E_ = emb.get_shape()[0];
  V_ = emb.get_shape()[1];
  H_ = m_.num_heads_;
  KVH_ = m_.num_kv_heads_;
  D_ = m_.head_dim_;
  F_ = m_.blocks[0].ffn.gate_proj.get_weight().get_shape()[1];
  max_seq_ = kv.get_max_seq_len();
  scale_ = 1.0f / std::sqrt(static_cast<float>(D_));
  if (H_ * D_ != E_ || H_ % KVH_ != 0) throw std::invalid_argument("DecodeGraph: inconsistent head layout");
  if (m_.lm_head.get_weight().get_shape()[1] != V_) throw std::invalid_argument("DecodeGraph: LM head width");
  for (auto &b : m_.blocks)
    for (nn::Linear *l : {&b.attention.q_proj, &b.attention.k_proj, &b.attention.v_proj, &b.attention.o_proj,
                          &b.ffn.gate_proj, &b.ffn.up_proj, &b.ffn.down_proj})
      if (!l->get_bias().is_empty()) throw std::invalid_argument("DecodeGraph: biased projections unsupported");
  // the fused step needs Q8_0 projections with rows of whole 16-byte words
  fused_ = !exact_matmul() && D_ == 64;
  auto q8 = [&](nn::Linear &l) {
    const Tensor &w = l.get_weight();
    return w.dtype() == DataType::Q8_0 && w.get_shape()[0] % 256 == 0;
  };
  for (auto &b : m_.blocks)
    fused_ = fused_ && q8(b.attention.q_proj) && q8(b.attention.k_proj) && q8(b.attention.v_proj) &&
             q8(b.attention.o_proj) && q8(b.ffn.gate_proj) && q8(b.ffn.up_proj) && q8(b.ffn.down_proj);
  fused_ = fused_ && q8(m_.lm_head);
  tb_check(tb_stream_create(&stream_));
  ids_ = static_cast<int32_t *>(buf(16));
  pos_ = static_cast<int32_t *>(buf(16));
  idx_ = static_cast<int64_t *>(buf(16));
  hist_ = static_cast<int32_t *>(buf(sizeof(int32_t) * (size_t)max_seq_));
  if (temperature_ > 0.f) uniform_ = static_cast<double *>(buf(sizeof(double) * (size_t)max_seq_));
  margins_ = static_cast<float *>(buf(sizeof(float) * (size_t)max_seq_));
  const size_t f = sizeof(float);
  x_ = static_cast<float *>(buf(f * E_));
  xn_ = static_cast<float *>(buf(f * E_));
  h_ = static_cast<float *>(buf(f * E_));
  q_ = static_cast<float *>(buf(f * E_));
  k_ = static_cast<float *>(buf(f * KVH_ * D_));
  v_ = static_cast<float *>(buf(f * KVH_ * D_));
  ctx_ = static_cast<float *>(buf(f * E_));
  ao_ = static_cast<float *>(buf(f * E_));
  g_ = static_cast<float *>(buf(f * F_));
  u_ = static_cast<float *>(buf(f * F_));
  sw_ = static_cast<float *>(buf(f * F_));
  fo_ = static_cast<float *>(buf(f * E_));
  logits_ = static_cast<float *>(buf(f * V_));
  if (fused_ && persistent_decode()) setup_persistent();
}

// The single-kernel step needs hidden 2048, head_dim 64, ffn 2048/4096/8192,
// <= 4 query heads per key/value head, max_seq <= 2048, Q8_0 embedding and LM
// head, one epsilon per norm kind; otherwise the fused graph stays in use.
void DecodeGraph::setup_persistent() {
  const Tensor &emb = m_.tok_emb.get_weight();
  const Tensor &lm = m_.lm_head.get_weight();
  const nn::TransformerBlock &b0 = m_.blocks[0];
  bool ok = E_ == 2048 && D_ == 64 && (F_ == 2048 || F_ == 4096 || F_ == 8192) && H_ / KVH_ <= 4 && KVH_ <= 56 &&
            max_seq_ <= 2048 && emb.dtype() == DataType::Q8_0 && lm.dtype() == DataType::Q8_0 &&
            (reinterpret_cast<uintptr_t>(lm.get_storage()->device_data()) & 15) == 0 &&
            (reinterpret_cast<uintptr_t>(emb.get_storage()->device_data()) & 15) == 0;
  for (const auto &b : m_.blocks)
    ok = ok && b.attention_norm.epsilon == b0.attention_norm.epsilon && b.ffn_norm.epsilon == b0.ffn_norm.epsilon;
  if (!ok) return;
  std::vector<tb_decode_layer> layers(m_.blocks.size());
  auto wptr = [](nn::Linear &l) { return (const void *)l.get_weight().get_storage()->device_data(); };
  for (size_t l = 0; l < m_.blocks.size(); ++l) {
    nn::TransformerBlock &b = m_.blocks[l];
    tb_decode_layer &d = layers[l];
    d.wq = wptr(b.attention.q_proj);
    d.wk = wptr(b.attention.k_proj);
    d.wv = wptr(b.attention.v_proj);
    d.wo = wptr(b.attention.o_proj);
    d.w_gate = wptr(b.ffn.gate_proj);
    d.w_up = wptr(b.ffn.up_proj);
    d.w_down = wptr(b.ffn.down_proj);
    d.attn_norm = static_cast<const float *>(b.attention_norm.get_weight().device_ptr());
    d.ffn_norm = static_cast<const float *>(b.ffn_norm.get_weight().device_ptr());
    d.k_cache = static_cast<float *>(kv_.get_k_cache((int)l).device_ptr());
    d.v_cache = static_cast<float *>(kv_.get_v_cache((int)l).device_ptr());
  }
  tb_decode_layer *ldev = static_cast<tb_decode_layer *>(buf(sizeof(tb_decode_layer) * layers.size()));
  tb_check(tb_upload(ldev, layers.data(), sizeof(tb_decode_layer) * layers.size(), stream_));
  nn::MultiHeadAttention &a0 = m_.blocks[0].attention;
  tb_decode_model &pm = pm_;
  pm.n_layers = (int32_t)m_.blocks.size();
  pm.hidden = (int64_t)E_;
  pm.ffn = (int64_t)F_;
  pm.heads = (int64_t)H_;
  pm.kv_heads = (int64_t)KVH_;
  pm.head_dim = (int64_t)D_;
  pm.vocab = (int64_t)V_;
  pm.max_seq = max_seq_;
  pm.rope_max_seq = (int64_t)a0.rope.max_seq_len;
  pm.eps_attn = b0.attention_norm.epsilon;
  pm.eps_ffn = b0.ffn_norm.epsilon;
  pm.eps_final = m_.norm.epsilon;
  pm.attn_scale = scale_;
  pm.layers_dev = ldev;
  pm.tok_emb = emb.get_storage()->device_data();
  pm.lm_head = lm.get_storage()->device_data();
  pm.final_norm = static_cast<const float *>(m_.norm.get_weight().device_ptr());
  pm.rope_cos = static_cast<const float *>(a0.rope.dev_cos->device_ptr());
  pm.rope_sin = static_cast<const float *>(a0.rope.dev_sin->device_ptr());
  pm.token_dev = ids_;
  pm.pos_dev = pos_;
  pm.logits = logits_;
  size_t ws = 0;
  tb_check(tb_decode_workspace_bytes(&pm, &ws));
  pm.workspace = buf(ws);
  pm.workspace_bytes = ws;
  tb_check(tb_memset(pm.workspace, 0, ws, stream_));
  tb_check(tb_sync(stream_));
  persistent_ = true;
}

void DecodeGraph::enqueue_step_persistent() {
  tb_check(tb_decode_step_persistent(&pm_, stream_));
  enqueue_pick(stream_);
}

DecodeGraph::~DecodeGraph() {
  if (graph_) tb_graph_destroy(graph_);
  if (stream_) {
    tb_sync(stream_);
    tb_stream_destroy(stream_);
  }
  for (int i = 0; i < n_arena_; ++i) tb_free(arena_[i]);
}

namespace {
// y[1, N] = x[1, K] . W for the projection's quantized (or fp32) weight.
void linear(nn::Linear &l, const float *x, float *y, tb_stream s) {
  const Tensor &w = l.get_weight();
  const int64_t K = (int64_t)w.get_shape()[0], N = (int64_t)w.get_shape()[1];
  const int dt = tb_dtype_of(w.dtype());
  if (dt != TB_Q8_0 && dt != TB_Q4_0) throw std::invalid_argument("DecodeGraph: projection weights must be Q8_0/Q4_0");
  if (exact_matmul())
    tb_check(tb_matmul_quant_exact(dt, x, 1, K, w.get_storage()->device_data(), N, y, s));
  else
    tb_check(tb_matmul_quant(dt, x, 1, K, w.get_storage()->device_data(), N, y, s));
}

tb_view vec_view(const float *p, int64_t n) {
  tb_view v{};
  v.data = const_cast<float *>(p);
  v.dtype = TB_F32;
  v.rank = 2;
  v.shape[0] = 1;
  v.shape[1] = n;
  v.strides[0] = n;
  v.strides[1] = 1;
  return v;
}

// [1, heads, 1, D] over a contiguous [heads * D] vector: the B, H, S, D view
// RoPE::apply_in_place receives from attention.cpp for one token.
tb_view head_view(float *p, int64_t heads, int64_t D) {
  tb_view v{};
  v.data = p;
  v.dtype = TB_F32;
  v.rank = 4;
  v.shape[0] = 1;
  v.shape[1] = heads;
  v.shape[2] = 1;
  v.shape[3] = D;
  v.strides[0] = heads * D;
  v.strides[1] = D;
  v.strides[2] = heads * D;
  v.strides[3] = 1;
  return v;
}
}  // namespace

void DecodeGraph::enqueue_step_fused() {
  tb_stream s = stream_;
  const int64_t E = (int64_t)E_, F = (int64_t)F_, V = (int64_t)V_, KV = (int64_t)(KVH_ * D_);
  auto wptr = [](nn::Linear &l) { return (const void *)l.get_weight().get_storage()->device_data(); };
  auto gptr = [](nn::RMSNorm &n) { return static_cast<const float *>(n.get_weight().device_ptr()); };
  const Tensor &emb = m_.tok_emb.get_weight();
  tb_check(tb_embedding(tb_dtype_of(emb.dtype()), emb.get_storage()->device_data(), E, V, ids_, 1, x_, s));
  for (size_t l = 0; l < m_.blocks.size(); ++l) {
    nn::TransformerBlock &b = m_.blocks[l];
    nn::MultiHeadAttention &a = b.attention;
    tb_gemv_segment qkv[3] = {{wptr(a.q_proj), E, q_, nullptr},
                              {wptr(a.k_proj), KV, k_, nullptr},
                              {wptr(a.v_proj), KV, v_, nullptr}};
    tb_check(tb_gemv_q8_0_multi(x_, E, gptr(b.attention_norm), b.attention_norm.epsilon, qkv, 3, s));
    float *kc = static_cast<float *>(kv_.get_k_cache((int)l).device_ptr());
    float *vc = static_cast<float *>(kv_.get_v_cache((int)l).device_ptr());
    tb_check(tb_rope_attention_decode(q_, k_, v_, (int64_t)H_, (int64_t)KVH_, (int64_t)D_,
                                      static_cast<const float *>(a.rope.dev_cos->device_ptr()),
                                      static_cast<const float *>(a.rope.dev_sin->device_ptr()),
                                      (int64_t)a.rope.max_seq_len, kc, vc, max_seq_, scale_, pos_, ctx_, s));
    tb_gemv_segment o = {wptr(a.o_proj), E, h_, x_};  // h = x + O ctx
    tb_check(tb_gemv_q8_0_multi(ctx_, E, nullptr, 0.f, &o, 1, s));
    tb_check(tb_gemv_q8_0_swiglu(h_, E, gptr(b.ffn_norm), b.ffn_norm.epsilon, wptr(b.ffn.gate_proj),
                                 wptr(b.ffn.up_proj), F, sw_, s));
    tb_gemv_segment d = {wptr(b.ffn.down_proj), E, x_, h_};  // x = h + down sw
    tb_check(tb_gemv_q8_0_multi(sw_, F, nullptr, 0.f, &d, 1, s));
  }
  // the LM head (128256 rows) runs faster on the tensor-core GEMV than fused
  tb_check(tb_rmsnorm(TB_F32, x_, gptr(m_.norm), xn_, 1, E, m_.norm.epsilon, s));
  linear(m_.lm_head, xn_, logits_, s);
  enqueue_pick(s);
}

void DecodeGraph::enqueue_step() {
  if (persistent_) return enqueue_step_persistent();
  if (fused_) return enqueue_step_fused();
  tb_stream s = stream_;
  const int64_t E = (int64_t)E_, F = (int64_t)F_, V = (int64_t)V_;
  const Tensor &emb = m_.tok_emb.get_weight();
  tb_check(tb_embedding(tb_dtype_of(emb.dtype()), emb.get_storage()->device_data(), E, V, ids_, 1, x_, s));
  for (size_t l = 0; l < m_.blocks.size(); ++l) {
    nn::TransformerBlock &b = m_.blocks[l];
    nn::MultiHeadAttention &a = b.attention;
    tb_check(tb_rmsnorm(TB_F32, x_, static_cast<const float *>(b.attention_norm.get_weight().device_ptr()), xn_, 1,
                        E, b.attention_norm.epsilon, s));
    linear(a.q_proj, xn_, q_, s);
    linear(a.k_proj, xn_, k_, s);
    linear(a.v_proj, xn_, v_, s);
    const float *cs = static_cast<const float *>(a.rope.dev_cos->device_ptr());
    const float *sn = static_cast<const float *>(a.rope.dev_sin->device_ptr());
    tb_view vq = head_view(q_, (int64_t)H_, (int64_t)D_), vk = head_view(k_, (int64_t)KVH_, (int64_t)D_);
    tb_check(tb_rope_at(&vq, cs, sn, (int64_t)D_, (int64_t)a.rope.max_seq_len, pos_, s));
    tb_check(tb_rope_at(&vk, cs, sn, (int64_t)D_, (int64_t)a.rope.max_seq_len, pos_, s));
    float *kc = static_cast<float *>(kv_.get_k_cache((int)l).device_ptr());
    float *vc = static_cast<float *>(kv_.get_v_cache((int)l).device_ptr());
    tb_check(tb_kv_append(kc, vc, k_, v_, (int64_t)(KVH_ * D_), max_seq_, pos_, s));
    tb_check(tb_attention_decode(q_, kc, vc, (int64_t)H_, (int64_t)KVH_, (int64_t)D_, max_seq_, scale_, pos_, ctx_, s));
    linear(a.o_proj, ctx_, ao_, s);
    tb_view vx = vec_view(x_, E), va = vec_view(ao_, E), vh = vec_view(h_, E);
    tb_check(tb_binary(0, &vx, &va, &vh, s));
    tb_check(tb_rmsnorm(TB_F32, h_, static_cast<const float *>(b.ffn_norm.get_weight().device_ptr()), xn_, 1, E,
                        b.ffn_norm.epsilon, s));
    linear(b.ffn.gate_proj, xn_, g_, s);
    linear(b.ffn.up_proj, xn_, u_, s);
    tb_check(tb_swiglu(TB_F32, g_, u_, sw_, F, s));
    linear(b.ffn.down_proj, sw_, fo_, s);
    tb_view vf = vec_view(fo_, E);
    tb_check(tb_binary(0, &vh, &vf, &vx, s));
  }
  tb_check(tb_rmsnorm(TB_F32, x_, static_cast<const float *>(m_.norm.get_weight().device_ptr()), xn_, 1, E,
                      m_.norm.epsilon, s));
  linear(m_.lm_head, xn_, logits_, s);
  enqueue_pick(s);
}

void DecodeGraph::enqueue_pick(tb_stream s) {
  const int64_t V = (int64_t)V_;
  if (uniform_)
    tb_check(tb_sample_top_p_at(logits_, V, temperature_, top_p_, uniform_, pos_, max_seq_, idx_, s));
  else
    tb_check(tb_argmax(logits_, 1, V, idx_, s));
  if (margins_on_) tb_check(tb_decode_margin(logits_, V, idx_, pos_, max_seq_, margins_, s));
  tb_check(tb_decode_advance(idx_, ids_, pos_, hist_, max_seq_, s));
}

void DecodeGraph::generate(int first, size_t steps, int *out_ids, float *margins, const double *uniforms) {
  if (steps == 0) return;
  if (uniform_ && !uniforms) throw std::invalid_argument("DecodeGraph: sampling needs a uniform number per step");
  const int pos0 = kv_.get_current_seq_len();
  if (first < 0 || (size_t)first >= V_)
    throw std::out_of_range("Token ID " + std::to_string(first) + " exceeds vocabulary size " + std::to_string(V_));
  if ((size_t)pos0 + steps > (size_t)max_seq_) throw std::out_of_range("KV cache is full.");
  uint32_t flags = 0;
  tb_check(tb_take_device_errors(&flags));  // start from a clean error word
  const int32_t init[2] = {first, pos0};
  tb_check(tb_upload(ids_, &init[0], sizeof(int32_t), stream_));
  tb_check(tb_upload(pos_, &init[1], sizeof(int32_t), stream_));
  if (uniform_) tb_check(tb_upload(uniform_ + pos0, uniforms, sizeof(double) * steps, stream_));
  // the first step runs eagerly: it sets every kernel's attributes before capture
  enqueue_step();
  if (steps > 1) {
    if (!graph_) {
      tb_check(tb_capture_begin(stream_));
      try {
        enqueue_step();
      } catch (...) {
        tb_graph g = nullptr;
        tb_capture_end(stream_, &g);
        if (g) tb_graph_destroy(g);
        throw;
      }
      tb_check(tb_capture_end(stream_, &graph_));
    }
    for (size_t i = 1; i < steps; ++i) tb_check(tb_graph_launch(graph_, stream_));
  }
  std::vector<int32_t> hist(steps);
  tb_check(tb_download(hist.data(), hist_ + pos0, sizeof(int32_t) * steps, stream_));
  if (margins) tb_check(tb_download(margins, margins_ + pos0, sizeof(float) * steps, stream_));
  tb_check(tb_sync(stream_));
  tb_check(tb_take_device_errors(&flags));
  if (flags & 2u) throw std::out_of_range("Sequence position exceeds RoPE cache size.");
  if (flags) throw std::runtime_error("DecodeGraph: device error flags " + std::to_string(flags));
  for (size_t i = 0; i < steps; ++i) out_ids[i] = hist[i];
  kv_.increment_seq_len((int)steps);
}

}  // namespace turbo
