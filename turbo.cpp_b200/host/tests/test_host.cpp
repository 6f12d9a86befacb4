// test_host.cpp -- the reference's unit-test cases (tests/test_tensor.cpp,
// test_nn.cpp, test_rope.cpp, test_quant.cpp) and its exception semantics, run
// against the device Tensor/nn API.  Exit status = number of failed checks.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "turbo/core/kv_cache.hpp"
#include "turbo/core/sampler.hpp"
#include "turbo/nn/embedding.hpp"
#include "turbo/nn/linear.hpp"
#include "turbo/nn/rmsnorm.hpp"
#include "turbo/nn/rope.hpp"
#include "turbo/nn/softmax.hpp"
#include "turbo/nn/swiglu.hpp"
#include "turbo/tensor/tensor.hpp"

using namespace turbo;

static int g_fail = 0, g_pass = 0;
#define CHECK(cond, what)                                                  \
  do {                                                                     \
    if (cond) {                                                            \
      ++g_pass;                                                            \
    } else {                                                               \
      ++g_fail;                                                            \
      std::printf("FAIL %s:%d %s\n", __FILE__, __LINE__, what);            \
    }                                                                      \
  } while (0)
#define NEAR(a, b, tol, what) CHECK(std::fabs((double)(a) - (double)(b)) < (tol), what)
template <class E, class F> static bool throws(F f) {
  try {
    f();
  } catch (const E &) {
    return true;
  } catch (...) {
    return false;
  }
  return false;
}

static uint16_t f2h(float f) {  // float -> IEEE half (test values are exact halves)
  uint32_t x;
  std::memcpy(&x, &f, 4);
  uint32_t e = (x >> 23) & 0xFF, m = x & 0x7FFFFF;
  return (uint16_t)(((x >> 16) & 0x8000) | ((e - 112) << 10) | (m >> 13));
}

int main() {
  // test_tensor.cpp:11-44 NumericallyStableSoftmax
  {
    Tensor logits({1.0f, 2.0f, 3.0f, 10.0f, 100.0f, 10.0f}, {2, 3});
    nn::Softmax sm(-1);
    Tensor p = sm.forward(logits);
    const float expect[6] = {0.0900f, 0.2447f, 0.6652f, 0.0f, 1.0f, 0.0f};
    for (size_t i = 0; i < 6; ++i) NEAR(p.at({i / 3, i % 3}), expect[i], 1e-4, "softmax KAT");
    CHECK(throws<std::invalid_argument>([&] { sm.forward(Tensor()); }), "softmax of empty tensor");
  }
  // test_nn.cpp:8-42 LinearForwardPass (weights set through at(): host shadow)
  {
    nn::Linear lin(3, 2);
    lin.get_weight().at({0, 0}) = 1.0f;
    lin.get_weight().at({0, 1}) = 2.0f;
    lin.get_weight().at({1, 0}) = 3.0f;
    lin.get_weight().at({1, 1}) = 4.0f;
    lin.get_weight().at({2, 0}) = 5.0f;
    lin.get_weight().at({2, 1}) = 6.0f;
    lin.get_bias().at({0}) = 0.5f;
    lin.get_bias().at({1}) = -0.5f;
    Tensor X({1.0f, 1.0f, 1.0f, 2.0f, 0.0f, 1.0f}, {2, 3});
    Tensor Y = lin.forward(X);
    CHECK(Y.at({0, 0}) == 9.5f && Y.at({0, 1}) == 11.5f && Y.at({1, 0}) == 7.5f && Y.at({1, 1}) == 9.5f,
          "linear KAT");
  }
  // test_nn.cpp:44-79: the reference's 1-argument SwiGLU throws runtime_error
  {
    nn::SwiGLU sw;
    Tensor X({1.0f, 2.0f, 3.0f, 4.0f}, {1, 4});
    CHECK(throws<std::runtime_error>([&] { sw.forward(X); }), "swiglu 1-arg deprecated");
    Tensor g({1.0f, 2.0f}, {1, 2}), u({3.0f, 4.0f}, {1, 2});
    Tensor y = sw.forward(g, u);
    NEAR(y.at({0, 0}), 2.19317f, 1e-4, "swiglu value 0");
    NEAR(y.at({0, 1}), 7.04637f, 1e-4, "swiglu value 1");
    Tensor bad({1.0f, 2.0f, 3.0f}, {1, 3});
    CHECK(throws<std::invalid_argument>([&] { sw.forward(g, bad); }), "swiglu shape mismatch");
  }
  // test_nn.cpp:124-133 EmbeddingOutOfBounds
  {
    nn::Embedding emb(3, 4);
    Tensor bad({5.0f}, {1});
    CHECK(throws<std::out_of_range>([&] { emb.forward(bad); }), "embedding out of range");
    Tensor ids({0.0f, 2.0f}, {2});
    Tensor e = emb.forward(ids);
    CHECK(e.get_shape() == std::vector<size_t>({2, 4}) && e.at({1, 3}) == 0.0f, "embedding of zeros");
  }
  // test_nn.cpp:135-170 RMSNormForwardPass
  {
    nn::RMSNorm rms(4, 1e-5f);
    rms.get_weight().at({0}) = 0.5f;
    rms.get_weight().at({1}) = 1.0f;
    rms.get_weight().at({2}) = 1.5f;
    rms.get_weight().at({3}) = 2.0f;
    Tensor X({1.0f, 2.0f, 3.0f, 4.0f}, {1, 4});
    Tensor Y = rms.forward(X);
    NEAR(Y.at({0, 0}), 0.182574f, 1e-4, "rmsnorm 0");
    NEAR(Y.at({0, 1}), 0.730296f, 1e-4, "rmsnorm 1");
    NEAR(Y.at({0, 2}), 1.643167f, 1e-4, "rmsnorm 2");
    NEAR(Y.at({0, 3}), 2.921186f, 1e-4, "rmsnorm 3");
    Tensor wrong({1.0f, 2.0f, 3.0f}, {1, 3});
    CHECK(throws<std::invalid_argument>([&] { rms.forward(wrong); }), "rmsnorm hidden mismatch");
  }
  // test_rope.cpp:4-34 RoPEForwardPass
  {
    nn::RoPE rope(4, 10);
    Tensor X({1.0f, 2.0f, 3.0f, 4.0f, 1.0f, 2.0f, 3.0f, 4.0f}, {2, 4});
    rope.apply_in_place(X, 0);
    CHECK(X.at({0, 0}) == 1.0f && X.at({0, 1}) == 2.0f && X.at({0, 2}) == 3.0f && X.at({0, 3}) == 4.0f,
          "rope position 0 unchanged");
    NEAR(X.at({1, 0}), -1.9840f, 1e-3, "rope x0");
    NEAR(X.at({1, 2}), 2.4623f, 1e-3, "rope x2");
    CHECK(throws<std::out_of_range>([&] { rope.apply_in_place(X, 9); }), "rope past the table");
    CHECK(throws<std::invalid_argument>([&] { nn::RoPE odd(3, 4); }), "rope odd head dim");
  }
  // test_quant.cpp:7-32 / 34-65: block dot products that cancel to 0 (matmul form)
  {
    std::vector<uint8_t> q8(34);
    uint16_t h = f2h(0.5f);
    std::memcpy(q8.data(), &h, 2);
    for (int i = 0; i < 32; ++i) q8[2 + i] = (uint8_t)(int8_t)((i % 2 == 0) ? 2 : -2);
    Tensor W({32, 1}, DataType::Q8_0, q8.data());
    Tensor X(std::vector<float>(32, 1.0f), {1, 32});
    NEAR(X.matmul(W).at({0, 0}), 0.0f, 1e-5, "q8_0 dot KAT");
    std::vector<uint8_t> q4(18);
    std::memcpy(q4.data(), &h, 2);
    for (int i = 0; i < 16; ++i) q4[2 + i] = 0x6A;
    Tensor W4({32, 1}, DataType::Q4_0, q4.data());
    NEAR(X.matmul(W4).at({0, 0}), 0.0f, 1e-5, "q4_0 dot KAT");
  }
  // Tensor semantics the reference callers rely on (src/tensor/tensor.cpp)
  {
    Tensor a({1, 2, 3, 4, 5, 6}, {2, 3});
    Tensor e;
    Tensor s = e + a;  // operator+ returns the other operand when one is empty
    CHECK(s.get_storage() == a.get_storage(), "empty + a returns a");
    Tensor c = a.contiguous();
    CHECK(c.get_storage() == a.get_storage(), "contiguous() of a contiguous tensor shares storage");
    Tensor t = a.transpose();
    CHECK(throws<std::runtime_error>([&] { t.reshape({6}); }), "reshape of a non-contiguous view");
    Tensor tc = t.contiguous();
    CHECK(tc.at({2, 1}) == 6.0f && tc.at({0, 1}) == 4.0f, "contiguous of a transpose");
    CHECK(throws<std::out_of_range>([&] { a.transpose(0, 5); }), "transpose out of range");
    CHECK(throws<std::invalid_argument>([&] { a.slice(3, 0); }), "slice dim out of range");
    CHECK(throws<std::out_of_range>([&] { a.slice(0, 1, 3); }), "slice range out of range");
    Tensor row({10, 20, 30}, {3});
    Tensor b = a + row;  // broadcast
    CHECK(b.at({1, 2}) == 36.0f && b.at({0, 0}) == 11.0f, "broadcast add");
    Tensor bad({1, 2}, {2});
    CHECK(throws<std::invalid_argument>([&] { a + bad; }), "not broadcastable");
    Tensor m = a * 0.5f;
    CHECK(m.at({1, 1}) == 2.5f, "scalar multiply");
    Tensor z = Tensor::zeros({2, 3});
    CHECK(throws<std::invalid_argument>([&] { z.copy_(t); }), "copy_ shape mismatch");
    z.copy_(a);
    CHECK(z.at({1, 0}) == 4.0f, "copy_");
    CHECK(throws<std::invalid_argument>([&] { a.matmul(Tensor({1, 2}, {2})); }), "matmul rank < 2");
    Tensor p = a.matmul(a.transpose());
    CHECK(p.at({0, 0}) == 14.0f && p.at({1, 0}) == 32.0f && p.at({1, 1}) == 77.0f, "fp32 matmul");
  }
  // KV cache write through a slice view (attention.cpp:66-84)
  {
    KVCache kv(8, 1, 2, 4);
    Tensor k({1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16}, {1, 2, 2, 4});  // [B, S, H, D]
    Tensor kt = k.transpose(1, 2);  // [B, H, S, D]
    kv.get_k_cache(0).slice(0, 3, 5).copy_(kt.squeeze(0).transpose(0, 1));
    const Tensor &cache = kv.get_k_cache(0);
    CHECK(cache.at({3, 0, 0}) == 1.0f && cache.at({3, 1, 3}) == 8.0f && cache.at({4, 0, 0}) == 9.0f &&
              cache.at({2, 0, 0}) == 0.0f,
          "kv cache append");
  }
  // greedy_sample: first index of the maximum, NaN never wins
  {
    const float v[5] = {1.0f, 3.0f, NAN, 3.0f, -INFINITY};
    CHECK(greedy_sample(v, 5) == 1, "greedy_sample tie");
    const float w[3] = {NAN, -INFINITY, NAN};
    CHECK(greedy_sample(w, 3) == 0, "greedy_sample all NaN/-inf");
  }
  // sample_top_p: a nucleus of one is the greedy choice; equal probabilities go by id
  {
    const float v[6] = {0.5f, 2.0f, -1.0f, 7.0f, 1.0f, 6.5f};
    CHECK(sample_top_p(v, 6, 0.8f, 1e-6f) == 3, "sample_top_p tiny top_p");
    std::vector<float> flat(1000, 0.0f);
    Tensor logits(flat, {1, 1000});
    // 500 equal probabilities reach top_p 0.5; u = 0.25 takes the 125th of them
    CHECK(sample_top_p(logits, 1.0f, 0.5f, 0.25) == 124, "sample_top_p ties by id");
    CHECK(sample_top_p(logits, 1.0f, 0.5f, 0.0) == 0, "sample_top_p u = 0");
    bool in_nucleus = true;
    for (int i = 0; i < 20; ++i) in_nucleus = in_nucleus && sample_top_p(flat.data(), 1000, 1.0f, 0.5f) < 500;
    CHECK(in_nucleus, "sample_top_p host draws stay in the nucleus");
  }
  std::printf("%d passed, %d failed\n", g_pass, g_fail);
  return g_fail;
}
