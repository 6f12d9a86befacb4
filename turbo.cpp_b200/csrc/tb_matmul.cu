// tb_matmul.cu -- the quantized matmul entry point (Tensor::matmul Q8_0/Q4_0
// branches, src/tensor/tensor.cpp:328-432): shape checks and dispatch.
#include <algorithm>

#include "tb_internal.cuh"

namespace tb {
tb_status launch_q8_0(const float *x, int64_t M, int64_t K, const void *w, int64_t N, float *y,
                      bool exact, cudaStream_t s, const DeviceState *st);
tb_status launch_q4_0_exact(const uint8_t *xq, int64_t M, int64_t K, const void *w, int64_t N,
                            float *y, cudaStream_t s, const DeviceState *st);
bool gemm_f16_eligible(int64_t M, int64_t K, const float *x, const void *w);
tb_status launch_gemm_f16(int dtype, const float *x, int64_t M, int64_t K, const void *w, int64_t N, float *y,
                          cudaStream_t s, const DeviceState *st);
}  // namespace tb

using namespace tb;

namespace {
tb_status matmul_quant(int dtype, const float *x, int64_t M, int64_t K, const void *w, int64_t N,
                       float *y, bool exact, tb_stream stream) {
  if (dtype != TB_Q8_0 && dtype != TB_Q4_0)
    return fail(TB_EINVAL, "tb_matmul_quant: dtype must be TB_Q8_0 or TB_Q4_0");
  if (M < 0 || K < 0 || N < 0) return fail(TB_EINVAL, "tb_matmul_quant: negative extent");
  if (K % 32 != 0) return fail(TB_EINVAL, "tb_matmul_quant: K=%lld is not a multiple of 32", (long long)K);
  if (M == 0 || N == 0) return TB_OK;
  if (K == 0) return tb_memset(y, 0, (size_t)(M * N) * sizeof(float), stream);
  if (!x || !w || !y) return fail(TB_EINVAL, "tb_matmul_quant: null pointer");
  if (N > 0x7FFFFFFF || K > 0x7FFFFFFF || M > 0x7FFFFFFF) return fail(TB_EINVAL, "tb_matmul_quant: extent too large");
  DeviceState *st;
  TB_TRY(device_state(&st));
  cudaStream_t s = as_stream(stream);
  // prefill-sized M: tcgen05 tensor cores (within 1e-5 of sum |w x|)
  if (!exact && gemm_f16_eligible(M, K, x, w)) return launch_gemm_f16(dtype, x, M, K, w, N, y, s, st);
  if (dtype == TB_Q8_0) return launch_q8_0(x, M, K, w, N, y, exact, s, st);
  // Q4_0: X rows -> Q8_0 (tensor.cpp:413-421) into stream-ordered scratch.
  size_t xq_bytes = (size_t)M * (size_t)(K / 32) * 34;
  void *xq = nullptr;
  cudaError_t e = cudaMallocAsync(&xq, xq_bytes, s);
  if (e != cudaSuccess) return fail(TB_ENOMEM, "tb_matmul_quant: scratch of %zu bytes: %s", xq_bytes, cudaGetErrorString(e));
  tb_status rs = tb_quantize_q8_0(x, M, K, xq, stream);
  if (rs == TB_OK) rs = launch_q4_0_exact((const uint8_t *)xq, M, K, w, N, y, s, st);
  e = cudaFreeAsync(xq, s);
  if (rs == TB_OK && e != cudaSuccess) return fail(TB_ECUDA, "tb_matmul_quant: free scratch: %s", cudaGetErrorString(e));
  return rs;
}
}  // namespace

extern "C" tb_status tb_matmul_quant(int dtype, const float *x, int64_t M, int64_t K,
                                     const void *w, int64_t N, float *y, tb_stream stream) {
  return matmul_quant(dtype, x, M, K, w, N, y, false, stream);
}

extern "C" tb_status tb_matmul_quant_exact(int dtype, const float *x, int64_t M, int64_t K,
                                           const void *w, int64_t N, float *y, tb_stream stream) {
  return matmul_quant(dtype, x, M, K, w, N, y, true, stream);
}
