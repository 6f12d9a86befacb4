// tb_selfcheck.cu -- device self-check of the exp implementations used by the
// softmax and SwiGLU kernels, over every fp32 bit pattern.  Test code: built
// into its own library (libturbo_b200_selfcheck.so), not the product one; it
// shares only the device functions of tb_internal.cuh.
#include "tb_internal.cuh"

namespace tb {
namespace {

// Distance in units in the last place between two floats (NaN == NaN; a NaN
// against a number counts as 2^32).
__device__ __forceinline__ unsigned long long ulp_dist(float a, float b) {
  const bool na = a != a, nb = b != b;
  if (na || nb) return (na && nb) ? 0ull : (1ull << 32);
  int32_t ia = __float_as_int(a), ib = __float_as_int(b);
  ia = ia < 0 ? (int32_t)(0x80000000u - (uint32_t)ia) : ia;  // -0.0 -> 0
  ib = ib < 0 ? (int32_t)(0x80000000u - (uint32_t)ib) : ib;
  const long long d = (long long)ia - (long long)ib;
  return (unsigned long long)(d < 0 ? -d : d);
}

// out[0]: inputs where exp_cr differs from exp_ref; out[1]: largest such
// distance (ulp); out[2]: inputs x in [-87, 0] where __expf (the softmax
// kernels' exp) is further from exp_ref than its documented 2 + 1.173|x| ulp;
// out[3]: its largest distance over x in [-20, 0].
__global__ void exp_check_kernel(unsigned long long *out) {
  __shared__ double tab[64];
  exp_cr_table_init(tab);
  __syncthreads();
  unsigned long long n_cr = 0, max_cr = 0, n_fast = 0, max_fast = 0;
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  for (unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; i < (1ull << 32);
       i += stride) {
    const float x = __uint_as_float((uint32_t)i);
    const float ref = exp_ref(x);
    const unsigned long long dc = ulp_dist(exp_cr(x, tab), ref);
    n_cr += dc != 0;
    max_cr = dc > max_cr ? dc : max_cr;
    if (x >= -87.0f && x <= 0.0f) {
      const unsigned long long df = ulp_dist(__expf(x), ref);
      n_fast += (double)df > 2.0 + floor(1.173 * fabs((double)x));
      if (x >= -20.0f) max_fast = df > max_fast ? df : max_fast;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    n_cr += __shfl_xor_sync(0xffffffffu, n_cr, o);
    n_fast += __shfl_xor_sync(0xffffffffu, n_fast, o);
    const unsigned long long a = __shfl_xor_sync(0xffffffffu, max_cr, o);
    const unsigned long long b = __shfl_xor_sync(0xffffffffu, max_fast, o);
    max_cr = a > max_cr ? a : max_cr;
    max_fast = b > max_fast ? b : max_fast;
  }
  if ((threadIdx.x & 31) == 0) {
    atomicAdd(out + 0, n_cr);
    atomicMax(out + 1, max_cr);
    atomicAdd(out + 2, n_fast);
    atomicMax(out + 3, max_fast);
  }
}

}  // namespace
}  // namespace tb

using namespace tb;

// counts[0]: inputs where exp_cr differs from the double-precision exp rounded
// to float; counts[1]: its largest distance in ulp; counts[2]: inputs in
// [-87, 0] where __expf exceeds its documented 2 + 1.173|x| ulp; counts[3]:
// its largest distance over [-20, 0].  Synchronous, on the current device.
// Returns TB_EINVAL for a null pointer, TB_ECUDA for a CUDA failure.
extern "C" __attribute__((visibility("default"))) int tb_selfcheck_exp(uint64_t *counts) {
  if (!counts) return TB_EINVAL;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  unsigned long long *d = nullptr;
  if (e == cudaSuccess) e = cudaMalloc(&d, 4 * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMemset(d, 0, 4 * sizeof(unsigned long long));
  if (e == cudaSuccess) {
    exp_check_kernel<<<sms * 8, 256>>>(d);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMemcpy(counts, d, 4 * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
  if (d) cudaFree(d);
  return e == cudaSuccess ? TB_OK : TB_ECUDA;
}
