// Test helper (built by tests/test_gpu_division.py): compares the quantizer's
// division (div_rn with __frcp_rn, innerq_b200/csrc/common.cuh) with CUDA's
// IEEE fp32 '/' for every fp16 numerator and every positive finite fp16
// divisor, bit for bit.
#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"

__global__ void div_check_kernel(unsigned long long* n_bad, unsigned int* first_bad) {
  const uint16_t bbits = (uint16_t)(blockIdx.x + 1);  // 0x0001 .. 0x7bff
  const float b = __half2float(__ushort_as_half(bbits));
  const float rb = __frcp_rn(b);
  unsigned long long bad = 0;
  for (int i = threadIdx.x; i < 2 * 0x7c00; i += blockDim.x) {
    const uint16_t abits = (uint16_t)(i < 0x7c00 ? i : 0x8000 + (i - 0x7c00));
    const float a = __half2float(__ushort_as_half(abits));
    const float want = a / b;
    const float got = innerq::div_rn(a, b, rb);
    if (__float_as_uint(want) != __float_as_uint(got)) {
      ++bad;
      atomicCAS(first_bad, 0xffffffffu, ((unsigned int)abits << 16) | bbits);
    }
  }
  if (bad) atomicAdd(n_bad, bad);
}

// the quantizers' constant divisors 2^k - 1, with the compile-time reciprocal
template <int Q>
__global__ void div_const_kernel(unsigned long long* n_bad, unsigned int* first_bad) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < 2 * 0x7c00; i += gridDim.x * blockDim.x) {
    const uint16_t abits = (uint16_t)(i < 0x7c00 ? i : 0x8000 + (i - 0x7c00));
    const float a = __half2float(__ushort_as_half(abits));
    if (__float_as_uint(a / (float)Q) != __float_as_uint(innerq::div_rn(a, (float)Q, 1.f / (float)Q))) {
      atomicAdd(n_bad, 1ull);
      atomicCAS(first_bad, 0xffffffffu, ((unsigned int)abits << 16) | Q);
    }
  }
}

extern "C" int div_check(unsigned long long* n_bad, unsigned int* first_bad) {
  unsigned long long* d_n;
  unsigned int* d_f;
  if (cudaMalloc(&d_n, sizeof(*d_n)) != cudaSuccess) return -1;
  if (cudaMalloc(&d_f, sizeof(*d_f)) != cudaSuccess) return -1;
  cudaMemset(d_n, 0, sizeof(*d_n));
  cudaMemset(d_f, 0xff, sizeof(*d_f));
  div_check_kernel<<<0x7bff, 256>>>(d_n, d_f);
  div_const_kernel<1><<<64, 256>>>(d_n, d_f);
  div_const_kernel<3><<<64, 256>>>(d_n, d_f);
  div_const_kernel<7><<<64, 256>>>(d_n, d_f);
  div_const_kernel<15><<<64, 256>>>(d_n, d_f);
  cudaError_t e = cudaDeviceSynchronize();
  cudaMemcpy(n_bad, d_n, sizeof(*d_n), cudaMemcpyDeviceToHost);
  cudaMemcpy(first_bad, d_f, sizeof(*d_f), cudaMemcpyDeviceToHost);
  cudaFree(d_n);
  cudaFree(d_f);
  return e == cudaSuccess ? 0 : -2;
}
