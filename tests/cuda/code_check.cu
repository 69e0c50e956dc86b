// Test helper (built by tests/test_gpu_division.py): the quantizers' codes
// from per-group cuts (code_cuts / code_by_cuts, innerq_b200/csrc/common.cuh)
// against rint(clamp(rnd_dt(a / s))) with CUDA's IEEE fp32 '/', for every
// non-negative finite fp16 (bf16) a and every positive finite fp16 (bf16) s,
// for qmax 1, 3, 7 and 15.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"

template <int DT, int QMAX>
__device__ unsigned long long check_one(float a, float s, const float* cut) {
  const int want = innerq::code_of(innerq::rnd<DT>(a / s), (float)QMAX);
  return innerq::code_by_cuts<QMAX>(a, cut) != want;
}

template <int DT>
__global__ void code_check_kernel(int n_a, unsigned long long* n_bad, unsigned int* first_bad) {
  constexpr int MB = DT == innerq::F16 ? 10 : 7;
  const uint16_t sbits = (uint16_t)(blockIdx.x + 1);
  const float s = innerq::to_f<DT>(sbits);
  const double sd = s;
  float c1[1], c3[3], c7[7], c15[15];
  innerq::code_cuts<MB, 1>(sd, c1);
  innerq::code_cuts<MB, 3>(sd, c3);
  innerq::code_cuts<MB, 7>(sd, c7);
  innerq::code_cuts<MB, 15>(sd, c15);
  unsigned long long bad = 0;
  for (int i = threadIdx.x; i < n_a; i += blockDim.x) {
    const float a = innerq::to_f<DT>((uint16_t)i);
    const unsigned long long b = check_one<DT, 1>(a, s, c1) + check_one<DT, 3>(a, s, c3) +
                                 check_one<DT, 7>(a, s, c7) + check_one<DT, 15>(a, s, c15);
    if (b) {
      bad += b;
      atomicCAS(first_bad, 0xffffffffu, ((unsigned int)i << 16) | sbits);
    }
  }
  if (bad) atomicAdd(n_bad, bad);
}

// dtype 0: fp16 (a, s up to 0x7bff), 1: bf16 (up to 0x7f7f)
extern "C" int code_check(int dtype, unsigned long long* n_bad, unsigned int* first_bad) {
  unsigned long long* d_n;
  unsigned int* d_f;
  if (cudaMalloc(&d_n, sizeof(*d_n)) != cudaSuccess) return -1;
  if (cudaMalloc(&d_f, sizeof(*d_f)) != cudaSuccess) return -1;
  cudaMemset(d_n, 0, sizeof(*d_n));
  cudaMemset(d_f, 0xff, sizeof(*d_f));
  if (dtype == 0) code_check_kernel<innerq::F16><<<0x7bff, 256>>>(0x7c00, d_n, d_f);
  else code_check_kernel<innerq::BF16><<<0x7f7f, 256>>>(0x7f80, d_n, d_f);
  cudaError_t e = cudaDeviceSynchronize();
  cudaMemcpy(n_bad, d_n, sizeof(*d_n), cudaMemcpyDeviceToHost);
  cudaMemcpy(first_bad, d_f, sizeof(*d_f), cudaMemcpyDeviceToHost);
  cudaFree(d_n);
  cudaFree(d_f);
  return e == cudaSuccess ? 0 : -2;
}
