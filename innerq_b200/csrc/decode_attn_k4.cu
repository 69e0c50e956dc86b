// Instantiations of the fused decode attention kernel for 4-bit keys.
#include "decode_attn.cuh"
#include "innerq_internal.h"

namespace innerq {

template <int BV, int R>
static cudaError_t go(const DevArgs& a, int dt, dim3 grid, cudaStream_t s) {
  if (dt == F16)
    decode_attn_kernel<4, BV, R, F16><<<grid, kWarps * 32, 0, s>>>(a);
  else
    decode_attn_kernel<4, BV, R, BF16><<<grid, kWarps * 32, 0, s>>>(a);
  return cudaGetLastError();
}

template <int BV>
static cudaError_t go_r(const DevArgs& a, int R, int dt, dim3 grid, cudaStream_t s) {
  switch (R) {
    case 1: return go<BV, 1>(a, dt, grid, s);
    case 2: return go<BV, 2>(a, dt, grid, s);
    case 4: return go<BV, 4>(a, dt, grid, s);
    case 8: return go<BV, 8>(a, dt, grid, s);
    default: return cudaErrorNotSupported;
  }
}

cudaError_t launch_attn_k4(const DevArgs& a, int bv, int R, int dt, dim3 grid, cudaStream_t s) {
  switch (bv) {
    case 2: return go_r<2>(a, R, dt, grid, s);
    case 3: return go_r<3>(a, R, dt, grid, s);
    case 4: return go_r<4>(a, R, dt, grid, s);
    default: return cudaErrorNotSupported;
  }
}

}  // namespace innerq
