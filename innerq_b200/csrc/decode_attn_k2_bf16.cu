// Instantiations of the fused decode attention kernel: 2-bit keys, BF16 activations.
#include <cuda_runtime.h>

#include "decode_attn.cuh"
#include "innerq_internal.h"

namespace innerq {

namespace {
template <int BV, int RP, int NG, int VCH>
cudaError_t go(const DevArgs& a, dim3 grid, cudaStream_t s) {
  auto kern = decode_attn_kernel<2, BV, RP, BF16, NG, VCH>;
  const int smem = attn_dyn_smem(2, BV, NG, a.k.asym, a.v.asym, RP);
  int dev = 0;
  cudaGetDevice(&dev);
  static int set_bytes[64] = {0};
  if (dev >= 0 && dev < 64 && smem > set_bytes[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    set_bytes[dev] = smem;
  }
  return launch_after_prep(kern, grid, smem, s, a);
}

template <int BV, int RP>
cudaError_t go_ng(const DevArgs& a, int ng, dim3 grid, cudaStream_t s) {
  switch (ng) {
    case 4: return a.v.chan ? go<BV, RP, 4, 1>(a, grid, s) : go<BV, RP, 4, 0>(a, grid, s);
    case 2: return a.v.chan ? go<BV, RP, 2, 1>(a, grid, s) : go<BV, RP, 2, 0>(a, grid, s);
    case 1: return a.v.chan ? go<BV, RP, 1, 1>(a, grid, s) : go<BV, RP, 1, 0>(a, grid, s);
    default: return cudaErrorNotSupported;
  }
}

template <int BV>
cudaError_t go_r(const DevArgs& a, int rp, int ng, dim3 grid, cudaStream_t s) {
  return rp == 4 ? go_ng<BV, 4>(a, ng, grid, s) : go_ng<BV, 8>(a, ng, grid, s);
}
}  // namespace

cudaError_t launch_attn_k2_bf16(const DevArgs& a, int bv, int rp, int ng, dim3 grid, cudaStream_t s) {
  switch (bv) {
    case 2: return go_r<2>(a, rp, ng, grid, s);
    case 3: return go_r<3>(a, rp, ng, grid, s);
    case 4: return go_r<4>(a, rp, ng, grid, s);
    default: return cudaErrorNotSupported;
  }
}

}  // namespace innerq
