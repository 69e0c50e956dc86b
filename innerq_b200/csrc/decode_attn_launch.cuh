// Launch of one fused decode attention instantiation (shared by the
// decode_attn_k*_*.cu translation units, one per key width, dtype and
// geometry source, so the instantiations compile in parallel).
#pragma once
#include <cuda_runtime.h>

#include "decode_attn.cuh"
#include "innerq_internal.h"

namespace innerq {

template <int BK, int DT, int BV, int RP, int NG, int VCH, int GM, int VHY = 0, int KOT = 0>
cudaError_t attn_go(const DevArgs& a, dim3 grid, cudaStream_t s) {
  auto kern = decode_attn_kernel<BK, BV, RP, DT, NG, VCH, GM, VHY, KOT>;
  const int smem = attn_dyn_smem(BK, BV, NG, a.k.asym, a.v.asym, RP, VHY);
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

template <int BK, int DT, int BV, int RP, int GM>
cudaError_t attn_go_ng(const DevArgs& a, int ng, dim3 grid, cudaStream_t s) {
  // hybrid values (token groups; keys in groups of 32, argument-fed geometry)
  if (a.v.hyb) {
    if constexpr (GM == 0) {
      if (ng == 4 && !a.v.chan) return attn_go<BK, DT, BV, RP, 4, 0, 0, 1>(a, grid, s);
    }
    return cudaErrorNotSupported;
  }
  // keys grouped over tokens (KIVI): GQA <= 4 (make_plan)
  if (a.k.otok) {
    if constexpr (RP == 4) {
      return a.v.chan ? attn_go<BK, DT, BV, 4, 4, 1, GM, 0, 1>(a, grid, s) : attn_go<BK, DT, BV, 4, 4, 0, GM, 0, 1>(a, grid, s);
    }
    return cudaErrorNotSupported;
  }
  // value groups over tokens (VCH 0) or channels (VCH 1)
  switch (ng) {
    case 4: return a.v.chan ? attn_go<BK, DT, BV, RP, 4, 1, GM>(a, grid, s) : attn_go<BK, DT, BV, RP, 4, 0, GM>(a, grid, s);
    case 2: return a.v.chan ? attn_go<BK, DT, BV, RP, 2, 1, GM>(a, grid, s) : attn_go<BK, DT, BV, RP, 2, 0, GM>(a, grid, s);
    case 1: return a.v.chan ? attn_go<BK, DT, BV, RP, 1, 1, GM>(a, grid, s) : attn_go<BK, DT, BV, RP, 1, 0, GM>(a, grid, s);
    default: return cudaErrorNotSupported;
  }
}

template <int BK, int DT, int GM>
cudaError_t launch_attn(const DevArgs& a, int bv, int rp, int ng, dim3 grid, cudaStream_t s) {
  switch (bv) {
    case 2: return rp == 4 ? attn_go_ng<BK, DT, 2, 4, GM>(a, ng, grid, s) : attn_go_ng<BK, DT, 2, 8, GM>(a, ng, grid, s);
    case 3: return rp == 4 ? attn_go_ng<BK, DT, 3, 4, GM>(a, ng, grid, s) : attn_go_ng<BK, DT, 3, 8, GM>(a, ng, grid, s);
    case 4: return rp == 4 ? attn_go_ng<BK, DT, 4, 4, GM>(a, ng, grid, s) : attn_go_ng<BK, DT, 4, 8, GM>(a, ng, grid, s);
    default: return cudaErrorNotSupported;
  }
}

}  // namespace innerq
