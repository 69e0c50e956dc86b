// Instantiations of the query-prep kernel that runs before every attention
// pass (one CTA per (batch, KV head)).
#include <cuda_runtime.h>

#include "decode_attn.cuh"
#include "innerq_internal.h"

namespace innerq {

namespace {
template <int DT, int RP>
cudaError_t go(const DevArgs& a, int ng, cudaStream_t s) {
  const dim3 grid(a.Hkv, a.B, 1);
  switch (ng) {
    case 4: qprep_kernel<DT, RP, 4><<<grid, kWarps * 32, 0, s>>>(a); break;
    case 2: qprep_kernel<DT, RP, 2><<<grid, kWarps * 32, 0, s>>>(a); break;
    case 1: qprep_kernel<DT, RP, 1><<<grid, kWarps * 32, 0, s>>>(a); break;
    default: return cudaErrorNotSupported;
  }
  return cudaGetLastError();
}
}  // namespace

int64_t qprep_bytes(int rp) { return rp == 4 ? sizeof(QPrep<4>) : sizeof(QPrep<8>); }

cudaError_t launch_qprep(const DevArgs& a, int rp, int ng, int bf16, cudaStream_t s) {
  if (bf16) return rp == 4 ? go<BF16, 4>(a, ng, s) : go<BF16, 8>(a, ng, s);
  return rp == 4 ? go<F16, 4>(a, ng, s) : go<F16, 8>(a, ng, s);
}

}  // namespace innerq
