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
    case 4: return launch_pdl(qprep_kernel<DT, RP, 4>, grid, dim3(kWarps * 32), 0, s, a);
    case 2: return launch_pdl(qprep_kernel<DT, RP, 2>, grid, dim3(kWarps * 32), 0, s, a);
    case 1: return launch_pdl(qprep_kernel<DT, RP, 1>, grid, dim3(kWarps * 32), 0, s, a);
    default: return cudaErrorNotSupported;
  }
}
}  // namespace

int64_t qprep_bytes(int rp) { return rp == 4 ? sizeof(QPrep<4>) : sizeof(QPrep<8>); }

cudaError_t launch_qprep(const DevArgs& a, int rp, int ng, int bf16, cudaStream_t s) {
  if (bf16) return rp == 4 ? go<BF16, 4>(a, ng, s) : go<BF16, 8>(a, ng, s);
  return rp == 4 ? go<F16, 4>(a, ng, s) : go<F16, 8>(a, ng, s);
}

}  // namespace innerq
