// Fused decode attention instantiations: 4-bit keys, BF16 activations, geometry from the launch arguments.
#include "decode_attn_launch.cuh"

namespace innerq {

cudaError_t launch_attn_k4_bf16(const DevArgs& a, int bv, int rp, int ng, dim3 grid, cudaStream_t s) {
  return launch_attn<4, BF16, 0>(a, bv, rp, ng, grid, s);
}

}  // namespace innerq
