// Fused decode attention instantiations: 3-bit keys, F16 activations, geometry from the launch arguments.
#include "decode_attn_launch.cuh"

namespace innerq {

cudaError_t launch_attn_k3_f16(const DevArgs& a, int bv, int rp, int ng, dim3 grid, cudaStream_t s) {
  return launch_attn<3, F16, 0>(a, bv, rp, ng, grid, s);
}

}  // namespace innerq
