// Fused decode attention instantiations: 3-bit keys, F16 activations, graph mode (geometry from the device step counter).
#include "decode_attn_launch.cuh"

namespace innerq {

cudaError_t launch_attn_k3_f16_graph(const DevArgs& a, int bv, int rp, int ng, dim3 grid, cudaStream_t s) {
  return launch_attn<3, F16, 1>(a, bv, rp, ng, grid, s);
}

}  // namespace innerq
