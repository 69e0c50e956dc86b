// Fused decode attention instantiations: 4-bit keys, BF16 activations, graph mode (geometry from the device step counter).
#include "decode_attn_launch.cuh"

namespace innerq {

cudaError_t launch_attn_k4_bf16_graph(const DevArgs& a, int bv, int rp, int ng, dim3 grid, cudaStream_t s) {
  return launch_attn<4, BF16, 1>(a, bv, rp, ng, grid, s);
}

}  // namespace innerq
