// Fused decode attention instantiations: 2-bit keys, BF16 activations, graph mode (geometry from the device step counter).
#include "decode_attn_launch.cuh"

namespace innerq {

cudaError_t launch_attn_k2_bf16_graph(const DevArgs& a, int bv, int rp, int ng, dim3 grid, cudaStream_t s) {
  return launch_attn<2, BF16, 1>(a, bv, rp, ng, grid, s);
}

}  // namespace innerq
