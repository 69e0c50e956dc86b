// Decode attention for callers that cannot allocate device memory.
//
// Some hosts of this library cannot call cudaMalloc on the decode path: a
// runtime whose device memory is owned by a fixed arena handed out up front,
// or a serving loop that forbids allocation after warm-up so its memory
// footprint stays fixed.  innerq_decode_attn needs a caller-provided
// workspace for its split-KV partials; this variant takes its workspace from
// a fixed array in device memory that every GPU loading the library holds
// until the process exits.
#include <cuda_runtime.h>
#include <mutex>

#include "../../include/innerq_b200.h"
#include "innerq_internal.h"

namespace {

constexpr int64_t kScratchBytes = INNERQ_NOALLOC_SCRATCH_BYTES;

// Split-KV partials of innerq_decode_attn_noalloc.  In host code this name is
// only a stand-in for the symbol; the device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {nullptr};

}  // namespace

extern "C" {

int innerq_decode_attn_noalloc(const innerq_attn_args* args, void* out, int64_t o_sb,
                               int64_t o_sh, float* lse, void* stream) {
  // arguments first: a rejected call neither touches the scratch nor loads
  // the module that holds it; the plan's own status (INNERQ_ERR_ARG or
  // INNERQ_ERR_UNSUPPORTED) is returned unchanged
  const int rc = innerq_attn_plan(args, nullptr, nullptr);
  if (rc != INNERQ_OK) return rc;  // innerq_last_error() holds the reason
  const int64_t need = innerq_decode_attn_workspace(args);
  if (need < 0) return INNERQ_ERR_ARG;
  if (need > kScratchBytes) {
    return innerq::set_last_error(INNERQ_ERR_ARG,
             "noalloc: split-KV partials need %lld bytes, above the fixed %lld-byte scratch; pass a "
             "smaller n_splits or a smaller batch, or use innerq_decode_attn with a workspace",
             (long long)need, (long long)kScratchBytes);
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    return innerq::set_last_error(INNERQ_ERR_CUDA, "noalloc: no usable current CUDA device");
  }
  void* ptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_addr[dev]) {
      // once per device, with that device current
      cudaError_t e = cudaGetSymbolAddress(&g_addr[dev], g_scratch);
      if (e != cudaSuccess) {
        g_addr[dev] = nullptr;
        return innerq::set_last_error(INNERQ_ERR_CUDA, "noalloc: cudaGetSymbolAddress: %s",
                                      cudaGetErrorString(e));
      }
    }
    ptr = g_addr[dev];
  }
  // Every partial row is written by the attention pass before the merge reads
  // it, so nothing in the scratch has to start at zero.
  return innerq_decode_attn(args, ptr, kScratchBytes, out, o_sb, o_sh, lse, stream);
}

}  // extern "C"
