// Internal launcher declarations shared by the C-ABI layer (capi.cu) and the
// kernel translation units.  Not part of the public ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace innerq {
struct DevArgs;

cudaError_t launch_norm_factor(const void* x, int dt, int B, int H, int T, int64_t sb, int64_t sh,
                               int64_t st, void* f, cudaStream_t s);
cudaError_t launch_pack(const void* x, int dt, int B, int H, int T, int64_t sb, int64_t sh,
                        int64_t st, int bits, int group, int asym, int role_v, int over_token,
                        const void* nf, void* codes, void* scale, void* zero, int64_t cap_tiles,
                        int64_t t_off, cudaStream_t s);
cudaError_t launch_unpack_ref(const void* codes, const void* scale, const void* zero, int dt, int B,
                              int H, int64_t n, int bits, int group, int asym, int role_v,
                              int over_token, int64_t cap_tiles, int64_t t_begin, int32_t* oc,
                              void* os, void* osc, void* oz, cudaStream_t s);
cudaError_t launch_dequant(const void* codes, const void* scale, const void* zero, int dt, int B,
                           int H, int64_t n, int bits, int group, int asym, int role_v,
                           int over_token, int64_t cap_tiles, int64_t t_begin, const void* nf,
                           void* out, int64_t ob, int64_t oh, int64_t ot, cudaStream_t s);
cudaError_t launch_lse_merge(const float* po, const float* pm, const float* pl, int rows,
                             int rows_per_b, int n_splits, int dt, void* out, int64_t o_b,
                             int64_t o_h, float* lse, cudaStream_t s, int n_ranks = 1,
                             int64_t rank_stride = 0);
cudaError_t launch_dequant_ref(const int32_t* c, const void* s, const void* zs, int dt, int64_t n_outer,
                               int T, int D, int group, int asym, int over_token, float* out,
                               cudaStream_t st);
// record the message innerq_last_error() returns on this thread; returns code
int set_last_error(int code, const char* fmt, ...);
// decode attention, one translation unit per (K bits, dtype); rp = query heads
// per KV head padded to 4 or 8, ng = K channel groups per token (4, 2, 1)
#define INNERQ_DECL_ATTN(name) \
  cudaError_t name(const DevArgs& a, int bv, int rp, int ng, dim3 grid, cudaStream_t s);
INNERQ_DECL_ATTN(launch_attn_k2_f16)
INNERQ_DECL_ATTN(launch_attn_k2_bf16)
INNERQ_DECL_ATTN(launch_attn_k3_f16)
INNERQ_DECL_ATTN(launch_attn_k3_bf16)
INNERQ_DECL_ATTN(launch_attn_k4_f16)
INNERQ_DECL_ATTN(launch_attn_k4_bf16)
INNERQ_DECL_ATTN(launch_attn_k2_f16_graph)
INNERQ_DECL_ATTN(launch_attn_k2_bf16_graph)
INNERQ_DECL_ATTN(launch_attn_k3_f16_graph)
INNERQ_DECL_ATTN(launch_attn_k3_bf16_graph)
INNERQ_DECL_ATTN(launch_attn_k4_f16_graph)
INNERQ_DECL_ATTN(launch_attn_k4_bf16_graph)
#undef INNERQ_DECL_ATTN
// graph-mode decode append of one side (quant_pack.cu); mode 0: channel
// groups / row layout, 1: token groups / col layout, 2: channel groups / col
// layout, 3: no quantization
struct AppendArgs {
  const void* x; int64_t x_sb, x_sh;
  void* fifo; int64_t f_sb, f_sh, f_st; int fifo_cap;
  void* codes; void* scale; void* zero; int64_t cap_tiles;
  const void* norm_f;
  int dt, B, H, bits, group, asym, mode, flush, n_q, n_rec, r0, max_steps;
};
cudaError_t launch_append_step(const AppendArgs& a, const int64_t* step, cudaStream_t s);
// the query-prep pass that precedes every attention launch (qprep.cu)
cudaError_t launch_qprep(const DevArgs& a, int rp, int ng, int bf16, cudaStream_t s);
int64_t qprep_bytes(int rp);  // one (batch, KV head) block
}  // namespace innerq
