/*
 * innerq_b200 — C ABI of the B200 (sm_100a) InnerQ decode hot path.
 *
 * Every entry point takes plain device pointers, sizes and element strides,
 * enqueues work on the caller's CUDA stream (`stream`, a cudaStream_t passed
 * as void*; NULL = the legacy default stream) and allocates nothing.  Every
 * entry point returns INNERQ_OK (0) or a negative INNERQ_ERR_* status;
 * innerq_last_error() then describes the failure (per calling thread).
 *
 * Geometry: head_dim D must be 128.  Tensors named [B][H][T][D] are indexed
 * with element strides (sb, sh, st) and a contiguous last dimension.
 * Element types are 16-bit: `dtype` = INNERQ_DT_F16 or INNERQ_DT_BF16 for the
 * model activations and for stored scales / zero points / normalisation
 * factors (the reference keeps those in the input dtype).
 *
 * Packed store of one of K or V ("side"), per (b, h):
 *   codes  [B][H][cap_tiles][innerq_tile_bytes(bits)]   32 tokens per tile
 *   scale  channel groups: [B][H][cap_tiles * 32][D / group]   (tile-swizzled)
 *          token groups:   [B][H][cap_tiles * 32 / group][D]   (dim-swizzled)
 *   zero   same shape as scale, asymmetric mode only
 * Role K uses the row layout (tokens are rows of the QK^T A operand) and role
 * V the col layout (dims are rows of the PV A operand); see
 * innerq_b200/csrc/common.cuh for the bit-level layout.
 *
 * Built: bits 2, 3, 4; group 32/64/128; symmetric or asymmetric; either
 * group axis for either role (the store, pack, unpack and dequant entry
 * points).  The fused decode attention reads K with channel groups (the
 * reference default, cache.py:87) or with token groups (KIVI; GQA <= 4,
 * eager launches, no key normalisation, the values' sink size) and V with
 * token groups (cache.py:88 default), channel groups or hybrid token groups;
 * it refuses the rest with INNERQ_ERR_UNSUPPORTED (materialise those with
 * innerq_dequant).  Scales / zero points of token groups are [groups][D] per
 * (batch, head): values in the col layout's dim order, keys in natural order.
 * Values grouped over channels must be appended into a zero-filled store
 * (their codes share words across tokens).
 */
#ifndef INNERQ_B200_H
#define INNERQ_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define INNERQ_ABI_VERSION 5

enum {
  INNERQ_OK = 0,
  INNERQ_ERR_ARG = -1,         /* bad size, pointer, alignment or stride */
  INNERQ_ERR_UNSUPPORTED = -2, /* valid for the reference, not built here */
  INNERQ_ERR_CUDA = -3         /* a CUDA launch or runtime call failed */
};
enum { INNERQ_DT_F16 = 0, INNERQ_DT_BF16 = 1 };
enum { INNERQ_SYM = 0, INNERQ_ASYM = 1, INNERQ_HYBRID = 2 };  /* quant.py:43-56 QMode */
enum { INNERQ_ROLE_K = 0, INNERQ_ROLE_V = 1 };

/* Version of this ABI (INNERQ_ABI_VERSION). */
int innerq_abi_version(void);
/* Message of the last failing call on this thread ("" if none). */
const char* innerq_last_error(void);

/* Bytes of one packed 32-token tile of one (b, h) at `bits` (D = 128). */
int64_t innerq_tile_bytes(int bits);

/*
 * Key normalisation factor f[b][h][d] = dtype(sqrt(max_t |x[b][h][t][d]|)).
 * Replaces the factor computation of InnerqDynamicLayer.normalize_keys
 * (src/innerq/cache.py:121-126).  out_f is contiguous [B][H][D].
 */
int innerq_norm_factor(const void* x, int dtype, int B, int H, int T, int D, int64_t sb,
                       int64_t sh, int64_t st, void* out_f, void* stream);

/*
 * Quantize T tokens x[B][H][T][D] and pack them into a store at packed token
 * index t_offset (the cache-append quantizer).  Replaces quantize_sym /
 * quantize_asym and their channel-/token-dim wrappers
 * (src/innerq/quant.py:58-81, 95-119) as called by
 * InnerqDynamicLayer.initialize_*_q / quantize_new_* (cache.py:187-210,
 * 314-365), with the torch.cat onto the store replaced by an in-place write.
 * norm_f (nullable, [B][H][D]) divides x first, in the dtype (cache.py:125).
 * Token groups need T % group == 0 and t_offset % group == 0.  The store
 * must hold t_offset + T tokens (cap_tiles * 32).
 */
int innerq_quant_pack(const void* x, int dtype, int B, int H, int T, int D, int64_t sb,
                      int64_t sh, int64_t st, int bits, int group, int mode, int role,
                      int over_token, const void* norm_f, void* codes, void* scale, void* zero,
                      int64_t cap_tiles, int64_t t_offset, void* stream);

/*
 * Reference-format views of packed tokens [t_begin, t_begin + n): the int32
 * codes, sign tensor and scale / zero-point tensors that quant.py:58-131
 * returns (magnitudes + dtype signs for symmetric, raw codes + min for
 * asymmetric).  out_sign / out_zero may be NULL.  All outputs contiguous:
 * codes and signs [B][H][n][D]; scale and zero [B][H][n][D/group] (channel
 * groups) or [B][H][n/group][D] (token groups).
 */
int innerq_unpack_ref(const void* codes, const void* scale, const void* zero, int dtype, int B,
                      int H, int64_t t_begin, int64_t n, int D, int bits, int group, int mode,
                      int role, int over_token, int64_t cap_tiles, int32_t* out_codes,
                      void* out_sign, void* out_scale, void* out_zero, void* stream);

/*
 * Materialise dequantized tokens [t_begin, t_begin + n) in the model dtype
 * exactly as InnerqDynamicLayer.get_*_deq (cache.py:235-281) does:
 * dtype(fp32(c) * fp32(s) * sign [+ fp32(min)] [* fp32(norm_f)]).
 * out is [B][H][n][D] with strides (ob, oh, ot).
 */
int innerq_dequant(const void* codes, const void* scale, const void* zero, int dtype, int B, int H,
                   int64_t t_begin, int64_t n, int D, int bits, int group, int mode, int role,
                   int over_token, int64_t cap_tiles, const void* norm_f, void* out, int64_t ob,
                   int64_t oh, int64_t ot, void* stream);

/*
 * Dequantize reference-format tensors to fp32: the dequantize_{channeldim,
 * tokendim}_{sym,asym} functions of src/innerq/quant.py:83-93, 121-131.
 * codes int32 [n_outer][T][D]; scale (dtype) [n_outer][T][D/group] for
 * channel groups or [n_outer][T/group][D] for token groups; zp_or_sign is the
 * dtype sign tensor [n_outer][T][D] (symmetric) or the zero point shaped like
 * scale (asymmetric).  out fp32 [n_outer][T][D].  Any D divisible by group.
 */
int innerq_dequant_ref(const int32_t* codes, const void* scale, const void* zp_or_sign, int dtype,
                       int64_t n_outer, int T, int D, int group, int mode, int over_token,
                       float* out, void* stream);

/* One side (K or V) of the cache as the fused decode attention reads it.
 * Token order is [sink | quantized | recent] (cache.py:235-276). */
typedef struct {
  const void* codes;   /* packed store (NULL when n_q == 0) */
  const void* scale;
  const void* zero;    /* asymmetric only */
  int64_t cap_tiles;
  const void* sink;    /* [B][H][n_sink][D] dtype, strides below */
  int64_t sink_sb, sink_sh, sink_st;
  const void* recent;  /* [B][H][n_recent][D] dtype */
  int64_t rec_sb, rec_sh, rec_st;
  int32_t n_sink, n_q, n_recent;
  int32_t bits;        /* 2, 3, 4 (ignored when n_q == 0) */
  int32_t group;
  int32_t mode;        /* INNERQ_SYM / INNERQ_ASYM */
  int32_t over_token;  /* groups over tokens: 1 (V default; K for KIVI) or channels: 0 */
  /* Graph mode only (innerq_attn_args.step set), else 0: n_q / n_recent are
   * the counts at step 0, `recent` is the FIFO buffer base, r0 the window's
   * FIFO offset at step 0 and flush the side's flush size (0: no quantization).
   * max_steps: the steps the buffers were reserved for; the kernel reads the
   * state after min(*step, max_steps) steps, so a counter run past the
   * reservation never reads outside the buffers (the caller checks the count). */
  int32_t r0, flush, max_steps;
  /* Hybrid values (mode INNERQ_HYBRID, quant.py:133-176; values grouped over
   * tokens, read by innerq_decode_attn only): codes / scale above hold the
   * symmetric `bits`-bit set, codes2 / scale2 / zero2 the asymmetric
   * (bits - 1)-bit set in a store of cap_tiles2 tiles, and mask one bit per
   * (token group, dim), 16 bytes per group ([B][H][cap_tiles2 * 32 / group]),
   * bit col_scale_idx(dim) (the dim order of the value scales) set where the
   * group keeps its symmetric codes.  Unused (NULL, 0) otherwise. */
  const void* codes2;
  const void* scale2;
  const void* zero2;
  const void* mask;
  int64_t cap_tiles2;
} innerq_side;

typedef struct {
  int32_t struct_size; /* sizeof(innerq_attn_args) */
  int32_t dtype;
  int32_t B, Hq, Hkv, D;
  const void* q;       /* [B][Hq][D] with strides (q_sb, q_sh) */
  int64_t q_sb, q_sh;
  const void* key_norm;/* [B][Hkv][D] contiguous normalisation factor, or NULL */
  innerq_side k, v;
  float softmax_scale; /* the reference consumer uses head_dim^-0.5 */
  int32_t n_splits;    /* 0 = choose for the GPU; else exactly this split-KV count (splits
                        * past the last tile publish m = -inf, l = 0) */
  int32_t tile_lo, tile_hi; /* 0,0 = all tiles; else a sub-range (context sharding) */
  /* Graph mode: device counter of decode steps appended since the state in k
   * and v (innerq_append_step advances the cache, the caller the counter), so
   * one recorded CUDA graph serves every step; NULL: the state in k, v is
   * current.  The split count is fixed when the plan is made. */
  const int64_t* step;
} innerq_attn_args;

/* Number of 32-token tiles the fused kernel iterates for these args, and the
 * split count it will use (n_splits resolved). */
int innerq_attn_plan(const innerq_attn_args* args, int32_t* n_tiles, int32_t* n_splits);

/* Workspace bytes innerq_decode_attn needs: the split-KV partials and the
 * per-(batch, KV head) query blocks the attention pass reads. */
int64_t innerq_decode_attn_workspace(const innerq_attn_args* args);

/*
 * Fused decode attention for one query token per sequence:
 *   out[b][hq] = softmax(q[b][hq] . K[b][hq/G]^T * scale) V[b][hq/G]
 * reading the packed K/V and fp16 sink / recent tokens directly.  Replaces
 * InnerqDynamicLayer.get_deq_tensors (cache.py:278-281) followed by the HF
 * sdpa consumer.  workspace (>= innerq_decode_attn_workspace bytes, 16-byte
 * aligned) holds the split partials and the query blocks.  out [B][Hq][D] dtype with strides
 * (o_sb, o_sh); lse (nullable, [B][Hq] fp32) receives log2-sum-exp2 of the
 * scaled logits.
 */
int innerq_decode_attn(const innerq_attn_args* args, void* workspace, int64_t workspace_bytes,
                       void* out, int64_t o_sb, int64_t o_sh, float* lse, void* stream);

/*
 * Partials only: part_o [B][Hq][n_splits][D] fp32 (unnormalised), part_m and
 * part_l [B][Hq][n_splits] (log2-domain running max and sum).  For context
 * sharding across GPUs: gather the partials, then innerq_lse_merge.
 * workspace (>= innerq_decode_attn_workspace bytes, 16-byte aligned) holds the
 * query blocks.
 */
int innerq_decode_attn_partials(const innerq_attn_args* args, float* part_o, float* part_m,
                                float* part_l, void* workspace, int64_t workspace_bytes,
                                void* stream);

/*
 * One decode-step append of one side in graph mode (cache.py:283-307 then
 * 314-380: append the new token to the recent window, then quantize and pack
 * the oldest `flush` tokens when the window holds at least that many), with
 * the step taken from the device counter `step` (this step counted), so the
 * launch can be recorded in a CUDA graph once and replayed.  The FIFO and the
 * packed store must already hold the capacity the replays need.  One launch.
 */
typedef struct {
  int32_t struct_size;  /* sizeof(innerq_append_args) */
  int32_t dtype, B, H, D;
  const void* x;        /* the new token [B][H][D] with strides (x_sb, x_sh) */
  int64_t x_sb, x_sh;
  void* fifo;           /* recent FIFO buffer [B][H][*][D] */
  int64_t f_sb, f_sh, f_st;
  int32_t fifo_cap;     /* tokens the FIFO buffer holds */
  void* codes;          /* packed store of the side (see innerq_quant_pack) */
  void* scale;
  void* zero;
  int64_t cap_tiles;
  const void* norm_f;   /* key normalisation factor or NULL */
  int32_t bits;         /* 1-4, or 16: no quantization (the window only grows) */
  int32_t group, mode, role, over_token;
  int32_t flush;        /* the side's flush size */
  int32_t n_q, n_recent, r0;  /* packed count, window size and its FIFO offset at step 0 */
  int32_t max_steps;    /* steps the FIFO and the store were reserved for; a counter
                         * beyond it makes the launch write nothing */
} innerq_append_args;

int innerq_append_step(const innerq_append_args* args, const int64_t* step, void* stream);

/* Merge split partials: out[row] = sum_s 2^(m_s-M) O_s / sum_s 2^(m_s-M) l_s,
 * rows = B * rows_per_b, out row (b, h) at b*o_sb + h*o_sh. */
int innerq_lse_merge(const float* part_o, const float* part_m, const float* part_l, int B,
                     int rows_per_b, int n_splits, int D, int dtype, void* out, int64_t o_sb,
                     int64_t o_sh, float* lse, void* stream);

/*
 * Context sharding across ranks (no counterpart in the reference, which is
 * single-GPU): each rank computes the split partials of its own context chunk
 * into one block of innerq_partials_rank_floats(B, rows_per_b, n_splits, D)
 * floats laid out as [o: rows][n_splits][D] | [m: rows][n_splits] |
 * [l: rows][n_splits] (rows = B * rows_per_b; pass the three parts to
 * innerq_decode_attn_partials), the blocks of all ranks are gathered
 * rank_stride floats apart (one all-gather), and innerq_lse_merge_ranks
 * merges every rank's splits into out exactly as innerq_lse_merge merges one
 * rank's.  Returns -1 for bad sizes.
 */
int64_t innerq_partials_rank_floats(int B, int rows_per_b, int n_splits, int D);
int innerq_lse_merge_ranks(const float* parts, int n_ranks, int64_t rank_stride, int B,
                           int rows_per_b, int n_splits, int D, int dtype, void* out, int64_t o_sb,
                           int64_t o_sh, float* lse, void* stream);

/*
 * innerq_decode_attn without a caller workspace, for callers that cannot
 * allocate device memory at decode time (a fixed memory arena, or a serving
 * loop that forbids allocation after warm-up).  No counterpart in the
 * reference, which has no native entry points.
 *
 * The split-KV partials live in a file-scope device array of
 * INNERQ_NOALLOC_SCRATCH_BYTES.  A device takes that memory when the
 * library's module is loaded on it: with CUDA's lazy module loading (the
 * default of CUDA 12) that is the first valid call of this function on the
 * device, which looks up the array's address (cudaGetSymbolAddress) with the
 * device current; without lazy loading it is the library's first use of the
 * device.  Either way the memory stays taken until the process exits.  Make
 * the first call on each device before any stream capture.  Arguments are
 * checked first: a rejected call takes no memory.  Calls whose partials would
 * not fit are rejected with INNERQ_ERR_ARG (pass a smaller n_splits or
 * batch); other bad arguments get the status innerq_decode_attn gives them.  All calls share the
 * one array: calls that overlap on the GPU (two streams, two threads) race.
 * Nothing in it needs to start at zero.  Allocates nothing; arguments and
 * results as innerq_decode_attn.
 */
#define INNERQ_NOALLOC_SCRATCH_BYTES (64ll << 20)
int innerq_decode_attn_noalloc(const innerq_attn_args* args, void* out, int64_t o_sb,
                               int64_t o_sh, float* lse, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* INNERQ_B200_H */
