// C-ABI entry points of libinnerq_b200.so (declared in include/innerq_b200.h):
// argument validation, split-KV planning and kernel dispatch.
#include <cuda_runtime.h>

#include <algorithm>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include "../../include/innerq_b200.h"
#include "decode_attn.cuh"
#include "innerq_internal.h"

using namespace innerq;

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return INNERQ_OK;
  if (e == cudaErrorNotSupported)
    return fail(INNERQ_ERR_UNSUPPORTED, "%s: combination not supported", what);
  return fail(INNERQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned(const void* p, int n) { return ((uintptr_t)p % n) == 0; }

int check_common(int dtype, int D, int bits, int group, int mode, int role, int over_token) {
  if (dtype != INNERQ_DT_F16 && dtype != INNERQ_DT_BF16) return fail(INNERQ_ERR_ARG, "dtype %d", dtype);
  if (D != kD) return fail(INNERQ_ERR_UNSUPPORTED, "head_dim %d (only 128 is built)", D);
  if (bits < 1 || bits > 4) return fail(INNERQ_ERR_UNSUPPORTED, "bits %d (1 to 4 are built)", bits);
  if (mode != INNERQ_SYM && mode != INNERQ_ASYM) return fail(INNERQ_ERR_ARG, "mode %d", mode);
  if (group != 32 && group != 64 && group != 128)
    return fail(INNERQ_ERR_UNSUPPORTED, "group size %d (32, 64, 128 are built)", group);
  if (role != INNERQ_ROLE_K && role != INNERQ_ROLE_V) return fail(INNERQ_ERR_ARG, "role %d", role);
  return INNERQ_OK;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// a side with a packed part now, or one that will pack during graph-mode steps
inline bool packed(const innerq_side& s) { return s.n_q > 0 || s.flush > 0; }

struct Plan {
  int S, t_first, n_tiles, tile_lo, tile_hi, n_splits, tps, R, bk, bv;
};

int check_side(const innerq_side& s, int dtype, int role, const char* name) {
  if (s.n_sink < 0 || s.n_q < 0 || s.n_recent < 0) return fail(INNERQ_ERR_ARG, "%s: negative count", name);
  if (packed(s)) {
    const bool hyb = s.mode == INNERQ_HYBRID;
    int rc = check_common(dtype, kD, s.bits, s.group, hyb ? INNERQ_SYM : s.mode, role, s.over_token);
    if (rc) return rc;
    if (hyb) {
      if (role != INNERQ_ROLE_V || !s.over_token)
        return fail(INNERQ_ERR_UNSUPPORTED, "fused attention: hybrid %s must be values grouped over tokens", name);
      if (!s.codes2 || !s.scale2 || !s.zero2 || !s.mask || !aligned(s.codes2, 16) || !aligned(s.scale2, 16) ||
          !aligned(s.zero2, 16) || !aligned(s.mask, 16))
        return fail(INNERQ_ERR_ARG, "%s: hybrid stores missing or not 16-byte aligned", name);
      if ((int64_t)s.n_q > s.cap_tiles2 * 32) return fail(INNERQ_ERR_ARG, "%s: n_q beyond the asymmetric store", name);
    }
    if (s.bits < 2) return fail(INNERQ_ERR_UNSUPPORTED, "fused attention: %s bits %d (2, 3, 4)", name, s.bits);
    // keys grouped over tokens (the KIVI layout) are read too; make_plan
    // checks the rest of their conditions
    if (!s.codes || !s.scale || (s.mode == INNERQ_ASYM && !s.zero))
      return fail(INNERQ_ERR_ARG, "%s: missing store pointer", name);
    if (!aligned(s.codes, 16) || !aligned(s.scale, 16) || (s.zero && !aligned(s.zero, 16)))
      return fail(INNERQ_ERR_ARG, "%s: store pointers must be 16-byte aligned", name);
    if ((int64_t)s.n_q > s.cap_tiles * 32) return fail(INNERQ_ERR_ARG, "%s: n_q beyond capacity", name);
    // token-grouped values come in whole groups; channel-grouped ones may end
    // inside a tile (whose unwritten code slots are zero)
    if (role == INNERQ_ROLE_V && s.over_token && s.n_q % 32) return fail(INNERQ_ERR_ARG, "%s: n_q %% 32", name);
  }
  if (s.n_sink > 0 && (!s.sink || !aligned(s.sink, 4) || (s.sink_st % 2) || (s.sink_sh % 2) || (s.sink_sb % 2)))
    return fail(INNERQ_ERR_ARG, "%s: sink pointer / strides must be 4-byte aligned", name);
  if (s.n_recent > 0 && (!s.recent || !aligned(s.recent, 4) || (s.rec_st % 2) || (s.rec_sh % 2) || (s.rec_sb % 2)))
    return fail(INNERQ_ERR_ARG, "%s: recent pointer / strides must be 4-byte aligned", name);
  return INNERQ_OK;
}

// tokens a side's packed store holds after max_steps graph-mode steps (one
// token appended per step, `flush` packed whenever the window holds that many)
int64_t graph_packed_need(int n_q, int n_rec, int flush, int max_steps) {
  const int64_t k = flush > 0 ? std::min<int64_t>(max_steps, ((int64_t)n_rec + max_steps) / flush) : 0;
  return (int64_t)n_q + (int64_t)flush * k;
}

int check_graph_side(const innerq_side& s, const char* which) {
  if (s.max_steps < 0) return fail(INNERQ_ERR_ARG, "%s: max_steps %d", which, s.max_steps);
  if (s.flush > 0 && graph_packed_need(s.n_q, s.n_recent, s.flush, s.max_steps) > s.cap_tiles * 32)
    return fail(INNERQ_ERR_ARG, "%s: packed store of %lld tiles cannot take %d steps", which,
                (long long)s.cap_tiles, s.max_steps);
  return INNERQ_OK;
}

int make_plan(const innerq_attn_args* a, Plan& p) {
  if (!a) return fail(INNERQ_ERR_ARG, "null args");
  if (a->struct_size != (int32_t)sizeof(innerq_attn_args))
    return fail(INNERQ_ERR_ARG, "struct_size %d != %d (ABI mismatch)", a->struct_size, (int)sizeof(innerq_attn_args));
  if (a->dtype != INNERQ_DT_F16 && a->dtype != INNERQ_DT_BF16) return fail(INNERQ_ERR_ARG, "dtype");
  if (a->D != kD) return fail(INNERQ_ERR_UNSUPPORTED, "head_dim %d (only 128 is built)", a->D);
  if (a->B <= 0 || a->Hkv <= 0 || a->Hq <= 0 || a->Hq % a->Hkv) return fail(INNERQ_ERR_ARG, "head counts");
  p.R = a->Hq / a->Hkv;
  if (p.R != 1 && p.R != 2 && p.R != 4 && p.R != 8)
    return fail(INNERQ_ERR_UNSUPPORTED, "GQA ratio %d (1, 2, 4, 8 are built)", p.R);
  if (!a->q) return fail(INNERQ_ERR_ARG, "q is null");
  int rc = check_side(a->k, a->dtype, INNERQ_ROLE_K, "k");
  if (rc) return rc;
  rc = check_side(a->v, a->dtype, INNERQ_ROLE_V, "v");
  if (rc) return rc;
  if (a->step) {
    if ((rc = check_graph_side(a->k, "k"))) return rc;
    if ((rc = check_graph_side(a->v, "v"))) return rc;
  }
  if (packed(a->v) && a->v.mode == INNERQ_HYBRID) {
    if (a->step) return fail(INNERQ_ERR_UNSUPPORTED, "fused attention: hybrid values in graph mode");
    if (packed(a->k) && a->k.group != 32)
      return fail(INNERQ_ERR_UNSUPPORTED, "fused attention: hybrid values need keys in groups of 32 (use innerq_dequant)");
  }
  // keys grouped over tokens (KIVI, cache.py:87): the query is scaled per
  // token group inside the kernel; built for GQA <= 4, unnormalised keys,
  // the values' sink size, non-hybrid values
  if (packed(a->k) && a->k.over_token) {
    if (p.R > 4) return fail(INNERQ_ERR_UNSUPPORTED, "fused attention: keys grouped over tokens need GQA <= 4");
    if (a->key_norm) return fail(INNERQ_ERR_UNSUPPORTED, "fused attention: normalised keys grouped over tokens");
    if (a->k.n_sink != a->v.n_sink)
      return fail(INNERQ_ERR_UNSUPPORTED, "fused attention: keys grouped over tokens need the values' sink size");
    if (packed(a->v) && a->v.mode == INNERQ_HYBRID)
      return fail(INNERQ_ERR_UNSUPPORTED, "fused attention: keys grouped over tokens with hybrid values");
    if (packed(a->v) && !a->v.over_token && a->v.group != 32)
      return fail(INNERQ_ERR_UNSUPPORTED, "fused attention: keys grouped over tokens with values in channel groups of %d (32 is built)", a->v.group);
    if (a->k.n_q % 32) return fail(INNERQ_ERR_ARG, "k: n_q %% 32");
  }
  // values grouped over channels share the keys' channel-group count
  if (packed(a->v) && !a->v.over_token && packed(a->k) && !a->k.over_token && a->v.group != a->k.group)
    return fail(INNERQ_ERR_UNSUPPORTED,
                "fused attention: channel-grouped values need the keys' group size (%d vs %d; use innerq_dequant)",
                a->v.group, a->k.group);
  const int64_t Sk = (int64_t)a->k.n_sink + a->k.n_q + a->k.n_recent;
  const int64_t Sv = (int64_t)a->v.n_sink + a->v.n_q + a->v.n_recent;
  if (Sk != Sv) return fail(INNERQ_ERR_ARG, "K holds %lld tokens, V holds %lld", (long long)Sk, (long long)Sv);
  if (Sk > (1ll << 30)) return fail(INNERQ_ERR_ARG, "context too long");
  p.S = (int)Sk;
  const int vs = a->v.n_sink;
  p.t_first = packed(a->v) ? vs - 32 * ((vs + 31) / 32) : 0;
  p.n_tiles = (p.S - p.t_first + 31) / 32;
  p.tile_lo = a->tile_lo, p.tile_hi = a->tile_hi;
  if (p.tile_lo == 0 && p.tile_hi == 0) p.tile_hi = p.n_tiles;
  if (p.tile_lo < 0 || p.tile_hi > p.n_tiles || p.tile_lo > p.tile_hi)
    return fail(INNERQ_ERR_ARG, "tile range [%d, %d) outside [0, %d)", p.tile_lo, p.tile_hi, p.n_tiles);
  const int ntr = p.tile_hi - p.tile_lo;
  int splits = a->n_splits;
  if (splits <= 0) {
    // cost model: waves of resident CTAs x (tiles per CTA + per-CTA overhead
    // worth ~6 tiles: the query-block wait, the warp combine and the partial
    // write); the best split count balances wave quantisation against it
    const int64_t bh = (int64_t)a->B * a->Hkv;
    const int64_t slots = (int64_t)sm_count() * (p.R <= 4 ? 4 : 3);
    int64_t best = -1;
    splits = 1;
    for (int s = 1; s <= 256 && s <= (ntr > 0 ? ntr : 1); ++s) {
      const int64_t tpc = (ntr + s - 1) / s;
      const int64_t waves = (bh * s + slots - 1) / slots;
      const int64_t cost = waves * (tpc + 6);
      if (best < 0 || cost < best) { best = cost; splits = s; }
    }
  }
  if (splits > 65535) splits = 65535;
  p.tps = ntr > 0 ? (ntr + splits - 1) / splits : 1;
  // a chosen count drops the splits that would get no tile; a requested one
  // is kept exactly (its trailing splits may be empty and publish m = -inf),
  // so every rank of a context-sharded layer has the same partials layout
  p.n_splits = a->n_splits > 0 ? splits : (ntr > 0 ? (ntr + p.tps - 1) / p.tps : 1);
  p.bk = packed(a->k) ? a->k.bits : 4;
  p.bv = packed(a->v) ? a->v.bits : 4;
  return INNERQ_OK;
}

DevSide dev_side(const innerq_side& s) {
  DevSide d;
  d.codes = (const uint8_t*)s.codes;
  d.scale = (const uint16_t*)s.scale;
  d.zero = (const uint16_t*)s.zero;
  d.cap_tiles = s.cap_tiles;
  d.sink = (const uint16_t*)s.sink;
  d.sk_b = s.sink_sb; d.sk_h = s.sink_sh; d.sk_t = s.sink_st;
  d.rec = (const uint16_t*)s.recent;
  d.rc_b = s.rec_sb; d.rc_h = s.rec_sh; d.rc_t = s.rec_st;
  d.n_sink = s.n_sink; d.n_q = s.n_q; d.n_rec = s.n_recent;
  d.group = packed(s) ? s.group : 32;
  d.asym = packed(s) && s.mode == INNERQ_ASYM;  // hybrid: the symmetric set
  d.chan = 0;
  d.r0 = s.r0;
  d.flush = s.flush;
  d.max_steps = s.max_steps;
  d.hyb = packed(s) && s.mode == INNERQ_HYBRID;
  d.codes2 = (const uint8_t*)s.codes2;
  d.scale2 = (const uint16_t*)s.scale2;
  d.zero2 = (const uint16_t*)s.zero2;
  d.mask = (const uint16_t*)s.mask;
  d.cap_tiles2 = s.cap_tiles2;
  d.otok = packed(s) && s.over_token;
  return d;
}

int64_t part_bytes(const innerq_attn_args* a, const Plan& p) {
  const int64_t rows = (int64_t)a->B * a->Hq * p.n_splits;
  return rows * kD * 4 + 2 * ((rows * 4 + 255) / 256 * 256);
}

int64_t ws_bytes(const innerq_attn_args* a, const Plan& p) {
  const int rp = p.R <= 4 ? 4 : 8;
  return part_bytes(a, p) + (int64_t)a->B * a->Hkv * qprep_bytes(rp);
}

// prep pass + attention pass; qprep: the query-block region of a workspace
int run_partials(const innerq_attn_args* a, const Plan& p, float* po, float* pm, float* pl,
                 void* qprep, cudaStream_t st) {
  DevArgs d;
  d.k = dev_side(a->k);
  d.v = dev_side(a->v);
  d.v.chan = packed(a->v) && !a->v.over_token;
  d.q = (const uint16_t*)a->q;
  d.q_b = a->q_sb;
  d.q_h = a->q_sh;
  d.kf = (const uint16_t*)a->key_norm;
  d.B = a->B; d.Hq = a->Hq; d.Hkv = a->Hkv; d.S = p.S;
  d.t_first = p.t_first;
  d.tile_lo = p.tile_lo; d.tile_hi = p.tile_hi;
  d.tiles_per_split = p.tps; d.n_splits = p.n_splits;
  d.scale_log2 = a->softmax_scale * 1.4426950408889634f;
  d.po = po; d.pm = pm; d.pl = pl;
  d.step = a->step;
  d.qprep = qprep;
  d.R = p.R;
  dim3 grid(p.n_splits, a->Hkv, a->B);
  const int rp = p.R <= 4 ? 4 : 8;
  // keys grouped over tokens: the 4-group staging geometry (4 tiles' scales per stage)
  const int ng = packed(a->k) && !a->k.over_token ? kD / a->k.group : (d.v.chan && !packed(a->k) ? kD / a->v.group : 4);
  const bool bf = a->dtype == INNERQ_DT_BF16;
  cudaError_t e = launch_qprep(d, rp, ng, bf, st);
  if (e != cudaSuccess) return cuda_status(e, "qprep");
  if (a->step) {  // graph mode: separate instantiations
    switch (p.bk) {
      case 2: e = bf ? launch_attn_k2_bf16_graph(d, p.bv, rp, ng, grid, st) : launch_attn_k2_f16_graph(d, p.bv, rp, ng, grid, st); break;
      case 3: e = bf ? launch_attn_k3_bf16_graph(d, p.bv, rp, ng, grid, st) : launch_attn_k3_f16_graph(d, p.bv, rp, ng, grid, st); break;
      default: e = bf ? launch_attn_k4_bf16_graph(d, p.bv, rp, ng, grid, st) : launch_attn_k4_f16_graph(d, p.bv, rp, ng, grid, st); break;
    }
  } else {
    switch (p.bk) {
      case 2: e = bf ? launch_attn_k2_bf16(d, p.bv, rp, ng, grid, st) : launch_attn_k2_f16(d, p.bv, rp, ng, grid, st); break;
      case 3: e = bf ? launch_attn_k3_bf16(d, p.bv, rp, ng, grid, st) : launch_attn_k3_f16(d, p.bv, rp, ng, grid, st); break;
      default: e = bf ? launch_attn_k4_bf16(d, p.bv, rp, ng, grid, st) : launch_attn_k4_f16(d, p.bv, rp, ng, grid, st); break;
    }
  }
  return cuda_status(e, "decode_attn");
}

}  // namespace

int innerq::set_last_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

extern "C" {

int innerq_abi_version(void) { return INNERQ_ABI_VERSION; }
const char* innerq_last_error(void) { return g_err; }
int64_t innerq_tile_bytes(int bits) { return (bits >= 1 && bits <= 4) ? tile_bytes(bits) : -1; }

int innerq_norm_factor(const void* x, int dtype, int B, int H, int T, int D, int64_t sb, int64_t sh,
                       int64_t st, void* out_f, void* stream) {
  if (dtype != INNERQ_DT_F16 && dtype != INNERQ_DT_BF16) return fail(INNERQ_ERR_ARG, "dtype");
  if (D != kD) return fail(INNERQ_ERR_UNSUPPORTED, "head_dim %d", D);
  if (B <= 0 || H <= 0 || T <= 0 || !x || !out_f) return fail(INNERQ_ERR_ARG, "empty input");
  if (B > 65535 || H > 65535) return fail(INNERQ_ERR_ARG, "B and H must be <= 65535 (grid limits)");
  return cuda_status(launch_norm_factor(x, dtype, B, H, T, sb, sh, st, out_f, (cudaStream_t)stream),
                     "norm_factor");
}

int innerq_quant_pack(const void* x, int dtype, int B, int H, int T, int D, int64_t sb, int64_t sh,
                      int64_t st, int bits, int group, int mode, int role, int over_token,
                      const void* norm_f, void* codes, void* scale, void* zero, int64_t cap_tiles,
                      int64_t t_offset, void* stream) {
  int rc = check_common(dtype, D, bits, group, mode, role, over_token);
  if (rc) return rc;
  if (B < 0 || H < 0 || T < 0 || t_offset < 0) return fail(INNERQ_ERR_ARG, "negative size");
  if (B == 0 || H == 0 || T == 0) return INNERQ_OK;
  if (!x || !codes || !scale || (mode == INNERQ_ASYM && !zero)) return fail(INNERQ_ERR_ARG, "null pointer");
  if (!aligned(codes, 16) || !aligned(scale, 2)) return fail(INNERQ_ERR_ARG, "store alignment");
  if (t_offset + T > cap_tiles * 32) return fail(INNERQ_ERR_ARG, "store capacity %lld tokens < %lld",
                                                (long long)(cap_tiles * 32), (long long)(t_offset + T));
  if (B > 65535 || H > 65535) return fail(INNERQ_ERR_ARG, "B and H must be <= 65535 (grid limits)");
  if (over_token) {
    if (T % group || t_offset % group)
      return fail(INNERQ_ERR_ARG, "token groups need T (%d) and t_offset (%lld) divisible by group %d", T,
                  (long long)t_offset, group);
  } else {
    if (!aligned(x, 8) || (sb % 4) || (sh % 4) || (st % 4))
      return fail(INNERQ_ERR_ARG, "channel-group input must be 8-byte aligned rows");
  }
  if (norm_f && over_token) return fail(INNERQ_ERR_UNSUPPORTED, "normalisation with token groups");
  return cuda_status(launch_pack(x, dtype, B, H, T, sb, sh, st, bits, group, mode == INNERQ_ASYM,
                                 role == INNERQ_ROLE_V, over_token, norm_f, codes, scale, zero,
                                 cap_tiles, t_offset, (cudaStream_t)stream),
                     "quant_pack");
}

int innerq_unpack_ref(const void* codes, const void* scale, const void* zero, int dtype, int B, int H,
                      int64_t t_begin, int64_t n, int D, int bits, int group, int mode, int role,
                      int over_token, int64_t cap_tiles, int32_t* out_codes, void* out_sign,
                      void* out_scale, void* out_zero, void* stream) {
  int rc = check_common(dtype, D, bits, group, mode, role, over_token);
  if (rc) return rc;
  if (n < 0 || t_begin < 0 || t_begin + n > cap_tiles * 32) return fail(INNERQ_ERR_ARG, "token range");
  if (over_token && (t_begin % group || n % group)) return fail(INNERQ_ERR_ARG, "token-group range");
  if (n == 0) return INNERQ_OK;
  if (!codes || !scale || !out_codes || !out_scale || (mode == INNERQ_ASYM && !zero))
    return fail(INNERQ_ERR_ARG, "null pointer");
  return cuda_status(launch_unpack_ref(codes, scale, zero, dtype, B, H, n, bits, group,
                                       mode == INNERQ_ASYM, role == INNERQ_ROLE_V, over_token,
                                       cap_tiles, t_begin, out_codes, out_sign, out_scale, out_zero,
                                       (cudaStream_t)stream),
                     "unpack_ref");
}

int innerq_dequant(const void* codes, const void* scale, const void* zero, int dtype, int B, int H,
                   int64_t t_begin, int64_t n, int D, int bits, int group, int mode, int role,
                   int over_token, int64_t cap_tiles, const void* norm_f, void* out, int64_t ob,
                   int64_t oh, int64_t ot, void* stream) {
  int rc = check_common(dtype, D, bits, group, mode, role, over_token);
  if (rc) return rc;
  if (n < 0 || t_begin < 0 || t_begin + n > cap_tiles * 32) return fail(INNERQ_ERR_ARG, "token range");
  if (n == 0) return INNERQ_OK;
  if (!codes || !scale || !out || (mode == INNERQ_ASYM && !zero)) return fail(INNERQ_ERR_ARG, "null pointer");
  return cuda_status(launch_dequant(codes, scale, zero, dtype, B, H, n, bits, group,
                                    mode == INNERQ_ASYM, role == INNERQ_ROLE_V, over_token, cap_tiles,
                                    t_begin, norm_f, out, ob, oh, ot, (cudaStream_t)stream),
                     "dequant");
}

int innerq_dequant_ref(const int32_t* codes, const void* scale, const void* zp_or_sign, int dtype,
                       int64_t n_outer, int T, int D, int group, int mode, int over_token, float* out,
                       void* stream) {
  if (dtype != INNERQ_DT_F16 && dtype != INNERQ_DT_BF16) return fail(INNERQ_ERR_ARG, "dtype");
  if (mode != INNERQ_SYM && mode != INNERQ_ASYM) return fail(INNERQ_ERR_ARG, "mode");
  if (n_outer < 0 || T < 0 || D <= 0 || group <= 0) return fail(INNERQ_ERR_ARG, "sizes");
  if ((over_token ? T : D) % group) return fail(INNERQ_ERR_ARG, "group %d does not divide the grouped dim", group);
  if (n_outer == 0 || T == 0) return INNERQ_OK;
  if (!codes || !scale || !zp_or_sign || !out) return fail(INNERQ_ERR_ARG, "null pointer");
  return cuda_status(launch_dequant_ref(codes, scale, zp_or_sign, dtype, n_outer, T, D, group,
                                        mode == INNERQ_ASYM, over_token, out, (cudaStream_t)stream),
                     "dequant_ref");
}

int innerq_attn_plan(const innerq_attn_args* args, int32_t* n_tiles, int32_t* n_splits) {
  Plan p;
  int rc = make_plan(args, p);
  if (rc) return rc;
  if (n_tiles) *n_tiles = p.n_tiles;
  if (n_splits) *n_splits = p.n_splits;
  return INNERQ_OK;
}

int64_t innerq_decode_attn_workspace(const innerq_attn_args* args) {
  Plan p;
  if (make_plan(args, p)) return -1;
  return ws_bytes(args, p);
}

int innerq_decode_attn_partials(const innerq_attn_args* args, float* part_o, float* part_m,
                                float* part_l, void* workspace, int64_t workspace_bytes,
                                void* stream) {
  Plan p;
  int rc = make_plan(args, p);
  if (rc) return rc;
  if (!part_o || !part_m || !part_l) return fail(INNERQ_ERR_ARG, "null partials");
  const int64_t need = ws_bytes(args, p);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 16))
    return fail(INNERQ_ERR_ARG, "workspace %lld bytes < %lld needed (or misaligned)",
                (long long)workspace_bytes, (long long)need);
  return run_partials(args, p, part_o, part_m, part_l, (char*)workspace + part_bytes(args, p),
                      (cudaStream_t)stream);
}

int innerq_decode_attn(const innerq_attn_args* args, void* workspace, int64_t workspace_bytes,
                       void* out, int64_t o_sb, int64_t o_sh, float* lse, void* stream) {
  Plan p;
  int rc = make_plan(args, p);
  if (rc) return rc;
  if (!out) return fail(INNERQ_ERR_ARG, "out is null");
  const int64_t need = ws_bytes(args, p);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 16))
    return fail(INNERQ_ERR_ARG, "workspace %lld bytes < %lld needed (or misaligned)",
                (long long)workspace_bytes, (long long)need);
  const int64_t rows = (int64_t)args->B * args->Hq * p.n_splits;
  float* po = (float*)workspace;
  float* pm = po + rows * kD;
  float* pl = (float*)((char*)pm + (rows * 4 + 255) / 256 * 256);
  rc = run_partials(args, p, po, pm, pl, (char*)workspace + part_bytes(args, p), (cudaStream_t)stream);
  if (rc) return rc;
  return cuda_status(launch_lse_merge(po, pm, pl, args->B * args->Hq, args->Hq, p.n_splits,
                                      args->dtype, out, o_sb, o_sh, lse, (cudaStream_t)stream),
                     "lse_merge");
}

int innerq_append_step(const innerq_append_args* a, const int64_t* step, void* stream) {
  if (!a) return fail(INNERQ_ERR_ARG, "null args");
  if (a->struct_size != (int32_t)sizeof(innerq_append_args))
    return fail(INNERQ_ERR_ARG, "struct_size %d != %d (ABI mismatch)", a->struct_size,
                (int)sizeof(innerq_append_args));
  if (a->dtype != INNERQ_DT_F16 && a->dtype != INNERQ_DT_BF16) return fail(INNERQ_ERR_ARG, "dtype");
  if (a->D != kD) return fail(INNERQ_ERR_UNSUPPORTED, "head_dim %d (only 128 is built)", a->D);
  if (a->B <= 0 || a->H <= 0 || a->B > 65535 || a->H > 65535) return fail(INNERQ_ERR_ARG, "B, H");
  if (!step || !a->x || !a->fifo) return fail(INNERQ_ERR_ARG, "null pointer");
  if (a->n_q < 0 || a->n_recent < 0 || a->r0 < 0 || a->r0 + a->n_recent > a->fifo_cap)
    return fail(INNERQ_ERR_ARG, "FIFO state outside its buffer");
  if (a->max_steps < 0 || (int64_t)a->r0 + a->n_recent + a->max_steps > a->fifo_cap)
    return fail(INNERQ_ERR_ARG, "FIFO of %d tokens cannot take %d steps", a->fifo_cap, a->max_steps);
  if (a->bits != 16 && a->flush > 0 &&
      graph_packed_need(a->n_q, a->n_recent, a->flush, a->max_steps) > a->cap_tiles * 32)
    return fail(INNERQ_ERR_ARG, "packed store of %lld tiles cannot take %d steps",
                (long long)a->cap_tiles, a->max_steps);
  AppendArgs g;
  g.x = a->x; g.x_sb = a->x_sb; g.x_sh = a->x_sh;
  g.fifo = a->fifo; g.f_sb = a->f_sb; g.f_sh = a->f_sh; g.f_st = a->f_st; g.fifo_cap = a->fifo_cap;
  g.codes = a->codes; g.scale = a->scale; g.zero = a->zero; g.cap_tiles = a->cap_tiles;
  g.norm_f = a->norm_f;
  g.dt = a->dtype; g.B = a->B; g.H = a->H; g.bits = a->bits; g.group = a->group;
  g.asym = a->mode == INNERQ_ASYM; g.flush = a->flush;
  g.n_q = a->n_q; g.n_rec = a->n_recent; g.r0 = a->r0; g.max_steps = a->max_steps;
  if (a->bits == 16) {
    g.mode = 3;
  } else {
    int rc = check_common(a->dtype, a->D, a->bits, a->group, a->mode, a->role, a->over_token);
    if (rc) return rc;
    if (a->flush <= 0) return fail(INNERQ_ERR_ARG, "flush %d", a->flush);
    if (!a->codes || !a->scale || (a->mode == INNERQ_ASYM && !a->zero))
      return fail(INNERQ_ERR_ARG, "null store pointer");
    if (a->over_token) {
      if (a->flush % a->group || a->n_q % a->group)
        return fail(INNERQ_ERR_ARG, "token groups need flush (%d) and n_q (%d) divisible by group %d",
                    a->flush, a->n_q, a->group);
      if (a->norm_f) return fail(INNERQ_ERR_UNSUPPORTED, "normalisation with token groups");
      g.mode = a->role == INNERQ_ROLE_V ? 1 : 4;
    } else {
      if (a->norm_f && a->role == INNERQ_ROLE_V) return fail(INNERQ_ERR_ARG, "normalised values");
      g.mode = a->role == INNERQ_ROLE_V ? 2 : 0;
    }
  }
  return cuda_status(launch_append_step(g, step, (cudaStream_t)stream), "append_step");
}

int innerq_lse_merge(const float* part_o, const float* part_m, const float* part_l, int B,
                     int rows_per_b, int n_splits, int D, int dtype, void* out, int64_t o_sb,
                     int64_t o_sh, float* lse, void* stream) {
  if (D != kD) return fail(INNERQ_ERR_UNSUPPORTED, "head_dim %d", D);
  if (dtype != INNERQ_DT_F16 && dtype != INNERQ_DT_BF16) return fail(INNERQ_ERR_ARG, "dtype");
  if (B < 0 || rows_per_b < 0 || n_splits <= 0) return fail(INNERQ_ERR_ARG, "sizes");
  if (!part_o || !part_m || !part_l || !out) return fail(INNERQ_ERR_ARG, "null pointer");
  return cuda_status(launch_lse_merge(part_o, part_m, part_l, B * rows_per_b, rows_per_b, n_splits,
                                      dtype, out, o_sb, o_sh, lse, (cudaStream_t)stream),
                     "lse_merge");
}

int64_t innerq_partials_rank_floats(int B, int rows_per_b, int n_splits, int D) {
  if (B < 0 || rows_per_b < 0 || n_splits <= 0 || D != kD) return -1;
  const int64_t rows = (int64_t)B * rows_per_b * n_splits;
  return rows * (kD + 2);
}

int innerq_lse_merge_ranks(const float* parts, int n_ranks, int64_t rank_stride, int B,
                           int rows_per_b, int n_splits, int D, int dtype, void* out, int64_t o_sb,
                           int64_t o_sh, float* lse, void* stream) {
  if (D != kD) return fail(INNERQ_ERR_UNSUPPORTED, "head_dim %d", D);
  if (dtype != INNERQ_DT_F16 && dtype != INNERQ_DT_BF16) return fail(INNERQ_ERR_ARG, "dtype");
  if (B < 0 || rows_per_b < 0 || n_splits <= 0 || n_ranks <= 0) return fail(INNERQ_ERR_ARG, "sizes");
  if (!parts || !out) return fail(INNERQ_ERR_ARG, "null pointer");
  const int64_t block = innerq_partials_rank_floats(B, rows_per_b, n_splits, D);
  if (n_ranks > 1 && rank_stride < block)
    return fail(INNERQ_ERR_ARG, "rank stride %lld floats < the %lld of one rank's partials",
                (long long)rank_stride, (long long)block);
  const int64_t rs = (int64_t)B * rows_per_b * n_splits;
  return cuda_status(launch_lse_merge(parts, parts + rs * kD, parts + rs * kD + rs, B * rows_per_b,
                                      rows_per_b, n_splits, dtype, out, o_sb, o_sh, lse,
                                      (cudaStream_t)stream, n_ranks, rank_stride),
                     "lse_merge_ranks");
}

}  // extern "C"
