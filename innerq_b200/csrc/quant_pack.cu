// Cache-append quantize-and-pack, key normalisation factor, reference-format
// unpack and dequantize kernels.
//
// Arithmetic follows quant.py of mthcom/innerq op by op, each op computed in
// fp32 and rounded to the input dtype (fp16 or bf16, RNE), which is what a
// torch fp16/bf16 op does:
//   symmetric  (quant.py:95-111):  s = h(max|x| / (2^(b-1)-1)),
//                                  c = rint(clamp(h(|x| / s), 0, 2^(b-1)-1))
//   asymmetric (quant.py:58-73):   s = h(h(max-min) / (2^b-1)),
//                                  c = rint(clamp(h(h(x-min) / s), 0, 2^b-1))
// Division gives the IEEE fp32 '/' result (this file must not be built with
// fast math); with fp16 operands it is computed by Markstein's sequence from
// one correctly rounded reciprocal per divisor (div_rn in common.cuh).
// A group whose scale is 0 makes the reference divide 0/0 (NaN, stored as
// INT32_MIN); the packed format stores code 0 there, which dequantizes to the
// same value.
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "innerq_internal.h"

namespace innerq {

// warps of one split-merge CTA (splits are dealt to them)
constexpr int kMergeMaxWarps = 16;

template <int BITS>
__device__ __forceinline__ int qmax_sym() { return (1 << (BITS - 1)) - 1; }


// a / b as the IEEE fp32 '/' computes it for a non-negative numerator and a
// divisor shared by many numerators: fp16 operands take Markstein's sequence
// with one reciprocal per divisor (rb = __frcp_rn(b), computed by the caller);
// bf16 operands, whose range can underflow that sequence, use '/'.
template <int DT>
__device__ __forceinline__ float shared_div(float a, float b, float rb) {
  if (DT == F16) {
    // a zero or infinite divisor gives the IEEE quotient of a non-negative a
    // by select: a / 0 = inf (NaN for 0 / 0), a / inf = 0
    const float special = b == 0.f ? (a > 0.f ? INFINITY : NAN) : 0.f;
    const float q = div_rn(a, b, rb);
    return (b > 0.f && b < INFINITY) ? q : special;
  }
  return a / b;
}
template <int DT>
__device__ __forceinline__ float shared_rcp(float b) {
  return (DT == F16 && b > 0.f && b < INFINITY) ? __frcp_rn(b) : 0.f;
}
// a / q for the constant q = 2^k - 1 of a quantizer (IEEE result; fp16 a)
template <int DT, int Q>
__device__ __forceinline__ float div_qmax(float a) {
  if (DT == F16) return div_rn(a, (float)Q, 1.f / (float)Q);  // RN(1/Q) folds at compile time
  return a / (float)Q;
}

// --------------------------------------------------------------------------
// K normalisation factor (cache.py:124): f = sqrt(max_t |x|) per (b, h, d)
// --------------------------------------------------------------------------
template <int DT>
__global__ void norm_factor_kernel(const uint16_t* __restrict__ x, int64_t sb, int64_t sh,
                                   int64_t st, int H, int T, uint16_t* __restrict__ f) {
  const int bh = blockIdx.x, b = bh / H, h = bh % H, d = threadIdx.x;
  const uint16_t* p = x + b * sb + h * sh + d;
  float mx = 0.f;
  for (int t = 0; t < T; ++t) mx = fmaxf(mx, fabsf(to_f<DT>(p[(int64_t)t * st])));
  f[(int64_t)bh * kD + d] = from_f<DT>(sqrtf(mx));
}

// The same over chunks of 512 tokens: grid (chunks, H, B), 256 threads = 4 token
// rows x 64 dim pairs.  |x| >= 0 in fp16 / bf16 orders like its 16-bit
// pattern, so each chunk's maxima are combined as bit patterns in the output
// itself (zeroed first) with a compare-and-swap on the 32-bit word holding two
// adjacent dims; norm_sqrt_kernel then replaces each max m by rnd(sqrt(m)).
template <int DT>
__global__ void __launch_bounds__(256) norm_absmax_kernel(const uint16_t* __restrict__ x, int64_t sb,
                                                          int64_t sh, int64_t st, int T,
                                                          uint32_t* __restrict__ f_words) {
  __shared__ uint32_t red[4][64];
  const int h = blockIdx.y, b = blockIdx.z, H = gridDim.y;
  const int dp = threadIdx.x & 63, row = threadIdx.x >> 6;
  const int t0 = blockIdx.x * 512;
  const uint16_t* base = x + b * sb + h * sh + 2 * dp;
  uint32_t m0 = 0u, m1 = 0u;  // max |x| as 15-bit magnitude patterns
#pragma unroll 8
  for (int k = row; k < 512; k += 4) {
    if (t0 + k < T) {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(base + (int64_t)(t0 + k) * st);
      m0 = max(m0, w & 0x7fffu);
      m1 = max(m1, (w >> 16) & 0x7fffu);
    }
  }
  red[row][dp] = m0 | (m1 << 16);
  __syncthreads();
  if (row == 0) {
    uint32_t lo = 0u, hi = 0u;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      lo = max(lo, red[r][dp] & 0xffffu);
      hi = max(hi, red[r][dp] >> 16);
    }
    uint32_t* word = f_words + ((int64_t)b * H + h) * (kD / 2) + dp;
    uint32_t old = *word, assumed;
    do {
      assumed = old;
      const uint32_t nw = max(assumed & 0xffffu, lo) | (max(assumed >> 16, hi) << 16);
      if (nw == assumed) break;
      old = atomicCAS(word, assumed, nw);
    } while (old != assumed);
  }
}

template <int DT>
__global__ void norm_sqrt_kernel(uint16_t* __restrict__ f, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) f[i] = from_f<DT>(sqrtf(to_f<DT>(f[i])));
}

// --------------------------------------------------------------------------
// Channel groups (per-token groups along head_dim): one warp per token row.
// --------------------------------------------------------------------------
template <int DT, int BITS, int ROLEV>
__device__ __forceinline__ void pack_row_token(const uint2 raw, int t, int64_t bh, int lane,
                                               uint32_t* seg, const uint16_t* __restrict__ nf,
                                               int group, int asym, uint8_t* __restrict__ codes,
                                               uint16_t* __restrict__ scale, uint16_t* __restrict__ zero,
                                               int64_t cap_tiles, int64_t t_off) {
  float v[4] = {to_f<DT>(raw.x & 0xffff), to_f<DT>(raw.x >> 16), to_f<DT>(raw.y & 0xffff),
                to_f<DT>(raw.y >> 16)};
  if (nf) {  // cache.py:125 key_states / factor, in the dtype
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float f = to_f<DT>(nf[bh * kD + 4 * lane + i]);
      // signed numerator, and a zero factor is possible for a channel that was
      // all zero in the first chunk: IEEE '/' outside the fast range
      v[i] = rnd<DT>((DT == F16 && f > 0.f && f < INFINITY) ? div_rn(v[i], f, __frcp_rn(f)) : v[i] / f);
    }
  }
  const int gl = group >> 2;  // lanes per group (8, 16, 32): powers of two
  const int glog = 31 - __clz(gl);
  float s, z = 0.f;
  int u[4];
  if (!asym) {
    float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    for (int o = 1; o < gl; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float qmax = (float)qmax_sym<BITS>();
    s = rnd<DT>(div_qmax<DT, (1 << (BITS - 1)) - 1>(mx));
    const float rs = shared_rcp<DT>(s);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = code_of(rnd<DT>(shared_div<DT>(fabsf(v[i]), s, rs)), qmax);
      u[i] = (v[i] < 0.f ? -c : c) + (1 << (BITS - 1));
    }
  } else {
    float mn = fminf(fminf(v[0], v[1]), fminf(v[2], v[3]));
    float mx = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
    for (int o = 1; o < gl; o <<= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const float qmax = (float)((1 << BITS) - 1);
    s = rnd<DT>(div_qmax<DT, (1 << BITS) - 1>(rnd<DT>(mx - mn)));
    z = mn;
    const float rs = shared_rcp<DT>(s);
#pragma unroll
    for (int i = 0; i < 4; ++i) u[i] = code_of(rnd<DT>(shared_div<DT>(rnd<DT>(v[i] - mn), s, rs)), qmax);
  }
  const int64_t p = t_off + t;
  const int64_t ti = p >> 5;
  const int r = (int)(p & 31);
  const int ng = 32 >> glog;  // kD / group
  if ((lane & (gl - 1)) == 0) {
    const int g = lane >> glog;
    const int64_t si = (bh * cap_tiles + ti) * 32 * ng + row_scale_idx(r, g, ng);
    scale[si] = from_f<DT>(s);
    if (asym) zero[si] = from_f<DT>(z);
  }
  if (ROLEV) {
    // col layout (values grouped over channels): a token's codes are spread
    // over every lane chunk of its tile, sharing words with other tokens, so
    // OR them into the (zero-initialised) store word by word
    uint8_t* tb = codes + (bh * cap_tiles + ti) * tile_bytes(BITS);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const BitPos bp = col_pos(BITS, r, 4 * lane + i);
      const uint32_t uc = (uint32_t)u[i];
      if (BITS == 4 || BITS == 1) {
        atomicOr(reinterpret_cast<uint32_t*>(tb + bp.off), uc << bp.shift);
      } else {
        atomicOr(reinterpret_cast<uint32_t*>(tb + bp.off), (uc & 3u) << bp.shift);
        if (BITS == 3) atomicOr(reinterpret_cast<uint32_t*>(tb + bp.hoff), (uc >> 2) << bp.hshift);
      }
    }
    return;
  }
  // Row layout (keys): a token row's codes never share a 32-bit word with
  // another row, and this lane's 4 codes (dims 4*lane + i) all land in one
  // word: word kb = lane>>3 of the row's segment for lane2 = gid*4 + (lane&3),
  // at bit offsets 8i + (position of this lane among the word's sharers).
  // Build the word in registers, OR it across the sharing lanes with
  // shuffles, and store whole words (no atomics, no staging).
  (void)seg;
  const int half = (lane >> 2) & 1, kb = lane >> 3, tq = lane & 3;
  const int gid = r & 7, j = r >> 3, lane2 = gid * 4 + tq;
  uint8_t* tb = codes + (bh * cap_tiles + ti) * tile_bytes(BITS);
  if (BITS == 4) {
    uint32_t w = 0u;
#pragma unroll
    for (int i = 0; i < 4; ++i) w |= (uint32_t)u[i] << (8 * i + 4 * half);
    w |= __shfl_xor_sync(0xffffffffu, w, 4);
    if (!half) *reinterpret_cast<uint32_t*>(tb + j * 512 + lane2 * 16 + kb * 4) = w;
  } else if (BITS == 1) {
    uint32_t w = 0u;
#pragma unroll
    for (int i = 0; i < 4; ++i) w |= ((uint32_t)u[i] & 1u) << (8 * i + kb * 2 + half);
    w |= __shfl_xor_sync(0xffffffffu, w, 4);
    w |= __shfl_xor_sync(0xffffffffu, w, 8);
    w |= __shfl_xor_sync(0xffffffffu, w, 16);
    if (lane < 4) *reinterpret_cast<uint32_t*>(tb + lane2 * 16 + j * 4) = w;
  } else {
    // low two bits: word kb>>1 of the row's 8 bytes, crumb 4i + (kb&1)*2 + half
    uint32_t w = 0u, wh = 0u;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      w |= ((uint32_t)u[i] & 3u) << (8 * i + 4 * (kb & 1) + 2 * half);
      if (BITS == 3) wh |= (((uint32_t)u[i] >> 2) & 1u) << (8 * i + kb * 2 + half);
    }
    w |= __shfl_xor_sync(0xffffffffu, w, 4);
    w |= __shfl_xor_sync(0xffffffffu, w, 8);
    if ((lane & 12) == 0)
      *reinterpret_cast<uint32_t*>(tb + (j >> 1) * 512 + lane2 * 16 + (j & 1) * 8 + (kb >> 1) * 4) = w;
    if (BITS == 3) {
      wh |= __shfl_xor_sync(0xffffffffu, wh, 4);
      wh |= __shfl_xor_sync(0xffffffffu, wh, 8);
      wh |= __shfl_xor_sync(0xffffffffu, wh, 16);
      if (lane < 4) *reinterpret_cast<uint32_t*>(tb + 1024 + lane2 * 16 + j * 4) = wh;
    }
  }
}


template <int DT, int BITS, int ROLEV>
__global__ void __launch_bounds__(256)
pack_row_channel_kernel(const uint16_t* __restrict__ x, int64_t sb, int64_t sh, int64_t st,
                        int H, int T, const uint16_t* __restrict__ nf, int group, int asym,
                        uint8_t* __restrict__ codes, uint16_t* __restrict__ scale,
                        uint16_t* __restrict__ zero, int64_t cap_tiles, int64_t t_off) {
  __shared__ uint32_t wbuf[8][16];
  // grid (token blocks of 8 warps x 4 tokens, H, B); each warp loads its 4
  // token rows before working on them, so the loads are in flight together
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = (blockIdx.x * 8 + warp) * 4;
  if (t0 >= T) return;
  const int h = blockIdx.y, b = blockIdx.z;
  const int64_t bh = (int64_t)b * H + h;
  uint2 raw[4];
#pragma unroll
  for (int k = 0; k < 4; ++k)
    if (t0 + k < T)
      raw[k] = *reinterpret_cast<const uint2*>(x + b * sb + h * sh + (int64_t)(t0 + k) * st + 4 * lane);
  // unrolled so raw[] stays in registers
#pragma unroll
  for (int k = 0; k < 4; ++k)
    if (t0 + k < T)
      pack_row_token<DT, BITS, ROLEV>(raw[k], t0 + k, bh, lane, wbuf[warp], nf, group, asym, codes,
                                      scale, zero, cap_tiles, t_off);
}

// --------------------------------------------------------------------------
// Row layout (keys, channel groups), one thread per (token, 32-dim block):
// a warp covers 8 tokens x 4 blocks, a CTA of 8 warps 64 tokens of one
// (batch, head).  Each thread reads its 64 bytes with four 16-byte loads,
// reduces its group without shuffles (groups of 64 / 128 combine 2 / 4
// threads), and builds whole 32-bit words of the packed tile in registers.
// --------------------------------------------------------------------------

// dtype fraction bits (the cuts of common.cuh depend on them)
template <int DT> constexpr int kMantBits = DT == F16 ? 10 : 7;

// the cuts of a group of scale s >= 0.  The reference divides by a scale of 0
// too: a / 0 is inf for a > 0 (code qmax) and NaN for a = 0 (code 0), so every
// cut sits just above 0; a / inf is 0 (code 0), so every cut is inf.
template <int DT, int QM>
__device__ __forceinline__ void group_cuts(float s, float* cut) {
  if (s > 0.f && s < INFINITY) {
    code_cuts<kMantBits<DT>, QM>((double)s, cut);
  } else {
#pragma unroll
    for (int k = 0; k < QM; ++k) cut[k] = s == 0.f ? __uint_as_float(1u) : INFINITY;
  }
}

template <int DT, int BITS, int ASYM, int NORM>
__global__ void __launch_bounds__(256, 3)
pack_rows_kernel(const uint16_t* __restrict__ x, int64_t sb, int64_t sh, int64_t st, int T,
                 const uint16_t* __restrict__ nf, int group, uint8_t* __restrict__ codes,
                 uint16_t* __restrict__ scale, uint16_t* __restrict__ zero, int64_t cap_tiles,
                 int64_t t_off) {
  __shared__ __align__(8) float f_s[NORM ? kD : 2];
  __shared__ __align__(8) float rf_s[NORM ? kD : 2];
  // the factor pairs of word w of block kb: {f, f, rf, rf} of dims kb*32 + 2w,
  // +1; blocks 17 entries apart, so the 4 blocks a warp reads at once sit in
  // different banks
  __shared__ float4 fr_s[NORM ? 4 : 1][17];
  const int h = blockIdx.y, b = blockIdx.z, H = gridDim.y;
  const int64_t bh = (int64_t)b * H + h;
  // fp16 factors that are all positive and finite take the paired division
  // (Markstein's sequence on float pairs); others take the scalar path
  bool pair_div = false;
  if constexpr (NORM) {
    bool ok = true;
    if (threadIdx.x < kD) {
      const float f = to_f<DT>(nf[bh * kD + threadIdx.x]);
      f_s[threadIdx.x] = f;
      rf_s[threadIdx.x] = shared_rcp<DT>(f);
      ok = f > 0.f && f < INFINITY;
      float* fr = reinterpret_cast<float*>(&fr_s[threadIdx.x >> 5][(threadIdx.x & 31) >> 1]);
      fr[threadIdx.x & 1] = f;
      fr[2 + (threadIdx.x & 1)] = rf_s[threadIdx.x];
    }
    pair_div = __syncthreads_and(ok) && DT == F16;
  }
  const int lane = threadIdx.x & 31, kb = lane & 3;
  const int t = blockIdx.x * 64 + (threadIdx.x >> 5) * 8 + (lane >> 2);
  const bool valid = t < T;  // no early return: the group reductions shuffle
  // the thread's 32 values as 16 words of two 16-bit dtype values (element e
  // in half e & 1 of word e >> 1); converted where used to keep registers low
  uint32_t raw[16];
  {
    uint4 r4[4] = {};
    if (valid) {
      const uint4* p = reinterpret_cast<const uint4*>(x + b * sb + h * sh + (int64_t)t * st + kb * 32);
#pragma unroll
      for (int k = 0; k < 4; ++k) r4[k] = p[k];
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      raw[4 * k] = r4[k].x; raw[4 * k + 1] = r4[k].y; raw[4 * k + 2] = r4[k].z; raw[4 * k + 3] = r4[k].w;
    }
  }
  auto val = [&](int e) -> float {
    return to_f<DT>((uint16_t)((e & 1) ? (raw[e >> 1] >> 16) : (raw[e >> 1] & 0xffffu)));
  };
  if (NORM && !ASYM && pair_div) {
    // cache.py:125 key_states / factor in fp16, two elements at a time: the
    // magnitude's quotient (Markstein: q = |x| rf, r = |x| - q f exact,
    // RN(q + r rf) = RN(|x| / f)) rounded to fp16, the sign put back
#pragma unroll
    for (int w = 0; w < 16; ++w) {
      const uint32_t mag = raw[w] & 0x7fff7fffu;
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&mag));
      const float4 fr = fr_s[kb][w];
      const float2 f = make_float2(fr.x, fr.y), rf = make_float2(fr.z, fr.w);
      const float2 q = __fmul2_rn(a, rf);
      const float2 r = __ffma2_rn(make_float2(-q.x, -q.y), f, a);
      const __half2 h = __float22half2_rn(__ffma2_rn(r, rf, q));
      raw[w] = *reinterpret_cast<const uint32_t*>(&h) | (raw[w] & 0x80008000u);
    }
  } else if constexpr (NORM) {  // cache.py:125 key_states / factor, in the dtype (stored back as dtype bits)
#pragma unroll
    for (int w = 0; w < 16; ++w) {
      uint32_t nw = 0u;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int e = 2 * w + hf;
        const float f = f_s[kb * 32 + e];
        const float q = (DT == F16 && f > 0.f && f < INFINITY) ? div_rn(val(e), f, rf_s[kb * 32 + e])
                                                               : val(e) / f;
        nw |= (uint32_t)from_f<DT>(q) << (16 * hf);
      }
      raw[w] = nw;
    }
  }
  const int64_t p = t_off + t;
  const int64_t ti = p >> 5;
  const int r = (int)(p & 31), gid = r & 7, j = r >> 3;
  uint8_t* tb = codes + (bh * cap_tiles + ti) * tile_bytes(BITS);
  const int kpg = group >> 5;  // 32-dim blocks per group
  // the group max (and min) in the dtype (exact), codes two elements per
  // word (sym_codes2 / asym_codes2), moved into the row-layout words by byte
  // permutes
  constexpr int QM = ASYM ? (1 << BITS) - 1 : (1 << (BITS - 1)) - 1;
  float s, z = 0.f;
  if constexpr (!ASYM) {
    uint32_t m2 = 0u;
#pragma unroll
    for (int w = 0; w < 16; ++w) m2 = absmax2<DT>(m2, raw[w]);
    float mx = fmaxf(to_f<DT>((uint16_t)(m2 & 0xffffu)), to_f<DT>((uint16_t)(m2 >> 16)));
    if (group >= 64) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    if (group >= 128) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    s = rnd<DT>(div_qmax<DT, QM>(mx));
  } else {
    uint32_t hi = raw[0], lo = raw[0];
#pragma unroll
    for (int w = 1; w < 16; ++w) {
      hi = max2<DT>(hi, raw[w]);
      lo = min2<DT>(lo, raw[w]);
    }
    float mx = fmaxf(to_f<DT>((uint16_t)(hi & 0xffffu)), to_f<DT>((uint16_t)(hi >> 16)));
    float mn = fminf(to_f<DT>((uint16_t)(lo & 0xffffu)), to_f<DT>((uint16_t)(lo >> 16)));
    if (group >= 64) {
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, 1));
    }
    if (group >= 128) {
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, 2));
    }
    s = rnd<DT>(div_qmax<DT, QM>(rnd<DT>(mx - mn)));
    z = mn;
  }
  const uint32_t z2 = (uint32_t)from_f<DT>(z) * 0x00010001u;
  uint32_t cb[QM];
  {
    float cut[QM];
    group_cuts<DT, QM>(s, cut);
#pragma unroll
    for (int k = 0; k < QM; ++k) cb[k] = cut_bits<DT>(cut[k]) * 0x00010001u;
  }
  auto codes2 = [&](uint32_t w) -> uint32_t {
    if constexpr (ASYM) return asym_codes2<DT, BITS>(w, z2, cb);
    else return sym_codes2<DT, BITS>(w, cb);
  };
  if (valid && kb % kpg == 0) {
    const int ng = kD / group, g = kb / kpg;
    const int64_t si = (bh * cap_tiles + ti) * 32 * ng + row_scale_idx(r, g, ng);
    scale[si] = from_f<DT>(s);
    if (ASYM) zero[si] = from_f<DT>(z);
  }
  // word w holds elements 2w, 2w+1 = dims kb*32 + hf*16 + 4*tq + i with
  // hf = w >> 3, tq = (w >> 1) & 3, i = 2*(w & 1) + (half)
#pragma unroll
  for (int tq = 0; tq < 4; ++tq) {
    const int lane2 = gid * 4 + tq;
    uint32_t P[2];  // hf = 0, 1: the codes of i = 0..3 in bytes 0..3
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int w = hf * 8 + 2 * tq;
      P[hf] = __byte_perm(codes2(raw[w]), codes2(raw[w + 1]), 0x6420);
    }
    if constexpr (BITS == 4) {
      // nibble 2i + hf
      if (valid) *reinterpret_cast<uint32_t*>(tb + j * 512 + lane2 * 16 + kb * 4) = P[0] | (P[1] << 4);
    } else {
      // low two bits: crumb 4i + (kb&1)*2 + hf of word kb>>1, shared with
      // block kb^1; 3-bit: bit 2 at 8i + kb*2 + hf of plane H
      const int sh = (kb & 1) * 4;
      const uint32_t l0 = BITS == 3 ? P[0] & 0x03030303u : P[0];
      const uint32_t l1 = BITS == 3 ? P[1] & 0x03030303u : P[1];
      uint32_t w = (l0 << sh) | (l1 << (sh + 2));
      w |= __shfl_xor_sync(0xffffffffu, w, 1);
      if (valid && !(kb & 1))
        *reinterpret_cast<uint32_t*>(tb + (j >> 1) * 512 + lane2 * 16 + (j & 1) * 8 + (kb >> 1) * 4) = w;
      if constexpr (BITS == 3) {
        uint32_t wh = (((P[0] >> 2) & 0x01010101u) << (2 * kb)) | (((P[1] >> 2) & 0x01010101u) << (2 * kb + 1));
        wh |= __shfl_xor_sync(0xffffffffu, wh, 1);
        wh |= __shfl_xor_sync(0xffffffffu, wh, 2);
        if (valid && kb == 0) *reinterpret_cast<uint32_t*>(tb + 1024 + lane2 * 16 + j * 4) = wh;
      }
    }
  }
}

// --------------------------------------------------------------------------
// Col layout, token groups (V): one CTA of 128 threads (one per dim) per
// group of `group` tokens.
// --------------------------------------------------------------------------
// The col-layout words of a group's tiles (values, 2-4 bits) from the codes
// as words of 4 tokens per dim, cbt[dim][token / 4] (the layout map of
// common.cuh), stored straight to global memory by threads tid of nthr.
template <int BITS>
__device__ __forceinline__ void store_col_tiles(const uint32_t (*cbt)[33], uint8_t* __restrict__ codes,
                                                int64_t bh, int64_t cap_tiles, int64_t t_abs, int n_tiles,
                                                int tid, int nthr) {
  constexpr int TW = tile_bytes(BITS) / 4;
    // every word of the group's tiles from 2-8 word loads of 4 tokens' codes
    // (the col-layout map of common.cuh); stored straight to global memory
    const int64_t ti0 = t_abs / 32;
    uint32_t* dst = reinterpret_cast<uint32_t*>(codes + (bh * cap_tiles + ti0) * tile_bytes(BITS));
    for (int i = tid; i < n_tiles * TW; i += nthr) {
      const int k = i / TW, wi = i % TW;
      uint32_t w = 0u;
      if (BITS == 4) {
        const int pc = wi >> 7, L = (wi >> 2) & 31, c = wi & 3;
        const int hh = c >> 1, hf = c & 1, g8 = L >> 2, tq = L & 3;
        const int widx = 8 * k + hf * 4 + tq;
        const int d0 = pc * 16 + hh * 8 + g8;
        w = cbt[d0][widx] | (cbt[d0 + 64][widx] << 4);
      } else if (BITS == 2) {
        const int pc = wi >> 7, L = (wi >> 2) & 31, c = wi & 3;
        const int hh = c >> 1, hf = c & 1, g8 = L >> 2, tq = L & 3;
        const int widx = 8 * k + hf * 4 + tq;
#pragma unroll
        for (int q = 0; q < 4; ++q) w |= cbt[(2 * q + pc) * 16 + hh * 8 + g8][widx] << (2 * q);
      } else if (wi < 256) {  // 3-bit plane L
        const int L = (wi >> 2) & 31, mt = (wi >> 7) * 4 + (wi & 3);
        const int g8 = L >> 2, tq = L & 3;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int hh = c >> 1, hf = c & 1;
          w |= (cbt[mt * 16 + hh * 8 + g8][8 * k + hf * 4 + tq] & 0x03030303u) << (2 * c);
        }
      } else {  // 3-bit plane H
        const int wj = wi - 256, L = wj >> 2, mq = wj & 3;
        const int g8 = L >> 2, tq = L & 3;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int m1 = c >> 2, hh = (c >> 1) & 1, hf = c & 1;
          const int mt = 2 * mq + m1;
          w |= ((cbt[mt * 16 + hh * 8 + g8][8 * k + hf * 4 + tq] >> 2) & 0x01010101u) << c;
        }
      }
      dst[(int64_t)k * TW + wi] = w;
    }
}

// One group of `group` tokens of pair bh (x0: its first token, dim 0; token
// stride st), stored at packed position t_abs; 128 threads, one per dim.
template <int DT, int BITS, int ROLEV>
__device__ __forceinline__ void pack_col_group(const uint16_t* __restrict__ x0, int64_t st, int group,
                                               int asym, uint8_t* __restrict__ codes,
                                               uint16_t* __restrict__ scale, uint16_t* __restrict__ zero,
                                               int64_t cap_tiles, int64_t t_abs, int64_t bh) {
  // col layout (values), 2-4 bits: codes per dim as words of 4 tokens,
  // [dim][token/4] (+1 pad word: conflict-free); otherwise [token][dim] bytes
  constexpr bool kWords = ROLEV && BITS >= 2;
  __shared__ uint8_t cb[kWords ? 1 : 128][kWords ? 1 : kD];
  __shared__ uint32_t cbt[kWords ? kD : 1][kWords ? 33 : 1];
  __shared__ __align__(16) uint32_t tw[kWords ? 4 : 4 * tile_bytes(4) / 4];
  const int d = threadIdx.x;
  const uint16_t* xp = x0 + d;
  float s, z = 0.f;
  if (!asym) {
    float mx = 0.f;
    for (int t = 0; t < group; ++t) mx = fmaxf(mx, fabsf(to_f<DT>(xp[(int64_t)t * st])));
    const float qmax = (float)qmax_sym<BITS>();
    s = rnd<DT>(div_qmax<DT, (1 << (BITS - 1)) - 1>(mx));
    const float rs = shared_rcp<DT>(s);
    uint32_t w4 = 0u;
    for (int t = 0; t < group; ++t) {
      const float v = to_f<DT>(xp[(int64_t)t * st]);
      const int c = code_of(rnd<DT>(shared_div<DT>(fabsf(v), s, rs)), qmax);
      const uint32_t uc = (uint32_t)((v < 0.f ? -c : c) + (1 << (BITS - 1)));
      if (kWords) {
        w4 |= uc << (8 * (t & 3));
        if ((t & 3) == 3) { cbt[d][t >> 2] = w4; w4 = 0u; }
      } else {
        cb[t][d] = (uint8_t)uc;
      }
    }
  } else {
    float mn = INFINITY, mx = -INFINITY;
    for (int t = 0; t < group; ++t) {
      const float v = to_f<DT>(xp[(int64_t)t * st]);
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
    const float qmax = (float)((1 << BITS) - 1);
    s = rnd<DT>(div_qmax<DT, (1 << BITS) - 1>(rnd<DT>(mx - mn)));
    z = mn;
    const float rs = shared_rcp<DT>(s);
    uint32_t w4 = 0u;
    for (int t = 0; t < group; ++t) {
      const float v = to_f<DT>(xp[(int64_t)t * st]);
      const uint32_t uc = (uint32_t)code_of(rnd<DT>(shared_div<DT>(rnd<DT>(v - mn), s, rs)), qmax);
      if (kWords) {
        w4 |= uc << (8 * (t & 3));
        if ((t & 3) == 3) { cbt[d][t >> 2] = w4; w4 = 0u; }
      } else {
        cb[t][d] = (uint8_t)uc;
      }
    }
  }
  const int64_t groups_cap = cap_tiles * 32 / group;
  const int64_t gglob = t_abs / group;
  // values: the col layout's dim order; keys (grouped over tokens): natural
  // dim order, so a lane of the attention pass reads its 4 dims as one word pair
  const int64_t si = (bh * groups_cap + gglob) * kD + (ROLEV ? col_scale_idx(d) : d);
  scale[si] = from_f<DT>(s);
  if (asym) zero[si] = from_f<DT>(z);
  __syncthreads();
  const int n_tiles = group / 32;
  constexpr int TW = tile_bytes(BITS) / 4;
  if constexpr (kWords) {
    store_col_tiles<BITS>(cbt, codes, bh, cap_tiles, t_abs, n_tiles, threadIdx.x, blockDim.x);
    return;
  }
  // assemble each 32-token tile of the group in shared memory with the layout map
  for (int i = threadIdx.x; i < n_tiles * TW; i += blockDim.x) tw[i] = 0u;
  __syncthreads();
  for (int t = 0; t < group; ++t) {
    const uint32_t uc = cb[t][d];
    const BitPos bp = ROLEV ? col_pos(BITS, t & 31, d) : row_pos(BITS, t & 31, d);
    uint32_t* w = tw + (t >> 5) * TW;
    if (BITS == 4 || BITS == 1) {
      atomicOr(&w[bp.off >> 2], uc << bp.shift);
    } else {
      atomicOr(&w[bp.off >> 2], (uc & 3u) << bp.shift);
      if (BITS == 3) atomicOr(&w[bp.hoff >> 2], (uc >> 2) << bp.hshift);
    }
  }
  __syncthreads();
  const int64_t ti0 = t_abs / 32;
  uint4* dst = reinterpret_cast<uint4*>(codes + (bh * cap_tiles + ti0) * tile_bytes(BITS));
  const uint4* src = reinterpret_cast<const uint4*>(tw);
  for (int i = threadIdx.x; i < n_tiles * TW / 4; i += blockDim.x) dst[i] = src[i];
}

// Values, token groups, 2-4 bits (col layout): one CTA of 64 threads per
// group, each thread two adjacent dims read as 4-byte words (a warp reads 128
// contiguous bytes of a token row).  The group is read in chunks of 32 tokens
// held in registers: once for its max (min) and, for groups above 32 tokens,
// once more for the codes (from L2).  Codes use fast_code's exact rounding.
template <int DT, int BITS, int ASYM>
__global__ void __launch_bounds__(64)
pack_cols_kernel(const uint16_t* __restrict__ x, int64_t sb, int64_t sh, int64_t st, int group,
                 uint8_t* __restrict__ codes, uint16_t* __restrict__ scale, uint16_t* __restrict__ zero,
                 int64_t cap_tiles, int64_t t_off) {
  __shared__ uint32_t cbt[kD][33];
  const int gi = blockIdx.x, h = blockIdx.y, b = blockIdx.z, H = gridDim.y;
  const int64_t bh = (int64_t)b * H + h;
  const int dp = threadIdx.x;  // dims 2dp, 2dp+1
  const uint16_t* x0 = x + b * sb + h * sh + (int64_t)gi * group * st + 2 * dp;
  // a chunk of 32 tokens as words of the two dims' 16-bit values, converted
  // where used (keeps the registers, and so the occupancy, of the 4-bit codes)
  uint32_t raw[32];
  auto load = [&](int c0) {
#pragma unroll
    for (int t = 0; t < 32; ++t) raw[t] = *reinterpret_cast<const uint32_t*>(x0 + (int64_t)(c0 + t) * st);
  };
  // per-dim max (and min) in the dtype (exact), codes of both dims of a
  // token word at once
  // (sym_codes2 / asym_codes2), 4 tokens' codes gathered into the
  // [dim][token / 4] byte words by byte permutes
  constexpr int QM = ASYM ? (1 << BITS) - 1 : (1 << (BITS - 1)) - 1;
  uint32_t hi = 0u, lo = 0u;  // asymmetric: both start at the first token's values
  for (int c0 = 0; c0 < group; c0 += 32) {
    load(c0);
    if (ASYM && c0 == 0) hi = lo = raw[0];
#pragma unroll
    for (int t = 0; t < 32; ++t) {
      if constexpr (ASYM) {
        hi = max2<DT>(hi, raw[t]);
        lo = min2<DT>(lo, raw[t]);
      } else {
        hi = absmax2<DT>(hi, raw[t]);
      }
    }
  }
  float s[2], z[2] = {0.f, 0.f};
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const float mx = to_f<DT>((uint16_t)(e ? hi >> 16 : hi & 0xffffu));
    if constexpr (ASYM) {
      z[e] = to_f<DT>((uint16_t)(e ? lo >> 16 : lo & 0xffffu));
      s[e] = rnd<DT>(div_qmax<DT, QM>(rnd<DT>(mx - z[e])));
    } else {
      s[e] = rnd<DT>(div_qmax<DT, QM>(mx));
    }
  }
  const uint32_t z2 = lo;  // the zero points (the minima) as dtype bits
  uint32_t cb[QM];
  {
    float cut[2][QM];
    group_cuts<DT, QM>(s[0], cut[0]);
    group_cuts<DT, QM>(s[1], cut[1]);
#pragma unroll
    for (int k = 0; k < QM; ++k) cb[k] = cut_bits<DT>(cut[0][k]) | (cut_bits<DT>(cut[1][k]) << 16);
  }
  auto codes2 = [&](uint32_t w) -> uint32_t {
    if constexpr (ASYM) return asym_codes2<DT, BITS>(w, z2, cb);
    else return sym_codes2<DT, BITS>(w, cb);
  };
  for (int c0 = 0; c0 < group; c0 += 32) {
    // 3 / 4 bits: the chunk is read again (from L2) rather than kept in
    // registers across the cut computation, which would cost occupancy
    if (group > 32 || BITS > 2) load(c0);
#pragma unroll
    for (int t4 = 0; t4 < 8; ++t4) {
      const uint32_t f0 = codes2(raw[4 * t4]), f1 = codes2(raw[4 * t4 + 1]);
      const uint32_t f2 = codes2(raw[4 * t4 + 2]), f3 = codes2(raw[4 * t4 + 3]);
      // [f0.b0, f1.b0, f0.b2, f1.b2], [f2.b0, f3.b0, f2.b2, f3.b2]
      const uint32_t p01 = __byte_perm(f0, f1, 0x6240), p23 = __byte_perm(f2, f3, 0x6240);
      cbt[2 * dp][(c0 >> 2) + t4] = __byte_perm(p01, p23, 0x5410);
      cbt[2 * dp + 1][(c0 >> 2) + t4] = __byte_perm(p01, p23, 0x7632);
    }
  }
  const int64_t groups_cap = cap_tiles * 32 / group;
  const int64_t t_abs = t_off + (int64_t)gi * group;
  const int64_t gglob = t_abs / group;
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int64_t si = (bh * groups_cap + gglob) * kD + col_scale_idx(2 * dp + e);
    scale[si] = from_f<DT>(s[e]);
    if (ASYM) zero[si] = from_f<DT>(z[e]);
  }
  __syncthreads();
  store_col_tiles<BITS>(cbt, codes, bh, cap_tiles, t_abs, group / 32, threadIdx.x, 64);
}

template <int DT, int BITS, int ROLEV>
__global__ void __launch_bounds__(128)
pack_col_token_kernel(const uint16_t* __restrict__ x, int64_t sb, int64_t sh, int64_t st,
                      int group, int asym, uint8_t* __restrict__ codes,
                      uint16_t* __restrict__ scale, uint16_t* __restrict__ zero,
                      int64_t cap_tiles, int64_t t_off) {
  const int gi = blockIdx.x, h = blockIdx.y, b = blockIdx.z, H = gridDim.y;
  pack_col_group<DT, BITS, ROLEV>(x + b * sb + h * sh + (int64_t)gi * group * st, st, group, asym, codes,
                                  scale, zero, cap_tiles, t_off + (int64_t)gi * group, (int64_t)b * H + h);
}

// --------------------------------------------------------------------------
// Graph-mode decode append of one side (cache.py:283-307, 314-380): the new
// token goes to the recent FIFO; when the window then holds >= flush tokens
// the oldest `flush` are quantized and packed.  The step comes from a device
// counter (steps taken, this one included) and the state at step 0, so the
// launch replays from a CUDA graph.  Grid (H, B), 128 threads.
// MODE 0: channel groups, row layout (keys); 1: token groups, col layout
// (values); 2: channel groups, col layout (values); 3: no quantization;
// 4: token groups, row layout (keys grouped over tokens, KIVI).
// --------------------------------------------------------------------------
struct AppendDev {
  const uint16_t* x;
  int64_t x_b, x_h;
  uint16_t* fifo;
  int64_t f_b, f_h, f_t;
  int fifo_cap;
  uint8_t* codes;
  uint16_t* scale;
  uint16_t* zero;
  int64_t cap_tiles;
  const uint16_t* nf;
  int group, asym, flush, n_q, n_rec, r0, max_steps;
};

template <int DT, int BITS, int MODE>
__global__ void __launch_bounds__(128) append_step_kernel(const AppendDev a, const int64_t* __restrict__ step) {
  __shared__ uint32_t seg_unused[16];
  const int h = blockIdx.x, b = blockIdx.y, H = gridDim.x, d = threadIdx.x;
  const int64_t bh = (int64_t)b * H + h;
  griddep_wait();  // earlier kernels on the stream (the step counter's update) are done
  griddep_launch_dependents();
  if (*step < 1 || *step > a.max_steps) return;  // outside the reserved steps: write nothing
  const int n1 = (int)*step, n0 = n1 - 1;
  uint16_t* fifo = a.fifo + b * a.f_b + h * a.f_h;
  const int pos = a.r0 + a.n_rec + n0;
  if (pos < a.fifo_cap) fifo[(int64_t)pos * a.f_t + d] = a.x[b * a.x_b + h * a.x_h + d];
  if (MODE == 3) return;
  const int k0 = min(n0, (a.n_rec + n0) / a.flush), k1 = min(n1, (a.n_rec + n1) / a.flush);
  if (k1 == k0) return;
  const int f0 = a.r0 + a.flush * k0;
  const int64_t t0 = (int64_t)a.n_q + (int64_t)a.flush * k0;
  if (f0 + a.flush > a.fifo_cap || t0 + a.flush > a.cap_tiles * 32) return;  // beyond the reserved capacity
  __syncthreads();  // the new token may be one of those flushed
  if (MODE == 1 || MODE == 4) {
    // token groups: values (col layout) or keys (row layout, KIVI)
    for (int g = 0; g < a.flush; g += a.group) {
      pack_col_group<DT, BITS, MODE == 1 ? 1 : 0>(fifo + (int64_t)(f0 + g) * a.f_t, a.f_t, a.group, a.asym, a.codes, a.scale,
                                  a.zero, a.cap_tiles, t0 + g, bh);
      __syncthreads();
    }
  } else {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = warp; i < a.flush; i += 4) {
      const uint2 raw = *reinterpret_cast<const uint2*>(fifo + (int64_t)(f0 + i) * a.f_t + 4 * lane);
      pack_row_token<DT, BITS, MODE == 2 ? 1 : 0>(raw, i, bh, lane, seg_unused, a.nf, a.group, a.asym, a.codes,
                                                  a.scale, a.zero, a.cap_tiles, t0);
    }
  }
}

// --------------------------------------------------------------------------
// Code extraction at (packed token p, dim d) for either layout
// --------------------------------------------------------------------------
__device__ __forceinline__ int extract_code(const uint8_t* store_bh, int bits, int role_v,
                                            int64_t p, int d) {
  const int64_t ti = p >> 5;
  const int r = (int)(p & 31);
  const uint8_t* tb = store_bh + ti * tile_bytes(bits);
  const BitPos bp = role_v ? col_pos(bits, r, d) : row_pos(bits, r, d);
  const uint32_t w = *reinterpret_cast<const uint32_t*>(tb + bp.off);
  if (bits == 4) return (w >> bp.shift) & 15u;
  if (bits == 1) return (w >> bp.shift) & 1u;
  int u = (w >> bp.shift) & 3u;
  if (bits == 3) {
    const uint32_t wh = *reinterpret_cast<const uint32_t*>(tb + bp.hoff);
    u |= ((wh >> bp.hshift) & 1u) << 2;
  }
  return u;
}

// scale / zero element index of (packed token p, dim d) inside one (b,h) store
__device__ __forceinline__ int64_t scale_index(int role_v, int over_token, int group,
                                               int64_t cap_tiles, int64_t p, int d) {
  if (!over_token) {  // channel groups: row-layout tiles
    const int ng = kD / group;
    return (p >> 5) * 32 * ng + row_scale_idx((int)(p & 31), d / group, ng);
  }
  return (p / group) * kD + (role_v ? col_scale_idx(d) : d);  // keys: natural dim order
}

// Reference-format views (quant.py return values): int32 codes (magnitudes
// for symmetric), fp16/bf16 signs, and scale / zero point tensors.
template <int DT>
__global__ void unpack_ref_kernel(const uint8_t* __restrict__ codes, const uint16_t* __restrict__ scale,
                                  const uint16_t* __restrict__ zero, int H, int64_t n, int bits,
                                  int group, int asym, int role_v, int over_token, int64_t cap_tiles,
                                  int64_t t_begin, int32_t* __restrict__ oc, uint16_t* __restrict__ os,
                                  uint16_t* __restrict__ osc, uint16_t* __restrict__ oz, int64_t total) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int d = (int)(i % kD);
  const int64_t tn = (i / kD) % n;
  const int64_t bh = i / (kD * n);
  const int64_t p = t_begin + tn;
  const int64_t groups_cap = cap_tiles * 32 / group;
  const int64_t per_bh_scales = over_token ? groups_cap * kD : cap_tiles * 32 * (kD / group);
  const int u = extract_code(codes + bh * cap_tiles * tile_bytes(bits), bits, role_v, p, d);
  if (asym) {
    oc[i] = u;
  } else {
    const int v = u - (1 << (bits - 1));
    oc[i] = v < 0 ? -v : v;
    if (os) os[i] = from_f<DT>(v > 0 ? 1.f : (v < 0 ? -1.f : 0.f));
  }
  const int64_t si = bh * per_bh_scales + scale_index(role_v, over_token, group, cap_tiles, p, d);
  if (!over_token) {
    if (d % group == 0) {
      const int64_t o = (bh * n + tn) * (kD / group) + d / group;
      osc[o] = scale[si];
      if (asym && oz) oz[o] = zero[si];
    }
  } else if (tn % group == 0) {
    const int64_t o = (bh * (n / group) + tn / group) * kD + d;
    osc[o] = scale[si];
    if (asym && oz) oz[o] = zero[si];
  }
}

// Materialised dequantization in the model dtype, exactly as cache.py:241-281:
// fp32(c)*fp32(s) (*sign | +zero) [*f], then cast to the dtype.
template <int DT>
__global__ void dequant_kernel(const uint8_t* __restrict__ codes, const uint16_t* __restrict__ scale,
                               const uint16_t* __restrict__ zero, int H, int64_t n, int bits, int group,
                               int asym, int role_v, int over_token, int64_t cap_tiles, int64_t t_begin,
                               const uint16_t* __restrict__ nf, uint16_t* __restrict__ out, int64_t ob,
                               int64_t oh, int64_t ot, int64_t total) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int d = (int)(i % kD);
  const int64_t tn = (i / kD) % n;
  const int64_t bh = i / (kD * n);
  const int64_t p = t_begin + tn;
  const int64_t groups_cap = cap_tiles * 32 / group;
  const int64_t per_bh_scales = over_token ? groups_cap * kD : cap_tiles * 32 * (kD / group);
  const int u = extract_code(codes + bh * cap_tiles * tile_bytes(bits), bits, role_v, p, d);
  const int64_t si = bh * per_bh_scales + scale_index(role_v, over_token, group, cap_tiles, p, d);
  const float s = to_f<DT>(scale[si]);
  float val;
  if (asym) {
    val = (float)u * s + to_f<DT>(zero[si]);
  } else {
    val = (float)(u - (1 << (bits - 1))) * s;
  }
  if (nf) val = val * to_f<DT>(nf[bh * kD + d]);
  const int b = (int)(bh / H), h = (int)(bh % H);
  out[b * ob + h * oh + tn * ot + d] = from_f<DT>(val);
}

// --------------------------------------------------------------------------
// Split-KV log-sum-exp merge: out = sum_s 2^(m_s-M) O_s / sum_s 2^(m_s-M) l_s
// --------------------------------------------------------------------------
template <int DT, int VEC>
__global__ void __launch_bounds__(kMergeMaxWarps * 32)
lse_merge_kernel(const float* __restrict__ po, const float* __restrict__ pm, const float* __restrict__ pl,
                 int n_splits, int rows_per_b, int n_ranks, int64_t rank_stride, uint16_t* __restrict__ out,
                 int64_t o_b, int64_t o_h, float* __restrict__ lse_out) {
  // One CTA per output row; n_ranks blocks of partials, rank_stride floats
  // apart (one block per rank of a context-sharded layer, gathered; 1 block
  // otherwise), each with n_splits partials per row.  The splits are dealt
  // to the CTA's warps (warp w takes splits w, w + nw, ...), a lane holds 4
  // dims, so a warp reads one split's 128-dim row per (16-byte) load and the
  // CTA has nw of them in flight; the warps' sums meet in shared memory.
  __shared__ float4 acc_s[kMergeMaxWarps][32];
  __shared__ float den_s[kMergeMaxWarps], max_s[kMergeMaxWarps];
  griddep_wait();  // the attention grid's partials are complete and visible
  griddep_launch_dependents();
  const int row = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int total = n_ranks * n_splits;
  // split j = (rank w, split sp): offset of its (m, l) entry; its o row
  // starts at w * rank_stride + (row * n_splits + sp) * kD
  auto at = [&](int j) -> int64_t {
    const int w = j / n_splits, sp = j - w * n_splits;
    return w * rank_stride + (int64_t)row * n_splits + sp;
  };
  auto at_o = [&](int j) -> int64_t {
    const int w = j / n_splits, sp = j - w * n_splits;
    return w * rank_stride + ((int64_t)row * n_splits + sp) * kD;
  };
  // the row's largest split maximum
  float M = -INFINITY;
  for (int j = threadIdx.x; j < total; j += blockDim.x) M = fmaxf(M, pm[at(j)]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  if (lane == 0) max_s[warp] = M;
  __syncthreads();
  M = max_s[0];
  for (int w = 1; w < nw; ++w) M = fmaxf(M, max_s[w]);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float den = 0.f;
  if (M != -INFINITY) {
#pragma unroll 4
    for (int j = warp; j < total; j += nw) {
      const int64_t r = at(j);
      const float m = pm[r];
      // an empty split contributes nothing
      const float wt = m == -INFINITY ? 0.f : exp2f(m - M);
      den += wt * pl[r];
      const float* src = po + at_o(j);
      float4 v;
      if constexpr (VEC) {
        v = *reinterpret_cast<const float4*>(src + 4 * lane);
      } else {
        v = make_float4(src[4 * lane], src[4 * lane + 1], src[4 * lane + 2], src[4 * lane + 3]);
      }
      acc.x += wt * v.x; acc.y += wt * v.y; acc.z += wt * v.z; acc.w += wt * v.w;
    }
  }
  acc_s[warp][lane] = acc;
  if (lane == 0) den_s[warp] = den;
  __syncthreads();
  if (warp != 0) return;
  float4 num = acc_s[0][lane];
  float dsum = den_s[0];
  for (int w = 1; w < nw; ++w) {
    const float4 t = acc_s[w][lane];
    num.x += t.x; num.y += t.y; num.z += t.z; num.w += t.w;
    dsum += den_s[w];
  }
  const int b = row / rows_per_b, h = row % rows_per_b;
  uint16_t* o = out + b * o_b + h * o_h + 4 * lane;
  o[0] = from_f<DT>(dsum > 0.f ? num.x / dsum : 0.f);
  o[1] = from_f<DT>(dsum > 0.f ? num.y / dsum : 0.f);
  o[2] = from_f<DT>(dsum > 0.f ? num.z / dsum : 0.f);
  o[3] = from_f<DT>(dsum > 0.f ? num.w / dsum : 0.f);
  if (lse_out && lane == 0) lse_out[row] = dsum > 0.f ? M + log2f(dsum) : -INFINITY;
}


// Dequantize reference-format tensors (quant.py:83-93, 121-131): int32 codes,
// dtype scale and dtype sign (symmetric) or zero point (asymmetric), fp32 out.
template <int DT>
__global__ void dequant_ref_kernel(const int32_t* __restrict__ c, const uint16_t* __restrict__ s,
                                   const uint16_t* __restrict__ zs, int T, int D, int group, int asym,
                                   int over_token, float* __restrict__ out, int64_t total) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int d = (int)(i % D);
  const int64_t t = (i / D) % T;
  const int64_t o = i / ((int64_t)D * T);
  const int64_t si = over_token ? (o * (T / group) + t / group) * D + d
                                : (o * T + t) * (D / group) + d / group;
  float v = (float)c[i] * to_f<DT>(s[si]);
  if (asym) v = v + to_f<DT>(zs[si]);
  else v = v * to_f<DT>(zs[i]);
  out[i] = v;
}

// ------------------------------------------------------------ launchers ---
#define DT_DISPATCH(dt, ...)            \
  if ((dt) == F16) {                    \
    constexpr int DTC = F16;            \
    __VA_ARGS__;                        \
  } else {                              \
    constexpr int DTC = BF16;           \
    __VA_ARGS__;                        \
  }
#define BITS_DISPATCH(bits, ...)        \
  if ((bits) == 1) {                    \
    constexpr int BC = 1;               \
    __VA_ARGS__;                        \
  } else if ((bits) == 2) {             \
    constexpr int BC = 2;               \
    __VA_ARGS__;                        \
  } else if ((bits) == 3) {             \
    constexpr int BC = 3;               \
    __VA_ARGS__;                        \
  } else {                              \
    constexpr int BC = 4;               \
    __VA_ARGS__;                        \
  }

cudaError_t launch_norm_factor(const void* x, int dt, int B, int H, int T, int64_t sb, int64_t sh,
                               int64_t st, void* f, cudaStream_t s) {
  const bool pairs = ((uintptr_t)x % 4 == 0) && sb % 2 == 0 && sh % 2 == 0 && st % 2 == 0 &&
                     (uintptr_t)f % 4 == 0;
  if (!pairs) {
    DT_DISPATCH(dt, norm_factor_kernel<DTC><<<B * H, kD, 0, s>>>(
                        (const uint16_t*)x, sb, sh, st, H, T, (uint16_t*)f));
    return cudaGetLastError();
  }
  const int64_t n = (int64_t)B * H * kD;
  cudaError_t e = cudaMemsetAsync(f, 0, n * sizeof(uint16_t), s);
  if (e != cudaSuccess) return e;
  const dim3 grid((unsigned)((T + 511) / 512), (unsigned)H, (unsigned)B);
  DT_DISPATCH(dt, norm_absmax_kernel<DTC><<<grid, 256, 0, s>>>((const uint16_t*)x, sb, sh, st, T, (uint32_t*)f));
  DT_DISPATCH(dt, norm_sqrt_kernel<DTC><<<(unsigned)((n + 255) / 256), 256, 0, s>>>((uint16_t*)f, n));
  return cudaGetLastError();
}

cudaError_t launch_append_step(const AppendArgs& g, const int64_t* step, cudaStream_t s) {
  AppendDev a;
  a.x = (const uint16_t*)g.x; a.x_b = g.x_sb; a.x_h = g.x_sh;
  a.fifo = (uint16_t*)g.fifo; a.f_b = g.f_sb; a.f_h = g.f_sh; a.f_t = g.f_st; a.fifo_cap = g.fifo_cap;
  a.codes = (uint8_t*)g.codes; a.scale = (uint16_t*)g.scale; a.zero = (uint16_t*)g.zero;
  a.cap_tiles = g.cap_tiles; a.nf = (const uint16_t*)g.norm_f;
  a.group = g.group; a.asym = g.asym; a.flush = g.flush; a.n_q = g.n_q; a.n_rec = g.n_rec; a.r0 = g.r0;
  a.max_steps = g.max_steps;
  const dim3 grid((unsigned)g.H, (unsigned)g.B, 1);
  const int dt = g.dt, bits = g.bits;
  cudaError_t e = cudaSuccess;
  switch (g.mode) {
    case 0: DT_DISPATCH(dt, BITS_DISPATCH(bits, e = launch_pdl(append_step_kernel<DTC, BC, 0>, grid, dim3(128), 0, s, a, step))); break;
    case 1: DT_DISPATCH(dt, BITS_DISPATCH(bits, e = launch_pdl(append_step_kernel<DTC, BC, 1>, grid, dim3(128), 0, s, a, step))); break;
    case 2: DT_DISPATCH(dt, BITS_DISPATCH(bits, e = launch_pdl(append_step_kernel<DTC, BC, 2>, grid, dim3(128), 0, s, a, step))); break;
    case 4: DT_DISPATCH(dt, BITS_DISPATCH(bits, e = launch_pdl(append_step_kernel<DTC, BC, 4>, grid, dim3(128), 0, s, a, step))); break;
    default: DT_DISPATCH(dt, (e = launch_pdl(append_step_kernel<DTC, 4, 3>, grid, dim3(128), 0, s, a, step))); break;
  }
  return e;
}

// rows of 16-byte aligned, 16-byte strided 16-bit values
static bool rows16(const void* x, int64_t sb, int64_t sh, int64_t st) {
  return (uintptr_t)x % 16 == 0 && sb % 8 == 0 && sh % 8 == 0 && st % 8 == 0;
}

cudaError_t launch_pack(const void* x, int dt, int B, int H, int T, int64_t sb, int64_t sh,
                        int64_t st, int bits, int group, int asym, int role_v, int over_token,
                        const void* nf, void* codes, void* scale, void* zero, int64_t cap_tiles,
                        int64_t t_off, cudaStream_t s) {
  if (!over_token && !role_v && bits >= 2 && rows16(x, sb, sh, st)) {
    // keys, channel groups: one thread per (token, 32-dim block)
    const dim3 grid((unsigned)((T + 63) / 64), (unsigned)H, (unsigned)B);
#define PACK_ROWS(A, N)                                                                          \
  DT_DISPATCH(dt, BITS_DISPATCH(bits, pack_rows_kernel<DTC, (BC < 2 ? 2 : BC), A, N><<<grid, 256, 0, s>>>( \
                                          (const uint16_t*)x, sb, sh, st, T, (const uint16_t*)nf,   \
                                          group, (uint8_t*)codes, (uint16_t*)scale, (uint16_t*)zero,  \
                                          cap_tiles, t_off)))
    if (asym && nf) {
      PACK_ROWS(1, 1);
    } else if (asym) {
      PACK_ROWS(1, 0);
    } else if (nf) {
      PACK_ROWS(0, 1);
    } else {
      PACK_ROWS(0, 0);
    }
#undef PACK_ROWS
  } else if (!over_token) {
    const dim3 grid((unsigned)((T + 31) / 32), (unsigned)H, (unsigned)B);
    if (role_v) {
      DT_DISPATCH(dt, BITS_DISPATCH(bits, pack_row_channel_kernel<DTC, BC, 1><<<grid, 256, 0, s>>>(
                                              (const uint16_t*)x, sb, sh, st, H, T,
                                              (const uint16_t*)nf, group, asym, (uint8_t*)codes,
                                              (uint16_t*)scale, (uint16_t*)zero, cap_tiles, t_off)));
    } else {
      DT_DISPATCH(dt, BITS_DISPATCH(bits, pack_row_channel_kernel<DTC, BC, 0><<<grid, 256, 0, s>>>(
                                              (const uint16_t*)x, sb, sh, st, H, T,
                                              (const uint16_t*)nf, group, asym, (uint8_t*)codes,
                                              (uint16_t*)scale, (uint16_t*)zero, cap_tiles, t_off)));
    }
  } else if (role_v && bits >= 2 && (uintptr_t)x % 4 == 0 && sb % 2 == 0 && sh % 2 == 0 && st % 2 == 0) {
    // values, token groups: 64 threads x 2 dims per group
    dim3 grid(T / group, H, B);
    if (asym) {
      DT_DISPATCH(dt, BITS_DISPATCH(bits, pack_cols_kernel<DTC, (BC < 2 ? 2 : BC), 1><<<grid, 64, 0, s>>>(
                                              (const uint16_t*)x, sb, sh, st, group, (uint8_t*)codes,
                                              (uint16_t*)scale, (uint16_t*)zero, cap_tiles, t_off)));
    } else {
      DT_DISPATCH(dt, BITS_DISPATCH(bits, pack_cols_kernel<DTC, (BC < 2 ? 2 : BC), 0><<<grid, 64, 0, s>>>(
                                              (const uint16_t*)x, sb, sh, st, group, (uint8_t*)codes,
                                              (uint16_t*)scale, (uint16_t*)zero, cap_tiles, t_off)));
    }
  } else {
    dim3 grid(T / group, H, B);
    if (role_v) {
      DT_DISPATCH(dt, BITS_DISPATCH(bits, pack_col_token_kernel<DTC, BC, 1><<<grid, 128, 0, s>>>(
                                              (const uint16_t*)x, sb, sh, st, group, asym,
                                              (uint8_t*)codes, (uint16_t*)scale, (uint16_t*)zero,
                                              cap_tiles, t_off)));
    } else {
      DT_DISPATCH(dt, BITS_DISPATCH(bits, pack_col_token_kernel<DTC, BC, 0><<<grid, 128, 0, s>>>(
                                              (const uint16_t*)x, sb, sh, st, group, asym,
                                              (uint8_t*)codes, (uint16_t*)scale, (uint16_t*)zero,
                                              cap_tiles, t_off)));
    }
  }
  return cudaGetLastError();
}

cudaError_t launch_unpack_ref(const void* codes, const void* scale, const void* zero, int dt, int B,
                              int H, int64_t n, int bits, int group, int asym, int role_v,
                              int over_token, int64_t cap_tiles, int64_t t_begin, int32_t* oc,
                              void* os, void* osc, void* oz, cudaStream_t s) {
  const int64_t total = (int64_t)B * H * n * kD;
  if (total == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((total + 255) / 256);
  DT_DISPATCH(dt, unpack_ref_kernel<DTC><<<grid, 256, 0, s>>>(
                      (const uint8_t*)codes, (const uint16_t*)scale, (const uint16_t*)zero, H, n,
                      bits, group, asym, role_v, over_token, cap_tiles, t_begin, oc,
                      (uint16_t*)os, (uint16_t*)osc, (uint16_t*)oz, total));
  return cudaGetLastError();
}

cudaError_t launch_dequant(const void* codes, const void* scale, const void* zero, int dt, int B,
                           int H, int64_t n, int bits, int group, int asym, int role_v,
                           int over_token, int64_t cap_tiles, int64_t t_begin, const void* nf,
                           void* out, int64_t ob, int64_t oh, int64_t ot, cudaStream_t s) {
  const int64_t total = (int64_t)B * H * n * kD;
  if (total == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((total + 255) / 256);
  DT_DISPATCH(dt, dequant_kernel<DTC><<<grid, 256, 0, s>>>(
                      (const uint8_t*)codes, (const uint16_t*)scale, (const uint16_t*)zero, H, n,
                      bits, group, asym, role_v, over_token, cap_tiles, t_begin,
                      (const uint16_t*)nf, (uint16_t*)out, ob, oh, ot, total));
  return cudaGetLastError();
}

cudaError_t launch_lse_merge(const float* po, const float* pm, const float* pl, int rows,
                             int rows_per_b, int n_splits, int dt, void* out, int64_t o_b,
                             int64_t o_h, float* lse, cudaStream_t s, int n_ranks,
                             int64_t rank_stride) {
  if (rows == 0) return cudaSuccess;
  cudaError_t e = cudaSuccess;
  // one warp per split up to kMergeMaxWarps; 16-byte loads when aligned
  const int nw = (int)std::min<int64_t>(kMergeMaxWarps, std::max<int64_t>(1, (int64_t)n_splits * n_ranks));
  const bool vec = (uintptr_t)po % 16 == 0 && (n_ranks == 1 || rank_stride % 4 == 0);
  if (vec) {
    DT_DISPATCH(dt, e = launch_pdl(lse_merge_kernel<DTC, 1>, dim3(rows), dim3(32 * nw), 0, s, po, pm, pl,
                                   n_splits, rows_per_b, n_ranks, rank_stride, (uint16_t*)out, o_b, o_h, lse));
  } else {
    DT_DISPATCH(dt, e = launch_pdl(lse_merge_kernel<DTC, 0>, dim3(rows), dim3(32 * nw), 0, s, po, pm, pl,
                                   n_splits, rows_per_b, n_ranks, rank_stride, (uint16_t*)out, o_b, o_h, lse));
  }
  return e;
}

cudaError_t launch_dequant_ref(const int32_t* c, const void* s, const void* zs, int dt, int64_t n_outer,
                               int T, int D, int group, int asym, int over_token, float* out,
                               cudaStream_t st) {
  const int64_t total = n_outer * T * D;
  if (total == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((total + 255) / 256);
  DT_DISPATCH(dt, dequant_ref_kernel<DTC><<<grid, 256, 0, st>>>(c, (const uint16_t*)s,
                                                                (const uint16_t*)zs, T, D, group, asym,
                                                                over_token, out, total));
  return cudaGetLastError();
}

}  // namespace innerq
