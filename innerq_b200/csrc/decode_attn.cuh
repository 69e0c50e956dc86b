// Fused InnerQ decode attention over [sink fp16 | packed middle | recent fp16].
//
// Replaces, for one decode step of one layer, the reference sequence
//   cache.py:235-281  get_deq_tensors()  (full fp32 dequant + concat + cast)
//   HF sdpa           softmax(q K^T * scale) V   (GQA via repeat_kv)
// with one pass that reads the packed codes once and dequantizes in registers.
//
// Work decomposition: grid (split, kv_head, batch), 4 warps per CTA.  The
// token axis is cut into 32-token tiles aligned to the V packed grid; each CTA
// owns a contiguous range of tiles (a split) and each warp takes every 4th
// tile of that range with its own online-softmax state.  The CTA writes an
// unnormalised partial (O, m, l) per query head; lse_merge() combines splits
// (and GPUs when context chunks are sharded).
//
// Inner products use mma.sync m16n8k16 with register-resident A fragments:
//   QK^T: A = K tile [token][dim] decoded from the row layout, B = q*f split
//         into fp16 hi+lo columns (8 columns = 4 query heads x {hi,lo}), one
//         accumulator per channel group, scaled by the group scale in fp32.
//   PV:   A = V^T tile [dim][token] decoded from the col layout, B = P split
//         into hi+lo, scaled by the (token-group, dim) scale in fp32.
// The hi/lo split keeps ~22 mantissa bits, so results match an fp32
// dequantize-then-matmul to ~1e-6 relative.
#pragma once
#include "common.cuh"

namespace innerq {

struct DevSide {
  const uint8_t* codes;
  const uint16_t* scale;
  const uint16_t* zero;
  int64_t cap_tiles;
  const uint16_t* sink;
  int64_t sk_b, sk_h, sk_t;
  const uint16_t* rec;
  int64_t rc_b, rc_h, rc_t;
  int n_sink, n_q, n_rec;
  int group;
  int asym;
};

struct DevArgs {
  DevSide k, v;
  const uint16_t* q;
  int64_t q_b, q_h;
  const uint16_t* kf;  // key normalisation factor [B][Hkv][D] or null
  int B, Hq, Hkv, S;
  int t_first;         // token index of tile 0 (<= 0)
  int tile_lo, tile_hi;
  int tiles_per_split, n_splits;
  float scale_log2;    // softmax scale * log2(e)
  float* po;           // [B][Hq][n_splits][D]
  float* pm;           // [B][Hq][n_splits]
  float* pl;
};

constexpr int kWarps = 4;

template <int R>
struct AttnSmem {
  static constexpr int NT = (R + 3) / 4;
  float q_s[R][kD];     // q * f * 2^e_p
  float qd_s[R][kD];    // q * 2^e_d
  float qsum_s[R][8];   // asym K: per channel group sum of q_s
  uint2 bd_s[NT][8][32];
  float p_s[kWarps][R][kTile];
  float red_s[2][kWarps];
  float cm_s[kWarps][R];
  float cl_s[kWarps][R];
  float co_s[kWarps][R][kD];
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// reduce across the 8 lanes that share tq (lane bits 2..4)
__device__ __forceinline__ float gid_max(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
  return v;
}
__device__ __forceinline__ float gid_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  v += __shfl_xor_sync(0xffffffffu, v, 16);
  return v;
}

// per-row K words of one packed token row (row layout)
template <int BITS> struct KRow { uint32_t w[BITS == 4 ? 4 : 3]; };

template <int BITS>
__device__ __forceinline__ void load_krow(KRow<BITS>& r, const uint8_t* tilebase, int lane2, int j) {
  if constexpr (BITS == 4) {
    uint4 v = *reinterpret_cast<const uint4*>(tilebase + lane2 * 64 + j * 16);
    r.w[0] = v.x; r.w[1] = v.y; r.w[2] = v.z; r.w[3] = v.w;
  } else if constexpr (BITS == 2) {
    uint2 v = *reinterpret_cast<const uint2*>(tilebase + lane2 * 32 + j * 8);
    r.w[0] = v.x; r.w[1] = v.y; r.w[2] = 0;
  } else {
    uint2 v = *reinterpret_cast<const uint2*>(tilebase + lane2 * 32 + j * 8);
    r.w[0] = v.x; r.w[1] = v.y;
    r.w[2] = *reinterpret_cast<const uint32_t*>(tilebase + 1024 + lane2 * 16 + j * 4);
  }
}

// fp16 pair for (kb, hi8) of a packed K row
template <int BITS>
__device__ __forceinline__ uint32_t krow_pair(const KRow<BITS>& r, int kb, int hi8, uint32_t bias) {
  if constexpr (BITS == 4) {
    return Dec<4>::pair(r.w[kb >> 1], (kb & 1) * 2 + hi8, bias);
  } else if constexpr (BITS == 2) {
    return Dec<2>::pair(r.w[kb >> 2], (kb & 3) * 2 + hi8, bias);
  } else {
    return Dec3::pair(r.w[kb >> 2], (kb & 3) * 2 + hi8, r.w[2], kb * 2 + hi8, bias);
  }
}

// per-lane V chunk (col layout)
template <int BITS> struct VChunk { uint32_t w[BITS == 4 ? 16 : (BITS == 2 ? 8 : 12)]; };

template <int BITS>
__device__ __forceinline__ void load_vchunk(VChunk<BITS>& c, const uint8_t* tilebase, int lane) {
  if constexpr (BITS == 4) {
    const uint4* p = reinterpret_cast<const uint4*>(tilebase + lane * 64);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 v = p[i];
      c.w[4 * i] = v.x; c.w[4 * i + 1] = v.y; c.w[4 * i + 2] = v.z; c.w[4 * i + 3] = v.w;
    }
  } else {
    const uint4* p = reinterpret_cast<const uint4*>(tilebase + lane * 32);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      uint4 v = p[i];
      c.w[4 * i] = v.x; c.w[4 * i + 1] = v.y; c.w[4 * i + 2] = v.z; c.w[4 * i + 3] = v.w;
    }
    if constexpr (BITS == 3) {
      uint4 v = *reinterpret_cast<const uint4*>(tilebase + 1024 + lane * 16);
      c.w[8] = v.x; c.w[9] = v.y; c.w[10] = v.z; c.w[11] = v.w;
    }
  }
}

template <int BITS>
__device__ __forceinline__ uint32_t vchunk_pair(const VChunk<BITS>& c, int mt, int h, int kb,
                                                int hi8, uint32_t bias) {
  if constexpr (BITS == 4) {
    return Dec<4>::pair(c.w[mt * 2 + h], kb * 2 + hi8, bias);
  } else if constexpr (BITS == 2) {
    return Dec<2>::pair(c.w[mt], h * 4 + kb * 2 + hi8, bias);
  } else {
    return Dec3::pair(c.w[mt], h * 4 + kb * 2 + hi8, c.w[8 + (mt >> 1)],
                      (mt & 1) * 8 + h * 4 + kb * 2 + hi8, bias);
  }
}

// Dense (fp16/bf16) K row pointer for token t, or null when t is not a dense
// token of this side.
__device__ __forceinline__ const uint16_t* dense_row(const DevSide& s, int b, int h, int t, int S) {
  if (t < 0 || t >= S) return nullptr;
  if (t < s.n_sink) return s.sink + b * s.sk_b + h * s.sk_h + (int64_t)t * s.sk_t;
  int r = t - s.n_sink - s.n_q;
  if (r >= 0) return s.rec + b * s.rc_b + h * s.rc_h + (int64_t)r * s.rc_t;
  return nullptr;
}

template <int BK, int BV, int R, int DT>
__global__ void __launch_bounds__(kWarps * 32)
decode_attn_kernel(const DevArgs a) {
  constexpr int NT = (R + 3) / 4;
  __shared__ AttnSmem<R> sm;
  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tq = lane & 3;
  const int tile_beg = a.tile_lo + split * a.tiles_per_split;
  const int tile_end = min(tile_beg + a.tiles_per_split, a.tile_hi);
  const int S = a.S;

  // ---------------------------------------------------------------- prologue
  float amax_p = 0.f, amax_d = 0.f;
  for (int i = threadIdx.x; i < R * kD; i += kWarps * 32) {
    int h = i / kD, d = i % kD;
    float qv = to_f<DT>(a.q[b * a.q_b + (int64_t)(hk * R + h) * a.q_h + d]);
    float f = a.kf ? to_f<DT>(a.kf[((int64_t)b * a.Hkv + hk) * kD + d]) : 1.f;
    float qp = qv * f;
    sm.q_s[h][d] = qp;
    sm.qd_s[h][d] = qv;
    amax_p = fmaxf(amax_p, fabsf(qp));
    amax_d = fmaxf(amax_d, fabsf(qv));
  }
  amax_p = warp_max(amax_p);
  amax_d = warp_max(amax_d);
  if (lane == 0) { sm.red_s[0][warp] = amax_p; sm.red_s[1][warp] = amax_d; }
  __syncthreads();
  amax_p = fmaxf(fmaxf(sm.red_s[0][0], sm.red_s[0][1]), fmaxf(sm.red_s[0][2], sm.red_s[0][3]));
  amax_d = fmaxf(fmaxf(sm.red_s[1][0], sm.red_s[1][1]), fmaxf(sm.red_s[1][2], sm.red_s[1][3]));
  int ex;
  int e_p = 0, e_d = 0;
  if (amax_p > 0.f) { frexpf(amax_p, &ex); e_p = 15 - ex; }
  if (amax_d > 0.f) { frexpf(amax_d, &ex); e_d = 15 - ex; }
  for (int i = threadIdx.x; i < R * kD; i += kWarps * 32) {
    int h = i / kD, d = i % kD;
    sm.q_s[h][d] = ldexpf(sm.q_s[h][d], e_p);
    sm.qd_s[h][d] = ldexpf(sm.qd_s[h][d], e_d);
  }
  __syncthreads();
  const int ng = kD / a.k.group;  // channel groups per K token (valid for the packed K path)
  if (a.k.asym) {
    for (int i = threadIdx.x; i < R * ng; i += kWarps * 32) {
      int h = i / ng, g = i % ng;
      float s = 0.f;
      for (int d = g * a.k.group; d < (g + 1) * a.k.group; ++d) s += sm.q_s[h][d];
      sm.qsum_s[h][g] = s;
    }
  }
  // dense-K B fragments (dtype hi/lo)
  for (int i = threadIdx.x; i < NT * 8 * 32; i += kWarps * 32) {
    int nt = i / 256, kb = (i / 32) % 8, ln = i % 32;
    int g2 = ln >> 2, t2 = ln & 3;
    int head = nt * 4 + (g2 >> 1), part = g2 & 1;
    uint16_t v[4];
    const int dd[4] = {kb * 16 + 2 * t2, kb * 16 + 2 * t2 + 1, kb * 16 + 2 * t2 + 8, kb * 16 + 2 * t2 + 9};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float x = head < R ? sm.qd_s[head][dd[u]] : 0.f;
      uint16_t hi, lo;
      split_hilo<DT>(x, hi, lo);
      v[u] = part ? lo : hi;
    }
    sm.bd_s[nt][kb][ln] = make_uint2(pack2(v[0], v[1]), pack2(v[2], v[3]));
  }
  // packed-K B fragments in registers (fp16 hi/lo of q*f*2^e_p)
  uint32_t bk[NT][8][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    int head = nt * 4 + (gid >> 1), part = gid & 1;
#pragma unroll
    for (int kb = 0; kb < 8; ++kb) {
      uint16_t v[4];
      const int dd[4] = {kb * 16 + 2 * tq, kb * 16 + 2 * tq + 1, kb * 16 + 2 * tq + 8, kb * 16 + 2 * tq + 9};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float x = head < R ? sm.q_s[head][dd[u]] : 0.f;
        uint16_t hi, lo;
        split_hilo<F16>(x, hi, lo);
        v[u] = part ? lo : hi;
      }
      bk[nt][kb][0] = pack2(v[0], v[1]);
      bk[nt][kb][1] = pack2(v[2], v[3]);
    }
  }
  __syncthreads();

  const float cp = ldexpf(a.scale_log2, -e_p);
  const float cd = ldexpf(a.scale_log2, -e_d);
  const int ks = a.k.n_sink, nqk = a.k.n_q;
  const int vs = a.v.n_sink, nqv = a.v.n_q;
  const uint32_t kbias = bias_pair(a.k.asym ? 0 : (1 << (BK - 1)));
  const uint32_t vbias = bias_pair(a.v.asym ? 0 : (1 << (BV - 1)));
  const int64_t kbh = (int64_t)b * a.Hkv + hk;
  const uint8_t* kcodes = a.k.codes ? a.k.codes + kbh * a.k.cap_tiles * tile_bytes(BK) : nullptr;
  const uint16_t* kscale = a.k.scale ? a.k.scale + kbh * a.k.cap_tiles * 32 * ng : nullptr;
  const uint16_t* kzero = a.k.zero ? a.k.zero + kbh * a.k.cap_tiles * 32 * ng : nullptr;
  const uint8_t* vcodes = a.v.codes ? a.v.codes + kbh * a.v.cap_tiles * tile_bytes(BV) : nullptr;
  const int64_t vgroups_cap = a.v.codes ? a.v.cap_tiles * 32 / a.v.group : 0;
  const uint16_t* vscale = a.v.scale ? a.v.scale + kbh * vgroups_cap * kD : nullptr;
  const uint16_t* vzero = a.v.zero ? a.v.zero + kbh * vgroups_cap * kD : nullptr;

  float m_run[NT], l_run[NT], o[NT][8][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    m_run[nt] = -INFINITY;
    l_run[nt] = 0.f;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) o[nt][mt][0] = o[nt][mt][1] = 0.f;
  }

  // ---------------------------------------------------------------- tiles
  for (int tile = tile_beg + warp; tile < tile_end; tile += kWarps) {
    const int t0 = a.t_first + tile * kTile;
    float x[NT][4];
    // row sources: 1 packed, 2 dense, 0 masked
    int src[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int t = t0 + gid + 8 * j;
      src[j] = (t < 0 || t >= S) ? 0 : ((t >= ks && t < ks + nqk) ? 1 : 2);
    }
    const int lo_t = max(t0, 0), hi_t = min(t0 + kTile, S);
    const bool kp_any = nqk > 0 && lo_t < ks + nqk && hi_t > ks;
    const bool kd_any = (lo_t < min(ks, hi_t)) || (hi_t > max(ks + nqk, lo_t));

    float lp[NT][4], ld[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) lp[nt][j] = ld[nt][j] = 0.f;

    if (kp_any) {
      KRow<BK> rw[4];
      float sc[4][4], zc[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int p = t0 + gid + 8 * j - ks;
#pragma unroll
        for (int g = 0; g < 4; ++g) { sc[j][g] = 0.f; zc[j][g] = 0.f; }
        if (src[j] == 1) {
          const int ti = p >> 5, r = p & 31;
          load_krow<BK>(rw[j], kcodes + (int64_t)ti * tile_bytes(BK), (r & 7) * 4 + tq, r >> 3);
          const int64_t so = (int64_t)ti * 32 * ng + ((r & 7) * 4 + (r >> 3)) * ng;
#pragma unroll
          for (int g = 0; g < 4; ++g)
            if (g < ng) sc[j][g] = to_f<DT>(kscale[so + g]);
          if (a.k.asym) {
#pragma unroll
            for (int g = 0; g < 4; ++g)
              if (g < ng) zc[j][g] = to_f<DT>(kzero[so + g]);
          }
        } else {
#pragma unroll
          for (int u = 0; u < (BK == 4 ? 4 : 3); ++u) rw[j].w[u] = 0;
        }
      }
      // k-blocks per channel group: 2 (G=32), 4 (G=64), 8 (G=128)
      const int kpg_shift = a.k.group == 32 ? 1 : (a.k.group == 64 ? 2 : 3);
      const int kpg_mask = (1 << kpg_shift) - 1;
      float acc[2][NT][4];
#pragma unroll
      for (int kb = 0; kb < 8; ++kb) {
        if ((kb & kpg_mask) == 0) {
#pragma unroll
          for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
              acc[mt][nt][0] = acc[mt][nt][1] = acc[mt][nt][2] = acc[mt][nt][3] = 0.f;
        }
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          uint32_t af[4];
          af[0] = krow_pair<BK>(rw[2 * mt], kb, 0, kbias);
          af[1] = krow_pair<BK>(rw[2 * mt + 1], kb, 0, kbias);
          af[2] = krow_pair<BK>(rw[2 * mt], kb, 1, kbias);
          af[3] = krow_pair<BK>(rw[2 * mt + 1], kb, 1, kbias);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) mma_f16(acc[mt][nt], af, bk[nt][kb]);
        }
        if ((kb & kpg_mask) == kpg_mask) {
          const int g = kb >> kpg_shift;
          float s[4], z[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            s[j] = g == 0 ? sc[j][0] : g == 1 ? sc[j][1] : g == 2 ? sc[j][2] : sc[j][3];
            z[j] = g == 0 ? zc[j][0] : g == 1 ? zc[j][1] : g == 2 ? zc[j][2] : zc[j][3];
          }
#pragma unroll
          for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              lp[nt][2 * mt] += s[2 * mt] * (acc[mt][nt][0] + acc[mt][nt][1]);
              lp[nt][2 * mt + 1] += s[2 * mt + 1] * (acc[mt][nt][2] + acc[mt][nt][3]);
            }
          if (a.k.asym) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const int head = nt * 4 + tq;
              const float qs = head < R ? sm.qsum_s[head][g] : 0.f;
#pragma unroll
              for (int j = 0; j < 4; ++j) lp[nt][j] += z[j] * qs;
            }
          }
        }
      }
    }
    if (kd_any) {
      const uint16_t* rp[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        rp[j] = src[j] == 2 ? dense_row(a.k, b, hk, t0 + gid + 8 * j, S) : nullptr;
#pragma unroll
      for (int kb = 0; kb < 8; ++kb) {
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          uint32_t af[4];
          const uint16_t* r0 = rp[2 * mt];
          const uint16_t* r1 = rp[2 * mt + 1];
          int c0 = kb * 16 + 2 * tq;
          af[0] = r0 ? *reinterpret_cast<const uint32_t*>(r0 + c0) : 0u;
          af[1] = r1 ? *reinterpret_cast<const uint32_t*>(r1 + c0) : 0u;
          af[2] = r0 ? *reinterpret_cast<const uint32_t*>(r0 + c0 + 8) : 0u;
          af[3] = r1 ? *reinterpret_cast<const uint32_t*>(r1 + c0 + 8) : 0u;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            uint2 bb = sm.bd_s[nt][kb][lane];
            uint32_t bf[2] = {bb.x, bb.y};
            float c[4] = {0.f, 0.f, 0.f, 0.f};
            mma_dt<DT>(c, af, bf);
            ld[nt][2 * mt] += c[0] + c[1];
            ld[nt][2 * mt + 1] += c[2] + c[3];
          }
        }
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const bool head_ok = nt * 4 + tq < R;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        x[nt][j] = (!head_ok || src[j] == 0) ? -INFINITY
                   : (src[j] == 1 ? lp[nt][j] * cp : ld[nt][j] * cd);
    }

    // ------------------------------------------------------------ softmax
    float psum[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float mx = fmaxf(fmaxf(x[nt][0], x[nt][1]), fmaxf(x[nt][2], x[nt][3]));
      mx = gid_max(mx);
      const float m_new = fmaxf(m_run[nt], mx);
      float alpha = 1.f, ps = 0.f;
      float p[4];
      if (m_new == -INFINITY) {
        p[0] = p[1] = p[2] = p[3] = 0.f;
      } else {
        alpha = exp2f(m_run[nt] - m_new);
#pragma unroll
        for (int j = 0; j < 4; ++j) { p[j] = exp2f(x[nt][j] - m_new); ps += p[j]; }
      }
      m_run[nt] = m_new;
      l_run[nt] = l_run[nt] * alpha + ps;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) { o[nt][mt][0] *= alpha; o[nt][mt][1] *= alpha; }
      psum[nt] = ps;
      const int head = nt * 4 + tq;
      if (head < R) {
#pragma unroll
        for (int j = 0; j < 4; ++j) sm.p_s[warp][head][gid + 8 * j] = p[j];
      }
    }
    __syncwarp();

    // ------------------------------------------------------------------ PV
    const bool vpacked = nqv > 0 && t0 >= vs && t0 + kTile <= vs + nqv;
    if (vpacked) {
      if (a.v.asym) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) psum[nt] = gid_sum(psum[nt]);
      }
      uint32_t pb[NT][2][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int head = nt * 4 + (gid >> 1), part = gid & 1;
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          uint16_t v[4];
          const int rr[4] = {kb * 16 + 2 * tq, kb * 16 + 2 * tq + 1, kb * 16 + 2 * tq + 8, kb * 16 + 2 * tq + 9};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float pv = head < R ? sm.p_s[warp][head][rr[u]] : 0.f;
            uint16_t hi, lo;
            split_hilo<F16>(pv, hi, lo);
            v[u] = part ? lo : hi;
          }
          pb[nt][kb][0] = pack2(v[0], v[1]);
          pb[nt][kb][1] = pack2(v[2], v[3]);
        }
      }
      const int pv_tok = t0 - vs;
      VChunk<BV> vc;
      load_vchunk<BV>(vc, vcodes + (int64_t)(pv_tok >> 5) * tile_bytes(BV), lane);
      const int gg = pv_tok / a.v.group;
      uint16_t sv[16], zv[16];
      {
        const uint4* sp = reinterpret_cast<const uint4*>(vscale + (int64_t)gg * kD + gid * 16);
        uint4 s0 = sp[0], s1 = sp[1];
        const uint32_t sw[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
        for (int u = 0; u < 8; ++u) { sv[2 * u] = sw[u] & 0xffff; sv[2 * u + 1] = sw[u] >> 16; }
        if (a.v.asym) {
          const uint4* zp = reinterpret_cast<const uint4*>(vzero + (int64_t)gg * kD + gid * 16);
          uint4 z0 = zp[0], z1 = zp[1];
          const uint32_t zw[8] = {z0.x, z0.y, z0.z, z0.w, z1.x, z1.y, z1.z, z1.w};
#pragma unroll
          for (int u = 0; u < 8; ++u) { zv[2 * u] = zw[u] & 0xffff; zv[2 * u + 1] = zw[u] >> 16; }
        }
      }
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        float acc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          uint32_t af[4];
          af[0] = vchunk_pair<BV>(vc, mt, 0, kb, 0, vbias);
          af[1] = vchunk_pair<BV>(vc, mt, 1, kb, 0, vbias);
          af[2] = vchunk_pair<BV>(vc, mt, 0, kb, 1, vbias);
          af[3] = vchunk_pair<BV>(vc, mt, 1, kb, 1, vbias);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) mma_f16(acc[nt], af, pb[nt][kb]);
        }
        const float s0 = to_f<DT>(sv[mt * 2]), s1 = to_f<DT>(sv[mt * 2 + 1]);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          o[nt][mt][0] += s0 * (acc[nt][0] + acc[nt][1]);
          o[nt][mt][1] += s1 * (acc[nt][2] + acc[nt][3]);
          if (a.v.asym) {
            o[nt][mt][0] += to_f<DT>(zv[mt * 2]) * psum[nt];
            o[nt][mt][1] += to_f<DT>(zv[mt * 2 + 1]) * psum[nt];
          }
        }
      }
    } else {
      // dense V tile (sink / recent / masked rows)
      uint32_t pb[NT][2][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int head = nt * 4 + (gid >> 1), part = gid & 1;
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          uint16_t v[4];
          const int rr[4] = {kb * 16 + 2 * tq, kb * 16 + 2 * tq + 1, kb * 16 + 2 * tq + 8, kb * 16 + 2 * tq + 9};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float pv = head < R ? sm.p_s[warp][head][rr[u]] : 0.f;
            uint16_t hi, lo;
            split_hilo<DT>(pv, hi, lo);
            v[u] = part ? lo : hi;
          }
          pb[nt][kb][0] = pack2(v[0], v[1]);
          pb[nt][kb][1] = pack2(v[2], v[3]);
        }
      }
      const uint16_t* vp[2][4];
#pragma unroll
      for (int kb = 0; kb < 2; ++kb) {
        const int rr[4] = {kb * 16 + 2 * tq, kb * 16 + 2 * tq + 1, kb * 16 + 2 * tq + 8, kb * 16 + 2 * tq + 9};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          int t = t0 + rr[u];
          bool dense = t >= 0 && t < S && !(t >= vs && t < vs + nqv);
          vp[kb][u] = dense ? dense_row(a.v, b, hk, t, S) : nullptr;
        }
      }
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int d0 = mt * 16 + gid;
        float acc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          uint16_t e[4][2];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            e[u][0] = vp[kb][u] ? vp[kb][u][d0] : (uint16_t)0;
            e[u][1] = vp[kb][u] ? vp[kb][u][d0 + 8] : (uint16_t)0;
          }
          uint32_t af[4];
          af[0] = pack2(e[0][0], e[1][0]);
          af[1] = pack2(e[0][1], e[1][1]);
          af[2] = pack2(e[2][0], e[3][0]);
          af[3] = pack2(e[2][1], e[3][1]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) mma_dt<DT>(acc[nt], af, pb[nt][kb]);
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          o[nt][mt][0] += acc[nt][0] + acc[nt][1];
          o[nt][mt][1] += acc[nt][2] + acc[nt][3];
        }
      }
    }
    __syncwarp();
  }

  // ------------------------------------------------------- combine warps
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const float l = gid_sum(l_run[nt]);
    const int head = nt * 4 + tq;
    if (head < R) {
      if (gid == 0) { sm.cm_s[warp][head] = m_run[nt]; sm.cl_s[warp][head] = l; }
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        sm.co_s[warp][head][mt * 16 + gid] = o[nt][mt][0];
        sm.co_s[warp][head][mt * 16 + 8 + gid] = o[nt][mt][1];
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < R * kD; i += kWarps * 32) {
    const int head = i / kD, d = i % kD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sm.cm_s[w][head]);
    float ov = 0.f, lv = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float mw = sm.cm_s[w][head];
        const float wt = mw == -INFINITY ? 0.f : exp2f(mw - M);
        ov += wt * sm.co_s[w][head][d];
        lv += wt * sm.cl_s[w][head];
      }
    }
    const int64_t row = ((int64_t)b * a.Hq + hk * R + head) * a.n_splits + split;
    a.po[row * kD + d] = ov;
    if (d == 0) { a.pm[row] = M; a.pl[row] = lv; }
  }
}

}  // namespace innerq
