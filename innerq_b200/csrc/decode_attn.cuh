// Fused InnerQ decode attention over [sink fp16 | packed middle | recent fp16].
//
// Replaces, for one decode step of one layer, the reference sequence
//   cache.py:235-281  get_deq_tensors()  (full fp32 dequant + concat + cast)
//   HF sdpa           softmax(q K^T * scale) V   (GQA via repeat_kv)
// with one pass that reads the packed codes once and dequantizes in registers.
//
// Work decomposition: grid (split, kv_head, batch), 4 warps per CTA.  The token
// axis is cut into 32-token tiles aligned to the V packed grid; each CTA owns a
// contiguous range of tiles (a split) and each warp takes every 4th tile of that
// range with its own online-softmax state.  The CTA writes an unnormalised
// partial (O, m, l) per query head; lse_merge combines splits (and GPUs when
// context chunks are sharded).
//
// Staging: the 4 warps take 4 consecutive tiles at a time (a stage).  Stages
// whose K and V are all packed (the whole middle of the cache) are fetched by
// the TMA engine with a handful of cp.async.bulk copies into a CTA ring of
// stages_for(RP) slots, completion tracked by one mbarrier per slot (no
// multicast); the last warp to finish with a slot issues its refill.
// Boundary tiles (sink, recent, the K/V packed/dense seams) load directly
// from global memory.
//
// The query side (digits, B fragments, group sums) of each (batch, KV head)
// is built once by qprep_kernel; each CTA bulk-copies that block while its
// first KV stages are in flight (programmatic dependent launch).
//
// Arithmetic: packed codes are multiplied on the tensor cores with
// mma.sync m16n8k32 u8 x s8/u8 -> s32, so every partial dot product is exact:
//   QK^T: A = K codes [token][dim] (u8), B = q*f*2^e rounded to a 22-bit
//         integer (21 / 20 bits for groups of 64 / 128, so one group's sum
//         fits int32) and split into three balanced int8 digits.
//         logit = 2^-e * sum_g s_g * (sum_{d in g} u_d q_d - off * sum_{d in g} q_d)
//   PV:   A = V codes [dim][token] (u8), B = exp2(x - tile max) as a 16-bit
//         fixed-point value split into two u8 digits; scaled per tile by
//         exp2(tile max - running max) / 65535 and by the (group, dim) scale.
// B columns (d2, d1) and (d0, 0) per head; the offset-binary correction
// off * sum q enters as the accumulator input of the d0 column.  The logits
// carry ~2^-21 of max|q| rounding; the probabilities 2^-17 of each tile's
// largest weight.
// Dense (fp16 / bf16) rows use m16n8k16 with hi/lo-split B operands.
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
  int chan;   // values grouped over channels (scales per token and channel group)
  // graph mode (DevArgs::step set): n_q / n_rec are the counts at step 0, rec
  // the FIFO base, r0 the window's FIFO offset at step 0, flush the flush size,
  // max_steps the steps its buffers were reserved for
  int r0, flush, max_steps;
  // hybrid values (token groups): codes / scale are the symmetric set;
  // codes2 / scale2 / zero2 the asymmetric (bits - 1)-bit set (cap_tiles2),
  // mask 8 16-bit words per group, bit col_scale_idx(dim) set where the group
  // keeps its symmetric codes
  int hyb;
  const uint8_t* codes2;
  const uint16_t* scale2;
  const uint16_t* zero2;
  const uint16_t* mask;
  int64_t cap_tiles2;
  int otok;  // keys grouped over tokens (scales per (token group, dim))
};

// A side's geometry after n decode steps of graph mode: each step appends one
// token to the recent FIFO, then flushes `flush` tokens whenever it holds at
// least that many (at most one flush per step), so after n steps
// min(n, (n_rec0 + n) / flush) flushes have happened.
struct SideNow { int nq, nrec, r0; };
__device__ __forceinline__ SideNow side_after(const DevSide& s, int n) {
  SideNow o;
  const int k = s.flush > 0 ? min(n, (s.n_rec + n) / s.flush) : 0;
  o.nq = s.n_q + s.flush * k;
  o.nrec = s.n_rec + n - s.flush * k;
  o.r0 = s.r0 + s.flush * k;
  return o;
}

struct DevArgs {
  DevSide k, v;
  const uint16_t* q;
  int64_t q_b, q_h;
  const uint16_t* kf;  // key normalisation factor [B][Hkv][D] or null
  int B, Hq, Hkv, S, R;
  int t_first;         // token index of tile 0 (<= 0)
  int tile_lo, tile_hi;
  int tiles_per_split, n_splits;
  float scale_log2;    // softmax scale * log2(e)
  const void* qprep;   // [B][Hkv] QPrep<RP> blocks written by qprep_kernel
  float* po;           // [B][Hq][n_splits][D]
  float* pm;           // [B][Hq][n_splits]
  float* pl;
  const int64_t* step;  // graph mode: device count of decode steps taken (else null)
};

constexpr int kWarps = 4;
// staging ring depth (stages of kWarps tiles); 2 keeps 4 CTAs per SM
__host__ __device__ constexpr int stages_for(int rp) { return 2; }
// bounded mbarrier wait: each try suspends the warp for up to ~100 us (hint,
// in ns) instead of spinning; 1 << 16 tries bound the wait to seconds
constexpr uint32_t kWaitLimit = 1u << 16;

// bytes of one staged tile (K codes, K scales [, K zeros], V codes, V scales
// [, V zeros] [, hybrid: asymmetric V codes, their scales and zeros, the mask])
__host__ __device__ inline int stage_bytes(int bk, int bv, int ng, int kasym, int vasym, int hyb = 0) {
  return tile_bytes(bk) + 64 * ng * (1 + kasym) + tile_bytes(bv) + 256 * (1 + vasym) +
         (hyb ? tile_bytes(bv - 1) + 256 + 256 + 16 : 0);
}
__host__ __device__ inline int attn_dyn_smem(int bk, int bv, int ng, int kasym, int vasym, int rp, int hyb = 0) {
  return kWarps * stages_for(rp) * stage_bytes(bk, bv, ng, kasym, vasym, hyb);
}

// ------------------------------------------------------------ PTX helpers ---
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 100000;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t limit) {
  for (uint32_t it = 0; it < limit; ++it)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
// plain (non-multicast) bulk copy global -> this CTA's shared memory
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 2^x with the MUFU approximation (ex2.approx.ftz.f32: ~2 ulp; 2^-inf = 0)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

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

// words of one packed K token row (row layout): b=4: 4, b=2: 2, b=3: L0 L1 H
template <int BITS> struct KRow { uint32_t w[BITS == 4 ? 4 : 3]; };

template <int BITS>
__device__ __forceinline__ void load_krows(KRow<BITS> rw[4], const uint8_t* tb, int lane) {
  // the lane's four rows of one fully packed tile (shared or global memory);
  // piece k of the lane at k*512 + lane*16
  if constexpr (BITS == 4) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 v = *reinterpret_cast<const uint4*>(tb + j * 512 + lane * 16);
      rw[j].w[0] = v.x; rw[j].w[1] = v.y; rw[j].w[2] = v.z; rw[j].w[3] = v.w;
    }
  } else {
    const uint4 v0 = *reinterpret_cast<const uint4*>(tb + lane * 16);
    const uint4 v1 = *reinterpret_cast<const uint4*>(tb + 512 + lane * 16);
    rw[0].w[0] = v0.x; rw[0].w[1] = v0.y; rw[1].w[0] = v0.z; rw[1].w[1] = v0.w;
    rw[2].w[0] = v1.x; rw[2].w[1] = v1.y; rw[3].w[0] = v1.z; rw[3].w[1] = v1.w;
    if constexpr (BITS == 3) {
      const uint4 h = *reinterpret_cast<const uint4*>(tb + 1024 + lane * 16);
      rw[0].w[2] = h.x; rw[1].w[2] = h.y; rw[2].w[2] = h.z; rw[3].w[2] = h.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) rw[j].w[2] = 0;
    }
  }
}

template <int BITS>
__device__ __forceinline__ void load_krow(KRow<BITS>& r, const uint8_t* tb, int lane2, int j) {
  // one row of a tile, for tiles whose rows come from different places
  if constexpr (BITS == 4) {
    const uint4 v = *reinterpret_cast<const uint4*>(tb + j * 512 + lane2 * 16);
    r.w[0] = v.x; r.w[1] = v.y; r.w[2] = v.z; r.w[3] = v.w;
  } else {
    const uint2 v = *reinterpret_cast<const uint2*>(tb + (j >> 1) * 512 + lane2 * 16 + (j & 1) * 8);
    r.w[0] = v.x; r.w[1] = v.y;
    r.w[2] = BITS == 3 ? *reinterpret_cast<const uint32_t*>(tb + 1024 + lane2 * 16 + j * 4) : 0u;
  }
}

template <int BITS> struct VChunk { uint32_t w[BITS == 4 ? 16 : (BITS == 2 ? 8 : (BITS == 3 ? 12 : 4))]; };

template <int BITS>
__device__ __forceinline__ void load_vchunk(VChunk<BITS>& c, const uint8_t* tb, int lane) {
  if constexpr (BITS == 1) {
    const uint4 v = *reinterpret_cast<const uint4*>(tb + lane * 16);
    c.w[0] = v.x; c.w[1] = v.y; c.w[2] = v.z; c.w[3] = v.w;
  } else if constexpr (BITS == 4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 v = *reinterpret_cast<const uint4*>(tb + i * 512 + lane * 16);
      c.w[4 * i] = v.x; c.w[4 * i + 1] = v.y; c.w[4 * i + 2] = v.z; c.w[4 * i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint4 v = *reinterpret_cast<const uint4*>(tb + i * 512 + lane * 16);
      c.w[4 * i] = v.x; c.w[4 * i + 1] = v.y; c.w[4 * i + 2] = v.z; c.w[4 * i + 3] = v.w;
    }
    if constexpr (BITS == 3) {
      const uint4 v = *reinterpret_cast<const uint4*>(tb + 1024 + lane * 16);
      c.w[8] = v.x; c.w[9] = v.y; c.w[10] = v.z; c.w[11] = v.w;
    }
  }
}

// a pair of 16-bit dtype values packed in a word -> two floats
template <int DT> __device__ __forceinline__ float2 pair_to_f2(uint32_t w);
template <> __device__ __forceinline__ float2 pair_to_f2<F16>(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
template <> __device__ __forceinline__ float2 pair_to_f2<BF16>(uint32_t w) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}

// 16 16-bit values (32 B) as 8 float pairs
template <int DT>
__device__ __forceinline__ void load16(float2 out[8], const uint16_t* p) {
  const uint4 a = reinterpret_cast<const uint4*>(p)[0], b = reinterpret_cast<const uint4*>(p)[1];
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int u = 0; u < 8; ++u) out[u] = pair_to_f2<DT>(w[u]);
}

__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }

// dense (fp16 / bf16) row pointer for token t of a side, or null
// (nq: the side's packed count now; r0: FIFO offset of the recent window)
__device__ __forceinline__ const uint16_t* dense_row(const DevSide& s, int b, int h, int t, int S, int nq,
                                                     int r0) {
  if (t < 0 || t >= S) return nullptr;
  if (t < s.n_sink) return s.sink + b * s.sk_b + h * s.sk_h + (int64_t)t * s.sk_t;
  const int r = t - s.n_sink - nq;
  if (r >= 0) return s.rec + b * s.rc_b + h * s.rc_h + (int64_t)(r + r0) * s.rc_t;
  return nullptr;
}


// a tile whose 32 K rows and 32 V rows all sit in the packed stores, both
// tile-aligned: it is staged by the bulk-copy ring
__device__ __forceinline__ bool is_fast_tile(const DevArgs& a, int nqk, int nqv, int tile) {
  const int t0 = a.t_first + tile * kTile;
  const int ks = a.k.n_sink, vs = a.v.n_sink;
  return nqk > 0 && t0 >= ks && t0 + kTile <= ks + nqk && ((t0 - ks) & 31) == 0 && nqv > 0 &&
         t0 >= vs && t0 + kTile <= vs + nqv;
}

// Everything the attention pass needs from the query of one (batch, KV head),
// built once by qprep_kernel and bulk-copied into each CTA of that pair.
template <int RP>
struct QPrep {
  static constexpr int NT = RP / 4;
  // packed-K B fragments (three int8 digits of q*f*2^e_p): n-tile nt < NT holds
  // (d2, d1) of heads 4nt..4nt+3; n-tile NT holds d0 (GQA <= 4: (d0, 0) per
  // head; GQA 8: (d0 of head q, d0 of head q+4), so 8 heads need 3 n-tiles)
  static constexpr int kBTiles = NT + 1;
  uint2 bk[kBTiles][4][32];
  int qsum[RP][4];          // sum of the integer query over each K channel group
  int e_p, e_d, pad0, pad1; // exponents of the packed / dense query scalings
  uint2 bd[NT][8][32];      // dense-K B fragments (dtype hi/lo of q*2^e_d)
  // bytes every CTA copies; the dense fragments follow only where needed
  static constexpr uint32_t kHead = sizeof(uint2) * kBTiles * 4 * 32 + sizeof(int) * (RP * 4 + 4);
  static constexpr uint32_t kDense = sizeof(uint2) * NT * 8 * 32;
};
static_assert(QPrep<4>::kHead % 16 == 0 && QPrep<8>::kHead % 16 == 0, "bulk copy granularity");
static_assert(sizeof(QPrep<4>) == QPrep<4>::kHead + QPrep<4>::kDense, "QPrep layout");
static_assert(sizeof(QPrep<8>) == QPrep<8>::kHead + QPrep<8>::kDense, "QPrep layout");

template <int RP>
struct AttnStatic {
  static constexpr int NT = RP / 4;
  static constexpr int kStages = stages_for(RP);
  alignas(128) QPrep<RP> qp;  // this pair's query block (bulk-copied)
  uint64_t bars[kStages];     // "stage full" barriers of the CTA's staging ring
  uint64_t prep_bar;          // the query block has landed
  int cnt[kStages];           // warps done with each stage
  float p_s[kWarps][RP][kTile];
  uint8_t pd_s[kWarps][RP][2][kTile];
  float cm_s[kWarps][RP];
  float cl_s[kWarps][RP];
  int geo[9];                 // graph mode: this step's S, packed K / V counts, K / V FIFO
                              // offsets, the split's tile range, the packed tile run
};

// balanced base-256 digits of an integer |v| < 2^23: v = d2*65536 + d1*256 + d0
__device__ __forceinline__ void digits3(int v, int& d0, int& d1, int& d2) {
  d0 = ((v + 128) & 255) - 128;
  const int v1 = (v - d0) >> 8;
  d1 = ((v1 + 128) & 255) - 128;
  d2 = (v1 - d1) >> 8;
}

// Logits (before the softmax scale) of the lane's 4 token rows for its
// head(s) from packed K words: lp[nt][j] += sum_g s[j][g] * (sum_d u q - off*sum_d q)
// (+ z[j][g] * sum_d q for asymmetric keys).  All partial sums are exact int32.
// Rows j = 2m, 2m+1 travel as one float pair (.x, .y): lp[nt][m], sc[m][g].
template <int BK, int NT, int NG, bool KASYM>
__device__ __forceinline__ void k_packed_logits(const KRow<BK> rw[4], const float2 sc[2][NG],
                                                const float2 zc[2][NG], const uint2 (*bks)[4][32],
                                                const float ctf[NT][NG], const float qsf[NT][NG],
                                                int lane, float2 lp[NT][2]) {
  constexpr int KPG = 4 / NG;
  if constexpr (NT == 2) {
    // 8 heads: two (d2, d1) n-tiles and one shared d0 n-tile (head q / q+4)
    int accP[2][2][4], accD[2][4];  // [nt][mt][c], [mt][c]
#pragma unroll
    for (int kb = 0; kb < 4; ++kb) {
      const int g = kb / KPG;
      const bool first = kb % KPG == 0;
      const uint2 p0 = bks[0][kb][lane], p1 = bks[1][kb][lane], pd = bks[2][kb][lane];
      const uint32_t bp0[2] = {p0.x, p0.y}, bp1[2] = {p1.x, p1.y}, bd[2] = {pd.x, pd.y};
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const uint32_t af[4] = {row_frag<BK>(rw[2 * mt].w, kb, 0), row_frag<BK>(rw[2 * mt + 1].w, kb, 0),
                                row_frag<BK>(rw[2 * mt].w, kb, 1), row_frag<BK>(rw[2 * mt + 1].w, kb, 1)};
        if (first) {
          imma_u8s8(accP[0][mt], af, bp0, 0, 0, 0, 0);
          imma_u8s8(accP[1][mt], af, bp1, 0, 0, 0, 0);
          imma_u8s8(accD[mt], af, bd, 0, 0, 0, 0);
        } else {
          imma_u8s8(accP[0][mt], af, bp0, accP[0][mt][0], accP[0][mt][1], accP[0][mt][2], accP[0][mt][3]);
          imma_u8s8(accP[1][mt], af, bp1, accP[1][mt][0], accP[1][mt][1], accP[1][mt][2], accP[1][mt][3]);
          imma_u8s8(accD[mt], af, bd, accD[mt][0], accD[mt][1], accD[mt][2], accD[mt][3]);
        }
      }
      if (kb % KPG == KPG - 1) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) {
            float tf[2];
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
              const uint32_t t = (uint32_t)accP[nt][mt][2 * rr] * 65536u +
                                 (uint32_t)accP[nt][mt][2 * rr + 1] * 256u + (uint32_t)accD[mt][2 * rr + nt];
              tf[rr] = (float)(int)t;
            }
            const float2 tc = __fadd2_rn(make_float2(tf[0], tf[1]), f2(-ctf[nt][g]));
            lp[nt][mt] = __ffma2_rn(sc[mt][g], tc, lp[nt][mt]);
            if constexpr (KASYM) lp[nt][mt] = __ffma2_rn(zc[mt][g], f2(qsf[nt][g]), lp[nt][mt]);
          }
      }
    }
  } else {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    int acc[2][2][4];  // [mt][digit n-tile: (d2,d1) / (d0,-)][c]
#pragma unroll
    for (int kb = 0; kb < 4; ++kb) {
      const int g = kb / KPG;
      const bool first = kb % KPG == 0;
      const uint2 b0 = bks[nt][kb][lane], b1 = bks[NT][kb][lane];
      const uint32_t bf0[2] = {b0.x, b0.y}, bf1[2] = {b1.x, b1.y};
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const uint32_t af[4] = {row_frag<BK>(rw[2 * mt].w, kb, 0), row_frag<BK>(rw[2 * mt + 1].w, kb, 0),
                                row_frag<BK>(rw[2 * mt].w, kb, 1), row_frag<BK>(rw[2 * mt + 1].w, kb, 1)};
        if (first) {
          imma_u8s8(acc[mt][0], af, bf0, 0, 0, 0, 0);
          imma_u8s8(acc[mt][1], af, bf1, 0, 0, 0, 0);
        } else {
          imma_u8s8(acc[mt][0], af, bf0, acc[mt][0][0], acc[mt][0][1], acc[mt][0][2], acc[mt][0][3]);
          imma_u8s8(acc[mt][1], af, bf1, acc[mt][1][0], acc[mt][1][1], acc[mt][1][2], acc[mt][1][3]);
        }
      }
      if (kb % KPG == KPG - 1) {
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          float tf[2];
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            // sum_d u q (|.| < 2^31); intermediate terms wrap modulo 2^32
            const uint32_t t = (uint32_t)acc[mt][0][2 * rr] * 65536u +
                               (uint32_t)acc[mt][0][2 * rr + 1] * 256u + (uint32_t)acc[mt][1][2 * rr];
            tf[rr] = (float)(int)t;
          }
          // offset-binary correction off * sum_d q in fp32 (an MMA accumulator
          // input would cost register moves on every MMA)
          const float2 tc = __fadd2_rn(make_float2(tf[0], tf[1]), f2(-ctf[nt][g]));
          lp[nt][mt] = __ffma2_rn(sc[mt][g], tc, lp[nt][mt]);
          if constexpr (KASYM) lp[nt][mt] = __ffma2_rn(zc[mt][g], f2(qsf[nt][g]), lp[nt][mt]);
        }
      }
    }
  }
  }
}

// Logits (q . k) of the lane's 4 token rows for its head (lane tq) from a
// packed K tile whose scales / zero points run per (token group, dim), the
// KIVI layout (cache.py:87, quant.py:58-93): k = s_d u + z_d (asymmetric) or
// s_d (u - off) (symmetric), so q . k = sum_d (q_d s_d) u + sum_d q_d z_d.
// The scaled query q_d s_d changes with the tile's group, so its integer
// digits are built here, per tile: each lane makes the B-fragment bytes of
// head gid/2 for its 32 dims (kb*32 + 4tq + i, kb*32 + 16 + 4tq + i), scaled
// by 2^e so the group's largest |q_d s_d| fits QB bits; with codes below
// 2^BK the 128-dim integer sum stays exact in int32 (QB = 24 - BK).
// sp / zp: the group's 128 scales / zero points (natural dim order), qk: the
// pair's query in fp32, [4 heads][128].  Rows j = 2m, 2m+1 as one float pair.
template <int BK, int DT, bool KASYM>
__device__ __forceinline__ void k_tok_logits(const KRow<BK> rw[4], const uint16_t* sp, const uint16_t* zp,
                                             const float (*qk)[kD], int lane, float2 lp[2]) {
  constexpr int QB = 24 - BK;
  const int gid = lane >> 2, tq = lane & 3, hb = gid >> 1, plane = gid & 1;
  float qs[4][8];
  float mx = 0.f, zs = 0.f;
#pragma unroll
  for (int kb = 0; kb < 4; ++kb)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int d = kb * 32 + hf * 16 + 4 * tq;
      const float4 q4 = *reinterpret_cast<const float4*>(&qk[hb][d]);
      const uint2 s2 = *reinterpret_cast<const uint2*>(sp + d);
      const float2 sa = pair_to_f2<DT>(s2.x), sb = pair_to_f2<DT>(s2.y);
      const float qv[4] = {q4.x, q4.y, q4.z, q4.w}, sv[4] = {sa.x, sa.y, sb.x, sb.y};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        qs[kb][hf * 4 + i] = qv[i] * sv[i];
        mx = fmaxf(mx, fabsf(qs[kb][hf * 4 + i]));
      }
      if constexpr (KASYM) {
        const uint2 z2 = *reinterpret_cast<const uint2*>(zp + d);
        const float2 za = pair_to_f2<DT>(z2.x), zb = pair_to_f2<DT>(z2.y);
        zs = fmaf(qv[0], za.x, fmaf(qv[1], za.y, fmaf(qv[2], zb.x, fmaf(qv[3], zb.y, zs))));
      }
    }
  // the head's largest |q s| and sums over its 128 dims: the 4 lanes tq of a gid
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  int e = 0;
  if (mx > 0.f) {
    int ex;
    frexpf(mx, &ex);
    e = QB - ex;
  }
  const float mul = ldexpf(1.f, e);
  int qsum = 0;
  uint32_t bA[4][2], bB[4][2];  // n-tile 0: d2 / d1 of head hb; n-tile 1: d0 of head hb / 0
#pragma unroll
  for (int kb = 0; kb < 4; ++kb)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      int dA[4], dB[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int v = __float2int_rn(qs[kb][hf * 4 + i] * mul);
        qsum += v;
        int d0, d1, d2;
        digits3(v, d0, d1, d2);
        dA[i] = plane ? d1 : d2;
        dB[i] = plane ? 0 : d0;
      }
      bA[kb][hf] = __byte_perm(__byte_perm(dA[0], dA[1], 0x0040), __byte_perm(dA[2], dA[3], 0x0040), 0x5410);
      bB[kb][hf] = __byte_perm(__byte_perm(dB[0], dB[1], 0x0040), __byte_perm(dB[2], dB[3], 0x0040), 0x5410);
    }
  qsum += __shfl_xor_sync(0xffffffffu, qsum, 1);
  qsum += __shfl_xor_sync(0xffffffffu, qsum, 2);
  if constexpr (KASYM) {
    zs += __shfl_xor_sync(0xffffffffu, zs, 1);
    zs += __shfl_xor_sync(0xffffffffu, zs, 2);
  }
  int acc[2][2][4];  // [mt][n-tile][c]
#pragma unroll
  for (int kb = 0; kb < 4; ++kb)
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const uint32_t af[4] = {row_frag<BK>(rw[2 * mt].w, kb, 0), row_frag<BK>(rw[2 * mt + 1].w, kb, 0),
                              row_frag<BK>(rw[2 * mt].w, kb, 1), row_frag<BK>(rw[2 * mt + 1].w, kb, 1)};
      if (kb == 0) {
        imma_u8s8(acc[mt][0], af, bA[kb], 0, 0, 0, 0);
        imma_u8s8(acc[mt][1], af, bB[kb], 0, 0, 0, 0);
      } else {
        imma_u8s8(acc[mt][0], af, bA[kb], acc[mt][0][0], acc[mt][0][1], acc[mt][0][2], acc[mt][0][3]);
        imma_u8s8(acc[mt][1], af, bB[kb], acc[mt][1][0], acc[mt][1][1], acc[mt][1][2], acc[mt][1][3]);
      }
    }
  // this lane's accumulator columns belong to head tq, whose scaling, integer
  // sum and zero term the lanes gid = 2tq computed
  const int src = 8 * tq;
  const float inv = ldexpf(1.f, -__shfl_sync(0xffffffffu, e, src));
  // symmetric: sum_d qi (u - off), exact in int32 (|.| < 128 * 2^(BK-1) * 2^QB)
  const int corr = KASYM ? 0 : (1 << (BK - 1)) * __shfl_sync(0xffffffffu, qsum, src);
  const float zt = KASYM ? __shfl_sync(0xffffffffu, zs, src) : 0.f;
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    float tf[2];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const uint32_t t = (uint32_t)acc[mt][0][2 * rr] * 65536u + (uint32_t)acc[mt][0][2 * rr + 1] * 256u +
                         (uint32_t)acc[mt][1][2 * rr];
      tf[rr] = fmaf((float)((int)t - corr), inv, zt);
    }
    lp[mt] = make_float2(tf[0], tf[1]);
  }
}

// O[nt][mt][h] += fv * (s * (sum_t u p - off * sum_t p) [+ z * sum_t p]) for one
// packed V tile (integer MMA, probabilities as two u8 digits)
template <int BV, int NT, bool VASYM>
__device__ __forceinline__ void v_packed_accumulate(const VChunk<BV>& vc, const float2 sv[8],
                                                    const float2 zv[8], const uint32_t pb[NT][2],
                                                    const float offp[NT], const float fv[NT],
                                                    const float zf[NT], float2 o[NT][8]) {
  // m-tile mt's sums carry col_scale(mt) (a power of two): exact to undo here
  float2 svf[NT][8];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int u = 0; u < 8; ++u) svf[nt][u] = __fmul2_rn(sv[u], f2(fv[nt] * (1.f / col_scale<BV>(u))));
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    const uint32_t af[4] = {col_frag<BV>(vc.w, mt, 0, 0), col_frag<BV>(vc.w, mt, 1, 0),
                            col_frag<BV>(vc.w, mt, 0, 1), col_frag<BV>(vc.w, mt, 1, 1)};
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      int acc[4];
      imma_u8u8(acc, af, pb[nt], 0, 0, 0, 0);
      const float t0 = (float)(acc[0] * 256 + acc[1]), t1 = (float)(acc[2] * 256 + acc[3]);
      const float2 tc = __fadd2_rn(make_float2(t0, t1), f2(-offp[nt] * col_scale<BV>(mt)));  // off * sum_t p
      o[nt][mt] = __ffma2_rn(svf[nt][mt], tc, o[nt][mt]);
      if constexpr (VASYM) o[nt][mt] = __ffma2_rn(zv[mt], f2(zf[nt]), o[nt][mt]);
    }
  }
}

// A fragment of the asymmetric (BV - 1)-bit set of a hybrid V tile, scaled
// like the symmetric BV-bit fragment of the same m-tile (col_scale<BV>(mt)),
// so one fp32 scale per dim undoes either
template <int BV>
__device__ __forceinline__ uint32_t asym_frag(const uint32_t* w, int mt, int h, int half) {
  if constexpr (BV == 2) {  // 1-bit plane: bit (mt&1)*4 + h*2 + half of word mt>>1
    return ((w[mt >> 1] >> ((mt & 1) * 4 + h * 2 + half)) & 0x01010101u) << (2 * (mt >> 1));
  } else if constexpr (BV == 3) {  // 2-bit set, crumb position mt>>1, moved to bit 0
    return (w[(mt & 1) * 4 + h * 2 + half] >> (2 * (mt >> 1))) & 0x03030303u;
  } else {  // 3-bit set (factor 1) under a 4-bit layout (factor 16 for m-tiles 4-7)
    return col_frag<3>(w, mt, h, half) << (mt < 4 ? 0 : 4);
  }
}

// PV of one packed tile of hybrid values (quant.py:133-176): per dim the
// group's mask picks the symmetric codes (scale s, offset 2^(BV-1)) or the
// asymmetric ones (scale s2, zero z2):
//   O[nt][mt][h] += fv * (S * sum_t u p + Cz * sum_t p),
//   (S, Cz) = mask ? (s, -2^(BV-1) s) : (s2, z2)
template <int BV, int NT>
__device__ __forceinline__ void v_hybrid_accumulate(const VChunk<BV>& vc, const VChunk<BV - 1>& va,
                                                    const float2 sv[8], const float2 sa[8],
                                                    const float2 za[8], uint32_t mk,
                                                    const uint32_t pb[NT][2], const int psum[NT],
                                                    const float fv[NT], float2 o[NT][8]) {
  constexpr float kOff = (float)(1 << (BV - 1));
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    const bool s0 = (mk >> (2 * mt)) & 1u, s1 = (mk >> (2 * mt + 1)) & 1u;  // dims (mt, h 0 / 1)
    const float2 S = make_float2(s0 ? sv[mt].x : sa[mt].x, s1 ? sv[mt].y : sa[mt].y);
    const float2 Cz = make_float2(s0 ? -kOff * sv[mt].x : za[mt].x, s1 ? -kOff * sv[mt].y : za[mt].y);
    const uint32_t af[4] = {s0 ? col_frag<BV>(vc.w, mt, 0, 0) : asym_frag<BV>(va.w, mt, 0, 0),
                            s1 ? col_frag<BV>(vc.w, mt, 1, 0) : asym_frag<BV>(va.w, mt, 1, 0),
                            s0 ? col_frag<BV>(vc.w, mt, 0, 1) : asym_frag<BV>(va.w, mt, 0, 1),
                            s1 ? col_frag<BV>(vc.w, mt, 1, 1) : asym_frag<BV>(va.w, mt, 1, 1)};
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      int acc[4];
      imma_u8u8(acc, af, pb[nt], 0, 0, 0, 0);
      const float2 t = make_float2((float)(acc[0] * 256 + acc[1]), (float)(acc[2] * 256 + acc[3]));
      o[nt][mt] = __ffma2_rn(__fmul2_rn(S, f2(fv[nt] * (1.f / col_scale<BV>(mt)))), t, o[nt][mt]);
      o[nt][mt] = __ffma2_rn(Cz, f2((float)psum[nt] * fv[nt]), o[nt][mt]);
    }
  }
}

// scales / zero points of the lane's 4 rows (row layout, [g][j]), 8*NG bytes at
// p, as pairs of rows: out[m][g] = (row 2m, row 2m+1)
template <int DT, int NG>
__device__ __forceinline__ void load_kscales(float2 out[2][NG], const uint16_t* p) {
  uint32_t w[2 * NG];
  if constexpr (NG == 4) {
    const uint4 a = reinterpret_cast<const uint4*>(p)[0], b = reinterpret_cast<const uint4*>(p)[1];
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w; w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
  } else if constexpr (NG == 2) {
    const uint4 a = reinterpret_cast<const uint4*>(p)[0];
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
  } else {
    const uint2 a = reinterpret_cast<const uint2*>(p)[0];
    w[0] = a.x; w[1] = a.y;
  }
#pragma unroll
  for (int g = 0; g < NG; ++g)
#pragma unroll
    for (int m = 0; m < 2; ++m) out[m][g] = pair_to_f2<DT>(w[2 * g + m]);
}

// BK/BV: code bits; RP: query heads per KV head padded to 4 or 8; DT: dtype;
// NG: K channel groups per token (4, 2, 1 for groups of 32, 64, 128); VCH:
// values grouped over channels too (same group size as the keys) instead of
// over tokens; GM: graph mode (geometry from the device step counter; a
// separate instantiation, because carrying that path costs the argument-fed
// kernel ~10% through register allocation)
template <int BK, int BV, int RP, int DT, int NG, int VCH, int GM, int VHY = 0, int KOT = 0>
__global__ void __launch_bounds__(kWarps * 32, RP == 4 ? 4 : 4)
decode_attn_kernel(const DevArgs a) {
  static_assert(!KOT || (RP == 4 && NG == 4 && !VHY), "keys over tokens: GQA <= 4, non-hybrid");
  constexpr int NT = RP / 4;
  constexpr int kStages = stages_for(RP);
  extern __shared__ __align__(128) uint8_t dyn[];
  __shared__ AttnStatic<RP> sm;
  // channel-grouped values: probability digits per (channel group, head)
  __shared__ __align__(16) uint8_t pdc_s[VCH ? kWarps : 1][VCH ? NG : 1][RP][2][kTile];
  // keys grouped over tokens: the pair's query heads in fp32
  __shared__ __align__(16) float qk_s[KOT ? RP : 1][KOT ? kD : 4];
  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tq = lane & 3;
  const int R = a.R;
  // this step's geometry: from the arguments, or in graph mode from the
  // device step counter (the grid, i.e. the split count, stays fixed)
  int S = a.S, nqk = a.k.n_q, nqv = a.v.n_q, kr0 = 0, vr0 = 0;
  int tile_lo = a.tile_lo, tile_hi = a.tile_hi, tps = a.tiles_per_split;
  if constexpr (GM) {
    // a counter past the reservation reads the last reserved state, never
    // beyond the buffers
    const int n = (int)min(*a.step, (int64_t)min(a.k.max_steps, a.v.max_steps));
    const SideNow kn = side_after(a.k, n), vn = side_after(a.v, n);
    nqk = kn.nq; nqv = vn.nq; kr0 = kn.r0; vr0 = vn.r0;
    S = a.k.n_sink + kn.nq + kn.nrec;
    tile_lo = 0;
    tile_hi = (S - a.t_first + kTile - 1) / kTile;
    tps = (tile_hi + a.n_splits - 1) / a.n_splits;
  }
  const int tile_beg = tile_lo + split * tps;
  const int tile_end = min(tile_beg + tps, tile_hi);
  const int ks = a.k.n_sink;
  const int vs = a.v.n_sink;
  const int kasym = a.k.asym, vasym = a.v.asym;
  const int SB = stage_bytes(BK, BV, NG, kasym, vasym, VHY);
  const int koff = kasym ? 0 : (1 << (BK - 1));
  const int voff = vasym ? 0 : (1 << (BV - 1));


  const int64_t kbh = (int64_t)b * a.Hkv + hk;
  const uint8_t* kcodes = a.k.codes ? a.k.codes + kbh * a.k.cap_tiles * tile_bytes(BK) : nullptr;
  // K scales: per (token, channel group) [tiles][32][NG], or (keys grouped
  // over tokens) per (token group, dim) [groups][128]
  const int kgs = a.k.group == 32 ? 5 : (a.k.group == 64 ? 6 : 7);
  const int64_t ksc_pair = KOT ? ((a.k.cap_tiles * 32) >> kgs) * kD : a.k.cap_tiles * 32 * NG;
  const uint16_t* kscale = a.k.scale ? a.k.scale + kbh * ksc_pair : nullptr;
  const uint16_t* kzero = a.k.zero ? a.k.zero + kbh * ksc_pair : nullptr;
  const uint8_t* vcodes = a.v.codes ? a.v.codes + kbh * a.v.cap_tiles * tile_bytes(BV) : nullptr;
  // V token-group size is 32, 64 or 128: divide by shifting
  const int vgs = a.v.group == 32 ? 5 : (a.v.group == 64 ? 6 : 7);
  const int64_t vgroups_cap = a.v.codes ? (a.v.cap_tiles * 32) >> vgs : 0;
  // token groups: [groups][128] per pair; channel groups: [tiles][32][NG] like K
  const int64_t vsc_pair = VCH ? a.v.cap_tiles * 32 * NG : vgroups_cap * kD;
  const uint16_t* vscale = a.v.scale ? a.v.scale + kbh * vsc_pair : nullptr;
  const uint16_t* vzero = a.v.zero ? a.v.zero + kbh * vsc_pair : nullptr;
  // hybrid values: the asymmetric set and the per-(group, dim) mask
  constexpr int TBV2 = VHY ? tile_bytes(BV - 1) : 0;
  const int64_t vgroups_cap2 = VHY ? (a.v.cap_tiles2 * 32) >> vgs : 0;
  const uint8_t* vcodes2 = VHY ? a.v.codes2 + kbh * a.v.cap_tiles2 * TBV2 : nullptr;
  const uint16_t* vscale2 = VHY ? a.v.scale2 + kbh * vgroups_cap2 * kD : nullptr;
  const uint16_t* vzero2 = VHY ? a.v.zero2 + kbh * vgroups_cap2 * kD : nullptr;
  const uint16_t* vmask = VHY ? a.v.mask + kbh * vgroups_cap2 * 8 : nullptr;

  // One ring per CTA: stage i holds the kWarps consecutive tiles
  // tile_beg + kWarps*i + w (warp w takes tile w).  Layout of a stage:
  // [K codes x4 | K scales x4 | K zeros x4 | V codes x4 | V scales | V zeros]
  const int TBK = tile_bytes(BK), TBV = tile_bytes(BV);
  const int o_ks = kWarps * TBK;
  const int o_kz = o_ks + kWarps * 64 * NG;
  const int o_vc = o_kz + (kasym ? kWarps * 64 * NG : 0);
  const int o_vs = o_vc + kWarps * TBV;
  const int o_vz = o_vs + kWarps * 256;
  const int o_vc2 = o_vz + (vasym ? kWarps * 256 : 0);  // hybrid regions
  const int o_vs2 = o_vc2 + kWarps * TBV2;
  const int o_vz2 = o_vs2 + kWarps * 256;
  const int o_vm = o_vz2 + kWarps * 256;
  const int SBC = kWarps * SB;  // bytes of a stage (same total as kWarps per-tile slots)
  uint8_t* ring = dyn;

  // packed tiles form one contiguous run [fast_lo, fast_hi) of tile indices
  int fast_lo = 0, fast_hi = 0;
  if (nqk > 0 && nqv > 0 && ((vs - ks) & 31) == 0) {
    const int lo_tok = max(ks, vs), hi_tok = min(ks + nqk, vs + nqv);
    fast_lo = (lo_tok - a.t_first + 31) >> 5;
    fast_hi = (hi_tok - a.t_first) >> 5;  // floor: the tile must end inside
  }
  const int n_st = (tile_end - tile_beg + kWarps - 1) / kWarps;
  if constexpr (GM) {
    // graph mode: the tile loop reads this step's geometry from shared memory
    // (it cannot be re-derived from the launch arguments, and kept in
    // registers across the loop it spills); written before thread 0's first
    // copies and read by the others after the barrier below
    if (threadIdx.x == 0) {
      sm.geo[0] = S; sm.geo[1] = nqk; sm.geo[2] = nqv; sm.geo[3] = kr0; sm.geo[4] = vr0;
      sm.geo[5] = tile_beg; sm.geo[6] = tile_end; sm.geo[7] = fast_lo; sm.geo[8] = fast_hi;
    }
  }
  auto gTB = [&]() -> int { if constexpr (GM) return sm.geo[5]; else return tile_beg; };
  auto gTE = [&]() -> int { if constexpr (GM) return sm.geo[6]; else return tile_end; };
  auto stage_fast = [&](int i) -> bool {
    const int ta = gTB() + kWarps * i, tb = min(ta + kWarps, gTE()) - 1;
    if constexpr (GM) return ta >= sm.geo[7] && tb < sm.geo[8];
    else return ta >= fast_lo && tb < fast_hi;
  };
  // issued by one thread: the last warp to release the slot (or thread 0 at start)
  auto issue = [&](int i) {
    if (i >= n_st) return;
    const int slot = i % kStages;
    uint64_t* bar = &sm.bars[slot];
    if (!stage_fast(i)) {
      mbar_arrive(bar);
      return;
    }
    const int ta = gTB() + kWarps * i, n_in = min(kWarps, gTE() - ta);
    const int t0 = a.t_first + ta * kTile;
    const int64_t tk = (t0 - ks) >> 5, tv = (t0 - vs) >> 5;
    const int64_t g0 = (t0 - vs) >> vgs, g1 = (t0 + n_in * kTile - 1 - vs) >> vgs;
    const uint32_t nvg = (uint32_t)(g1 - g0 + 1);
    uint8_t* st = ring + slot * SBC;
    // keys grouped over tokens: the stage's token groups' scales (256 B each)
    const int64_t kg0 = (t0 - ks) >> kgs;
    const uint32_t nkg = KOT ? (uint32_t)(((t0 + n_in * kTile - 1 - ks) >> kgs) - kg0 + 1) : 0u;
    const uint32_t kb = KOT ? n_in * TBK + nkg * 256 * (1 + kasym) : n_in * (TBK + 64 * NG * (1 + kasym));
    const uint32_t vb = n_in * TBV + (VCH ? n_in * 64 * NG : nvg * 256) * (1 + vasym) +
                        (VHY ? n_in * TBV2 + nvg * (256 + 256 + 16) : 0);
    fence_proxy_async();
    mbar_arrive_tx(bar, kb + vb);
    bulk_g2s(st, kcodes + tk * TBK, n_in * TBK, bar);
    if (KOT) {
      bulk_g2s(st + o_ks, kscale + kg0 * kD, nkg * 256, bar);
      if (kasym) bulk_g2s(st + o_kz, kzero + kg0 * kD, nkg * 256, bar);
    } else {
      bulk_g2s(st + o_ks, kscale + tk * 32 * NG, n_in * 64 * NG, bar);
      if (kasym) bulk_g2s(st + o_kz, kzero + tk * 32 * NG, n_in * 64 * NG, bar);
    }
    bulk_g2s(st + o_vc, vcodes + tv * TBV, n_in * TBV, bar);
    if (VCH) {
      bulk_g2s(st + o_vs, vscale + tv * 32 * NG, n_in * 64 * NG, bar);
      if (vasym) bulk_g2s(st + o_vz, vzero + tv * 32 * NG, n_in * 64 * NG, bar);
    } else {
      bulk_g2s(st + o_vs, vscale + g0 * kD, nvg * 256, bar);
      if (vasym) bulk_g2s(st + o_vz, vzero + g0 * kD, nvg * 256, bar);
    }
    if constexpr (VHY) {
      bulk_g2s(st + o_vc2, vcodes2 + tv * TBV2, n_in * TBV2, bar);
      bulk_g2s(st + o_vs2, vscale2 + g0 * kD, nvg * 256, bar);
      bulk_g2s(st + o_vz2, vzero2 + g0 * kD, nvg * 256, bar);
      bulk_g2s(st + o_vm, vmask + g0 * 8, nvg * 16, bar);
    }
  };

  float m_run[NT], l_run[NT];
  float2 o[NT][8];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    m_run[nt] = -INFINITY;
    l_run[nt] = 0.f;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) o[nt][mt] = make_float2(0.f, 0.f);
  }

  // dense-K B fragments are needed only by CTAs that meet a sink / recent /
  // seam tile (packed tiles form one contiguous run)
  const bool any_dense =
      tile_end > tile_beg && !(is_fast_tile(a, nqk, nqv, tile_beg) && is_fast_tile(a, nqk, nqv, tile_end - 1));
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.bars[s], 1);
      sm.cnt[s] = 0;
    }
    mbar_init(&sm.prep_bar, 1);
    mbar_fence_init();
    // the KV tiles do not depend on the prep kernel: start them at once
#pragma unroll 1
    for (int s = 0; s < kStages; ++s) issue(s);
  }
  griddep_wait();  // the prep kernel's query blocks are complete and visible
  if (threadIdx.x == 0) {
    const uint8_t* src = reinterpret_cast<const uint8_t*>(a.qprep) + ((int64_t)b * a.Hkv + hk) * sizeof(QPrep<RP>);
    constexpr uint32_t kH = QPrep<RP>::kHead, kDn = QPrep<RP>::kDense;
    mbar_arrive_tx(&sm.prep_bar, kH + (any_dense ? kDn : 0u));
    bulk_g2s(&sm.qp, src, kH, &sm.prep_bar);
    if (any_dense) bulk_g2s(&sm.qp.bd, src + kH, kDn, &sm.prep_bar);
  }
  if constexpr (KOT) {
    for (int i = threadIdx.x; i < RP * kD; i += kWarps * 32) {
      const int h = i / kD, d = i % kD;
      qk_s[h][d] = h < R ? to_f<DT>(a.q[b * a.q_b + (int64_t)(hk * R + h) * a.q_h + d]) : 0.f;
    }
  }
  __syncthreads();  // barrier initialisation (and graph-mode geometry) visible to every thread
  bool failed = !mbar_wait_bounded(&sm.prep_bar, 0, kWaitLimit);
  int i_done = 0;
  float ctf[NT][NG];  // K offset correction per channel group: off * sum q
  float qsf[NT][NG];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      const int qs = sm.qp.qsum[nt * 4 + tq][g];
      ctf[nt][g] = (float)(koff * qs);
      qsf[nt][g] = (float)qs;
    }
  const float cp = ldexpf(a.scale_log2, -sm.qp.e_p);
  const float cd = ldexpf(a.scale_log2, -sm.qp.e_d);

  // ---------------------------------------------------------------- tiles
  // this step's geometry inside the loop: launch arguments, or (graph mode)
  // shared memory
  auto gS = [&]() -> int { if constexpr (GM) return sm.geo[0]; else return a.S; };
  auto gNQK = [&]() -> int { if constexpr (GM) return sm.geo[1]; else return a.k.n_q; };
  auto gNQV = [&]() -> int { if constexpr (GM) return sm.geo[2]; else return a.v.n_q; };
  auto gKR0 = [&]() -> int { if constexpr (GM) return sm.geo[3]; else return 0; };
  auto gVR0 = [&]() -> int { if constexpr (GM) return sm.geo[4]; else return 0; };
#pragma unroll 1
  for (int i = 0; i < (failed ? 0 : n_st); ++i) {
    const int slot = i % kStages;
    if (!mbar_wait_bounded(&sm.bars[slot], (uint32_t)((i / kStages) & 1), kWaitLimit)) {
      failed = true;
      break;
    }
    i_done = i + 1;
    const int tile = gTB() + kWarps * i + warp;
    const int t0 = a.t_first + tile * kTile;
    const bool fast = stage_fast(i);
    const uint8_t* sg = ring + slot * SBC;
    if (tile < gTE()) {
    float x[NT][4];

    // ----------------------------------------------------------- QK^T
    if (fast) {
      KRow<BK> rw[4];
      float2 sc[2][NG], zc[2][NG];
      load_krows<BK>(rw, sg + warp * TBK, lane);
      if constexpr (!KOT) {
        load_kscales<DT, NG>(sc, reinterpret_cast<const uint16_t*>(sg + o_ks + warp * 64 * NG) + gid * 4 * NG);
        if (kasym)
          load_kscales<DT, NG>(zc, reinterpret_cast<const uint16_t*>(sg + o_kz + warp * 64 * NG) + gid * 4 * NG);
      }
      float2 lp[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) lp[nt][0] = lp[nt][1] = make_float2(0.f, 0.f);
      if constexpr (KOT) {
        // the tile's token group among the groups staged with this stage
        const int kgo = ((t0 - ks) >> kgs) - ((a.t_first + (tile - warp) * kTile - ks) >> kgs);
        const uint16_t* sp = reinterpret_cast<const uint16_t*>(sg + o_ks) + kgo * kD;
        const uint16_t* zp = reinterpret_cast<const uint16_t*>(sg + o_kz) + kgo * kD;
        if (kasym) k_tok_logits<BK, DT, true>(rw, sp, zp, qk_s, lane, lp[0]);
        else k_tok_logits<BK, DT, false>(rw, sp, zp, qk_s, lane, lp[0]);
      } else {
        if (kasym) k_packed_logits<BK, NT, NG, true>(rw, sc, zc, sm.qp.bk, ctf, qsf, lane, lp);
        else k_packed_logits<BK, NT, NG, false>(rw, sc, zc, sm.qp.bk, ctf, qsf, lane, lp);
      }
      const float cpk = KOT ? a.scale_log2 : cp;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const bool head_ok = nt * 4 + tq < R;
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          const float2 xs = __fmul2_rn(lp[nt][m], f2(cpk));
          x[nt][2 * m] = head_ok ? xs.x : -INFINITY;
          x[nt][2 * m + 1] = head_ok ? xs.y : -INFINITY;
        }
      }
    } else {
      int src[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = t0 + gid + 8 * j;
        src[j] = (t < 0 || t >= gS()) ? 0 : ((t >= ks && t < ks + gNQK()) ? 1 : 2);
      }
      const int S = gS(), nqk = gNQK();
      const int lo_t = max(t0, 0), hi_t = min(t0 + kTile, S);
      const bool kp_any = nqk > 0 && lo_t < ks + nqk && hi_t > ks;
      const bool kd_any = (lo_t < min(ks, hi_t)) || (hi_t > max(ks + nqk, lo_t));
      float2 lp[NT][2];
      float ld[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        lp[nt][0] = lp[nt][1] = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 4; ++j) ld[nt][j] = 0.f;
      }
      if (KOT && kp_any) {
        if constexpr (KOT) {
          // keys grouped over tokens: the tile is wholly packed (its token
          // groups start at the sink, which the values share)
          KRow<BK> rw[4];
          const int64_t ti = (t0 - ks) >> 5;
          load_krows<BK>(rw, kcodes + ti * tile_bytes(BK), lane);
          const int64_t g = (t0 - ks) >> kgs;
          if (kasym) k_tok_logits<BK, DT, true>(rw, kscale + g * kD, kzero + g * kD, qk_s, lane, lp[0]);
          else k_tok_logits<BK, DT, false>(rw, kscale + g * kD, nullptr, qk_s, lane, lp[0]);
        }
      } else if (kp_any) {
        KRow<BK> rw[4];
        float sc[4][NG], zc[4][NG];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
          for (int g = 0; g < NG; ++g) sc[j][g] = zc[j][g] = 0.f;
#pragma unroll
          for (int u = 0; u < (BK == 4 ? 4 : 3); ++u) rw[j].w[u] = 0u;
          if (src[j] == 1) {
            const int p = t0 + gid + 8 * j - ks;
            const int ti = p >> 5, r = p & 31;
            load_krow<BK>(rw[j], kcodes + (int64_t)ti * tile_bytes(BK), (r & 7) * 4 + tq, r >> 3);
            const int64_t so = (int64_t)ti * 32 * NG;
#pragma unroll
            for (int g = 0; g < NG; ++g) {
              sc[j][g] = to_f<DT>(kscale[so + row_scale_idx(r, g, NG)]);
              zc[j][g] = kasym ? to_f<DT>(kzero[so + row_scale_idx(r, g, NG)]) : 0.f;
            }
          }
        }
        float2 sc2[2][NG], zc2[2][NG];
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
          for (int g = 0; g < NG; ++g) {
            sc2[m][g] = make_float2(sc[2 * m][g], sc[2 * m + 1][g]);
            zc2[m][g] = make_float2(zc[2 * m][g], zc[2 * m + 1][g]);
          }
        if (kasym) k_packed_logits<BK, NT, NG, true>(rw, sc2, zc2, sm.qp.bk, ctf, qsf, lane, lp);
        else k_packed_logits<BK, NT, NG, false>(rw, sc2, zc2, sm.qp.bk, ctf, qsf, lane, lp);
      }
      if (kd_any) {
        const uint16_t* rp[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) rp[j] = src[j] == 2 ? dense_row(a.k, b, hk, t0 + gid + 8 * j, S, nqk, gKR0()) : nullptr;
#pragma unroll
        for (int kb = 0; kb < 8; ++kb)
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) {
            const uint16_t* r0 = rp[2 * mt];
            const uint16_t* r1 = rp[2 * mt + 1];
            const int c0 = kb * 16 + 2 * tq;
            const uint32_t af[4] = {r0 ? *reinterpret_cast<const uint32_t*>(r0 + c0) : 0u,
                                    r1 ? *reinterpret_cast<const uint32_t*>(r1 + c0) : 0u,
                                    r0 ? *reinterpret_cast<const uint32_t*>(r0 + c0 + 8) : 0u,
                                    r1 ? *reinterpret_cast<const uint32_t*>(r1 + c0 + 8) : 0u};
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const uint2 bb = sm.qp.bd[nt][kb][lane];
              const uint32_t bf[2] = {bb.x, bb.y};
              float c[4] = {0.f, 0.f, 0.f, 0.f};
              mma_dt<DT>(c, af, bf);
              ld[nt][2 * mt] += c[0] + c[1];
              ld[nt][2 * mt + 1] += c[2] + c[3];
            }
          }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const bool head_ok = nt * 4 + tq < R;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          x[nt][j] = (!head_ok || src[j] == 0)
                         ? -INFINITY
                         : (src[j] == 1 ? (j & 1 ? lp[nt][j >> 1].y : lp[nt][j >> 1].x) * (KOT ? a.scale_log2 : cp)
                                        : ld[nt][j] * cd);
      }
    }

    // ------------------------------------------------------------ softmax
    const int nqv = gNQV();
    const bool vpacked = nqv > 0 && t0 >= vs && t0 + kTile <= vs + nqv;
    // channel-grouped values may end inside a tile: its packed rows take the
    // packed path and its dense rows the dense path
    const bool vseam = VCH && nqv > 0 && t0 >= vs && t0 < vs + nqv && t0 + kTile > vs + nqv;
    float fv[NT];
    int psum[NT];
    // channel-grouped values: per (head, group) tile factor, offset term, zero term
    float fvg[VCH ? NT : 1][VCH ? NG : 1], offg[VCH ? NT : 1][VCH ? NG : 1], zsg[VCH ? NT : 1][VCH ? NG : 1];
    float2 vsc[VCH ? 2 : 1][VCH ? NG : 1], vzc[VCH ? 2 : 1][VCH ? NG : 1];
    if (VCH && (vpacked || vseam)) {
      // the lane's 4 tokens' V scales (and zero points), rows 2m, 2m+1 paired
      const uint16_t* sp;
      const uint16_t* zp = nullptr;
      if (fast) {
        sp = reinterpret_cast<const uint16_t*>(sg + o_vs + warp * 64 * NG) + gid * 4 * NG;
        if (vasym) zp = reinterpret_cast<const uint16_t*>(sg + o_vz + warp * 64 * NG) + gid * 4 * NG;
      } else {
        const int64_t ti = (t0 - vs) >> 5;
        sp = vscale + ti * 32 * NG + gid * 4 * NG;
        if (vasym) zp = vzero + ti * 32 * NG + gid * 4 * NG;
      }
      if constexpr (VCH) {
        load_kscales<DT, NG>(vsc, sp);
        if (vasym) load_kscales<DT, NG>(vzc, zp);
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const float mx = gid_max(fmaxf(fmaxf(x[nt][0], x[nt][1]), fmaxf(x[nt][2], x[nt][3])));
      const float m_new = fmaxf(m_run[nt], mx);
      float pt[4] = {0.f, 0.f, 0.f, 0.f};
      float alpha = 1.f, wt = 0.f;
      if (mx != -INFINITY) {
        alpha = m_new == m_run[nt] ? 1.f : ex2(m_run[nt] - m_new);
        wt = ex2(mx - m_new);
#pragma unroll
        for (int j = 0; j < 4; ++j) pt[j] = ex2(x[nt][j] - mx);
      }
      m_run[nt] = m_new;
      l_run[nt] = l_run[nt] * alpha + wt * ((pt[0] + pt[1]) + (pt[2] + pt[3]));
      if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) o[nt][mt] = __fmul2_rn(o[nt][mt], f2(alpha));
      }
      const int head = nt * 4 + tq;
      if (VCH && (vpacked || vseam)) {
        if constexpr (VCH) {
        // p * s per channel group, 16-bit fixed point relative to the group's
        // largest product in this tile (65000: stays below 2^16 after rounding).
        // Rows past the packed end (a seam tile) are selected out: their
        // scale slots were never written.
        bool pin[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) pin[j] = vpacked || t0 + gid + 8 * j < vs + nqv;
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          const float2 p01 = __fmul2_rn(make_float2(pt[0], pt[1]), vsc[0][g]);
          const float2 p23 = __fmul2_rn(make_float2(pt[2], pt[3]), vsc[VCH ? 1 : 0][g]);
          const float pr[4] = {pin[0] ? p01.x : 0.f, pin[1] ? p01.y : 0.f, pin[2] ? p23.x : 0.f,
                               pin[3] ? p23.y : 0.f};
          const float mg = gid_max(fmaxf(fmaxf(pr[0], pr[1]), fmaxf(pr[2], pr[3])));
          const float inv = mg > 0.f ? __fdividef(65000.f, mg) : 0.f;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int v = __float_as_int(fmaf(pr[j], inv, 12582912.f)) - 0x4B400000;
            pdc_s[warp][g][head][0][gid + 8 * j] = (uint8_t)(v >> 8);
            pdc_s[warp][g][head][1][gid + 8 * j] = (uint8_t)(v & 255);
          }
          fvg[nt][g] = wt * mg * (1.f / 65000.f);
          if (vasym) {
            const float2 z01 = __fmul2_rn(make_float2(pt[0], pt[1]), vzc[0][g]);
            const float2 z23 = __fmul2_rn(make_float2(pt[2], pt[3]), vzc[VCH ? 1 : 0][g]);
            const float zr = (pin[0] ? z01.x : 0.f) + (pin[1] ? z01.y : 0.f) + (pin[2] ? z23.x : 0.f) +
                             (pin[3] ? z23.y : 0.f);
            zsg[nt][g] = wt * gid_sum(zr);
          } else {
            zsg[nt][g] = 0.f;
          }
        }
        }
      } else if (vpacked) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          // round to nearest on the FMA pipe: adding 1.5*2^23 leaves the integer
          // in the low mantissa bits (pt*65535 < 2^22)
          const int v = __float_as_int(fmaf(pt[j], 65535.f, 12582912.f)) - 0x4B400000;
          sm.pd_s[warp][head][0][gid + 8 * j] = (uint8_t)(v >> 8);
          sm.pd_s[warp][head][1][gid + 8 * j] = (uint8_t)(v & 255);
        }
        fv[nt] = wt * (1.f / 65535.f);
      }
      if (!vpacked) {
#pragma unroll
        for (int j = 0; j < 4; ++j) sm.p_s[warp][head][gid + 8 * j] = pt[j] * wt;
      }
    }
    __syncwarp();

    // ------------------------------------------------------------------ PV
    if (VCH && (vpacked || vseam)) {
      if constexpr (VCH) {
      VChunk<BV> vc;
      if (fast) load_vchunk<BV>(vc, sg + o_vc + warp * TBV, lane);
      else load_vchunk<BV>(vc, vcodes + (int64_t)((t0 - vs) >> 5) * tile_bytes(BV), lane);
      constexpr int MPG = 8 / NG;  // 16-dim m-tiles per channel group
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int g = mt / MPG;
        const uint32_t af[4] = {col_frag<BV>(vc.w, mt, 0, 0), col_frag<BV>(vc.w, mt, 1, 0),
                                col_frag<BV>(vc.w, mt, 0, 1), col_frag<BV>(vc.w, mt, 1, 1)};
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int head = nt * 4 + (gid >> 1), digit = gid & 1;
          const uint32_t pb[2] = {*reinterpret_cast<const uint32_t*>(&pdc_s[warp][g][head][digit][4 * tq]),
                                  *reinterpret_cast<const uint32_t*>(&pdc_s[warp][g][head][digit][16 + 4 * tq])};
          if (mt % MPG == 0) {
            // the group's digit sums of head tq (+4nt), hi and lo: an
            // all-ones A operand sums each B column over the 32 tokens
            const uint32_t ones[4] = {0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u};
            int sacc[4];
            imma_u8u8(sacc, ones, pb, 0, 0, 0, 0);
            offg[nt][g] = (float)(voff * (sacc[0] * 256 + sacc[1]));
          }
          int acc[4];
          imma_u8u8(acc, af, pb, 0, 0, 0, 0);
          const float t0f = (float)(acc[0] * 256 + acc[1]), t1f = (float)(acc[2] * 256 + acc[3]);
          const float2 tc = __fadd2_rn(make_float2(t0f, t1f), f2(-offg[nt][g] * col_scale<BV>(mt)));
          o[nt][mt] = __ffma2_rn(f2(fvg[nt][g] * (1.f / col_scale<BV>(mt))), tc, o[nt][mt]);
          if (vasym) o[nt][mt] = __fadd2_rn(o[nt][mt], f2(zsg[nt][g]));
        }
      }
      }
    } else if (vpacked) {
      uint32_t pb[NT][2];
      float offp[NT];
      float zf[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int head = nt * 4 + (gid >> 1), digit = gid & 1;
        pb[nt][0] = *reinterpret_cast<const uint32_t*>(&sm.pd_s[warp][head][digit][4 * tq]);
        pb[nt][1] = *reinterpret_cast<const uint32_t*>(&sm.pd_s[warp][head][digit][16 + 4 * tq]);
        // the tile's probability sum of head tq (+4nt): an all-ones A operand
        // sums each digit column (hi, lo) over the 32 tokens
        {
          const uint32_t ones[4] = {0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u};
          int acc[4];
          imma_u8u8(acc, ones, pb[nt], 0, 0, 0, 0);
          psum[nt] = acc[0] * 256 + acc[1];
        }
        offp[nt] = (float)(voff * psum[nt]);
        zf[nt] = (float)psum[nt] * fv[nt];
      }
      VChunk<BV> vc;
      float2 sv[8], zv[8];
      if constexpr (VHY) {
        VChunk<BV - 1> va;
        uint32_t mk;
        if (fast) {
          const int gi = ((t0 - vs) >> vgs) - ((a.t_first + (tile - warp) * kTile - vs) >> vgs);
          load_vchunk<BV>(vc, sg + o_vc + warp * TBV, lane);
          load_vchunk<BV - 1>(va, sg + o_vc2 + warp * TBV2, lane);
          load16<DT>(sv, reinterpret_cast<const uint16_t*>(sg + o_vs + gi * 256) + gid * 16);
          load16<DT>(zv, reinterpret_cast<const uint16_t*>(sg + o_vs2 + gi * 256) + gid * 16);
          float2 z2[8];
          load16<DT>(z2, reinterpret_cast<const uint16_t*>(sg + o_vz2 + gi * 256) + gid * 16);
          mk = reinterpret_cast<const uint16_t*>(sg + o_vm + gi * 16)[gid];
          v_hybrid_accumulate<BV, NT>(vc, va, sv, zv, z2, mk, pb, psum, fv, o);
        } else {
          const int pv = t0 - vs;
          load_vchunk<BV>(vc, vcodes + (int64_t)(pv >> 5) * tile_bytes(BV), lane);
          load_vchunk<BV - 1>(va, vcodes2 + (int64_t)(pv >> 5) * TBV2, lane);
          const int64_t gg = pv >> vgs;
          load16<DT>(sv, vscale + gg * kD + gid * 16);
          load16<DT>(zv, vscale2 + gg * kD + gid * 16);
          float2 z2[8];
          load16<DT>(z2, vzero2 + gg * kD + gid * 16);
          mk = vmask[gg * 8 + gid];
          v_hybrid_accumulate<BV, NT>(vc, va, sv, zv, z2, mk, pb, psum, fv, o);
        }
      } else {
      if (fast) {
        const int gofs = (((t0 - vs) >> vgs) - ((a.t_first + (tile - warp) * kTile - vs) >> vgs)) * 256;
        load_vchunk<BV>(vc, sg + o_vc + warp * TBV, lane);
        load16<DT>(sv, reinterpret_cast<const uint16_t*>(sg + o_vs + gofs) + gid * 16);
        if (vasym) load16<DT>(zv, reinterpret_cast<const uint16_t*>(sg + o_vz + gofs) + gid * 16);
      } else {
        const int pv = t0 - vs;
        load_vchunk<BV>(vc, vcodes + (int64_t)(pv >> 5) * tile_bytes(BV), lane);
        const int64_t gg = pv >> vgs;
        load16<DT>(sv, vscale + gg * kD + gid * 16);
        if (vasym) load16<DT>(zv, vzero + gg * kD + gid * 16);
      }
      if (vasym) v_packed_accumulate<BV, NT, true>(vc, sv, zv, pb, offp, fv, zf, o);
      else v_packed_accumulate<BV, NT, false>(vc, sv, zv, pb, offp, fv, zf, o);
      }
    }
    if (!vpacked) {
      // dense V rows (sink / recent / masked rows), probabilities as dtype hi/lo
      uint32_t pb[NT][2][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int head = nt * 4 + (gid >> 1), part = gid & 1;
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          const int rr[4] = {kb * 16 + 2 * tq, kb * 16 + 2 * tq + 1, kb * 16 + 2 * tq + 8, kb * 16 + 2 * tq + 9};
          uint16_t v[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint16_t hi, lo;
            split_hilo<DT>(sm.p_s[warp][head][rr[u]], hi, lo);
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
          const int t = t0 + rr[u];
          const int S = gS();
          const bool dense = t >= 0 && t < S && !(t >= vs && t < vs + nqv);
          vp[kb][u] = dense ? dense_row(a.v, b, hk, t, S, nqv, gVR0()) : nullptr;
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
          const uint32_t af[4] = {pack2(e[0][0], e[1][0]), pack2(e[0][1], e[1][1]),
                                  pack2(e[2][0], e[3][0]), pack2(e[2][1], e[3][1])};
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) mma_dt<DT>(acc[nt], af, pb[nt][kb]);
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          o[nt][mt].x += acc[nt][0] + acc[nt][1];
          o[nt][mt].y += acc[nt][2] + acc[nt][3];
        }
      }
    }
    }  // tile < tile_end
    __syncwarp();
    if (lane == 0) {
      // the last warp to finish with this slot refills it
      if (atomicAdd(&sm.cnt[slot], 1) == kWarps - 1) {
        sm.cnt[slot] = 0;
        issue(i + kStages);
      }
    }
  }

  // the tiles are done: the merge grid (launched as this grid's programmatic
  // dependent) may be scheduled as CTAs finish; it waits for this grid's
  // completion before reading the partials
  griddep_launch_dependents();

  if (failed) {
    // a staged tile never arrived: wait (bounded) for this warp's copies still
    // in flight, then publish NaN so the caller sees the failure
#pragma unroll 1
    for (int i = i_done; i < min(n_st, i_done + kStages); ++i)
      mbar_wait_bounded(&sm.bars[i % kStages], (uint32_t)((i / kStages) & 1), kWaitLimit / 16);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) { m_run[nt] = NAN; l_run[nt] = NAN; }
  }

  // ------------------------------------------------------- combine warps
  __syncthreads();  // the ring is idle; reuse it for the per-warp outputs
  float* co_s = reinterpret_cast<float*>(dyn);  // [kWarps][RP][128]
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const float l = gid_sum(l_run[nt]);
    const int head = nt * 4 + tq;
    if (gid == 0) { sm.cm_s[warp][head] = m_run[nt]; sm.cl_s[warp][head] = l; }
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      co_s[(warp * RP + head) * kD + mt * 16 + gid] = o[nt][mt].x;
      co_s[(warp * RP + head) * kD + mt * 16 + 8 + gid] = o[nt][mt].y;
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
        const float wt = ex2(mw - M);  // 0 for an empty warp (mw = -inf)
        ov += wt * co_s[(w * RP + head) * kD + d];
        lv += wt * sm.cl_s[w][head];
      }
    }
    const int64_t row = ((int64_t)b * a.Hq + hk * R + head) * a.n_splits + split;
    a.po[row * kD + d] = ov;
    if (d == 0) { a.pm[row] = M; a.pl[row] = lv; }
  }
}

// The query side of the attention pass for one (batch, KV head): grid (Hkv, B),
// 128 threads.  q*f (f = the key normalisation factor, 1 without) is scaled by
// 2^e_p so its largest entry just fits QBITS bits, rounded to an integer and
// split into three balanced int8 digits laid out as the m16n8k32 B fragments
// the packed-K MMA reads; q alone, scaled by 2^e_d, gives the dtype hi/lo B
// fragments of the dense (sink / recent) rows.
template <int DT, int RP, int NG>
__global__ void __launch_bounds__(kWarps * 32) qprep_kernel(const DevArgs a) {
  // the previous kernel on the stream (an append of this layer's token, a
  // merge) has completed and its memory is visible once this returns; only
  // then may the attention grid start its KV copies
  griddep_wait();
  griddep_launch_dependents();
  constexpr int NT = RP / 4;
  constexpr int KPG = 4 / NG;                                // 32-dim k-blocks per channel group
  constexpr int QBITS = NG == 4 ? 22 : (NG == 2 ? 21 : 20);  // |q int| < 2^QBITS: a group sum fits int32
  __shared__ float q_s[RP * kD];   // q*f
  __shared__ float qd_s[RP * kD];  // q, then q*2^e_d
  __shared__ int qi_s[RP * kD];    // integer q*f*2^e_p
  __shared__ __align__(16) int8_t dg_s[3][RP * kD];  // balanced digits d0, d1, d2
  __shared__ float red_s[2][kWarps];
  const int hk = blockIdx.x, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int R = a.R;
  QPrep<RP>& out = reinterpret_cast<QPrep<RP>*>(const_cast<void*>(a.qprep))[(int64_t)b * a.Hkv + hk];
  float amax_p = 0.f, amax_d = 0.f;
  for (int i = threadIdx.x; i < RP * kD; i += kWarps * 32) {
    const int h = i / kD, d = i % kD;
    float qv = 0.f, f = 1.f;
    if (h < R) {
      qv = to_f<DT>(a.q[b * a.q_b + (int64_t)(hk * R + h) * a.q_h + d]);
      if (a.kf) f = to_f<DT>(a.kf[((int64_t)b * a.Hkv + hk) * kD + d]);
    }
    const float qp = qv * f;
    q_s[i] = qp;
    qd_s[i] = qv;
    amax_p = fmaxf(amax_p, fabsf(qp));
    amax_d = fmaxf(amax_d, fabsf(qv));
  }
  amax_p = warp_max(amax_p);
  amax_d = warp_max(amax_d);
  if (lane == 0) { red_s[0][warp] = amax_p; red_s[1][warp] = amax_d; }
  __syncthreads();
  amax_p = fmaxf(fmaxf(red_s[0][0], red_s[0][1]), fmaxf(red_s[0][2], red_s[0][3]));
  amax_d = fmaxf(fmaxf(red_s[1][0], red_s[1][1]), fmaxf(red_s[1][2], red_s[1][3]));
  int ex, e_p = 0, e_d = 0;
  if (amax_p > 0.f) { frexpf(amax_p, &ex); e_p = QBITS - ex; }
  if (amax_d > 0.f) { frexpf(amax_d, &ex); e_d = 15 - ex; }
  for (int i = threadIdx.x; i < RP * kD; i += kWarps * 32) {
    const int qi = __float2int_rn(ldexpf(q_s[i], e_p));
    qi_s[i] = qi;
    qd_s[i] = ldexpf(qd_s[i], e_d);
    int d0, d1, d2;
    digits3(qi, d0, d1, d2);
    dg_s[0][i] = (int8_t)d0;
    dg_s[1][i] = (int8_t)d1;
    dg_s[2][i] = (int8_t)d2;
  }
  if (threadIdx.x == 0) { out.e_p = e_p; out.e_d = e_d; out.pad0 = out.pad1 = 0; }
  __syncthreads();
  // per (head, channel group) sums of the integer query: one warp per head
  for (int h = warp; h < RP; h += kWarps) {
    int s[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) s[c] = qi_s[h * kD + c * 32 + lane];
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s[c] += __shfl_xor_sync(0xffffffffu, s[c], o);
    if (lane < 4) {
      int t = 0;
#pragma unroll
      for (int c = 0; c < 4; ++c) t += (c / KPG == lane) ? s[c] : 0;
      out.qsum[h][lane] = t;
    }
  }
  // packed-K B fragments (m16n8k32), column n = g2 of an n-tile: n-tile
  // ntk < NT holds (d2, d1) of head 4*ntk + n/2; n-tile NT holds d0 of head
  // n/2 (n even; n odd empty) for up to 4 heads, or of head n/2 + 4*(n&1) for
  // 8.  Each fragment word is one 32-bit read of 4 consecutive digit bytes.
  for (int i = threadIdx.x; i < QPrep<RP>::kBTiles * 4 * 32; i += kWarps * 32) {
    const int ntk = i / 128, kb = (i / 32) % 4, ln = i % 32;
    const int g2 = ln >> 2, t2 = ln & 3;
    const int which = g2 & 1;
    int head, plane;
    if (ntk < NT) {
      head = ntk * 4 + (g2 >> 1);
      plane = which ? 1 : 2;
    } else if (NT == 1) {
      head = g2 >> 1;
      plane = which ? -1 : 0;
    } else {
      head = (g2 >> 1) + 4 * which;
      plane = 0;
    }
    uint32_t wrd[2] = {0u, 0u};
    if (plane >= 0) {
      const int8_t* src = &dg_s[plane][head * kD + kb * 32 + 4 * t2];
      wrd[0] = *reinterpret_cast<const uint32_t*>(src);
      wrd[1] = *reinterpret_cast<const uint32_t*>(src + 16);
    }
    out.bk[ntk][kb][ln] = make_uint2(wrd[0], wrd[1]);
  }
  // dense-K B fragments (m16n8k16, dtype hi/lo of q * 2^e_d)
  for (int i = threadIdx.x; i < NT * 8 * 32; i += kWarps * 32) {
    const int nt = i / 256, kb = (i / 32) % 8, ln = i % 32;
    const int g2 = ln >> 2, t2 = ln & 3;
    const int head = nt * 4 + (g2 >> 1), part = g2 & 1;
    const int dd[4] = {kb * 16 + 2 * t2, kb * 16 + 2 * t2 + 1, kb * 16 + 2 * t2 + 8, kb * 16 + 2 * t2 + 9};
    uint16_t v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      uint16_t hi, lo;
      split_hilo<DT>(qd_s[head * kD + dd[u]], hi, lo);
      v[u] = part ? lo : hi;
    }
    out.bd[nt][kb][ln] = make_uint2(pack2(v[0], v[1]), pack2(v[2], v[3]));
  }
}

// Launch of the attention grid as a programmatic dependent of the prep grid
// launched just before it on the same stream.
template <typename K>
inline cudaError_t launch_after_prep(K kern, dim3 grid, int smem, cudaStream_t s, const DevArgs& a) {
  return launch_pdl(kern, grid, dim3(kWarps * 32, 1, 1), smem, s, a);
}

}  // namespace innerq
