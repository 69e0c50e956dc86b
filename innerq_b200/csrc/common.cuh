// Shared device helpers for the InnerQ B200 kernels: dtype rounding, the packed
// tile layouts, code extraction into integer-MMA fragments, mma.sync wrappers.
//
// Packed layouts (D = 128, tiles of 32 tokens, b = bits per code).  A lane's
// words are grouped in 16-byte pieces stored piece-major: piece k of lane L
// sits at byte k*512 + L*16 of its plane, so each 128-bit load of one piece
// by a whole warp reads 512 contiguous bytes (no shared-memory bank
// conflicts after the tile is bulk-copied).  Below, "word w of lane L" is
// word w%4 of piece w/4.  Both
// layouts hand each lane of the consuming warp exactly the bytes of its
// m16n8k32 integer-MMA A fragments (a0: row gid, k 4tq..4tq+3; a1: row gid+8;
// a2: row gid, k 16+4tq..; a3: row gid+8, k 16+4tq..), so a 4-bit word
// expands to two fragment registers with at most one shift and two LOP3s.
//
// "row" layout (K, channel groups; A = K[token][dim]):
//   Lane L = 4*gid + tq owns tokens r = gid + 8*j (j = 0..3) at dims
//   d = kb*32 + half*16 + 4*tq + i (kb = 0..3, half = 0..1, i = 0..3).
//     b=4: lane chunk 64 B = 4 rows x 4 words; word kb, nibble 2i + half
//     b=2: lane chunk 32 B = 4 rows x 2 words; word kb>>1,
//          crumb 4i + (kb&1)*2 + half
//     b=3: low 2 bits as b=2 in plane L (1024 B / tile); bit 2 in plane H
//          (512 B / tile, 1 word per row): bit 8i + kb*2 + half
//   Scales / zero points (ng = D/G per token) per tile: [gid 8][g ng][j 4], so
//   rows j = 2m, 2m+1 (the two rows of one MMA m-tile) share a 32-bit word.
//
// "col" layout (V, token groups; A = V^T[dim][token]):
//   Lane L = 4*gid + tq owns dims d = mt*16 + h*8 + gid (mt = 0..7, h = 0..1)
//   at tokens r = half*16 + 4*tq + i.
//     b=4: 16 words; word (mt&3)*4 + h*2 + half, bits 8i + 4*(mt>>2): m-tiles
//          0-3 sit in the low nibbles and 4-7 in the high nibbles of the same
//          bytes, so each fragment register is one AND (the high-nibble ones
//          hold 16*u, undone in the fp32 scale)
//     b=2:  8 words; word (mt&1)*4 + h*2 + half, bits 8i + 2*(mt>>1): crumb
//          position p = mt>>1 gives 4^p * u
//     b=3: plane L 8 words: word mt, crumb 4i + h*2 + half; plane H 4 words:
//          word mt>>1, bit 8i + (mt&1)*4 + h*2 + half
//   Scales / zero points (one per (group, dim)): [gid 8][mt 8][h 2].
//
// b=1 (the asymmetric half of hybrid mode) is a single plane laid out like
// plane H of b=3.
//
// Symmetric codes are stored offset-binary: u = sign*code + 2^(b-1) (1..2^b-1);
// asymmetric codes are stored as is (0..2^b-1).
#pragma once
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace innerq {

constexpr int kD = 128;        // head_dim supported by the packed kernels
constexpr int kTile = 32;      // tokens per tile

enum DType { F16 = 0, BF16 = 1 };

__host__ __device__ constexpr int tile_bytes(int bits) { return 512 * bits; }

// ---------------------------------------------------------------- dtype ---
template <int DT> __device__ __forceinline__ float to_f(uint16_t v);
template <> __device__ __forceinline__ float to_f<F16>(uint16_t v) {
  return __half2float(__ushort_as_half(v));
}
template <> __device__ __forceinline__ float to_f<BF16>(uint16_t v) {
  return __bfloat162float(__ushort_as_bfloat16(v));
}
template <int DT> __device__ __forceinline__ uint16_t from_f(float v);
template <> __device__ __forceinline__ uint16_t from_f<F16>(float v) {
  return __half_as_ushort(__float2half_rn(v));
}
template <> __device__ __forceinline__ uint16_t from_f<BF16>(float v) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}
// one torch op in the input dtype: fp32 result rounded to the dtype (RNE)
template <int DT> __device__ __forceinline__ float rnd(float v) { return to_f<DT>(from_f<DT>(v)); }

// hi/lo split of an fp32 value into two 16-bit values of dtype DT
template <int DT> __device__ __forceinline__ void split_hilo(float v, uint16_t& hi, uint16_t& lo) {
  hi = from_f<DT>(v);
  lo = from_f<DT>(v - to_f<DT>(hi));
}

__device__ __forceinline__ uint32_t pack2(uint16_t lo, uint16_t hi) {
  return (uint32_t)lo | ((uint32_t)hi << 16);
}

// Correctly rounded a / b given rb = RN(1/b): Markstein's division
// (P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Develop. 34(1), 1990).  q = RN(a*rb) is
// within one ulp of a/b, the remainder r = a - q*b is exact in one FMA, and
// RN(q + r*rb) = RN(a/b) provided no intermediate overflows or underflows.
// Called only with fp16 operands (exact in fp32, |a| <= 65504 and
// 2^-24 <= b <= 65504), where that holds; a GPU test compares it bit for bit
// with the IEEE '/' over every pair of fp16 values.
__device__ __forceinline__ float div_rn(float a, float b, float rb) {
  const float q = __fmul_rn(a, rb);
  const float r = __fmaf_rn(-q, b, a);
  // an exact quotient keeps q (and with it the sign of a zero a)
  return r == 0.f ? q : __fmaf_rn(r, rb, q);
}

// rint(clamp(q, 0, qmax)) with a NaN quotient (0 / 0 scale) giving code 0:
// fmaxf returns its non-NaN operand; adding 1.5 * 2^23 rounds to the nearest
// integer, ties to even, like rintf (q <= 15 here)
__device__ __forceinline__ int code_of(float q, float qmax) {
  return __float_as_int(fminf(fmaxf(q, 0.f), qmax) + 12582912.f) - 0x4B400000;
}

// ------------------------------------------------- codes by thresholds ---
// The reference's code of a >= 0 in a group of scale s > 0 is
//   c(a) = rint(clamp(rnd_dt(RN32(a / s)), 0, qmax))          (quant.py:71-72, 107-109)
// (RN32: the fp32 quotient of a torch half op, rnd_dt: rounding to fp16 /
// bf16, rint ties to even).  c is non-decreasing in a, so c(a) >= k exactly
// when a passes a cut that depends only on k, the dtype and s:
//   * rint(v) >= k for a dtype value v  <=>  v >= H_k, with H_k = k - 1/2 for
//     even k (the tie rounds up to k) and the next dtype value after k - 1/2
//     for odd k;
//   * rnd_dt(y) >= H_k for an fp32 value y  <=>  y >= Y_k, with Y_k the
//     midpoint between H_k and the dtype value below it, moved up one fp32 ulp
//     when H_k's significand is odd (a tie then rounds down);
//   * RN32(a / s) >= Y_k  <=>  a / s > M_k, or a / s == M_k when Y_k's fp32
//     significand is even (the tie rounds up), M_k the midpoint between Y_k
//     and the fp32 value below it.
// M_k * s has at most 25 + 11 significant bits, exact in fp64, and a is an
// fp32 value, so the cut in a is the fp32 value just at or above M_k * s.
// Per group: one fp64 product and rounding per k; per element: a comparison
// tree over the qmax cuts.  Tested against the fp32 division for every pair
// of non-negative fp16 / bf16 values (tests/cuda/code_check.cu).
__host__ __device__ constexpr double pow2_floor(double v) {
  double p = 1.0;
  while (p * 2.0 <= v) p *= 2.0;
  while (p > v) p *= 0.5;
  return p;
}
// spacing of a binary float with `mb` fraction bits at v > 0 (normal range)
__host__ __device__ constexpr double ulp_at(double v, int mb) { return pow2_floor(v) / (double)(1ll << mb); }
__host__ __device__ constexpr double ulp_below(double v, int mb) {
  return pow2_floor(v) == v ? 0.5 * ulp_at(v, mb) : ulp_at(v, mb);
}
__host__ __device__ constexpr bool odd_at(double v, int mb) { return ((long long)(v / ulp_at(v, mb))) & 1; }
// dtype fraction bits: fp16 10, bf16 7; fp32 23
__host__ __device__ constexpr double cut_h(int k, int mb) {
  return (k & 1) ? (k - 0.5) + ulp_at(k - 0.5, mb) : k - 0.5;
}
__host__ __device__ constexpr double cut_y(int k, int mb) {
  const double h = cut_h(k, mb);
  const double mid = h - 0.5 * ulp_below(h, mb);
  return odd_at(h, mb) ? mid + ulp_at(mid, 23) : mid;
}
__host__ __device__ constexpr double cut_m(int k, int mb) {
  const double y = cut_y(k, mb);
  return y - 0.5 * ulp_below(y, 23);
}
__host__ __device__ constexpr bool cut_even(int k, int mb) { return !odd_at(cut_y(k, mb), 23); }

// the fp32 cut of code k for scale s (as fp64): a passes it iff c(a) >= k
template <int MB, int K>
__device__ __forceinline__ float code_cut(double sd) {
  constexpr double m = cut_m(K, MB);
  constexpr bool even = cut_even(K, MB);
  const double t = m * sd;
  float a = __double2float_ru(t);
  if (!even && (double)a == t) a = __uint_as_float(__float_as_uint(a) + 1u);  // strictly above
  return a;
}

template <int MB, int QMAX, int K = 1>
__device__ __forceinline__ void code_cuts(double sd, float* cut) {
  if constexpr (K <= QMAX) {
    cut[K - 1] = code_cut<MB, K>(sd);
    code_cuts<MB, QMAX, K + 1>(sd, cut);
  }
}

// c(a) from the cuts (QMAX = 1, 3, 7, 15): a binary search by selects
template <int QMAX>
__device__ __forceinline__ int code_by_cuts(float a, const float* cut) {
  if constexpr (QMAX == 1) {
    return a >= cut[0];
  } else if constexpr (QMAX == 3) {
    const int b1 = a >= cut[1];
    const int b0 = a >= (b1 ? cut[2] : cut[0]);
    return 2 * b1 + b0;
  } else if constexpr (QMAX == 7) {
    const int b2 = a >= cut[3];
    const int b1 = a >= (b2 ? cut[5] : cut[1]);
    const float c0 = b2 ? (b1 ? cut[6] : cut[4]) : (b1 ? cut[2] : cut[0]);
    return 4 * b2 + 2 * b1 + (a >= c0);
  } else {
    const int b3 = a >= cut[7];
    const int b2 = a >= (b3 ? cut[11] : cut[3]);
    const float c1 = b3 ? (b2 ? cut[13] : cut[9]) : (b2 ? cut[5] : cut[1]);
    const int b1 = a >= c1;
    const int i0 = 8 * b3 + 4 * b2 + 2 * b1;  // cut index i0 (+1 - 1)
    float c0 = cut[0];
#pragma unroll
    for (int i = 2; i < 16; i += 2) c0 = i0 == i ? cut[i] : c0;
    return i0 + (a >= c0);
  }
}

// --------------------------------- symmetric codes, two elements at a time ---
// For a dtype value a, a >= cut (fp32) exactly when a >= ru(cut), the
// smallest dtype value at or above the cut.  So with the cuts rounded up to
// the dtype, the code magnitude of |a| is the number of cuts it reaches, and
// both 16-bit elements of a word are coded by packed dtype instructions (on
// the FMA pipe): per cut, a packed compare giving 1.0 / 0.0 and a packed FMA
// adding sign(a) * that to an accumulator that starts at BASE + 2^(b-1), with
// BASE = 1024 (fp16) or 128 (bf16): there consecutive integers are consecutive
// bit patterns, so the low byte of each half ends up holding the offset-binary
// code u = 2^(b-1) + sign * c exactly.  A NaN element compares false: code 0.
template <int DT> __device__ __forceinline__ uint32_t cut_bits(float cut);
template <> __device__ __forceinline__ uint32_t cut_bits<F16>(float cut) {
  return __half_as_ushort(__float2half_ru(cut));
}
template <> __device__ __forceinline__ uint32_t cut_bits<BF16>(float cut) {
  return __bfloat16_as_ushort(__float2bfloat16_ru(cut));
}

template <int DT> struct Pair;
template <> struct Pair<F16> {
  using T = __half2;
  static constexpr uint32_t kOne = 0x3c003c00u, kBase = 0x64006400u;  // 1.0, 1024.0
};
template <> struct Pair<BF16> {
  using T = __nv_bfloat162;
  static constexpr uint32_t kOne = 0x3f803f80u, kBase = 0x43004300u;  // 1.0, 128.0
};
template <int DT> __device__ __forceinline__ typename Pair<DT>::T as_pair(uint32_t w) {
  return *reinterpret_cast<const typename Pair<DT>::T*>(&w);
}
template <int DT> __device__ __forceinline__ uint32_t pair_bits(typename Pair<DT>::T v) {
  return *reinterpret_cast<const uint32_t*>(&v);
}
// max(m, |a|) per half, in the dtype (exact)
template <int DT> __device__ __forceinline__ uint32_t absmax2(uint32_t m, uint32_t a) {
  return pair_bits<DT>(__hmax2(as_pair<DT>(m), __habs2(as_pair<DT>(a))));
}

// max(m, a) / min(m, a) per half, in the dtype (exact)
template <int DT> __device__ __forceinline__ uint32_t max2(uint32_t m, uint32_t a) {
  return pair_bits<DT>(__hmax2(as_pair<DT>(m), as_pair<DT>(a)));
}
template <int DT> __device__ __forceinline__ uint32_t min2(uint32_t m, uint32_t a) {
  return pair_bits<DT>(__hmin2(as_pair<DT>(m), as_pair<DT>(a)));
}

// Asymmetric codes c = #{cuts at or below rnd_dt(a - z)} of the two elements
// of w in bytes 0 and 2; z2: the two zero points (the group minima) as dtype
// bits.  The packed subtraction rounds a - z once to the dtype; the
// reference's fp32 subtraction then dtype rounding gives the same value,
// because the difference of two dtype values is exact in fp32 unless their
// exponents lie more than 13 (fp16; 16 for bf16) apart, and then both
// roundings return the larger operand.
template <int DT, int BITS>
__device__ __forceinline__ uint32_t asym_codes2(uint32_t w, uint32_t z2, const uint32_t* cb) {
  constexpr int QM = (1 << BITS) - 1;
  const auto d = __hsub2(as_pair<DT>(w), as_pair<DT>(z2));
  if constexpr (BITS == 4) {
    // 15 cuts: a binary search per half, four packed compares (all-ones /
    // all-zero masks) and per-half selects of the next cut by bit logic
    auto ge = [&](uint32_t c) -> uint32_t { return __hge2_mask(d, as_pair<DT>(c)); };
    auto sel = [](uint32_t m, uint32_t a, uint32_t b) -> uint32_t { return (m & a) | (~m & b); };
    const uint32_t m3 = ge(cb[7]);
    const uint32_t m2 = ge(sel(m3, cb[11], cb[3]));
    const uint32_t m1 = ge(sel(m3, sel(m2, cb[13], cb[9]), sel(m2, cb[5], cb[1])));
    const uint32_t c0 = sel(m3, sel(m2, sel(m1, cb[14], cb[12]), sel(m1, cb[10], cb[8])),
                            sel(m2, sel(m1, cb[6], cb[4]), sel(m1, cb[2], cb[0])));
    const uint32_t m0 = ge(c0);
    return (m3 & 0x00080008u) | (m2 & 0x00040004u) | (m1 & 0x00020002u) | (m0 & 0x00010001u);
  } else {
    auto acc = as_pair<DT>(Pair<DT>::kBase);
#pragma unroll
    for (int k = 0; k < QM; ++k) acc = __hadd2(acc, __hge2(d, as_pair<DT>(cb[k])));
    return pair_bits<DT>(acc);
  }
}

// Offset-binary symmetric codes of the two elements of w in bytes 0 and 2;
// cb[k]: the cut of code k + 1 rounded up to the dtype, for (half 0, half 1)
template <int DT, int BITS>
__device__ __forceinline__ uint32_t sym_codes2(uint32_t w, const uint32_t* cb) {
  constexpr int QM = (1 << (BITS - 1)) - 1;
  const auto a = __habs2(as_pair<DT>(w));
  const auto sg = as_pair<DT>((w & 0x80008000u) | Pair<DT>::kOne);  // +-1.0
  auto acc = as_pair<DT>(Pair<DT>::kBase + (1u << (BITS - 1)) * 0x00010001u);
#pragma unroll
  for (int k = 0; k < QM; ++k) acc = __hfma2(__hge2(a, as_pair<DT>(cb[k])), sg, acc);
  return pair_bits<DT>(acc);
}

// ------------------------------------------- programmatic dependent launch ---
// Every kernel of the decode step is launched as the programmatic dependent of
// the previous kernel on its stream (launch_pdl), so its launch and prologue
// overlap the tail of that kernel.  The rules that keep stream order:
//   * each kernel calls griddep_wait() before it reads or writes memory that
//     an earlier kernel on the stream produces or reads, and before it ends;
//     the wait returns once the previous grid has completed and its memory is
//     visible, so by induction every earlier kernel has completed too;
//   * griddep_launch_dependents() lets the next grid start early; a kernel
//     calls it only after its own wait.
// Without a programmatic predecessor the wait returns at once.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ------------------------------------------------------------------ mma ---
__device__ __forceinline__ void mma_f16(float c[4], const uint32_t a[4], const uint32_t b[2]) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
__device__ __forceinline__ void mma_bf16(float c[4], const uint32_t a[4], const uint32_t b[2]) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
template <int DT> __device__ __forceinline__ void mma_dt(float c[4], const uint32_t a[4], const uint32_t b[2]);
template <> __device__ __forceinline__ void mma_dt<F16>(float c[4], const uint32_t a[4], const uint32_t b[2]) { mma_f16(c, a, b); }
template <> __device__ __forceinline__ void mma_dt<BF16>(float c[4], const uint32_t a[4], const uint32_t b[2]) { mma_bf16(c, a, b); }

// integer MMA: u8 codes x s8 / u8 digits, exact int32 accumulation
__device__ __forceinline__ void mma_u8s8(int c[4], const uint32_t a[4], const uint32_t b[2]) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
__device__ __forceinline__ void mma_u8u8(int c[4], const uint32_t a[4], const uint32_t b[2]) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// same, with a separate accumulator input c (d = a*b + c); passing literal
// zeros or per-thread constants for c avoids materialising zeroed registers
__device__ __forceinline__ void imma_u8s8(int d[4], const uint32_t a[4], const uint32_t b[2], int c0,
                                          int c1, int c2, int c3) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(c0), "r"(c1), "r"(c2),
        "r"(c3));
}
__device__ __forceinline__ void imma_u8u8(int d[4], const uint32_t a[4], const uint32_t b[2], int c0,
                                          int c1, int c2, int c3) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(c0), "r"(c1), "r"(c2),
        "r"(c3));
}

// ------------------------------------------------------ code extraction ---
// One m16n8k32 A-fragment register (4 codes as bytes) from packed words.
// Row layout (K): w = the words of one token row (b=3: L0, L1, H).
template <int BITS>
__device__ __forceinline__ uint32_t row_frag(const uint32_t* w, int kb, int half) {
  if constexpr (BITS == 4) {
    return (w[kb] >> (4 * half)) & 0x0F0F0F0Fu;
  } else {
    const uint32_t l = (w[kb >> 1] >> (2 * ((kb & 1) * 2 + half))) & 0x03030303u;
    if constexpr (BITS == 2) return l;
    return l | (((w[2] >> (kb * 2 + half)) & 0x01010101u) << 2);
  }
}
// Col layout (V): the lane's chunk words (b=3: 8 L words then 4 H words).
// The register holds col_scale<BITS>(mt) * code per byte.
template <int BITS>
__device__ __forceinline__ uint32_t col_frag(const uint32_t* w, int mt, int h, int half) {
  if constexpr (BITS == 4) {
    return w[(mt & 3) * 4 + h * 2 + half] & (mt < 4 ? 0x0F0F0F0Fu : 0xF0F0F0F0u);
  } else if constexpr (BITS == 2) {
    return w[(mt & 1) * 4 + h * 2 + half] & (0x03030303u << (2 * (mt >> 1)));
  } else {
    const uint32_t l = (w[mt] >> (2 * (h * 2 + half))) & 0x03030303u;
    return l | (((w[8 + (mt >> 1)] >> ((mt & 1) * 4 + h * 2 + half)) & 0x01010101u) << 2);
  }
}
template <int BITS>
__host__ __device__ constexpr int col_scale(int mt) {
  return BITS == 4 ? (mt < 4 ? 1 : 16) : (BITS == 2 ? 1 << (2 * (mt >> 1)) : 1);
}

// --------------------------------------------------- layout index helpers ---
// Byte offset (of a 32-bit word) + bit shift of the code of token-in-tile r,
// dim d; hoff / hshift locate bit 2 of a 3-bit code in plane H.
struct BitPos { int off; int shift; int hoff; int hshift; };

__host__ __device__ inline BitPos row_pos(int bits, int r, int d) {
  const int gid = r & 7, j = r >> 3;
  const int kb = d >> 5, half = (d >> 4) & 1, tq = (d >> 2) & 3, i = d & 3;
  const int lane = gid * 4 + tq;
  BitPos p{0, 0, 0, 0};
  if (bits == 1) {  // a single bit plane laid out like plane H of b=3
    p.off = lane * 16 + j * 4;
    p.shift = 8 * i + kb * 2 + half;
  } else if (bits == 4) {
    p.off = j * 512 + lane * 16 + kb * 4;
    p.shift = 4 * (2 * i + half);
  } else {
    p.off = (j >> 1) * 512 + lane * 16 + (j & 1) * 8 + (kb >> 1) * 4;
    p.shift = 2 * (4 * i + (kb & 1) * 2 + half);
    if (bits == 3) {
      p.hoff = 1024 + lane * 16 + j * 4;
      p.hshift = 8 * i + kb * 2 + half;
    }
  }
  return p;
}

__host__ __device__ inline BitPos col_pos(int bits, int r, int d) {
  const int mt = d >> 4, h = (d >> 3) & 1, gid = d & 7;
  const int half = r >> 4, tq = (r >> 2) & 3, i = r & 3;
  const int lane = gid * 4 + tq;
  BitPos p{0, 0, 0, 0};
  if (bits == 1) {
    p.off = lane * 16 + (mt >> 1) * 4;
    p.shift = 8 * i + (mt & 1) * 4 + h * 2 + half;
  } else if (bits == 4) {
    p.off = (mt & 3) * 512 + lane * 16 + (h * 2 + half) * 4;
    p.shift = 8 * i + 4 * (mt >> 2);
  } else if (bits == 2) {
    p.off = (mt & 1) * 512 + lane * 16 + (h * 2 + half) * 4;
    p.shift = 8 * i + 2 * (mt >> 1);
  } else {
    p.off = (mt >> 2) * 512 + lane * 16 + (mt & 3) * 4;
    p.shift = 2 * (4 * i + h * 2 + half);
    p.hoff = 1024 + lane * 16 + (mt >> 1) * 4;
    p.hshift = 8 * i + (mt & 1) * 4 + h * 2 + half;
  }
  return p;
}

// scale index inside a row-layout tile (channel groups)
__host__ __device__ inline int row_scale_idx(int r, int g, int ng) {
  return ((r & 7) * ng + g) * 4 + (r >> 3);
}
// scale index inside a col-layout group (token groups)
__host__ __device__ inline int col_scale_idx(int d) {
  return (d & 7) * 16 + (d >> 4) * 2 + ((d >> 3) & 1);
}

}  // namespace innerq
