// Shared device helpers for the InnerQ B200 kernels: dtype rounding, the packed
// tile layouts, code extraction into fp16 pairs, and mma.sync wrappers.
//
// Packed layouts (D = 128, tiles of 32 tokens, b = bits per code):
//
// "row" layout (K, channel groups; the A operand is K[token][dim]):
//   tile = 32 tokens = 512*b bytes.  Lane L = 4*gid + tq of the consuming warp
//   owns the 32 codes of tokens r = gid + 8*j (j = 0..3) at dims
//   kb*16 + {2tq, 2tq+1, 2tq+8, 2tq+9} (kb = 0..7), i.e. exactly the
//   m16n8k16 A-fragment elements.  Row-local code index c = kb*4 + hi8*2 + e.
//     b=4: lane chunk 64 B = 4 rows x 16 B; word w = kb>>1, nibble (kb&1)*2+hi8 + 4e
//     b=2: lane chunk 32 B = 4 rows x  8 B; word w = kb>>2, crumb  (kb&3)*2+hi8 + 8e
//     b=3: low 2 bits as b=2 in plane L (1024 B / tile), bit 2 in plane H
//          (512 B / tile, 4 B per row): bit (kb*2+hi8) + 16e
//   Scales / zero points (channel groups, ng = D/G per token) per tile:
//     [gid 8][j 4][ng] 16-bit values.
//
// "col" layout (V, token groups; the A operand is V^T[dim][token]):
//   Lane L = 4*gid + tq owns dims d = mt*16 + h*8 + gid (mt = 0..7, h = 0..1)
//   at tokens kb*16 + {2tq, 2tq+1, 2tq+8, 2tq+9} (kb = 0..1).
//     b=4: 16 words; word mt*2+h, nibble (kb*2+hi8) + 4e
//     b=2:  8 words; word mt,     crumb  (h*4+kb*2+hi8) + 8e
//     b=3: plane L as b=2; plane H 4 words: word mt>>1, bit ((mt&1)*8+h*4+kb*2+hi8) + 16e
//   Scales / zero points (token groups, one per (group, dim)): [gid 8][mt 8][h 2].
//
// Symmetric codes are stored offset-binary: u = sign*code + 2^(b-1) (1..2^b-1);
// asymmetric codes are stored as is (0..2^b-1).
#pragma once
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

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

// hi/lo split of an fp32 value into two 16-bit values of dtype DT packed as
// the low (first) element of a pair
template <int DT> __device__ __forceinline__ void split_hilo(float v, uint16_t& hi, uint16_t& lo) {
  hi = from_f<DT>(v);
  lo = from_f<DT>(v - to_f<DT>(hi));
}

__device__ __forceinline__ uint32_t pack2(uint16_t lo, uint16_t hi) {
  return (uint32_t)lo | ((uint32_t)hi << 16);
}

// ------------------------------------------------------------------ mma ---
__device__ __forceinline__ void mma_f16(float c[4], const uint32_t a[4], const uint32_t b[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
__device__ __forceinline__ void mma_bf16(float c[4], const uint32_t a[4], const uint32_t b[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
template <int DT> __device__ __forceinline__ void mma_dt(float c[4], const uint32_t a[4], const uint32_t b[2]);
template <> __device__ __forceinline__ void mma_dt<F16>(float c[4], const uint32_t a[4], const uint32_t b[2]) { mma_f16(c, a, b); }
template <> __device__ __forceinline__ void mma_dt<BF16>(float c[4], const uint32_t a[4], const uint32_t b[2]) { mma_bf16(c, a, b); }

// ------------------------------------------------------ code extraction ---
// fp16 pair (1024 + x, 1024 + y) from the two fields of a word selected by
// mask at shift s; then subtract the 1024 + offset bias exactly in fp16.
__device__ __forceinline__ uint32_t magic_pair(uint32_t w, int shift, uint32_t mask) {
  return ((w >> shift) & mask) | 0x64006400u;
}
__device__ __forceinline__ uint32_t hsub_u32(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t hfma_u32(uint32_t a, uint32_t b, uint32_t c) {
  __half2 r = __hfma2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b),
                      *reinterpret_cast<__half2*>(&c));
  return *reinterpret_cast<uint32_t*>(&r);
}
// bias constant (1024 + off) as an fp16 pair; off <= 8 so the sum is exact
__host__ __device__ constexpr uint32_t bias_pair(int off) {
  // fp16 of 1024 + k for 0 <= k < 1024 is 0x6400 + k
  return (uint32_t)(0x6400 + off) | ((uint32_t)(0x6400 + off) << 16);
}

// Decode pair p (elements at field p and p + fields/2) of a b-bit word as
// signed fp16 values (u - off).  For b = 3 the caller supplies the L word
// (2-bit pair index pl) and the H word (1-bit pair index ph).
template <int BITS> struct Dec;
template <> struct Dec<4> {
  static __device__ __forceinline__ uint32_t pair(uint32_t w, int p, uint32_t bias) {
    return hsub_u32(magic_pair(w, 4 * p, 0x000F000Fu), bias);
  }
};
template <> struct Dec<2> {
  static __device__ __forceinline__ uint32_t pair(uint32_t w, int p, uint32_t bias) {
    return hsub_u32(magic_pair(w, 2 * p, 0x00030003u), bias);
  }
};
struct Dec3 {
  static __device__ __forceinline__ uint32_t pair(uint32_t wl, int pl, uint32_t wh, int ph,
                                                  uint32_t bias) {
    uint32_t lo = hsub_u32(magic_pair(wl, 2 * pl, 0x00030003u), bias);       // l - off
    uint32_t hi = hsub_u32(magic_pair(wh, ph, 0x00010001u), 0x64006400u);    // h in {0,1}
    return hfma_u32(hi, 0x44004400u /* 4.0 */, lo);                            // 4h + l - off
  }
};

// --------------------------------------------------- layout index helpers ---
// Byte offset + bit shift of the code of token-in-tile r, dim d, row layout.
struct BitPos { int off; int shift; int hoff; int hshift; };

__host__ __device__ inline BitPos row_pos(int bits, int r, int d) {
  int gid = r & 7, j = r >> 3;
  int kb = d >> 4, dd = d & 15, tq = (dd & 7) >> 1, e = dd & 1, hi8 = dd >> 3;
  int lane = gid * 4 + tq;
  BitPos p{0, 0, 0, 0};
  if (bits == 4) {
    int w = kb >> 1, nib = (kb & 1) * 2 + hi8 + 4 * e;
    p.off = lane * 64 + j * 16 + w * 4;
    p.shift = 4 * nib;
  } else {  // 2-bit, or the L plane of 3-bit
    int w = kb >> 2, cr = (kb & 3) * 2 + hi8 + 8 * e;
    p.off = lane * 32 + j * 8 + w * 4;
    p.shift = 2 * cr;
    if (bits == 3) {
      p.hoff = 1024 + lane * 16 + j * 4;
      p.hshift = kb * 2 + hi8 + 16 * e;
    }
  }
  return p;
}

__host__ __device__ inline BitPos col_pos(int bits, int r, int d) {
  int mt = d >> 4, h = (d >> 3) & 1, gid = d & 7;
  int kb = r >> 4, rr = r & 15, tq = (rr & 7) >> 1, e = rr & 1, hi8 = rr >> 3;
  int lane = gid * 4 + tq;
  BitPos p{0, 0, 0, 0};
  if (bits == 4) {
    p.off = lane * 64 + (mt * 2 + h) * 4;
    p.shift = 4 * (kb * 2 + hi8 + 4 * e);
  } else {
    p.off = lane * 32 + mt * 4;
    p.shift = 2 * (h * 4 + kb * 2 + hi8 + 8 * e);
    if (bits == 3) {
      p.hoff = 1024 + lane * 16 + (mt >> 1) * 4;
      p.hshift = (mt & 1) * 8 + h * 4 + kb * 2 + hi8 + 16 * e;
    }
  }
  return p;
}

// scale index inside a row-layout tile (channel groups)
__host__ __device__ inline int row_scale_idx(int r, int g, int ng) {
  return ((r & 7) * 4 + (r >> 3)) * ng + g;
}
// scale index inside a col-layout group (token groups)
__host__ __device__ inline int col_scale_idx(int d) {
  return (d & 7) * 16 + (d >> 4) * 2 + ((d >> 3) & 1);
}

}  // namespace innerq
