// EXLR8 trellis codec on the device: codeword -> exact E4M3-rounded value,
// the direct K4 codeword extraction, and the generic K sliding windows.
//
// Format (exlr8/trellis.py:43-50,78-102; metal/fast_decode_common.metal:4-26):
// a 16-bit trellis state cw is hashed as (cw * 0xCBAC1FED mod 2^32) &
// 0x8FFF8FFF ^ 0x3B603B60; the two 16-bit halves are float16 numbers, their
// float16 sum rounded to E4M3 (nearest, ties to even) is the weight.  The
// E4M3 rounding here is the hardware float16x2 -> e4m3x2 conversion
// (round-to-nearest, finite saturation) and back, which the test-suite checks
// against the reference codebook over all 65,536 states.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace exlr8 {

constexpr uint32_t kMcgMul = 0xCBAC1FEDu;
constexpr uint32_t kMcgMask = 0x8FFF8FFFu;
constexpr uint32_t kMcgXor = 0x3B603B60u;

// Round an f16x2 to the nearest E4M3 pair and widen it back to f16x2.
__device__ __forceinline__ uint32_t round_e4m3_f16x2(uint32_t h2) {
  uint32_t r;
  asm("{\n .reg .b16 t;\n cvt.rn.satfinite.e4m3x2.f16x2 t, %1;\n cvt.rn.f16x2.e4m3x2 %0, t;\n}\n"
      : "=r"(r)
      : "r"(h2));
  return r;
}

// Float16 half sums of two hashed products pa = cw_a * C, pb = cw_b * C,
// packed as an f16x2 (low half = a): each product is masked as a whole (its
// two halves are the two float16 numbers of its codeword) and the halves of
// each product are added, then the two sums are packed.  One mask per
// product and one pack per pair cost one integer-pipe instruction less per
// pair than gathering the low and the high halves of both products first,
// and the float16 additions are the same, so the result is identical.
__device__ __forceinline__ uint32_t hashed_pair_sum(uint32_t pa, uint32_t pb, uint32_t mask, uint32_t xorv) {
  uint32_t qa, qb, r;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(qa) : "r"(pa), "r"(mask), "r"(xorv));
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(qb) : "r"(pb), "r"(mask), "r"(xorv));
  asm("{\n .reg .b16 al, ah, bl, bh, sa, sb;\n mov.b32 {al, ah}, %1;\n mov.b32 {bl, bh}, %2;\n"
      " add.rn.f16 sa, al, ah;\n add.rn.f16 sb, bl, bh;\n mov.b32 %0, {sa, sb};\n}\n"
      : "=r"(r)
      : "r"(qa), "r"(qb));
  return r;
}

// Values of two 16-bit states as an f16x2 (low half = state a).
__device__ __forceinline__ uint32_t decode_pair(uint32_t cw_a, uint32_t cw_b) {
  return round_e4m3_f16x2(hashed_pair_sum(cw_a * kMcgMul, cw_b * kMcgMul, kMcgMask, kMcgXor));
}

__device__ __forceinline__ float decode_value(uint32_t cw) {
  uint32_t r = decode_pair(cw & 0xFFFFu, cw & 0xFFFFu);
  return __half2float(__ushort_as_half(static_cast<uint16_t>(r & 0xFFFFu)));
}

// The eight codewords of lane l of a K4 tile: the stream window (prior:word)
// where word is tile word l and prior is word l-1 (cyclic).  Codeword j ends
// 4*(7-j) bits above bit 0 of word (fast_decode_linear.metal:147-155).
__device__ __forceinline__ void k4_codewords(uint32_t word, uint32_t prior, uint32_t cw[8]) {
  cw[0] = __funnelshift_r(word, prior, 28) & 0xFFFFu;
  cw[1] = __funnelshift_r(word, prior, 24) & 0xFFFFu;
  cw[2] = __funnelshift_r(word, prior, 20) & 0xFFFFu;
  cw[3] = word >> 16;
  cw[4] = (word >> 12) & 0xFFFFu;
  cw[5] = (word >> 8) & 0xFFFFu;
  cw[6] = (word >> 4) & 0xFFFFu;
  cw[7] = word & 0xFFFFu;
}

// mma.sync m16n8k16 A-fragment registers of one decoded 16x16 tile.  With the
// tile used as A = W^T (rows = output columns, k = input rows), the trellis
// tensor-core permutation places codeword j of lane l at exactly the fragment
// element the instruction expects: {a0,a1}=j0,j1  {a2,a3}=j4,j5
// {a4,a5}=j2,j3  {a6,a7}=j6,j7.
__device__ __forceinline__ void tile_fragment(const uint32_t cw[8], uint32_t a[4]) {
  a[0] = decode_pair(cw[0], cw[1]);
  a[1] = decode_pair(cw[4], cw[5]);
  a[2] = decode_pair(cw[2], cw[3]);
  a[3] = decode_pair(cw[6], cw[7]);
}

// Generic K: per lane two 64-bit windows (groups of four codewords); the
// window of group g is words (left, right) of the tile, codeword 4g+q sits at
// shift + (3-q)*K (trellis.metal:33-40, decode.metal:19-23).
struct GenericGeometry {
  uint32_t left[2], right[2], shift[2];
};

__device__ __forceinline__ GenericGeometry generic_geometry(int k, int lane) {
  GenericGeometry g;
  const uint32_t words = 8u * k;
#pragma unroll
  for (int grp = 0; grp < 2; ++grp) {
    uint32_t last_bit = (lane * 8u + grp * 4u + 4u) * k + 256u * k;
    uint32_t last_word = (last_bit - 1u) / 32u;
    g.left[grp] = (last_word - 1u) % words;
    g.right[grp] = last_word % words;
    g.shift[grp] = (last_word + 1u) * 32u - last_bit;
  }
  return g;
}

__device__ __forceinline__ void generic_codewords(const uint32_t* tile, int k, const GenericGeometry& g,
                                                  uint32_t cw[8]) {
#pragma unroll
  for (int grp = 0; grp < 2; ++grp) {
    uint64_t merged = (static_cast<uint64_t>(tile[g.left[grp]]) << 32) | tile[g.right[grp]];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      cw[grp * 4 + q] = static_cast<uint32_t>(merged >> (g.shift[grp] + (3 - q) * k)) & 0xFFFFu;
    }
  }
}

// Storage index (in tiles) of tile (tk, tn) of matrix e: side 1/0 output
// blocks first, side 2 input blocks first (fast_decode_linear.metal:91-95).
__device__ __forceinline__ int64_t tile_index(int64_t e, int tk, int tn, int in_tiles, int out_tiles, int side) {
  if (side == 2) {
    return ((((e * (in_tiles / 8) + tk / 8) * (out_tiles / 8) + tn / 8) * 8 + tk % 8) * 8) + tn % 8;
  }
  return ((e * (out_tiles / 8) + tn / 8) * in_tiles + tk) * 8 + tn % 8;
}

// Inner weight [r][c] of matrix e (decode.metal:9-35): the 16-bit codeword
// of position (r % 16, c % 16) read from the two words its bits straddle in
// the tile's 8k-word ring, then the codebook value.
__device__ __forceinline__ float trellis_weight(const uint32_t* __restrict__ words, int64_t e, int k, int in_tiles,
                                                int out_tiles, int side, int r, int c) {
  const int lr = r & 15, lc = c & 15;
  const uint32_t lane = (lc & 7) * 4 + ((lr & 7) >> 1);
  const uint32_t slot = (lr & 1) + ((lr & 8) >> 2) + ((lc & 8) >> 1);
  const uint32_t code = lane * 8 + slot;
  const uint32_t nwords = 8u * k;
  const uint32_t last_bit = (code + 1) * k + 256u * k;
  const uint32_t last_word = (last_bit - 1) / 32;
  const uint32_t shift = (last_word + 1) * 32 - last_bit;
  const uint32_t* tile = words + tile_index(e, r >> 4, c >> 4, in_tiles, out_tiles, side) * nwords;
  const uint64_t merged = (static_cast<uint64_t>(tile[(last_word - 1) % nwords]) << 32) | tile[last_word % nwords];
  return decode_value(static_cast<uint32_t>(merged >> shift) & 0xFFFFu);
}

}  // namespace exlr8
