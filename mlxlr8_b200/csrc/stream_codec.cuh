// The decode GEMV's codec-to-tensor-core path, shared by the streaming
// kernel and the codec throughput probe: K4 tile fragments from the trellis
// codes (or from static-cache E4M3 bytes) and the mma.sync that consumes
// them.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "codec.cuh"

namespace exlr8 {

// A fragment of one tile from its static-cache bytes: lane l's eight bytes are
// codewords 0-7 of the lane in order, E4M3-coded; the exact float16 values go
// to the same registers as the codec's (j0,j1 | j4,j5 | j2,j3 | j6,j7).
__device__ __forceinline__ void e4m3_fragment(uint2 b, uint32_t a[4]) {
  asm("{\n .reg .b16 l0, h0, l1, h1;\n mov.b32 {l0, h0}, %4;\n mov.b32 {l1, h1}, %5;\n"
      " cvt.rn.f16x2.e4m3x2 %0, l0;\n cvt.rn.f16x2.e4m3x2 %1, l1;\n"
      " cvt.rn.f16x2.e4m3x2 %2, h0;\n cvt.rn.f16x2.e4m3x2 %3, h1;\n}\n"
      : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
      : "r"(b.x), "r"(b.y));
}

__device__ __forceinline__ void mma_f16(float c[4], const uint32_t a[4], uint2 b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y));
}

// Exact E4M3 values (as f16x2, low half = a) of two hashed products.
__device__ __forceinline__ uint32_t pair_from_products(uint32_t pa, uint32_t pb, uint32_t mask, uint32_t xorv) {
  return round_e4m3_f16x2(hashed_pair_sum(pa, pb, mask, xorv));
}

// A fragment of one K4 tile from tile word l and word l-1.  The high
// codeword of each window is a plain shift: on B200 a 32-bit multiply-high
// (the other way to take it) runs well below the half rate of the other
// integer operations, and measured 5% slower over the whole decode.  The
// window shifts stay funnel shifts.
__device__ __forceinline__ void k4_fragment(uint32_t word, uint32_t prior, uint32_t mask, uint32_t xorv,
                                            uint32_t a[4]) {
  const uint32_t v0 = word;                              // (cw3 : cw7)
  const uint32_t v4 = __funnelshift_r(word, prior, 4);   // (cw2 : cw6)
  const uint32_t v8 = __funnelshift_r(word, prior, 8);   // (cw1 : cw5)
  const uint32_t v12 = __funnelshift_r(word, prior, 12); // (cw0 : cw4)
  const uint32_t h0 = v0 >> 16, h4 = v4 >> 16, h8 = v8 >> 16, h12 = v12 >> 16;
  const uint32_t ph0 = h0 * kMcgMul, ph4 = h4 * kMcgMul, ph8 = h8 * kMcgMul, ph12 = h12 * kMcgMul;
  // v*C - ph*2^16 (mod 2^32), one multiply-add each.
  const uint32_t pl0 = v0 * kMcgMul + ph0 * 0xFFFF0000u, pl4 = v4 * kMcgMul + ph4 * 0xFFFF0000u;
  const uint32_t pl8 = v8 * kMcgMul + ph8 * 0xFFFF0000u, pl12 = v12 * kMcgMul + ph12 * 0xFFFF0000u;
  a[0] = pair_from_products(ph12, ph8, mask, xorv);  // j0, j1
  a[1] = pair_from_products(pl12, pl8, mask, xorv);  // j4, j5
  a[2] = pair_from_products(ph4, ph0, mask, xorv);   // j2, j3
  a[3] = pair_from_products(pl4, pl0, mask, xorv);   // j6, j7
}

}  // namespace exlr8
