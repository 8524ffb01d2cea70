// bf16 dense GEMV rows on mma.sync for the shared expert (bf16 x bf16
// products are exact in float32).  Lane (gid, tig) loads 16 bytes of two
// weight rows (gid, gid+8) and 16 bytes of token gid at k = 8*tig..8*tig+7
// of each 32-wide step; the step is two m16n8k16 MMAs whose k order is
// permuted identically in A and B.
#pragma once

#include <stdint.h>

namespace exlr8 {

// Streaming 128-bit load (no L1 allocation).  Plain (not volatile) asm, so
// that the compiler may issue a batch of these ahead of their uses.
__device__ __forceinline__ uint4 ldg128_stream(const void* p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}

__device__ __forceinline__ void mma_bf16(float c[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One warp: rows n0..n0+15 of W ([n][k] bf16; W1 optional second matrix with
// the same shape sharing the x loads), k steps [s0, s1) of 32, all tokens;
// writes float32 partials p0/p1 [tokens][n] of this split.  The loads of
// kUnroll k steps are issued as one batch before their MMAs.
template <int kUnroll = 4>
__device__ __forceinline__ void dense_rows(const uint16_t* __restrict__ x, int tokens, const uint16_t* __restrict__ w0,
                                           const uint16_t* __restrict__ w1, int n, int k, int n0, int s0, int s1,
                                           float* __restrict__ p0, float* __restrict__ p1, int lane) {
  const int gid = lane >> 2, tig = lane & 3;
  const uint16_t* a0 = w0 + static_cast<int64_t>(n0 + gid) * k + 8 * tig;
  const uint16_t* a1 = a0 + static_cast<int64_t>(8) * k;
  const uint16_t* b0 = w1 ? w1 + static_cast<int64_t>(n0 + gid) * k + 8 * tig : nullptr;
  const uint16_t* b1 = w1 ? b0 + static_cast<int64_t>(8) * k : nullptr;
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  for (int t0 = 0; t0 < tokens; t0 += 8) {
    const bool has_token = t0 + gid < tokens;
    const uint16_t* xr = x + static_cast<int64_t>(has_token ? t0 + gid : 0) * k + 8 * tig;
    float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
    for (int st = s0; st < s1; st += kUnroll) {
      uint4 ra[kUnroll], rb[kUnroll], rc[kUnroll], rd[kUnroll], xv[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const bool in = st + u < s1;
        const int o = (st + u) * 32;
        ra[u] = in ? ldg128_stream(a0 + o) : zero;
        rb[u] = in ? ldg128_stream(a1 + o) : zero;
        rc[u] = in && w1 ? ldg128_stream(b0 + o) : zero;
        rd[u] = in && w1 ? ldg128_stream(b1 + o) : zero;
        xv[u] = in && has_token ? *reinterpret_cast<const uint4*>(xr + o) : zero;
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        mma_bf16(c0, ra[u].x, rb[u].x, ra[u].y, rb[u].y, xv[u].x, xv[u].y);
        mma_bf16(c0, ra[u].z, rb[u].z, ra[u].w, rb[u].w, xv[u].z, xv[u].w);
        if (w1) {
          mma_bf16(c1, rc[u].x, rd[u].x, rc[u].y, rd[u].y, xv[u].x, xv[u].y);
          mma_bf16(c1, rc[u].z, rd[u].z, rc[u].w, rd[u].w, xv[u].z, xv[u].w);
        }
      }
    }
    // c0,c1: row gid, tokens 2tig, 2tig+1; c2,c3: row gid+8.
    const int ta = t0 + 2 * tig, tb = ta + 1;
    if (ta < tokens) {
      p0[static_cast<int64_t>(ta) * n + n0 + gid] = c0[0];
      p0[static_cast<int64_t>(ta) * n + n0 + gid + 8] = c0[2];
      if (w1) {
        p1[static_cast<int64_t>(ta) * n + n0 + gid] = c1[0];
        p1[static_cast<int64_t>(ta) * n + n0 + gid + 8] = c1[2];
      }
    }
    if (tb < tokens) {
      p0[static_cast<int64_t>(tb) * n + n0 + gid] = c0[1];
      p0[static_cast<int64_t>(tb) * n + n0 + gid + 8] = c0[3];
      if (w1) {
        p1[static_cast<int64_t>(tb) * n + n0 + gid] = c1[1];
        p1[static_cast<int64_t>(tb) * n + n0 + gid + 8] = c1[3];
      }
    }
  }
}

}  // namespace exlr8
