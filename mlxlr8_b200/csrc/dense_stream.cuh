// The bf16 shared expert inside the trellis stream kernel: one extra warp per
// CTA streams the dense weight rows while the other warps decode trellis
// codes.  The trellis units are bound by their decode arithmetic and leave
// most of the HBM bandwidth unused; the dense rows are bound by HBM and need
// almost no arithmetic, so the two overlap within the same CTAs.
//
// A dense unit is (16-row group of W, K split).  For each 128-wide K chunk
// of its units the dense warp loads the 16 rows of W (and of W1, which shares
// the x loads) as two 2-D tensor-map boxes of 16 rows x 64 values per matrix
// (128-byte swizzle, no multicast), and the tokens' x rows with 1-D bulk
// copies, into a 4-deep ring of shared-memory buffers completing on
// mbarriers.  (Sixteen 256-byte row copies per matrix and chunk, the earlier
// form, kept the SM's copy engine so busy that the trellis code stages
// behind them arrived late: the boxes cut the copies per chunk from 33 to 5.)
// It multiplies with ldmatrix + mma.sync (bf16 x bf16, float32 accumulation;
// the products are exact) and writes float32 partials [splits][tokens][n]
// per unit.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "dense_warp.cuh"
#include "stream.cuh"
#include "tma.cuh"

namespace exlr8 {

constexpr int kDenseRows = 16;                              // rows of W per unit
constexpr int kDenseChunk = 128;                            // K values per staged chunk
constexpr int kDenseTokens = 16;                            // tokens per pass
constexpr int kDenseBuffers = 4;                            // chunks in flight per dense warp
constexpr int kDenseRowBytes = kDenseChunk * 2 + 16;        // x rows, padded: ldmatrix rows on distinct banks
constexpr int kDenseBoxBytes = kDenseRows * 128;            // 16 rows x 64 bf16 values, 128-byte swizzle
constexpr int kDenseMatBytes = 2 * kDenseBoxBytes;          // one matrix's chunk: two boxes
constexpr int kDenseXOffset = 2 * kDenseMatBytes;           // W0, W1, then the x rows
constexpr int kDenseBufBytes = (kDenseXOffset + kDenseTokens * kDenseRowBytes + 1023) / 1024 * 1024;
constexpr int kDenseSmemBytes = kDenseBuffers * kDenseBufBytes + 1024;  // + alignment of the ring to 1 KB

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Orders this thread's earlier shared-memory reads before later bulk copies
// (async proxy) into the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// K splits of a dense matrix with k inputs: the largest count <= max_splits
// that cuts k into whole 128-wide chunks.
inline int dense_split_count(int k, int max_splits) {
  const int chunks = k / kDenseChunk;
  int s = max_splits < chunks ? max_splits : chunks;
  while (s > 1 && chunks % s) --s;
  return s < 1 ? 1 : s;
}

// 2-D tiled tensor-map load (no multicast) of the box at (x, y) into `dst`.
__device__ __forceinline__ void dense_tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Issues the loads of one chunk (rows n0.., K values kc..kc+127, tokens
// t0..t0+nt-1) into `dst` (1 KB aligned), completing on `bar`.  The box x
// coordinates kc and kc + 64 are multiples of 64 bf16 values (128 bytes).
__device__ __forceinline__ void dense_issue_chunk(const DenseUnits& d, const CUtensorMap* w0, const CUtensorMap* w1,
                                                  int n0, int kc, int t0, int nt, unsigned char* dst, uint64_t* bar,
                                                  int lane) {
  const int mats = d.w1 ? 2 : 1;
  constexpr uint32_t kSeg = kDenseChunk * 2;
  fence_proxy_async_smem();
  if (lane == 0) {
    mbar_arrive_expect_tx(bar, static_cast<uint32_t>(mats * kDenseMatBytes) + static_cast<uint32_t>(nt) * kSeg);
    dense_tma_2d(dst, w0, kc, n0, bar);
    dense_tma_2d(dst + kDenseBoxBytes, w0, kc + 64, n0, bar);
    if (mats == 2) {
      dense_tma_2d(dst + kDenseMatBytes, w1, kc, n0, bar);
      dense_tma_2d(dst + kDenseMatBytes + kDenseBoxBytes, w1, kc + 64, n0, bar);
    }
  }
  __syncwarp();
  if (lane < nt)
    bulk_copy_g2s(dst + kDenseXOffset + lane * kDenseRowBytes, d.x + static_cast<int64_t>(t0 + lane) * d.k + kc,
                  kSeg, bar);
}

// ldmatrix address of 16-byte column `col16` (0..15) of row `r` of a matrix
// chunk: two 128-byte-swizzled boxes of 16 rows x 128 bytes.
__device__ __forceinline__ uint32_t dense_a_addr(uint32_t mat, int r, int col16) {
  return mat + (col16 >> 3) * kDenseBoxBytes + r * 128 + (((col16 & 7) ^ (r & 7)) << 4);
}

// One chunk's products: per 16-wide K step, A (16 rows of W, W1) and B (up
// to 16 tokens of x) come from ldmatrix; acc[mat][token block][4] follows
// the m16n8k16 accumulator layout.
__device__ __forceinline__ void dense_chunk_products(const unsigned char* src, bool two, bool second_block, int lane,
                                                     float acc[2][2][4]) {
  const uint32_t base = smem_u32(src);
  const int ar = lane & 15, ac = lane >> 4;  // A: row, and the half (8 values) of the 16-wide K step
  const uint32_t b_row = base + kDenseXOffset + ((lane & 7) + (lane >> 4) * 8) * kDenseRowBytes +
                         ((lane >> 3) & 1) * 16;
#pragma unroll
  for (int ks = 0; ks < kDenseChunk / 16; ++ks) {
    uint32_t b0, b1, b2, b3;
    ldsm_x4(b_row + ks * 32, b0, b1, b2, b3);
    uint32_t a0, a1, a2, a3;
    ldsm_x4(dense_a_addr(base, ar, 2 * ks + ac), a0, a1, a2, a3);
    mma_bf16(acc[0][0], a0, a1, a2, a3, b0, b1);
    if (second_block) mma_bf16(acc[0][1], a0, a1, a2, a3, b2, b3);
    if (two) {
      ldsm_x4(dense_a_addr(base + kDenseMatBytes, ar, 2 * ks + ac), a0, a1, a2, a3);
      mma_bf16(acc[1][0], a0, a1, a2, a3, b0, b1);
      if (second_block) mma_bf16(acc[1][1], a0, a1, a2, a3, b2, b3);
    }
  }
}

// The dense warp's loop over its units: CTA b takes units b, b + grid, ...
// (a static assignment: no counter to reset between calls).  `buf` is
// kDenseSmemBytes of shared memory, `bars` kDenseBuffers mbarriers
// initialised with count 1; `w0`, `w1` the tensor maps of d.w0 / d.w1.
// Returns false when a bounded wait timed out.
__device__ __forceinline__ bool dense_warp_run(const DenseUnits& d, const CUtensorMap* w0, const CUtensorMap* w1,
                                               unsigned char* buf_raw, uint64_t* bars, int lane) {
  unsigned char* buf = buf_raw + ((1024u - (smem_u32(buf_raw) & 1023u)) & 1023u);  // boxes need 1 KB alignment
  const int groups = d.n / kDenseRows;
  const int chunks = d.k / d.splits / kDenseChunk;
  const bool two = d.w1 != nullptr;
  uint32_t issued = 0, consumed = 0;  // chunk sequence numbers (buffer = seq % kDenseBuffers)
  for (int unit = blockIdx.x; unit < d.units; unit += gridDim.x) {
    const int g = unit % groups, split = unit / groups;
    const int n0 = g * kDenseRows, k0 = split * (d.k / d.splits);
    for (int t0 = 0; t0 < d.tokens; t0 += kDenseTokens) {
      const int nt = min(kDenseTokens, d.tokens - t0);
      float acc[2][2][4];
#pragma unroll
      for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[a][b][i] = 0.0f;
      // Keep up to kDenseBuffers chunks of this pass in flight.
      for (int c = 0; c < chunks && c < kDenseBuffers; ++c, ++issued)
        dense_issue_chunk(d, w0, w1, n0, k0 + c * kDenseChunk, t0, nt,
                          buf + (issued % kDenseBuffers) * kDenseBufBytes, &bars[issued % kDenseBuffers], lane);
      for (int c = 0; c < chunks; ++c, ++consumed) {
        const uint32_t b = consumed % kDenseBuffers;
        if (!mbar_wait(&bars[b], (consumed / kDenseBuffers) & 1u)) return false;
        dense_chunk_products(buf + b * kDenseBufBytes, two, nt > 8, lane, acc);
        __syncwarp();
        const int refill = c + kDenseBuffers;
        if (refill < chunks) {
          dense_issue_chunk(d, w0, w1, n0, k0 + refill * kDenseChunk, t0, nt, buf + b * kDenseBufBytes, &bars[b],
                            lane);
          ++issued;
        }
      }
      // Accumulator (row gid / gid + 8, tokens 2 tig, 2 tig + 1) of each block.
      const int gid = lane >> 2, tig = lane & 3;
      const int64_t part = static_cast<int64_t>(split) * d.tokens * d.n;
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        if (m == 1 && !two) break;
        float* p = (m == 0 ? d.p0 : d.p1) + part;
#pragma unroll
        for (int nb = 0; nb < 2; ++nb) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int t = nb * 8 + 2 * tig + h;
            if (t < nt) {
              p[static_cast<int64_t>(t0 + t) * d.n + n0 + gid] = acc[m][nb][h];
              p[static_cast<int64_t>(t0 + t) * d.n + n0 + gid + 8] = acc[m][nb][2 + h];
            }
          }
        }
      }
    }
  }
  return true;
}

}  // namespace exlr8
