// Grouped block-scaled expert GEMM on the sm_100a tensor cores:
// weights (E2M1 MXFP4, or trellis codes decoded to their exact E4M3 values)
// times E4M3 hi/lo activation planes, E8M0 scales per 32 values,
// float32 accumulators in TMEM.
//
// It plays the role of the expert matrix products of the reference:
//   * MXFP4: MLX gather_qmm(mode="mxfp4", group_size=32) in the joined path
//     (exlr8 joined_mxfp4.py:109-113 gate+up, 122-126 down);
//   * trellis: the segmented MMA GEMM of grouped_expert_mlp
//     (fast_prefill.py:188-211, metal/fast_prefill.metal), whose per-stage
//     tile decode becomes decoder warps writing E4M3 tiles into shared
//     memory.
//
// Shape of the work: a unit is (projection, chunk, weight block).  The chunk
// is up to kMxMaxN consecutive slot rows of one expert (the MMA N side, so an
// expert with 140 rows costs 144 columns, not two 128-row tiles); the weight
// block is two 128-row tiles of that expert (two TMEM accumulators of
// M = 128).  Each 128-value K step of a unit issues 2 accumulators x 2
// activation planes (hi, lo) x 4 MMAs of K = 32; hi and lo share their scale
// columns.
//
// CTA, one persistent CTA per SM:
//   warp 0      producer: unit scheduler (global atomic), TMA of activation
//               planes and scales, TMA (MXFP4) or bulk copy (trellis codes)
//               of the weights
//   warp 1      MMA issuer (one thread) and TMEM owner
//   epilogue    TMEM -> float32 rows of `out`: 8 warps for MXFP4 (two per
//               TMEM sub-partition, alternating 16-column groups, so the
//               accumulators drain in half the time while the MMA waits),
//               4 warps for trellis (warps 2-5)
//   warp 6      (trellis) code producer: bulk copies of trellis codes into a
//               4-stage ring ahead of the decoders
//   warps 7-22  (trellis) decoders: codes -> E4M3 weight tiles
// Every mbarrier wait is bounded; a timeout records an error in
// chunks.header[4] and the role leaves its loop, so the kernel always ends.

#include <cuda.h>

#include <atomic>
#include <cstring>
#include <mutex>

#include "codec.cuh"
#include "mx_gemm.cuh"
#include "tensor_map.cuh"
#include "umma.cuh"

namespace exlr8 {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool encode_tiled_2d(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t inner, uint64_t rows,
                     uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t es[2] = {1, 1};
  return fn(map, type, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace {

template <int kK>
struct GemmTraits {
  static constexpr bool kTrellis = kK != 0;
  static constexpr int kStages = kTrellis ? 2 : 3;       // operand ring (weight image + activation planes)
  static constexpr int kCodeStages = kTrellis ? 4 : 0;   // trellis code ring, ahead of the decoders
  static constexpr int kDecoderWarps = kTrellis ? 16 : 0;
  static constexpr int kEpiWarps = kTrellis ? 4 : 8;    // a multiple of 4 (one per TMEM sub-partition)
  static constexpr int kCodeWarp = 2 + kEpiWarps;       // trellis code producer
  static constexpr int kThreads = 64 + 32 * kEpiWarps + (kTrellis ? 32 + 32 * kDecoderWarps : 0);
  static constexpr uint32_t kTileA = 128 * 128;          // one 128-row weight tile image
  static constexpr uint32_t kTileB = kMxMaxN * 128;      // one activation plane tile
  static constexpr uint32_t kTrellisTile = 32 * (kK > 0 ? kK : 1);  // bytes of one 16x16 trellis tile
  static constexpr uint32_t kCodeBytes = kTrellis ? 64 * kTrellisTile : 0;  // per accumulator and code stage
  static constexpr uint32_t kOffA0 = 0, kOffA1 = kTileA;
  static constexpr uint32_t kOffBhi = 2 * kTileA, kOffBlo = 2 * kTileA + kTileB;
  static constexpr uint32_t kOffSfa = 2 * kTileA + 2 * kTileB;  // 2 x 512 (MXFP4)
  static constexpr uint32_t kOffSfb = kOffSfa + 1024;           // 2 x 512
  static constexpr uint32_t kStageBytes = (kOffSfb + 1024 + 1023) / 1024 * 1024;
  static constexpr uint32_t kCodeStageBytes = 2 * kCodeBytes;
  static constexpr uint32_t kSmemBytes =
      kStages * kStageBytes + kCodeStages * kCodeStageBytes + 1024 + (kTrellis ? 512 : 0);
};

constexpr int kSchedSlots = 4;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemAcc1 = 256, kTmemSfa = 496, kTmemSfb = 504;

enum : int { kErrSched = 1, kErrStage = 2, kErrFull = 3, kErrAcc = 4, kErrAccEmpty = 5, kErrDrain = 6, kErrCodes = 7 };

struct GemmMaps {
  CUtensorMap w;      // MXFP4 weights
  CUtensorMap hi[2];  // activation planes per projection
  CUtensorMap lo[2];
};

template <int kStages, int kCodeStages>
struct GemmShared {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t codes_full[kCodeStages > 0 ? kCodeStages : 1];
  uint64_t codes_empty[kCodeStages > 0 ? kCodeStages : 1];
  uint64_t acc_full;
  uint64_t acc_empty;
  uint64_t sched_full[kSchedSlots];
  uint64_t sched_empty[kSchedSlots];
  uint64_t drain;
  int sched[kSchedSlots];
  int stop[kCodeStages > 0 ? kCodeStages : 1];
  int two[kCodeStages > 0 ? kCodeStages : 1];  // the code stage's unit uses accumulator 1
  uint32_t tmem;
};

__device__ __forceinline__ void record_error(int32_t* header, int code) { atomicCAS(&header[4], 0, code); }

struct UnitInfo {
  int proj, chunk, block, expert, start, rows, n16;
  bool two;  // accumulator 1 holds rows of the matrix (false for a last half block)
};

__device__ __forceinline__ UnitInfo unit_info(const ExpertGemmArgs& g, int unit, int blocks, int per_proj) {
  const MxChunks& c = g.chunks;
  UnitInfo u;
  u.proj = unit / per_proj;
  const int r = unit % per_proj;
  u.chunk = r / blocks;
  u.block = r % blocks;
  u.expert = c.chunk_expert[u.chunk];
  u.start = c.chunk_start[u.chunk];
  u.rows = c.chunk_rows[u.chunk];
  u.n16 = (u.rows + 15) & ~15;
  u.two = g.paired || 256 * u.block + 128 < g.out_features;
  return u;
}

// First output row, within the projection's expert matrix, of accumulator a.
__device__ __forceinline__ int acc_row(const ExpertGemmArgs& g, const UnitInfo& u, int a) {
  if (g.paired) return (a ? g.out_features / 2 : 0) + 128 * u.block;
  return 256 * u.block + 128 * a;
}

// E4M3 pair of two hashed products (low byte = a), the exact value of the
// codewords (fast_decode_common.metal:4-26 exlr8_decode2).
__device__ __forceinline__ uint32_t e4m3_pair_from_products(uint32_t pa, uint32_t pb, uint32_t mask, uint32_t xorv) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f16x2 %0, %1;" : "=h"(r) : "r"(hashed_pair_sum(pa, pb, mask, xorv)));
  return r;
}

// Decode one 16x16 tile (k rows tk, o cols tn of the 128x128 block) into
// the SW128 E4M3 image of the weight tile A[o][k]: lane l = 4g + t writes
// A[g][2t..2t+1], A[g+8][2t..], A[g][2t+8..], A[g+8][2t+8..] (the trellis
// lane/slot -> (row, col) map of trellis.py:97-99).
// The high codeword of each window is a plain shift (a 32-bit multiply-high
// runs well below the half rate of the other integer operations on B200).
template <int kK>
__device__ __forceinline__ void decode_tile(const uint32_t* __restrict__ tile, uint8_t* __restrict__ a_img, int tk,
                                            int tn, int lane, uint32_t mask, uint32_t xorv,
                                            const GenericGeometry& geo) {
  uint32_t p[4];
  if constexpr (kK == 4) {
    const uint32_t word = tile[lane], prior = tile[(lane + 31) & 31];
    const uint32_t v0 = word, v4 = __funnelshift_r(word, prior, 4);
    const uint32_t v8 = __funnelshift_r(word, prior, 8), v12 = __funnelshift_r(word, prior, 12);
    const uint32_t ph0 = (v0 >> 16) * kMcgMul, ph4 = (v4 >> 16) * kMcgMul;
    const uint32_t ph8 = (v8 >> 16) * kMcgMul, ph12 = (v12 >> 16) * kMcgMul;
    // Low codeword's product: v * C minus the high codeword's product * 2^16.
    const uint32_t pl0 = v0 * kMcgMul + ph0 * 0xFFFF0000u, pl4 = v4 * kMcgMul + ph4 * 0xFFFF0000u;
    const uint32_t pl8 = v8 * kMcgMul + ph8 * 0xFFFF0000u, pl12 = v12 * kMcgMul + ph12 * 0xFFFF0000u;
    p[0] = e4m3_pair_from_products(ph12, ph8, mask, xorv);  // codewords 0, 1
    p[1] = e4m3_pair_from_products(pl12, pl8, mask, xorv);  // 4, 5
    p[2] = e4m3_pair_from_products(ph4, ph0, mask, xorv);   // 2, 3
    p[3] = e4m3_pair_from_products(pl4, pl0, mask, xorv);   // 6, 7
  } else {
    uint32_t cw[8];
    generic_codewords(tile, kK, geo, cw);
    p[0] = e4m3_pair_from_products(cw[0] * kMcgMul, cw[1] * kMcgMul, mask, xorv);
    p[1] = e4m3_pair_from_products(cw[4] * kMcgMul, cw[5] * kMcgMul, mask, xorv);
    p[2] = e4m3_pair_from_products(cw[2] * kMcgMul, cw[3] * kMcgMul, mask, xorv);
    p[3] = e4m3_pair_from_products(cw[6] * kMcgMul, cw[7] * kMcgMul, mask, xorv);
  }
  const int gq = lane >> 2, t = lane & 3;
  const int r0 = tn * 16 + gq;
  const uint32_t chunk = static_cast<uint32_t>((tk ^ gq) << 4);  // (r & 7) == gq for r0 and r0 + 8
  uint8_t* row0 = a_img + r0 * 128 + chunk + 2 * t;
  uint8_t* row1 = row0 + 8 * 128;
  *reinterpret_cast<uint16_t*>(row0) = static_cast<uint16_t>(p[0]);
  *reinterpret_cast<uint16_t*>(row1) = static_cast<uint16_t>(p[1]);
  *reinterpret_cast<uint16_t*>(row0 + 8) = static_cast<uint16_t>(p[2]);
  *reinterpret_cast<uint16_t*>(row1 + 8) = static_cast<uint16_t>(p[3]);
}

// Byte offset of the 128x128 code block (expert e, 128-row output block nb,
// 128-value input block kt): 64 consecutive tiles for either storage side
// (tile index formulas of fast_decode_linear.metal:91-95).
__device__ __forceinline__ int64_t code_block_offset(int64_t e, int nb, int kt, int in_features, int out_features,
                                                     int side, uint32_t tile_bytes) {
  const int64_t it = in_features / 16, ot = out_features / 16;
  int64_t tile;
  if (side == 2) tile = ((e * it / 8 + kt) * (ot / 8) + nb) * 64;
  else tile = ((e * ot / 8 + nb) * it + static_cast<int64_t>(kt) * 8) * 8;
  return tile * tile_bytes;
}

template <int kK>
__global__ void __launch_bounds__(GemmTraits<kK>::kThreads, 1)
    expert_gemm_kernel(const __grid_constant__ GemmMaps maps, const ExpertGemmArgs g) {
  using T = GemmTraits<kK>;
  constexpr int kStages = T::kStages, kCodeStages = T::kCodeStages;
  extern __shared__ uint8_t smem_raw[];
  __shared__ GemmShared<kStages, kCodeStages> sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Offsetting the shared array itself (not an integer round trip) keeps the
  // pointer in the shared window: the stage accesses compile to shared loads
  // and stores.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* code_ring = smem + kStages * T::kStageBytes;
  uint8_t* unit_scales = code_ring + kCodeStages * T::kCodeStageBytes;  // trellis: 512 bytes of E8M0 1.0
  int32_t* header = g.chunks.header;
  const int blocks = g.paired ? g.out_features / 256 : (g.out_features + 255) / 256;
  const int ktiles = g.in_features / kMxKTile;
  const int kblocks = g.in_features / 32;

  // Zero the operand stages once: the gap bytes of E2M1 images are never
  // written by the TMA and must read as zero.
  for (uint32_t i = threadIdx.x; i < kStages * T::kStageBytes / 16; i += T::kThreads)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  if constexpr (T::kTrellis) {
    for (uint32_t i = threadIdx.x; i < 512 / 16; i += T::kThreads)
      reinterpret_cast<uint4*>(unit_scales)[i] = make_uint4(0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sh.full[s], 1 + T::kDecoderWarps);
      mbar_init(&sh.empty[s], 1);
    }
    for (int c = 0; c < kCodeStages; ++c) {
      mbar_init(&sh.codes_full[c], 1);
      mbar_init(&sh.codes_empty[c], T::kDecoderWarps);
      sh.stop[c] = 0;
      sh.two[c] = 1;
    }
    mbar_init(&sh.acc_full, 1);
    mbar_init(&sh.acc_empty, T::kEpiWarps);
    for (int i = 0; i < kSchedSlots; ++i) {
      mbar_init(&sh.sched_full[i], 1);
      mbar_init(&sh.sched_empty[i], 1 + T::kEpiWarps + (T::kTrellis ? 1 : 0));
    }
    mbar_init(&sh.drain, 1);
    mbar_fence_init();
    if constexpr (!T::kTrellis) prefetch_tensor_map(&maps.w);
    for (int p = 0; p < g.projections; ++p) {
      prefetch_tensor_map(&maps.hi[p]);
      prefetch_tensor_map(&maps.lo[p]);
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (warp == 1) tmem_alloc(&sh.tmem, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem;
  const int per_proj = g.chunks.header[0] * blocks;
  const int total = per_proj * g.projections;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- scheduler + operand producer ----------------
      uint32_t use = 0;  // stage uses issued
      bool failed = false;
      for (int i = 0;; ++i) {
        int unit = failed ? -1 : atomicAdd(&header[g.counter_index], 1);
        if (unit >= total) unit = -1;
        const int slot = i % kSchedSlots;
        if (i >= kSchedSlots && !mbar_wait(&sh.sched_empty[slot], ((i / kSchedSlots) - 1) & 1)) {
          record_error(header, kErrSched);
          break;
        }
        sh.sched[slot] = unit;
        mbar_arrive(&sh.sched_full[slot]);
        if (unit < 0) break;
        const UnitInfo u = unit_info(g, unit, blocks, per_proj);
        const int64_t w0 = static_cast<int64_t>(u.expert) * g.out_features + acc_row(g, u, 0);
        const int64_t w1 = static_cast<int64_t>(u.expert) * g.out_features + acc_row(g, u, 1);
        const int nb = (u.n16 + 127) / 128;
        const uint32_t na = u.two ? 2u : 1u;
        const uint32_t bytes = (T::kTrellis ? 0u : na * (128 * 64 + 512)) + 2 * u.n16 * 128 + nb * 512;
        const CUtensorMap* hmap = &maps.hi[u.proj];
        const CUtensorMap* lmap = &maps.lo[u.proj];
        const uint8_t* xs = g.x_scales[u.proj];
        for (int kt = 0; kt < ktiles; ++kt, ++use) {
          const int s = use % kStages;
          if (use >= kStages && !mbar_wait(&sh.empty[s], ((use / kStages) - 1) & 1)) {
            record_error(header, kErrStage);
            failed = true;
            break;
          }
          uint8_t* st = smem + s * T::kStageBytes;
          mbar_arrive_expect_tx(&sh.full[s], bytes);
          if constexpr (!T::kTrellis) {
            const uint8_t* wsc = g.weight_scales[u.proj];
            tma_load_2d(st + T::kOffA0, &maps.w, kt * kMxKTile, static_cast<int>(w0), &sh.full[s]);
            bulk_copy_g2s(st + T::kOffSfa, wsc + mx_scale_offset(w0, 4 * kt, kblocks), 512, &sh.full[s]);
            if (u.two) {
              tma_load_2d(st + T::kOffA1, &maps.w, kt * kMxKTile, static_cast<int>(w1), &sh.full[s]);
              bulk_copy_g2s(st + T::kOffSfa + 512, wsc + mx_scale_offset(w1, 4 * kt, kblocks), 512, &sh.full[s]);
            }
          }
          for (int r = 0; r < u.n16; r += 16) {
            tma_load_2d(st + T::kOffBhi + r * 128, hmap, kt * kMxKTile, u.start + r, &sh.full[s]);
            tma_load_2d(st + T::kOffBlo + r * 128, lmap, kt * kMxKTile, u.start + r, &sh.full[s]);
          }
          for (int b = 0; b < nb; ++b)
            bulk_copy_g2s(st + T::kOffSfb + b * 512, xs + mx_scale_offset(u.start + 128 * b, 4 * kt, kblocks), 512,
                          &sh.full[s]);
        }
        if (failed) continue;  // the next iteration publishes the stop marker
      }
      // Wait for the copies still in flight before the CTA can exit.
      for (uint32_t k = 0; k < static_cast<uint32_t>(kStages) && k < use; ++k) {
        const uint32_t last = use - 1 - k;
        if (!mbar_wait(&sh.full[last % kStages], (last / kStages) & 1)) record_error(header, kErrDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      if constexpr (T::kTrellis) {
        tc_copy_scales(tmem + kTmemSfa, umma_desc_rows16(smem_u32(unit_scales)));
        tc_copy_scales(tmem + kTmemSfa + 4, umma_desc_rows16(smem_u32(unit_scales)));
      }
      uint32_t use = 0;
      for (int j = 0;; ++j) {
        const int slot = j % kSchedSlots;
        if (!mbar_wait(&sh.sched_full[slot], (j / kSchedSlots) & 1)) {
          record_error(header, kErrSched);
          break;
        }
        const int unit = sh.sched[slot];
        mbar_arrive(&sh.sched_empty[slot]);
        if (unit < 0) break;
        const UnitInfo u = unit_info(g, unit, blocks, per_proj);
        if (j >= 1 && !mbar_wait(&sh.acc_empty, (j - 1) & 1)) {
          record_error(header, kErrAccEmpty);
          break;
        }
        tc_fence_after();
        const uint32_t idesc = mx_idesc(T::kTrellis ? kFmtE4M3 : kFmtE2M1, kFmtE4M3, u.n16);
        const int nb = (u.n16 + 127) / 128;
        bool ok = true;
        for (int kt = 0; kt < ktiles; ++kt, ++use) {
          const int s = use % kStages;
          if (!mbar_wait(&sh.full[s], (use / kStages) & 1)) {
            record_error(header, kErrFull);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(smem + s * T::kStageBytes);
          if constexpr (!T::kTrellis) {
            tc_copy_scales(tmem + kTmemSfa, umma_desc_rows16(st + T::kOffSfa));
            if (u.two) tc_copy_scales(tmem + kTmemSfa + 4, umma_desc_rows16(st + T::kOffSfa + 512));
          }
          for (int b = 0; b < nb; ++b)
            tc_copy_scales(tmem + kTmemSfb + 4 * b, umma_desc_rows16(st + T::kOffSfb + 512 * b));
#pragma unroll
          for (int a = 0; a < 2; ++a) {
            if (a == 1 && !u.two) break;
#pragma unroll
            for (int t = 0; t < 2; ++t) {
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const uint32_t id = idesc | (static_cast<uint32_t>(kk) << 4) | (static_cast<uint32_t>(kk) << 29);
                const uint64_t da = umma_desc_sw128(st + (a ? T::kOffA1 : T::kOffA0) + kk * 32);
                const uint64_t db = umma_desc_sw128(st + (t ? T::kOffBlo : T::kOffBhi) + kk * 32);
                tc_mma_mx(tmem + a * kTmemAcc1, da, db, id,
                          (tmem + kTmemSfa + 4 * a) | (static_cast<uint32_t>(kk) << 30),
                          (tmem + kTmemSfb) | (static_cast<uint32_t>(kk) << 30), (kt | t | kk) != 0);
              }
            }
          }
          tc_commit(&sh.empty[s]);
        }
        if (!ok) break;
        tc_commit(&sh.acc_full);
      }
      tc_commit(&sh.drain);
      if (!mbar_wait(&sh.drain, 0)) record_error(header, kErrDrain);
    }
  } else if (warp < 2 + T::kEpiWarps) {
    // ---------------- epilogue ----------------
    constexpr int kParts = T::kEpiWarps / 4;
    const int quad = warp & 3;         // TMEM sub-partition this warp may read
    const int part = (warp - 2) >> 2;  // its 16-column groups: part, part + kParts, ...
    for (int j = 0;; ++j) {
      const int slot = j % kSchedSlots;
      if (!mbar_wait(&sh.sched_full[slot], (j / kSchedSlots) & 1)) {
        if (lane == 0) record_error(header, kErrSched);
        break;
      }
      const int unit = sh.sched[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.sched_empty[slot]);
      if (unit < 0) break;
      const UnitInfo u = unit_info(g, unit, blocks, per_proj);
      if (!mbar_wait(&sh.acc_full, j & 1)) {
        if (lane == 0) record_error(header, kErrAcc);
        break;
      }
      tc_fence_after();
      const int64_t base = static_cast<int64_t>(u.proj) * g.proj_offset + 32 * quad + lane;
      float* dst0 = g.out + static_cast<int64_t>(u.start) * g.out_stride + base + acc_row(g, u, 0);
      float* dst1 = g.out + static_cast<int64_t>(u.start) * g.out_stride + base + acc_row(g, u, 1);
      const uint32_t lane_addr = tmem + (static_cast<uint32_t>(32 * quad) << 16);
#pragma unroll 1
      for (int c0 = 16 * part; c0 < u.n16; c0 += 16 * kParts) {
        // Both accumulators' 16 columns in flight before one wait.
        uint32_t v0[16], v1[16];
        tc_ld16(lane_addr + c0, v0);
        if (u.two) tc_ld16(lane_addr + kTmemAcc1 + c0, v1);
        tc_wait_ld();
        const int n = min(16, u.rows - c0);
#pragma unroll
        for (int c = 0; c < 16; ++c)
          if (c < n) dst0[static_cast<int64_t>(c0 + c) * g.out_stride] = __uint_as_float(v0[c]);
        if (u.two) {
#pragma unroll
          for (int c = 0; c < 16; ++c)
            if (c < n) dst1[static_cast<int64_t>(c0 + c) * g.out_stride] = __uint_as_float(v1[c]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.acc_empty);
    }
  } else if constexpr (T::kTrellis) {
    if (warp == T::kCodeWarp) {
      if (lane == 0) {
        // ---------------- code producer (trellis) ----------------
        uint32_t cuse = 0;
        for (int j = 0;; ++j) {
          const int slot = j % kSchedSlots;
          if (!mbar_wait(&sh.sched_full[slot], (j / kSchedSlots) & 1)) {
            record_error(header, kErrSched);
            break;
          }
          const int unit = sh.sched[slot];
          mbar_arrive(&sh.sched_empty[slot]);
          if (unit < 0) break;
          const UnitInfo u = unit_info(g, unit, blocks, per_proj);
          const uint8_t* codes = static_cast<const uint8_t*>(g.weights[u.proj]);
          const int nb0 = acc_row(g, u, 0) / 128, nb1 = acc_row(g, u, 1) / 128;
          bool ok = true;
          for (int kt = 0; kt < ktiles; ++kt, ++cuse) {
            const int c = cuse % kCodeStages;
            if (cuse >= static_cast<uint32_t>(kCodeStages) &&
                !mbar_wait(&sh.codes_empty[c], ((cuse / kCodeStages) - 1) & 1)) {
              record_error(header, kErrCodes);
              ok = false;
              break;
            }
            uint8_t* dst = code_ring + c * T::kCodeStageBytes;
            sh.two[c] = u.two;
            mbar_arrive_expect_tx(&sh.codes_full[c], (u.two ? 2u : 1u) * T::kCodeBytes);
            bulk_copy_g2s(dst, codes + code_block_offset(u.expert, nb0, kt, g.in_features, g.out_features, g.side,
                                                         T::kTrellisTile),
                          T::kCodeBytes, &sh.codes_full[c]);
            if (u.two)
              bulk_copy_g2s(dst + T::kCodeBytes,
                            codes + code_block_offset(u.expert, nb1, kt, g.in_features, g.out_features, g.side,
                                                      T::kTrellisTile),
                            T::kCodeBytes, &sh.codes_full[c]);
          }
          if (!ok) break;
        }
        // Copies in flight land before the CTA exits.  (This comes before the
        // stop marker: the marker completes one more phase of a codes_full
        // barrier, after which the parity of the use four back on that stage
        // would read as pending again.)
        for (uint32_t k = 1; k <= static_cast<uint32_t>(kCodeStages) && k <= cuse; ++k) {
          const uint32_t last = cuse - k;
          if (!mbar_wait(&sh.codes_full[last % kCodeStages], (last / kCodeStages) & 1))
            record_error(header, kErrDrain);
        }
        // Stop marker for the decoders on the next code stage.
        const int c = cuse % kCodeStages;
        if (cuse < static_cast<uint32_t>(kCodeStages) ||
            mbar_wait(&sh.codes_empty[c], ((cuse / kCodeStages) - 1) & 1)) {
          sh.stop[c] = 1;
          mbar_arrive(&sh.codes_full[c]);
        } else {
          record_error(header, kErrCodes);
        }
      }
    } else {
      // ---------------- decoders (warps 7-22) ----------------
      // Warp d decodes tile column d % 8 of accumulator d / 8.
      const int dw = warp - (T::kCodeWarp + 1);
      const int tn = dw & 7, acc = dw >> 3;
      const GenericGeometry geo = generic_geometry(kK == 4 ? 3 : kK, lane);
      const uint32_t mask = g.mcg_mask, xorv = g.mcg_xor;
      for (uint32_t use = 0;; ++use) {
        const int c = use % kCodeStages, s = use % kStages;
        if (!mbar_wait(&sh.codes_full[c], (use / kCodeStages) & 1)) {
          if (lane == 0) record_error(header, kErrCodes);
          break;
        }
        if (sh.stop[c]) break;
        // The operand stage is free once the MMAs of its previous use finished.
        if (use >= static_cast<uint32_t>(kStages) && !mbar_wait(&sh.empty[s], ((use / kStages) - 1) & 1)) {
          if (lane == 0) record_error(header, kErrStage);
          break;
        }
        uint8_t* st = smem + s * T::kStageBytes;
        if (acc == 0 || sh.two[c]) {
          const uint32_t* codes =
              reinterpret_cast<const uint32_t*>(code_ring + c * T::kCodeStageBytes + acc * T::kCodeBytes);
          uint8_t* img = st + (acc ? T::kOffA1 : T::kOffA0);
#pragma unroll 4
          for (int tk = 0; tk < 8; ++tk)
            decode_tile<kK>(codes + (tk * 8 + tn) * (T::kTrellisTile / 4), img, tk, tn, lane, mask, xorv,
                            geo);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sh.codes_empty[c]);
          mbar_arrive(&sh.full[s]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_free(tmem, kTmemCols);
}

// ---------------------------------------------------------------------------
// MXFP4 on an SM pair (cta_group::2).  A pair unit is (chunk, pair block):
// CTA r of the two-CTA cluster owns weight block 2 * pair_block + r (two
// accumulators of 128 rows, as in the one-SM kernel) and stages half of the
// chunk's activation rows (B columns r * N/2 ...); one M = 256 MMA covers
// both CTAs' rows.  Against the one-SM kernel each CTA stages half the
// activation bytes per K step, so four stages fit instead of three, and the
// tensor core reads half of B from each SM's shared memory.  The even CTA's
// producer takes pair units from the launch's global counter and hands each
// to both CTAs through a small ring (a remote shared store plus a remote
// arrive for the odd CTA), so pairs stay balanced however uneven the chunks.
//
//   warp 0      producer (each CTA): its weight tiles and scales, its half
//               of both activation planes and the activation scales, all
//               counted on the even CTA's full barrier; the even CTA's also
//               schedules
//   warp 1      MMA issuer (even CTA), TMEM owner (both)
//   warps 2-17  epilogue (each CTA): its TMEM -> float32 rows of `out`
// Every wait is bounded as in the one-SM kernel; the CTAs leave together
// through a cluster barrier, after every copy and commit that targets the
// other CTA has landed.
// ---------------------------------------------------------------------------
struct PairTraits {
  static constexpr int kStages = 4;
  static constexpr int kEpiWarps = 16;  // four per TMEM sub-partition: the accumulators drain in a quarter of the time
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr uint32_t kTileA = 128 * 128;
  static constexpr uint32_t kTileB = (kMxMaxN / 2) * 128;  // this CTA's half of a plane
  static constexpr uint32_t kOffA0 = 0, kOffA1 = kTileA;
  static constexpr uint32_t kOffBhi = 2 * kTileA, kOffBlo = 2 * kTileA + kTileB;
  static constexpr uint32_t kOffSfa = 2 * kTileA + 2 * kTileB;  // 2 x 512
  static constexpr uint32_t kOffSfb = kOffSfa + 1024;           // 2 x 512 (N <= 160)
  static constexpr uint32_t kStageBytes = (kOffSfb + 1024 + 1023) / 1024 * 1024;
  static constexpr uint32_t kSmemBytes = kStages * kStageBytes + 1024;
};
static_assert(PairTraits::kOffBlo % 1024 == 0 && PairTraits::kOffBhi % 1024 == 0, "SW128 tiles start on 1 KB");
static_assert(PairTraits::kSmemBytes + 256 <= 232448, "pair stages exceed shared memory");

struct PairMaps {
  CUtensorMap w;       // E2M1 weights, box 128 rows x 128 values
  CUtensorMap wsc;     // weight scale blocks viewed as [blocks][256] u16, box one 512-byte block
  CUtensorMap hi, lo;  // activation planes, box 8 rows x 128 values
  CUtensorMap xsc;     // activation scale blocks, as wsc
};

struct PairShared {
  uint64_t full[PairTraits::kStages];   // even CTA: both CTAs' bytes of a stage
  uint64_t empty[PairTraits::kStages];  // each CTA: its stage may be refilled
  uint64_t acc_full;                    // each CTA: its accumulators hold a unit
  uint64_t acc_empty;                   // even CTA: both CTAs' epilogues drained them
  uint64_t sched_full[kSchedSlots];     // each CTA: sched[slot] holds the next unit
  uint64_t sched_empty[kSchedSlots];    // even CTA: every reader of the slot in both CTAs is done
  uint64_t drain;
  int sched[kSchedSlots];               // pair unit, -1 = no more
  uint32_t tmem;
};

// Readers of a schedule slot, all counted on the even CTA's sched_empty: its
// MMA issuer and epilogue warps, the odd CTA's producer and epilogue warps.
constexpr int kPairSchedReaders = 2 + 2 * PairTraits::kEpiWarps;

// Next pair unit of this CTA's reader number j: waits for slot j % kSchedSlots
// (acquire at cluster scope: the even CTA wrote it) and reads it.  Returns
// -2 on timeout.
__device__ __forceinline__ int pair_sched_take(PairShared& sh, int j) {
  const int slot = j % kSchedSlots;
  if (!mbar_wait_cluster(&sh.sched_full[slot], (j / kSchedSlots) & 1)) return -2;
  return static_cast<volatile int*>(sh.sched)[slot];
}

// Releases slot j % kSchedSlots (one arrival on the even CTA's sched_empty).
__device__ __forceinline__ void pair_sched_release(PairShared& sh, int j) {
  mbar_arrive_cluster(cluster_addr(smem_u32(&sh.sched_empty[j % kSchedSlots]), 0));
}

__device__ __forceinline__ UnitInfo pair_unit(const ExpertGemmArgs& g, int unit, int pair_blocks, uint32_t rank) {
  const MxChunks& c = g.chunks;
  UnitInfo u;
  u.proj = 0;
  u.chunk = unit / pair_blocks;
  u.block = 2 * (unit % pair_blocks) + static_cast<int>(rank);
  u.expert = c.chunk_expert[u.chunk];
  u.start = c.chunk_start[u.chunk];
  u.rows = c.chunk_rows[u.chunk];
  u.n16 = (u.rows + 15) & ~15;
  u.two = true;
  return u;
}

__global__ void __launch_bounds__(PairTraits::kThreads, 1)
    expert_gemm_pair_kernel(const __grid_constant__ PairMaps maps, const ExpertGemmArgs g) {
  using T = PairTraits;
  constexpr int kStages = T::kStages;
  extern __shared__ uint8_t smem_raw[];
  __shared__ PairShared sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  int32_t* header = g.chunks.header;
  const uint32_t rank = cluster_rank();
  const int pair_blocks = g.out_features / 512;
  const int ktiles = g.in_features / kMxKTile;
  const int kb4 = g.in_features / kMxKTile;  // 512-byte scale blocks per 128 rows
  const int total = header[0] * pair_blocks;

  for (uint32_t i = threadIdx.x; i < kStages * T::kStageBytes / 16; i += T::kThreads)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    mbar_init(&sh.acc_full, 1);
    mbar_init(&sh.acc_empty, 2 * T::kEpiWarps);
    for (int i = 0; i < kSchedSlots; ++i) {
      mbar_init(&sh.sched_full[i], 1);
      mbar_init(&sh.sched_empty[i], kPairSchedReaders);
    }
    mbar_init(&sh.drain, 1);
    mbar_fence_init();
    prefetch_tensor_map(&maps.w);
    prefetch_tensor_map(&maps.wsc);
    prefetch_tensor_map(&maps.hi);
    prefetch_tensor_map(&maps.lo);
    prefetch_tensor_map(&maps.xsc);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (warp == 1) tmem_alloc2(&sh.tmem, kTmemCols);
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem = sh.tmem;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer (each CTA; the even one schedules) ----------------
      uint32_t use = 0;
      bool failed = false;
      for (int i = 0; !failed; ++i) {
        int unit;
        if (rank == 0) {
          unit = atomicAdd(&header[g.counter_index], 1);
          if (unit >= total) unit = -1;
          const int slot = i % kSchedSlots;
          if (i >= kSchedSlots && !mbar_wait_cluster(&sh.sched_empty[slot], ((i / kSchedSlots) - 1) & 1)) {
            record_error(header, kErrSched);
            unit = -1;
            failed = true;
          }
          // This CTA's copy, then the odd CTA's (remote store, ordered before
          // the remote arrive by its release).
          sh.sched[slot] = unit;
          const uint32_t peer_slot = cluster_addr(smem_u32(&sh.sched[slot]), 1);
          asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer_slot), "r"(unit) : "memory");
          mbar_arrive(&sh.sched_full[slot]);
          mbar_arrive_cluster(cluster_addr(smem_u32(&sh.sched_full[slot]), 1));
        } else {
          unit = pair_sched_take(sh, i);
          if (unit == -2) {
            record_error(header, kErrSched);
            break;
          }
          pair_sched_release(sh, i);
        }
        if (unit < 0) break;
        const UnitInfo u = pair_unit(g, unit, pair_blocks, rank);
        const int64_t w0 = static_cast<int64_t>(u.expert) * g.out_features + acc_row(g, u, 0);
        const int64_t w1 = static_cast<int64_t>(u.expert) * g.out_features + acc_row(g, u, 1);
        const int half = u.n16 / 2, nb = (u.n16 + 127) / 128;
        // Bytes of one CTA; the even CTA expects both CTAs' (the same shape).
        const uint32_t bytes = 2 * (128 * 64 + 512) + 2 * half * 128 + nb * 512;
        const int row0 = u.start + static_cast<int>(rank) * half;
        for (int kt = 0; kt < ktiles; ++kt, ++use) {
          const int s = use % kStages;
          if (use >= kStages && !mbar_wait(&sh.empty[s], ((use / kStages) - 1) & 1)) {
            record_error(header, kErrStage);
            failed = true;
            break;
          }
          uint8_t* st = smem + s * T::kStageBytes;
          const uint32_t bar = cluster_addr(smem_u32(&sh.full[s]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&sh.full[s], 2 * bytes);
          tma2_load_2d(st + T::kOffA0, &maps.w, kt * kMxKTile, static_cast<int>(w0), bar);
          tma2_load_2d(st + T::kOffSfa, &maps.wsc, 0, static_cast<int>((w0 / 128) * kb4 + kt), bar);
          tma2_load_2d(st + T::kOffA1, &maps.w, kt * kMxKTile, static_cast<int>(w1), bar);
          tma2_load_2d(st + T::kOffSfa + 512, &maps.wsc, 0, static_cast<int>((w1 / 128) * kb4 + kt), bar);
          for (int r = 0; r < half; r += 8) {
            tma2_load_2d(st + T::kOffBhi + r * 128, &maps.hi, kt * kMxKTile, row0 + r, bar);
            tma2_load_2d(st + T::kOffBlo + r * 128, &maps.lo, kt * kMxKTile, row0 + r, bar);
          }
          for (int b = 0; b < nb; ++b)
            tma2_load_2d(st + T::kOffSfb + b * 512, &maps.xsc, 0, (u.start / 128 + b) * kb4 + kt, bar);
        }
      }
      // The MMA issuer's last commits to this CTA's stages (they follow the
      // MMAs, which followed both CTAs' copies of those stages).
      for (uint32_t k = 1; k <= static_cast<uint32_t>(kStages) && k <= use; ++k) {
        const uint32_t last = use - k;
        if (!mbar_wait(&sh.empty[last % kStages], (last / kStages) & 1)) record_error(header, kErrDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer (even CTA) ----------------
      uint32_t use = 0;
      for (int j = 0;; ++j) {
        const int unit = pair_sched_take(sh, j);
        if (unit == -2) {
          record_error(header, kErrSched);
          break;
        }
        pair_sched_release(sh, j);
        if (unit < 0) break;
        const UnitInfo u = pair_unit(g, unit, pair_blocks, rank);
        if (j >= 1 && !mbar_wait_cluster(&sh.acc_empty, (j - 1) & 1)) {
          record_error(header, kErrAccEmpty);
          break;
        }
        tc_fence_after();
        const uint32_t idesc = mx_idesc_pair(kFmtE2M1, kFmtE4M3, u.n16);
        const int nb = (u.n16 + 127) / 128;
        bool ok = true;
        for (int kt = 0; kt < ktiles; ++kt, ++use) {
          const int s = use % kStages;
          if (!mbar_wait(&sh.full[s], (use / kStages) & 1)) {
            record_error(header, kErrFull);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(smem + s * T::kStageBytes);
          tc2_copy_scales(tmem + kTmemSfa, umma_desc_rows16(st + T::kOffSfa));
          tc2_copy_scales(tmem + kTmemSfa + 4, umma_desc_rows16(st + T::kOffSfa + 512));
          for (int b = 0; b < nb; ++b)
            tc2_copy_scales(tmem + kTmemSfb + 4 * b, umma_desc_rows16(st + T::kOffSfb + 512 * b));
#pragma unroll
          for (int a = 0; a < 2; ++a) {
#pragma unroll
            for (int t = 0; t < 2; ++t) {
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const uint32_t id = idesc | (static_cast<uint32_t>(kk) << 4) | (static_cast<uint32_t>(kk) << 29);
                const uint64_t da = umma_desc_sw128(st + (a ? T::kOffA1 : T::kOffA0) + kk * 32);
                const uint64_t db = umma_desc_sw128(st + (t ? T::kOffBlo : T::kOffBhi) + kk * 32);
                tc2_mma_mx(tmem + a * kTmemAcc1, da, db, id,
                           (tmem + kTmemSfa + 4 * a) | (static_cast<uint32_t>(kk) << 30),
                           (tmem + kTmemSfb) | (static_cast<uint32_t>(kk) << 30), (kt | t | kk) != 0);
              }
            }
          }
          tc2_commit(cluster_addr(smem_u32(&sh.empty[s]), 0));
          tc2_commit(cluster_addr(smem_u32(&sh.empty[s]), 1));
        }
        if (!ok) break;
        tc2_commit(cluster_addr(smem_u32(&sh.acc_full), 0));
        tc2_commit(cluster_addr(smem_u32(&sh.acc_full), 1));
      }
      tc2_commit(cluster_addr(smem_u32(&sh.drain), 0));
      if (!mbar_wait(&sh.drain, 0)) record_error(header, kErrDrain);
    }
  } else {
    // ---------------- epilogue (each CTA, warps 2-17) ----------------
    constexpr int kParts = T::kEpiWarps / 4;
    const int quad = warp & 3;
    const int part = (warp - 2) >> 2;
    const uint32_t lead_acc_empty = cluster_addr(smem_u32(&sh.acc_empty), 0);
    for (int j = 0;; ++j) {
      const int unit = pair_sched_take(sh, j);
      __syncwarp();
      if (unit == -2) {
        if (lane == 0) record_error(header, kErrSched);
        break;
      }
      if (lane == 0) pair_sched_release(sh, j);
      if (unit < 0) break;
      const UnitInfo u = pair_unit(g, unit, pair_blocks, rank);
      if (!mbar_wait(&sh.acc_full, j & 1)) {
        if (lane == 0) record_error(header, kErrAcc);
        break;
      }
      tc_fence_after();
      const int64_t base = 32 * quad + lane;
      float* dst0 = g.out + static_cast<int64_t>(u.start) * g.out_stride + base + acc_row(g, u, 0);
      float* dst1 = g.out + static_cast<int64_t>(u.start) * g.out_stride + base + acc_row(g, u, 1);
      const uint32_t lane_addr = tmem + (static_cast<uint32_t>(32 * quad) << 16);
#pragma unroll 1
      for (int c0 = 16 * part; c0 < u.n16; c0 += 16 * kParts) {
        uint32_t v0[16], v1[16];
        tc_ld16(lane_addr + c0, v0);
        tc_ld16(lane_addr + kTmemAcc1 + c0, v1);
        tc_wait_ld();
        const int n = min(16, u.rows - c0);
#pragma unroll
        for (int c = 0; c < 16; ++c)
          if (c < n) dst0[static_cast<int64_t>(c0 + c) * g.out_stride] = __uint_as_float(v0[c]);
#pragma unroll
        for (int c = 0; c < 16; ++c)
          if (c < n) dst1[static_cast<int64_t>(c0 + c) * g.out_stride] = __uint_as_float(v1[c]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(lead_acc_empty);
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no copy, commit or arrive still targets the other CTA
  tc_fence_after();
  if (warp == 1) tmem_free2(tmem, kTmemCols);
}

bool encode_2d(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t inner, uint64_t rows,
               uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows) {
  return encode_tiled_2d(map, type, base, inner, rows, row_bytes, box_inner, box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

int sm_count_cached() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return sms;
}

template <int kK>
cudaError_t launch_variant(const ExpertGemmArgs& args, const GemmMaps& maps, cudaStream_t s) {
  using T = GemmTraits<kK>;
  static bool configured = false;
  if (!configured) {
    const cudaError_t err =
        cudaFuncSetAttribute(expert_gemm_kernel<kK>, cudaFuncAttributeMaxDynamicSharedMemorySize, T::kSmemBytes);
    if (err != cudaSuccess) return err;
    configured = true;
  }
  expert_gemm_kernel<kK><<<sm_count_cached(), T::kThreads, T::kSmemBytes, s>>>(maps, args);
  return cudaGetLastError();
}

// The SM-pair form for MXFP4 when the shape allows it: one projection,
// weight blocks in pairs (out_features a multiple of 512) and an even SM count.
bool pair_eligible(const ExpertGemmArgs& a) {
  return a.trellis_k == 0 && a.projections == 1 && a.out_features % 512 == 0 && a.in_features % kMxKTile == 0 &&
         sm_count_cached() % 2 == 0 && gemm_pair_enabled();
}

cudaError_t launch_pair(const ExpertGemmArgs& args, cudaStream_t s) {
  using T = PairTraits;
  PairMaps maps;
  memset(&maps, 0, sizeof(maps));
  const uint64_t wrows = static_cast<uint64_t>(args.experts) * args.out_features;
  const uint64_t kb4 = static_cast<uint64_t>(args.in_features) / kMxKTile;
  if (!encode_2d(&maps.w, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, args.weights[0], args.in_features, wrows,
                 args.in_features / 2, 128, 128) ||
      !encode_tiled_2d(&maps.wsc, CU_TENSOR_MAP_DATA_TYPE_UINT16, args.weight_scales[0], 256, wrows / 128 * kb4, 512,
                       256, 1, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !encode_2d(&maps.hi, CU_TENSOR_MAP_DATA_TYPE_UINT8, args.x_hi[0], args.in_features, args.padded_rows,
                 args.in_features, 128, 8) ||
      !encode_2d(&maps.lo, CU_TENSOR_MAP_DATA_TYPE_UINT8, args.x_lo[0], args.in_features, args.padded_rows,
                 args.in_features, 128, 8) ||
      !encode_tiled_2d(&maps.xsc, CU_TENSOR_MAP_DATA_TYPE_UINT16, args.x_scales[0], 256,
                       static_cast<uint64_t>(args.padded_rows) / 128 * kb4, 512, 256, 1, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  static bool configured = false;
  if (!configured) {
    const cudaError_t err = cudaFuncSetAttribute(expert_gemm_pair_kernel,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, T::kSmemBytes);
    if (err != cudaSuccess) return err;
    configured = true;
  }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(static_cast<unsigned>(sm_count_cached()));
  cfg.blockDim = dim3(T::kThreads);
  cfg.dynamicSmemBytes = T::kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, expert_gemm_pair_kernel, maps, args);
}

}  // namespace

static std::atomic<int> g_gemm_pair{1};

bool gemm_pair_enabled() { return g_gemm_pair.load(std::memory_order_relaxed) != 0; }

int set_gemm_pair(int enable) { return enable < 0 ? g_gemm_pair.load() : g_gemm_pair.exchange(enable != 0 ? 1 : 0); }

cudaError_t launch_expert_gemm(const ExpertGemmArgs& args, cudaStream_t s) {
  if (pair_eligible(args)) return launch_pair(args, s);
  GemmMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (args.trellis_k == 0) {
    const uint64_t wrows = static_cast<uint64_t>(args.experts) * args.out_features;
    if (!encode_2d(&maps.w, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, args.weights[0], args.in_features, wrows,
                   args.in_features / 2, 128, 128))
      return cudaErrorInvalidValue;
  }
  for (int p = 0; p < args.projections; ++p) {
    if (!encode_2d(&maps.hi[p], CU_TENSOR_MAP_DATA_TYPE_UINT8, args.x_hi[p], args.in_features, args.padded_rows,
                   args.in_features, 128, 16) ||
        !encode_2d(&maps.lo[p], CU_TENSOR_MAP_DATA_TYPE_UINT8, args.x_lo[p], args.in_features, args.padded_rows,
                   args.in_features, 128, 16))
      return cudaErrorInvalidValue;
  }
  switch (args.trellis_k) {
    case 0: return launch_variant<0>(args, maps, s);
    case 3: return launch_variant<3>(args, maps, s);
    case 4: return launch_variant<4>(args, maps, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace exlr8
