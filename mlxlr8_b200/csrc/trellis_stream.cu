// Streaming trellis GEMV for selected experts (decode / small batches).
//
// Replaces metal/fast_decode_linear.metal (exlr8 v0.1.21).  One persistent
// CTA per SM slot; warp 4 is the producer, warps 0-3 consume.
//
//   producer: takes work units (row group of one expert, projection, 128-wide
//     output block, K split) from a global counter and streams each unit's
//     packed tiles -- one contiguous run of 8 output tiles per K tile -- plus
//     the unit rows' activation fragment records (one per 128-wide K block,
//     with the block's unscale) into a ring of shared-memory stages with 1-D
//     bulk copies (cp.async.bulk, no multicast) completing on mbarriers.  A
//     stage is one 128-wide K block.  Units follow each other through the
//     ring without draining.
//   consumers: each of the eight warps owns one of the eight 16x16 output
//     tiles and takes the stage's 8 K tiles at once (eight independent decode
//     chains per warp).  A lane reads word l and word l-1 of a tile; every 32-bit window
//     of that 64-bit stream carries two codewords, whose hashes come from three
//     integer multiplies (V*C, (V>>16)*C and V*C - ((V>>16)*C << 16)), so the
//     codeword masks disappear.  The half sums are rounded to E4M3 and placed
//     directly in mma.sync m16n8k16 A fragments (the trellis tensor-core
//     permutation is that layout); B holds float16 hi/lo pieces of up to four
//     rows (eight columns) per fragment group; each stage's float32 products
//     are added into the unit's accumulators times the block's unscale.
//   static cache: a unit whose expert is cached (StreamParams::hot) streams
//     the expert's exact E4M3 bytes instead, kHotTiles K tiles per stage, and
//     its consumers convert them into the same A fragments (bit-equal).
//   output: per unit, float32 partial sums [proj][slot][split][out].
//   dense warp (warp 9): the bf16 shared expert's rows (stream.cuh
//   DenseUnits, dense_stream.cuh), streamed beside the trellis units.

#include "codec.cuh"
#include "stream_codec.cuh"
#include "common.cuh"
#include "dense_stream.cuh"
#include "launch.cuh"
#include "stream.cuh"
#include "tma.cuh"
#include "tensor_map.cuh"

namespace exlr8 {

constexpr int kConsumers = 8;
constexpr int kProducerWarp = kConsumers;
constexpr int kDenseWarp = kConsumers + 1;
constexpr int kStreamThreads = (kConsumers + 2) * 32;
constexpr int kStages = 4;
constexpr int kPlanCache = 160;  // plan groups / slots cached in shared memory (decode: <= 144 slots)
constexpr int kStageTiles = 8;                       // K tiles per stage
constexpr int kFragRowBytes = kStageTiles * 64 + 64;  // padded: rows hit different banks
static_assert(kFragRowBytes >= kFragBlockBytes, "a fragment record fits its stage row");

// kHot: a stage of static-cache bytes covering kHotTiles K tiles; kBlockStart
// / kBlockEnd: the stage opens / closes its 128-wide K block (code stages do
// both).
enum : int { kFirst = 1, kLast = 2, kEnd = 4, kHot = 8, kBlockStart = 16, kBlockEnd = 32 };

template <int K>
struct StageGeometry {
  static constexpr int kTileWords = 8 * K;
  static constexpr int kCodeBytes = kStageTiles * 8 * kTileWords * 4;
  static constexpr int kFragBytes = kMaxGroupRows * kFragRowBytes;
  static constexpr int kStageBytes = kCodeBytes + kFragBytes;
  static constexpr int kRingBytes = kStages * kStageBytes;
  static constexpr int kSmemBytes = kRingBytes + kDenseSmemBytes;  // ring, then the dense warp's buffers
  // K tiles of static-cache bytes per stage (8 output tiles x 256 bytes per
  // K tile) that fit the code area: a power of two dividing kStageTiles.
  static constexpr int kHotTiles = kCodeBytes >= 4 * 8 * 256 ? 4 : 2;
  static_assert(kHotTiles * 8 * 256 <= kCodeBytes, "a hot stage fits the code area");
};

struct UnitInfo {
  int group, proj, nb, split;
};

// Unit indices stay below 2^31 (rows <= 2^20, projections <= 2, 128-wide
// output blocks <= 48 at GLM size, splits <= 16), so 32-bit arithmetic
// suffices; the producer decodes each unit once and passes its fields to
// the consumers through shared memory.
__device__ __forceinline__ UnitInfo decode_unit(uint32_t unit, const StreamParams& p, uint32_t nblocks) {
  UnitInfo u;
  const uint32_t splits = static_cast<uint32_t>(p.splits), projections = static_cast<uint32_t>(p.projections);
  const uint32_t a = unit / splits, b = a / nblocks;
  u.split = static_cast<int>(unit - a * splits);
  u.nb = static_cast<int>(a - b * nblocks);
  u.proj = static_cast<int>(b % projections);
  u.group = static_cast<int>(b / projections);
  return u;
}

template <int K>
__global__ void __launch_bounds__(kStreamThreads, 2) trellis_stream_kernel(const __grid_constant__ StreamParams p) {
  using G = StageGeometry<K>;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t full_bar[kStages];
  __shared__ __align__(8) uint64_t empty_bar[kStages];
  __shared__ int4 meta[kStages];  // unit, first K tile, K tiles, flags
  // First stage of a unit: [0] rows of the unit's group, [1 + r] slot of row r,
  // then the unit's projection, output block and split (the consumers read
  // the unit from here, not from the global plan).
  constexpr int kUnitProj = kMaxGroupRows + 1, kUnitBlock = kMaxGroupRows + 2, kUnitSplit = kMaxGroupRows + 3;
  __shared__ int unit_rows[kStages][kMaxGroupRows + 4];
  __shared__ __align__(8) uint64_t dense_bar[kDenseBuffers];
  __shared__ int plan_cache[4][kPlanCache];  // group expert, start, count; slot order (producer)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int it = p.in_features / 16, ot = p.out_features / 16, nblocks = ot / 8;
  pdl_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kConsumers);
    }
    for (int b = 0; b < kDenseBuffers; ++b) mbar_init(&dense_bar[b], 1);
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kDenseWarp) {
    // ---------------- dense warp ----------------
    // The gate/up launch's dense rows need nothing from the kernels before
    // it in the chain (stream.cuh DenseUnits::early): they stream while the
    // routing and the fragment prep finish.
    if (!p.dense.early) pdl_wait();
    if (p.dense.units > 0 && !dense_warp_run(p.dense, &p.dense_w0, &p.dense_w1, smem + G::kRingBytes, dense_bar, lane)) {
      if (lane == 0) atomicOr(&p.plan.header[9], 4);
      // Copies already issued target valid addresses and land within
      // microseconds; give them that time before this warp retires.
      for (int i = 0; i < 1000; ++i) __nanosleep(1000);
    }
    return;
  }

  pdl_wait();  // the plan, fragments and partial buffers belong to earlier kernels

  if (warp == kProducerWarp) {
    // ---------------- producer ----------------
    // The plan's groups and slot order (decode batches: at most kPlanCache of
    // each) are cached in shared memory by the whole warp, so that a unit
    // boundary costs no global round trip; larger plans are read in place.
    const int groups = p.plan.header[0];
    const bool cached = groups <= kPlanCache && p.nslots <= kPlanCache;
    if (cached) {
      for (int g = lane; g < groups; g += 32) {
        plan_cache[0][g] = p.plan.group_expert[g];
        plan_cache[1][g] = p.plan.group_start[g];
        plan_cache[2][g] = p.plan.group_count[g];
      }
      for (int i = lane; i < p.nslots; i += 32) plan_cache[3][i] = p.plan.order[i];
      __syncwarp();
    }
    if (lane != 0) return;
    const int64_t total = static_cast<int64_t>(groups) * p.projections * nblocks * p.splits;
    int stage = 0;
    uint32_t phase = 0;
    bool failed = false;
    // Each CTA's first unit is its index; later units come from the counter,
    // fetched one unit ahead so that the atomic's round trip overlaps the
    // current unit's stages.
    int64_t unit = blockIdx.x;
    for (;;) {
      const int64_t next = static_cast<int64_t>(gridDim.x) + atomicAdd(&p.plan.header[p.counter], 1);
      if (!mbar_wait(&empty_bar[stage], phase ^ 1u)) {
        failed = true;
        break;
      }
      if (unit >= total) {
        meta[stage] = make_int4(0, 0, 0, kEnd);
        mbar_arrive(&full_bar[stage]);
        break;
      }
      const UnitInfo u = decode_unit(static_cast<uint32_t>(unit), p, static_cast<uint32_t>(nblocks));
      const int expert = cached ? plan_cache[0][u.group] : p.plan.group_expert[u.group];
      const int start = cached ? plan_cache[1][u.group] : p.plan.group_start[u.group];
      const int nr = cached ? plan_cache[2][u.group] : p.plan.group_count[u.group];
      const int kt0 = u.split * p.kt_per_split;
      const int kt1 = min(kt0 + p.kt_per_split, it);
      const uint32_t* words = p.packed[u.proj];
      int slots[kMaxGroupRows];
#pragma unroll
      for (int r = 0; r < kMaxGroupRows; ++r)
        slots[r] = r < nr ? (cached ? plan_cache[3][start + r] : p.plan.order[start + r]) : -1;
      // A cached expert streams its E4M3 bytes, kHotTiles K tiles per stage
      // (twice the bytes of K4 codes, no decode); others stream codes, one
      // 128-wide K block per stage.
      int hslot = p.expert_to_slot != nullptr ? p.expert_to_slot[expert] : -1;
      if (hslot >= p.hot_slots) hslot = -1;
      const int step = hslot >= 0 ? G::kHotTiles : kStageTiles;
      for (int kt = kt0; kt < kt1; kt += step) {
        if (kt != kt0) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u)) {
            failed = true;
            break;
          }
        }
        const int n = min(step, kt1 - kt);
        const int block_flags = (kt % kStageTiles == 0 ? kBlockStart : 0) |
                                ((kt + n) % kStageTiles == 0 || kt + n >= kt1 ? kBlockEnd : 0);
        meta[stage] = make_int4(static_cast<int>(unit), kt, n,
                                (kt == kt0 ? kFirst : 0) | (kt + step >= kt1 ? kLast : 0) | block_flags |
                                    (hslot >= 0 ? kHot : 0));
        if (kt == kt0) {
          unit_rows[stage][0] = nr;
#pragma unroll
          for (int r = 0; r < kMaxGroupRows; ++r) unit_rows[stage][1 + r] = slots[r];
          unit_rows[stage][kUnitProj] = u.proj;
          unit_rows[stage][kUnitBlock] = u.nb;
          unit_rows[stage][kUnitSplit] = u.split;
        }
        unsigned char* base = smem + stage * G::kStageBytes;
        if (hslot >= 0) {
          const uint32_t hot_bytes = static_cast<uint32_t>(n) * 8u * 256u;
          mbar_arrive_expect_tx(&full_bar[stage], hot_bytes + static_cast<uint32_t>(nr) * kFragBlockBytes);
          const unsigned char* src = p.hot[u.proj] + tile_index(hslot, kt, u.nb * 8, it, ot, p.side) * 256;
          bulk_copy_g2s(base, src, hot_bytes, &full_bar[stage]);
        } else {
          const uint32_t code_bytes = static_cast<uint32_t>(n) * 8u * G::kTileWords * 4u;
          mbar_arrive_expect_tx(&full_bar[stage], code_bytes + static_cast<uint32_t>(nr) * kFragBlockBytes);
          const uint32_t* src = words + tile_index(expert, kt, u.nb * 8, it, ot, p.side) * G::kTileWords;
          bulk_copy_g2s(base, src, code_bytes, &full_bar[stage]);
        }
#pragma unroll
        for (int r = 0; r < kMaxGroupRows; ++r) {
          if (r >= nr) break;
          const int slot = slots[r];
          const unsigned char* fsrc =
              p.frag + ((static_cast<int64_t>(u.proj) * p.nslots + slot) * (it / 8) + kt / 8) * kFragBlockBytes;
          bulk_copy_g2s(base + G::kCodeBytes + r * kFragRowBytes, fsrc, kFragBlockBytes, &full_bar[stage]);
        }
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (failed) break;
      unit = next;
    }
    if (failed) {
      atomicOr(&p.plan.header[9], 1);
      // Copies already issued target valid addresses and land within
      // microseconds; give them that time before this thread retires.
      for (int i = 0; i < 1000; ++i) __nanosleep(1000);
    }
    return;
  }

  // ---------------- consumers ----------------
  const int gid = lane >> 2, tig = lane & 3;
  const uint32_t mcg_mask = p.mcg_mask, mcg_xor = p.mcg_xor;
  int stage = 0;
  uint32_t phase = 0;
  float acc[2][4];
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[c][i] = 0.0f;
  UnitInfo u{};
  int nr = 0, ncg = 1, slot_a = -1, slot_b = -1;
  float st[2][4];  // the current 128-wide K block's products (hot stages carry them across stages)
  GenericGeometry geo;
  if (K != 4) geo = generic_geometry(K, lane);
  const int r0 = gid >> 1, fpos = (gid & 1) * 4 + tig;

  for (;;) {
    if (!mbar_wait(&full_bar[stage], phase)) {
      if (lane == 0) atomicOr(&p.plan.header[9], 2);
      break;
    }
    const int4 m = meta[stage];
    if (m.w & kEnd) break;
    if (m.w & kFirst) {
      u.proj = unit_rows[stage][kUnitProj];
      u.nb = unit_rows[stage][kUnitBlock];
      u.split = unit_rows[stage][kUnitSplit];
      nr = unit_rows[stage][0];
      ncg = (nr + 3) >> 2;
      slot_a = unit_rows[stage][1 + tig];
      slot_b = unit_rows[stage][5 + tig];
    }
    const unsigned char* base = smem + stage * G::kStageBytes;
    const uint32_t* codes = reinterpret_cast<const uint32_t*>(base);
    const uint2* frag = reinterpret_cast<const uint2*>(base + G::kCodeBytes);
    // A code stage holds one 128-wide K block (kStageTiles K tiles), a hot
    // stage kHotTiles K tiles of one; both carry the block's records.  Record
    // rows past the unit's rows hold stale bytes: they only feed the
    // accumulator columns of absent slots, which are reset and never stored.
    const uint2* f0 = frag + (r0 * kFragRowBytes) / 8 + fpos;
    const uint2* f1 = frag + ((4 + r0) * kFragRowBytes) / 8 + fpos;
    if (m.w & kBlockStart) {
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int i = 0; i < 4; ++i) st[c][i] = 0.0f;
    }
    if (m.w & kHot) {
      // Static-cache bytes: the same values in the same MMA order as the
      // codec path, so a cached expert's products are bit-equal.
      const int kb = m.y % kStageTiles;
#pragma unroll
      for (int kk = 0; kk < G::kHotTiles; ++kk) {
        const uint2 b = *reinterpret_cast<const uint2*>(base + (kk * 8 + warp) * 256 + lane * 8);
        uint32_t a[4];
        e4m3_fragment(b, a);
        mma_f16(st[0], a, f0[(kb + kk) * 8]);
        if (ncg > 1) mma_f16(st[1], a, f1[(kb + kk) * 8]);
      }
    } else if (K == 4) {
      uint32_t word[kStageTiles], prior[kStageTiles];
#pragma unroll
      for (int kk = 0; kk < kStageTiles; ++kk) {
        const uint32_t* tile = codes + (kk * 8 + warp) * 32;
        word[kk] = tile[lane];
        prior[kk] = tile[(lane + 31) & 31];
      }
      if (ncg > 1) {
#pragma unroll
        for (int kk = 0; kk < kStageTiles; ++kk) {
          uint32_t a[4];
          k4_fragment(word[kk], prior[kk], mcg_mask, mcg_xor, a);
          mma_f16(st[0], a, f0[kk * 8]);
          mma_f16(st[1], a, f1[kk * 8]);
        }
      } else {
#pragma unroll
        for (int kk = 0; kk < kStageTiles; ++kk) {
          uint32_t a[4];
          k4_fragment(word[kk], prior[kk], mcg_mask, mcg_xor, a);
          mma_f16(st[0], a, f0[kk * 8]);
        }
      }
    } else {
#pragma unroll
      for (int kk = 0; kk < kStageTiles; ++kk) {
        uint32_t cw[8], a[4];
        generic_codewords(codes + (kk * 8 + warp) * G::kTileWords, K, geo, cw);
        tile_fragment(cw, a);
        mma_f16(st[0], a, f0[kk * 8]);
        if (ncg > 1) mma_f16(st[1], a, f1[kk * 8]);
      }
    }
    // This lane's accumulator columns belong to unit rows tig and 4 + tig;
    // their block unscales sit in the fragment record headers.
    if (m.w & kBlockEnd) {
      const float* hdr = reinterpret_cast<const float*>(base + G::kCodeBytes + 512);
      const float us0 = tig < nr ? hdr[tig * (kFragRowBytes / 4)] : 0.0f;
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[0][i] = fmaf(st[0][i], us0, acc[0][i]);
      if (ncg > 1) {
        const float us1 = 4 + tig < nr ? hdr[(4 + tig) * (kFragRowBytes / 4)] : 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[1][i] = fmaf(st[1][i], us1, acc[1][i]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[stage]);
    if (m.w & kLast) {
      const int64_t ubase = static_cast<int64_t>(u.proj) * p.nslots;
      const int col = u.nb * 128 + warp * 16 + gid;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int slot = c == 0 ? slot_a : slot_b;
        if (slot >= 0) {
          float* dst = p.partial + ((ubase + slot) * p.splits + u.split) * p.out_features + col;
          dst[0] = acc[c][0] + acc[c][1];
          dst[8] = acc[c][2] + acc[c][3];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[c][i] = 0.0f;
      }
    }
    if (++stage == kStages) {
      stage = 0;
      phase ^= 1u;
    }
  }
}

template <int K>
static cudaError_t launch_stream_k(const StreamParams& p, cudaStream_t s) {
  // Attribute and occupancy are queried once per process (the launch shape is
  // fixed: one persistent CTA per resident slot).
  static int grid = 0;
  const int smem = StageGeometry<K>::kSmemBytes;
  if (grid == 0) {
    cudaError_t err =
        cudaFuncSetAttribute(trellis_stream_kernel<K>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return err;
    int device = 0, sms = 0, per_sm = 0;
    if ((err = cudaGetDevice(&device)) != cudaSuccess) return err;
    if ((err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) return err;
    if ((err = prefer_shared_carveout(trellis_stream_kernel<K>)) != cudaSuccess) return err;
    if ((err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, trellis_stream_kernel<K>, kStreamThreads,
                                                             smem)) != cudaSuccess)
      return err;
    grid = sms * (per_sm < 1 ? 1 : per_sm);
  }
  return launch_pdl(trellis_stream_kernel<K>, dim3(grid), dim3(kStreamThreads), static_cast<size_t>(smem), s, p);
}

bool encode_dense_maps(StreamParams& p) {
  const DenseUnits& d = p.dense;
  if (d.units <= 0) return true;
  const uint64_t row_bytes = static_cast<uint64_t>(d.k) * 2;
  if (!encode_tiled_2d(&p.dense_w0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, d.w0, static_cast<uint64_t>(d.k),
                       static_cast<uint64_t>(d.n), row_bytes, 64, kDenseRows, CU_TENSOR_MAP_SWIZZLE_128B))
    return false;
  if (d.w1 == nullptr) {
    p.dense_w1 = p.dense_w0;
    return true;
  }
  return encode_tiled_2d(&p.dense_w1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, d.w1, static_cast<uint64_t>(d.k),
                         static_cast<uint64_t>(d.n), row_bytes, 64, kDenseRows, CU_TENSOR_MAP_SWIZZLE_128B);
}

cudaError_t launch_stream(const StreamParams& p, cudaStream_t s) {
  switch (p.k) {
    case 2: return launch_stream_k<2>(p, s);
    case 3: return launch_stream_k<3>(p, s);
    default: return launch_stream_k<4>(p, s);
  }
}

}  // namespace exlr8
