// Streaming MXFP4 GEMV for the joined experts at decode batch sizes.
//
// Replaces, for up to 16 token rows, the ordered-gather GEMV and the MLX
// gather_qmm products of exlr8 joined_mxfp4.py:72-134.  Same shape as the
// trellis stream (trellis_stream.cu): one persistent CTA per resident slot,
// warp 8 produces, warps 0-7 consume.
//
//   producer: takes units (plan group, 128-row output block, K split) from a
//     global counter and streams each unit's K range, 256 inputs per stage,
//     into a ring of shared-memory stages: the codes of the unit's 128 rows as
//     one 2-D TMA tile (128 rows x 128 bytes, 128-byte swizzle: wide rows keep
//     the tensor copy efficient), their E8M0 scales as two 512-byte blocks of
//     the prepared layout (one copy), and two activation records per unit row,
//     all completing on the stage's mbarrier.
//   consumers: warp w owns output rows 16w..16w+15 of the block.  Per 32-wide
//     K block a lane reads one code word of row g and of row g + 8 (eight
//     E2M1 values each; the swizzle keeps the 32 lanes on distinct banks),
//     converts them pairwise to float16 (exact) and runs two mma.sync
//     m16n8k16 steps against float16 hi/lo activation pieces (the MXFP4 K
//     order of joined_stream.cuh); the block's float32 product is added times
//     the row's E8M0 scale, and each stage's sum times the activation block's
//     unscale, so the result equals the float32 product of the dequantised
//     weights with the activations to about 22 significant bits.
//   output: float32 partials [plane][slot][split][plane_rows]; the joined
//     gate/up matrix (2m rows) lands as the gate plane and the up plane.

#include "common.cuh"
#include "joined_stream.cuh"
#include "launch.cuh"
#include "mx_gemm.cuh"
#include "tensor_map.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace exlr8 {

namespace {

constexpr int kJConsumers = 8;
constexpr int kJProducerWarp = kJConsumers;
constexpr int kJThreads = (kJConsumers + 1) * 32;
constexpr int kJStages = 4;
constexpr int kJBlocks = 2;                      // 128-wide K blocks per stage
constexpr int kJRowBytes = kJBlocks * 64;        // 256 E2M1 codes of one row
constexpr int kJCodeBytes = 128 * kJRowBytes;    // 128 rows
constexpr int kJScaleBytes = kJBlocks * 512;     // 128 rows x 8 E8M0
constexpr int kJFragRowBytes = 8 * 64 + 64;  // record rows padded onto different banks
constexpr int kJFragOffset = kJCodeBytes + kJScaleBytes;
constexpr int kJStageBytes = (kJFragOffset + kJBlocks * kMaxGroupRows * kJFragRowBytes + 1023) / 1024 * 1024;
constexpr int kJSmemBytes = kJStages * kJStageBytes + 1024;  // + alignment slack for the 128-byte swizzle
static_assert(kJFragRowBytes >= kFragBlockBytes, "a fragment record fits its stage row");

enum : int { kFirst = 1, kLast = 2, kEnd = 4 };

// One 32-block of one column group: the eight E2M1 codes of rows g (w0) and
// g + 8 (w1) converted to float16 straight into the A operands of the
// block's two MMA steps (pairs (k, k + 1) of codes 0-3 for the first, 4-7 for
// the second), d = A0 * b0 + A1 * b1.  One asm statement, so the converted
// values need no register moves before the MMAs.
__device__ __forceinline__ void block_mma(float d[4], uint32_t w0, uint32_t w1, uint2 b0, uint2 b1) {
  asm volatile(
      "{\n"
      " .reg .b8 p0, p1, p2, p3, q0, q1, q2, q3;\n"
      " .reg .b32 a0, a1, a2, a3, z;\n"
      " mov.b32 {p0, p1, p2, p3}, %4;\n"
      " mov.b32 {q0, q1, q2, q3}, %5;\n"
      " mov.b32 z, 0;\n"
      " cvt.rn.f16x2.e2m1x2 a0, p0;\n"
      " cvt.rn.f16x2.e2m1x2 a1, q0;\n"
      " cvt.rn.f16x2.e2m1x2 a2, p1;\n"
      " cvt.rn.f16x2.e2m1x2 a3, q1;\n"
      " mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {a0,a1,a2,a3}, {%6,%7}, {z,z,z,z};\n"
      " cvt.rn.f16x2.e2m1x2 a0, p2;\n"
      " cvt.rn.f16x2.e2m1x2 a1, q2;\n"
      " cvt.rn.f16x2.e2m1x2 a2, p3;\n"
      " cvt.rn.f16x2.e2m1x2 a3, q3;\n"
      " mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {a0,a1,a2,a3}, {%8,%9}, {%0,%1,%2,%3};\n"
      "}\n"
      : "=&f"(d[0]), "=&f"(d[1]), "=&f"(d[2]), "=&f"(d[3])
      : "r"(w0), "r"(w1), "r"(b0.x), "r"(b0.y), "r"(b1.x), "r"(b1.y));
}

// Four 8x16-byte shared-memory matrices; lane l gives the row address of
// matrix l / 8, row l % 8, and receives word (l % 4) of row (l / 4) of each.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& d0, uint32_t& d1, uint32_t& d2, uint32_t& d3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
               : "r"(addr));
}

// 2^(s - 127) of the four E8M0 bytes of a scale word: each byte moved to the
// float exponent field.  A zero code gives 0 rather than 2^-127: its products
// lie below 6 * 2^-127 of the activations, far under a float32 ulp of any sum
// they join.
__device__ __forceinline__ void e8m0x4(uint32_t word, float f[4]) {
  f[0] = __uint_as_float((word << 23) & 0x7F800000u);
  f[1] = __uint_as_float((word << 15) & 0x7F800000u);
  f[2] = __uint_as_float((word << 7) & 0x7F800000u);
  f[3] = __uint_as_float((word >> 1) & 0x7F800000u);
}

struct UnitInfo {
  int group, nb, split;
};

// Unit indices stay below 2^31, so 32-bit arithmetic suffices; the producer
// decodes each unit once and hands its fields to the consumers through
// shared memory.
__device__ __forceinline__ UnitInfo decode_unit(uint32_t unit, uint32_t splits, uint32_t nblocks) {
  UnitInfo u;
  const uint32_t a = unit / splits;
  u.split = static_cast<int>(unit - a * splits);
  u.group = static_cast<int>(a / nblocks);
  u.nb = static_cast<int>(a - static_cast<uint32_t>(u.group) * nblocks);
  return u;
}

constexpr int kJPlanCache = 160;

__global__ void __launch_bounds__(kJThreads, 2) joined_stream_kernel(const __grid_constant__ JoinedStreamParams p) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kJStages];
  __shared__ __align__(8) uint64_t empty_bar[kJStages];
  __shared__ int4 meta[kJStages];  // unit, first K block, K blocks (1 or 2), flags
  // First stage of a unit: rows, slots, then the unit's output block and split.
  constexpr int kUnitBlock = kMaxGroupRows + 1, kUnitSplit = kMaxGroupRows + 2;
  __shared__ int unit_rows[kJStages][kMaxGroupRows + 3];
  __shared__ int plan_cache[4][kJPlanCache];
  // The 128-byte swizzle repeats every 1024 bytes: stages start on 1024.
  // (Offsetting the shared array itself keeps the pointer in the shared
  // window, so the stage reads compile to shared-memory loads.)
  unsigned char* ring = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kblocks = p.in_features / 128, nblocks = p.out_features / 128;
  pdl_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kJStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kJConsumers);
    }
    mbar_fence_init();
  }
  __syncthreads();
  pdl_wait();  // the plan, the records and the partial buffers belong to earlier kernels

  if (warp == kJProducerWarp) {
    // ---------------- producer ----------------
    const int groups = p.plan.header[0];
    const bool cached = groups <= kJPlanCache && p.nslots <= kJPlanCache;
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
    prefetch_tensor_map(&p.codes);
    const int64_t total = static_cast<int64_t>(groups) * nblocks * p.splits;
    int stage = 0;
    uint32_t phase = 0;
    bool failed = false;
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
      const UnitInfo u = decode_unit(static_cast<uint32_t>(unit), static_cast<uint32_t>(p.splits),
                                     static_cast<uint32_t>(nblocks));
      const int expert = cached ? plan_cache[0][u.group] : p.plan.group_expert[u.group];
      const int start = cached ? plan_cache[1][u.group] : p.plan.group_start[u.group];
      const int nr = cached ? plan_cache[2][u.group] : p.plan.group_count[u.group];
      const int kb0 = u.split * p.kb_per_split;
      const int kb1 = min(kb0 + p.kb_per_split, kblocks);
      const int64_t row0 = static_cast<int64_t>(expert) * p.out_features + static_cast<int64_t>(u.nb) * 128;
      const uint8_t* sblocks = p.scales + (row0 / 128) * kblocks * 512;
      int slots[kMaxGroupRows];
#pragma unroll
      for (int r = 0; r < kMaxGroupRows; ++r)
        slots[r] = r < nr ? (cached ? plan_cache[3][start + r] : p.plan.order[start + r]) : -1;
      for (int kb = kb0; kb < kb1; kb += kJBlocks) {
        if (kb != kb0) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u)) {
            failed = true;
            break;
          }
        }
        const int nb = min(kJBlocks, kb1 - kb);
        meta[stage] = make_int4(static_cast<int>(unit), kb, nb,
                                (kb == kb0 ? kFirst : 0) | (kb + kJBlocks >= kb1 ? kLast : 0));
        if (kb == kb0) {
          unit_rows[stage][0] = nr;
#pragma unroll
          for (int r = 0; r < kMaxGroupRows; ++r) unit_rows[stage][1 + r] = slots[r];
          unit_rows[stage][kUnitBlock] = u.nb;
          unit_rows[stage][kUnitSplit] = u.split;
        }
        unsigned char* base = ring + stage * kJStageBytes;
        // The tensor tile is always 128 x 128 bytes: past the end of a row it
        // is zero-filled (and counted), and the consumers skip that half.
        mbar_arrive_expect_tx(&full_bar[stage], kJCodeBytes + static_cast<uint32_t>(nb) * 512u +
                                                    static_cast<uint32_t>(nr * nb) * kFragBlockBytes);
        tma_load_2d(base, &p.codes, kb * 64, static_cast<int>(row0), &full_bar[stage]);
        bulk_copy_g2s(base + kJCodeBytes, sblocks + kb * 512, static_cast<uint32_t>(nb) * 512u, &full_bar[stage]);
#pragma unroll
        for (int r = 0; r < kMaxGroupRows; ++r) {
          if (r >= nr) break;
          const unsigned char* fsrc = p.frag + (static_cast<int64_t>(slots[r]) * kblocks + kb) * kFragBlockBytes;
          for (int q = 0; q < nb; ++q)
            bulk_copy_g2s(base + kJFragOffset + (q * kMaxGroupRows + r) * kJFragRowBytes, fsrc + q * kFragBlockBytes,
                          kFragBlockBytes, &full_bar[stage]);
        }
        if (++stage == kJStages) {
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
  const int r0 = warp * 16 + gid, r1 = r0 + 8;  // rows of the 128-row block
  // Code words come in by ldmatrix: for each pair of 32-blocks (c, c + 1) of
  // the stage's 256 inputs, matrices 0-3 are (rows 0-7, c), (rows 8-15, c),
  // (rows 0-7, c + 1), (rows 8-15, c + 1) of the warp's 16 rows, so lane
  // (g, tig) receives word tig of rows g and g + 8 of both blocks.  Lane l
  // addresses row (l % 8) + 8 ((l / 8) % 2) of block c + l / 16; 16-byte
  // chunk c of row r sits at chunk c ^ (r & 7) (128-byte swizzle).
  const int lrow = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
  uint32_t code_off[2 * kJBlocks];  // [q * 2 + pair]
#pragma unroll
  for (int cp = 0; cp < 2 * kJBlocks; ++cp)
    code_off[cp] = static_cast<uint32_t>(lrow * kJRowBytes + (((2 * cp + (lane >> 4)) ^ (lane & 7)) << 4));
  const int sc0_off = kJCodeBytes + (r0 & 31) * 16 + (r0 >> 5) * 4;
  const int sc1_off = kJCodeBytes + (r1 & 31) * 16 + (r1 >> 5) * 4;
  int stage = 0;
  uint32_t phase = 0;
  float acc[2][4];
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[c][i] = 0.0f;
  UnitInfo u{};
  int nr = 0, ncg = 1, slot_a = -1, slot_b = -1;
  const int rr0 = gid >> 1, fpos = (gid & 1) * 4 + tig;

  for (;;) {
    if (!mbar_wait(&full_bar[stage], phase)) {
      if (lane == 0) atomicOr(&p.plan.header[9], 2);
      break;
    }
    const int4 m = meta[stage];
    if (m.w & kEnd) break;
    if (m.w & kFirst) {
      u.nb = unit_rows[stage][kUnitBlock];
      u.split = unit_rows[stage][kUnitSplit];
      nr = unit_rows[stage][0];
      ncg = (nr + 3) >> 2;
      slot_a = unit_rows[stage][1 + tig];
      slot_b = unit_rows[stage][5 + tig];
    }
    const unsigned char* base = ring + stage * kJStageBytes;
    // Record rows past the unit's rows hold stale bytes: they only feed the
    // accumulator columns of absent slots, which are never stored.
    const uint2* frag = reinterpret_cast<const uint2*>(base + kJFragOffset);
    const float* hdr = reinterpret_cast<const float*>(base + kJFragOffset + 512);
    float us[2][kJBlocks];
#pragma unroll
    for (int q = 0; q < kJBlocks; ++q) {
      us[0][q] = tig < nr ? hdr[(q * kMaxGroupRows + tig) * (kJFragRowBytes / 4)] : 0.0f;
      us[1][q] = 4 + tig < nr ? hdr[(q * kMaxGroupRows + 4 + tig) * (kJFragRowBytes / 4)] : 0.0f;
    }
#pragma unroll
    for (int q = 0; q < kJBlocks; ++q) {
      if (q < m.z) {
        uint32_t w0[4], w1[4];
        const uint32_t sbase = smem_u32(base);
        ldsm_x4(sbase + code_off[q * 2], w0[0], w1[0], w0[1], w1[1]);
        ldsm_x4(sbase + code_off[q * 2 + 1], w0[2], w1[2], w0[3], w1[3]);
        float fs0[4], fs1[4];
        e8m0x4(*reinterpret_cast<const uint32_t*>(base + sc0_off + q * 512), fs0);
        e8m0x4(*reinterpret_cast<const uint32_t*>(base + sc1_off + q * 512), fs1);
        const uint2* f0 = frag + ((q * kMaxGroupRows + rr0) * kJFragRowBytes) / 8 + fpos;
        const uint2* f1 = frag + ((q * kMaxGroupRows + 4 + rr0) * kJFragRowBytes) / 8 + fpos;
        float st[2][4];
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int i = 0; i < 4; ++i) st[c][i] = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          // Rows g / g + 8; A pairs (k 8tig + 4h .. +1) and (8tig + 4h + 2 .. +3).
          float blk[4];
          block_mma(blk, w0[j], w1[j], f0[(2 * j) * 8], f0[(2 * j + 1) * 8]);
          st[0][0] = fmaf(blk[0], fs0[j], st[0][0]);
          st[0][1] = fmaf(blk[1], fs0[j], st[0][1]);
          st[0][2] = fmaf(blk[2], fs1[j], st[0][2]);
          st[0][3] = fmaf(blk[3], fs1[j], st[0][3]);
          if (ncg > 1) {
            float blk1[4];
            block_mma(blk1, w0[j], w1[j], f1[(2 * j) * 8], f1[(2 * j + 1) * 8]);
            st[1][0] = fmaf(blk1[0], fs0[j], st[1][0]);
            st[1][1] = fmaf(blk1[1], fs0[j], st[1][1]);
            st[1][2] = fmaf(blk1[2], fs1[j], st[1][2]);
            st[1][3] = fmaf(blk1[3], fs1[j], st[1][3]);
          }
        }
        // Each 128-wide block's products times its activation unscale.
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[0][i] = fmaf(st[0][i], us[0][q], acc[0][i]);
        if (ncg > 1) {
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[1][i] = fmaf(st[1][i], us[1][q], acc[1][i]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[stage]);
    if (m.w & kLast) {
      const int row = u.nb * 128 + r0;
      const int plane = (u.nb * 128) / p.plane_rows;
      const int col = row - plane * p.plane_rows;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int slot = c == 0 ? slot_a : slot_b;
        if (slot >= 0) {
          float* dst = p.partial +
                       ((static_cast<int64_t>(plane) * p.nslots + slot) * p.splits + u.split) * p.plane_rows + col;
          dst[0] = acc[c][0] + acc[c][1];
          dst[8] = acc[c][2] + acc[c][3];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[c][i] = 0.0f;
      }
    }
    if (++stage == kJStages) {
      stage = 0;
      phase ^= 1u;
    }
  }
}

int g_grid = 0;

cudaError_t configure() {
  if (g_grid != 0) return cudaSuccess;
  cudaError_t err =
      cudaFuncSetAttribute(joined_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kJSmemBytes);
  if (err != cudaSuccess) return err;
  int device = 0, sms = 0, per_sm = 0;
  if ((err = cudaGetDevice(&device)) != cudaSuccess) return err;
  if ((err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) return err;
  if ((err = prefer_shared_carveout(joined_stream_kernel)) != cudaSuccess) return err;
  if ((err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, joined_stream_kernel, kJThreads, kJSmemBytes)) !=
      cudaSuccess)
    return err;
  g_grid = sms * (per_sm < 1 ? 1 : per_sm);
  return cudaSuccess;
}

}  // namespace

bool joined_code_map(CUtensorMap* map, const void* codes, int64_t rows, int in_features) {
  return encode_tiled_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, codes, static_cast<uint64_t>(in_features / 2),
                         static_cast<uint64_t>(rows), static_cast<uint64_t>(in_features / 2), kJRowBytes, 128,
                         CU_TENSOR_MAP_SWIZZLE_128B);
}

int joined_stream_ctas() {
  if (configure() != cudaSuccess) return 296;
  return g_grid;
}

cudaError_t launch_joined_stream(const JoinedStreamParams& p, cudaStream_t s) {
  const cudaError_t err = configure();
  if (err != cudaSuccess) return err;
  return launch_pdl(joined_stream_kernel, dim3(g_grid), dim3(kJThreads), static_cast<size_t>(kJSmemBytes), s, p);
}

}  // namespace exlr8
