// Grouped block-scaled expert GEMM (E2M1 weights x E4M3 hi/lo activations,
// E8M0 scales per 32 values) on the sm_100a tensor cores.
//
// Roles the matrix product of one MLX `gather_qmm(mode="mxfp4",
// group_size=32)` call plays in the joined path (exlr8 joined_mxfp4.py:
// 109-113 gate+up, 122-126 down): every sorted slot row times its expert's
// weight rows, float32 out.
//
// Shape of the work: a unit is (chunk, weight block).  The chunk is up to
// kMxMaxN consecutive slot rows of one expert (the MMA N side, so an expert
// with 140 rows costs 144 columns, not two 128-row tiles); the weight block
// is two 128-row tiles of that expert (two TMEM accumulators of M = 128).
// Each 128-value K step of a unit issues 2 accumulators x 2 activation
// planes (hi, lo) x 4 MMAs of K = 32.  Activation hi and lo planes share
// one scale per 32 values, so their MMAs read the same scale columns.
//
// CTA = 6 warps, one persistent CTA per SM:
//   warp 0   TMA producer: unit scheduler (global atomic) + stage loads
//   warp 1   MMA issuer (one thread) and TMEM owner
//   warps 2-5  epilogue: TMEM -> float32 rows of `out`
// Every mbarrier wait is bounded; a timeout records an error in
// chunks.header[4] and the role leaves its loop, so the kernel always ends.

#include <cuda.h>
#include <mutex>

#include "mx_gemm.cuh"
#include "umma.cuh"

namespace exlr8 {

namespace {

constexpr int kStages = 3;
constexpr int kSchedSlots = 4;
constexpr uint32_t kTileA = 128 * 128;                       // one weight tile image (E2M1 with gaps)
constexpr uint32_t kTileB = kMxMaxN * 128;                   // one activation plane tile
constexpr uint32_t kOffA0 = 0, kOffA1 = kTileA, kOffBhi = 2 * kTileA, kOffBlo = 2 * kTileA + kTileB;
constexpr uint32_t kOffSfa = 2 * kTileA + 2 * kTileB;        // 2 x 512
constexpr uint32_t kOffSfb = kOffSfa + 1024;                 // 2 x 512
constexpr uint32_t kStageBytes = kOffSfb + 1024;
static_assert(kStageBytes % 1024 == 0, "stage must keep 1 KB alignment");
constexpr uint32_t kSmemBytes = kStages * kStageBytes + 1024;  // + alignment slack
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemAcc1 = 256, kTmemSfa = 496, kTmemSfb = 504;

enum : int { kErrSched = 1, kErrStage = 2, kErrFull = 3, kErrAcc = 4, kErrAccEmpty = 5, kErrDrain = 6, kErrAlign = 7 };

struct MxShared {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full;
  uint64_t acc_empty;
  uint64_t sched_full[kSchedSlots];
  uint64_t sched_empty[kSchedSlots];
  uint64_t drain;
  int sched[kSchedSlots];
  uint32_t tmem;
};

__device__ __forceinline__ void record_error(int32_t* header, int code) { atomicCAS(&header[4], 0, code); }

struct UnitInfo {
  int chunk, block, expert, start, rows, n16;
};

__device__ __forceinline__ UnitInfo unit_info(const MxChunks& c, int unit, int blocks) {
  UnitInfo u;
  u.chunk = unit / blocks;
  u.block = unit % blocks;
  u.expert = c.chunk_expert[u.chunk];
  u.start = c.chunk_start[u.chunk];
  u.rows = c.chunk_rows[u.chunk];
  u.n16 = (u.rows + 15) & ~15;
  return u;
}

// First weight row (global, over experts * out_features) of accumulator a.
__device__ __forceinline__ int64_t weight_row(const MxGemmArgs& g, const UnitInfo& u, int a) {
  const int64_t base = static_cast<int64_t>(u.expert) * g.out_features;
  if (g.paired) return base + (a ? g.out_features / 2 : 0) + 128 * u.block;
  return base + 256 * u.block + 128 * a;
}

__global__ void __launch_bounds__(kThreads, 1)
    mx_gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap hmap,
                   const __grid_constant__ CUtensorMap lmap, const MxGemmArgs g) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ MxShared sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  int32_t* header = g.chunks.header;
  const int blocks = g.paired ? g.out_features / 256 : g.out_features / 256;
  const int ktiles = g.in_features / kMxKTile;
  const int kblocks = g.in_features / 32;

  // Zero the stages once: the gap bytes of E2M1 images are never written by
  // the TMA and must read as zero.
  for (uint32_t i = threadIdx.x; i < kStages * kStageBytes / 16; i += kThreads)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    mbar_init(&sh.acc_full, 1);
    mbar_init(&sh.acc_empty, 4);
    for (int i = 0; i < kSchedSlots; ++i) {
      mbar_init(&sh.sched_full[i], 1);
      mbar_init(&sh.sched_empty[i], 5);
    }
    mbar_init(&sh.drain, 1);
    mbar_fence_init();
    prefetch_tensor_map(&wmap);
    prefetch_tensor_map(&hmap);
    prefetch_tensor_map(&lmap);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (warp == 1) tmem_alloc(&sh.tmem, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer ----------------
      const int total = header[0] * blocks;
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
        const UnitInfo u = unit_info(g.chunks, unit, blocks);
        const int64_t w0 = weight_row(g, u, 0), w1 = weight_row(g, u, 1);
        const int nb = (u.n16 + 127) / 128;
        const uint32_t bytes = 2 * (128 * 64) + 2 * u.n16 * 128 + 1024 + nb * 512;
        for (int kt = 0; kt < ktiles; ++kt, ++use) {
          const int s = use % kStages;
          if (use >= kStages && !mbar_wait(&sh.empty[s], ((use / kStages) - 1) & 1)) {
            record_error(header, kErrStage);
            failed = true;
            break;
          }
          uint8_t* st = smem + s * kStageBytes;
          mbar_arrive_expect_tx(&sh.full[s], bytes);
          tma_load_2d(st + kOffA0, &wmap, kt * kMxKTile, static_cast<int>(w0), &sh.full[s]);
          tma_load_2d(st + kOffA1, &wmap, kt * kMxKTile, static_cast<int>(w1), &sh.full[s]);
          for (int r = 0; r < u.n16; r += 16) {
            tma_load_2d(st + kOffBhi + r * 128, &hmap, kt * kMxKTile, u.start + r, &sh.full[s]);
            tma_load_2d(st + kOffBlo + r * 128, &lmap, kt * kMxKTile, u.start + r, &sh.full[s]);
          }
          bulk_copy_g2s(st + kOffSfa, g.weight_scales + mx_scale_offset(w0, 4 * kt, kblocks), 512, &sh.full[s]);
          bulk_copy_g2s(st + kOffSfa + 512, g.weight_scales + mx_scale_offset(w1, 4 * kt, kblocks), 512,
                        &sh.full[s]);
          for (int b = 0; b < nb; ++b)
            bulk_copy_g2s(st + kOffSfb + b * 512, g.x_scales + mx_scale_offset(u.start + 128 * b, 4 * kt, kblocks),
                          512, &sh.full[s]);
        }
        if (failed) {
          // Publish the stop marker for the consumers of the next slot.
          continue;
        }
      }
      // Wait for the copies still in flight before the CTA can exit.
      for (uint32_t k = 0; k < kStages && k < use; ++k) {
        const uint32_t last = use - 1 - k;
        if (!mbar_wait(&sh.full[last % kStages], (last / kStages) & 1)) record_error(header, kErrDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
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
        const UnitInfo u = unit_info(g.chunks, unit, blocks);
        if (j >= 1 && !mbar_wait(&sh.acc_empty, (j - 1) & 1)) {
          record_error(header, kErrAccEmpty);
          break;
        }
        tc_fence_after();
        const uint32_t idesc = mx_idesc(kFmtE2M1, kFmtE4M3, u.n16);
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
          const uint32_t st = smem_u32(smem + s * kStageBytes);
          tc_copy_scales(tmem + kTmemSfa, umma_desc_rows16(st + kOffSfa));
          tc_copy_scales(tmem + kTmemSfa + 4, umma_desc_rows16(st + kOffSfa + 512));
          for (int b = 0; b < nb; ++b) tc_copy_scales(tmem + kTmemSfb + 4 * b, umma_desc_rows16(st + kOffSfb + 512 * b));
#pragma unroll
          for (int a = 0; a < 2; ++a) {
#pragma unroll
            for (int t = 0; t < 2; ++t) {
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const uint32_t id = idesc | (static_cast<uint32_t>(kk) << 4) | (static_cast<uint32_t>(kk) << 29);
                const uint64_t da = umma_desc_sw128(st + (a ? kOffA1 : kOffA0) + kk * 32);
                const uint64_t db = umma_desc_sw128(st + (t ? kOffBlo : kOffBhi) + kk * 32);
                tc_mma_mx(tmem + a * kTmemAcc1, da, db, id, (tmem + kTmemSfa + 4 * a) | (static_cast<uint32_t>(kk) << 30),
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
  } else {
    // ---------------- epilogue (warps 2-5) ----------------
    const int quad = warp & 3;  // TMEM sub-partition this warp may read
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
      const UnitInfo u = unit_info(g.chunks, unit, blocks);
      if (!mbar_wait(&sh.acc_full, j & 1)) {
        if (lane == 0) record_error(header, kErrAcc);
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int a = 0; a < 2; ++a) {
        const int64_t feature = weight_row(g, u, a) - static_cast<int64_t>(u.expert) * g.out_features + 32 * quad + lane;
        float* dst = g.out + static_cast<int64_t>(u.start) * g.out_features + feature;
#pragma unroll 1
        for (int c0 = 0; c0 < u.n16; c0 += 16) {
          uint32_t v[16];
          tc_ld16(tmem + (static_cast<uint32_t>(32 * quad) << 16) + a * kTmemAcc1 + c0, v);
          tc_wait_ld();
#pragma unroll
          for (int c = 0; c < 16; ++c)
            if (c0 + c < u.rows) dst[static_cast<int64_t>(c0 + c) * g.out_features] = __uint_as_float(v[c]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.acc_empty);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_free(tmem, kTmemCols);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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

thread_local int g_encode_status = 0;

bool encode_2d(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t inner, uint64_t rows,
               uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) {
    g_encode_status = -1;
    return false;
  }
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = fn(map, type, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  g_encode_status = static_cast<int>(r);
  return r == CUDA_SUCCESS;
}

}  // namespace

int mx_gemm_status() { return g_encode_status; }

cudaError_t launch_mx_gemm(const MxGemmArgs& args, cudaStream_t s) {
  static int sms = 0;
  static bool configured = false;
  if (!configured) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err == cudaSuccess) err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (err == cudaSuccess)
      err = cudaFuncSetAttribute(mx_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (err != cudaSuccess) return err;
    configured = true;
  }
  CUtensorMap wmap, hmap, lmap;
  const uint64_t wrows = static_cast<uint64_t>(args.experts) * args.out_features;
  if (!encode_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, args.weights, args.in_features, wrows,
                 args.in_features / 2, 128, 128) ||
      !encode_2d(&hmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, args.x_hi, args.in_features, args.padded_rows,
                 args.in_features, 128, 16) ||
      !encode_2d(&lmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, args.x_lo, args.in_features, args.padded_rows,
                 args.in_features, 128, 16))
    return cudaErrorInvalidValue;
  mx_gemm_kernel<<<sms, kThreads, kSmemBytes, s>>>(wmap, hmap, lmap, args);
  return cudaGetLastError();
}

}  // namespace exlr8
