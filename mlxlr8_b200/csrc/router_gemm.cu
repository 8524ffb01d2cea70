// Router gate product for prefill batches on the tensor cores:
// logits[T][256] = x[T][h] . Wg[256][h]^T in float32 (model.py:366-371,
// dense.py:158-159: the gate runs on x.astype(float32) with float32 weights).
//
// Operands are bf16 pieces whose products sum to the float32 product: the
// weight w = w1 + w2 + w3 (w1 = bf16(w), w2 = bf16(w - w1), w3 =
// bf16(w - w1 - w2), 24 significant bits), and x itself when it is bf16 (a
// bf16 value is exact), else x = x1 + x2 (+ x3 for float32).  The kernel
// accumulates every piece product x_i . w_j with i + j <= 2 (the dropped
// terms are below 2^-24 of the product) into one TMEM accumulator, so the
// logits equal a float32 dot product up to summation order.
//
// Tile: 128 tokens (M) x 128 experts (N); the K range is split over
// gridDim.z CTAs whose float32 partials are summed in split order by
// router_sum_kernel.  Warp 0 loads (TMA), warp 1 issues the MMAs, warps 2-5
// drain TMEM.  A stage holds the pieces of one 64-wide K tile, and the ring
// has as many stages as twelve 16 KB tiles allow (three for bf16 tokens
// against the three weight pieces, six for the plain bf16 GEMM).  Waits are
// bounded; a timeout sets error[0].

#include <cuda.h>
#include <cuda_bf16.h>
#include <mutex>

#include "common.cuh"
#include "router_gemm.cuh"
#include "umma.cuh"

namespace exlr8 {

namespace {

constexpr int kRgKTile = 64;                  // bf16 values per 128-byte row
constexpr uint32_t kRgTile = 128 * 128;       // one 128-row operand tile
constexpr int kRgRingTiles = 12;              // tiles of all stages together
constexpr int kRgMaxStages = 6;
constexpr uint32_t kRgSmem = kRgRingTiles * kRgTile + 1024;
constexpr int kRgThreads = 192;

struct RgShared {
  uint64_t full[kRgMaxStages];
  uint64_t empty[kRgMaxStages];
  uint64_t acc_full;
  uint32_t tmem;
};

// partial[split][row][n0 + c] (row stride n) of x . W^T over this CTA's K
// range; the weight piece j occupies rows [j * n, (j + 1) * n) of wmap.
__global__ void __launch_bounds__(kRgThreads, 1)
    bf16_gemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                     int x_pieces, int w_pieces, int tokens, int hidden, int n, int ktiles_per_split,
                     float* __restrict__ partial, int32_t* __restrict__ error) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ RgShared sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Offsetting the shared array itself (not an integer round trip) keeps the
  // pointer in the shared window: the stage accesses compile to shared loads
  // and stores.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int m0 = blockIdx.x * 128, n0 = blockIdx.y * 128, split = blockIdx.z;
  const int kt0 = split * ktiles_per_split;
  const int ktiles = min(ktiles_per_split, hidden / kRgKTile - kt0);
  const int stage_tiles = x_pieces + w_pieces;
  const int stages = min(kRgMaxStages, kRgRingTiles / stage_tiles);
  const uint32_t stage_stride = stage_tiles * kRgTile;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    mbar_init(&sh.acc_full, 1);
    mbar_fence_init();
    prefetch_tensor_map(&xmap);
    prefetch_tensor_map(&wmap);
  }
  if (warp == 1) tmem_alloc(&sh.tmem, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem;
  const uint32_t stage_bytes = stage_tiles * kRgTile;

  if (warp == 0) {
    if (lane == 0) {
      int kt = 0;
      for (; kt < ktiles; ++kt) {
        const int s = kt % stages;
        if (kt >= stages && !mbar_wait(&sh.empty[s], ((kt / stages) - 1) & 1)) {
          atomicCAS(error, 0, 1);
          break;
        }
        uint8_t* st = smem + s * stage_stride;
        const int k = (kt0 + kt) * kRgKTile;
        mbar_arrive_expect_tx(&sh.full[s], stage_bytes);
        for (int i = 0; i < x_pieces; ++i) tma_load_2d(st + i * kRgTile, &xmap, k, i * tokens + m0, &sh.full[s]);
        for (int j = 0; j < w_pieces; ++j)
          tma_load_2d(st + (x_pieces + j) * kRgTile, &wmap, k, j * n + n0, &sh.full[s]);
      }
      // Copies still in flight must land before the CTA exits.
      for (int u = max(0, kt - stages); u < kt; ++u)
        if (!mbar_wait(&sh.full[u % stages], (u / stages) & 1)) atomicCAS(error, 0, 2);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = bf16_idesc(128);
      bool ok = true;
      for (int kt = 0; kt < ktiles; ++kt) {
        const int s = kt % stages;
        if (!mbar_wait(&sh.full[s], (kt / stages) & 1)) {
          atomicCAS(error, 0, 3);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t st = smem_u32(smem + s * stage_stride);
        for (int i = 0; i < x_pieces; ++i) {
          for (int j = 0; j < w_pieces && i + j <= 2; ++j) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              tc_mma_f16(tmem, umma_desc_sw128(st + i * kRgTile + kk * 32),
                         umma_desc_sw128(st + (x_pieces + j) * kRgTile + kk * 32), idesc,
                         (kt | i | j | kk) != 0);
            }
          }
        }
        tc_commit(&sh.empty[s]);
      }
      tc_commit(&sh.acc_full);
      (void)ok;
    }
  } else {
    const int quad = warp & 3;
    const bool ok = mbar_wait(&sh.acc_full, 0);
    if (!ok && lane == 0) atomicCAS(error, 0, 4);
    tc_fence_after();
    if (ok) {
      float* dst = partial + static_cast<int64_t>(split) * tokens * n;
#pragma unroll 1
      for (int c0 = 0; c0 < 128; c0 += 16) {
        uint32_t v[16];
        tc_ld16(tmem + (static_cast<uint32_t>(32 * quad) << 16) + c0, v);
        tc_wait_ld();
        const int row = m0 + 32 * quad + lane;
        if (row < tokens) {
          float4* out = reinterpret_cast<float4*>(dst + static_cast<int64_t>(row) * n + n0 + c0);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            out[q] = ktiles > 0 ? make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                              __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_free(tmem, 128);
}

// Gate weight pieces: w [256][h] float32 -> bf16 [3][256][h].
__global__ void router_weight_pieces_kernel(const float* __restrict__ w, int64_t n, __nv_bfloat16* __restrict__ out) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float v = w[i];
    const __nv_bfloat16 a = __float2bfloat16_rn(v);
    const float r1 = v - __bfloat162float(a);
    const __nv_bfloat16 b = __float2bfloat16_rn(r1);
    const __nv_bfloat16 c = __float2bfloat16_rn(r1 - __bfloat162float(b));
    out[i] = a;
    out[n + i] = b;
    out[2 * n + i] = c;
  }
}

// Activation pieces for float16 / float32 x: [pieces][tokens][h] bf16.
__global__ void router_x_pieces_kernel(const void* __restrict__ x, int x_dtype, int64_t n, int pieces,
                                       __nv_bfloat16* __restrict__ out) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float v = load_act(x, x_dtype, i);
    for (int p = 0; p < pieces; ++p) {
      const __nv_bfloat16 b = __float2bfloat16_rn(v);
      out[p * n + i] = b;
      v -= __bfloat162float(b);
    }
  }
}

// h[t][j] = T(SwiGLU(T(sum g), T(sum u))) over split partials [splits][t][m]
// (the dense shared expert's gate/up finish; sums in split order).
__global__ void dense_swiglu_kernel(const float* __restrict__ gp, const float* __restrict__ up, int splits, int64_t n,
                                    int act_dtype, void* __restrict__ h) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float g = gp[i], u = up[i];
    for (int k = 1; k < splits; ++k) {
      g += gp[k * n + i];
      u += up[k * n + i];
    }
    store_act(h, act_dtype, i, swiglu_typed(act_dtype, g, u));
  }
}

// logits = sum over splits in split order.
__global__ void router_sum_kernel(const float* __restrict__ partial, int splits, int64_t n, float* __restrict__ logits) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float s = partial[i];
    for (int k = 1; k < splits; ++k) s += partial[k * n + i];
    logits[i] = s;
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn rg_encode_fn() {
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

bool rg_encode(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows) {
  if (rows == 0) return false;
  EncodeTiledFn fn = rg_encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {inner * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kRgKTile), 128};
  const cuuint32_t es[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return sms;
}

}  // namespace

cudaError_t launch_dense_swiglu(const float* gate_partial, const float* up_partial, int splits, int64_t n,
                                int act_dtype, void* h, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  dense_swiglu_kernel<<<sm_count() * 8, 256, 0, s>>>(gate_partial, up_partial, splits, n, act_dtype, h);
  return cudaGetLastError();
}

// K splits so that the grid fills the SMs in one wave (one CTA per SM: the
// ring takes most of shared memory); every split gets at least one 64-wide
// K tile.
int bf16_gemm_splits(int tokens, int k, int n) {
  const int mtiles = (tokens + 127) / 128;
  const int ntiles = n / 128;
  const int ktiles = k / kRgKTile;
  int splits = sm_count() / (mtiles * ntiles);
  if (splits > 8) splits = 8;
  if (splits > ktiles) splits = ktiles;
  if (splits < 1) splits = 1;
  const int per = (ktiles + splits - 1) / splits;
  return (ktiles + per - 1) / per;
}

int router_gemm_splits(int tokens, int hidden) { return bf16_gemm_splits(tokens, hidden, 256); }

size_t router_gemm_workspace(int tokens, int hidden, int x_dtype) {
  const int pieces = x_dtype == kBF16 ? 0 : (x_dtype == kF16 ? 2 : 3);
  const size_t splits = static_cast<size_t>(router_gemm_splits(tokens, hidden));
  auto up = [](size_t v) { return (v + 255) / 256 * 256; };
  return up(3ull * 256 * hidden * 2) + up(static_cast<size_t>(pieces) * tokens * hidden * 2) +
         up(splits * tokens * 256 * 4) + up(16);
}

static cudaError_t configure_bf16_gemm() {
  static bool configured = false;
  if (!configured) {
    cudaError_t err = cudaFuncSetAttribute(bf16_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kRgSmem);
    if (err != cudaSuccess) return err;
    configured = true;
  }
  return cudaSuccess;
}

cudaError_t launch_dense_gemm(const uint16_t* a, int rows, int k, const uint16_t* b, int n, int splits,
                              float* partial, int32_t* error, cudaStream_t s) {
  cudaError_t err = configure_bf16_gemm();
  if (err != cudaSuccess) return err;
  CUtensorMap amap, bmap;
  if (!rg_encode(&amap, a, k, rows) || !rg_encode(&bmap, b, k, n)) return cudaErrorInvalidValue;
  const int ktiles = k / kRgKTile;
  const int per = (ktiles + splits - 1) / splits;
  dim3 grid((rows + 127) / 128, n / 128, splits);
  bf16_gemm_kernel<<<grid, kRgThreads, kRgSmem, s>>>(amap, bmap, 1, 1, rows, k, n, per, partial, error);
  return cudaGetLastError();
}

cudaError_t launch_router_gemm(const void* x, int x_dtype, int tokens, int hidden, const float* gate_weight,
                               float* logits, void* workspace, cudaStream_t s) {
  {
    const cudaError_t err = configure_bf16_gemm();
    if (err != cudaSuccess) return err;
  }
  auto up = [](size_t v) { return (v + 255) / 256 * 256; };
  char* ws = static_cast<char*>(workspace);
  __nv_bfloat16* wp = reinterpret_cast<__nv_bfloat16*>(ws);
  ws += up(3ull * 256 * hidden * 2);
  const int pieces = x_dtype == kBF16 ? 1 : (x_dtype == kF16 ? 2 : 3);
  const void* xa = x;
  if (x_dtype != kBF16) {
    __nv_bfloat16* xp = reinterpret_cast<__nv_bfloat16*>(ws);
    ws += up(static_cast<size_t>(pieces) * tokens * hidden * 2);
    router_x_pieces_kernel<<<sm_count() * 8, 256, 0, s>>>(x, x_dtype, static_cast<int64_t>(tokens) * hidden, pieces,
                                                          xp);
    xa = xp;
  }
  const int splits = router_gemm_splits(tokens, hidden);
  float* partial = reinterpret_cast<float*>(ws);
  ws += up(static_cast<size_t>(splits) * tokens * 256 * 4);
  int32_t* error = reinterpret_cast<int32_t*>(ws);
  cudaError_t err = cudaMemsetAsync(error, 0, sizeof(int32_t), s);
  if (err != cudaSuccess) return err;
  router_weight_pieces_kernel<<<sm_count() * 4, 256, 0, s>>>(gate_weight, 256ll * hidden, wp);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  CUtensorMap xmap, wmap;
  if (!rg_encode(&xmap, xa, hidden, static_cast<uint64_t>(pieces) * tokens) || !rg_encode(&wmap, wp, hidden, 3 * 256))
    return cudaErrorInvalidValue;
  const int ktiles = hidden / kRgKTile;
  const int per = (ktiles + splits - 1) / splits;
  dim3 grid((tokens + 127) / 128, 2, splits);
  bf16_gemm_kernel<<<grid, kRgThreads, kRgSmem, s>>>(xmap, wmap, pieces, 3, tokens, hidden, 256, per,
                                                     splits == 1 ? logits : partial, error);
  err = cudaGetLastError();
  if (err != cudaSuccess || splits == 1) return err;
  const int64_t n = static_cast<int64_t>(tokens) * 256;
  router_sum_kernel<<<sm_count() * 4, 256, 0, s>>>(partial, splits, n, logits);
  return cudaGetLastError();
}

}  // namespace exlr8
