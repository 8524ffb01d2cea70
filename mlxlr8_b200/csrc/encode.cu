// MXFP4 quantisation and the load-time trellis -> MXFP4 re-encode of the
// joined experts (exlr8 joined_mxfp4.py:12-47).
//
// Quantisation follows MLX 0.32.3 quantize(w, mode="mxfp4") (group 32, the
// Metal fp_quantize kernel with its fp8_e8m0 / fp4_e2m1 conversions), per
// block of 32 consecutive values along the last axis:
//   x     = amax / 6                       (6 = largest E2M1 magnitude)
//   e     = round(log2 x) (float32 log2, half away from zero), clamped to
//           [-127, 127]; E8M0 code e + 127 (amax = 0 gives code 0, which
//           decodes as 2^-127)
//   q_j   = v_j / 2^e (2^-127 for code 0)
//   code  = nearest E2M1 value to |q_j| (0, .5, 1, 1.5, 2, 3, 4, 6; ties to
//           the even code; above 6 saturates), sign bit 3 = signbit(q_j)
// The float32 log2 is the correctly rounded one, computed through float64.
// Eight codes per uint32, low nibble first; one scale byte per block.

#include "common.cuh"
#include "codec.cuh"

namespace exlr8 {

namespace {

// round(log2 x), x = amax / 6.  Away from the boundary significand sqrt(2)
// the exact log2 is at least 64 significand steps (>= 7.5e-6) from n + 1/2,
// more than half a float32 ulp of any |n + 1/2| <= 127.5, so the rounded
// float32 log2 rounds the same way as the exact one and n = exponent +
// (significand > sqrt 2).  The test runs on amax * float(1/6), which is
// within one ulp of the correctly rounded quotient (and gives the same n as
// it outside the window); inside the window (or for a subnormal quotient)
// the quotient is divided exactly and its float32 log2 formed through
// float64.
constexpr int kSqrt2Mantissa = 0x3504F3;  // largest significand below sqrt(2)
constexpr int kBoundaryWindow = 64;

__device__ __forceinline__ int e8m0_code(float amax) {
  if (!(amax <= 3.4028234663852886e38f)) return 255;  // inf / nan
  if (amax == 0.0f) return 0;
  const uint32_t bits = __float_as_uint(__fmul_rn(amax, 0.16666667163372039794921875f));
  const int biased = static_cast<int>(bits >> 23);
  const int mant = static_cast<int>(bits & 0x7FFFFFu);
  int n;
  if (biased != 0 && abs(mant - kSqrt2Mantissa) > kBoundaryWindow) {
    n = biased - 127 + (mant > kSqrt2Mantissa ? 1 : 0);
  } else {
    const float x = __fdiv_rn(amax, 6.0f);
    if (x == 0.0f) return 0;  // log2 -> -inf, clamped to -127
    n = static_cast<int>(roundf(__double2float_rn(log2(static_cast<double>(x)))));
  }
  n = n < -127 ? -127 : (n > 127 ? 127 : n);
  return n + 127;
}

// max that returns NaN when either operand is NaN (a block holding a NaN
// has a non-finite maximum, code 255).
__device__ __forceinline__ float max_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

// Three-operand form (sm_100).
__device__ __forceinline__ float max3_nan(float a, float b, float c) {
  float d;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 1 / 2^e of a scale code (exact: 2^127 for code 0, 2^-127 for code 254).
// Multiplying by it equals dividing by the decoded scale bit for bit.
__device__ __forceinline__ float e8m0_reciprocal(int code) {
  const int e = code == 0 ? -127 : code - 127;
  return e == 127 ? __uint_as_float(0x00400000u) : __uint_as_float(static_cast<uint32_t>(127 - e) << 23);
}

// E2M1 code of q by comparison: nearest magnitude, ties to the even code,
// saturating at 6, sign bit 3 = signbit(q), NaN -> 7.
__device__ __forceinline__ uint32_t e2m1_code(float q) {
  const uint32_t sign = (__float_as_uint(q) >> 31) << 3;
  const float a = fabsf(q);
  if (a != a) return 7u;
  uint32_t m;
  if (a > 5.0f) m = 7;
  else if (a >= 3.5f) m = 6;
  else if (a > 2.5f) m = 5;
  else if (a >= 1.75f) m = 4;
  else if (a > 1.25f) m = 3;
  else if (a >= 0.75f) m = 2;
  else if (a > 0.25f) m = 1;
  else m = 0;
  return sign | m;
}

// Eight finite values -> eight E2M1 codes, q[0] in the low nibble: the
// hardware conversion rounds to nearest even with finite saturation.
__device__ __forceinline__ uint32_t e2m1x8(const float q[8]) {
  uint32_t out;
  asm("{\n"
      " .reg .b8 b0, b1, b2, b3;\n"
      " cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n"
      " cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n"
      " cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n"
      " cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n"
      " mov.b32 %0, {b0, b1, b2, b3};\n"
      "}\n"
      : "=r"(out)
      : "f"(q[0]), "f"(q[1]), "f"(q[2]), "f"(q[3]), "f"(q[4]), "f"(q[5]), "f"(q[6]), "f"(q[7]));
  return out;
}

// Codes of eight values under scale `code`.  A non-finite block (code 255,
// an infinity or NaN in the block) takes the comparison path, v / inf being
// +-0 or NaN.
__device__ __forceinline__ uint32_t quantize8(const float v[8], int code) {
  if (code == 255) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) word |= e2m1_code(__fdiv_rn(v[j], __uint_as_float(0x7F800000u))) << (4 * j);
    return word;
  }
  const float inv = e8m0_reciprocal(code);
  float q[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) q[j] = __fmul_rn(v[j], inv);
  return e2m1x8(q);
}

// Rows of `in_features` floats; one thread per (row, block of 32).
__global__ void __launch_bounds__(256) mxfp4_quantize_kernel(const float* __restrict__ w, int64_t rows,
                                                             int in_features, uint32_t* __restrict__ codes,
                                                             uint8_t* __restrict__ scales) {
  const int blocks = in_features / 32;
  const int64_t total = rows * blocks;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float4* src = reinterpret_cast<const float4*>(w + t * 32);
    float v[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 f = src[i];
      v[4 * i] = f.x, v[4 * i + 1] = f.y, v[4 * i + 2] = f.z, v[4 * i + 3] = f.w;
    }
    float amax = fabsf(v[0]);
#pragma unroll
    for (int j = 1; j < 31; j += 2) amax = max3_nan(amax, fabsf(v[j]), fabsf(v[j + 1]));
    amax = max_nan(amax, fabsf(v[31]));
    const int code = e8m0_code(amax);
    uint32_t words[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) words[q] = quantize8(v + 8 * q, code);
    scales[t] = static_cast<uint8_t>(code);
    reinterpret_cast<uint4*>(codes)[t] = make_uint4(words[0], words[1], words[2], words[3]);
  }
}

// ---- fused trellis decode + fold + quantise ------------------------------
//
// CTA task = (matrix e, 128-row input chunk, group of 8 output tiles = 128
// columns); warp w takes output tile tn = 8 * group + w and the chunk's eight
// 16x16 tiles, two per 32-row block.  In the tensor-core layout of a decoded
// tile, lane l holds columns c0 = l / 4 and c0 + 8 at rows 2a, 2a+1, 2a+8,
// 2a+9 (a = l % 4): codeword pairs (0,1), (2,3) for c0 and (4,5), (6,7) for
// c0 + 8.  The four lanes of a column reduce the block maximum by shuffles;
// each lane then codes its eight values of a column in a block into one word
// whose byte j is byte a of code word j of that block, and a 4x4 byte
// transpose through shared memory yields the row-major code words.
constexpr int kEncodeWarps = 8;
constexpr int kEncodeThreads = kEncodeWarps * 32;

// Lane `lane`'s word of each of the eight K4 tiles of a task (streamed:
// the words are read once).
__device__ __forceinline__ void load_task_words(const uint32_t* __restrict__ packed, int64_t e, int chunk, int tn,
                                                int in_tiles, int out_tiles, int side, int lane, uint32_t w[8]) {
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const uint32_t* p = packed + tile_index(e, chunk * 8 + t, tn, in_tiles, out_tiles, side) * 32 + lane;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(w[t]) : "l"(p));
  }
}

struct EncodeTask {
  int64_t e;
  int chunk, group;
};

__device__ __forceinline__ EncodeTask encode_task(int64_t task, int chunks, int groups) {
  EncodeTask t;
  t.e = task / (static_cast<int64_t>(chunks) * groups);
  const int rem = static_cast<int>(task - t.e * chunks * groups);
  t.chunk = rem / groups;
  t.group = rem % groups;
  return t;
}

// The raw fold operands of input row i of matrix e (scale, unit), loaded for
// the next task while the current one computes.
__device__ __forceinline__ float2 load_fold(const void* in_scale, const void* unit, int scale_dtype, int64_t e,
                                            int in_features, int64_t i) {
  float2 r;
  if (scale_dtype == kF32) {
    r.x = static_cast<const float*>(in_scale)[e * in_features + i];
    r.y = unit ? static_cast<const float*>(unit)[i] : 1.0f;
  } else {
    const __half s = static_cast<const __half*>(in_scale)[e * in_features + i];
    const __half u = unit ? static_cast<const __half*>(unit)[i] : __float2half(1.0f);
    r.x = __half2float(s);
    r.y = __half2float(u);
  }
  return r;
}

// scale * unit in the scale dtype (fp16 * fp16 rounds to fp16), as float.
__device__ __forceinline__ float fold_product(float2 r, int scale_dtype) {
  if (scale_dtype == kF32) return __fmul_rn(r.x, r.y);
  return __half2float(__hmul(__float2half(r.x), __float2half(r.y)));
}

template <bool kFold, bool kDirectK4>
__global__ void __launch_bounds__(kEncodeThreads) mxfp4_encode_trellis_kernel(
    const uint32_t* __restrict__ packed, int64_t matrices, int k, int in_features, int out_features, int side,
    const void* __restrict__ in_scale, const void* __restrict__ unit, int scale_dtype, uint32_t* __restrict__ codes,
    uint8_t* __restrict__ scales, int64_t rows_per_matrix, int64_t row_offset) {
  __shared__ float fold[128];
  // [warp][column][block * 4 + lane a]; a 20-word column stride keeps the
  // lanes' stores on distinct banks.
  __shared__ __align__(16) uint32_t stage[kEncodeWarps][16][20];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c0 = lane >> 2, a = lane & 3;
  const int in_tiles = in_features / 16, out_tiles = out_features / 16;
  const int chunks = in_features / 128, groups = out_features / 128;
  const int64_t tasks = matrices * chunks * groups;
  const uint32_t nwords = 8u * k;
  const GenericGeometry geo = generic_geometry(k, lane);
  uint32_t cur[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float2 fcur = make_float2(1.0f, 1.0f);
  if (static_cast<int64_t>(blockIdx.x) < tasks) {
    const EncodeTask t0 = encode_task(blockIdx.x, chunks, groups);
    if (kDirectK4) load_task_words(packed, t0.e, t0.chunk, t0.group * 8 + warp, in_tiles, out_tiles, side, lane, cur);
    if (kFold && threadIdx.x < 128)
      fcur = load_fold(in_scale, unit, scale_dtype, t0.e, in_features, static_cast<int64_t>(t0.chunk) * 128 + threadIdx.x);
  }
  for (int64_t task = blockIdx.x; task < tasks; task += gridDim.x) {
    const EncodeTask tk0 = encode_task(task, chunks, groups);
    const int64_t e = tk0.e;
    const int chunk = tk0.chunk;
    const int tn = tk0.group * 8 + warp;
    if (kFold) {
      if (threadIdx.x < 128) fold[threadIdx.x] = fold_product(fcur, scale_dtype);
      __syncthreads();
    }
    // Prefetch the next task's words and fold operands.
    uint32_t nxt[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float2 fnext = make_float2(1.0f, 1.0f);
    const int64_t next = task + gridDim.x;
    if (next < tasks) {
      const EncodeTask tn1 = encode_task(next, chunks, groups);
      if (kDirectK4)
        load_task_words(packed, tn1.e, tn1.chunk, tn1.group * 8 + warp, in_tiles, out_tiles, side, lane, nxt);
      if (kFold && threadIdx.x < 128)
        fnext = load_fold(in_scale, unit, scale_dtype, tn1.e, in_features,
                          static_cast<int64_t>(tn1.chunk) * 128 + threadIdx.x);
    }
    int code[2][4];
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) {
      float v[2][8];  // [column j][tile t * 4 + (rows 2a, 2a+1, 2a+8, 2a+9)]
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        uint32_t cw[8];
        if (kDirectK4) {
          const uint32_t word = cur[blk * 2 + t];
          k4_codewords(word, __shfl_sync(0xffffffffu, word, (lane + 31) & 31), cw);
        } else {
          const int tk = chunk * 8 + blk * 2 + t;
          generic_codewords(packed + tile_index(e, tk, tn, in_tiles, out_tiles, side) * nwords, k, geo, cw);
        }
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {
          const uint32_t h2 = decode_pair(cw[2 * pr], cw[2 * pr + 1]);
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h2));
          v[pr >> 1][t * 4 + (pr & 1) * 2] = f.x;
          v[pr >> 1][t * 4 + (pr & 1) * 2 + 1] = f.y;
        }
        if (kFold) {
          const float2 f0 = *reinterpret_cast<const float2*>(&fold[blk * 32 + t * 16 + 2 * a]);
          const float2 f1 = *reinterpret_cast<const float2*>(&fold[blk * 32 + t * 16 + 2 * a + 8]);
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            v[j][t * 4 + 0] = __fmul_rn(v[j][t * 4 + 0], f0.x);
            v[j][t * 4 + 1] = __fmul_rn(v[j][t * 4 + 1], f0.y);
            v[j][t * 4 + 2] = __fmul_rn(v[j][t * 4 + 2], f1.x);
            v[j][t * 4 + 3] = __fmul_rn(v[j][t * 4 + 3], f1.y);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float amax = max3_nan(fabsf(v[j][0]), fabsf(v[j][1]), fabsf(v[j][2]));
        amax = max3_nan(amax, fabsf(v[j][3]), fabsf(v[j][4]));
        amax = max3_nan(amax, fabsf(v[j][5]), fabsf(v[j][6]));
        amax = max_nan(amax, fabsf(v[j][7]));
        amax = max_nan(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = max_nan(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        code[j][blk] = e8m0_code(amax);
        stage[warp][c0 + 8 * j][blk * 4 + a] = quantize8(v[j], code[j][blk]);
      }
    }
    __syncwarp();
    const int64_t row0 = e * rows_per_matrix + row_offset + static_cast<int64_t>(tn) * 16;
#pragma unroll
    for (int it = 0; it < 2; ++it) {
      const int col = (lane >> 2) + 8 * it, blk = lane & 3;
      const uint4 b = *reinterpret_cast<const uint4*>(&stage[warp][col][blk * 4]);
      const uint32_t lo01 = __byte_perm(b.x, b.y, 0x5140), hi01 = __byte_perm(b.x, b.y, 0x7362);
      const uint32_t lo23 = __byte_perm(b.z, b.w, 0x5140), hi23 = __byte_perm(b.z, b.w, 0x7362);
      const uint4 out = make_uint4(__byte_perm(lo01, lo23, 0x5410), __byte_perm(lo01, lo23, 0x7632),
                                   __byte_perm(hi01, hi23, 0x5410), __byte_perm(hi01, hi23, 0x7632));
      *reinterpret_cast<uint4*>(codes + (row0 + col) * (in_features / 8) + (chunk * 4 + blk) * 4) = out;
    }
    if (a == 0) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint32_t packed_codes = static_cast<uint32_t>(code[j][0]) | (static_cast<uint32_t>(code[j][1]) << 8) |
                                      (static_cast<uint32_t>(code[j][2]) << 16) |
                                      (static_cast<uint32_t>(code[j][3]) << 24);
        *reinterpret_cast<uint32_t*>(scales + (row0 + c0 + 8 * j) * (in_features / 32) + chunk * 4) = packed_codes;
      }
    }
    __syncwarp();
    if (kFold) __syncthreads();  // fold[] is rewritten by the next task
#pragma unroll
    for (int t = 0; t < 8; ++t) cur[t] = nxt[t];
    fcur = fnext;
  }
}

int grid_for(int64_t total) {
  const int64_t want = (total + 255) / 256;
  return static_cast<int>(want < 148 * 16 ? want : 148 * 16);
}

template <bool kFold, bool kDirectK4>
int encode_grid(int64_t tasks) {
  static int per_sm = 0, sms = 0;
  if (per_sm == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mxfp4_encode_trellis_kernel<kFold, kDirectK4>,
                                                      kEncodeThreads, 0) != cudaSuccess ||
        per_sm <= 0) {
      per_sm = 2;
      sms = 148;
    }
  }
  const int64_t resident = static_cast<int64_t>(per_sm) * sms;
  return static_cast<int>(tasks < resident ? tasks : resident);
}

template <bool kFold, bool kDirectK4>
cudaError_t launch_encode(const uint32_t* packed, int64_t matrices, int k, int in_features, int out_features,
                          int side, const void* in_scale, const void* unit, int scale_dtype, uint32_t* codes,
                          uint8_t* scales, int64_t rows_per_matrix, int64_t row_offset, int64_t tasks,
                          cudaStream_t s) {
  mxfp4_encode_trellis_kernel<kFold, kDirectK4><<<encode_grid<kFold, kDirectK4>(tasks), kEncodeThreads, 0, s>>>(
      packed, matrices, k, in_features, out_features, side, in_scale, unit, scale_dtype, codes, scales,
      rows_per_matrix, row_offset);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_mxfp4_quantize(const float* w, int64_t rows, int in_features, uint32_t* codes, uint8_t* scales,
                                  cudaStream_t s) {
  const int64_t total = rows * (in_features / 32);
  if (total == 0) return cudaSuccess;
  mxfp4_quantize_kernel<<<grid_for(total), 256, 0, s>>>(w, rows, in_features, codes, scales);
  return cudaGetLastError();
}

cudaError_t launch_mxfp4_encode_trellis(const uint32_t* packed, int64_t matrices, int k, int in_features,
                                        int out_features, int side, const void* in_scale, const void* unit,
                                        int scale_dtype, uint32_t* codes, uint8_t* scales, int64_t rows_per_matrix,
                                        int64_t row_offset, cudaStream_t s) {
  const int64_t tasks = matrices * (in_features / 128) * (out_features / 128);
  if (tasks == 0) return cudaSuccess;
  const bool fold = in_scale != nullptr;
  if (fold && k == 4)
    return launch_encode<true, true>(packed, matrices, k, in_features, out_features, side, in_scale, unit,
                                     scale_dtype, codes, scales, rows_per_matrix, row_offset, tasks, s);
  if (fold)
    return launch_encode<true, false>(packed, matrices, k, in_features, out_features, side, in_scale, unit,
                                      scale_dtype, codes, scales, rows_per_matrix, row_offset, tasks, s);
  if (k == 4)
    return launch_encode<false, true>(packed, matrices, k, in_features, out_features, side, in_scale, unit,
                                      scale_dtype, codes, scales, rows_per_matrix, row_offset, tasks, s);
  return launch_encode<false, false>(packed, matrices, k, in_features, out_features, side, in_scale, unit,
                                     scale_dtype, codes, scales, rows_per_matrix, row_offset, tasks, s);
}

}  // namespace exlr8
