// Joined MXFP4 expert path (exlr8 joined_mxfp4.py): dispatch segments for the
// grouped tcgen05 GEMM, activation preparation, the fused gate/up finish and
// the weight scale re-layout.
//
//   joined_segment_kernel     -- segments of the expert-sorted slots
//                                (the grouping of MLX gather_qmm's sorted
//                                RHS indices, joined_mxfp4.py:98-104)
//   joined_rowmap_kernel      -- padded row <-> slot maps
//   joined_prep_kernel        -- xh = H(x * unit) (joined_mxfp4.py:96,
//                                metal/fast_decode_prep.metal) quantised
//                                for the GEMM
//   joined_gate_finish_kernel -- metal/joined_gate_finish.metal, quantised
//                                for the down GEMM
//   mx_prepare_scales_kernel  -- E8M0 [rows][k/32] -> 512-byte block layout
//
// GEMM activations are two E4M3 planes (hi, lo) that share one E8M0 scale
// per 32 values: s = 2^e with amax / s <= 448, hi = e4m3(v / s),
// lo = e4m3(v / s - hi).  hi + lo keeps about eight significant bits of
// every value relative to its block maximum, so the float32-accumulated
// products stay within 1e-3 of the float32 reference path.

#include <cuda_fp8.h>

#include "common.cuh"
#include "joined.cuh"
#include "mx_gemm.cuh"
#include "trellis_gemv.cuh"

namespace exlr8 {

namespace {

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// E8M0 code of the smallest power of two s with amax / s <= 448.
__device__ __forceinline__ int e8m0_code(float amax) {
  if (!(amax > 0.f)) return 1;                  // zero block (or NaN): any scale, values are zero
  if (!(amax < 3.0e38f)) return 254;            // overflow: saturate
  const uint32_t bits = __float_as_uint(amax);
  int e = static_cast<int>((bits >> 23) & 0xFFu) - 127;
  if (e == -127) return 1;                      // float32 subnormal block maximum
  e += ((bits & 0x7FFFFFu) > 0x600000u) ? -7 : -8;  // mantissa above 1.75 needs one more binade
  const int code = e + 127;
  return code < 1 ? 1 : (code > 254 ? 254 : code);
}

// 2^(127 - code) for code in [1, 254].
__device__ __forceinline__ float e8m0_inverse(int code) {
  return code <= 253 ? __uint_as_float(static_cast<uint32_t>(254 - code) << 23) : __uint_as_float(0x00400000u);
}

__device__ __forceinline__ uint8_t to_e4m3(float v) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}

__device__ __forceinline__ float from_e4m3(uint8_t b) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(b), __NV_E4M3);
  return __half2float(__half(h));
}

// Quantise one 128-value block held in Hadamard layout (value lane + 32 j in
// v[j]) into row `row` of the hi/lo planes and the block-layout scales.
__device__ __forceinline__ void quantize_block(const float (&v)[4], int64_t row, int block, int features,
                                               uint8_t* __restrict__ hi, uint8_t* __restrict__ lo,
                                               uint8_t* __restrict__ scales, int lane) {
  const int64_t base = row * features + block * 128 + lane;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int code = e8m0_code(warp_max(fabsf(v[j])));
    const float scaled = v[j] * e8m0_inverse(code);
    const uint8_t h = to_e4m3(scaled);
    const uint8_t l = to_e4m3(scaled - from_e4m3(h));
    hi[base + 32 * j] = h;
    lo[base + 32 * j] = l;
    if (lane == j) scales[mx_scale_offset(row, 4 * block + j, features / 32)] = static_cast<uint8_t>(code);
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// Segments: one CTA.  Expert e's sorted rows start at padded_start[e] (a
// multiple of kMxRowAlign); an expert with at most kMxMaxN rows is one chunk,
// a larger one is cut into 128-row chunks and a last chunk of 113..240 rows.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int chunk_count(int rows) {
  if (rows <= 0) return 0;
  if (rows <= kMxMaxN) return 1;
  return (rows - kMxMaxN + kMxRowAlign - 1) / kMxRowAlign + 1;
}

__global__ void __launch_bounds__(1024) joined_segment_kernel(PlanView plan, int experts, MxChunks c) {
  __shared__ int s_pad[1024], s_chunk[1024];
  const int tid = threadIdx.x;
  // Blocked exclusive scans over experts (experts <= 32 * 1024 handled by
  // one pass per 1024 experts with a running carry).
  int pad_carry = 0, chunk_carry = 0;
  for (int e0 = 0; e0 < experts; e0 += 1024) {
    const int e = e0 + tid;
    const int rows = e < experts ? plan.expert_count[e] : 0;
    const int pad = (rows + kMxRowAlign - 1) / kMxRowAlign * kMxRowAlign;
    const int nch = chunk_count(rows);
    s_pad[tid] = pad;
    s_chunk[tid] = nch;
    __syncthreads();
    for (int off = 1; off < 1024; off <<= 1) {
      const int a = tid >= off ? s_pad[tid - off] : 0;
      const int b = tid >= off ? s_chunk[tid - off] : 0;
      __syncthreads();
      s_pad[tid] += a;
      s_chunk[tid] += b;
      __syncthreads();
    }
    const int pad_start = pad_carry + s_pad[tid] - pad;
    const int chunk_start = chunk_carry + s_chunk[tid] - nch;
    if (e < experts) {
      c.padded_start[e] = pad_start;
      for (int k = 0; k < nch; ++k) {
        const int first = k * kMxRowAlign;
        c.chunk_expert[chunk_start + k] = e;
        c.chunk_start[chunk_start + k] = pad_start + first;
        c.chunk_rows[chunk_start + k] = (k == nch - 1) ? rows - first : kMxRowAlign;
      }
    }
    pad_carry += s_pad[1023];
    chunk_carry += s_chunk[1023];
    __syncthreads();
  }
  if (tid == 0) {
    c.padded_start[experts] = pad_carry;
    c.header[0] = chunk_carry;
    c.header[1] = pad_carry;
    c.header[2] = 0;
    c.header[3] = 0;
    c.header[4] = 0;
  }
}

// One CTA per expert: row_slot over the expert's padded segment, slot_row for
// its slots (slot_row starts as -1 for slots outside every expert).
__global__ void __launch_bounds__(256) joined_rowmap_kernel(PlanView plan, MxChunks c) {
  const int e = blockIdx.x;
  const int rows = plan.expert_count[e];
  const int first = plan.expert_start[e];
  const int pad_start = c.padded_start[e];
  const int pad = (rows + kMxRowAlign - 1) / kMxRowAlign * kMxRowAlign;
  for (int i = threadIdx.x; i < pad; i += blockDim.x) {
    const int slot = i < rows ? plan.order[first + i] : -1;
    c.row_slot[pad_start + i] = slot;
    if (slot >= 0) c.slot_row[slot] = pad_start + i;
  }
}

// xh = H(x[token] * unit) for every padded row (zeros for padding), one warp
// per (row, 128-block).
__global__ void __launch_bounds__(256) joined_prep_kernel(const void* __restrict__ x, int act_dtype,
                                                          const void* __restrict__ unit, int scale_dtype,
                                                          int slots_per_token, MxChunks c, int hidden,
                                                          uint8_t* __restrict__ hi, uint8_t* __restrict__ lo,
                                                          uint8_t* __restrict__ scales) {
  const int lane = threadIdx.x & 31;
  const int blocks = hidden / 128;
  const int64_t items = static_cast<int64_t>(c.header[1]) * blocks;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); item < items;
       item += warps) {
    const int64_t row = item / blocks;
    const int block = static_cast<int>(item % blocks);
    const int slot = c.row_slot[row];
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (slot >= 0) {
      const int64_t token = slot / slots_per_token;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = block * 128 + lane + 32 * j;
        v[j] = __fmul_rn(load_act(x, act_dtype, token * hidden + col), load_scale(unit, scale_dtype, col));
      }
      hadamard128(v, lane);
    }
    quantize_block(v, row, block, hidden, hi, lo, scales, lane);
  }
}

// metal/joined_gate_finish.metal: gate and up halves of the joined product,
// Hadamard, out scales, typed SwiGLU, down in scale, Hadamard; quantised into
// the down GEMM's activation planes.
__global__ void __launch_bounds__(256) joined_gate_finish_kernel(
    const float* __restrict__ gu, const uint32_t* __restrict__ ids, MxChunks c, const void* __restrict__ gate_out,
    const void* __restrict__ up_out, const void* __restrict__ down_in, int scale_dtype, int intermediate, int act_dtype,
    uint8_t* __restrict__ hi, uint8_t* __restrict__ lo, uint8_t* __restrict__ scales) {
  const int lane = threadIdx.x & 31;
  const int blocks = intermediate / 128;
  const int64_t items = static_cast<int64_t>(c.header[1]) * blocks;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); item < items;
       item += warps) {
    const int64_t row = item / blocks;
    const int block = static_cast<int>(item % blocks);
    const int slot = c.row_slot[row];
    float h[4] = {0.f, 0.f, 0.f, 0.f};
    if (slot >= 0) {
      const int64_t e = ids[slot];
      const float* g_row = gu + row * 2 * intermediate + block * 128 + lane;
      float g[4], u[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        g[j] = __ldcs(g_row + 32 * j);
        u[j] = __ldcs(g_row + intermediate + 32 * j);
      }
      hadamard128(g, lane);
      hadamard128(u, lane);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t si = e * intermediate + block * 128 + lane + 32 * j;
        const float act = swiglu_typed(act_dtype, __fmul_rn(g[j], load_scale(gate_out, scale_dtype, si)),
                                       __fmul_rn(u[j], load_scale(up_out, scale_dtype, si)));
        h[j] = __fmul_rn(act, load_scale(down_in, scale_dtype, si));
      }
      hadamard128(h, lane);
    }
    quantize_block(h, row, block, intermediate, hi, lo, scales, lane);
  }
}

// E8M0 scales [rows][k/32] -> block layout [rows/128][k/128][512].
__global__ void mx_prepare_scales_kernel(const uint8_t* __restrict__ in, int64_t rows, int kblocks,
                                         uint8_t* __restrict__ out) {
  const int64_t n = rows * kblocks;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / kblocks;
    const int64_t kb = i % kblocks;
    out[mx_scale_offset(r, kb, kblocks)] = in[i];
  }
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------

static int worker_grid() {
  static int grid = 0;
  if (grid == 0) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    grid = sms * 8;
  }
  return grid;
}

cudaError_t launch_joined_segments(PlanView plan, int experts, int slots, MxChunks c, cudaStream_t s) {
  cudaError_t err = cudaMemsetAsync(c.slot_row, 0xFF, static_cast<size_t>(slots) * sizeof(int32_t), s);
  if (err != cudaSuccess) return err;
  joined_segment_kernel<<<1, 1024, 0, s>>>(plan, experts, c);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  joined_rowmap_kernel<<<experts, 256, 0, s>>>(plan, c);
  return cudaGetLastError();
}

cudaError_t launch_joined_prep(const void* x, int act_dtype, const void* unit, int scale_dtype, int slots_per_token,
                               MxChunks c, int hidden, uint8_t* hi, uint8_t* lo, uint8_t* scales, cudaStream_t s) {
  joined_prep_kernel<<<worker_grid(), 256, 0, s>>>(x, act_dtype, unit, scale_dtype, slots_per_token, c, hidden, hi,
                                                   lo, scales);
  return cudaGetLastError();
}

cudaError_t launch_joined_gate_finish(const float* gu, const uint32_t* ids, MxChunks c, const void* gate_out,
                                      const void* up_out, const void* down_in, int scale_dtype, int intermediate,
                                      int act_dtype, uint8_t* hi, uint8_t* lo, uint8_t* scales, cudaStream_t s) {
  joined_gate_finish_kernel<<<worker_grid(), 256, 0, s>>>(gu, ids, c, gate_out, up_out, down_in, scale_dtype,
                                                          intermediate, act_dtype, hi, lo, scales);
  return cudaGetLastError();
}

cudaError_t launch_mx_prepare_scales(const uint8_t* in, int64_t rows, int kblocks, uint8_t* out, cudaStream_t s) {
  const int64_t n = rows * kblocks;
  if (n == 0) return cudaSuccess;
  const int64_t want = (n + 255) / 256;
  const unsigned grid = static_cast<unsigned>(want < 65535 ? want : 65535);
  mx_prepare_scales_kernel<<<grid, 256, 0, s>>>(in, rows, kblocks, out);
  return cudaGetLastError();
}

}  // namespace exlr8
