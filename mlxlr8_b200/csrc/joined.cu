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

#include <type_traits>

#include "common.cuh"
#include "joined.cuh"
#include "mx_gemm.cuh"
#include "trellis_gemv.cuh"

namespace exlr8 {

namespace {

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

// Quantise one 128-value block held in Hadamard layout (value lane + 32 j in
// v[j]) for the hi/lo planes and the block-layout scales.  A warp-private
// shared buffer (128 floats) turns the block around so that lane
// l holds values 4l .. 4l+3: a 32-value scale block is then 8 lanes (three
// shuffles for its maximum) and each plane is one 128-byte warp store.
struct QuantWords {
  uint32_t hi, lo;  // four E4M3 bytes of values 4l .. 4l+3
  int code;         // E8M0 scale of the lane's 32-value block
};

__device__ __forceinline__ QuantWords quantize_words(const float (&v)[4], float* __restrict__ tbuf, int lane) {
#pragma unroll
  for (int j = 0; j < 4; ++j) tbuf[lane + 32 * j] = v[j];
  __syncwarp();
  const float4 q = reinterpret_cast<const float4*>(tbuf)[lane];
  __syncwarp();
  float amax = fmaxf(fmaxf(fabsf(q.x), fabsf(q.y)), fmaxf(fabsf(q.z), fabsf(q.w)));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
  const int code = e8m0_code(amax);
  const float inv = e8m0_inverse(code);
  const float2 s01 = make_float2(q.x * inv, q.y * inv), s23 = make_float2(q.z * inv, q.w * inv);
  const __nv_fp8x2_storage_t h01 = __nv_cvt_float2_to_fp8x2(s01, __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t h23 = __nv_cvt_float2_to_fp8x2(s23, __NV_SATFINITE, __NV_E4M3);
  const float2 b01 = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(h01, __NV_E4M3)));
  const float2 b23 = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(h23, __NV_E4M3)));
  const __nv_fp8x2_storage_t l01 =
      __nv_cvt_float2_to_fp8x2(make_float2(s01.x - b01.x, s01.y - b01.y), __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t l23 =
      __nv_cvt_float2_to_fp8x2(make_float2(s23.x - b23.x, s23.y - b23.y), __NV_SATFINITE, __NV_E4M3);
  QuantWords w;
  w.hi = static_cast<uint32_t>(h01) | (static_cast<uint32_t>(h23) << 16);
  w.lo = static_cast<uint32_t>(l01) | (static_cast<uint32_t>(l23) << 16);
  w.code = code;
  return w;
}

__device__ __forceinline__ void store_words(const QuantWords& w, int64_t row, int block, int features,
                                            uint8_t* __restrict__ hi, uint8_t* __restrict__ lo,
                                            uint8_t* __restrict__ scales, int lane) {
  const int64_t base = row * features + block * 128 + 4 * lane;
  *reinterpret_cast<uint32_t*>(hi + base) = w.hi;
  *reinterpret_cast<uint32_t*>(lo + base) = w.lo;
  if ((lane & 7) == 0) scales[mx_scale_offset(row, 4 * block + (lane >> 3), features / 32)] = static_cast<uint8_t>(w.code);
}

}  // namespace

// ---------------------------------------------------------------------------
// Segments: one CTA.  Expert e's sorted rows start at padded_start[e] (a
// multiple of kMxRowAlign); an expert with at most kMxMaxN rows is one chunk,
// a larger one is cut into 128-row chunks and a last chunk of 33..160 rows.
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

constexpr int kRowWarps = 8;     // warps per CTA of the row kernels
constexpr int kBlockGroup = 8;   // 128-blocks per warp item of the row kernels

// xh = H(x[token] * unit), quantised once per token and stored into the
// padded row of each of the token's slots.  Padding rows are left as they
// are: they only feed MMA columns whose results are never stored.
template <int kAct, int kScale>
__global__ void __launch_bounds__(kRowWarps * 32) joined_prep_kernel(const void* __restrict__ x,
                                                                     const void* __restrict__ unit,
                                                                     int slots_per_token, int tokens, MxChunks c,
                                                                     int hidden, uint8_t* __restrict__ hi,
                                                                     uint8_t* __restrict__ lo,
                                                                     uint8_t* __restrict__ scales) {
  __shared__ __align__(16) float tbuf[kRowWarps][128];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int blocks = hidden / 128;
  const int groups = (blocks + kBlockGroup - 1) / kBlockGroup;
  const int64_t items = static_cast<int64_t>(tokens) * groups;
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * kRowWarps + warp; item < items;
       item += static_cast<int64_t>(gridDim.x) * kRowWarps) {
    const int token = static_cast<int>(item / groups);
    const int b0 = static_cast<int>(item % groups) * kBlockGroup, b1 = min(b0 + kBlockGroup, blocks);
    const int my_row = lane < slots_per_token ? c.slot_row[static_cast<int64_t>(token) * slots_per_token + lane] : -1;
    const int64_t xrow = static_cast<int64_t>(token) * hidden;
    for (int block = b0; block < b1; ++block) {
      float v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = block * 128 + lane + 32 * j;
        v[j] = __fmul_rn(load_act(x, kAct, xrow + col), load_scale(unit, kScale, col));
      }
      hadamard128(v, lane);
      const QuantWords w = quantize_words(v, tbuf[warp], lane);
      for (int r = 0; r < slots_per_token; ++r) {
        const int row = __shfl_sync(0xffffffffu, my_row, r);
        if (row >= 0) store_words(w, row, block, hidden, hi, lo, scales, lane);
      }
    }
  }
}

// Trellis prefill inputs (fast_prefill.py:188-211 prep): per slot and
// projection p, H(x[row] * in_scale_p[e]) quantised into the slot's padded
// row of plane set p.  One warp per slot; x row = slot (per_slot) or
// slot / slots_per_token.
template <int kAct, int kScale>
__global__ void __launch_bounds__(kRowWarps * 32) trellis_prep_kernel(
    const void* __restrict__ x, int per_slot, int slots_per_token, int nslots, const uint32_t* __restrict__ ids,
    MxChunks c, const void* __restrict__ in0, const void* __restrict__ in1, int projections, int hidden,
    uint8_t* __restrict__ hi0, uint8_t* __restrict__ lo0, uint8_t* __restrict__ sc0, uint8_t* __restrict__ hi1,
    uint8_t* __restrict__ lo1, uint8_t* __restrict__ sc1) {
  __shared__ __align__(16) float tbuf[kRowWarps][128];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int blocks = hidden / 128;
  const int groups = (blocks + kBlockGroup - 1) / kBlockGroup;
  const int64_t items = static_cast<int64_t>(nslots) * groups;
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * kRowWarps + warp; item < items;
       item += static_cast<int64_t>(gridDim.x) * kRowWarps) {
    const int slot = static_cast<int>(item / groups);
    const int b0 = static_cast<int>(item % groups) * kBlockGroup, b1 = min(b0 + kBlockGroup, blocks);
    const int row = c.slot_row[slot];
    if (row < 0) continue;
    const int64_t e = ids[slot];
    const int64_t xrow = static_cast<int64_t>(per_slot ? slot : slot / slots_per_token) * hidden;
    for (int block = b0; block < b1; ++block) {
      float xv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) xv[j] = load_act(x, kAct, xrow + block * 128 + lane + 32 * j);
      for (int p = 0; p < projections; ++p) {
        const void* in = p ? in1 : in0;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          v[j] = __fmul_rn(xv[j], load_scale(in, kScale, e * hidden + block * 128 + lane + 32 * j));
        hadamard128(v, lane);
        store_words(quantize_words(v, tbuf[warp], lane), row, block, hidden, p ? hi1 : hi0, p ? lo1 : lo0,
                    p ? sc1 : sc0, lane);
      }
    }
  }
}

// metal/joined_gate_finish.metal: gate and up halves of the joined product,
// Hadamard, out scales, typed SwiGLU, down in scale, Hadamard; quantised into
// the down GEMM's activation planes.  One warp per padded row.
template <int kAct, int kScale>
__global__ void __launch_bounds__(kRowWarps * 32, 5) joined_gate_finish_kernel(
    const float* __restrict__ gu, const uint32_t* __restrict__ ids, int slots, MxChunks c,
    const void* __restrict__ gate_out, const void* __restrict__ up_out, const void* __restrict__ down_in,
    int intermediate, uint8_t* __restrict__ hi, uint8_t* __restrict__ lo, uint8_t* __restrict__ scales) {
  __shared__ __align__(16) float tbuf[kRowWarps][128];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int blocks = intermediate / 128;
  const int groups = (blocks + kBlockGroup - 1) / kBlockGroup;
  const int64_t items = static_cast<int64_t>(slots) * groups;
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * kRowWarps + warp; item < items;
       item += static_cast<int64_t>(gridDim.x) * kRowWarps) {
    const int slot = static_cast<int>(item / groups);
    const int b0 = static_cast<int>(item % groups) * kBlockGroup, b1 = min(b0 + kBlockGroup, blocks);
    const int row = c.slot_row[slot];
    if (row < 0) continue;
    const int64_t e = ids[slot];
    const float* g_row = gu + static_cast<int64_t>(row) * 2 * intermediate + lane;
    for (int block = b0; block < b1; ++block) {
      // The block's gate and up values and its three scale vectors' entries
      // go out together (one round trip per block).
      float g[4], u[4], h[4], sg[4], su[4], sd[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        g[j] = __ldcs(g_row + block * 128 + 32 * j);
        u[j] = __ldcs(g_row + intermediate + block * 128 + 32 * j);
        const int64_t si = e * intermediate + block * 128 + lane + 32 * j;
        sg[j] = load_scale(gate_out, kScale, si);
        su[j] = load_scale(up_out, kScale, si);
        sd[j] = load_scale(down_in, kScale, si);
      }
      hadamard128(g, lane);
      hadamard128(u, lane);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float act = swiglu_typed(kAct, __fmul_rn(g[j], sg[j]), __fmul_rn(u[j], su[j]));
        h[j] = __fmul_rn(act, sd[j]);
      }
      hadamard128(h, lane);
      store_words(quantize_words(h, tbuf[warp], lane), row, block, intermediate, hi, lo, scales, lane);
    }
  }
}

// JoinedMXFP4.finish for prefill batches: one CTA (nine warps, one per slot)
// per token and group of four 128-blocks.  Per slot T(H(v) * down_out[e]);
// then the routed sum in the order of metal/fast_decode_finish_fused.metal
// (slot 0, then (slot r + 0) + total for r = 1..7), T(routed),
// T(routed + shared) and T(residual + combined).
constexpr int kFinishGroup = 4;

template <int kAct, int kScale>
__global__ void __launch_bounds__(288) joined_finish_kernel(const float* __restrict__ v,
                                                            const int32_t* __restrict__ slot_row,
                                                            const uint32_t* __restrict__ ids, int features,
                                                            int experts, const void* __restrict__ out_scale,
                                                            const float* __restrict__ scores,
                                                            const void* __restrict__ residual,
                                                            const float* __restrict__ shared_values, int shared_splits,
                                                            int tokens, void* __restrict__ out) {
  __shared__ float products[9][kFinishGroup * 128];
  const int lane = threadIdx.x & 31, slot = threadIdx.x >> 5;
  const int64_t token = blockIdx.x;
  const bool dense_shared = slot == 8 && shared_values != nullptr;
  const int64_t e = ids[token * 9 + slot];
  const int prow = dense_shared ? -1 : slot_row[token * 9 + slot];
  const bool ok = e < experts && prow >= 0;
  const float score = slot < 8 ? scores[token * 8 + slot] : 1.0f;
  const float* src = v + static_cast<int64_t>(ok ? prow : 0) * features + lane;
  const int blocks = features / 128;
  {
    const int b0 = blockIdx.y * kFinishGroup;
    const int nb = min(kFinishGroup, blocks - b0);
    // The residual of the (at most two) columns this thread sums below, loaded
    // with the slot rows so that the sum phase waits on no memory.
    const int64_t base = token * features + b0 * 128;
    const int c_a = threadIdx.x, c_b = threadIdx.x + 288;
    const float res_a = c_a < nb * 128 ? load_act(residual, kAct, base + c_a) : 0.0f;
    const float res_b = c_b < nb * 128 ? load_act(residual, kAct, base + c_b) : 0.0f;
    if (dense_shared) {
      // Dense shared expert: float32 split partials [splits][tokens][h], summed
      // in split order and cast.  The group's sixteen values of one split go
      // out together: one round trip per split, not per value.  (A branch of
      // its own, one split in flight: the slot warps' registers stay those of
      // the slot path alone.)
      const int64_t total = static_cast<int64_t>(tokens) * features;
      const float* part = shared_values + base + lane;
      float acc[kFinishGroup][4];
#pragma unroll
      for (int g = 0; g < kFinishGroup; ++g)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[g][j] = 0.f;
#pragma unroll 1
      for (int sp = 0; sp < shared_splits; ++sp) {
        float q[kFinishGroup][4];
#pragma unroll
        for (int g = 0; g < kFinishGroup; ++g)
#pragma unroll
          for (int j = 0; j < 4; ++j) q[g][j] = g < nb ? __ldcg(part + sp * total + g * 128 + 32 * j) : 0.f;
#pragma unroll
        for (int g = 0; g < kFinishGroup; ++g)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[g][j] += q[g][j];
      }
#pragma unroll
      for (int g = 0; g < kFinishGroup; ++g)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (g < nb) products[8][g * 128 + lane + 32 * j] = round_to(kAct, acc[g][j]);
    } else {
      float val[kFinishGroup][4];
#pragma unroll
      for (int g = 0; g < kFinishGroup; ++g)
#pragma unroll
        for (int j = 0; j < 4; ++j) val[g][j] = (ok && g < nb) ? __ldcs(src + (b0 + g) * 128 + 32 * j) : 0.0f;
#pragma unroll
      for (int g = 0; g < kFinishGroup; ++g) {
        if (g >= nb) break;
        hadamard128(val[g], lane);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int col = (b0 + g) * 128 + lane + 32 * j;
          const float value =
              ok ? round_to(kAct, __fmul_rn(val[g][j], load_scale(out_scale, kScale, e * features + col))) : 0.0f;
          products[slot][g * 128 + lane + 32 * j] = slot < 8 ? __fmul_rn(value, score) : value;
        }
      }
    }
    __syncthreads();
    static_assert(kFinishGroup * 128 <= 2 * 288, "two columns per thread cover the group");
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = h ? c_b : c_a;
      if (c >= nb * 128) break;
      float total = __fadd_rn(products[0][c], 0.0f);
#pragma unroll
      for (int r = 1; r < 8; ++r) total = __fadd_rn(__fadd_rn(products[r][c], 0.0f), total);
      const float routed = round_to(kAct, total);
      const float combined = round_to(kAct, __fadd_rn(routed, round_to(kAct, products[8][c])));
      store_act(out, kAct, base + c, __fadd_rn(h ? res_b : res_a, combined));
    }
    __syncthreads();
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

template <typename F>
static cudaError_t dispatch_types(int act_dtype, int scale_dtype, F&& f) {
  const bool f16s = scale_dtype == kF16;
  switch (act_dtype) {
    case kF32: return f16s ? f(std::integral_constant<int, kF32>{}, std::integral_constant<int, kF16>{})
                           : f(std::integral_constant<int, kF32>{}, std::integral_constant<int, kF32>{});
    case kF16: return f16s ? f(std::integral_constant<int, kF16>{}, std::integral_constant<int, kF16>{})
                           : f(std::integral_constant<int, kF16>{}, std::integral_constant<int, kF32>{});
    default: return f16s ? f(std::integral_constant<int, kBF16>{}, std::integral_constant<int, kF16>{})
                         : f(std::integral_constant<int, kBF16>{}, std::integral_constant<int, kF32>{});
  }
}

cudaError_t launch_joined_prep(const void* x, int act_dtype, const void* unit, int scale_dtype, int slots_per_token,
                               int tokens, MxChunks c, int hidden, uint8_t* hi, uint8_t* lo, uint8_t* scales,
                               cudaStream_t s) {
  return dispatch_types(act_dtype, scale_dtype, [&](auto a, auto sc) {
    joined_prep_kernel<decltype(a)::value, decltype(sc)::value>
        <<<worker_grid(), kRowWarps * 32, 0, s>>>(x, unit, slots_per_token, tokens, c, hidden, hi, lo, scales);
    return cudaGetLastError();
  });
}

cudaError_t launch_joined_gate_finish(const float* gu, const uint32_t* ids, int slots, MxChunks c,
                                      const void* gate_out, const void* up_out, const void* down_in, int scale_dtype,
                                      int intermediate, int act_dtype, uint8_t* hi, uint8_t* lo, uint8_t* scales,
                                      cudaStream_t s) {
  return dispatch_types(act_dtype, scale_dtype, [&](auto a, auto sc) {
    joined_gate_finish_kernel<decltype(a)::value, decltype(sc)::value>
        <<<worker_grid(), kRowWarps * 32, 0, s>>>(gu, ids, slots, c, gate_out, up_out, down_in, intermediate, hi,
                                                  lo, scales);
    return cudaGetLastError();
  });
}

cudaError_t launch_joined_finish(const float* v, const int32_t* slot_row, const uint32_t* ids, int tokens,
                                 int features, int experts, const void* out_scale, int scale_dtype,
                                 const float* scores, const void* residual, const float* shared_values,
                                 int shared_splits, int act_dtype, void* out, cudaStream_t s) {
  if (tokens == 0) return cudaSuccess;
  return dispatch_types(act_dtype, scale_dtype, [&](auto a, auto sc) {
    const dim3 grid(tokens, (features / 128 + kFinishGroup - 1) / kFinishGroup);
    joined_finish_kernel<decltype(a)::value, decltype(sc)::value><<<grid, 288, 0, s>>>(
        v, slot_row, ids, features, experts, out_scale, scores, residual, shared_values, shared_splits, tokens, out);
    return cudaGetLastError();
  });
}

cudaError_t launch_trellis_prep(const void* x, int act_dtype, int per_slot, int slots_per_token, int nslots,
                                const uint32_t* ids, MxChunks c, const void* in0, const void* in1, int scale_dtype,
                                int projections, int hidden, uint8_t* hi0, uint8_t* lo0, uint8_t* sc0, uint8_t* hi1,
                                uint8_t* lo1, uint8_t* sc1, cudaStream_t s) {
  return dispatch_types(act_dtype, scale_dtype, [&](auto a, auto sc) {
    trellis_prep_kernel<decltype(a)::value, decltype(sc)::value><<<worker_grid(), kRowWarps * 32, 0, s>>>(
        x, per_slot, slots_per_token, nslots, ids, c, in0, in1, projections, hidden, hi0, lo0, sc0, hi1, lo1, sc1);
    return cudaGetLastError();
  });
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
