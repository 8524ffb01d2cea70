// Trellis expert kernels around the streaming GEMV (trellis_stream.cu):
// dispatch plan, activation fragments, gate/up finish and output finishes.
//
// Reference roles (exlr8 v0.1.21):
//   plan_kernel             -- fast_prefill.py:19-46 (sort slots by expert, segments)
//   prep_frag_kernel        -- metal/fast_decode_prep.metal (x * in_scale, Hadamard-128)
//   gate_finish_frag_kernel -- metal/fast_decode_gate_finish.metal
//   finish_kernel           -- metal/fast_decode_finish.metal
//   finish_fused_kernel     -- metal/fast_decode_finish_fused.metal
//
// Activations reach the tensor cores as float16 hi/lo pieces (hi = f16(v),
// lo = f16(v - hi)) of the value times a power-of-two scale chosen per
// (row, K split), so products keep about 22 significant bits and the
// float32 accumulation sees the full range.

#include "common.cuh"
#include "codec.cuh"
#include "stream.cuh"
#include "trellis_gemv.cuh"
#include "plan.cuh"

namespace exlr8 {

// ---------------------------------------------------------------------------
// Plan
// ---------------------------------------------------------------------------

static inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

size_t plan_bytes(int rows, int experts) {
  size_t n = 16;                              // header
  n += static_cast<size_t>(rows);             // order
  n += 3 * static_cast<size_t>(rows);         // groups (at most one per row)
  n += 2 * static_cast<size_t>(experts);      // expert count / start
  return align_up(n * sizeof(int32_t), 256);
}

PlanView plan_view(void* base, int rows, int experts) {
  PlanView v;
  int32_t* p = static_cast<int32_t*>(base);
  v.header = p;
  p += 16;
  v.order = p;
  p += rows;
  v.group_expert = p;
  p += rows;
  v.group_start = p;
  p += rows;
  v.group_count = p;
  p += rows;
  v.expert_count = p;
  p += experts;
  v.expert_start = p;
  v.zero = nullptr;
  v.zero_count = 0;
  return v;
}

constexpr int kPlanThreads = 1024;

__global__ void __launch_bounds__(kPlanThreads) plan_kernel(const uint32_t* __restrict__ ids, int rows,
                                                            int experts, int period, int skip_slot, PlanView plan) {
  extern __shared__ int sm[];
  plan_body(ids, rows, experts, period, skip_slot, plan, sm);
}

cudaError_t launch_plan(const uint32_t* ids, int rows, int experts, int period, int skip_slot, PlanView plan,
                        cudaStream_t s) {
  const size_t smem = plan_smem_bytes(experts, kPlanThreads / 32);
  if (smem > 48 * 1024) {
    cudaError_t err = cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
    if (err != cudaSuccess) return err;
  }
  plan_kernel<<<1, kPlanThreads, smem, s>>>(ids, rows, experts, period > 0 ? period : 1, skip_slot, plan);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Activation fragments.  One CTA per (K split, slot, projection): the split's
// 128-wide blocks are transformed into shared memory, the split maximum picks
// a power-of-two scale, and the scaled values are written as float16 hi/lo
// B fragments (see stream.cuh).
// ---------------------------------------------------------------------------

constexpr int kFragThreads = 256;

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float split_piece(float v, int piece) {
  const float hi = __half2float(__float2half_rn(v));
  return piece ? v - hi : hi;
}

// Scale exponent for a split maximum: the scaled maximum lies in [2^14, 2^15).
__device__ __forceinline__ int piece_exponent(float m) {
  int ex = 0;
  if (m > 0.0f && m < 3.0e38f) {
    frexpf(m, &ex);
    ex -= 15;
  }
  return ex;
}

// vals: the split's transformed values (kt_count*16 floats) in shared memory.
__device__ __forceinline__ void write_fragments(const float* vals, int kt_count, float scale, uint2* dst) {
  for (int idx = threadIdx.x; idx < kt_count * 8; idx += blockDim.x) {
    const int ktl = idx >> 3, piece = (idx >> 2) & 1, tig = idx & 3;
    const float* v = vals + ktl * 16;
    uint2 b;
    b.x = pack_half2(split_piece(v[2 * tig] * scale, piece), split_piece(v[2 * tig + 1] * scale, piece));
    b.y = pack_half2(split_piece(v[2 * tig + 8] * scale, piece), split_piece(v[2 * tig + 9] * scale, piece));
    dst[idx] = b;
  }
}

__device__ __forceinline__ float block_max(float m, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  float r = 0.0f;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) r = fmaxf(r, red[w]);
  return r;
}

__global__ void __launch_bounds__(kFragThreads) prep_frag_kernel(
    const void* __restrict__ x, int x_dtype, int per_slot, int slots_per_token, const uint32_t* __restrict__ ids,
    int nslots, const void* __restrict__ in0, const void* __restrict__ in1, int scale_dtype, int features,
    int experts, int kt_split, int splits, uint2* __restrict__ frag, float* __restrict__ unscale) {
  extern __shared__ float vals[];
  __shared__ float red[kFragThreads / 32];
  const int split = blockIdx.x, slot = blockIdx.y, proj = blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int it = features / 16;
  const int kt0 = split * kt_split;
  const int kt_count = min(kt_split, it - kt0);
  const uint32_t e = ids[slot];
  const bool ok = e < static_cast<uint32_t>(experts);
  const int64_t row = per_slot ? slot : slot / slots_per_token;
  const void* scale = proj ? in1 : in0;
  float m = 0.0f;
  for (int b = warp; b < kt_count / 8; b += kFragThreads / 32) {
    const int c0 = kt0 * 16 + b * 128;
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = c0 + lane + 32 * j;
      v[j] = ok ? __fmul_rn(load_act(x, x_dtype, row * features + col),
                            load_scale(scale, scale_dtype, static_cast<int64_t>(e) * features + col))
                : 0.0f;
    }
    hadamard128(v, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      vals[b * 128 + lane + 32 * j] = v[j];
      m = fmaxf(m, fabsf(v[j]));
    }
  }
  const float mx = block_max(m, red);  // contains the barrier that publishes vals
  const int ex = piece_exponent(mx);
  const int64_t rbase = static_cast<int64_t>(proj) * nslots + slot;
  write_fragments(vals, kt_count, ldexpf(1.0f, -ex), frag + (rbase * it + kt0) * 8);
  if (threadIdx.x == 0) unscale[rbase * splits + split] = ldexpf(1.0f, ex);
}

cudaError_t launch_prep_frag(const void* x, int x_dtype, int per_slot, int slots_per_token, const uint32_t* ids,
                             int nslots, const void* in0, const void* in1, int scale_dtype, int features, int experts,
                             int projections, int kt_split, int splits, uint2* frag, float* unscale, cudaStream_t s) {
  const size_t smem = static_cast<size_t>(kt_split) * 16 * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t err =
        cudaFuncSetAttribute(prep_frag_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (err != cudaSuccess) return err;
  }
  dim3 grid(splits, nslots, projections);
  prep_frag_kernel<<<grid, kFragThreads, smem, s>>>(x, x_dtype, per_slot, slots_per_token, ids, nslots, in0, in1,
                                                     scale_dtype, features, experts, kt_split, splits, frag, unscale);
  return cudaGetLastError();
}

// gate/up split sum, Hadamard, output scales, typed SwiGLU, down input scale,
// Hadamard -> down fragments.  One CTA per (down K split, slot).
__global__ void __launch_bounds__(kFragThreads) gate_finish_frag_kernel(
    const float* __restrict__ partial, int gu_splits, const uint32_t* __restrict__ ids, int nslots,
    const void* __restrict__ out_gate, const void* __restrict__ out_up, const void* __restrict__ in_down,
    int scale_dtype, int features, int experts, int act_dtype, int kt_split, int splits, uint2* __restrict__ frag,
    float* __restrict__ unscale) {
  extern __shared__ float vals[];
  __shared__ float red[kFragThreads / 32];
  const int split = blockIdx.x, slot = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int it = features / 16;
  const int kt0 = split * kt_split;
  const int kt_count = min(kt_split, it - kt0);
  const int64_t e = ids[slot];
  const bool ok = e < experts;
  float m = 0.0f;
  for (int b = warp; b < kt_count / 8; b += kFragThreads / 32) {
    const int c0 = kt0 * 16 + b * 128;
    float gate[4] = {0.f, 0.f, 0.f, 0.f}, up[4] = {0.f, 0.f, 0.f, 0.f};
    if (ok) {
      // Splits outer, columns inner, unrolled: all loads of a step in flight.
      const float* pg = partial + static_cast<int64_t>(slot) * gu_splits * features + c0 + lane;
      const float* pu = partial + (static_cast<int64_t>(nslots) + slot) * gu_splits * features + c0 + lane;
#pragma unroll 4
      for (int s = 0; s < gu_splits; ++s) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          gate[j] += pg[static_cast<int64_t>(s) * features + 32 * j];
          up[j] += pu[static_cast<int64_t>(s) * features + 32 * j];
        }
      }
    }
    hadamard128(gate, lane);
    hadamard128(up, lane);
    float act[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t si = e * features + c0 + lane + 32 * j;
      act[j] = ok ? __fmul_rn(swiglu_typed(act_dtype, __fmul_rn(gate[j], load_scale(out_gate, scale_dtype, si)),
                                           __fmul_rn(up[j], load_scale(out_up, scale_dtype, si))),
                              load_scale(in_down, scale_dtype, si))
                  : 0.0f;
    }
    hadamard128(act, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      vals[b * 128 + lane + 32 * j] = act[j];
      m = fmaxf(m, fabsf(act[j]));
    }
  }
  const float mx = block_max(m, red);
  const int ex = piece_exponent(mx);
  write_fragments(vals, kt_count, ldexpf(1.0f, -ex), frag + (static_cast<int64_t>(slot) * it + kt0) * 8);
  if (threadIdx.x == 0) unscale[static_cast<int64_t>(slot) * splits + split] = ldexpf(1.0f, ex);
}

cudaError_t launch_gate_finish_frag(const float* partial, int gu_splits, const uint32_t* ids, int nslots,
                                    const void* out_gate, const void* out_up, const void* in_down, int scale_dtype,
                                    int features, int experts, int act_dtype, int kt_split, int splits, uint2* frag,
                                    float* unscale, cudaStream_t s) {
  const size_t smem = static_cast<size_t>(kt_split) * 16 * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t err = cudaFuncSetAttribute(gate_finish_frag_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
    if (err != cudaSuccess) return err;
  }
  dim3 grid(splits, nslots);
  gate_finish_frag_kernel<<<grid, kFragThreads, smem, s>>>(partial, gu_splits, ids, nslots, out_gate, out_up, in_down,
                                                            scale_dtype, features, experts, act_dtype, kt_split,
                                                            splits, frag, unscale);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Finishes
// ---------------------------------------------------------------------------

// Split sum, Hadamard, signed output scale, cast to the activation type.
__global__ void __launch_bounds__(128) finish_kernel(const float* __restrict__ partial, int splits,
                                                     const int32_t* __restrict__ row_map,
                                                     const uint32_t* __restrict__ ids, int nslots,
                                                     const void* __restrict__ out_scale, int scale_dtype,
                                                     int features, int experts, int act_dtype,
                                                     void* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int block = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int slot = blockIdx.y;
  if (block * 128 >= features) return;
  const int64_t e = ids[slot];
  const int64_t prow = row_map ? row_map[slot] : static_cast<int64_t>(slot) * splits;
  if (e >= experts || prow < 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) store_act(out, act_dtype, static_cast<int64_t>(slot) * features + block * 128 + lane + 32 * j, 0.0f);
    return;
  }
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  const float* ps = partial + prow * features + block * 128 + lane;
#pragma unroll 4
  for (int s = 0; s < splits; ++s) {
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] += ps[static_cast<int64_t>(s) * features + 32 * j];
  }
  hadamard128(v, lane);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int col = block * 128 + lane + 32 * j;
    store_act(out, act_dtype, static_cast<int64_t>(slot) * features + col,
              __fmul_rn(v[j], load_scale(out_scale, scale_dtype, e * features + col)));
  }
}

cudaError_t launch_finish(const float* partial, int splits, const int32_t* row_map, const uint32_t* ids, int nslots,
                          const void* out_scale, int scale_dtype, int features, int experts, int act_dtype, void* out,
                          cudaStream_t s) {
  dim3 grid((features / 128 + 3) / 4, nslots);
  finish_kernel<<<grid, 128, 0, s>>>(partial, splits, row_map, ids, nslots, out_scale, scale_dtype, features, experts,
                                     act_dtype, out);
  return cudaGetLastError();
}

// Nine slots per token (eight routed + shared), one warp per slot: expert
// finish (split sum, Hadamard, out scale, cast), then warp 0 forms the routed
// weighted sum in the order slot 0, then (slot r + 0) + total for r = 1..7,
// T(routed), T(routed + T(shared)), T(residual + combined)
// (metal/fast_decode_finish_fused.metal:52-62).  When shared_values is given
// it holds the typed shared-expert output [tokens][h] and slot 8 of partial is
// not read.  shared_values are the dense shared expert's float32 split
// partials, summed and cast here.
__global__ void __launch_bounds__(288) finish_fused_kernel(const float* __restrict__ partial, int splits,
                                                           const int32_t* __restrict__ row_map,
                                                           const uint32_t* __restrict__ ids, int tokens,
                                                           const void* __restrict__ out_scale, int scale_dtype,
                                                           int features, int experts,
                                                           const float* __restrict__ scores,
                                                           const void* __restrict__ residual,
                                                           const void* __restrict__ shared_values, int shared_splits,
                                                           int act_dtype, void* __restrict__ out) {
  __shared__ float products[9][128];
  const int lane = threadIdx.x & 31, slot = threadIdx.x >> 5;
  const int block = blockIdx.x, token = blockIdx.y;
  const int row = token * 9 + slot;
  if (slot == 8 && shared_values != nullptr) {
    // Dense shared expert: float32 split partials [shared_splits][tokens][h].
    const int64_t total = static_cast<int64_t>(tokens) * features;
    float a[4] = {0.f, 0.f, 0.f, 0.f};
    const float* sv = static_cast<const float*>(shared_values) + static_cast<int64_t>(token) * features + block * 128 + lane;
#pragma unroll 4
    for (int sp = 0; sp < shared_splits; ++sp) {
#pragma unroll
      for (int j = 0; j < 4; ++j) a[j] += __ldcg(sv + sp * total + 32 * j);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) products[8][lane + 32 * j] = round_to(act_dtype, a[j]);
  } else {
    const int64_t e = ids[row];
    const int64_t prow = row_map ? row_map[row] : static_cast<int64_t>(row) * splits;
    const bool ok = e < experts && prow >= 0;  // an out-of-range id contributes zero
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (ok) {
      const float* ps = partial + prow * features + block * 128 + lane;
#pragma unroll 4
      for (int s = 0; s < splits; ++s) {
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] += ps[static_cast<int64_t>(s) * features + 32 * j];
      }
    }
    hadamard128(v, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = block * 128 + lane + 32 * j;
      const float value =
          ok ? round_to(act_dtype, __fmul_rn(v[j], load_scale(out_scale, scale_dtype, e * features + col))) : 0.0f;
      products[slot][lane + 32 * j] = slot < 8 ? __fmul_rn(value, scores[token * 8 + slot]) : value;
    }
  }
  __syncthreads();
  if (slot != 0) return;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = lane + 32 * j;
    float total = __fadd_rn(products[0][c], 0.0f);
#pragma unroll
    for (int r = 1; r < 8; ++r) total = __fadd_rn(__fadd_rn(products[r][c], 0.0f), total);
    const int64_t off = static_cast<int64_t>(token) * features + block * 128 + c;
    const float routed = round_to(act_dtype, total);
    const float combined = round_to(act_dtype, __fadd_rn(routed, round_to(act_dtype, products[8][c])));
    store_act(out, act_dtype, off, __fadd_rn(load_act(residual, act_dtype, off), combined));
  }
}

cudaError_t launch_finish_fused(const float* partial, int splits, const int32_t* row_map, const uint32_t* ids, int tokens,
                                const void* out_scale, int scale_dtype, int features, int experts,
                                const float* scores, const void* residual, const void* shared_values,
                                int shared_splits, int act_dtype, void* out, cudaStream_t s) {
  dim3 grid(features / 128, tokens);
  finish_fused_kernel<<<grid, 288, 0, s>>>(partial, splits, row_map, ids, tokens, out_scale, scale_dtype, features, experts,
                                           scores, residual, shared_values, shared_splits, act_dtype, out);
  return cudaGetLastError();
}

}  // namespace exlr8
