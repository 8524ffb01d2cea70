// Router: float32 gate GEMV (logits = x @ Wg^T) and the sigmoid + bias top-8
// selection with renormalisation (exlr8 fast_router.metal:1-42,
// model.py:111-132).

#include "common.cuh"
#include "router.cuh"
#include "plan.cuh"
#include "trellis_gemv.cuh"
#include "launch.cuh"

namespace exlr8 {

constexpr int kGateWarps = 8;
constexpr int kGateTokens = 8;
constexpr int kGateChunk = 6;  // float4 weight loads in flight per lane (hidden 6144: all of them)

// Four consecutive activations (index a multiple of 4) as floats.
__device__ __forceinline__ float4 load_act4(const void* base, int dtype, int64_t i) {
  if (dtype == kF32) return *reinterpret_cast<const float4*>(static_cast<const float*>(base) + i);
  const uint2 v = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(base) + i);
  if (dtype == kF16) {
    const __half2 a = *reinterpret_cast<const __half2*>(&v.x), b = *reinterpret_cast<const __half2*>(&v.y);
    return make_float4(__low2float(a), __high2float(a), __low2float(b), __high2float(b));
  }
  const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&v.x);
  const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&v.y);
  return make_float4(__low2float(a), __high2float(a), __low2float(b), __high2float(b));
}

// One CTA per expert row of Wg; the 8 warps split the hidden dimension; each
// warp keeps partial dot products for up to kGateTokens tokens at a time.
// In the decode chain this kernel is the chain head: a plain launch, fully
// ordered after earlier work in the stream (later kernels of the chain rely
// on it); it lets the routing kernel launch early.
__global__ void __launch_bounds__(kGateWarps * 32) gate_logits_kernel(const void* __restrict__ x, int x_dtype,
                                                                      int tokens, int hidden,
                                                                      const float* __restrict__ wg,
                                                                      float* __restrict__ logits, int experts) {
  pdl_launch_dependents();  // the routing kernel may launch and wait for this grid
  __shared__ float red[kGateWarps][kGateTokens];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int e = blockIdx.x;
  const float* w = wg + static_cast<int64_t>(e) * hidden;
  const int per_warp = (hidden / 4 + kGateWarps - 1) / kGateWarps;  // float4 groups
  const int g0 = warp * per_warp;
  const int g1 = min(g0 + per_warp, hidden / 4);
  for (int t0 = 0; t0 < tokens; t0 += kGateTokens) {
    float acc[kGateTokens];
#pragma unroll
    for (int t = 0; t < kGateTokens; ++t) acc[t] = 0.f;
    // All of a lane's weight loads of a chunk are issued before any use.
    for (int gc = g0 + lane; gc < g1; gc += 32 * kGateChunk) {
      float4 wv[kGateChunk];
#pragma unroll
      for (int i = 0; i < kGateChunk; ++i)
        wv[i] = gc + 32 * i < g1 ? reinterpret_cast<const float4*>(w)[gc + 32 * i] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int t = 0; t < kGateTokens; ++t) {
        if (t0 + t < tokens) {
#pragma unroll
          for (int i = 0; i < kGateChunk; ++i) {
            if (gc + 32 * i < g1) {
              const float4 xv = load_act4(x, x_dtype, static_cast<int64_t>(t0 + t) * hidden + 4 * (gc + 32 * i));
              acc[t] = fmaf(xv.x, wv[i].x, acc[t]);
              acc[t] = fmaf(xv.y, wv[i].y, acc[t]);
              acc[t] = fmaf(xv.z, wv[i].z, acc[t]);
              acc[t] = fmaf(xv.w, wv[i].w, acc[t]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < kGateTokens; ++t) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], off);
    }
    if (lane == 0) {
#pragma unroll
      for (int t = 0; t < kGateTokens; ++t) red[warp][t] = acc[t];
    }
    __syncthreads();
    if (threadIdx.x < kGateTokens && t0 + static_cast<int>(threadIdx.x) < tokens) {
      float s = 0.f;
#pragma unroll
      for (int w2 = 0; w2 < kGateWarps; ++w2) s += red[w2][threadIdx.x];
      logits[static_cast<int64_t>(t0 + threadIdx.x) * experts + e] = s;
    }
    __syncthreads();
  }
}

cudaError_t launch_gate_logits(const void* x, int x_dtype, int tokens, int hidden, const float* wg, float* logits,
                               int experts, cudaStream_t s) {
  static const cudaError_t carve = prefer_shared_carveout(gate_logits_kernel);
  if (carve != cudaSuccess) return carve;
  gate_logits_kernel<<<experts, kGateWarps * 32, 0, s>>>(x, x_dtype, tokens, hidden, wg, logits, experts);
  return cudaGetLastError();
}

// Selection for one row of 256 logits by one warp.  Lane l owns experts
// i*32 + l.  Each of the eight rounds takes the largest remaining
// sigmoid(l)+bias (lowest expert id on a tie), records its sigmoid, and
// removes it; lane r keeps the round-r winner.  Weights are divided by
// 1e-20 + their sum (accumulated in rank order) and multiplied by `scale`;
// slot 8 holds the shared expert id.  With `ids_copy` the nine ids are also
// written there (shared memory).  The rounds stay a loop: the routing runs
// once per launch on one SM, where straight-line code would be fetched cold.
__device__ __forceinline__ void route_warp(const float* logits, const float* __restrict__ bias, uint32_t* ids,
                                           float* scores, float scale, uint32_t shared_id, int lane,
                                           uint32_t* ids_copy = nullptr) {
  float original[8], choice[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = i * 32 + lane;
    original[i] = sigmoid_select(__ldcg(logits + e));
    choice[i] = __fadd_rn(original[i], bias[e]);
  }
  float my_selected = 0.0f;
  uint32_t my_winner = 0u;
#pragma unroll 1
  for (int rank = 0; rank < 8; ++rank) {
    float best = -INFINITY;
    uint32_t index = 256u;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t e = i * 32 + lane;
      if (choice[i] > best || (choice[i] == best && e < index)) {
        best = choice[i];
        index = e;
      }
    }
    float top = best;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) top = fmaxf(top, __shfl_xor_sync(0xffffffffu, top, off));
    const uint32_t winner = __reduce_min_sync(0xffffffffu, best == top ? index : 256u);
    const int slot = static_cast<int>(winner >> 5);
    float mine = original[0];
#pragma unroll
    for (int i = 1; i < 8; ++i)
      if (i == slot) mine = original[i];
    const float selected = __shfl_sync(0xffffffffu, mine, winner & 31);
    if (lane == rank) {
      my_selected = selected;
      my_winner = winner;
    }
    if (lane == static_cast<int>(winner & 31)) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i == slot) choice[i] = -INFINITY;
    }
  }
  float total = 1e-20f;
#pragma unroll
  for (int r = 0; r < 8; ++r) total = __fadd_rn(total, __shfl_sync(0xffffffffu, my_selected, r));
  if (lane < 8) {
    ids[lane] = my_winner;
    scores[lane] = __fmul_rn(__fdiv_rn(my_selected, total), scale);
    if (ids_copy) ids_copy[lane] = my_winner;
  } else if (lane == 8) {
    ids[8] = shared_id;
    if (ids_copy) ids_copy[8] = shared_id;
  }
}

__global__ void __launch_bounds__(128) route_kernel(const float* __restrict__ logits, const float* __restrict__ bias,
                                                    int rows, uint32_t* __restrict__ ids,
                                                    float* __restrict__ scores, float scale, uint32_t shared_id) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (row >= rows) return;
  route_warp(logits + static_cast<int64_t>(row) * 256, bias, ids + static_cast<int64_t>(row) * 9,
             scores + static_cast<int64_t>(row) * 8, scale, shared_id, lane);
}

// Routing and dispatch plan of the decode chain: one CTA, launched with
// programmatic dependent launch after gate_logits_kernel; it waits for the
// gate grid, routes every token (one warp per token) and builds the plan of
// the 9 * tokens slots in place of a separate plan kernel.
__global__ void __launch_bounds__(kGateWarps * 32) route_plan_kernel(
    const float* __restrict__ logits, const float* __restrict__ bias, int tokens, uint32_t* __restrict__ ids,
    float* __restrict__ scores, int plan_experts, int skip_slot, PlanView plan) {
  pdl_launch_dependents();  // the prep kernel may launch and wait for this grid
  extern __shared__ int sm[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  pdl_wait();
  const int rows = tokens * 9;
  if (rows <= kSmallPlanRows) {
    // Decode batches: the ids stay in shared memory for the plan.
    uint32_t* s_ids = reinterpret_cast<uint32_t*>(sm);
    for (int t = warp; t < tokens; t += kGateWarps)
      route_warp(logits + static_cast<int64_t>(t) * 256, bias, ids + static_cast<int64_t>(t) * 9,
                 scores + static_cast<int64_t>(t) * 8, 2.5f, 256u, lane, s_ids + t * 9);
    __syncthreads();
    small_plan_body(s_ids, rows, plan_experts, 9, skip_slot, plan, sm + rows);
    return;
  }
  for (int t = warp; t < tokens; t += kGateWarps)
    route_warp(logits + static_cast<int64_t>(t) * 256, bias, ids + static_cast<int64_t>(t) * 9,
               scores + static_cast<int64_t>(t) * 8, 2.5f, 256u, lane);
  __syncthreads();
  plan_body(ids, rows, plan_experts, 9, skip_slot, plan, sm);
}

cudaError_t launch_route_plan(const float* logits, const float* bias, int tokens, uint32_t* ids, float* scores,
                              int plan_experts, int skip_slot, PlanView plan, cudaStream_t s) {
  size_t smem = plan_smem_bytes(plan_experts, kGateWarps);
  if (smem < 5 * kSmallPlanRows * sizeof(int)) smem = 5 * kSmallPlanRows * sizeof(int);
  if (smem > 48 * 1024) {
    cudaError_t err =
        cudaFuncSetAttribute(route_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (err != cudaSuccess) return err;
  }
  static const cudaError_t carve = prefer_shared_carveout(route_plan_kernel);
  if (carve != cudaSuccess) return carve;
  return launch_pdl(route_plan_kernel, dim3(1), dim3(kGateWarps * 32), smem, s, logits, bias, tokens, ids, scores,
                    plan_experts, skip_slot, plan);
}

cudaError_t launch_route(const float* logits, const float* bias, int rows, uint32_t* ids, float* scores,
                         float scale, uint32_t shared_id, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  route_kernel<<<(rows + 3) / 4, 128, 0, s>>>(logits, bias, rows, ids, scores, scale, shared_id);
  return cudaGetLastError();
}

}  // namespace exlr8
