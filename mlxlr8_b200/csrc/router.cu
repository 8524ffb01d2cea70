// Router: float32 gate GEMV (logits = x @ Wg^T) and the sigmoid + bias top-8
// selection with renormalisation (exlr8 fast_router.metal:1-42,
// model.py:111-132).

#include "common.cuh"
#include "router.cuh"

namespace exlr8 {

constexpr int kGateWarps = 8;
constexpr int kGateTokens = 8;

// One CTA per expert row of Wg; the 8 warps split the hidden dimension; each
// warp keeps partial dot products for up to kGateTokens tokens at a time.
__global__ void __launch_bounds__(kGateWarps * 32) gate_logits_kernel(const void* __restrict__ x, int x_dtype,
                                                                      int tokens, int hidden,
                                                                      const float* __restrict__ wg,
                                                                      float* __restrict__ logits, int experts) {
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
    for (int g = g0 + lane; g < g1; g += 32) {
      const float4 wv = reinterpret_cast<const float4*>(w)[g];
#pragma unroll
      for (int t = 0; t < kGateTokens; ++t) {
        if (t0 + t < tokens) {
          const int64_t base = static_cast<int64_t>(t0 + t) * hidden + 4 * g;
          acc[t] = fmaf(load_act(x, x_dtype, base), wv.x, acc[t]);
          acc[t] = fmaf(load_act(x, x_dtype, base + 1), wv.y, acc[t]);
          acc[t] = fmaf(load_act(x, x_dtype, base + 2), wv.z, acc[t]);
          acc[t] = fmaf(load_act(x, x_dtype, base + 3), wv.w, acc[t]);
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
  gate_logits_kernel<<<experts, kGateWarps * 32, 0, s>>>(x, x_dtype, tokens, hidden, wg, logits, experts);
  return cudaGetLastError();
}

// One warp per row of 256 logits.  Lane l owns experts i*32 + l.  Each of
// the eight rounds takes the largest remaining sigmoid(l)+bias (lowest expert
// id on a tie), records its sigmoid, and removes it.  Weights are divided by
// 1e-20 + their sum (accumulated in rank order) and multiplied by `scale`;
// slot 8 holds the shared expert id.
__global__ void __launch_bounds__(128) route_kernel(const float* __restrict__ logits, const float* __restrict__ bias,
                                                    int rows, uint32_t* __restrict__ ids,
                                                    float* __restrict__ scores, float scale, uint32_t shared_id) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (row >= rows) return;
  float original[8], choice[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = i * 32 + lane;
    original[i] = sigmoid_select(logits[static_cast<int64_t>(row) * 256 + e]);
    choice[i] = __fadd_rn(original[i], bias[e]);
  }
  float selected[8];
  uint32_t winners[8];
#pragma unroll
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
    selected[rank] = __shfl_sync(0xffffffffu, mine, winner & 31);
    winners[rank] = winner;
    if (lane == static_cast<int>(winner & 31)) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i == slot) choice[i] = -INFINITY;
    }
  }
  if (lane == 0) {
    float total = 1e-20f;
#pragma unroll
    for (int i = 0; i < 8; ++i) total = __fadd_rn(total, selected[i]);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      ids[static_cast<int64_t>(row) * 9 + i] = winners[i];
      scores[static_cast<int64_t>(row) * 8 + i] = __fmul_rn(__fdiv_rn(selected[i], total), scale);
    }
    ids[static_cast<int64_t>(row) * 9 + 8] = shared_id;
  }
}

cudaError_t launch_route(const float* logits, const float* bias, int rows, uint32_t* ids, float* scores,
                         float scale, uint32_t shared_id, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  route_kernel<<<(rows + 3) / 4, 128, 0, s>>>(logits, bias, rows, ids, scores, scale, shared_id);
  return cudaGetLastError();
}

}  // namespace exlr8
