// Standalone dispatch plan and combine of the reference's grouped path.
//
//   dispatch_table_kernel -- the block table of exlr8 fast_prefill.py:19-46
//                            (_segment_table, _plan) from the plan's
//                            per-expert counts and starts; rows whose id is
//                            out of range go after every valid row
//   gather_ids_kernel     -- sorted_ids[i] = ids[order[i]]
//   combine_kernel        -- model.py:415-418 on per-slot expert outputs, in
//                            the float32 order of
//                            metal/fast_decode_finish_fused.metal:52-62
//
// The stable counting sort itself is the library's plan (trellis_gemv.cu
// launch_plan: one CTA for small row counts, per-chunk histograms + one scan
// CTA + stable per-chunk scatter for large ones).

#include "common.cuh"
#include "dispatch.cuh"
#include "trellis_gemv.cuh"

namespace exlr8 {

namespace {

constexpr int kTableThreads = 1024;

// One CTA.  Experts <= kTableThreads: thread e owns expert e.
__global__ void __launch_bounds__(kTableThreads) dispatch_table_kernel(PlanView plan, const uint32_t* __restrict__ ids,
                                                                       int rows, int experts, int block_rows,
                                                                       uint32_t* __restrict__ table, int64_t capacity,
                                                                       int32_t* __restrict__ count) {
  __shared__ int warp_sum[kTableThreads / 32];
  __shared__ int s_valid;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = tid < experts ? plan.expert_count[tid] : 0;
  const int blocks = (c + block_rows - 1) / block_rows;
  // Block-wide exclusive scan of the per-expert block counts.
  int inc = blocks;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, inc, off);
    if (lane >= off) inc += v;
  }
  if (lane == 31) warp_sum[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int w = warp_sum[lane];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += v;
    }
    warp_sum[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  const int first = (warp > 0 ? warp_sum[warp - 1] : 0) + inc - blocks;
  if (tid < experts) {
    const int start = plan.expert_start[tid];
    for (int j = 0; j < blocks; ++j) {
      const int64_t col = first + j;
      if (col >= capacity) break;
      table[col] = static_cast<uint32_t>(tid);
      table[capacity + col] = static_cast<uint32_t>(start + j * block_rows);
      table[2 * capacity + col] = static_cast<uint32_t>(min(block_rows, c - j * block_rows));
    }
  }
  if (tid == kTableThreads - 1) {
    *count = warp_sum[kTableThreads / 32 - 1];
    s_valid = rows - plan.header[8];
  }
  __syncthreads();
  if (plan.header[8] == 0) return;
  // Rows with an out-of-range id follow the valid ones, in row order.
  int placed = s_valid;
  for (int base = 0; base < rows; base += kTableThreads) {
    const int i = base + tid;
    const bool bad = i < rows && ids[i] >= static_cast<uint32_t>(experts);
    const unsigned m = __ballot_sync(0xffffffffu, bad);
    if (lane == 0) warp_sum[warp] = __popc(m);
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < kTableThreads / 32; ++w) {
      before += w < warp ? warp_sum[w] : 0;
      total += warp_sum[w];
    }
    if (bad) plan.order[placed + before + __popc(m & ((1u << lane) - 1u))] = i;
    placed += total;
    __syncthreads();
  }
}

__global__ void gather_ids_kernel(const uint32_t* __restrict__ ids, const int32_t* __restrict__ order, int rows,
                                  uint32_t* __restrict__ order_out, uint32_t* __restrict__ sorted_ids) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += gridDim.x * blockDim.x) {
    const int o = order[i];
    order_out[i] = static_cast<uint32_t>(o);
    sorted_ids[i] = ids[o];
  }
}

// One thread per (token, feature): values [tokens][9][features] typed, the
// ninth slot the shared expert's output.
template <int kAct>
__global__ void combine_kernel(const void* __restrict__ values, const float* __restrict__ scores,
                               const void* __restrict__ residual, int64_t tokens, int features,
                               void* __restrict__ out) {
  const int64_t n = tokens * features;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / features, c = i - t * features;
    const int64_t v0 = t * 9 * features + c;
    float v[9];
#pragma unroll
    for (int r = 0; r < 9; ++r) v[r] = load_act(values, kAct, v0 + r * features);
    const float res = load_act(residual, kAct, i);
    float total = __fadd_rn(__fmul_rn(v[0], scores[t * 8]), 0.0f);
#pragma unroll
    for (int r = 1; r < 8; ++r) total = __fadd_rn(__fadd_rn(__fmul_rn(v[r], scores[t * 8 + r]), 0.0f), total);
    const float routed = round_to(kAct, total);
    const float combined = round_to(kAct, __fadd_rn(routed, v[8]));
    store_act(out, kAct, i, __fadd_rn(res, combined));
  }
}

int sm_count_dispatch() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return sms;
}

}  // namespace

cudaError_t launch_dispatch_plan(const uint32_t* ids, int rows, int experts, int block_rows, PlanView plan,
                                 uint32_t* order, uint32_t* sorted_ids, uint32_t* table, int64_t capacity,
                                 int32_t* count, cudaStream_t s) {
  cudaError_t err = launch_plan(ids, rows, experts, 1, -1, plan, s);
  if (err != cudaSuccess) return err;
  dispatch_table_kernel<<<1, kTableThreads, 0, s>>>(plan, ids, rows, experts, block_rows, table, capacity, count);
  if ((err = cudaGetLastError()) != cudaSuccess) return err;
  if (rows == 0) return cudaSuccess;
  const int grid = min(sm_count_dispatch() * 4, (rows + 255) / 256);
  gather_ids_kernel<<<grid, 256, 0, s>>>(ids, plan.order, rows, order, sorted_ids);
  return cudaGetLastError();
}

cudaError_t launch_combine(const void* values, const float* scores, const void* residual, int64_t tokens,
                           int features, int act_dtype, void* out, cudaStream_t s) {
  const int64_t n = tokens * features;
  if (n == 0) return cudaSuccess;
  const int64_t want = (n + 255) / 256;
  const int grid = static_cast<int>(want < sm_count_dispatch() * 16 ? want : sm_count_dispatch() * 16);
  switch (act_dtype) {
    case kF32: combine_kernel<kF32><<<grid, 256, 0, s>>>(values, scores, residual, tokens, features, out); break;
    case kF16: combine_kernel<kF16><<<grid, 256, 0, s>>>(values, scores, residual, tokens, features, out); break;
    default: combine_kernel<kBF16><<<grid, 256, 0, s>>>(values, scores, residual, tokens, features, out); break;
  }
  return cudaGetLastError();
}

}  // namespace exlr8
