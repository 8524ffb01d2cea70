// Expert parallelism: dispatch of routed slots to the ranks that own their
// experts, and the combine of the returned slot values (the exchange step of
// the expert-parallel MoE layer; the reference runs all 257 experts on one
// device, model.py:385-418).
//
// Layout of one exchange (capacity C rows per destination rank):
//   send_x    [ranks][C][hidden]  activation rows in the activation dtype
//   send_meta [ranks][C]          local expert id of the row, -1 = empty
//   slot_pos  [tokens * 8]        destination rank * C + row of each routed
//                                 slot, -1 when its id is out of range
//   counts    [ranks]             rows per destination (overflow: an error)
// Rows go to their destination in slot order (token-major), so the exchange
// is deterministic.

#include "common.cuh"
#include "ep.cuh"

namespace exlr8 {

namespace {

constexpr int kDispatchThreads = 1024;

// Positions: one CTA walks the tokens * 8 routed slots in order and gives each
// one the next row of its destination rank (warp ballots per destination).
__global__ void __launch_bounds__(kDispatchThreads) ep_positions_kernel(
    const uint32_t* __restrict__ ids, int tokens, int ranks, int experts_per_rank, int capacity,
    int32_t* __restrict__ send_meta, int32_t* __restrict__ slot_pos, int32_t* __restrict__ counts,
    int32_t* __restrict__ status) {
  __shared__ int s_base[32];   // running rows per destination (ranks <= 32)
  __shared__ int s_warp[32][32];  // [warp][dest] counts of the current chunk
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = kDispatchThreads / 32;
  const int slots = tokens * 8;
  const int routed = ranks * experts_per_rank;
  if (tid < 32) s_base[tid] = 0;
  __syncthreads();
  for (int chunk = 0; chunk < slots; chunk += kDispatchThreads) {
    const int i = chunk + tid;
    int dest = -1, local = -1;
    if (i < slots) {
      const uint32_t e = ids[static_cast<int64_t>(i / 8) * 9 + i % 8];
      if (e < static_cast<uint32_t>(routed)) {
        dest = static_cast<int>(e) / experts_per_rank;
        local = static_cast<int>(e) % experts_per_rank;
      }
    }
    // Per-warp counts and in-warp ranks for every destination.
    int rank_in_warp = 0;
    for (int d = 0; d < ranks; ++d) {
      const unsigned m = __ballot_sync(0xffffffffu, dest == d);
      if (dest == d) rank_in_warp = __popc(m & ((1u << lane) - 1u));
      if (lane == 0) s_warp[warp][d] = __popc(m);
    }
    __syncthreads();
    if (dest >= 0) {
      int pos = s_base[dest] + rank_in_warp;
      for (int w = 0; w < warp; ++w) pos += s_warp[w][dest];
      if (pos < capacity) {
        slot_pos[i] = dest * capacity + pos;
        send_meta[static_cast<int64_t>(dest) * capacity + pos] = local;
      } else {
        slot_pos[i] = -1;
        atomicAdd(&status[0], 1);  // capacity overflow: the slot is lost
      }
    } else if (i < slots) {
      slot_pos[i] = -1;
    }
    __syncthreads();
    if (tid < ranks) {
      int add = 0;
      for (int w = 0; w < nwarps; ++w) add += s_warp[w][tid];
      s_base[tid] += add;
    }
    __syncthreads();
  }
  if (tid < ranks) counts[tid] = min(s_base[tid], capacity);
}

// Row copies: x[token] -> send_x[slot_pos], 16 bytes per thread.
__global__ void ep_copy_kernel(const uint4* __restrict__ x, int row_vecs, int tokens,
                               const int32_t* __restrict__ slot_pos, uint4* __restrict__ send_x) {
  const int64_t total = static_cast<int64_t>(tokens) * 8 * row_vecs;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t slot = i / row_vecs;
    const int v = static_cast<int>(i % row_vecs);
    const int pos = slot_pos[slot];
    if (pos >= 0) send_x[static_cast<int64_t>(pos) * row_vecs + v] = x[(slot / 8) * row_vecs + v];
  }
}

// Combine (metal/fast_decode_finish_fused.metal:52-62 order): slot values are
// already T(H(v) * out_scale); products value * score, routed sum slot 0 then
// (slot r + 0) + total, T(routed), T(routed + shared), T(residual + combined).
template <int kAct>
__global__ void ep_combine_kernel(const void* __restrict__ values, const int32_t* __restrict__ slot_pos,
                                  const float* __restrict__ scores, const void* __restrict__ shared,
                                  const void* __restrict__ residual, int tokens, int hidden, void* __restrict__ out) {
  const int64_t total = static_cast<int64_t>(tokens) * hidden;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / hidden;
    const int c = static_cast<int>(i % hidden);
    float prod[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int pos = slot_pos[t * 8 + r];
      const float v = pos >= 0 ? load_act(values, kAct, static_cast<int64_t>(pos) * hidden + c) : 0.0f;
      prod[r] = __fmul_rn(v, scores[t * 8 + r]);
    }
    float sum = __fadd_rn(prod[0], 0.0f);
#pragma unroll
    for (int r = 1; r < 8; ++r) sum = __fadd_rn(__fadd_rn(prod[r], 0.0f), sum);
    const float routed = round_to(kAct, sum);
    const float combined = round_to(kAct, __fadd_rn(routed, round_to(kAct, load_act(shared, kAct, i))));
    store_act(out, kAct, i, __fadd_rn(load_act(residual, kAct, i), combined));
  }
}

template <int kAct>
__global__ void sum_cast_kernel(const float* __restrict__ partial, int splits, int64_t n, void* __restrict__ out) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float a = 0.f;
    for (int sp = 0; sp < splits; ++sp) a += partial[sp * n + i];
    store_act(out, kAct, i, a);
  }
}

int grid_for(int64_t n, int threads) {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const int64_t want = (n + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sms) * 8;
  return static_cast<int>(want < 1 ? 1 : (want < cap ? want : cap));
}

}  // namespace

cudaError_t launch_ep_dispatch(const uint32_t* ids, int tokens, const void* x, int x_dtype, int hidden, int ranks,
                               int experts_per_rank, int capacity, void* send_x, int32_t* send_meta,
                               int32_t* slot_pos, int32_t* counts, int32_t* status, cudaStream_t s) {
  cudaError_t err = cudaMemsetAsync(send_meta, 0xFF, static_cast<size_t>(ranks) * capacity * sizeof(int32_t), s);
  if (err == cudaSuccess) err = cudaMemsetAsync(status, 0, sizeof(int32_t), s);
  if (err != cudaSuccess) return err;
  if (tokens == 0) return cudaMemsetAsync(counts, 0, static_cast<size_t>(ranks) * sizeof(int32_t), s);
  ep_positions_kernel<<<1, kDispatchThreads, 0, s>>>(ids, tokens, ranks, experts_per_rank, capacity, send_meta,
                                                     slot_pos, counts, status);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  const int elem = x_dtype == kF32 ? 4 : 2;
  const int row_vecs = hidden * elem / 16;
  const int64_t total = static_cast<int64_t>(tokens) * 8 * row_vecs;
  ep_copy_kernel<<<grid_for(total, 256), 256, 0, s>>>(static_cast<const uint4*>(x), row_vecs, tokens, slot_pos,
                                                      static_cast<uint4*>(send_x));
  return cudaGetLastError();
}

cudaError_t launch_ep_combine(const void* values, int x_dtype, const int32_t* slot_pos, const float* scores,
                              const void* shared, const void* residual, int tokens, int hidden, void* out,
                              cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(tokens) * hidden;
  if (total == 0) return cudaSuccess;
  const int grid = grid_for(total, 256);
  if (x_dtype == kF32)
    ep_combine_kernel<kF32><<<grid, 256, 0, s>>>(values, slot_pos, scores, shared, residual, tokens, hidden, out);
  else if (x_dtype == kF16)
    ep_combine_kernel<kF16><<<grid, 256, 0, s>>>(values, slot_pos, scores, shared, residual, tokens, hidden, out);
  else
    ep_combine_kernel<kBF16><<<grid, 256, 0, s>>>(values, slot_pos, scores, shared, residual, tokens, hidden, out);
  return cudaGetLastError();
}

cudaError_t launch_sum_cast(const float* partial, int splits, int64_t n, int act_dtype, void* out, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const int grid = grid_for(n, 256);
  if (act_dtype == kF32) sum_cast_kernel<kF32><<<grid, 256, 0, s>>>(partial, splits, n, out);
  else if (act_dtype == kF16) sum_cast_kernel<kF16><<<grid, 256, 0, s>>>(partial, splits, n, out);
  else sum_cast_kernel<kBF16><<<grid, 256, 0, s>>>(partial, splits, n, out);
  return cudaGetLastError();
}

}  // namespace exlr8
