// Dispatch plan shared by the plan kernel and the fused router kernel.
#pragma once

#include <stdint.h>

#include "trellis_gemv.cuh"

namespace exlr8 {

// Single-CTA stable counting sort of the slot expert ids, then groups of at
// most kMaxGroupRows rows.  Ids outside [0, experts) are counted in
// header[8] and left out of every group.  Works for any block size that is a
// multiple of 32.
__device__ __forceinline__ void plan_body(const uint32_t* __restrict__ ids, int rows, int experts, int period, int skip_slot,
                          PlanView plan, int* sm) {
  const int nwarps = blockDim.x >> 5;
  int* hist = sm;                        // [experts]
  int* base = hist + experts;            // [experts]
  int* gbase = base + experts;           // [experts]
  int* wcount = gbase + experts;         // [nwarps][experts]
  __shared__ int s_total_groups;
  __shared__ int s_bad;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  for (int e = tid; e < experts; e += blockDim.x) hist[e] = 0;
  for (int i = tid; i < plan.zero_count; i += blockDim.x) plan.zero[i] = 0;
  if (tid == 0) s_bad = 0;
  __syncthreads();
  for (int i = tid; i < rows; i += blockDim.x) {
    if (skip_slot >= 0 && i % period == skip_slot) continue;
    uint32_t e = ids[i];
    if (e < static_cast<uint32_t>(experts)) atomicAdd(&hist[e], 1);
    else atomicAdd(&s_bad, 1);
  }
  __syncthreads();
  // Exclusive scans of row counts and group counts (one warp).
  if (warp == 0) {
    const int per = (experts + 31) / 32;
    const int first = lane * per;
    int rsum = 0, gsum = 0;
    for (int e = first; e < min(first + per, experts); ++e) {
      rsum += hist[e];
      gsum += (hist[e] + kMaxGroupRows - 1) / kMaxGroupRows;
    }
    int rinc = rsum, ginc = gsum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      int r = __shfl_up_sync(0xffffffffu, rinc, off);
      int g = __shfl_up_sync(0xffffffffu, ginc, off);
      if (lane >= off) {
        rinc += r;
        ginc += g;
      }
    }
    int rrun = rinc - rsum, grun = ginc - gsum;
    for (int e = first; e < min(first + per, experts); ++e) {
      base[e] = rrun;
      gbase[e] = grun;
      plan.expert_start[e] = rrun;
      plan.expert_count[e] = hist[e];
      rrun += hist[e];
      grun += (hist[e] + kMaxGroupRows - 1) / kMaxGroupRows;
    }
    if (lane == 31) s_total_groups = ginc;
  }
  __syncthreads();
  // Groups.
  for (int e = tid; e < experts; e += blockDim.x) {
    const int n = hist[e];
    for (int c = 0; c * kMaxGroupRows < n; ++c) {
      const int g = gbase[e] + c;
      plan.group_expert[g] = e;
      plan.group_start[g] = base[e] + c * kMaxGroupRows;
      plan.group_count[g] = min(kMaxGroupRows, n - c * kMaxGroupRows);
    }
  }
  __syncthreads();
  // Stable scatter, one chunk of blockDim slots at a time.
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int chunk = 0; chunk < rows; chunk += blockDim.x) {
    for (int j = tid; j < nwarps * experts; j += blockDim.x) wcount[j] = 0;
    __syncthreads();
    const int i = chunk + tid;
    const bool skipped = i < rows && skip_slot >= 0 && i % period == skip_slot;
    const uint32_t raw = (i < rows && !skipped) ? ids[i] : 0xFFFFFFFFu;
    const bool valid = raw < static_cast<uint32_t>(experts);
    const uint32_t key = valid ? raw : 0xFFFFFFFFu;
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    const int leader = __ffs(peers) - 1;
    const int rank = __popc(peers & lt_mask);
    if (valid && lane == leader) wcount[warp * experts + key] = __popc(peers);
    __syncthreads();
    if (valid) {
      int prior = 0;
      for (int w = 0; w < warp; ++w) prior += wcount[w * experts + key];
      plan.order[base[key] + prior + rank] = i;
    }
    __syncthreads();
    if (valid && lane == leader) atomicAdd(&base[key], __popc(peers));
    __syncthreads();
  }
  if (tid == 0) {
    plan.header[0] = s_total_groups;
    plan.header[1] = rows;
    for (int c = 2; c < 8; ++c) plan.header[c] = 0;
    plan.header[8] = s_bad;
    plan.header[9] = 0;
  }
}

// Plan of at most kSmallPlanRows slots (decode batches) whose ids are already
// in shared memory: one thread per slot ranks it by (expert id, slot) against
// every other slot, so the sort needs no global round trip.  Produces the
// same order, groups and header as plan_body (the per-expert counts and
// starts, which only the prefill path reads, are not written).  `scratch`
// holds 4 * rows ints of shared memory.
constexpr int kSmallPlanRows = 256;

__device__ __forceinline__ void small_plan_body(const uint32_t* s_ids, int rows, int experts, int period,
                                                int skip_slot, PlanView plan, int* scratch) {
  __shared__ int s_bad, s_groups;
  uint32_t* key = reinterpret_cast<uint32_t*>(scratch);
  int* rank = scratch + rows;
  int* within = rank + rows;
  int* count = within + rows;
  const int tid = threadIdx.x;
  if (tid == 0) {
    s_bad = 0;
    s_groups = 0;
  }
  for (int i = tid; i < rows; i += blockDim.x) {
    const uint32_t e = s_ids[i];
    const bool skipped = skip_slot >= 0 && i % period == skip_slot;
    key[i] = !skipped && e < static_cast<uint32_t>(experts) ? e : 0xFFFFFFFFu;
  }
  __syncthreads();
  for (int i = tid; i < rows; i += blockDim.x) {
    const uint32_t k = key[i];
    if (k == 0xFFFFFFFFu) {
      if (!(skip_slot >= 0 && i % period == skip_slot)) atomicAdd(&s_bad, 1);
      continue;
    }
    int r = 0, w = 0, c = 0;
    for (int j = 0; j < rows; ++j) {
      const uint32_t kj = key[j];
      r += kj < k || (kj == k && j < i);
      w += kj == k && j < i;
      c += kj == k;
    }
    rank[i] = r;
    within[i] = w;
    count[i] = c;
    plan.order[r] = i;
  }
  __syncthreads();
  for (int i = tid; i < rows; i += blockDim.x) {
    const uint32_t k = key[i];
    if (k == 0xFFFFFFFFu || within[i] % kMaxGroupRows != 0) continue;
    int g = within[i] / kMaxGroupRows;  // groups of this expert before this one
    for (int j = 0; j < rows; ++j)      // plus every group of the smaller ids
      if (key[j] < k && within[j] == 0) g += (count[j] + kMaxGroupRows - 1) / kMaxGroupRows;
    plan.group_expert[g] = static_cast<int>(k);
    plan.group_start[g] = rank[i];
    plan.group_count[g] = min(kMaxGroupRows, count[i] - within[i]);
    atomicAdd(&s_groups, 1);
  }
  __syncthreads();
  if (tid == 0) {
    plan.header[0] = s_groups;
    plan.header[1] = rows;
    for (int c = 2; c < 8; ++c) plan.header[c] = 0;
    plan.header[8] = s_bad;
    plan.header[9] = 0;
  }
}

}  // namespace exlr8
