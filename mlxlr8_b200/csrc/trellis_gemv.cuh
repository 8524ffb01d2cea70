// Parameter blocks and launch helpers of the trellis expert kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace exlr8 {

constexpr int kMaxGroupRows = 8;  // rows (expert slots) sharing one decoded tile

// Device-side dispatch plan: slots sorted by expert and cut into groups of at
// most kMaxGroupRows rows of one expert.  Written by plan_kernel.
struct PlanView {
  int32_t* header;        // [0] groups, [1] rows, [2..7] work counters
  int32_t* order;         // [rows] slot index, sorted by expert (stable)
  int32_t* group_expert;  // [max_groups]
  int32_t* group_start;   // [max_groups] offset into order
  int32_t* group_count;   // [max_groups]
  int32_t* expert_count;  // [experts] rows per expert
  int32_t* expert_start;  // [experts] first position in order
  int32_t* zero;          // counters of later kernels, zeroed by the plan (may be null)
  int zero_count;
  int32_t* chunk_hist;    // [chunks][experts + 1] scratch of the multi-CTA plan (large row counts)
};

// Shared memory of plan_body for `warps` warps.
inline size_t plan_smem_bytes(int experts, int warps) {
  return static_cast<size_t>(3 + warps) * experts * sizeof(int);
}

size_t plan_bytes(int rows, int experts);
PlanView plan_view(void* base, int rows, int experts);

// Rows i with i % period == skip_slot are left out (skip_slot < 0: none).
cudaError_t launch_plan(const uint32_t* ids, int rows, int experts, int period, int skip_slot, PlanView plan,
                        cudaStream_t s);
// row_map (nullable): slot -> row of `partial` holding that slot's single
// (unsplit) product; a negative row contributes zero.  Without it slot r
// reads rows r * splits .. r * splits + splits - 1.
cudaError_t launch_finish(const float* partial, int splits, const int32_t* row_map, const uint32_t* ids, int nslots,
                          const void* out_scale, int scale_dtype, int features, int experts, int act_dtype, void* out,
                          cudaStream_t s);
cudaError_t launch_finish_fused(const float* partial, int splits, const int32_t* row_map, const uint32_t* ids, int tokens,
                                const void* out_scale, int scale_dtype, int features, int experts,
                                const float* scores, const void* residual, const void* shared_values,
                                int shared_splits, int act_dtype, void* out, cudaStream_t s);

}  // namespace exlr8
