// Standalone dispatch plan (expert sort + block table) and combine.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "trellis_gemv.cuh"

namespace exlr8 {

constexpr int kDispatchMaxExperts = 1024;

// Stable sort of `rows` slot ids by expert (plan in `plan`, sized by
// plan_bytes(rows, experts)), then order/sorted_ids [rows] and the block
// table [3][capacity] (expert, first sorted row, length) with *count columns.
cudaError_t launch_dispatch_plan(const uint32_t* ids, int rows, int experts, int block_rows, PlanView plan,
                                 uint32_t* order, uint32_t* sorted_ids, uint32_t* table, int64_t capacity,
                                 int32_t* count, cudaStream_t s);

// out[t] = T(residual[t] + T(T(sum_r values[t][r] * scores[t][r]) + values[t][8])).
cudaError_t launch_combine(const void* values, const float* scores, const void* residual, int64_t tokens,
                           int features, int act_dtype, void* out, cudaStream_t s);

}  // namespace exlr8
