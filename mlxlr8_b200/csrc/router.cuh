// Router launch helpers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "trellis_gemv.cuh"

namespace exlr8 {

// Gate GEMV logits = x @ Wg^T, one CTA per expert row; a plain launch (the
// head of the decode kernel chain).
cudaError_t launch_gate_logits(const void* x, int x_dtype, int tokens, int hidden, const float* wg, float* logits,
                               int experts, cudaStream_t s);
// Routing + dispatch plan of the decode chain (one CTA, programmatic
// dependent launch after launch_gate_logits).
cudaError_t launch_route_plan(const float* logits, const float* bias, int tokens, uint32_t* ids, float* scores,
                              int plan_experts, int skip_slot, PlanView plan, cudaStream_t s);
cudaError_t launch_route(const float* logits, const float* bias, int rows, uint32_t* ids, float* scores,
                         float scale, uint32_t shared_id, cudaStream_t s);

}  // namespace exlr8
