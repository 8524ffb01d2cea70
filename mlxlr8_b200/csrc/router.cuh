// Router launch helpers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "trellis_gemv.cuh"

namespace exlr8 {

cudaError_t launch_gate_logits(const void* x, int x_dtype, int tokens, int hidden, const float* wg, float* logits,
                               int experts, cudaStream_t s);
// Gate GEMV + route + dispatch plan in one launch (the last CTA routes and
// plans); `done` is a workspace int that the launch zeroes first.
cudaError_t launch_router_plan(const void* x, int x_dtype, int tokens, int hidden, const float* wg, float* logits,
                               const float* bias, uint32_t* ids, float* scores, int* done, int plan_experts,
                               int skip_slot, PlanView plan, cudaStream_t s);
cudaError_t launch_route(const float* logits, const float* bias, int rows, uint32_t* ids, float* scores,
                         float scale, uint32_t shared_id, cudaStream_t s);

}  // namespace exlr8
