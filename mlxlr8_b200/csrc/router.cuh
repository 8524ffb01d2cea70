// Router launch helpers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace exlr8 {

cudaError_t launch_gate_logits(const void* x, int x_dtype, int tokens, int hidden, const float* wg, float* logits,
                               int experts, cudaStream_t s);
cudaError_t launch_route(const float* logits, const float* bias, int rows, uint32_t* ids, float* scores,
                         float scale, uint32_t shared_id, cudaStream_t s);

}  // namespace exlr8
