// Residual add + RMS norm (norm.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace exlr8 {

// h = T(x + residual) (residual may be null), out = T(w * T(h * rsqrt(mean(h^2) + eps))).
cudaError_t launch_residual_rms(const void* x, const void* residual, const void* w, int act_dtype, int64_t rows,
                                int hidden, float eps, void* h_out, void* out, cudaStream_t s);

}  // namespace exlr8
