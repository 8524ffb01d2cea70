// Dense helpers: codebook probe, whole-matrix trellis decode/dequantize and
// the bf16 shared expert.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace exlr8 {

cudaError_t launch_codebook(const uint32_t* states, float* values, int64_t n, int paired, cudaStream_t s);
cudaError_t launch_decode_matrix(const uint32_t* words, int64_t expert, int k, int in_features, int out_features,
                                 int side, float* inner, cudaStream_t s);
cudaError_t launch_dequantize(const float* inner, const void* suh, const void* svh, int scale_dtype,
                              int in_features, int out_features, float* weight, cudaStream_t s);

// bf16 shared expert: y[t][n] = sum_k x[t][k] * W[n][k] (float32 accumulate)
// written as float32 split-K partials [splits][tokens][n].
cudaError_t launch_dense_bf16_gemv(const uint16_t* x, int tokens, const uint16_t* w, int n, int k, int splits,
                                   float* partial, cudaStream_t s);
// Typed SwiGLU of the summed gate/up partials -> bf16 h [tokens][n].
cudaError_t launch_dense_swiglu(const float* gate_partial, const float* up_partial, int splits, int tokens, int n,
                                int act_dtype, void* h, cudaStream_t s);
// Sum split partials and cast -> typed values [tokens][n].
cudaError_t launch_dense_cast(const float* partial, int splits, int tokens, int n, int act_dtype, void* out,
                              cudaStream_t s);

}  // namespace exlr8
