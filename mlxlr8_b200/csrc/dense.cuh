// Codebook probe and whole-matrix trellis decode/dequantize.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace exlr8 {

cudaError_t launch_codebook(const uint32_t* states, float* values, int64_t n, int paired, cudaStream_t s);
cudaError_t launch_decode_matrix(const uint32_t* words, int64_t expert, int k, int in_features, int out_features,
                                 int side, float* inner, cudaStream_t s);
cudaError_t launch_dequantize(const float* inner, const void* suh, const void* svh, int scale_dtype,
                              int in_features, int out_features, float* weight, cudaStream_t s);

// bf16 shared expert.  Gate and up in one pass, the last CTA of each 64-row
// block writing h = SwiGLU(T(g), T(u)) in the activation type; `counters`
// ([n/64] ints) must be zero at launch.  Partials are [splits][tokens][n].
// max_ctas > 0 caps the grid (the kernels loop over their work items).
cudaError_t launch_dense_gate_up(const uint16_t* x, int tokens, const uint16_t* wg, const uint16_t* wu, int n, int k,
                                 int splits, float* gate_partial, float* up_partial, int* counters, int act_dtype,
                                 void* h, int max_ctas, cudaStream_t s);
cudaError_t launch_dense_gemv(const uint16_t* x, int tokens, const uint16_t* w, int n, int k, int splits,
                              float* partial, int max_ctas, cudaStream_t s);

}  // namespace exlr8
