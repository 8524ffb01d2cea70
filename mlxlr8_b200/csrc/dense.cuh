// Codebook probe and whole-matrix trellis decode/dequantize.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace exlr8 {

cudaError_t launch_codebook(const uint32_t* states, float* values, int64_t n, int paired, cudaStream_t s);
// Exact E4M3 bytes of `tiles` stored trellis tiles (256 bytes per tile, tile order kept).
cudaError_t launch_expand_static(const uint32_t* words, int64_t tiles, int k, uint32_t* out, cudaStream_t s);
cudaError_t launch_decode_matrix(const uint32_t* words, int64_t expert, int k, int in_features, int out_features,
                                 int side, float* inner, cudaStream_t s);
// Normalised Hadamard-128 of every 128-value block of `blocks` blocks
// (float32 in and out; in place allowed): the warp transform the expert
// kernels apply to their inputs and outputs.
cudaError_t launch_hadamard128(const float* x, int64_t blocks, float* out, cudaStream_t s);
cudaError_t launch_dequantize(const float* inner, const void* suh, const void* svh, int scale_dtype,
                              int in_features, int out_features, float* weight, cudaStream_t s);

// MXFP4 (MLX quantize mode="mxfp4", group 32) of float rows, and the fused
// decode + in-scale fold + quantise of every matrix of a trellis buffer
// (W^T rows land at (e * rows_per_matrix + row_offset + o)).  Codes and the
// float rows must be 16-byte aligned.
cudaError_t launch_mxfp4_quantize(const float* w, int64_t rows, int in_features, uint32_t* codes, uint8_t* scales,
                                  cudaStream_t s);
cudaError_t launch_mxfp4_encode_trellis(const uint32_t* packed, int64_t matrices, int k, int in_features,
                                        int out_features, int side, const void* in_scale, const void* unit,
                                        int scale_dtype, uint32_t* codes, uint8_t* scales, int64_t rows_per_matrix,
                                        int64_t row_offset, cudaStream_t s);

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
