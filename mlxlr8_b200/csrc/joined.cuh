// Launchers of the joined MXFP4 path (joined.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "mx_gemm.cuh"
#include "trellis_gemv.cuh"

namespace exlr8 {

// Segments, chunks and row maps from an expert plan over `slots` slots.
cudaError_t launch_joined_segments(PlanView plan, int experts, int slots, MxChunks c, cudaStream_t s);

// GEMM activations of the gate/up product: H(x[token] * unit) per padded row.
cudaError_t launch_joined_prep(const void* x, int act_dtype, const void* unit, int scale_dtype, int slots_per_token,
                               int tokens, MxChunks c, int hidden, uint8_t* hi, uint8_t* lo, uint8_t* scales,
                               cudaStream_t s);

// gate/up float32 rows -> GEMM activations of the down product.
cudaError_t launch_joined_gate_finish(const float* gu, const uint32_t* ids, int slots, MxChunks c,
                                      const void* gate_out, const void* up_out, const void* down_in, int scale_dtype,
                                      int intermediate, int act_dtype, uint8_t* hi, uint8_t* lo, uint8_t* scales,
                                      cudaStream_t s);

// Per-slot finish and routing-weighted combine with the residual (nine slots
// per token, slot 8 = shared) reading slot rows through slot_row.
// shared_values (nullable): float32 split partials [shared_splits][tokens][h]
// of a dense shared expert that replaces slot 8.
cudaError_t launch_joined_finish(const float* v, const int32_t* slot_row, const uint32_t* ids, int tokens,
                                 int features, int experts, const void* out_scale, int scale_dtype,
                                 const float* scores, const void* residual, const float* shared_values,
                                 int shared_splits, int act_dtype, void* out, cudaStream_t s);

// Trellis prefill GEMM inputs: per slot and projection, H(x * in_scale[e]).
cudaError_t launch_trellis_prep(const void* x, int act_dtype, int per_slot, int slots_per_token, int nslots,
                                const uint32_t* ids, MxChunks c, const void* in0, const void* in1, int scale_dtype,
                                int projections, int hidden, uint8_t* hi0, uint8_t* lo0, uint8_t* sc0, uint8_t* hi1,
                                uint8_t* lo1, uint8_t* sc1, cudaStream_t s);

cudaError_t launch_mx_prepare_scales(const uint8_t* in, int64_t rows, int kblocks, uint8_t* out, cudaStream_t s);

}  // namespace exlr8
