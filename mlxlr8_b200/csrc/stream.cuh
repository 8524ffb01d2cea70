// Streaming trellis GEMV, activation-fragment producers and their layouts.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "trellis_gemv.cuh"

namespace exlr8 {

// Activation fragments: for every (projection, slot, K tile) 64 bytes =
// [piece hi/lo][tig 0..3] uint2, the mma.sync m16n8k16 B-fragment words of
// one row: {x[2t], x[2t+1]} and {x[2t+8], x[2t+9]} as float16 pieces.  Each
// (projection, slot, K split) has one power-of-two scale; `unscale` holds its
// inverse.
struct StreamParams {
  const uint32_t* packed[2];
  const uint2* frag;     // [proj][nslots][in_tiles][8]
  const float* unscale;  // [proj][nslots][splits]
  float* partial;        // [proj][nslots][splits][out_features]
  PlanView plan;
  int counter;
  int k, side, in_features, out_features, kt_per_split, splits, projections, nslots;
  uint32_t unit16;  // 65536
  uint32_t mcg_mask, mcg_xor;  // 0x8FFF8FFF, 0x3B603B60 (runtime values: one LOP3 each)
};

// K tiles per split: a multiple of 8 (one 128-wide Hadamard block) so that
// fragments and scales can be produced one split at a time.
inline int kt_per_split(int in_features, int splits) {
  const int it = in_features / 16;
  int per = (it + splits - 1) / splits;
  per = (per + 7) / 8 * 8;
  return per;
}
inline int split_count(int in_features, int per) { return (in_features / 16 + per - 1) / per; }

cudaError_t launch_stream(const StreamParams& p, cudaStream_t s);

// xh = H(x[row] * in_scale_p[e]) written as fragments + unscales
// (metal/fast_decode_prep.metal).
cudaError_t launch_prep_frag(const void* x, int x_dtype, int per_slot, int slots_per_token, const uint32_t* ids,
                             int nslots, const void* in0, const void* in1, int scale_dtype, int features, int experts,
                             int projections, int kt_split, int splits, uint2* frag, float* unscale, cudaStream_t s);

// gate/up finish (metal/fast_decode_gate_finish.metal) producing the down
// projection's fragments + unscales.
cudaError_t launch_gate_finish_frag(const float* partial, int gu_splits, const uint32_t* ids, int nslots,
                                    const void* out_gate, const void* out_up, const void* in_down, int scale_dtype,
                                    int features, int experts, int act_dtype, int kt_split, int splits, uint2* frag,
                                    float* unscale, cudaStream_t s);

}  // namespace exlr8
