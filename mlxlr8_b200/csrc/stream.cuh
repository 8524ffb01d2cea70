// Streaming trellis GEMV, activation-fragment producers and their layouts.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "trellis_gemv.cuh"

namespace exlr8 {

// Activation fragments: one 528-byte record per (projection, slot, 128-wide
// K block): eight K tiles of 64 bytes -- [piece hi/lo][tig 0..3] uint2, the
// mma.sync m16n8k16 B-fragment words of one row, {x[2t], x[2t+1]} and
// {x[2t+8], x[2t+9]} as float16 pieces of the block's values times 2^-ex --
// then a 16-byte header whose first float is the block's unscale 2^ex.  The
// power-of-two scale is chosen per block (the scaled block maximum lies in
// [2^14, 2^15)), so every block is produced independently.
constexpr int kFragBlockBytes = 8 * 64 + 16;

inline size_t frag_bytes(int64_t rows, int features, int projections) {
  return static_cast<size_t>(projections) * static_cast<size_t>(rows) * static_cast<size_t>(features / 128) *
         kFragBlockBytes;
}

// The bf16 shared expert rides along as dense units, streamed by one extra
// warp per CTA (dense_stream.cuh) beside the trellis warps.  A dense unit is
// (16-row group of W, K split); W1 (optional) shares the x rows.  Partials
// are float32 [splits][tokens][n].  Requirements: n % 16 == 0, k a multiple
// of 128 * splits, W, W1 and x 16-byte aligned (the tensor maps of W, W1
// need k * 2 bytes between rows, a multiple of 16).
struct DenseUnits {
  const uint16_t* w0;  // [n][k] bf16 (gate, or down)
  const uint16_t* w1;  // [n][k] bf16 (up) or null
  const uint16_t* x;   // [tokens][k] bf16
  float* p0;           // [splits][tokens][n] partials of w0
  float* p1;           // same for w1
  int n, k, tokens, splits, units;  // units = (n / 16) * splits, 0 = none
  // 1: the inputs (W, W1, x) and outputs (p0, p1) do not depend on the
  // kernels launched since the head of the call's kernel chain, so the dense
  // warp starts without waiting for its predecessor grid (launch.cuh).  The
  // chain head is launched with full stream ordering, which makes that safe.
  int early;
};

struct StreamParams {
  // Tensor maps of the dense rows W0 / W1 ([n][k] bf16; boxes of 16 rows x 64
  // values, 128-byte swizzle), read by the dense warp; encoded on the host
  // when dense.units > 0 (encode_dense_maps).
  CUtensorMap dense_w0, dense_w1;
  const uint32_t* packed[2];
  // Static hot-expert cache (optional): the exact E4M3 bytes of the cached
  // experts per projection, the stored tile order with 256 bytes per tile and
  // in_features * out_features bytes per cache slot; expert_to_slot[e] is the
  // slot of expert e or -1.  Units of cached experts stream these bytes.
  const unsigned char* hot[2];
  const int32_t* expert_to_slot;
  int64_t hot_slots;  // slots in hot[]: a map entry outside [0, hot_slots) reads as "not cached"
  const unsigned char* frag;  // [proj][nslots][in_features / 128] records of kFragBlockBytes
  float* partial;             // [proj][nslots][splits][out_features]
  PlanView plan;
  DenseUnits dense;
  int counter;
  int k, side, in_features, out_features, kt_per_split, splits, projections, nslots;
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

// Encodes p.dense_w0 / p.dense_w1 for p.dense (no-op without dense units);
// false when the encode fails.
bool encode_dense_maps(StreamParams& p);

// xh = H(x[row] * in_scale_p[e]) written as fragment records
// (metal/fast_decode_prep.metal).  frag holds frag_bytes(nslots, features,
// projections).  The scale of channel c is in_scale_p[e * scale_stride + c]
// (scale_stride < 0: features; 0: one vector for every expert, the joined
// path's unit).  mx_order writes the MXFP4 K order (joined_stream.cuh).
cudaError_t launch_prep_frag(const void* x, int x_dtype, int per_slot, int slots_per_token, const uint32_t* ids,
                             int nslots, const void* in0, const void* in1, int scale_dtype, int features, int experts,
                             int projections, unsigned char* frag, cudaStream_t s, int scale_stride = -1,
                             int mx_order = 0, int skip_empty = 0);

// gate/up finish (metal/fast_decode_gate_finish.metal) producing the down
// projection's fragment records (frag_bytes(nslots, features, 1)).  With
// dense_tokens > 0 it also writes the bf16 shared expert's
// h = SwiGLU(T(g), T(u)) [dense_tokens][features] (activation type) from its
// split partials dense_g/dense_u [dense_splits][dense_tokens][features].
// skip_empty: the slot list is sparse (most ids out of range); such slots
// are skipped before their partials are loaded, at the cost of waiting for
// the id first.
cudaError_t launch_gate_finish_frag(const float* partial, int gu_splits, const uint32_t* ids, int nslots,
                                    const void* out_gate, const void* out_up, const void* in_down, int scale_dtype,
                                    int features, int experts, int act_dtype, unsigned char* frag,
                                    const float* dense_g, const float* dense_u, int dense_splits, int dense_tokens,
                                    void* dense_h, cudaStream_t s, int mx_order = 0, int skip_empty = 0);

}  // namespace exlr8
