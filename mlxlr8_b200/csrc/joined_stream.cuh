// Streaming MXFP4 GEMV of the joined experts for decode batches (the role of
// metal/joined_gather_order.metal and MLX gather_qmm at small row counts,
// exlr8 joined_mxfp4.py:72-87,90-134).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "stream.cuh"

namespace exlr8 {

// Work unit: (plan group of <= 8 slots of one expert, 128-row output block,
// K split); a stage is one 128-wide K block of the unit's 128 rows.
//
// Activation records (kFragBlockBytes each, the layout of stream.cuh) use
// the MXFP4 K order: K tile s of a 128-wide block is the two MMA steps of
// 32-block j = s / 2, half h = s % 2, and lane tig's B words hold
// x[32j + 8 tig + 4h + {0, 1}] and x[32j + 8 tig + 4h + {2, 3}], so that one
// 32-bit code word (eight E2M1 values, k = 32j + 8 tig .. + 7) of a weight
// row feeds both steps of its block.
struct JoinedStreamParams {
  CUtensorMap codes;         // uint8 [experts * out_features][in_features / 2]: box 128 B x 128 rows, 128-byte swizzle
  const uint8_t* scales;     // E8M0 of the same rows in the 512-byte block layout (mx_scale_offset)
  const unsigned char* frag; // [nslots][in_features / 128] activation records, MXFP4 K order
  float* partial;            // [out_features / plane_rows][nslots][splits][plane_rows]
  PlanView plan;
  int counter;               // plan header entry used as the unit counter
  int in_features, out_features, plane_rows, kb_per_split, splits, nslots;
};

// Tensor map of joined codes [rows][in_features / 2] for the stream kernel.
bool joined_code_map(CUtensorMap* map, const void* codes, int64_t rows, int in_features);

cudaError_t launch_joined_stream(const JoinedStreamParams& p, cudaStream_t s);

// Number of persistent stream CTAs (for split heuristics).
int joined_stream_ctas();

}  // namespace exlr8
