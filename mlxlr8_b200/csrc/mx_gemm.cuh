// Grouped block-scaled expert GEMM on tcgen05 (kind::mxf8f6f4) and the
// dispatch tables it consumes.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace exlr8 {

constexpr int kMxMaxN = 160;      // slot rows per chunk (MMA N)
constexpr int kMxKTile = 128;     // K values per pipeline stage
constexpr int kMxRowAlign = 128;  // expert segments start on this row multiple

// Slots sorted by expert, each expert's segment padded to a multiple of
// kMxRowAlign rows, cut into chunks of at most kMxMaxN rows whose starts are
// multiples of kMxRowAlign.  Written on the device by the segment kernels.
struct MxChunks {
  int32_t* header;        // [0] chunks, [1] padded rows, [2..3] unit counters, [4] error
  int32_t* chunk_start;   // [max_chunks] padded row of the first row
  int32_t* chunk_rows;    // [max_chunks] valid rows (<= kMxMaxN)
  int32_t* chunk_expert;  // [max_chunks]
  int32_t* padded_start;  // [experts + 1]
  int32_t* row_slot;      // [padded rows] slot index, -1 for padding
  int32_t* slot_row;      // [slots] padded row, -1 when the slot has no expert
};

// Largest padded row count for `slots` sorted slots over `experts` experts.
inline int64_t mx_padded_rows(int64_t slots, int64_t experts) {
  return (slots + experts * (kMxRowAlign - 1) + kMxRowAlign - 1) / kMxRowAlign * kMxRowAlign;
}
inline int64_t mx_max_chunks(int64_t slots, int64_t experts) { return slots / kMxRowAlign + experts + 1; }

// One grouped product: for every projection p, chunk (expert e) and output
// row o < out_features of p:  out[r][p * proj_offset + o] =
// sum_k W_pe[o][k] X_p[r][k] over the chunk's padded rows r, where
// X = (hi + lo) E4M3 planes sharing one E8M0 scale per 32 values of k, and
// W is either
//   * MXFP4 (trellis_k == 0): E2M1 codes [experts * out][in / 2] with E8M0
//     scales per 32 values in the 512-byte block layout (mx_scale_offset), or
//   * trellis codes (trellis_k == 3 or 4, EXLR8 packed bytes, storage side
//     `side`), decoded in the kernel to their exact E4M3 values.
struct ExpertGemmArgs {
  const void* weights[2];
  const uint8_t* weight_scales[2];  // MXFP4 only
  const uint8_t* x_hi[2];           // [padded rows][in_features] E4M3, per projection
  const uint8_t* x_lo[2];
  const uint8_t* x_scales[2];       // [padded rows / 128][in_features / 128][512]
  MxChunks chunks;
  int counter_index;                // header slot of this launch's unit counter
  int64_t experts;
  int64_t padded_rows;              // allocated rows of the activation planes
  int in_features;
  int out_features;                 // per projection
  int projections;                  // 1 or 2
  int paired;                       // MXFP4 joined gate|up: accumulator 1 covers rows out_features / 2 + ...
  int trellis_k;                    // 0, 3 or 4
  int side;                         // trellis storage side (1: gate/up, 2: down)
  uint32_t mcg_mask, mcg_xor;       // trellis hash constants (kept in registers for one LOP3)
  float* out;
  int64_t out_stride;               // floats between consecutive rows of out
  int64_t proj_offset;              // column offset of projection 1
};

// Byte of the scale of (row, k-block kb) inside the 512-byte block layout
// [rows / 128][k_blocks / 4][512].
__host__ __device__ inline int64_t mx_scale_offset(int64_t row, int64_t kb, int64_t k_blocks) {
  return ((row / 128) * (k_blocks / 4) + kb / 4) * 512 + (row % 32) * 16 + ((row % 128) / 32) * 4 + kb % 4;
}

cudaError_t launch_expert_gemm(const ExpertGemmArgs& args, cudaStream_t s);

// Whether MXFP4 products whose shape allows it run on SM pairs
// (cta_group::2); on by default.  The one-SM kernel computes the same sums.
bool gemm_pair_enabled();
// Sets the switch (enable 0 or 1) and returns its previous value; enable < 0
// only reads it.
int set_gemm_pair(int enable);

}  // namespace exlr8
