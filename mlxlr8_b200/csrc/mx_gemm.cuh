// Grouped block-scaled expert GEMM on tcgen05 (kind::mxf8f6f4) and the
// dispatch tables it consumes.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace exlr8 {

constexpr int kMxMaxN = 160;    // slot rows per chunk (MMA N)
constexpr int kMxKTile = 128;   // K values per pipeline stage
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

// One grouped projection: out[p][o] = sum_k W_e[o][k] X[p][k] for every
// padded row p of every chunk (expert e) and every output o < out_features,
// where W is E2M1 x E8M0 (per 32 values of k) and X = (hi + lo) E4M3 planes
// sharing one E8M0 scale per 32 values.  Weight and activation scales are in
// the 512-byte block layout (mx_scale_offset).
struct MxGemmArgs {
  const void* weights;         // [experts * out_features][in_features / 2] packed E2M1
  const uint8_t* weight_scales;  // [experts * out_features / 128][in_features / 128][512]
  const uint8_t* x_hi;         // [padded rows][in_features] E4M3
  const uint8_t* x_lo;
  const uint8_t* x_scales;     // [padded rows / 128][in_features / 128][512]
  MxChunks chunks;
  int counter_index;           // header slot of this launch's unit counter
  int64_t experts;
  int64_t padded_rows;         // allocated rows of x_hi / x_lo
  int in_features;
  int out_features;
  int paired;                  // accumulator 1 covers rows out_features / 2 + (those of accumulator 0)
  float* out;                  // [padded rows][out_features]
};

// Byte of the scale of (row, k-block kb) inside the 512-byte block layout
// [rows / 128][k_blocks / 4][512].
__host__ __device__ inline int64_t mx_scale_offset(int64_t row, int64_t kb, int64_t k_blocks) {
  return ((row / 128) * (k_blocks / 4) + kb / 4) * 512 + (row % 32) * 16 + ((row % 128) / 32) * 4 + kb % 4;
}

cudaError_t launch_mx_gemm(const MxGemmArgs& args, cudaStream_t s);
int mx_gemm_status();  // 0, or a driver error from tensor-map encoding

}  // namespace exlr8
