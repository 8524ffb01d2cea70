// Expert-parallel dispatch and combine kernels (ep.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace exlr8 {

// Routed slots of `ids` [tokens][9] (slots 0..7; expert e lives on rank
// e / experts_per_rank as local expert e % experts_per_rank) packed into
// per-destination rows.  status[0] counts slots lost to capacity overflow.
cudaError_t launch_ep_dispatch(const uint32_t* ids, int tokens, const void* x, int x_dtype, int hidden, int ranks,
                               int experts_per_rank, int capacity, void* send_x, int32_t* send_meta,
                               int32_t* slot_pos, int32_t* counts, int32_t* status, cudaStream_t s);

// Routing-weighted combine of the returned slot values with the shared
// expert's typed output and the residual.
cudaError_t launch_ep_combine(const void* values, int x_dtype, const int32_t* slot_pos, const float* scores,
                              const void* shared, const void* residual, int tokens, int hidden, void* out,
                              cudaStream_t s);

// out[i] = T(sum over splits of partial[s][i]).
cudaError_t launch_sum_cast(const float* partial, int splits, int64_t n, int act_dtype, void* out, cudaStream_t s);

// ---- peer-memory exchange (ep_peer.cu) --------------------------------------
//
// Each rank owns one region of device memory that every other rank maps with
// CUDA IPC.  Layout for `ranks` ranks, at most `max_capacity` rows per
// (source, owner) pair and `elem`-byte activations; a call with capacity
// C <= max_capacity uses C as the row stride of every area:
//   [0, 4)          epoch: exchanges this rank has completed
//   [256, 512)      arrived[src]: epoch + 1 once src's rows for this call landed
//   [512, 768)      returned[owner]: epoch + 1 once owner's values landed
//   [768, 1024)     caps[src]: the row capacity C src used for this call (all
//                   ranks must agree: they pass the same token count)
//   [1024, 1280)    sent[dst]: CTAs of this rank's send kernels done with dst
//   [1280, 1536)    back[src]: CTAs of this rank's return kernels done with src
//                   (the last CTA of a peer raises the flag and resets the
//                   count for the next call)
//   meta            int32 [ranks][C]: local expert id of each received row, -1 empty
//   rows            [ranks][C][hidden]: received activation rows
//   back            [ranks][C][hidden]: slot values returned by each owner
constexpr int kPeerMaxRanks = 64;

struct PeerLayout {
  size_t meta, rows, back, total;
};

__host__ __device__ inline PeerLayout peer_layout(int ranks, int max_capacity, int hidden, int elem) {
  PeerLayout l;
  const size_t rows_bytes = static_cast<size_t>(ranks) * max_capacity * hidden * elem;
  l.meta = 1536;
  l.rows = l.meta + ((static_cast<size_t>(ranks) * max_capacity * 4 + 255) / 256) * 256;
  l.back = l.rows + ((rows_bytes + 255) / 256) * 256;
  l.total = l.back + ((rows_bytes + 255) / 256) * 256;
  return l;
}

// Dispatch of this rank's routed slots straight into the owners' regions:
// rows and local expert ids (slot order per owner), slot_pos as for
// launch_ep_dispatch, then the `arrived` flag of this rank in every owner's
// region; then waits (bounded) until every source's rows for this call have
// arrived here.  status[0] counts slots lost to capacity overflow, status[1]
// gets bit 0 when a wait timed out and bit 2 when a source used another
// capacity (token count) than this rank.
cudaError_t launch_ep_send(const uint32_t* ids, int tokens, const void* x, int x_dtype, int hidden, int ranks,
                           int rank, int experts_per_rank, int capacity, int max_capacity, const uint64_t* peers,
                           void* local, int32_t* slot_pos, int32_t* status, cudaStream_t s);

// Return of the owner's slot values (values [ranks][C][hidden], rows of
// source s at [s]) into each source's `back` area, then this rank's
// `returned` flag there; waits (bounded) for every owner's values for this
// call; then advances this rank's epoch.  status[1] gets bit 1 on timeout.
cudaError_t launch_ep_return(const void* values, int x_dtype, int hidden, int ranks, int rank, int capacity,
                             int max_capacity, const uint64_t* peers, void* local, int32_t* status, cudaStream_t s);

// 16-byte stores of `bytes` (a multiple of 16) from src to dst (dst may be a
// peer GPU's memory mapped with CUDA IPC).
cudaError_t launch_peer_write(void* dst, const void* src, int64_t bytes, cudaStream_t s);

}  // namespace exlr8
