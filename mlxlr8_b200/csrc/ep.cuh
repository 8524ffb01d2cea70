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

}  // namespace exlr8
