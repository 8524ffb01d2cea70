// Tensor-core router gate product for prefill batches (router_gemm.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace exlr8 {

// Token count from which the joined layer uses the tensor-core gate product.
constexpr int kRouterGemmMinTokens = 64;

int router_gemm_splits(int tokens, int hidden);
// Scratch of launch_router_gemm (weight pieces, activation pieces, partials).
size_t router_gemm_workspace(int tokens, int hidden, int x_dtype);
// logits [tokens][256] float32 = x . gate_weight^T; hidden % 64 == 0, x and
// workspace 16-byte aligned.
cudaError_t launch_router_gemm(const void* x, int x_dtype, int tokens, int hidden, const float* gate_weight,
                               float* logits, void* workspace, cudaStream_t s);

}  // namespace exlr8
