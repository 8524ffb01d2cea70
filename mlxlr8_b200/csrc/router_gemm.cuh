// Tensor-core router gate product for prefill batches (router_gemm.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace exlr8 {

// Token count from which the joined layer uses the tensor-core gate product.
constexpr int kRouterGemmMinTokens = 64;

int router_gemm_splits(int tokens, int hidden);

// Dense bf16 products on the tensor cores for prefill batches: float32
// partials [splits][rows][n] of a[rows][k] . b[n][k]^T (k % 64 == 0,
// n % 128 == 0, a and b 16-byte aligned).  `error` (one int, zero at launch)
// records a timed-out wait.
int bf16_gemm_splits(int rows, int k, int n);
cudaError_t launch_dense_gemm(const uint16_t* a, int rows, int k, const uint16_t* b, int n, int splits,
                              float* partial, int32_t* error, cudaStream_t s);
// h = T(SwiGLU(T(sum g), T(sum u))) over gate/up split partials of n values.
cudaError_t launch_dense_swiglu(const float* gate_partial, const float* up_partial, int splits, int64_t n,
                                int act_dtype, void* h, cudaStream_t s);
// Scratch of launch_router_gemm (weight pieces, activation pieces, partials).
size_t router_gemm_workspace(int tokens, int hidden, int x_dtype);
// logits [tokens][256] float32 = x . gate_weight^T; hidden % 64 == 0, x and
// workspace 16-byte aligned.
cudaError_t launch_router_gemm(const void* x, int x_dtype, int tokens, int hidden, const float* gate_weight,
                               float* logits, void* workspace, cudaStream_t s);

}  // namespace exlr8
