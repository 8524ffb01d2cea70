// Residual add + RMS norm in front of each MoE block (exlr8 model.py:373-384;
// the fused form of fast_norm.py residual_rms_pair): one CTA per row,
//   h   = T(x + residual)
//   out = T(w * T(h * rsqrt(sum(h * h) / hidden + eps)))
// T() rounds to the activation type; the sum of squares is float32 (plain
// multiply and add, no contraction), reduced over the CTA.  Launched with
// programmatic dependent launch: in a block stack the next block's gate
// kernel becomes resident (and prefetches its weights) while this one runs.

#include "common.cuh"
#include "launch.cuh"

namespace exlr8 {

namespace {

constexpr int kNormThreads = 256;

template <int kAct>
__global__ void __launch_bounds__(kNormThreads) residual_rms_kernel(const void* __restrict__ x,
                                                                    const void* __restrict__ residual,
                                                                    const void* __restrict__ w, int hidden,
                                                                    float eps, void* __restrict__ h_out,
                                                                    void* __restrict__ out) {
  pdl_launch_dependents();
  __shared__ float red[kNormThreads / 32];
  __shared__ float s_inv;
  pdl_wait();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * hidden;
  float acc = 0.0f;
  for (int i = threadIdx.x; i < hidden; i += kNormThreads) {
    float h = load_act(x, kAct, base + i);
    if (residual) h = round_to(kAct, __fadd_rn(h, load_act(residual, kAct, base + i)));
    if (h_out) store_act(h_out, kAct, base + i, h);
    acc = __fadd_rn(acc, __fmul_rn(h, h));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float total = 0.0f;
    for (int wi = 0; wi < kNormThreads / 32; ++wi) total = __fadd_rn(total, red[wi]);
    s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(hidden)), eps)));
  }
  __syncthreads();
  const float inv = s_inv;
  for (int i = threadIdx.x; i < hidden; i += kNormThreads) {
    float h = load_act(x, kAct, base + i);
    if (residual) h = round_to(kAct, __fadd_rn(h, load_act(residual, kAct, base + i)));
    const float normed = round_to(kAct, __fmul_rn(h, inv));
    store_act(out, kAct, base + i, __fmul_rn(load_act(w, kAct, i), normed));
  }
}

}  // namespace

cudaError_t launch_residual_rms(const void* x, const void* residual, const void* w, int act_dtype, int64_t rows,
                                int hidden, float eps, void* h_out, void* out, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>(rows));
  if (act_dtype == kF32)
    return launch_pdl(residual_rms_kernel<kF32>, grid, dim3(kNormThreads), 0, s, x, residual, w, hidden, eps, h_out,
                      out);
  if (act_dtype == kF16)
    return launch_pdl(residual_rms_kernel<kF16>, grid, dim3(kNormThreads), 0, s, x, residual, w, hidden, eps, h_out,
                      out);
  return launch_pdl(residual_rms_kernel<kBF16>, grid, dim3(kNormThreads), 0, s, x, residual, w, hidden, eps, h_out,
                    out);
}

}  // namespace exlr8
