// Shared device helpers for the exlr8 B200 kernels: activation types, typed
// rounding (the T(...) casts of the exlr8 Metal kernels), warp Hadamard-128.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/exlr8_b200.h"

namespace exlr8 {

// Activation element types (match EXLR8_DTYPE_* in the public header).
enum DType : int { kF32 = EXLR8_DTYPE_F32, kF16 = EXLR8_DTYPE_F16, kBF16 = EXLR8_DTYPE_BF16 };

__device__ __forceinline__ float load_act(const void* base, int dtype, int64_t i) {
  if (dtype == kF32) return static_cast<const float*>(base)[i];
  if (dtype == kF16) return __half2float(static_cast<const __half*>(base)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
}

__device__ __forceinline__ void store_act(void* base, int dtype, int64_t i, float v) {
  if (dtype == kF32) static_cast<float*>(base)[i] = v;
  else if (dtype == kF16) static_cast<__half*>(base)[i] = __float2half_rn(v);
  else static_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
}

// Round a float to the activation type and back: the value T(v) as a float.
__device__ __forceinline__ float round_to(int dtype, float v) {
  if (dtype == kF32) return v;
  if (dtype == kF16) return __half2float(__float2half_rn(v));
  return __bfloat162float(__float2bfloat16_rn(v));
}

// Scale vectors are fp16 in EXLR8 checkpoints (experts.py:97-115); fp32 is
// accepted as well.
__device__ __forceinline__ float load_scale(const void* base, int dtype, int64_t i) {
  if (dtype == kF32) return static_cast<const float*>(base)[i];
  return __half2float(static_cast<const __half*>(base)[i]);
}

// Normalised Hadamard-128 over one warp.  Lane l holds v[j] = element
// l + 32*j.  Stages run over index bits 1, 2, 4, ..., 64 in that order with
// (a+b, a-b) butterflies, then a multiply by float(1/sqrt(128)); this is the
// order of the reference transform, so results are bit-identical to it.
// A cross-lane butterfly is one fused multiply-add with a per-lane sign:
// fma(+1, v, o) = v + o and fma(-1, v, o) = o - v, each one rounding of the
// exact sum (signed zeros included), the same bits as the add or subtract.
__device__ __forceinline__ void hadamard128(float v[4], int lane) {
#pragma unroll
  for (int bit = 1; bit < 32; bit <<= 1) {
    const float sign = (lane & bit) ? -1.0f : 1.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float other = __shfl_xor_sync(0xffffffffu, v[j], bit);
      v[j] = fmaf(sign, v[j], other);
    }
  }
  float a0 = v[0] + v[1], a1 = v[0] - v[1], a2 = v[2] + v[3], a3 = v[2] - v[3];
  v[0] = a0 + a2;
  v[1] = a1 + a3;
  v[2] = a0 - a2;
  v[3] = a1 - a3;
  const float s = 0.08838834764831845f;
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] *= s;
}

// Typed SwiGLU T(T(g*sigmoid(g))*u) where every step of the typed sigmoid
// rounds to T: tail = T(1/T(1+T(exp(|g|)))), sigmoid = g<0 ? tail : T(1-tail).
__device__ __forceinline__ float swiglu_typed(int dtype, float gate, float up) {
  float g = round_to(dtype, gate);
  float u = round_to(dtype, up);
  float e = round_to(dtype, expf(fabsf(g)));
  float tail = round_to(dtype, 1.0f / round_to(dtype, 1.0f + e));
  float sig = g < 0.0f ? tail : round_to(dtype, 1.0f - tail);
  return round_to(dtype, round_to(dtype, g * sig) * u);
}

// Sigmoid as 1/(1+exp(|v|)) with a sign select, float32.
__device__ __forceinline__ float sigmoid_select(float v) {
  float y = 1.0f / (1.0f + expf(fabsf(v)));
  return v < 0.0f ? y : 1.0f - y;
}

}  // namespace exlr8
