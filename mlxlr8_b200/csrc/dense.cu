// Dense helpers: codebook probe, whole-matrix trellis decode and dequantize
// (exlr8 trellis.py:199-214, metal/decode.metal), and the bf16 shared expert
// GEMV used when the shared expert is stored as bf16 matrices.

#include "common.cuh"
#include "codec.cuh"
#include "dense.cuh"

namespace exlr8 {

__global__ void codebook_kernel(const uint32_t* __restrict__ states, float* __restrict__ values, int64_t n,
                                int paired) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (paired) {
    if (2 * i + 1 < n) {
      const uint32_t r = decode_pair(states[2 * i] & 0xFFFFu, states[2 * i + 1] & 0xFFFFu);
      values[2 * i] = __half2float(__ushort_as_half(static_cast<uint16_t>(r & 0xFFFFu)));
      values[2 * i + 1] = __half2float(__ushort_as_half(static_cast<uint16_t>(r >> 16)));
    } else if (2 * i < n) {
      values[2 * i] = decode_value(states[2 * i]);
    }
  } else if (i < n) {
    values[i] = decode_value(states[i]);
  }
}

cudaError_t launch_codebook(const uint32_t* states, float* values, int64_t n, int paired, cudaStream_t s) {
  const int64_t work = paired ? (n + 1) / 2 : n;
  if (work == 0) return cudaSuccess;
  codebook_kernel<<<static_cast<unsigned>((work + 255) / 256), 256, 0, s>>>(states, values, n, paired);
  return cudaGetLastError();
}

// One thread per weight of matrix `expert`: inner[r][c] (decode.metal:9-35).
__global__ void decode_matrix_kernel(const uint32_t* __restrict__ words, int64_t expert, int k, int in_features,
                                     int out_features, int side, float* __restrict__ inner) {
  const int64_t index = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (index >= static_cast<int64_t>(in_features) * out_features) return;
  const int r = static_cast<int>(index / out_features), c = static_cast<int>(index % out_features);
  const int tk = r >> 4, tn = c >> 4, lr = r & 15, lc = c & 15;
  const uint32_t lane = (lc & 7) * 4 + ((lr & 7) >> 1);
  const uint32_t slot = (lr & 1) + ((lr & 8) >> 2) + ((lc & 8) >> 1);
  const uint32_t code = lane * 8 + slot;
  const uint32_t nwords = 8u * k;
  const uint32_t last_bit = (code + 1) * k + 256u * k;
  const uint32_t last_word = (last_bit - 1) / 32;
  const uint32_t shift = (last_word + 1) * 32 - last_bit;
  const uint32_t* tile = words + tile_index(expert, tk, tn, in_features / 16, out_features / 16, side) * nwords;
  const uint64_t merged = (static_cast<uint64_t>(tile[(last_word - 1) % nwords]) << 32) | tile[last_word % nwords];
  inner[index] = decode_value(static_cast<uint32_t>(merged >> shift) & 0xFFFFu);
}

cudaError_t launch_decode_matrix(const uint32_t* words, int64_t expert, int k, int in_features, int out_features,
                                 int side, float* inner, cudaStream_t s) {
  const int64_t n = static_cast<int64_t>(in_features) * out_features;
  decode_matrix_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(words, expert, k, in_features,
                                                                               out_features, side, inner);
  return cudaGetLastError();
}

// weight[o][i] = H_i(H_o(inner)^T)[o][i] * svh[o] * suh[i], one CTA per
// 128x128 block (trellis.py:105-109 order: transform along out, transpose,
// transform along in, then the two scales).
__global__ void __launch_bounds__(256) dequantize_kernel(const float* __restrict__ inner,
                                                         const void* __restrict__ suh, const void* __restrict__ svh,
                                                         int scale_dtype, int in_features, int out_features,
                                                         float* __restrict__ weight) {
  extern __shared__ float tile[];  // [128 in][129]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ib = blockIdx.y, ob = blockIdx.x;
  for (int idx = threadIdx.x; idx < 128 * 128; idx += blockDim.x) {
    const int i = idx >> 7, o = idx & 127;
    tile[i * 129 + o] = inner[static_cast<int64_t>(ib * 128 + i) * out_features + ob * 128 + o];
  }
  __syncthreads();
  for (int i = warp; i < 128; i += 8) {  // transform along out for each input row
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = tile[i * 129 + lane + 32 * j];
    hadamard128(v, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) tile[i * 129 + lane + 32 * j] = v[j];
  }
  __syncthreads();
  for (int o = warp; o < 128; o += 8) {  // transform along in for each output column
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = tile[(lane + 32 * j) * 129 + o];
    hadamard128(v, lane);
    const int64_t orow = ob * 128 + o;
    const float so = load_scale(svh, scale_dtype, orow);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int icol = ib * 128 + lane + 32 * j;
      weight[orow * in_features + icol] = __fmul_rn(__fmul_rn(v[j], so), load_scale(suh, scale_dtype, icol));
    }
  }
}

cudaError_t launch_dequantize(const float* inner, const void* suh, const void* svh, int scale_dtype, int in_features,
                              int out_features, float* weight, cudaStream_t s) {
  const size_t smem = 128 * 129 * sizeof(float);
  cudaError_t err =
      cudaFuncSetAttribute(dequantize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  dim3 grid(out_features / 128, in_features / 128);
  dequantize_kernel<<<grid, 256, smem, s>>>(inner, suh, svh, scale_dtype, in_features, out_features, weight);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// bf16 dense GEMV on mma.sync (bf16 x bf16 products are exact in float32).
// Lane (gid, tig) loads 16 bytes of two weight rows (gid, gid+8) and 16 bytes
// of token gid at k = 8*tig..8*tig+7 of each 32-wide step; the step is two
// m16n8k16 MMAs whose k order is permuted identically in A and B.
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint4 ldg128_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void mma_bf16(float c[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

constexpr int kDenseWarps = 4;
constexpr int kDenseUnroll = 4;

__global__ void __launch_bounds__(kDenseWarps * 32) dense_bf16_gemv_kernel(const uint16_t* __restrict__ x, int tokens,
                                                                           const uint16_t* __restrict__ w, int n,
                                                                           int k, int splits,
                                                                           float* __restrict__ partial) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const int n0 = (blockIdx.x * kDenseWarps + warp) * 16;
  if (n0 >= n) return;
  const int split = blockIdx.y;
  const int steps = k / 32;
  const int per = (steps + splits - 1) / splits;
  const int s0 = split * per, s1 = min(s0 + per, steps);
  const uint16_t* w0 = w + static_cast<int64_t>(n0 + gid) * k + 8 * tig;
  const uint16_t* w1 = w0 + static_cast<int64_t>(8) * k;
  for (int t0 = 0; t0 < tokens; t0 += 8) {
    const bool has_token = t0 + gid < tokens;
    const uint16_t* xr = x + static_cast<int64_t>(has_token ? t0 + gid : 0) * k + 8 * tig;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int st = s0;
    for (; st + kDenseUnroll <= s1; st += kDenseUnroll) {
      uint4 a[kDenseUnroll], b[kDenseUnroll], xv[kDenseUnroll];
#pragma unroll
      for (int u = 0; u < kDenseUnroll; ++u) {
        a[u] = ldg128_stream(w0 + (st + u) * 32);
        b[u] = ldg128_stream(w1 + (st + u) * 32);
        xv[u] = has_token ? *reinterpret_cast<const uint4*>(xr + (st + u) * 32) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kDenseUnroll; ++u) {
        mma_bf16(acc, a[u].x, b[u].x, a[u].y, b[u].y, xv[u].x, xv[u].y);
        mma_bf16(acc, a[u].z, b[u].z, a[u].w, b[u].w, xv[u].z, xv[u].w);
      }
    }
    for (; st < s1; ++st) {
      const uint4 a = ldg128_stream(w0 + st * 32);
      const uint4 b = ldg128_stream(w1 + st * 32);
      const uint4 xv = has_token ? *reinterpret_cast<const uint4*>(xr + st * 32) : make_uint4(0, 0, 0, 0);
      mma_bf16(acc, a.x, b.x, a.y, b.y, xv.x, xv.y);
      mma_bf16(acc, a.z, b.z, a.w, b.w, xv.z, xv.w);
    }
    // c0,c1: row gid, tokens 2tig, 2tig+1; c2,c3: row gid+8.
    const int ta = t0 + 2 * tig, tb = ta + 1;
    float* out = partial + static_cast<int64_t>(split) * tokens * n;
    if (ta < tokens) {
      out[static_cast<int64_t>(ta) * n + n0 + gid] = acc[0];
      out[static_cast<int64_t>(ta) * n + n0 + gid + 8] = acc[2];
    }
    if (tb < tokens) {
      out[static_cast<int64_t>(tb) * n + n0 + gid] = acc[1];
      out[static_cast<int64_t>(tb) * n + n0 + gid + 8] = acc[3];
    }
  }
}

cudaError_t launch_dense_bf16_gemv(const uint16_t* x, int tokens, const uint16_t* w, int n, int k, int splits,
                                   float* partial, cudaStream_t s) {
  dim3 grid((n / 16 + kDenseWarps - 1) / kDenseWarps, splits);
  dense_bf16_gemv_kernel<<<grid, kDenseWarps * 32, 0, s>>>(x, tokens, w, n, k, splits, partial);
  return cudaGetLastError();
}

__global__ void dense_swiglu_kernel(const float* __restrict__ gp, const float* __restrict__ up, int splits, int tokens,
                                    int n, int act_dtype, void* __restrict__ h) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = static_cast<int64_t>(tokens) * n;
  if (i >= total) return;
  float g = 0.f, u = 0.f;
  for (int s = 0; s < splits; ++s) {
    g += gp[s * total + i];
    u += up[s * total + i];
  }
  store_act(h, act_dtype, i, swiglu_typed(act_dtype, g, u));
}

cudaError_t launch_dense_swiglu(const float* gate_partial, const float* up_partial, int splits, int tokens, int n,
                                int act_dtype, void* h, cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(tokens) * n;
  dense_swiglu_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(gate_partial, up_partial, splits,
                                                                                 tokens, n, act_dtype, h);
  return cudaGetLastError();
}

__global__ void dense_cast_kernel(const float* __restrict__ partial, int splits, int tokens, int n, int act_dtype,
                                  void* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = static_cast<int64_t>(tokens) * n;
  if (i >= total) return;
  float a = 0.f;
  for (int s = 0; s < splits; ++s) a += partial[s * total + i];
  store_act(out, act_dtype, i, a);
}

cudaError_t launch_dense_cast(const float* partial, int splits, int tokens, int n, int act_dtype, void* out,
                              cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(tokens) * n;
  dense_cast_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(partial, splits, tokens, n, act_dtype,
                                                                               out);
  return cudaGetLastError();
}

}  // namespace exlr8
