// Codebook probe and whole-matrix trellis decode / dequantize
// (exlr8 trellis.py:199-214, metal/decode.metal).

#include "common.cuh"
#include "codec.cuh"
#include "dense.cuh"
#include "dense_warp.cuh"

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

// One warp per 128-value block; lane l holds elements l + 32 j, the layout of
// every in-kernel use of hadamard128.
__global__ void hadamard128_kernel(const float* __restrict__ x, int64_t blocks, float* __restrict__ out) {
  const int64_t block = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (block >= blocks) return;
  float v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = x[block * 128 + lane + 32 * j];
  hadamard128(v, lane);
#pragma unroll
  for (int j = 0; j < 4; ++j) out[block * 128 + lane + 32 * j] = v[j];
}

cudaError_t launch_hadamard128(const float* x, int64_t blocks, float* out, cudaStream_t s) {
  if (blocks == 0) return cudaSuccess;
  hadamard128_kernel<<<static_cast<unsigned>((blocks + 7) / 8), 256, 0, s>>>(x, blocks, out);
  return cudaGetLastError();
}

// One thread per weight of matrix `expert`: inner[r][c] (decode.metal:9-35).
__global__ void decode_matrix_kernel(const uint32_t* __restrict__ words, int64_t expert, int k, int in_features,
                                     int out_features, int side, float* __restrict__ inner) {
  const int64_t index = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (index >= static_cast<int64_t>(in_features) * out_features) return;
  const int r = static_cast<int>(index / out_features), c = static_cast<int>(index % out_features);
  inner[index] = trellis_weight(words, expert, k, in_features / 16, out_features / 16, side, r, c);
}

cudaError_t launch_decode_matrix(const uint32_t* words, int64_t expert, int k, int in_features, int out_features,
                                 int side, float* inner, cudaStream_t s) {
  const int64_t n = static_cast<int64_t>(in_features) * out_features;
  decode_matrix_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(words, expert, k, in_features,
                                                                               out_features, side, inner);
  return cudaGetLastError();
}

// E4M3 byte of a float16 that is already an E4M3 number: sign in bit 7; a
// float16 exponent field of 9 or more is a normal number (field - 8, top three
// fraction bits); fields 6..8 are the subnormals m * 2^-9; zero keeps its sign.
__device__ __forceinline__ uint32_t e4m3_byte(uint32_t h) {
  const uint32_t field = (h >> 10) & 31u, fraction = h & 1023u;
  uint32_t code = (h >> 8) & 0x80u;
  if (field >= 9u) {
    code |= ((field - 8u) << 3) | (fraction >> 7);
  } else if (field >= 6u) {
    code |= (1024u + fraction) >> (16u - field);
  }
  return code;
}

// Static hot-expert cache expansion (static_cache.py:29-42): every stored
// tile of 8k words becomes 256 bytes in place of its index, byte p the E4M3
// code of codeword p of the tile's cyclic bitstream.  One thread per four
// codewords (one output word).
__global__ void expand_static_kernel(const uint32_t* __restrict__ words, int64_t tiles, int k,
                                     uint32_t* __restrict__ out) {
  const int64_t index = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (index >= tiles * 64) return;
  const uint32_t nwords = 8u * static_cast<uint32_t>(k);
  const uint32_t* tile = words + (index >> 6) * nwords;
  const uint32_t q = static_cast<uint32_t>(index & 63);
  uint32_t packed = 0;
#pragma unroll
  for (uint32_t j = 0; j < 4; ++j) {
    const uint32_t last_bit = (4u * q + j + 1u) * k + 256u * k;
    const uint32_t last_word = (last_bit - 1u) / 32u;
    const uint32_t shift = (last_word + 1u) * 32u - last_bit;
    const uint64_t merged = (static_cast<uint64_t>(tile[(last_word - 1u) % nwords]) << 32) | tile[last_word % nwords];
    const uint32_t cw = static_cast<uint32_t>(merged >> shift) & 0xFFFFu;
    packed |= e4m3_byte(decode_pair(cw, cw) & 0xFFFFu) << (8u * j);
  }
  out[index] = packed;
}

cudaError_t launch_expand_static(const uint32_t* words, int64_t tiles, int k, uint32_t* out, cudaStream_t s) {
  const int64_t n = tiles * 64;
  if (n == 0) return cudaSuccess;
  expand_static_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(words, tiles, k, out);
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
// bf16 shared expert (row-major bf16 [out][in] weights).
// ---------------------------------------------------------------------------

constexpr int kDenseWarps = 4;

// Gate and up products in one pass over x, split along k.  Work items are
// (64-row block, split), taken in a grid-stride loop so that the grid can be
// capped (one CTA per SM runs beside the trellis stream kernel); the CTA that
// completes the last split of a 64-row block writes h = SwiGLU(T(g), T(u))
// for it.  `counters` ([n/64]) must be zero at launch.
__global__ void __launch_bounds__(kDenseWarps * 32) dense_gate_up_kernel(
    const uint16_t* __restrict__ x, int tokens, const uint16_t* __restrict__ wg, const uint16_t* __restrict__ wu,
    int n, int k, int splits, float* __restrict__ gp, float* __restrict__ up, int* __restrict__ counters,
    int act_dtype, void* __restrict__ h) {
  __shared__ int s_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int row_blocks = (n / 16 + kDenseWarps - 1) / kDenseWarps;
  const int steps = k / 32;
  const int per = (steps + splits - 1) / splits;
  const int64_t total = static_cast<int64_t>(tokens) * n;
  for (int item = blockIdx.x; item < row_blocks * splits; item += gridDim.x) {
    const int rb = item % row_blocks, split = item / row_blocks;
    const int n0 = (rb * kDenseWarps + warp) * 16;
    const int s0 = split * per, s1 = min(s0 + per, steps);
    if (n0 < n) dense_rows(x, tokens, wg, wu, n, k, n0, s0, s1, gp + split * total, up + split * total, lane);
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      s_last = atomicAdd(&counters[rb], 1) == splits - 1;
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      const int rows = min(kDenseWarps * 16, n - rb * kDenseWarps * 16);
      for (int idx = threadIdx.x; idx < tokens * rows; idx += blockDim.x) {
        const int t = idx / rows;
        const int64_t i = static_cast<int64_t>(t) * n + rb * kDenseWarps * 16 + idx % rows;
        float g = 0.f, u = 0.f;
#pragma unroll 8
        for (int sp = 0; sp < splits; ++sp) {
          g += __ldcg(gp + sp * total + i);
          u += __ldcg(up + sp * total + i);
        }
        store_act(h, act_dtype, i, swiglu_typed(act_dtype, g, u));
      }
    }
    __syncthreads();  // s_last is rewritten by the next item
  }
}

static int capped_grid(int items, int max_ctas) { return max_ctas > 0 && items > max_ctas ? max_ctas : items; }

cudaError_t launch_dense_gate_up(const uint16_t* x, int tokens, const uint16_t* wg, const uint16_t* wu, int n, int k,
                                 int splits, float* gate_partial, float* up_partial, int* counters, int act_dtype,
                                 void* h, int max_ctas, cudaStream_t s) {
  const int items = (n / 16 + kDenseWarps - 1) / kDenseWarps * splits;
  dense_gate_up_kernel<<<capped_grid(items, max_ctas), kDenseWarps * 32, 0, s>>>(
      x, tokens, wg, wu, n, k, splits, gate_partial, up_partial, counters, act_dtype, h);
  return cudaGetLastError();
}

// y partials [splits][tokens][n] of x @ W^T, W bf16 [n][k]; items are
// (64-row block, split) in a grid-stride loop.
__global__ void __launch_bounds__(kDenseWarps * 32) dense_gemv_kernel(const uint16_t* __restrict__ x, int tokens,
                                                                      const uint16_t* __restrict__ w, int n, int k,
                                                                      int splits, float* __restrict__ partial) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int row_blocks = (n / 16 + kDenseWarps - 1) / kDenseWarps;
  const int steps = k / 32;
  const int per = (steps + splits - 1) / splits;
  for (int item = blockIdx.x; item < row_blocks * splits; item += gridDim.x) {
    const int rb = item % row_blocks, split = item / row_blocks;
    const int n0 = (rb * kDenseWarps + warp) * 16;
    if (n0 >= n) continue;
    const int s0 = split * per, s1 = min(s0 + per, steps);
    dense_rows(x, tokens, w, nullptr, n, k, n0, s0, s1, partial + split * static_cast<int64_t>(tokens) * n, nullptr,
               lane);
  }
}

cudaError_t launch_dense_gemv(const uint16_t* x, int tokens, const uint16_t* w, int n, int k, int splits,
                              float* partial, int max_ctas, cudaStream_t s) {
  const int items = (n / 16 + kDenseWarps - 1) / kDenseWarps * splits;
  dense_gemv_kernel<<<capped_grid(items, max_ctas), kDenseWarps * 32, 0, s>>>(x, tokens, w, n, k, splits, partial);
  return cudaGetLastError();
}

}  // namespace exlr8
