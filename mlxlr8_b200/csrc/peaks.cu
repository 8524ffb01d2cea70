// Tensor-core peak probe: the issue rate of tcgen05.mma on every SM for the
// two MMA kinds this library's GEMMs use, so that their throughput can be
// reported against the peak of the instruction they actually issue.
//
// One CTA per SM.  Operands are zero-filled shared-memory tiles (128 rows
// of A, N rows of B, 128-byte swizzled K-major rows) whose values do not
// matter for the rate; one thread issues `iters` x 4 MMAs (the four K
// steps of a 128-byte row) into one TMEM accumulator of M = 128 x N, then
// commits and waits (bounded) for the tensor pipe to drain.
//   kind 0: kind::f16, bf16 x bf16 -> f32, K = 16 per MMA
//   kind 1: kind::mxf8f6f4.block_scale, E4M3 x E4M3 with E8M0 scales, K = 32
// No TMA, no multicast, no global memory traffic.
//
// Codec probe: the decode GEMV's inner loop (stream_codec.cuh k4_fragment,
// the exact E4M3 trellis decode of a K4 tile, and its mma.sync) run on
// codes held in shared memory, with the stream kernel's occupancy (two CTAs
// of eight decoding warps per SM), each warp taking eight tiles per step.
// Its rate in weights per second is the compute ceiling of the trellis
// decode on this GPU, independent of HBM.

#include <cuda_runtime.h>

#include "capi_util.cuh"
#include "stream_codec.cuh"
#include "umma.cuh"

namespace exlr8 {

namespace {

constexpr int kPeakThreads = 128;
constexpr uint32_t kPeakTmemCols = 512;
constexpr uint32_t kPeakSfa = 496, kPeakSfb = 504;  // scale-factor columns (mxf8f6f4), after the N <= 256 accumulator

__global__ void __launch_bounds__(kPeakThreads, 1) mma_peak_kernel(int kind, int n, int iters,
                                                                   int32_t* __restrict__ status) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t done;
  __shared__ uint32_t tmem_base;
  const int warp = threadIdx.x >> 5;
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);  // 1 KB aligned (SW128 atoms)
  const uint32_t a_bytes = 128 * 128, b_bytes = static_cast<uint32_t>(n) * 128, sf_bytes = 3 * 512;
  for (uint32_t i = threadIdx.x; i < (a_bytes + b_bytes + sf_bytes) / 16; i += kPeakThreads)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0u, 0u, 0u, 0u);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic stores -> tensor-core reads
  if (threadIdx.x == 0) {
    mbar_init(&done, 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (warp == 0) tmem_alloc(&tmem_base, kPeakTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  if (threadIdx.x == 0) {
    const uint32_t a = smem_u32(smem), b = a + a_bytes, sf = b + b_bytes;
    if (kind == 1) {
      tc_copy_scales(tmem + kPeakSfa, umma_desc_rows16(sf));
      tc_copy_scales(tmem + kPeakSfb, umma_desc_rows16(sf + 512));
      tc_copy_scales(tmem + kPeakSfb + 4, umma_desc_rows16(sf + 1024));
    }
    const uint32_t idesc = kind == 1 ? mx_idesc(kFmtE4M3, kFmtE4M3, n) : bf16_idesc(n);
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint64_t da = umma_desc_sw128(a + kk * 32), db = umma_desc_sw128(b + kk * 32);
        const uint32_t acc = (it | kk) != 0;
        if (kind == 1) {
          tc_mma_mx(tmem, da, db, idesc | (static_cast<uint32_t>(kk) << 4) | (static_cast<uint32_t>(kk) << 29),
                    (tmem + kPeakSfa) | (static_cast<uint32_t>(kk) << 30),
                    (tmem + kPeakSfb) | (static_cast<uint32_t>(kk) << 30), acc);
        } else {
          tc_mma_f16(tmem, da, db, idesc, acc);
        }
      }
    }
    tc_commit(&done);
    if (!mbar_wait(&done, 0)) atomicOr(status, 1);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_free(tmem, kPeakTmemCols);
}

constexpr int kCodecThreads = 256;
constexpr int kCodecTiles = 64;  // K4 tiles of 32 words in shared memory

__global__ void __launch_bounds__(kCodecThreads, 2) codec_peak_kernel(int iters, uint32_t seed,
                                                                      float* __restrict__ sink) {
  __shared__ uint32_t codes[kCodecTiles * 32];
  for (int i = threadIdx.x; i < kCodecTiles * 32; i += kCodecThreads)
    codes[i] = (seed + static_cast<uint32_t>(i)) * 0x9E3779B9u ^ (static_cast<uint32_t>(blockIdx.x) << 16);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t mask = 0x8FFF8FFFu ^ (seed & 0x10u), xorv = 0x3B603B60u;  // runtime operands, as in the kernel
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const uint2 b = make_uint2(0x3C003C00u ^ lane, 0x38003800u ^ lane);
  for (int it = 0; it < iters; ++it) {
    uint32_t word[8], prior[8];
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t* tile = codes + ((warp * 8 + kk + it) & (kCodecTiles - 1)) * 32;
      word[kk] = tile[lane];
      prior[kk] = tile[(lane + 31) & 31];
    }
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t a[4];
      k4_fragment(word[kk], prior[kk], mask, xorv, a);
      mma_f16(acc, a, b);
    }
  }
  if (threadIdx.x == 0) sink[0] = acc[0] + acc[1] + acc[2] + acc[3];
}

}  // namespace

}  // namespace exlr8

using namespace exlr8;

extern "C" int exlr8_codec_peak(int iters, double* weights_per_s, float* sink, void* stream) {
  if (iters <= 0 || !weights_per_s || !sink) return EXLR8_ERR_ARG;
  cudaStream_t s = as_stream(stream);
  int device = 0, sms = 0;
  EXLR8_TRY(cudaGetDevice(&device));
  EXLR8_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  const int grid = 2 * sms;
  cudaEvent_t e0, e1;
  EXLR8_TRY(cudaEventCreate(&e0));
  EXLR8_TRY(cudaEventCreate(&e1));
  codec_peak_kernel<<<grid, kCodecThreads, 0, s>>>(iters / 10 + 1, 7u, sink);  // warm-up
  cudaEventRecord(e0, s);
  codec_peak_kernel<<<grid, kCodecThreads, 0, s>>>(iters, 7u, sink);
  cudaEventRecord(e1, s);
  cudaError_t err = cudaGetLastError();
  if (err == cudaSuccess) err = cudaEventSynchronize(e1);
  float ms = 0.f;
  if (err == cudaSuccess) err = cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  EXLR8_TRY(err);
  const double weights = static_cast<double>(grid) * (kCodecThreads / 32) * 8.0 * iters * 256.0;
  *weights_per_s = weights / (ms * 1e-3);
  return EXLR8_OK;
}

extern "C" int exlr8_tensor_peak(int kind, int n, int iters, double* tflops, int32_t* status, void* stream) {
  if ((kind != 0 && kind != 1) || n < 16 || n > 256 || n % 16 || iters <= 0 || !tflops || !status)
    return EXLR8_ERR_ARG;
  cudaStream_t s = as_stream(stream);
  int device = 0, sms = 0;
  EXLR8_TRY(cudaGetDevice(&device));
  EXLR8_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  const size_t smem = 1024 + 128 * 128 + static_cast<size_t>(n) * 128 + 3 * 512;
  EXLR8_TRY(cudaFuncSetAttribute(mma_peak_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem)));
  EXLR8_TRY(cudaMemsetAsync(status, 0, sizeof(int32_t), s));
  cudaEvent_t e0, e1;
  EXLR8_TRY(cudaEventCreate(&e0));
  EXLR8_TRY(cudaEventCreate(&e1));
  mma_peak_kernel<<<sms, kPeakThreads, smem, s>>>(kind, n, iters / 10 + 1, status);  // warm-up
  cudaEventRecord(e0, s);
  mma_peak_kernel<<<sms, kPeakThreads, smem, s>>>(kind, n, iters, status);
  cudaEventRecord(e1, s);
  cudaError_t err = cudaGetLastError();
  if (err == cudaSuccess) err = cudaEventSynchronize(e1);
  float ms = 0.f;
  if (err == cudaSuccess) err = cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  EXLR8_TRY(err);
  const double k = kind == 1 ? 32.0 : 16.0;
  const double flops = 2.0 * 128.0 * n * k * 4.0 * iters * sms;
  *tflops = flops / (ms * 1e-3) / 1e12;
  return EXLR8_OK;
}
