// Pinned host buffers read and written by the layer's own kernels.
//
// A decode step's inputs (x and residual) and its result are a few KB each.
// Moved by copy-engine copies they cost a DMA hand-off on each side of the
// step and cut the layer's programmatic-dependent-launch chain twice.
// Instead:
//   stage_in_kernel -- at the head of the chain, reads the pinned x and
//                      residual over PCIe (their device-accessible
//                      addresses) into the layer's device buffers;
//   the finish      -- writes the result straight into the pinned `out`,
//                      given its device-accessible address
//                      (exlr8_host_device_pointer).
// Only page-locked host memory (or device memory) is accepted: the pointer
// kind is checked with cudaPointerGetAttributes on the host, and a pageable
// pointer is refused there, never dereferenced by a kernel.

#include "capi_util.cuh"
#include "launch.cuh"

namespace exlr8 {

namespace {

constexpr int kStageThreads = 256;

// dst0 <- src0 and dst1 <- src1, `words` 16-byte words each.  The first
// words' host loads go out before the wait on the previous grid: the pinned
// inputs are written by the host before the launch, not by earlier kernels.
// The device stores come after it, since earlier kernels of the stream may
// still read the device buffers.
__global__ void __launch_bounds__(kStageThreads) stage_in_kernel(const uint4* __restrict__ src0,
                                                                  uint4* __restrict__ dst0,
                                                                  const uint4* __restrict__ src1,
                                                                  uint4* __restrict__ dst1, int64_t words) {
  pdl_launch_dependents();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kStageThreads;
  int64_t i = static_cast<int64_t>(blockIdx.x) * kStageThreads + threadIdx.x;
  uint4 a = make_uint4(0, 0, 0, 0), b = make_uint4(0, 0, 0, 0);
  if (i < words) {
    a = src0[i];
    b = src1[i];
  }
  pdl_wait();
  while (i < words) {
    const int64_t n = i + stride;
    uint4 na = make_uint4(0, 0, 0, 0), nb = make_uint4(0, 0, 0, 0);
    if (n < words) {
      na = src0[n];
      nb = src1[n];
    }
    dst0[i] = a;
    dst1[i] = b;
    a = na;
    b = nb;
    i = n;
  }
}

// Device-accessible address of `p`: device or managed memory as is,
// page-locked host memory at its mapped address; nullptr for anything else
// (pageable or unknown host memory).
void* device_address(const void* p) {
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    cudaGetLastError();  // an invalid pointer's error is not sticky: clear it
    return nullptr;
  }
  switch (attr.type) {
    case cudaMemoryTypeDevice:
    case cudaMemoryTypeManaged:
      return const_cast<void*>(p);
    case cudaMemoryTypeHost:
      if (attr.devicePointer == nullptr) return nullptr;
      if (attr.hostPointer == nullptr) return attr.devicePointer;
      // The two addresses name the same byte; keep p's offset from it.
      return static_cast<char*>(attr.devicePointer) +
             (reinterpret_cast<const char*>(p) - static_cast<const char*>(attr.hostPointer));
    default:
      return nullptr;
  }
}

}  // namespace

}  // namespace exlr8

using namespace exlr8;

extern "C" {

int exlr8_host_device_pointer(const void* ptr, void** device_ptr) {
  if (!ptr || !device_ptr) return EXLR8_ERR_ARG;
  void* d = device_address(ptr);
  if (!d) return EXLR8_ERR_ARG;
  *device_ptr = d;
  return EXLR8_OK;
}

int exlr8_stage_in(const void* src0, void* dst0, const void* src1, void* dst1, int64_t bytes, void* stream) {
  if (bytes < 0 || bytes % 16) return EXLR8_ERR_ARG;
  if (bytes == 0) return EXLR8_OK;
  if (!src0 || !dst0 || !src1 || !dst1) return EXLR8_ERR_ARG;
  if (!aligned16(src0) || !aligned16(dst0) || !aligned16(src1) || !aligned16(dst1)) return EXLR8_ERR_ALIGN;
  const void* s0 = device_address(src0);
  const void* s1 = device_address(src1);
  void* d0 = device_address(dst0);
  void* d1 = device_address(dst1);
  if (!s0 || !s1 || !d0 || !d1) return EXLR8_ERR_ARG;
  if (!aligned16(s0) || !aligned16(s1) || !aligned16(d0) || !aligned16(d1)) return EXLR8_ERR_ALIGN;
  const int64_t words = bytes / 16;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (words + kStageThreads - 1) / kStageThreads;
  const int64_t cap = static_cast<int64_t>(sms) * 8;
  const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
  return cuda_status(launch_pdl(stage_in_kernel, dim3(grid), dim3(kStageThreads), 0, as_stream(stream),
                                static_cast<const uint4*>(s0), static_cast<uint4*>(d0), static_cast<const uint4*>(s1),
                                static_cast<uint4*>(d1), words));
}

}  // extern "C"
