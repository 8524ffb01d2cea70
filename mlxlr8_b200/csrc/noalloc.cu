// exlr8_moe_layer_noalloc: the MoE layer for callers that cannot allocate
// device memory.
//
// Some hosts of this library hold device pointers but own no device
// allocator: an FFI caller that receives its tensors from another runtime,
// or a serving process whose memory pool is fixed at start-up and which must
// not call cudaMalloc (it may synchronise the device, fragment the pool, or
// fail once the pool holds all memory).  Such a caller cannot provide the
// workspace that exlr8_moe_layer takes.  This entry point uses instead one
// fixed scratch array that lives in this library's device module: every GPU
// that loads the library holds EXLR8_NOALLOC_SCRATCH_BYTES of it until the
// process exits.  Nothing here calls cudaMalloc, cudaFree or any allocating
// routine.
//
// The array's name is only a host-side handle: host code never passes it to
// a kernel.  The first call on each device, with that device current, looks
// up its device address with cudaGetSymbolAddress (checked) and keeps it for
// later calls; make that first call before any stream capture.
//
// All calls on a device share the array and it keeps the previous call's
// contents.  The layer's first kernel resets the work counters it needs at
// zero, and every other byte a call reads is written earlier in the same
// call.  Calls that overlap on the GPU (other streams, other threads) race on
// the array and must be serialised by the caller.

#include <cuda_runtime.h>

#include <mutex>

#include "../../include/exlr8_b200.h"
#include "capi_util.cuh"

namespace {

__device__ __align__(256) unsigned char g_noalloc_scratch[EXLR8_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_address[kMaxDevices] = {};

// Device address of the scratch array on the current device.
int noalloc_scratch(void** address) {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return EXLR8_ERR_CUDA;
  if (device < 0 || device >= kMaxDevices) return EXLR8_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_address[device] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return EXLR8_ERR_CUDA;
    g_noalloc_address[device] = p;
  }
  *address = g_noalloc_address[device];
  return EXLR8_OK;
}

}  // namespace

extern "C" int exlr8_moe_layer_noalloc(const void* x, int x_dtype, const void* residual, int64_t tokens,
                                       const float* gate_weight, const float* bias,
                                       const exlr8_trellis_experts* experts, const exlr8_dense_expert* shared,
                                       void* out, uint32_t* indices, float* scores, void* stream) {
  // The struct and the token count are validated before anything is sized
  // from them, with the same checks and status codes as exlr8_moe_layer.
  int64_t count = 0;
  const int checked = exlr8::moe_layer_preflight(experts, tokens, &count);
  if (checked != EXLR8_OK) return checked;
  const size_t need = exlr8_moe_layer_workspace(tokens, experts->hidden, experts->intermediate, count);
  if (need > EXLR8_NOALLOC_SCRATCH_BYTES) return EXLR8_ERR_STATIC_LIMIT;
  void* scratch = nullptr;
  const int status = noalloc_scratch(&scratch);
  if (status != EXLR8_OK) return status;
  return exlr8_moe_layer(x, x_dtype, residual, tokens, gate_weight, bias, experts, shared, out, indices, scores,
                         scratch, EXLR8_NOALLOC_SCRATCH_BYTES, stream);
}
