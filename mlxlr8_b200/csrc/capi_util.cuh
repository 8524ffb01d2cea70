// Helpers shared by the extern "C" entry points: CUDA status capture,
// opt-in launch timing, argument checks and workspace carving.
#pragma once

#include <cstdio>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/exlr8_b200.h"

namespace exlr8 {

extern thread_local char g_cuda_error[256];

inline int cuda_status(cudaError_t err) {
  if (err == cudaSuccess) return EXLR8_OK;
  std::snprintf(g_cuda_error, sizeof(g_cuda_error), "%s: %s", cudaGetErrorName(err), cudaGetErrorString(err));
  return EXLR8_ERR_CUDA;
}

#define EXLR8_TRY(expr)                          \
  do {                                           \
    int _st = ::exlr8::cuda_status(expr);        \
    if (_st != EXLR8_OK) return _st;             \
  } while (0)

#define EXLR8_CHECK(expr)                        \
  do {                                           \
    int _st = (expr);                            \
    if (_st != EXLR8_OK) return _st;             \
  } while (0)

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// ---- opt-in launch timing (exlr8_profile_*) --------------------------------
struct Profiler {
  bool on = false;
  int capacity = 0, used = 0;
  cudaEvent_t* events = nullptr;  // 2 * capacity
  int* kinds = nullptr;
};
extern thread_local Profiler g_prof;

struct ProfileScope {
  int slot = -1;
  cudaStream_t stream;
  ProfileScope(int kind, cudaStream_t s) : stream(s) {
    if (g_prof.on && g_prof.used < g_prof.capacity) {
      slot = g_prof.used++;
      g_prof.kinds[slot] = kind;
      cudaEventRecord(g_prof.events[2 * slot], s);
    }
  }
  ~ProfileScope() {
    if (slot >= 0) cudaEventRecord(g_prof.events[2 * slot + 1], stream);
  }
};

#define EXLR8_TIMED(kind, s, expr)   \
  do {                               \
    ::exlr8::ProfileScope _scope(kind, s); \
    EXLR8_TRY(expr);                 \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline bool valid_act(int d) { return d == EXLR8_DTYPE_F32 || d == EXLR8_DTYPE_F16 || d == EXLR8_DTYPE_BF16; }
inline bool valid_scale(int d) { return d == EXLR8_DTYPE_F32 || d == EXLR8_DTYPE_F16; }

// Workspace queries answer kBadSize for sizes that no call accepts, so that
// a query made before the call's own checks never divides by a zero split
// count or overflows.  Rows (tokens x slots) are at most 2^20 in every call.
constexpr size_t kBadSize = ~static_cast<size_t>(0);
inline bool sizes_ok(int64_t tokens, int64_t slots, int a, int b, int64_t experts) {
  return tokens >= 0 && slots > 0 && tokens <= (1 << 20) && slots <= 64 && tokens * slots <= (1 << 20) && a > 0 &&
         b > 0 && a % 128 == 0 && b % 128 == 0 && experts >= 0 && experts <= (1 << 20);
}

// The checks exlr8_moe_layer makes on its expert struct and token count
// before sizing anything (capi.cu); writes the matrix count.
int moe_layer_preflight(const exlr8_trellis_experts* ex, int64_t tokens, int64_t* experts);

constexpr size_t kAlign = 256;
inline size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// Linear workspace carve-out.
struct Carver {
  char* base;
  size_t used = 0;
  explicit Carver(void* b) : base(static_cast<char*>(b)) {}
  template <typename T>
  T* take(size_t bytes) {
    T* p = reinterpret_cast<T*>(base ? base + used : nullptr);
    used += align_up(bytes);
    return p;
  }
};

}  // namespace exlr8
