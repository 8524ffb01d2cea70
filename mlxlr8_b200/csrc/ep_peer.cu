// Expert-parallel exchange over peer memory (NVLink): the dispatch stores each
// routed row straight into its owner's region, the owner's values go back the
// same way, and per-source epoch flags (release stores, acquire loads at
// system scope) tell each side that a peer's rows have landed.  One kernel per
// direction replaces a dispatch kernel plus an NCCL all-to-all.
//
// Every wait is bounded: after kPeerSpinLimit polls the waiting CTA records a
// timeout in the status word for the host and returns.  Kernels of different
// ranks run on different GPUs; no two kernels that wait on each other share a
// GPU.  No TMA or multicast loads are used: remote memory is written with
// plain 16-byte stores and read only through the local region.
//
// Ordering across calls needs no double buffering: a source writes an
// owner's rows for call c + 1 only after it received the owner's values for
// call c, which the owner sends after its expert products of call c have read
// those rows; likewise for the values.

#include "common.cuh"
#include "ep.cuh"

namespace exlr8 {

namespace {

constexpr int kPeerThreads = 256;

// CTAs per peer in the send and return kernels: one per 16 rows of capacity,
// at most 16 (a single CTA per peer copied at a few tens of GB/s).
inline int peer_split(int capacity) {
  const int split = (capacity + 15) / 16;
  return split < 1 ? 1 : (split > 16 ? 16 : split);
}
constexpr uint32_t kPeerSpinLimit = 1u << 20;  // about 1 s of polling

__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void store_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Waits until *flag reaches `target` (epochs only grow); false on timeout.
__device__ bool wait_epoch(const uint32_t* flag, uint32_t target) {
  for (uint32_t i = 0; i < kPeerSpinLimit; ++i) {
    if (static_cast<int32_t>(load_acquire_sys(flag) - target) >= 0) return true;
    __nanosleep(i < 64 ? 32 : 1000);
  }
  return false;
}

__device__ __forceinline__ uint32_t* flags_at(unsigned char* region, int which) {
  return reinterpret_cast<uint32_t*>(region + 256 * which);  // which: 1 arrived, 2 returned, 3 caps
}

__device__ __forceinline__ uint32_t* counters_at(unsigned char* region, int which) {
  return reinterpret_cast<uint32_t*>(region + 1024 + 256 * which);  // which: 0 sent, 1 back
}

// One more CTA of this call is done with a peer (its copies fenced at system
// scope before); true for the last of the `split` CTAs of the peer, which
// resets the count for the next call (kernels of one stream run one after
// another, whatever split the next call uses) and orders everything after
// the others' copies.
__device__ __forceinline__ bool last_of_peer(uint32_t* counter, int split) {
  const uint32_t before = atomicAdd(counter, 1u);
  if (before != static_cast<uint32_t>(split) - 1u) return false;
  *counter = 0u;
  __threadfence_system();
  return true;
}

// CTAs (d, q) for owner d: every CTA ranks this rank's routed slots for d in
// slot order (the same ranking in each); CTA q copies rows q, q + split, ...
// (and q = 0 the local expert ids and slot positions) into d's region.  The
// last CTA of d then stores this rank's capacity and arrival flag there and
// waits until rank d's rows for this call have arrived in this rank's region.
__global__ void __launch_bounds__(kPeerThreads) ep_send_kernel(
    const uint32_t* __restrict__ ids, int tokens, const uint4* __restrict__ x, int row_vecs, int ranks, int rank,
    int experts_per_rank, int capacity, PeerLayout layout, const uint64_t* __restrict__ peers,
    unsigned char* __restrict__ local, int32_t* __restrict__ slot_pos, int32_t* __restrict__ status) {
  extern __shared__ int s_list[];  // [capacity] token of each row, [capacity] local expert id
  __shared__ int s_warp[kPeerThreads / 32];
  __shared__ int s_base;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int d = blockIdx.x, q = blockIdx.y, split = gridDim.y;
  const uint32_t target = *reinterpret_cast<volatile uint32_t*>(local) + 1u;
  unsigned char* owner = reinterpret_cast<unsigned char*>(peers[d]);
  const int slots = tokens * 8;
  const int routed = ranks * experts_per_rank;
  if (tid == 0) s_base = 0;
  __syncthreads();
  for (int chunk = 0; chunk < slots; chunk += kPeerThreads) {
    const int i = chunk + tid;
    int dest = -1, loc = -1;
    if (i < slots) {
      const uint32_t e = ids[static_cast<int64_t>(i / 8) * 9 + i % 8];
      if (e < static_cast<uint32_t>(routed)) {
        dest = static_cast<int>(e) / experts_per_rank;
        loc = static_cast<int>(e) % experts_per_rank;
      }
    }
    const unsigned m = __ballot_sync(0xffffffffu, dest == d);
    if (lane == 0) s_warp[warp] = __popc(m);
    __syncthreads();
    if (dest == d) {
      int pos = s_base + __popc(m & ((1u << lane) - 1u));
      for (int w = 0; w < warp; ++w) pos += s_warp[w];
      if (pos < capacity) {
        s_list[pos] = i / 8;
        s_list[capacity + pos] = loc;
        if (q == 0) slot_pos[i] = d * capacity + pos;
      } else if (q == 0) {
        slot_pos[i] = -1;
        atomicAdd(&status[0], 1);  // capacity overflow: the slot is lost
      }
    } else if (q == 0 && d == 0 && dest < 0 && i < slots) {
      slot_pos[i] = -1;  // id out of range: contributes zero
    }
    __syncthreads();
    if (tid == 0) {
      int add = 0;
      for (int w = 0; w < kPeerThreads / 32; ++w) add += s_warp[w];
      s_base += add;
    }
    __syncthreads();
  }
  const int count = min(s_base, capacity);
  if (q == 0) {
    int32_t* meta = reinterpret_cast<int32_t*>(owner + layout.meta) + static_cast<int64_t>(rank) * capacity;
    for (int j = tid; j < capacity; j += kPeerThreads) meta[j] = j < count ? s_list[capacity + j] : -1;
  }
  uint4* rows = reinterpret_cast<uint4*>(owner + layout.rows) + static_cast<int64_t>(rank) * capacity * row_vecs;
  for (int j = q; j < count; j += split) {
    const uint4* src = x + static_cast<int64_t>(s_list[j]) * row_vecs;
    uint4* dst = rows + static_cast<int64_t>(j) * row_vecs;
    for (int v = tid; v < row_vecs; v += kPeerThreads) dst[v] = src[v];
  }
  __threadfence_system();
  __syncthreads();
  if (tid == 0 && last_of_peer(counters_at(local, 0) + d, split)) {
    flags_at(owner, 3)[rank] = static_cast<uint32_t>(capacity);
    store_release_sys(flags_at(owner, 1) + rank, target);
    if (!wait_epoch(flags_at(local, 1) + d, target)) {
      atomicOr(&status[1], 1);
    } else if (flags_at(local, 3)[d] != static_cast<uint32_t>(capacity)) {
      atomicOr(&status[1], 4);  // source d's rows use another stride: its rows are misread
    }
  }
}

// CTAs (s, q) for source s: CTA q returns the values of source s's valid rows
// q, q + split, ... into s's `back` area; the last CTA of s raises the
// `returned` flag there and waits for owner s's values in this region.
__global__ void __launch_bounds__(kPeerThreads) ep_return_kernel(const uint4* __restrict__ values, int row_vecs,
                                                                 int rank, int capacity, PeerLayout layout,
                                                                 const uint64_t* __restrict__ peers,
                                                                 unsigned char* __restrict__ local,
                                                                 int32_t* __restrict__ status) {
  const int tid = threadIdx.x;
  const int src = blockIdx.x, q = blockIdx.y, split = gridDim.y;
  const uint32_t target = *reinterpret_cast<volatile uint32_t*>(local) + 1u;
  unsigned char* dst_region = reinterpret_cast<unsigned char*>(peers[src]);
  const int32_t* meta = reinterpret_cast<const int32_t*>(local + layout.meta) + static_cast<int64_t>(src) * capacity;
  uint4* back = reinterpret_cast<uint4*>(dst_region + layout.back) + static_cast<int64_t>(rank) * capacity * row_vecs;
  const uint4* v = values + static_cast<int64_t>(src) * capacity * row_vecs;
  for (int j = q; j < capacity; j += split) {
    if (meta[j] < 0) continue;  // rows are filled in order: the rest are empty as well
    for (int c = tid; c < row_vecs; c += kPeerThreads)
      back[static_cast<int64_t>(j) * row_vecs + c] = v[static_cast<int64_t>(j) * row_vecs + c];
  }
  __threadfence_system();
  __syncthreads();
  if (tid == 0 && last_of_peer(counters_at(local, 1) + src, split)) {
    store_release_sys(flags_at(dst_region, 2) + rank, target);
    if (!wait_epoch(flags_at(local, 2) + src, target)) atomicOr(&status[1], 2);
  }
}

// Grid-stride 16-byte copy from local memory to `dst`, which may be another
// GPU's memory mapped into this process (CUDA IPC): the store path the
// exchange kernels use, for measuring the per-direction NVLink bandwidth.
__global__ void peer_write_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src, int64_t vecs) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < vecs; i += stride) dst[i] = src[i];
}

// Runs after the return kernel: this rank's exchanges of the call are done.
__global__ void ep_epoch_kernel(unsigned char* __restrict__ local) {
  *reinterpret_cast<uint32_t*>(local) += 1u;
}

}  // namespace

cudaError_t launch_ep_send(const uint32_t* ids, int tokens, const void* x, int x_dtype, int hidden, int ranks,
                           int rank, int experts_per_rank, int capacity, int max_capacity, const uint64_t* peers,
                           void* local, int32_t* slot_pos, int32_t* status, cudaStream_t s) {
  cudaError_t err = cudaMemsetAsync(status, 0, 2 * sizeof(int32_t), s);
  if (err != cudaSuccess) return err;
  const int elem = x_dtype == kF32 ? 4 : 2;
  const PeerLayout layout = peer_layout(ranks, max_capacity, hidden, elem);
  const size_t smem = 2 * static_cast<size_t>(capacity) * sizeof(int);
  ep_send_kernel<<<dim3(ranks, peer_split(capacity)), kPeerThreads, smem, s>>>(
      ids, tokens, static_cast<const uint4*>(x), hidden * elem / 16, ranks, rank, experts_per_rank, capacity, layout,
      peers, static_cast<unsigned char*>(local), slot_pos, status);
  return cudaGetLastError();
}

cudaError_t launch_ep_return(const void* values, int x_dtype, int hidden, int ranks, int rank, int capacity,
                             int max_capacity, const uint64_t* peers, void* local, int32_t* status, cudaStream_t s) {
  const int elem = x_dtype == kF32 ? 4 : 2;
  const PeerLayout layout = peer_layout(ranks, max_capacity, hidden, elem);
  ep_return_kernel<<<dim3(ranks, peer_split(capacity)), kPeerThreads, 0, s>>>(
      static_cast<const uint4*>(values), hidden * elem / 16, rank, capacity, layout, peers,
      static_cast<unsigned char*>(local), status);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  ep_epoch_kernel<<<1, 1, 0, s>>>(static_cast<unsigned char*>(local));
  return cudaGetLastError();
}

cudaError_t launch_peer_write(void* dst, const void* src, int64_t bytes, cudaStream_t s) {
  const int64_t vecs = bytes / 16;
  if (vecs == 0) return cudaSuccess;
  int device = 0, sms = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err == cudaSuccess) err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (err != cudaSuccess) return err;
  peer_write_kernel<<<sms * 4, 512, 0, s>>>(static_cast<uint4*>(dst), static_cast<const uint4*>(src), vecs);
  return cudaGetLastError();
}

}  // namespace exlr8
