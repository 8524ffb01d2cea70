// Trellis expert kernels around the streaming GEMV (trellis_stream.cu):
// dispatch plan, activation fragments, gate/up finish and output finishes.
//
// Reference roles (exlr8 v0.1.21):
//   plan_kernel             -- fast_prefill.py:19-46 (sort slots by expert, segments)
//   prep_frag_kernel        -- metal/fast_decode_prep.metal (x * in_scale, Hadamard-128)
//   gate_finish_frag_kernel -- metal/fast_decode_gate_finish.metal
//   finish_kernel           -- metal/fast_decode_finish.metal
//   finish_fused_kernel     -- metal/fast_decode_finish_fused.metal
//
// Activations reach the tensor cores as float16 hi/lo pieces (hi = f16(v),
// lo = f16(v - hi)) of the value times a power-of-two scale chosen per
// (row, K split), so products keep about 22 significant bits and the
// float32 accumulation sees the full range.

#include "common.cuh"
#include "codec.cuh"
#include "stream.cuh"
#include "trellis_gemv.cuh"
#include "plan.cuh"
#include "launch.cuh"

namespace exlr8 {

// ---------------------------------------------------------------------------
// Plan
// ---------------------------------------------------------------------------

static inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Large row counts (prefill) are planned by several CTAs: a histogram per
// chunk of kPlanChunk slots, one CTA for the scans, and a stable scatter per
// chunk; smaller plans run in one CTA (plan_body).
constexpr int kPlanChunk = 4096;
constexpr int kPlanMultiMinRows = 4096;
constexpr int kPlanMultiMaxExperts = 2048;  // the scatter's shared counters: 17 x experts ints <= 139 KB
constexpr int kPlanChunkThreads = 512;

inline bool plan_multi(int rows, int experts) {
  return rows > kPlanMultiMinRows && experts <= kPlanMultiMaxExperts;
}
inline int plan_chunks(int rows) { return (rows + kPlanChunk - 1) / kPlanChunk; }

size_t plan_bytes(int rows, int experts) {
  size_t n = 16;                              // header
  n += static_cast<size_t>(rows);             // order
  n += 3 * static_cast<size_t>(rows);         // groups (at most one per row)
  n += 2 * static_cast<size_t>(experts);      // expert count / start
  if (plan_multi(rows, experts)) n += static_cast<size_t>(plan_chunks(rows)) * (experts + 1);  // chunk histograms
  return align_up(n * sizeof(int32_t), 256);
}

PlanView plan_view(void* base, int rows, int experts) {
  PlanView v;
  int32_t* p = static_cast<int32_t*>(base);
  v.header = p;
  p += 16;
  v.order = p;
  p += rows;
  v.group_expert = p;
  p += rows;
  v.group_start = p;
  p += rows;
  v.group_count = p;
  p += rows;
  v.expert_count = p;
  p += experts;
  v.expert_start = p;
  p += experts;
  v.chunk_hist = plan_multi(rows, experts) ? p : nullptr;
  v.zero = nullptr;
  v.zero_count = 0;
  return v;
}

constexpr int kPlanThreads = 1024;

__global__ void __launch_bounds__(kPlanThreads) plan_kernel(const uint32_t* __restrict__ ids, int rows,
                                                            int experts, int period, int skip_slot, PlanView plan) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ int sm[];
  plan_body(ids, rows, experts, period, skip_slot, plan, sm);
}

// Multi-CTA plan, step 1: per chunk of kPlanChunk slots, the slot count of
// every expert (and, in column `experts`, the ids out of range).
__global__ void __launch_bounds__(kPlanChunkThreads) plan_hist_kernel(const uint32_t* __restrict__ ids, int rows,
                                                                      int experts, int period, int skip_slot,
                                                                      int32_t* __restrict__ chunk_hist) {
  extern __shared__ int hist[];  // [experts + 1]
  for (int e = threadIdx.x; e <= experts; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int begin = blockIdx.x * kPlanChunk, end = min(begin + kPlanChunk, rows);
  for (int i = begin + threadIdx.x; i < end; i += blockDim.x) {
    if (skip_slot >= 0 && i % period == skip_slot) continue;
    const uint32_t e = ids[i];
    atomicAdd(&hist[e < static_cast<uint32_t>(experts) ? e : static_cast<uint32_t>(experts)], 1);
  }
  __syncthreads();
  int32_t* row = chunk_hist + static_cast<int64_t>(blockIdx.x) * (experts + 1);
  for (int e = threadIdx.x; e <= experts; e += blockDim.x) row[e] = hist[e];
}

// Step 2 (one CTA): expert totals and starts, groups of at most
// kMaxGroupRows rows, the header, and each chunk's first output position per
// expert (written over its histogram).
__global__ void __launch_bounds__(1024) plan_scan_kernel(int rows, int experts, int chunks, PlanView plan) {
  __shared__ int warp_rows[32], warp_groups[32];
  __shared__ int s_bad;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  for (int i = tid; i < plan.zero_count; i += blockDim.x) plan.zero[i] = 0;
  if (tid == 0) s_bad = 0;
  __syncthreads();
  if (tid < chunks) atomicAdd(&s_bad, plan.chunk_hist[static_cast<int64_t>(tid) * (experts + 1) + experts]);
  // Experts in blocks of blockDim: per expert its total and group count, a
  // block-wide exclusive scan, carried across blocks.
  int row_carry = 0, group_carry = 0;
  for (int e0 = 0; e0 < experts; e0 += blockDim.x) {
    const int e = e0 + tid;
    int total = 0;
    if (e < experts) {
      for (int c = 0; c < chunks; ++c) {
        int32_t* cell = plan.chunk_hist + static_cast<int64_t>(c) * (experts + 1) + e;
        const int n = *cell;
        *cell = total;  // offset of chunk c inside the expert's rows
        total += n;
      }
    }
    const int groups = (total + kMaxGroupRows - 1) / kMaxGroupRows;
    int r = total, g = groups;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int ru = __shfl_up_sync(0xffffffffu, r, off), gu = __shfl_up_sync(0xffffffffu, g, off);
      if (lane >= off) {
        r += ru;
        g += gu;
      }
    }
    if (lane == 31) {
      warp_rows[warp] = r;
      warp_groups[warp] = g;
    }
    __syncthreads();
    if (warp == 0) {
      int wr = lane < nwarps ? warp_rows[lane] : 0, wg = lane < nwarps ? warp_groups[lane] : 0;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int ru = __shfl_up_sync(0xffffffffu, wr, off), gu = __shfl_up_sync(0xffffffffu, wg, off);
        if (lane >= off) {
          wr += ru;
          wg += gu;
        }
      }
      if (lane < nwarps) {
        warp_rows[lane] = wr;
        warp_groups[lane] = wg;
      }
    }
    __syncthreads();
    const int row_base = row_carry + (warp > 0 ? warp_rows[warp - 1] : 0) + r - total;
    const int group_base = group_carry + (warp > 0 ? warp_groups[warp - 1] : 0) + g - groups;
    if (e < experts) {
      plan.expert_start[e] = row_base;
      plan.expert_count[e] = total;
      for (int c = 0; c < groups; ++c) {
        plan.group_expert[group_base + c] = e;
        plan.group_start[group_base + c] = row_base + c * kMaxGroupRows;
        plan.group_count[group_base + c] = min(kMaxGroupRows, total - c * kMaxGroupRows);
      }
      for (int c = 0; c < chunks; ++c) plan.chunk_hist[static_cast<int64_t>(c) * (experts + 1) + e] += row_base;
    }
    row_carry += warp_rows[nwarps - 1];
    group_carry += warp_groups[nwarps - 1];
    __syncthreads();
  }
  if (tid == 0) {
    plan.header[0] = group_carry;
    plan.header[1] = rows;
    for (int c = 2; c < 8; ++c) plan.header[c] = 0;
    plan.header[8] = s_bad;
    plan.header[9] = 0;
  }
}

// Step 3: each chunk scatters its slots in slot order to the positions the
// scan gave it (stable: earlier slots of an expert come first).
__global__ void __launch_bounds__(kPlanChunkThreads) plan_scatter_kernel(const uint32_t* __restrict__ ids, int rows,
                                                                         int experts, int period, int skip_slot,
                                                                         PlanView plan) {
  extern __shared__ int sm[];
  int* next = sm;                 // [experts] next output position per expert
  int* wcount = sm + experts;     // [warps][experts]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  const int32_t* start = plan.chunk_hist + static_cast<int64_t>(blockIdx.x) * (experts + 1);
  for (int e = tid; e < experts; e += blockDim.x) next[e] = start[e];
  const unsigned lt_mask = (1u << lane) - 1u;
  const int begin = blockIdx.x * kPlanChunk, end = min(begin + kPlanChunk, rows);
  for (int chunk = begin; chunk < end; chunk += blockDim.x) {
    for (int j = tid; j < nwarps * experts; j += blockDim.x) wcount[j] = 0;
    __syncthreads();
    const int i = chunk + tid;
    const bool skipped = i < end && skip_slot >= 0 && i % period == skip_slot;
    const uint32_t raw = (i < end && !skipped) ? ids[i] : 0xFFFFFFFFu;
    const bool valid = raw < static_cast<uint32_t>(experts);
    const uint32_t key = valid ? raw : 0xFFFFFFFFu;
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    const int leader = __ffs(peers) - 1;
    const int rank = __popc(peers & lt_mask);
    if (valid && lane == leader) wcount[warp * experts + key] = __popc(peers);
    __syncthreads();
    if (valid) {
      int prior = 0;
      for (int w = 0; w < warp; ++w) prior += wcount[w * experts + key];
      plan.order[next[key] + prior + rank] = i;
    }
    __syncthreads();
    if (valid && lane == leader) atomicAdd(&next[key], __popc(peers));
    __syncthreads();
  }
}

cudaError_t launch_plan(const uint32_t* ids, int rows, int experts, int period, int skip_slot, PlanView plan,
                        cudaStream_t s) {
  if (plan_multi(rows, experts) && plan.chunk_hist != nullptr) {
    // Plain launches: the plan heads its call's kernel chain.
    const int chunks = plan_chunks(rows);
    const int per = period > 0 ? period : 1;
    const size_t hist_smem = static_cast<size_t>(experts + 1) * sizeof(int);
    const size_t scatter_smem = static_cast<size_t>(1 + kPlanChunkThreads / 32) * experts * sizeof(int);
    static const cudaError_t attr = cudaFuncSetAttribute(
        plan_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
        static_cast<int>((1 + kPlanChunkThreads / 32) * kPlanMultiMaxExperts * sizeof(int)));
    if (attr != cudaSuccess) return attr;
    plan_hist_kernel<<<chunks, kPlanChunkThreads, hist_smem, s>>>(ids, rows, experts, per, skip_slot, plan.chunk_hist);
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    plan_scan_kernel<<<1, 1024, 0, s>>>(rows, experts, chunks, plan);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
    plan_scatter_kernel<<<chunks, kPlanChunkThreads, scatter_smem, s>>>(ids, rows, experts, per, skip_slot, plan);
    return cudaGetLastError();
  }
  const size_t smem = plan_smem_bytes(experts, kPlanThreads / 32);
  if (smem > 48 * 1024) {
    cudaError_t err = cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
    if (err != cudaSuccess) return err;
  }
  // The plan heads its call's kernel chain: a plain launch, fully ordered
  // after earlier work in the stream (later kernels of the chain rely on it).
  static const cudaError_t carve = prefer_shared_carveout(plan_kernel);
  if (carve != cudaSuccess) return carve;
  plan_kernel<<<1, kPlanThreads, smem, s>>>(ids, rows, experts, period > 0 ? period : 1, skip_slot, plan);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Activation fragments.  One warp per (projection, slot, 128-wide block):
// the block is transformed in registers, its maximum picks a power-of-two
// scale, and the scaled values are written as a float16 hi/lo fragment record
// (see stream.cuh) with the block's unscale in the record header.
// ---------------------------------------------------------------------------

constexpr int kFragWarps = 4;

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float split_piece(float v, int piece) {
  const float hi = __half2float(__float2half_rn(v));
  return piece ? v - hi : hi;
}

// Scale exponent for a block maximum: the scaled maximum lies in [2^14, 2^15).
__device__ __forceinline__ int piece_exponent(float m) {
  int ex = 0;
  if (m > 0.0f && m < 3.0e38f) {
    frexpf(m, &ex);
    ex -= 15;
  }
  return ex;
}

// v: the warp's transformed block (lane l holds element l + 32j); stage: 128
// floats of this warp's shared memory; dst: the block's fragment record.
// mx_order selects the MXFP4 K order of joined_stream.cuh (K tile s: pairs
// 32(s/2) + 8 tig + 4(s%2) + {0,1} and + {2,3}) instead of the tensor-core
// order (16 s + 2 tig + {0,1} and + {8,9}).
__device__ __forceinline__ void write_block_record(const float v[4], float* stage, int lane, unsigned char* dst,
                                                   int mx_order = 0) {
  float m = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    stage[lane + 32 * j] = v[j];
    m = fmaxf(m, fabsf(v[j]));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  const int ex = piece_exponent(m);
  const float scale = ldexpf(1.0f, -ex);
  __syncwarp();
  uint2* out = reinterpret_cast<uint2*>(dst);
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int idx = lane + 32 * q;
    const int ktl = idx >> 3, piece = (idx >> 2) & 1, tig = idx & 3;
    const int o0 = mx_order ? 32 * (ktl >> 1) + 8 * tig + 4 * (ktl & 1) : ktl * 16 + 2 * tig;
    const int o1 = mx_order ? o0 + 2 : o0 + 8;
    uint2 b;
    b.x = pack_half2(split_piece(stage[o0] * scale, piece), split_piece(stage[o0 + 1] * scale, piece));
    b.y = pack_half2(split_piece(stage[o1] * scale, piece), split_piece(stage[o1 + 1] * scale, piece));
    out[idx] = b;
  }
  if (lane < 4) reinterpret_cast<float*>(dst + 512)[lane] = lane == 0 ? ldexpf(1.0f, ex) : 0.0f;
  __syncwarp();
}

template <bool kSkipEmpty>
__global__ void __launch_bounds__(kFragWarps * 32) prep_frag_kernel(
    const void* __restrict__ x, int x_dtype, int per_slot, int slots_per_token, const uint32_t* __restrict__ ids,
    int nslots, const void* __restrict__ in0, const void* __restrict__ in1, int scale_dtype, int features,
    int experts, int projections, int scale_stride, int mx_order, unsigned char* __restrict__ frag) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float stage[kFragWarps][128];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int blocks = features / 128;
  const int64_t task = static_cast<int64_t>(blockIdx.x) * kFragWarps + warp;  // (proj * nslots + slot) * blocks + b
  if (task >= static_cast<int64_t>(projections) * nslots * blocks) return;
  const int b = static_cast<int>(task % blocks);
  const int64_t ps = task / blocks;
  const int slot = static_cast<int>(ps % nslots), proj = static_cast<int>(ps / nslots);
  const int64_t row = per_slot ? slot : slot / slots_per_token;
  const int c0 = b * 128 + lane;
  // Sparse slot lists (an expert-parallel owner's capacity rows) check the
  // id before loading the row; dense lists load both at once.
  const uint32_t e = ids[slot];
  const bool ok = e < static_cast<uint32_t>(experts);
  if (kSkipEmpty && !ok) return;
  float xv[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) xv[j] = load_act(x, x_dtype, row * features + c0 + 32 * j);
  if (!ok) return;  // no plan row reads the record of a slot without an expert
  const void* scale = proj ? in1 : in0;
  float v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    v[j] = ok ? __fmul_rn(xv[j], load_scale(scale, scale_dtype, static_cast<int64_t>(e) * scale_stride + c0 + 32 * j))
              : 0.0f;
  hadamard128(v, lane);
  write_block_record(v, stage[warp], lane, frag + task * kFragBlockBytes, mx_order);
}

cudaError_t launch_prep_frag(const void* x, int x_dtype, int per_slot, int slots_per_token, const uint32_t* ids,
                             int nslots, const void* in0, const void* in1, int scale_dtype, int features, int experts,
                             int projections, unsigned char* frag, cudaStream_t s, int scale_stride, int mx_order,
                             int skip_empty) {
  if (scale_stride < 0) scale_stride = features;
  const int64_t tasks = static_cast<int64_t>(projections) * nslots * (features / 128);
  if (tasks == 0) return cudaSuccess;
  const int64_t grid = (tasks + kFragWarps - 1) / kFragWarps;
  static const cudaError_t carve0 = prefer_shared_carveout(prep_frag_kernel<false>);
  static const cudaError_t carve1 = prefer_shared_carveout(prep_frag_kernel<true>);
  if (carve0 != cudaSuccess) return carve0;
  if (carve1 != cudaSuccess) return carve1;
  auto kernel = skip_empty ? prep_frag_kernel<true> : prep_frag_kernel<false>;
  return launch_pdl(kernel, dim3(static_cast<unsigned>(grid)), dim3(kFragWarps * 32), 0, s, x, x_dtype,
                    per_slot, slots_per_token, ids, nslots, in0, in1, scale_dtype, features, experts, projections,
                    scale_stride, mx_order, frag);
}

// gate/up split sum, Hadamard, output scales, typed SwiGLU, down input scale,
// Hadamard -> down fragment record.  One warp per (slot, 128-wide block of
// the intermediate features).  The partials of up to kGateFinishSplits
// splits and the id's three scale vectors are in flight together (the
// partials do not depend on the expert id; the scales need only the id),
// then the splits are summed in split order.  Warps past the slots' blocks
// form the bf16 shared expert's h = SwiGLU(T(g), T(u)), one per (token,
// 128-wide block).
constexpr int kGateFinishSplits = 16;  // splits loaded per round trip (the most gate_up_splits chooses)

template <bool kSkipEmpty>
__global__ void __launch_bounds__(kFragWarps * 32) gate_finish_frag_kernel(
    const float* __restrict__ partial, int gu_splits, const uint32_t* __restrict__ ids, int nslots,
    const void* __restrict__ out_gate, const void* __restrict__ out_up, const void* __restrict__ in_down,
    int scale_dtype, int features, int experts, int act_dtype, unsigned char* __restrict__ frag,
    const float* __restrict__ dense_g, const float* __restrict__ dense_u, int dense_splits, int dense_tokens,
    void* __restrict__ dense_h, int mx_order) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float stage[kFragWarps][128];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int blocks = features / 128;
  const int64_t task = static_cast<int64_t>(blockIdx.x) * kFragWarps + warp;  // slot * blocks + b
  const int64_t slot_tasks = static_cast<int64_t>(nslots) * blocks;
  if (task >= slot_tasks) {
    const int64_t d = task - slot_tasks;  // token * blocks + b
    if (d >= static_cast<int64_t>(dense_tokens) * blocks) return;
    const int64_t total = static_cast<int64_t>(dense_tokens) * features;
    const int64_t i0 = (d / blocks) * features + (d % blocks) * 128 + lane;
    float g[4] = {0.f, 0.f, 0.f, 0.f}, u[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
    for (int sp = 0; sp < dense_splits; ++sp) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        g[j] += __ldcg(dense_g + sp * total + i0 + 32 * j);
        u[j] += __ldcg(dense_u + sp * total + i0 + 32 * j);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) store_act(dense_h, act_dtype, i0 + 32 * j, swiglu_typed(act_dtype, g[j], u[j]));
    return;
  }
  const int b = static_cast<int>(task % blocks);
  const int slot = static_cast<int>(task / blocks);
  const int c0 = b * 128 + lane;
  const float* pg = partial + static_cast<int64_t>(slot) * gu_splits * features + c0;
  const float* pu = partial + (static_cast<int64_t>(nslots) + slot) * gu_splits * features + c0;
  const uint32_t id = ids[slot];
  float gate[4] = {0.f, 0.f, 0.f, 0.f}, up[4] = {0.f, 0.f, 0.f, 0.f};
  float sg[4], su[4], sd[4];
  const int64_t e = id;
  const bool ok = e < experts;
  // Sparse slot lists (an expert-parallel owner's fixed-capacity rows, most
  // of them empty): a slot without an expert has no plan row, so its record
  // is never read; skip its partials instead of loading them.  (Dense lists
  // do not wait for the id before loading.)
  if (kSkipEmpty && !ok) return;
  for (int s0 = 0; s0 < gu_splits; s0 += kGateFinishSplits) {
    float lg[kGateFinishSplits][4], lu[kGateFinishSplits][4];
#pragma unroll
    for (int sp = 0; sp < kGateFinishSplits; ++sp) {
      const bool have = s0 + sp < gu_splits;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t o = static_cast<int64_t>(s0 + sp) * features + 32 * j;
        lg[sp][j] = have ? __ldcg(pg + o) : 0.0f;
        lu[sp][j] = have ? __ldcg(pu + o) : 0.0f;
      }
    }
    if (s0 == 0) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t si = (ok ? e : 0) * features + c0 + 32 * j;
        sg[j] = load_scale(out_gate, scale_dtype, si);
        su[j] = load_scale(out_up, scale_dtype, si);
        sd[j] = load_scale(in_down, scale_dtype, si);
      }
    }
#pragma unroll
    for (int sp = 0; sp < kGateFinishSplits; ++sp) {
      if (s0 + sp < gu_splits) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          gate[j] += lg[sp][j];
          up[j] += lu[sp][j];
        }
      }
    }
  }
  if (gu_splits <= 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t si = (ok ? e : 0) * features + c0 + 32 * j;
      sg[j] = load_scale(out_gate, scale_dtype, si);
      su[j] = load_scale(out_up, scale_dtype, si);
      sd[j] = load_scale(in_down, scale_dtype, si);
    }
  }
  hadamard128(gate, lane);
  hadamard128(up, lane);
  float act[4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    act[j] = ok ? __fmul_rn(swiglu_typed(act_dtype, __fmul_rn(gate[j], sg[j]), __fmul_rn(up[j], su[j])), sd[j])
                : 0.0f;
  hadamard128(act, lane);
  write_block_record(act, stage[warp], lane, frag + task * kFragBlockBytes, mx_order);
}

cudaError_t launch_gate_finish_frag(const float* partial, int gu_splits, const uint32_t* ids, int nslots,
                                    const void* out_gate, const void* out_up, const void* in_down, int scale_dtype,
                                    int features, int experts, int act_dtype, unsigned char* frag,
                                    const float* dense_g, const float* dense_u, int dense_splits, int dense_tokens,
                                    void* dense_h, cudaStream_t s, int mx_order, int skip_empty) {
  if (!dense_h) dense_tokens = 0;
  const int64_t tasks = (static_cast<int64_t>(nslots) + dense_tokens) * (features / 128);
  if (tasks == 0) return cudaSuccess;
  const int64_t grid = (tasks + kFragWarps - 1) / kFragWarps;
  static const cudaError_t carve0 = prefer_shared_carveout(gate_finish_frag_kernel<false>);
  static const cudaError_t carve1 = prefer_shared_carveout(gate_finish_frag_kernel<true>);
  if (carve0 != cudaSuccess) return carve0;
  if (carve1 != cudaSuccess) return carve1;
  auto kernel = skip_empty ? gate_finish_frag_kernel<true> : gate_finish_frag_kernel<false>;
  return launch_pdl(kernel, dim3(static_cast<unsigned>(grid)), dim3(kFragWarps * 32), 0, s, partial, gu_splits, ids,
                    nslots, out_gate, out_up, in_down, scale_dtype, features, experts, act_dtype, frag, dense_g,
                    dense_u, dense_splits, dense_tokens, dense_h, mx_order);
}

// ---------------------------------------------------------------------------
// Finishes
// ---------------------------------------------------------------------------

// Split sum, Hadamard, signed output scale, cast to the activation type.
__global__ void __launch_bounds__(128) finish_kernel(const float* __restrict__ partial, int splits,
                                                     const int32_t* __restrict__ row_map,
                                                     const uint32_t* __restrict__ ids, int nslots,
                                                     const void* __restrict__ out_scale, int scale_dtype,
                                                     int features, int experts, int act_dtype,
                                                     void* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int block = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int slot = blockIdx.y;
  if (block * 128 >= features) return;
  const int64_t e = ids[slot];
  const int64_t prow = row_map ? row_map[slot] : static_cast<int64_t>(slot) * splits;
  if (e >= experts || prow < 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) store_act(out, act_dtype, static_cast<int64_t>(slot) * features + block * 128 + lane + 32 * j, 0.0f);
    return;
  }
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  const float* ps = partial + prow * features + block * 128 + lane;
#pragma unroll 4
  for (int s = 0; s < splits; ++s) {
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] += ps[static_cast<int64_t>(s) * features + 32 * j];
  }
  hadamard128(v, lane);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int col = block * 128 + lane + 32 * j;
    store_act(out, act_dtype, static_cast<int64_t>(slot) * features + col,
              __fmul_rn(v[j], load_scale(out_scale, scale_dtype, e * features + col)));
  }
}

cudaError_t launch_finish(const float* partial, int splits, const int32_t* row_map, const uint32_t* ids, int nslots,
                          const void* out_scale, int scale_dtype, int features, int experts, int act_dtype, void* out,
                          cudaStream_t s) {
  dim3 grid((features / 128 + 3) / 4, nslots);
  static const cudaError_t carve = prefer_shared_carveout(finish_kernel);
  if (carve != cudaSuccess) return carve;
  return launch_pdl(finish_kernel, grid, dim3(128), 0, s, partial, splits, row_map, ids, nslots, out_scale,
                    scale_dtype, features, experts, act_dtype, out);
}

// Nine slots per token (eight routed + shared), one warp per slot: expert
// finish (split sum, Hadamard, out scale, cast), then warp 0 forms the routed
// weighted sum in the order slot 0, then (slot r + 0) + total for r = 1..7,
// T(routed), T(routed + T(shared)), T(residual + combined)
// (metal/fast_decode_finish_fused.metal:52-62).  When shared_values is given
// it holds the typed shared-expert output [tokens][h] and slot 8 of partial is
// not read.  shared_values are the dense shared expert's float32 split
// partials, summed and cast here.
constexpr int kFinishSplits = 16;  // down-split partials loaded per round trip

__global__ void __launch_bounds__(288) finish_fused_kernel(const float* __restrict__ partial, int splits,
                                                           const int32_t* __restrict__ row_map,
                                                           const uint32_t* __restrict__ ids, int tokens,
                                                           const void* __restrict__ out_scale, int scale_dtype,
                                                           int features, int experts,
                                                           const float* __restrict__ scores,
                                                           const void* __restrict__ residual,
                                                           const void* __restrict__ shared_values, int shared_splits,
                                                           int act_dtype, void* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float products[9][128];
  const int lane = threadIdx.x & 31, slot = threadIdx.x >> 5;
  const int block = blockIdx.x, token = blockIdx.y;
  const int row = token * 9 + slot;
  const int64_t off0 = static_cast<int64_t>(token) * features + block * 128 + lane;
  // Loads that do not depend on the expert id go out first (one round trip),
  // then the id-dependent output scales.
  float res[4] = {0.f, 0.f, 0.f, 0.f};
  if (slot == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) res[j] = load_act(residual, act_dtype, off0 + 32 * j);
  }
  if (slot == 8 && shared_values != nullptr) {
    // Dense shared expert: float32 split partials [shared_splits][tokens][h].
    const int64_t total = static_cast<int64_t>(tokens) * features;
    float a[4] = {0.f, 0.f, 0.f, 0.f};
    const float* sv = static_cast<const float*>(shared_values) + off0;
#pragma unroll 8
    for (int sp = 0; sp < shared_splits; ++sp) {
#pragma unroll
      for (int j = 0; j < 4; ++j) a[j] += __ldcg(sv + sp * total + 32 * j);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) products[8][lane + 32 * j] = round_to(act_dtype, a[j]);
  } else {
    const int64_t e = ids[row];
    const float weight = slot < 8 ? scores[token * 8 + slot] : 1.0f;
    const int64_t prow = row_map ? row_map[row] : static_cast<int64_t>(row) * splits;
    const bool ok = e < experts && prow >= 0;  // an out-of-range id contributes zero
    // The output scales and up to kFinishSplits splits' partials go out
    // together, then the splits are summed in split order.
    float sc[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      sc[j] = load_scale(out_scale, scale_dtype, (ok ? e : 0) * features + block * 128 + lane + 32 * j);
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (prow >= 0) {
      const float* ps = partial + prow * features + block * 128 + lane;
      for (int s0 = 0; s0 < splits; s0 += kFinishSplits) {
        float lv[kFinishSplits][4];
#pragma unroll
        for (int sp = 0; sp < kFinishSplits; ++sp)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            lv[sp][j] = s0 + sp < splits ? __ldcg(ps + static_cast<int64_t>(s0 + sp) * features + 32 * j) : 0.0f;
#pragma unroll
        for (int sp = 0; sp < kFinishSplits; ++sp)
          if (s0 + sp < splits) {
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] += lv[sp][j];
          }
      }
    }
    hadamard128(v, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float value = ok ? round_to(act_dtype, __fmul_rn(v[j], sc[j])) : 0.0f;
      products[slot][lane + 32 * j] = slot < 8 ? __fmul_rn(value, weight) : value;
    }
  }
  __syncthreads();
  if (slot != 0) return;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = lane + 32 * j;
    float total = __fadd_rn(products[0][c], 0.0f);
#pragma unroll
    for (int r = 1; r < 8; ++r) total = __fadd_rn(__fadd_rn(products[r][c], 0.0f), total);
    const float routed = round_to(act_dtype, total);
    const float combined = round_to(act_dtype, __fadd_rn(routed, round_to(act_dtype, products[8][c])));
    store_act(out, act_dtype, off0 + 32 * j, __fadd_rn(res[j], combined));
  }
}

cudaError_t launch_finish_fused(const float* partial, int splits, const int32_t* row_map, const uint32_t* ids, int tokens,
                                const void* out_scale, int scale_dtype, int features, int experts,
                                const float* scores, const void* residual, const void* shared_values,
                                int shared_splits, int act_dtype, void* out, cudaStream_t s) {
  dim3 grid(features / 128, tokens);
  static const cudaError_t carve = prefer_shared_carveout(finish_fused_kernel);
  if (carve != cudaSuccess) return carve;
  return launch_pdl(finish_fused_kernel, grid, dim3(288), 0, s, partial, splits, row_map, ids, tokens, out_scale,
                    scale_dtype, features, experts, scores, residual, shared_values, shared_splits, act_dtype, out);
}

}  // namespace exlr8
