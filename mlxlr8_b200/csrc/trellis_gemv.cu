// Trellis expert kernels for small batches (decode): dispatch plan, input
// transform, tensor-core decode GEMV, gate/up finish and output finishes.
//
// Reference roles (exlr8 v0.1.21):
//   plan_kernel        -- fast_prefill.py:19-46 (sort slots by expert, segment table)
//   prep_kernel        -- metal/fast_decode_prep.metal (x * in_scale, Hadamard-128)
//   trellis_gemv_kernel-- metal/fast_decode_linear.metal (decode + dot, split-K partials)
//   gate_finish_kernel -- metal/fast_decode_gate_finish.metal
//   finish_kernel      -- metal/fast_decode_finish.metal
//   finish_fused_kernel-- metal/fast_decode_finish_fused.metal
//
// The GEMV decodes each 16x16 trellis tile straight into mma.sync A-fragment
// registers (the trellis tensor-core permutation is the m16n8k16 A layout),
// multiplies it with activations held as float16 hi/lo pairs (hi = f16(x),
// lo = f16(x - hi), a per-row power-of-two scale keeps them in range) and
// accumulates in float32 in the tensor cores.  Rows that share an expert
// share the decoded tile (up to kMaxGroupRows rows, 16 MMA columns).

#include "common.cuh"
#include "codec.cuh"
#include "trellis_gemv.cuh"

namespace exlr8 {

// ---------------------------------------------------------------------------
// Plan
// ---------------------------------------------------------------------------

static inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

size_t plan_bytes(int rows, int experts) {
  size_t n = 16;                              // header
  n += static_cast<size_t>(rows);             // order
  n += 3 * static_cast<size_t>(rows);         // groups (at most one per row)
  n += 2 * static_cast<size_t>(experts);      // expert count / start
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
  return v;
}

constexpr int kPlanThreads = 1024;

// Single-CTA stable counting sort of the slot expert ids, then groups of at
// most kMaxGroupRows rows.  Ids outside [0, experts) are counted in
// header[8] and left out of every group.
__global__ void __launch_bounds__(kPlanThreads) plan_kernel(const uint32_t* __restrict__ ids, int rows,
                                                            int experts, int period, int skip_slot, PlanView plan) {
  extern __shared__ int sm[];
  int* hist = sm;                        // [experts]
  int* base = hist + experts;            // [experts]
  int* gbase = base + experts;           // [experts]
  int* wcount = gbase + experts;         // [32][experts]
  __shared__ int s_total_groups;
  __shared__ int s_bad;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  for (int e = tid; e < experts; e += blockDim.x) hist[e] = 0;
  if (tid == 0) s_bad = 0;
  __syncthreads();
  for (int i = tid; i < rows; i += blockDim.x) {
    if (skip_slot >= 0 && i % period == skip_slot) continue;
    uint32_t e = ids[i];
    if (e < static_cast<uint32_t>(experts)) atomicAdd(&hist[e], 1);
    else atomicAdd(&s_bad, 1);
  }
  __syncthreads();
  // Exclusive scans of row counts and group counts (one warp).
  if (warp == 0) {
    const int per = (experts + 31) / 32;
    const int first = lane * per;
    int rsum = 0, gsum = 0;
    for (int e = first; e < min(first + per, experts); ++e) {
      rsum += hist[e];
      gsum += (hist[e] + kMaxGroupRows - 1) / kMaxGroupRows;
    }
    int rinc = rsum, ginc = gsum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      int r = __shfl_up_sync(0xffffffffu, rinc, off);
      int g = __shfl_up_sync(0xffffffffu, ginc, off);
      if (lane >= off) {
        rinc += r;
        ginc += g;
      }
    }
    int rrun = rinc - rsum, grun = ginc - gsum;
    for (int e = first; e < min(first + per, experts); ++e) {
      base[e] = rrun;
      gbase[e] = grun;
      plan.expert_start[e] = rrun;
      plan.expert_count[e] = hist[e];
      rrun += hist[e];
      grun += (hist[e] + kMaxGroupRows - 1) / kMaxGroupRows;
    }
    if (lane == 31) s_total_groups = ginc;
  }
  __syncthreads();
  // Groups.
  for (int e = tid; e < experts; e += blockDim.x) {
    const int n = hist[e];
    for (int c = 0; c * kMaxGroupRows < n; ++c) {
      const int g = gbase[e] + c;
      plan.group_expert[g] = e;
      plan.group_start[g] = base[e] + c * kMaxGroupRows;
      plan.group_count[g] = min(kMaxGroupRows, n - c * kMaxGroupRows);
    }
  }
  __syncthreads();
  // Stable scatter, one chunk of blockDim slots at a time.
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int chunk = 0; chunk < rows; chunk += blockDim.x) {
    for (int j = tid; j < 32 * experts; j += blockDim.x) wcount[j] = 0;
    __syncthreads();
    const int i = chunk + tid;
    const bool skipped = i < rows && skip_slot >= 0 && i % period == skip_slot;
    const uint32_t raw = (i < rows && !skipped) ? ids[i] : 0xFFFFFFFFu;
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
      plan.order[base[key] + prior + rank] = i;
    }
    __syncthreads();
    if (valid && lane == leader) atomicAdd(&base[key], __popc(peers));
    __syncthreads();
  }
  if (tid == 0) {
    plan.header[0] = s_total_groups;
    plan.header[1] = rows;
    for (int c = 2; c < 8; ++c) plan.header[c] = 0;
    plan.header[8] = s_bad;
  }
}

cudaError_t launch_plan(const uint32_t* ids, int rows, int experts, int period, int skip_slot, PlanView plan,
                        cudaStream_t s) {
  const size_t smem = (3 + 32) * static_cast<size_t>(experts) * sizeof(int);
  if (smem > 48 * 1024) {
    cudaError_t err = cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
    if (err != cudaSuccess) return err;
  }
  plan_kernel<<<1, kPlanThreads, smem, s>>>(ids, rows, experts, period > 0 ? period : 1, skip_slot, plan);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Prep: xh[p][slot] = H(x[row] * in_scale_p[expert])  (float32)
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(128) prep_kernel(const void* __restrict__ x, int x_dtype, int per_slot,
                                                   int slots_per_token, const uint32_t* __restrict__ ids, int nslots,
                                                   const void* __restrict__ in0, const void* __restrict__ in1,
                                                   int scale_dtype, int features, int experts,
                                                   float* __restrict__ xh) {
  const int lane = threadIdx.x & 31;
  const int block = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int slot = blockIdx.y;
  const int proj = blockIdx.z;
  if (block * 128 >= features) return;
  const uint32_t e = ids[slot];
  float* out = xh + (static_cast<int64_t>(proj) * nslots + slot) * features;
  if (e >= static_cast<uint32_t>(experts)) {  // unplanned row: zeros, never reads a scale
#pragma unroll
    for (int j = 0; j < 4; ++j) out[block * 128 + lane + 32 * j] = 0.0f;
    return;
  }
  const int64_t row = per_slot ? slot : slot / slots_per_token;
  const void* scale = proj ? in1 : in0;
  float v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int col = block * 128 + lane + 32 * j;
    v[j] = __fmul_rn(load_act(x, x_dtype, row * features + col),
                     load_scale(scale, scale_dtype, static_cast<int64_t>(e) * features + col));
  }
  hadamard128(v, lane);
#pragma unroll
  for (int j = 0; j < 4; ++j) out[block * 128 + lane + 32 * j] = v[j];
}

cudaError_t launch_prep(const void* x, int x_dtype, int per_slot, int slots_per_token, const uint32_t* ids,
                        int nslots, const void* in0, const void* in1, int scale_dtype, int features,
                        int experts, int projections, float* xh, cudaStream_t s) {
  dim3 grid((features / 128 + 3) / 4, nslots, projections);
  prep_kernel<<<grid, 128, 0, s>>>(x, x_dtype, per_slot, slots_per_token, ids, nslots, in0, in1, scale_dtype,
                                   features, experts, xh);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Decode GEMV
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t ld_stream(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.b32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ void mma_f16(float c[4], const uint32_t a[4], uint2 b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// hi or lo piece of a float as float16: hi = f16(v), lo = f16(v - hi).
__device__ __forceinline__ float split_piece(float v, int piece) {
  const float hi = __half2float(__float2half_rn(v));
  return piece ? v - hi : hi;
}

template <int K>
__global__ void __launch_bounds__(kGemvWarps * 32) trellis_gemv_kernel(GemvParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int s_unit;
  __shared__ int s_rows[kMaxGroupRows];
  __shared__ unsigned s_maxbits[kMaxGroupRows];
  __shared__ float s_scale[kMaxGroupRows];
  __shared__ float s_unscale[kMaxGroupRows];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int it = p.in_features / 16, ot = p.out_features / 16, nblocks = ot / 8;
  const int kt_per_split = (it + p.splits - 1) / p.splits;
  const int words_per_tile = 8 * K;
  const int groups = p.plan.header[0];
  const int64_t total = static_cast<int64_t>(groups) * p.projections * nblocks * p.splits;
  GenericGeometry geo;
  if (K != 4) geo = generic_geometry(K, lane);

  for (;;) {
    if (tid == 0) s_unit = atomicAdd(&p.plan.header[p.counter], 1);
    __syncthreads();
    const int64_t unit = s_unit;
    if (unit >= total) break;
    const int split = static_cast<int>(unit % p.splits);
    const int nb = static_cast<int>((unit / p.splits) % nblocks);
    const int proj = static_cast<int>((unit / (static_cast<int64_t>(p.splits) * nblocks)) % p.projections);
    const int g = static_cast<int>(unit / (static_cast<int64_t>(p.splits) * nblocks * p.projections));
    const int expert = p.plan.group_expert[g];
    const int start = p.plan.group_start[g];
    const int nr = p.plan.group_count[g];
    const int ncg = (nr + 3) / 4;
    const int kt0 = split * kt_per_split;
    const int kt1 = min(kt0 + kt_per_split, it);
    const int KT = kt1 - kt0;
    if (tid < nr) {
      s_rows[tid] = p.plan.order[start + tid];
      s_maxbits[tid] = 0u;
    }
    __syncthreads();
    const float* xbase = p.xh + static_cast<int64_t>(proj) * p.nslots * p.in_features;
    // Per-row power-of-two scale so that hi/lo float16 pieces cover the row.
    for (int idx = tid; idx < nr * KT * 16; idx += blockDim.x) {
      const int r = idx / (KT * 16), kk = idx % (KT * 16);
      const float v = xbase[static_cast<int64_t>(s_rows[r]) * p.in_features + kt0 * 16 + kk];
      atomicMax(&s_maxbits[r], __float_as_uint(fabsf(v)) & 0x7fffffffu);
    }
    __syncthreads();
    if (tid < nr) {
      const float m = __uint_as_float(s_maxbits[tid]);
      int ex = 0;
      if (m > 0.0f && m < 3.0e38f) {
        frexpf(m, &ex);
        ex -= 15;
      }
      s_scale[tid] = ldexpf(1.0f, -ex);
      s_unscale[tid] = ldexpf(1.0f, ex);
    }
    __syncthreads();
    // B fragments [KT][ncg][32] of (hi, lo) float16 pairs.
    uint2* bfrag = reinterpret_cast<uint2*>(smem);
    for (int idx = tid; idx < KT * ncg * 32; idx += blockDim.x) {
      const int l = idx & 31, cg = (idx >> 5) % ncg, ktl = idx / (32 * ncg);
      const int n = l >> 2, tig = l & 3;
      const int r = cg * 4 + (n >> 1), piece = n & 1;
      uint2 b = make_uint2(0u, 0u);
      if (r < nr) {
        const float* src = xbase + static_cast<int64_t>(s_rows[r]) * p.in_features + (kt0 + ktl) * 16;
        const float sc = s_scale[r];
        const float f0 = split_piece(src[2 * tig] * sc, piece);
        const float f1 = split_piece(src[2 * tig + 1] * sc, piece);
        const float f2 = split_piece(src[2 * tig + 8] * sc, piece);
        const float f3 = split_piece(src[2 * tig + 9] * sc, piece);
        b.x = pack_half2(f0, f1);
        b.y = pack_half2(f2, f3);
      }
      bfrag[idx] = b;
    }
    __syncthreads();

    float acc[8][2][4];
#pragma unroll
    for (int t = 0; t < 8; ++t)
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[t][c][i] = 0.0f;

    const uint32_t* packed = proj ? p.packed1 : p.packed0;
    if (K == 4) {
      uint32_t wcur[8], wnext[8];
      int ktl = warp;
      if (ktl < KT) {
        const uint32_t* words = packed + tile_index(expert, kt0 + ktl, nb * 8, it, ot, p.side) * 32;
#pragma unroll
        for (int t = 0; t < 8; ++t) wcur[t] = ld_stream(words + t * 32 + lane);
      }
      for (; ktl < KT; ktl += kGemvWarps) {
        const int nxt = ktl + kGemvWarps;
        if (nxt < KT) {
          const uint32_t* words = packed + tile_index(expert, kt0 + nxt, nb * 8, it, ot, p.side) * 32;
#pragma unroll
          for (int t = 0; t < 8; ++t) wnext[t] = ld_stream(words + t * 32 + lane);
        }
        uint2 b0 = bfrag[(ktl * ncg) * 32 + lane];
        uint2 b1 = ncg > 1 ? bfrag[(ktl * ncg + 1) * 32 + lane] : make_uint2(0u, 0u);
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const uint32_t prior = __shfl_sync(0xffffffffu, wcur[t], (lane + 31) & 31);
          uint32_t cw[8], a[4];
          k4_codewords(wcur[t], prior, cw);
          tile_fragment(cw, a);
          mma_f16(acc[t][0], a, b0);
          if (ncg > 1) mma_f16(acc[t][1], a, b1);
        }
#pragma unroll
        for (int t = 0; t < 8; ++t) wcur[t] = wnext[t];
      }
    } else {
      for (int ktl = warp; ktl < KT; ktl += kGemvWarps) {
        const uint32_t* words =
            packed + tile_index(expert, kt0 + ktl, nb * 8, it, ot, p.side) * words_per_tile;
        uint2 b0 = bfrag[(ktl * ncg) * 32 + lane];
        uint2 b1 = ncg > 1 ? bfrag[(ktl * ncg + 1) * 32 + lane] : make_uint2(0u, 0u);
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          uint32_t cw[8], a[4];
          generic_codewords(words + t * words_per_tile, K, geo, cw);
          tile_fragment(cw, a);
          mma_f16(acc[t][0], a, b0);
          if (ncg > 1) mma_f16(acc[t][1], a, b1);
        }
      }
    }
    __syncthreads();  // B fragments are dead; reuse shared memory for the warp reduction
    float4* red = reinterpret_cast<float4*>(smem);  // [warp][t][cg][lane]
#pragma unroll
    for (int t = 0; t < 8; ++t)
#pragma unroll
      for (int c = 0; c < 2; ++c)
        red[((warp * 8 + t) * 2 + c) * 32 + lane] = make_float4(acc[t][c][0], acc[t][c][1], acc[t][c][2], acc[t][c][3]);
    __syncthreads();
    for (int idx = tid; idx < 8 * ncg * 32; idx += blockDim.x) {
      const int l = idx & 31, c = (idx >> 5) % ncg, t = idx / (32 * ncg);
      float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < kGemvWarps; ++w) {
        const float4 v = red[((w * 8 + t) * 2 + c) * 32 + l];
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
      const int gid = l >> 2, tig = l & 3;
      const int r = c * 4 + tig;
      if (r < nr) {
        float* dst = p.partial +
                     ((static_cast<int64_t>(proj) * p.nslots + s_rows[r]) * p.splits + split) * p.out_features +
                     nb * 128 + t * 16 + gid;
        dst[0] = (s.x + s.y) * s_unscale[r];
        dst[8] = (s.z + s.w) * s_unscale[r];
      }
    }
    __syncthreads();
  }
}

static size_t gemv_smem(int in_features, int splits) {
  const int it = in_features / 16;
  const int kt = (it + splits - 1) / splits;
  const size_t frag = static_cast<size_t>(kt) * 2 * 32 * sizeof(uint2);
  const size_t red = static_cast<size_t>(kGemvWarps) * 8 * 2 * 32 * sizeof(float4);
  return frag > red ? frag : red;
}

template <int K>
static cudaError_t launch_gemv_k(const GemvParams& p, cudaStream_t s) {
  const size_t smem = gemv_smem(p.in_features, p.splits);
  cudaError_t err = cudaFuncSetAttribute(trellis_gemv_kernel<K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  int device = 0, sms = 0, per_sm = 0;
  cudaGetDevice(&device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, trellis_gemv_kernel<K>, kGemvWarps * 32, smem);
  if (per_sm < 1) per_sm = 1;
  trellis_gemv_kernel<K><<<sms * per_sm, kGemvWarps * 32, smem, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_gemv(const GemvParams& p, cudaStream_t s) {
  switch (p.k) {
    case 2: return launch_gemv_k<2>(p, s);
    case 3: return launch_gemv_k<3>(p, s);
    default: return launch_gemv_k<4>(p, s);
  }
}

// ---------------------------------------------------------------------------
// Finishes
// ---------------------------------------------------------------------------

// gate/up split sum, Hadamard, output scales, typed SwiGLU, down input scale,
// Hadamard -> down_xh (float32).  One warp per (slot, 128-block).
__global__ void __launch_bounds__(128) gate_finish_kernel(const float* __restrict__ partial, int splits,
                                                          const uint32_t* __restrict__ ids, int nslots,
                                                          const void* __restrict__ out_gate,
                                                          const void* __restrict__ out_up,
                                                          const void* __restrict__ in_down, int scale_dtype,
                                                          int features, int experts, int act_dtype,
                                                          float* __restrict__ down_xh) {
  const int lane = threadIdx.x & 31;
  const int block = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int slot = blockIdx.y;
  if (block * 128 >= features) return;
  const int64_t e = ids[slot];
  if (e >= experts) {
#pragma unroll
    for (int j = 0; j < 4; ++j) down_xh[static_cast<int64_t>(slot) * features + block * 128 + lane + 32 * j] = 0.0f;
    return;
  }
  float gate[4], up[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int col = block * 128 + lane + 32 * j;
    float g = 0.f, u = 0.f;
    for (int s = 0; s < splits; ++s) {
      g += partial[(static_cast<int64_t>(slot) * splits + s) * features + col];
      u += partial[((static_cast<int64_t>(nslots) + slot) * splits + s) * features + col];
    }
    gate[j] = g;
    up[j] = u;
  }
  hadamard128(gate, lane);
  hadamard128(up, lane);
  float act[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t si = e * features + block * 128 + lane + 32 * j;
    const float g = __fmul_rn(gate[j], load_scale(out_gate, scale_dtype, si));
    const float u = __fmul_rn(up[j], load_scale(out_up, scale_dtype, si));
    act[j] = __fmul_rn(swiglu_typed(act_dtype, g, u), load_scale(in_down, scale_dtype, si));
  }
  hadamard128(act, lane);
#pragma unroll
  for (int j = 0; j < 4; ++j) down_xh[static_cast<int64_t>(slot) * features + block * 128 + lane + 32 * j] = act[j];
}

cudaError_t launch_gate_finish(const float* partial, int splits, const uint32_t* ids, int nslots,
                               const void* out_gate, const void* out_up, const void* in_down, int scale_dtype,
                               int features, int experts, int act_dtype, float* down_xh, cudaStream_t s) {
  dim3 grid((features / 128 + 3) / 4, nslots);
  gate_finish_kernel<<<grid, 128, 0, s>>>(partial, splits, ids, nslots, out_gate, out_up, in_down, scale_dtype,
                                          features, experts, act_dtype, down_xh);
  return cudaGetLastError();
}

// Split sum, Hadamard, signed output scale, cast to the activation type.
__global__ void __launch_bounds__(128) finish_kernel(const float* __restrict__ partial, int splits,
                                                     const uint32_t* __restrict__ ids, int nslots,
                                                     const void* __restrict__ out_scale, int scale_dtype,
                                                     int features, int experts, int act_dtype,
                                                     void* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int block = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int slot = blockIdx.y;
  if (block * 128 >= features) return;
  const int64_t e = ids[slot];
  if (e >= experts) {
#pragma unroll
    for (int j = 0; j < 4; ++j) store_act(out, act_dtype, static_cast<int64_t>(slot) * features + block * 128 + lane + 32 * j, 0.0f);
    return;
  }
  float v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int col = block * 128 + lane + 32 * j;
    float a = 0.f;
    for (int s = 0; s < splits; ++s) a += partial[(static_cast<int64_t>(slot) * splits + s) * features + col];
    v[j] = a;
  }
  hadamard128(v, lane);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int col = block * 128 + lane + 32 * j;
    store_act(out, act_dtype, static_cast<int64_t>(slot) * features + col,
              __fmul_rn(v[j], load_scale(out_scale, scale_dtype, e * features + col)));
  }
}

cudaError_t launch_finish(const float* partial, int splits, const uint32_t* ids, int nslots, const void* out_scale,
                          int scale_dtype, int features, int experts, int act_dtype, void* out, cudaStream_t s) {
  dim3 grid((features / 128 + 3) / 4, nslots);
  finish_kernel<<<grid, 128, 0, s>>>(partial, splits, ids, nslots, out_scale, scale_dtype, features, experts,
                                     act_dtype, out);
  return cudaGetLastError();
}

// Nine slots per token (eight routed + shared): expert finish, routed
// weighted sum in the order slot 0, then (slot r + 0) + total for r = 1..7,
// T(routed), T(routed + T(shared)), T(residual + combined).  When
// shared_values is given it holds the typed shared-expert output [tokens][h]
// and slot 8 of partial is not read.
__global__ void __launch_bounds__(128) finish_fused_kernel(const float* __restrict__ partial, int splits,
                                                           const uint32_t* __restrict__ ids, int tokens,
                                                           const void* __restrict__ out_scale, int scale_dtype,
                                                           int features, int experts,
                                                           const float* __restrict__ scores,
                                                           const void* __restrict__ residual,
                                                           const void* __restrict__ shared_values, int act_dtype,
                                                           void* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int block = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int token = blockIdx.y;
  if (block * 128 >= features) return;
  float total[4], shared[4];
  for (int slot = 0; slot < 9; ++slot) {
    const int row = token * 9 + slot;
    if (slot == 8 && shared_values != nullptr) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        shared[j] = load_act(shared_values, act_dtype,
                             static_cast<int64_t>(token) * features + block * 128 + lane + 32 * j);
      break;
    }
    const int64_t e = ids[row];
    const bool ok = e < experts;  // an out-of-range id contributes zero
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = block * 128 + lane + 32 * j;
      float a = 0.f;
      if (ok)
        for (int s = 0; s < splits; ++s) a += partial[(static_cast<int64_t>(row) * splits + s) * features + col];
      v[j] = a;
    }
    hadamard128(v, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = block * 128 + lane + 32 * j;
      const float value =
          ok ? round_to(act_dtype, __fmul_rn(v[j], load_scale(out_scale, scale_dtype, e * features + col))) : 0.0f;
      if (slot < 8) {
        const float prod = __fmul_rn(value, scores[token * 8 + slot]);
        total[j] = slot == 0 ? __fadd_rn(prod, 0.0f) : __fadd_rn(__fadd_rn(prod, 0.0f), total[j]);
      } else {
        shared[j] = value;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t off = static_cast<int64_t>(token) * features + block * 128 + lane + 32 * j;
    const float routed = round_to(act_dtype, total[j]);
    const float combined = round_to(act_dtype, __fadd_rn(routed, round_to(act_dtype, shared[j])));
    store_act(out, act_dtype, off, __fadd_rn(load_act(residual, act_dtype, off), combined));
  }
}

cudaError_t launch_finish_fused(const float* partial, int splits, const uint32_t* ids, int tokens,
                                const void* out_scale, int scale_dtype, int features, int experts,
                                const float* scores, const void* residual, const void* shared_values, int act_dtype,
                                void* out, cudaStream_t s) {
  dim3 grid((features / 128 + 3) / 4, tokens);
  finish_fused_kernel<<<grid, 128, 0, s>>>(partial, splits, ids, tokens, out_scale, scale_dtype, features, experts,
                                           scores, residual, shared_values, act_dtype, out);
  return cudaGetLastError();
}

}  // namespace exlr8
