// extern "C" entry points of include/exlr8_b200.h: argument validation with
// the reference's error semantics, workspace layout and kernel sequencing.

#include <algorithm>
#include <cstdio>
#include <cstring>

#include "capi_util.cuh"
#include "codec.cuh"
#include "common.cuh"
#include "dense.cuh"
#include "dense_stream.cuh"
#include "dispatch.cuh"
#include "ep.cuh"
#include "joined.cuh"
#include "mx_gemm.cuh"
#include "norm.cuh"
#include "router.cuh"
#include "router_gemm.cuh"
#include "stream.cuh"
#include "trellis_gemv.cuh"

using namespace exlr8;

namespace exlr8 {
thread_local char g_cuda_error[256] = "";
thread_local Profiler g_prof;
}  // namespace exlr8

namespace {

constexpr int64_t kStreamCtasHint = 296;  // persistent stream CTAs on a B200 (2 per SM)

// K splits.  Gate/up follow fast_decode.py:216 (min(8, max(1, hidden // 768)));
// the down product splits once per 1024 inputs.  Splits are rounded to whole
// 128-wide blocks (stream.cuh kt_per_split).
struct Splits {
  int kt, count;
};
inline Splits make_splits(int in_features, int nominal, int cap = 8) {
  if (nominal < 1) nominal = 1;
  if (nominal > cap) nominal = cap;
  Splits s;
  s.kt = kt_per_split(in_features, nominal);
  s.count = split_count(in_features, s.kt);
  return s;
}
// Gate/up: at least the reference's count, and for small batches enough
// splits for >= 12 units per stream CTA (units are (row group, projection,
// 128-wide output block, split); the row count bounds the groups).
inline Splits gate_up_splits(int hidden, int intermediate, int64_t rows) {
  int nominal = hidden / 768;
  const int64_t per_split = (rows > 0 ? rows : 1) * 2 * (intermediate / 128);
  const int64_t want = (12 * kStreamCtasHint + per_split - 1) / per_split;
  if (want > nominal) nominal = static_cast<int>(want < 16 ? want : 16);
  return make_splits(hidden, nominal, 16);
}
// The down product splits once per 1024 inputs, and more for small batches:
// its units are (row group, 128-wide output block, split), and with few row
// groups whole-unit granularity would leave the last wave of the persistent
// stream CTAs (2 per SM, 296 on a B200) unbalanced.  Aim for >= 8 units per CTA.
inline Splits down_splits(int intermediate, int hidden, int64_t rows) {
  int nominal = intermediate / 1024;
  const int64_t per_split = (rows > 0 ? rows : 1) * (hidden / 128);
  const int64_t want = (8 * kStreamCtasHint + per_split - 1) / per_split;
  if (want > nominal) nominal = static_cast<int>(want < 8 ? want : 8);
  return make_splits(intermediate, nominal);
}
inline Splits linear_splits(int in_features) { return make_splits(in_features, in_features / 768); }
// K splits of the bf16 shared expert streamed beside the trellis units
// (units of 16 rows x one split; the partials are summed in split order).
inline int dense_gate_up_splits(int hidden) { return dense_split_count(hidden, 4); }
inline int dense_down_splits(int intermediate) { return dense_split_count(intermediate, 2); }

int format_status(int64_t packed_bytes, int k, int in_f, int out_f, int side, int64_t* matrices) {
  if (k != 2 && k != 3 && k != 4) return EXLR8_ERR_WIDTH;
  if (in_f <= 0 || out_f <= 0 || in_f % 128 || out_f % 128) return EXLR8_ERR_DIMS;
  if (side < 0 || side > 2) return EXLR8_ERR_SIDE;
  const int64_t size = static_cast<int64_t>(in_f) * out_f * k / 8;
  if (packed_bytes <= 0 || packed_bytes % size) return EXLR8_ERR_BYTES;
  if (matrices) *matrices = packed_bytes / size;
  return EXLR8_OK;
}

// Workspace of the trellis MLP over `rows` slots.
struct MlpLayout {
  Splits s1, s2;
  size_t plan, frag_gu, gu, frag_d, dpart;
  size_t total() const { return plan + frag_gu + gu + frag_d + dpart; }
};

// bf16 shared expert: K splits of the gate/up and down passes (enough warps
// in flight to stream the weights at full bandwidth for a few tokens).
constexpr int kDenseGateUpSplits = 32;
constexpr int kDenseDownSplits = 8;

MlpLayout mlp_layout(int64_t rows, int hidden, int inter, int64_t experts) {
  MlpLayout l;
  l.s1 = gate_up_splits(hidden, inter, rows);
  l.s2 = down_splits(inter, hidden, rows);
  l.plan = align_up(plan_bytes(static_cast<int>(rows), static_cast<int>(experts)));
  l.frag_gu = align_up(frag_bytes(rows, hidden, 2));
  l.gu = align_up(2 * rows * l.s1.count * static_cast<size_t>(inter) * sizeof(float));
  l.frag_d = align_up(frag_bytes(rows, inter, 1));
  l.dpart = align_up(rows * l.s2.count * static_cast<size_t>(hidden) * sizeof(float));
  return l;
}

struct DenseLayout {
  size_t gate, up, h, down, counters;
  size_t total() const { return gate + up + h + down + counters; }
};

DenseLayout dense_layout(int64_t tokens, int hidden, int inter) {
  DenseLayout l;
  l.gate = align_up(kDenseGateUpSplits * tokens * static_cast<size_t>(inter) * sizeof(float));
  l.up = l.gate;
  l.h = align_up(tokens * static_cast<size_t>(inter) * sizeof(float));
  l.down = align_up(kDenseDownSplits * tokens * static_cast<size_t>(hidden) * sizeof(float));
  l.counters = align_up((static_cast<size_t>(inter) / 64 + 1) * sizeof(int32_t));
  return l;
}

int check_experts(const exlr8_trellis_experts* ex, int64_t* matrices) {
  if (!ex) return EXLR8_ERR_ARG;
  if (!valid_scale(ex->scale_dtype)) return EXLR8_ERR_DTYPE;
  int64_t count = -1;
  for (int p = 0; p < 3; ++p) {
    const bool down = p == 2;
    const int a = down ? ex->intermediate : ex->hidden, b = down ? ex->hidden : ex->intermediate;
    int64_t m = 0;
    EXLR8_CHECK(format_status(ex->packed_bytes[p], ex->k, a, b, down ? 2 : 1, &m));
    if (!ex->packed[p] || !ex->in_scale[p] || !ex->out_scale[p]) return EXLR8_ERR_ARG;
    if (!aligned16(ex->packed[p])) return EXLR8_ERR_ALIGN;
    if (count >= 0 && m != count) return EXLR8_ERR_BYTES;
    count = m;
  }
  if (ex->scale_experts != count) return EXLR8_ERR_SCALES;
  *matrices = count;
  return EXLR8_OK;
}

}  // namespace

int exlr8::moe_layer_preflight(const exlr8_trellis_experts* ex, int64_t tokens, int64_t* experts) {
  EXLR8_CHECK(check_experts(ex, experts));
  if (tokens < 0) return EXLR8_ERR_ROWS;
  if (tokens > (1 << 20) || tokens * 9 > (1 << 20)) return EXLR8_ERR_UNSUPPORTED;
  return EXLR8_OK;
}

namespace {

StreamParams stream_params(const exlr8_trellis_experts* ex, PlanView plan, int counter, int rows) {
  StreamParams sp{};
  sp.plan = plan;
  sp.counter = counter;
  sp.k = ex ? ex->k : 4;
  sp.nslots = rows;
  sp.mcg_mask = 0x8FFF8FFFu;
  sp.mcg_xor = 0x3B603B60u;
  return sp;
}

// Buffers of one MLP call carved from the workspace.
struct MlpBuffers {
  PlanView plan;
  unsigned char* frag_gu;
  float* gu;
  unsigned char* frag_d;
  float* dpart;
  // dense shared expert (null when absent)
  float* dgate;
  float* dup;
  void* dh;
  float* ddown;
};

MlpBuffers carve_mlp(const MlpLayout& l, int64_t rows, int64_t experts, bool dense, int64_t tokens, int hidden,
                     int inter, Carver& c) {
  MlpBuffers b{};
  const int n = static_cast<int>(rows), e = static_cast<int>(experts);
  b.plan = plan_view(c.take<int32_t>(l.plan), n, e);
  b.frag_gu = c.take<unsigned char>(l.frag_gu);
  b.gu = c.take<float>(l.gu);
  b.frag_d = c.take<unsigned char>(l.frag_d);
  b.dpart = c.take<float>(l.dpart);
  if (dense) {
    const DenseLayout dl = dense_layout(tokens, hidden, inter);
    b.dgate = c.take<float>(dl.gate);
    b.dup = c.take<float>(dl.up);
    b.dh = c.take<void>(dl.h);
    b.ddown = c.take<float>(dl.down);
  }
  return b;
}

// The bf16 shared expert of a few tokens on its own (exlr8_shared_expert):
// gate/up with the SwiGLU into h, then the down partials
// [kDenseDownSplits][tokens][hidden].
int launch_dense_decode(const void* x, int x_dtype, int64_t tokens, const exlr8_dense_expert* shared, int h, int m,
                        float* dgate, float* dup, void* dh, float* ddown, int32_t* counters, cudaStream_t s) {
  const int t = static_cast<int>(tokens);
  EXLR8_TRY(cudaMemsetAsync(counters, 0, (m / 64 + 1) * sizeof(int32_t), s));
  EXLR8_TIMED(EXLR8_KERNEL_DENSE, s,
              launch_dense_gate_up(static_cast<const uint16_t*>(x), t, static_cast<const uint16_t*>(shared->gate),
                                   static_cast<const uint16_t*>(shared->up), m, h, kDenseGateUpSplits, dgate, dup,
                                   counters, x_dtype, dh, 0, s));
  EXLR8_TIMED(EXLR8_KERNEL_DENSE, s,
              launch_dense_gemv(static_cast<const uint16_t*>(dh), t, static_cast<const uint16_t*>(shared->down), h, m,
                                kDenseDownSplits, ddown, 0, s));
  return EXLR8_OK;
}

// The trellis MLP over all slots of `ids` ([rows] = tokens*slots) after the
// plan: activation fragments, the gate/up stream, the gate/up finish into the
// down fragments, the down stream.  Leaves fp32 down partials.  With
// `shared` the bf16 shared expert of the `tokens` rows of dense_x runs as
// dense units of the two stream launches (its SwiGLU in the gate/up finish)
// and leaves its down partials [dense_down_splits][tokens][hidden] in
// b.ddown.
int run_mlp_after_plan(const void* x, int x_dtype, int per_slot, int slots, const uint32_t* ids, int64_t rows,
                       const exlr8_trellis_experts* ex, int64_t experts, const exlr8_dense_expert* shared,
                       const void* dense_x, int64_t tokens, const MlpLayout& l, const MlpBuffers& b,
                       cudaStream_t s, const exlr8_static_cache* cache = nullptr, int sparse = 0) {
  const int h = ex->hidden, m = ex->intermediate;
  const int n = static_cast<int>(rows), e = static_cast<int>(experts), t = static_cast<int>(tokens);
  EXLR8_TIMED(EXLR8_KERNEL_PREP, s,
              launch_prep_frag(x, x_dtype, per_slot, slots, ids, n, ex->in_scale[0], ex->in_scale[1],
                               ex->scale_dtype, h, e, 2, b.frag_gu, s, -1, 0, sparse));
  StreamParams gp = stream_params(ex, b.plan, 2, n);
  gp.packed[0] = static_cast<const uint32_t*>(ex->packed[0]);
  gp.packed[1] = static_cast<const uint32_t*>(ex->packed[1]);
  gp.frag = b.frag_gu;
  gp.partial = b.gu;
  gp.side = 1;
  gp.in_features = h;
  gp.out_features = m;
  gp.kt_per_split = l.s1.kt;
  gp.splits = l.s1.count;
  gp.projections = 2;
  if (cache) {
    gp.hot[0] = cache->fp8[0];
    gp.hot[1] = cache->fp8[1];
    gp.expert_to_slot = cache->expert_to_slot;
    gp.hot_slots = cache->slots;
  }
  const int dsplits_gu = dense_gate_up_splits(h), dsplits_d = dense_down_splits(m);
  if (shared)
    gp.dense = DenseUnits{static_cast<const uint16_t*>(shared->gate), static_cast<const uint16_t*>(shared->up),
                          static_cast<const uint16_t*>(dense_x), b.dgate, b.dup, m, h, t, dsplits_gu,
                          (m / kDenseRows) * dsplits_gu, 1};
  if (!encode_dense_maps(gp)) return EXLR8_ERR_CUDA;
  EXLR8_TIMED(EXLR8_KERNEL_GATE_UP, s, launch_stream(gp, s));
  EXLR8_TIMED(EXLR8_KERNEL_GATE_FINISH, s,
              launch_gate_finish_frag(b.gu, l.s1.count, ids, n, ex->out_scale[0], ex->out_scale[1], ex->in_scale[2],
                                      ex->scale_dtype, m, e, x_dtype, b.frag_d, b.dgate, b.dup, dsplits_gu,
                                      shared ? t : 0, shared ? b.dh : nullptr, s, 0, sparse));
  StreamParams dp = stream_params(ex, b.plan, 3, n);
  dp.packed[0] = static_cast<const uint32_t*>(ex->packed[2]);
  dp.packed[1] = nullptr;
  dp.frag = b.frag_d;
  dp.partial = b.dpart;
  dp.side = 2;
  dp.in_features = m;
  dp.out_features = h;
  dp.kt_per_split = l.s2.kt;
  dp.splits = l.s2.count;
  dp.projections = 1;
  if (cache) {
    dp.hot[0] = cache->fp8[2];
    dp.expert_to_slot = cache->expert_to_slot;
    dp.hot_slots = cache->slots;
  }
  if (shared)
    dp.dense = DenseUnits{static_cast<const uint16_t*>(shared->down), nullptr, static_cast<const uint16_t*>(b.dh),
                          b.ddown, nullptr, h, m, t, dsplits_d, (h / kDenseRows) * dsplits_d, 0};
  if (!encode_dense_maps(dp)) return EXLR8_ERR_CUDA;
  EXLR8_TIMED(EXLR8_KERNEL_DOWN, s, launch_stream(dp, s));
  return EXLR8_OK;
}

int check_dense(const exlr8_dense_expert* sh, int x_dtype, int hidden, int inter) {
  if (!sh) return EXLR8_OK;
  if (!sh->gate || !sh->up || !sh->down) return EXLR8_ERR_ARG;
  if (x_dtype != EXLR8_DTYPE_BF16) return EXLR8_ERR_DTYPE;  // bf16 operands for the bf16 matrices
  if (!aligned16(sh->gate) || !aligned16(sh->up) || !aligned16(sh->down)) return EXLR8_ERR_ALIGN;
  if (hidden % 128 || inter % 128) return EXLR8_ERR_DIMS;
  return EXLR8_OK;
}

// ---- prefill: grouped trellis GEMM on the tensor cores --------------------
//
// The reference runs fast_expert_mlp up to 16 token rows and
// fast_prefill.grouped_expert_mlp above (experts.py:171-174).  Above the same
// threshold the trellis MLP runs as grouped tcgen05 GEMMs: slots sorted by
// expert in 128-row-aligned segments; per slot H(x * in_scale[e]) for gate
// and up as E4M3 hi/lo planes; one gate+up GEMM (two projections) whose
// decoder warps expand the trellis codes to E4M3 tiles; the gate/up finish;
// the down GEMM; the per-slot finish or the fused combine.
constexpr int64_t kPrefillMinTokens = 17;

struct PrefillBuffers {
  PlanView plan;
  int32_t* counters;
  MxChunks chunks;
  uint8_t *ghi, *glo, *gsc, *uhi, *ulo, *usc;
  float* gu;
  uint8_t *dhi, *dlo, *dsc;
  float* v;
  // dense bf16 shared expert on the tensor cores (split partials)
  float *dgate, *dup, *ddown;
  void* dh;
  int32_t* derr;
  int dsplits_gu, dsplits_d;
};

PrefillBuffers carve_prefill(int64_t tokens, int slots, int h, int m, int64_t experts, bool dense, Carver& c) {
  PrefillBuffers b{};
  const int64_t rows = tokens * slots;
  const int64_t padded = mx_padded_rows(rows, experts);
  const int64_t max_chunks = mx_max_chunks(rows, experts);
  b.plan = plan_view(c.take<char>(plan_bytes(static_cast<int>(rows), static_cast<int>(experts))),
                     static_cast<int>(rows), static_cast<int>(experts));
  b.counters = c.take<int32_t>((m / 64 + 1) * sizeof(int32_t));
  b.plan.zero = b.counters;
  b.plan.zero_count = m / 64;
  b.chunks.header = c.take<int32_t>(16 * sizeof(int32_t));
  b.chunks.chunk_start = c.take<int32_t>(max_chunks * sizeof(int32_t));
  b.chunks.chunk_rows = c.take<int32_t>(max_chunks * sizeof(int32_t));
  b.chunks.chunk_expert = c.take<int32_t>(max_chunks * sizeof(int32_t));
  b.chunks.padded_start = c.take<int32_t>((experts + 1) * sizeof(int32_t));
  b.chunks.row_slot = c.take<int32_t>(padded * sizeof(int32_t));
  b.chunks.slot_row = c.take<int32_t>(rows * sizeof(int32_t));
  b.ghi = c.take<uint8_t>(padded * h);
  b.glo = c.take<uint8_t>(padded * h);
  b.gsc = c.take<uint8_t>(padded * h / 32);
  b.uhi = c.take<uint8_t>(padded * h);
  b.ulo = c.take<uint8_t>(padded * h);
  b.usc = c.take<uint8_t>(padded * h / 32);
  b.gu = c.take<float>(padded * 2 * m * sizeof(float));
  b.dhi = c.take<uint8_t>(padded * m);
  b.dlo = c.take<uint8_t>(padded * m);
  b.dsc = c.take<uint8_t>(padded * m / 32);
  b.v = c.take<float>(padded * h * sizeof(float));
  if (dense) {
    const int t = static_cast<int>(tokens);
    b.dsplits_gu = bf16_gemm_splits(t, h, m);
    b.dsplits_d = bf16_gemm_splits(t, m, h);
    b.dgate = c.take<float>(static_cast<size_t>(b.dsplits_gu) * tokens * m * sizeof(float));
    b.dup = c.take<float>(static_cast<size_t>(b.dsplits_gu) * tokens * m * sizeof(float));
    b.dh = c.take<void>(static_cast<size_t>(tokens) * m * sizeof(uint16_t));
    b.ddown = c.take<float>(static_cast<size_t>(b.dsplits_d) * tokens * h * sizeof(float));
    b.derr = c.take<int32_t>(16);
  }
  return b;
}

size_t prefill_bytes(int64_t tokens, int slots, int h, int m, int64_t experts, bool dense) {
  Carver c(nullptr);
  carve_prefill(tokens, slots, h, m, experts, dense, c);
  return c.used;
}

// Everything up to the float32 down products b.v (and the dense shared
// expert's partials when `shared` is given).
int prefill_products(const void* x, int x_dtype, int per_slot, int slots, const uint32_t* ids, int64_t tokens,
                     const exlr8_trellis_experts* ex, int64_t experts, const exlr8_dense_expert* shared,
                     const PrefillBuffers& b, cudaStream_t s) {
  const int h = ex->hidden, m = ex->intermediate;
  const int64_t rows = tokens * slots;
  const int64_t padded = mx_padded_rows(rows, experts);
  const int e = static_cast<int>(experts), n = static_cast<int>(rows);
  EXLR8_TIMED(EXLR8_KERNEL_PLAN, s, launch_plan(ids, n, e, slots, shared ? 8 : -1, b.plan, s));
  EXLR8_TIMED(EXLR8_KERNEL_PLAN, s, launch_joined_segments(b.plan, e, n, b.chunks, s));
  EXLR8_TIMED(EXLR8_KERNEL_PREP, s,
              launch_trellis_prep(x, x_dtype, per_slot, slots, n, ids, b.chunks, ex->in_scale[0], ex->in_scale[1],
                                  ex->scale_dtype, 2, h, b.ghi, b.glo, b.gsc, b.uhi, b.ulo, b.usc, s));
  if (shared) {
    const int t = static_cast<int>(tokens);
    const uint16_t* xb = static_cast<const uint16_t*>(x);
    EXLR8_TRY(cudaMemsetAsync(b.derr, 0, sizeof(int32_t), s));
    EXLR8_TIMED(EXLR8_KERNEL_DENSE, s,
                launch_dense_gemm(xb, t, h, static_cast<const uint16_t*>(shared->gate), m, b.dsplits_gu, b.dgate,
                                  b.derr, s));
    EXLR8_TIMED(EXLR8_KERNEL_DENSE, s,
                launch_dense_gemm(xb, t, h, static_cast<const uint16_t*>(shared->up), m, b.dsplits_gu, b.dup, b.derr,
                                  s));
    EXLR8_TIMED(EXLR8_KERNEL_DENSE, s,
                launch_dense_swiglu(b.dgate, b.dup, b.dsplits_gu, tokens * m, x_dtype, b.dh, s));
    EXLR8_TIMED(EXLR8_KERNEL_DENSE, s,
                launch_dense_gemm(static_cast<const uint16_t*>(b.dh), t, m, static_cast<const uint16_t*>(shared->down),
                                  h, b.dsplits_d, b.ddown, b.derr, s));
  }
  ExpertGemmArgs g = {};
  g.weights[0] = ex->packed[0];
  g.weights[1] = ex->packed[1];
  g.x_hi[0] = b.ghi;
  g.x_lo[0] = b.glo;
  g.x_scales[0] = b.gsc;
  g.x_hi[1] = b.uhi;
  g.x_lo[1] = b.ulo;
  g.x_scales[1] = b.usc;
  g.chunks = b.chunks;
  g.counter_index = 2;
  g.experts = experts;
  g.padded_rows = padded;
  g.in_features = h;
  g.out_features = m;
  g.projections = 2;
  g.paired = 0;
  g.trellis_k = ex->k;
  g.side = 1;
  g.mcg_mask = kMcgMask;
  g.mcg_xor = kMcgXor;
  g.out = b.gu;
  g.out_stride = 2 * m;
  g.proj_offset = m;
  EXLR8_TIMED(EXLR8_KERNEL_GATE_UP, s, launch_expert_gemm(g, s));
  EXLR8_TIMED(EXLR8_KERNEL_GATE_FINISH, s,
              launch_joined_gate_finish(b.gu, ids, n, b.chunks, ex->out_scale[0], ex->out_scale[1], ex->in_scale[2],
                                        ex->scale_dtype, m, x_dtype, b.dhi, b.dlo, b.dsc, s));
  g.weights[0] = ex->packed[2];
  g.weights[1] = nullptr;
  g.x_hi[0] = b.dhi;
  g.x_lo[0] = b.dlo;
  g.x_scales[0] = b.dsc;
  g.counter_index = 3;
  g.in_features = m;
  g.out_features = h;
  g.projections = 1;
  g.side = 2;
  g.out = b.v;
  g.out_stride = h;
  g.proj_offset = 0;
  EXLR8_TIMED(EXLR8_KERNEL_DOWN, s, launch_expert_gemm(g, s));
  return EXLR8_OK;
}

// The trellis tensor-core path is built for K = 3 and 4 (the EXLR8 layer
// widths, experts.py:86); K = 2 keeps the streaming path.
inline bool use_prefill(int64_t tokens, const exlr8_trellis_experts* ex) {
  return tokens >= kPrefillMinTokens && (ex->k == 3 || ex->k == 4);
}
// The expert operators keep float32 activations on the streaming path at any
// row count: it accumulates in float32 from f16 hi/lo weight fragments and
// meets the reference's float32 tolerance (test_experts.py:147), which the
// GEMM's two E4M3 activation planes (about 1e-3 relative) do not.
inline bool use_prefill(int64_t tokens, const exlr8_trellis_experts* ex, int x_dtype) {
  return x_dtype != EXLR8_DTYPE_F32 && use_prefill(tokens, ex);
}

}  // namespace

extern "C" {

int exlr8_abi_version(void) { return EXLR8_ABI_VERSION; }

const char* exlr8_status_string(int status) {
  switch (status) {
    case EXLR8_OK: return "ok";
    case EXLR8_ERR_WIDTH: return "EXLR8 trellis width must be 2, 3, or 4";
    case EXLR8_ERR_DIMS: return "trellis dimensions must be positive multiples of 128";
    case EXLR8_ERR_SIDE: return "sharded_side must be 0, 1, or 2";
    case EXLR8_ERR_BYTES: return "packed byte count does not match the trellis dimensions";
    case EXLR8_ERR_SCALES: return "expert side vectors must contain full signed channel scales";
    case EXLR8_ERR_ROWS: return "activation rows do not match the expert indices";
    case EXLR8_ERR_WIDTH_X: return "activation width does not match in_features";
    case EXLR8_ERR_DTYPE: return "unsupported activation or scale dtype";
    case EXLR8_ERR_ALIGN: return "device pointers must be 16-byte aligned";
    case EXLR8_ERR_WORKSPACE: return "workspace is missing or too small";
    case EXLR8_ERR_ARG: return "invalid argument";
    case EXLR8_ERR_CUDA: return "CUDA runtime error";
    case EXLR8_ERR_ID_RANGE: return "Expert IDs must be in 0..256";
    case EXLR8_ERR_UNSUPPORTED: return "unsupported configuration";
    case EXLR8_ERR_STATIC_LIMIT:
      return "request needs more scratch than the fixed no-allocation buffer (EXLR8_NOALLOC_SCRATCH_BYTES)";
    default: return "unknown status";
  }
}

const char* exlr8_last_cuda_error(void) { return g_cuda_error; }

int exlr8_codebook(const uint32_t* states, float* values, int64_t count, int paired, void* stream) {
  if (count < 0 || (count > 0 && (!states || !values))) return EXLR8_ERR_ARG;
  return cuda_status(launch_codebook(states, values, count, paired, as_stream(stream)));
}

int exlr8_check_format(int64_t packed_bytes, int k, int in_features, int out_features, int sharded_side,
                       int64_t* matrices) {
  return format_status(packed_bytes, k, in_features, out_features, sharded_side, matrices);
}

int exlr8_decode_trellis(const void* packed, int64_t packed_bytes, int64_t matrix, int k, int in_features,
                         int out_features, int sharded_side, float* inner, void* stream) {
  int64_t count = 0;
  EXLR8_CHECK(format_status(packed_bytes, k, in_features, out_features, sharded_side, &count));
  if (!packed || !inner || matrix < 0 || matrix >= count) return EXLR8_ERR_ARG;
  return cuda_status(launch_decode_matrix(static_cast<const uint32_t*>(packed), matrix, k, in_features, out_features,
                                          sharded_side, inner, as_stream(stream)));
}

int exlr8_expand_static_trellis(const void* packed, int64_t packed_bytes, int k, int in_features, int out_features,
                                int sharded_side, uint8_t* out, void* stream) {
  int64_t count = 0;
  EXLR8_CHECK(format_status(packed_bytes, k, in_features, out_features, sharded_side, &count));
  if (!packed || !out) return EXLR8_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(packed) | reinterpret_cast<uintptr_t>(out)) & 3u) return EXLR8_ERR_ALIGN;
  return cuda_status(launch_expand_static(static_cast<const uint32_t*>(packed), packed_bytes / (32 * k), k,
                                          reinterpret_cast<uint32_t*>(out), as_stream(stream)));
}

size_t exlr8_dequantize_trellis_workspace(int in_features, int out_features) {
  return align_up(static_cast<size_t>(in_features) * out_features * sizeof(float));
}

int exlr8_dequantize_trellis(const void* packed, int64_t packed_bytes, const void* suh, const void* svh,
                             int scale_dtype, int k, int in_features, int out_features, int sharded_side,
                             float* weight, void* workspace, size_t workspace_bytes, void* stream) {
  int64_t count = 0;
  EXLR8_CHECK(format_status(packed_bytes, k, in_features, out_features, sharded_side, &count));
  if (count != 1) return EXLR8_ERR_BYTES;
  if (!packed || !suh || !svh || !weight) return EXLR8_ERR_ARG;
  if (!valid_scale(scale_dtype)) return EXLR8_ERR_DTYPE;
  if (!workspace || workspace_bytes < exlr8_dequantize_trellis_workspace(in_features, out_features))
    return EXLR8_ERR_WORKSPACE;
  float* inner = static_cast<float*>(workspace);
  EXLR8_TRY(launch_decode_matrix(static_cast<const uint32_t*>(packed), 0, k, in_features, out_features, sharded_side,
                                 inner, as_stream(stream)));
  return cuda_status(
      launch_dequantize(inner, suh, svh, scale_dtype, in_features, out_features, weight, as_stream(stream)));
}

int exlr8_hadamard128(const float* x, int64_t rows, int features, float* out, void* stream) {
  if (rows < 0 || features <= 0 || features % 128) return EXLR8_ERR_DIMS;
  if (rows == 0) return EXLR8_OK;
  if (!x || !out) return EXLR8_ERR_ARG;
  return cuda_status(launch_hadamard128(x, rows * (features / 128), out, as_stream(stream)));
}

int exlr8_mxfp4_quantize(const float* w, int64_t rows, int in_features, uint32_t* codes, uint8_t* scales,
                         void* stream) {
  if (rows < 0 || in_features <= 0 || in_features % 32) return EXLR8_ERR_DIMS;
  if (rows == 0) return EXLR8_OK;
  if (!w || !codes || !scales) return EXLR8_ERR_ARG;
  if (!aligned16(w) || !aligned16(codes)) return EXLR8_ERR_ALIGN;
  return cuda_status(launch_mxfp4_quantize(w, rows, in_features, codes, scales, as_stream(stream)));
}

int exlr8_mxfp4_encode_trellis(const void* packed, int64_t packed_bytes, int k, int in_features, int out_features,
                               int sharded_side, const void* in_scale, const void* unit, int scale_dtype,
                               uint32_t* codes, uint8_t* scales, int64_t rows_per_matrix, int64_t row_offset,
                               void* stream) {
  int64_t count = 0;
  EXLR8_CHECK(format_status(packed_bytes, k, in_features, out_features, sharded_side, &count));
  if (!packed || !codes || !scales || (unit && !in_scale)) return EXLR8_ERR_ARG;
  if (row_offset < 0 || rows_per_matrix < row_offset + out_features) return EXLR8_ERR_DIMS;
  if (in_scale && !valid_scale(scale_dtype)) return EXLR8_ERR_DTYPE;
  if (!aligned16(packed) || !aligned16(codes) || (reinterpret_cast<uintptr_t>(scales) & 3u)) return EXLR8_ERR_ALIGN;
  return cuda_status(launch_mxfp4_encode_trellis(static_cast<const uint32_t*>(packed), count, k, in_features,
                                                 out_features, sharded_side, in_scale, unit, scale_dtype, codes,
                                                 scales, rows_per_matrix, row_offset, as_stream(stream)));
}

int exlr8_route(const float* logits, const float* bias, int64_t rows, uint32_t* indices, float* scores,
                void* stream) {
  if (rows < 0 || (rows > 0 && (!logits || !bias || !indices || !scores))) return EXLR8_ERR_ARG;
  return cuda_status(launch_route(logits, bias, static_cast<int>(rows), indices, scores, 2.5f, 256u,
                                  as_stream(stream)));
}

size_t exlr8_dispatch_plan_workspace(int64_t rows, int experts) {
  if (rows < 0 || rows > (int64_t(1) << 30) || experts < 1 || experts > kDispatchMaxExperts) return kBadSize;
  return align_up(plan_bytes(static_cast<int>(rows), experts));
}

int exlr8_dispatch_plan(const uint32_t* ids, int64_t rows, int experts, int block_rows, uint32_t* order,
                        uint32_t* sorted_ids, uint32_t* table, int64_t table_capacity, int32_t* count,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (rows < 0 || rows > (int64_t(1) << 30) || experts < 1 || experts > kDispatchMaxExperts || block_rows < 1)
    return EXLR8_ERR_ARG;
  // The reference's table width: min(rows, rows / block_rows + experts) columns.
  const int64_t need = std::min<int64_t>(rows, rows / block_rows + experts);
  if (table_capacity < need || !count || (rows > 0 && (!ids || !order || !sorted_ids || !table)))
    return EXLR8_ERR_ARG;
  if (!workspace || workspace_bytes < exlr8_dispatch_plan_workspace(rows, experts)) return EXLR8_ERR_WORKSPACE;
  const PlanView plan = plan_view(workspace, static_cast<int>(rows), experts);
  return cuda_status(launch_dispatch_plan(ids, static_cast<int>(rows), experts, block_rows, plan, order, sorted_ids,
                                          table, table_capacity, count, as_stream(stream)));
}

int exlr8_combine(const void* values, const float* scores, const void* residual, int64_t tokens, int hidden,
                  int dtype, void* out, void* stream) {
  if (!valid_act(dtype)) return EXLR8_ERR_DTYPE;
  if (tokens < 0 || hidden <= 0) return EXLR8_ERR_ARG;
  if (tokens == 0) return EXLR8_OK;
  if (!values || !scores || !residual || !out) return EXLR8_ERR_ARG;
  return cuda_status(launch_combine(values, scores, residual, tokens, hidden, dtype, out, as_stream(stream)));
}

int exlr8_router(const void* x, int x_dtype, int64_t tokens, int hidden, const float* gate_weight, const float* bias,
                 float* logits, uint32_t* indices, float* scores, void* stream) {
  if (!valid_act(x_dtype)) return EXLR8_ERR_DTYPE;
  if (tokens < 0 || hidden <= 0 || hidden % 4) return EXLR8_ERR_ARG;
  if (tokens == 0) return EXLR8_OK;
  if (!x || !gate_weight || !bias || !logits || !indices || !scores) return EXLR8_ERR_ARG;
  if (!aligned16(gate_weight) || !aligned16(x)) return EXLR8_ERR_ALIGN;
  EXLR8_TRY(launch_gate_logits(x, x_dtype, static_cast<int>(tokens), hidden, gate_weight, logits, 256,
                               as_stream(stream)));
  return cuda_status(launch_route(logits, bias, static_cast<int>(tokens), indices, scores, 2.5f, 256u,
                                  as_stream(stream)));
}

size_t exlr8_expert_linear_workspace(int64_t tokens, int slots, int in_features, int out_features, int64_t experts) {
  if (!sizes_ok(tokens, slots, in_features, out_features, experts)) return kBadSize;
  const int64_t rows = tokens * slots;
  const Splits sp = linear_splits(in_features);
  return align_up(plan_bytes(static_cast<int>(rows), static_cast<int>(experts))) +
         align_up(frag_bytes(rows, in_features, 1)) +
         align_up(rows * sp.count * static_cast<size_t>(out_features) * sizeof(float));
}

int exlr8_expert_linear(const void* x, int x_dtype, int per_slot, const uint32_t* indices, int64_t tokens, int slots,
                        const void* packed, int64_t packed_bytes, const void* in_scale, const void* out_scale,
                        int scale_dtype, int64_t scale_experts, int k, int in_features, int out_features,
                        int sharded_side, void* out, void* workspace, size_t workspace_bytes, void* stream) {
  int64_t experts = 0;
  EXLR8_CHECK(format_status(packed_bytes, k, in_features, out_features, sharded_side, &experts));
  if (scale_experts != experts) return EXLR8_ERR_SCALES;
  if (!valid_act(x_dtype) || !valid_scale(scale_dtype)) return EXLR8_ERR_DTYPE;
  if (tokens < 0 || slots <= 0) return EXLR8_ERR_ROWS;
  const int64_t rows = tokens * slots;
  if (rows == 0) return EXLR8_OK;
  if (!x || !indices || !packed || !in_scale || !out_scale || !out) return EXLR8_ERR_ARG;
  if (!aligned16(packed)) return EXLR8_ERR_ALIGN;
  if (rows > (1 << 20)) return EXLR8_ERR_UNSUPPORTED;
  if (!workspace || workspace_bytes < exlr8_expert_linear_workspace(tokens, slots, in_features, out_features, experts))
    return EXLR8_ERR_WORKSPACE;
  cudaStream_t s = as_stream(stream);
  const Splits sp = linear_splits(in_features);
  const int n = static_cast<int>(rows), e = static_cast<int>(experts);
  Carver c(workspace);
  PlanView plan = plan_view(c.take<int32_t>(plan_bytes(n, e)), n, e);
  unsigned char* frag = c.take<unsigned char>(frag_bytes(rows, in_features, 1));
  float* part = c.take<float>(rows * sp.count * static_cast<size_t>(out_features) * sizeof(float));
  EXLR8_TRY(launch_plan(indices, n, e, slots, -1, plan, s));
  EXLR8_TRY(launch_prep_frag(x, x_dtype, per_slot, slots, indices, n, in_scale, in_scale, scale_dtype, in_features, e,
                             1, frag, s));
  StreamParams gp = stream_params(nullptr, plan, 2, n);
  gp.k = k;
  gp.packed[0] = static_cast<const uint32_t*>(packed);
  gp.packed[1] = nullptr;
  gp.frag = frag;
  gp.partial = part;
  gp.side = sharded_side;
  gp.in_features = in_features;
  gp.out_features = out_features;
  gp.kt_per_split = sp.kt;
  gp.splits = sp.count;
  gp.projections = 1;
  EXLR8_TRY(launch_stream(gp, s));
  return cuda_status(launch_finish(part, sp.count, nullptr, indices, n, out_scale, scale_dtype, out_features, e, x_dtype, out, s));
}

size_t exlr8_expert_mlp_workspace(int64_t tokens, int slots, int hidden, int intermediate, int64_t experts) {
  if (!sizes_ok(tokens, slots, hidden, intermediate, experts)) return kBadSize;
  const size_t decode = mlp_layout(tokens * slots, hidden, intermediate, experts).total();
  if (tokens < kPrefillMinTokens) return decode;
  const size_t prefill = prefill_bytes(tokens, slots, hidden, intermediate, experts, false);
  return prefill > decode ? prefill : decode;
}

static int expert_mlp(const void* x, int x_dtype, int per_slot, const uint32_t* indices, int64_t tokens, int slots,
                      const exlr8_trellis_experts* ex, const exlr8_static_cache* cache, void* out, void* workspace,
                      size_t workspace_bytes, void* stream) {
  int64_t experts = 0;
  EXLR8_CHECK(check_experts(ex, &experts));
  if (!valid_act(x_dtype)) return EXLR8_ERR_DTYPE;
  if (tokens < 0 || slots <= 0) return EXLR8_ERR_ROWS;
  const int64_t rows = tokens * slots;
  if (rows == 0) return EXLR8_OK;
  if (!x || !indices || !out) return EXLR8_ERR_ARG;
  if (rows > (1 << 20)) return EXLR8_ERR_UNSUPPORTED;
  if (!workspace || workspace_bytes < exlr8_expert_mlp_workspace(tokens, slots, ex->hidden, ex->intermediate, experts))
    return EXLR8_ERR_WORKSPACE;
  cudaStream_t s = as_stream(stream);
  if (use_prefill(tokens, ex, x_dtype)) {
    Carver pc(workspace);
    const PrefillBuffers pb = carve_prefill(tokens, slots, ex->hidden, ex->intermediate, experts, false, pc);
    EXLR8_CHECK(prefill_products(x, x_dtype, per_slot, slots, indices, tokens, ex, experts, nullptr, pb, s));
    ProfileScope scope(EXLR8_KERNEL_FINISH, s);
    return cuda_status(launch_finish(pb.v, 1, pb.chunks.slot_row, indices, static_cast<int>(rows), ex->out_scale[2],
                                     ex->scale_dtype, ex->hidden, static_cast<int>(experts), x_dtype, out, s));
  }
  const MlpLayout l = mlp_layout(rows, ex->hidden, ex->intermediate, experts);
  Carver c(workspace);
  const MlpBuffers b = carve_mlp(l, rows, experts, false, tokens, ex->hidden, ex->intermediate, c);
  EXLR8_TIMED(EXLR8_KERNEL_PLAN, s,
              launch_plan(indices, static_cast<int>(rows), static_cast<int>(experts), slots, -1, b.plan, s));
  EXLR8_CHECK(run_mlp_after_plan(x, x_dtype, per_slot, slots, indices, rows, ex, experts, nullptr, nullptr, tokens,
                                 l, b, s, cache));
  ProfileScope scope(EXLR8_KERNEL_FINISH, s);
  return cuda_status(launch_finish(b.dpart, l.s2.count, nullptr, indices, static_cast<int>(rows), ex->out_scale[2],
                                   ex->scale_dtype, ex->hidden, static_cast<int>(experts), x_dtype, out, s));
}

int exlr8_expert_mlp(const void* x, int x_dtype, int per_slot, const uint32_t* indices, int64_t tokens, int slots,
                     const exlr8_trellis_experts* ex, void* out, void* workspace, size_t workspace_bytes,
                     void* stream) {
  return expert_mlp(x, x_dtype, per_slot, indices, tokens, slots, ex, nullptr, out, workspace, workspace_bytes,
                    stream);
}

int exlr8_expert_mlp_cached(const void* x, int x_dtype, int per_slot, const uint32_t* indices, int64_t tokens,
                            int slots, const exlr8_trellis_experts* ex, const exlr8_static_cache* cache, void* out,
                            void* workspace, size_t workspace_bytes, void* stream) {
  if (!cache || !cache->expert_to_slot || cache->slots <= 0) return EXLR8_ERR_ARG;
  for (int p = 0; p < 3; ++p) {
    if (!cache->fp8[p]) return EXLR8_ERR_ARG;
    if (!aligned16(cache->fp8[p])) return EXLR8_ERR_ALIGN;
  }
  return expert_mlp(x, x_dtype, per_slot, indices, tokens, slots, ex, cache, out, workspace, workspace_bytes, stream);
}

size_t exlr8_expert_mlp_finish_workspace(int64_t tokens, int hidden, int intermediate, int64_t experts) {
  if (!sizes_ok(tokens, 9, hidden, intermediate, experts)) return kBadSize;
  const size_t decode = mlp_layout(tokens * 9, hidden, intermediate, experts).total() +
                        dense_layout(tokens, hidden, intermediate).total();
  if (tokens < kPrefillMinTokens) return decode;
  const size_t prefill = prefill_bytes(tokens, 9, hidden, intermediate, experts, true);
  return prefill > decode ? prefill : decode;
}

// Prefill counterpart of mlp_finish_after_plan (the plan runs inside).
static int prefill_finish(const void* x, int x_dtype, const uint32_t* indices, const float* scores,
                          const void* residual, int64_t tokens, const exlr8_trellis_experts* ex, int64_t experts,
                          const exlr8_dense_expert* shared, void* out, void* workspace, cudaStream_t s) {
  if (shared && !aligned16(x)) return EXLR8_ERR_ALIGN;  // tensor-map operand
  Carver pc(workspace);
  const PrefillBuffers pb = carve_prefill(tokens, 9, ex->hidden, ex->intermediate, experts, true, pc);
  EXLR8_CHECK(prefill_products(x, x_dtype, 0, 9, indices, tokens, ex, experts, shared, pb, s));
  ProfileScope scope(EXLR8_KERNEL_FINISH, s);
  return cuda_status(launch_joined_finish(pb.v, pb.chunks.slot_row, indices, static_cast<int>(tokens), ex->hidden,
                                          static_cast<int>(experts), ex->out_scale[2], ex->scale_dtype, scores,
                                          residual, shared ? pb.ddown : nullptr, pb.dsplits_d, x_dtype, out, s));
}

// Nine-slot MLP + combine after the plan exists in `b`.
static int mlp_finish_after_plan(const void* x, int x_dtype, const uint32_t* indices, const float* scores,
                                 const void* residual, int64_t tokens, const exlr8_trellis_experts* ex,
                                 int64_t experts, const exlr8_dense_expert* shared, void* out, const MlpLayout& l,
                                 const MlpBuffers& b, cudaStream_t s) {
  const int64_t rows = tokens * 9;
  EXLR8_CHECK(run_mlp_after_plan(x, x_dtype, 0, 9, indices, rows, ex, experts, shared, x, tokens, l, b, s));
  ProfileScope scope(EXLR8_KERNEL_FINISH, s);
  return cuda_status(launch_finish_fused(b.dpart, l.s2.count, nullptr, indices, static_cast<int>(tokens), ex->out_scale[2],
                                         ex->scale_dtype, ex->hidden, static_cast<int>(experts), scores, residual,
                                         shared ? b.ddown : nullptr, dense_down_splits(ex->intermediate), x_dtype,
                                         out, s));
}

int exlr8_expert_mlp_finish(const void* x, int x_dtype, const uint32_t* indices, const float* scores,
                            const void* residual, int64_t tokens, const exlr8_trellis_experts* ex,
                            const exlr8_dense_expert* shared, void* out, void* workspace, size_t workspace_bytes,
                            void* stream) {
  int64_t experts = 0;
  EXLR8_CHECK(check_experts(ex, &experts));
  if (!valid_act(x_dtype)) return EXLR8_ERR_DTYPE;
  EXLR8_CHECK(check_dense(shared, x_dtype, ex->hidden, ex->intermediate));
  if (shared && x && !aligned16(x)) return EXLR8_ERR_ALIGN;  // bulk-copied x rows of the shared expert
  if (tokens < 0) return EXLR8_ERR_ROWS;
  if (tokens == 0) return EXLR8_OK;
  if (!x || !indices || !scores || !residual || !out) return EXLR8_ERR_ARG;
  if (tokens * 9 > (1 << 20)) return EXLR8_ERR_UNSUPPORTED;
  if (!workspace || workspace_bytes < exlr8_expert_mlp_finish_workspace(tokens, ex->hidden, ex->intermediate, experts))
    return EXLR8_ERR_WORKSPACE;
  cudaStream_t s = as_stream(stream);
  if (use_prefill(tokens, ex, x_dtype))
    return prefill_finish(x, x_dtype, indices, scores, residual, tokens, ex, experts, shared, out, workspace, s);
  const int64_t rows = tokens * 9;
  const MlpLayout l = mlp_layout(rows, ex->hidden, ex->intermediate, experts);
  Carver c(workspace);
  const MlpBuffers b = carve_mlp(l, rows, experts, shared != nullptr, tokens, ex->hidden, ex->intermediate, c);
  EXLR8_TIMED(EXLR8_KERNEL_PLAN, s,
              launch_plan(indices, static_cast<int>(rows), static_cast<int>(experts), 9, shared ? 8 : -1, b.plan, s));
  return mlp_finish_after_plan(x, x_dtype, indices, scores, residual, tokens, ex, experts, shared, out, l, b, s);
}

size_t exlr8_moe_layer_workspace(int64_t tokens, int hidden, int intermediate, int64_t experts) {
  if (!sizes_ok(tokens, 9, hidden, intermediate, experts)) return kBadSize;
  size_t router = align_up(tokens * 256 * sizeof(float)) + align_up(tokens * 9 * sizeof(uint32_t)) +
                  align_up(tokens * 8 * sizeof(float));
  if (tokens >= kRouterGemmMinTokens)
    router += align_up(router_gemm_workspace(static_cast<int>(tokens), hidden, EXLR8_DTYPE_F32));
  return exlr8_expert_mlp_finish_workspace(tokens, hidden, intermediate, experts) + router;
}

int exlr8_moe_layer(const void* x, int x_dtype, const void* residual, int64_t tokens, const float* gate_weight,
                    const float* bias, const exlr8_trellis_experts* ex, const exlr8_dense_expert* shared, void* out,
                    uint32_t* indices, float* scores, void* workspace, size_t workspace_bytes, void* stream) {
  int64_t experts = 0;
  EXLR8_CHECK(check_experts(ex, &experts));
  if (!valid_act(x_dtype)) return EXLR8_ERR_DTYPE;
  EXLR8_CHECK(check_dense(shared, x_dtype, ex->hidden, ex->intermediate));
  if (!shared && experts < 257) return EXLR8_ERR_ID_RANGE;  // slot 8 routes to trellis matrix 256
  if (tokens < 0) return EXLR8_ERR_ROWS;
  if (tokens == 0) return EXLR8_OK;
  if (!x || !residual || !gate_weight || !bias || !out) return EXLR8_ERR_ARG;
  if (!aligned16(gate_weight) || !aligned16(x)) return EXLR8_ERR_ALIGN;
  if (ex->hidden % 4) return EXLR8_ERR_DIMS;
  if (tokens * 9 > (1 << 20)) return EXLR8_ERR_UNSUPPORTED;
  if (!workspace || workspace_bytes < exlr8_moe_layer_workspace(tokens, ex->hidden, ex->intermediate, experts))
    return EXLR8_ERR_WORKSPACE;
  cudaStream_t s = as_stream(stream);
  const int64_t rows = tokens * 9;
  const MlpLayout l = mlp_layout(rows, ex->hidden, ex->intermediate, experts);
  // The MLP part comes first so that the id-check header sits at offset 0.
  Carver c(workspace);
  const MlpBuffers b = carve_mlp(l, rows, experts, shared != nullptr, tokens, ex->hidden, ex->intermediate, c);
  Carver head(workspace);
  head.used = exlr8_expert_mlp_finish_workspace(tokens, ex->hidden, ex->intermediate, experts);
  float* logits = head.take<float>(tokens * 256 * sizeof(float));
  uint32_t* ids_buf = head.take<uint32_t>(tokens * 9 * sizeof(uint32_t));
  float* scores_buf = head.take<float>(tokens * 8 * sizeof(float));
  uint32_t* ids = indices ? indices : ids_buf;
  float* sc = scores ? scores : scores_buf;
  if (use_prefill(tokens, ex)) {
    if (tokens >= kRouterGemmMinTokens) {
      void* router_ws = head.take<char>(router_gemm_workspace(static_cast<int>(tokens), ex->hidden, EXLR8_DTYPE_F32));
      EXLR8_TIMED(EXLR8_KERNEL_ROUTER, s,
                  launch_router_gemm(x, x_dtype, static_cast<int>(tokens), ex->hidden, gate_weight, logits, router_ws,
                                     s));
    } else {
      EXLR8_TIMED(EXLR8_KERNEL_ROUTER, s,
                  launch_gate_logits(x, x_dtype, static_cast<int>(tokens), ex->hidden, gate_weight, logits, 256, s));
    }
    EXLR8_TIMED(EXLR8_KERNEL_ROUTER, s, launch_route(logits, bias, static_cast<int>(tokens), ids, sc, 2.5f, 256u, s));
    return prefill_finish(x, x_dtype, ids, sc, residual, tokens, ex, experts, shared, out, workspace, s);
  }
  EXLR8_TIMED(EXLR8_KERNEL_ROUTER, s,
              launch_gate_logits(x, x_dtype, static_cast<int>(tokens), ex->hidden, gate_weight, logits, 256, s));
  EXLR8_TIMED(EXLR8_KERNEL_PLAN, s,
              launch_route_plan(logits, bias, static_cast<int>(tokens), ids, sc, static_cast<int>(experts),
                                shared ? 8 : -1, b.plan, s));
  return mlp_finish_after_plan(x, x_dtype, ids, sc, residual, tokens, ex, experts, shared, out, l, b, s);
}

int exlr8_profile_enable(int enable, int capacity) {
  Profiler& p = g_prof;
  if (p.events) {
    for (int i = 0; i < 2 * p.capacity; ++i) cudaEventDestroy(p.events[i]);
    delete[] p.events;
    delete[] p.kinds;
    p.events = nullptr;
    p.kinds = nullptr;
  }
  p.on = false;
  p.used = 0;
  p.capacity = 0;
  if (!enable) return EXLR8_OK;
  if (capacity <= 0) return EXLR8_ERR_ARG;
  p.events = new cudaEvent_t[2 * capacity];
  p.kinds = new int[capacity];
  for (int i = 0; i < 2 * capacity; ++i) EXLR8_TRY(cudaEventCreate(&p.events[i]));
  p.capacity = capacity;
  p.on = true;
  return EXLR8_OK;
}

int exlr8_profile_read(int kind, int64_t* launches, double* total_ms) {
  if (!launches || !total_ms) return EXLR8_ERR_ARG;
  *launches = 0;
  *total_ms = 0.0;
  for (int i = 0; i < g_prof.used; ++i) {
    if (g_prof.kinds[i] != kind) continue;
    EXLR8_TRY(cudaEventSynchronize(g_prof.events[2 * i + 1]));
    float ms = 0.f;
    EXLR8_TRY(cudaEventElapsedTime(&ms, g_prof.events[2 * i], g_prof.events[2 * i + 1]));
    *launches += 1;
    *total_ms += ms;
  }
  return EXLR8_OK;
}

// ---- expert parallelism ---------------------------------------------------

int exlr8_ep_dispatch(const uint32_t* indices, int64_t tokens, const void* x, int x_dtype, int hidden, int ranks,
                      int experts_per_rank, int capacity, void* send_x, int32_t* send_meta, int32_t* slot_pos,
                      int32_t* counts, int32_t* status, void* stream) {
  if (!valid_act(x_dtype)) return EXLR8_ERR_DTYPE;
  if (tokens < 0 || hidden <= 0 || ranks <= 0 || ranks > 32 || experts_per_rank <= 0 || capacity < 0)
    return EXLR8_ERR_ARG;
  if ((hidden * (x_dtype == EXLR8_DTYPE_F32 ? 4 : 2)) % 16) return EXLR8_ERR_DIMS;
  if (tokens * 8 > (int64_t(1) << 24)) return EXLR8_ERR_UNSUPPORTED;
  if (!send_x || !send_meta || !counts || !status || (tokens > 0 && (!indices || !x || !slot_pos)))
    return EXLR8_ERR_ARG;
  if (!aligned16(x) || !aligned16(send_x)) return EXLR8_ERR_ALIGN;
  return cuda_status(launch_ep_dispatch(indices, static_cast<int>(tokens), x, x_dtype, hidden, ranks,
                                        experts_per_rank, capacity, send_x, send_meta, slot_pos, counts, status,
                                        as_stream(stream)));
}

int exlr8_ep_combine(const void* values, int x_dtype, const int32_t* slot_pos, const float* scores, const void* shared,
                     const void* residual, int64_t tokens, int hidden, void* out, void* stream) {
  if (!valid_act(x_dtype)) return EXLR8_ERR_DTYPE;
  if (tokens < 0 || hidden <= 0) return EXLR8_ERR_ARG;
  if (tokens == 0) return EXLR8_OK;
  if (!values || !slot_pos || !scores || !shared || !residual || !out) return EXLR8_ERR_ARG;
  EXLR8_TIMED(EXLR8_KERNEL_EP_COMBINE, as_stream(stream),
              launch_ep_combine(values, x_dtype, slot_pos, scores, shared, residual, static_cast<int>(tokens), hidden,
                                out, as_stream(stream)));
  return EXLR8_OK;
}

// ---- residual add + RMS norm in front of each MoE block ----------------------

int exlr8_residual_rms_norm(const void* x, const void* residual, const void* weight, int x_dtype, int64_t rows,
                            int hidden, float eps, void* h_out, void* out, void* stream) {
  if (!valid_act(x_dtype)) return EXLR8_ERR_DTYPE;
  if (rows < 0 || hidden <= 0) return EXLR8_ERR_ARG;
  if (rows == 0) return EXLR8_OK;
  if (!x || !weight || !out || !(eps >= 0.0f)) return EXLR8_ERR_ARG;
  if (rows > 0x7fffffff) return EXLR8_ERR_UNSUPPORTED;
  EXLR8_TIMED(EXLR8_KERNEL_NORM, as_stream(stream),
              launch_residual_rms(x, residual, weight, x_dtype, rows, hidden, eps, h_out, out, as_stream(stream)));
  return EXLR8_OK;
}

// ---- peer-memory exchange of the expert-parallel layer ---------------------

namespace {
int elem_size(int x_dtype) { return x_dtype == EXLR8_DTYPE_F32 ? 4 : 2; }
int check_peer_shape(int ranks, int max_capacity, int hidden, int x_dtype) {
  if (!valid_act(x_dtype)) return EXLR8_ERR_DTYPE;
  if (ranks < 1 || ranks > kPeerMaxRanks || max_capacity < 0 || max_capacity > 4096 || hidden <= 0)
    return EXLR8_ERR_ARG;
  if ((static_cast<int64_t>(hidden) * elem_size(x_dtype)) % 16) return EXLR8_ERR_DIMS;
  return EXLR8_OK;
}
}  // namespace

size_t exlr8_ep_peer_bytes(int ranks, int max_capacity, int hidden, int x_dtype) {
  if (check_peer_shape(ranks, max_capacity, hidden, x_dtype) != EXLR8_OK) return 0;
  return peer_layout(ranks, max_capacity, hidden, elem_size(x_dtype)).total;
}

int exlr8_ep_peer_offsets(int ranks, int max_capacity, int hidden, int x_dtype, size_t* meta, size_t* rows,
                          size_t* back) {
  EXLR8_CHECK(check_peer_shape(ranks, max_capacity, hidden, x_dtype));
  if (!meta || !rows || !back) return EXLR8_ERR_ARG;
  const PeerLayout l = peer_layout(ranks, max_capacity, hidden, elem_size(x_dtype));
  *meta = l.meta;
  *rows = l.rows;
  *back = l.back;
  return EXLR8_OK;
}

int exlr8_ep_peer_create(size_t bytes, void** region, void* ipc_handle) {
  if (!region || !ipc_handle || bytes == 0) return EXLR8_ERR_ARG;
  void* p = nullptr;
  EXLR8_TRY(cudaMalloc(&p, bytes));
  cudaError_t err = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t handle;
  if (err == cudaSuccess) err = cudaIpcGetMemHandle(&handle, p);
  if (err != cudaSuccess) {
    cudaFree(p);
    return cuda_status(err);
  }
  std::memcpy(ipc_handle, &handle, sizeof(handle));
  *region = p;
  return EXLR8_OK;
}

int exlr8_ep_peer_open(const void* ipc_handle, void** region) {
  if (!ipc_handle || !region) return EXLR8_ERR_ARG;
  cudaIpcMemHandle_t handle;
  std::memcpy(&handle, ipc_handle, sizeof(handle));
  return cuda_status(cudaIpcOpenMemHandle(region, handle, cudaIpcMemLazyEnablePeerAccess));
}

int exlr8_ep_peer_close(void* region) { return region ? cuda_status(cudaIpcCloseMemHandle(region)) : EXLR8_OK; }

int exlr8_ep_peer_destroy(void* region) { return region ? cuda_status(cudaFree(region)) : EXLR8_OK; }

int exlr8_ep_send(const uint32_t* indices, int64_t tokens, const void* x, int x_dtype, int hidden, int ranks, int rank,
                  int experts_per_rank, int max_capacity, const uint64_t* peers, void* region, int32_t* slot_pos,
                  int32_t* status, void* stream) {
  EXLR8_CHECK(check_peer_shape(ranks, max_capacity, hidden, x_dtype));
  if (tokens < 0 || tokens * 8 > max_capacity) return EXLR8_ERR_ROWS;
  if (rank < 0 || rank >= ranks || experts_per_rank <= 0) return EXLR8_ERR_ARG;
  if (!peers || !region || !status || (tokens > 0 && (!indices || !x || !slot_pos))) return EXLR8_ERR_ARG;
  if ((x && !aligned16(x)) || !aligned16(region)) return EXLR8_ERR_ALIGN;
  EXLR8_TIMED(EXLR8_KERNEL_EP_SEND, as_stream(stream),
              launch_ep_send(indices, static_cast<int>(tokens), x, x_dtype, hidden, ranks, rank, experts_per_rank,
                             static_cast<int>(tokens * 8), max_capacity, peers, region, slot_pos, status,
                             as_stream(stream)));
  return EXLR8_OK;
}

int exlr8_peer_write(void* dst, const void* src, int64_t bytes, void* stream) {
  if (bytes < 0 || bytes % 16) return EXLR8_ERR_ARG;
  if (bytes == 0) return EXLR8_OK;
  if (!dst || !src) return EXLR8_ERR_ARG;
  if (!aligned16(dst) || !aligned16(src)) return EXLR8_ERR_ALIGN;
  return cuda_status(launch_peer_write(dst, src, bytes, as_stream(stream)));
}

int exlr8_ep_return(const void* values, int x_dtype, int hidden, int ranks, int rank, int64_t tokens,
                    int max_capacity, const uint64_t* peers, void* region, int32_t* status, void* stream) {
  EXLR8_CHECK(check_peer_shape(ranks, max_capacity, hidden, x_dtype));
  if (tokens < 0 || tokens * 8 > max_capacity) return EXLR8_ERR_ROWS;
  if (rank < 0 || rank >= ranks) return EXLR8_ERR_ARG;
  if (!peers || !region || !status || (tokens > 0 && !values)) return EXLR8_ERR_ARG;
  if ((values && !aligned16(values)) || !aligned16(region)) return EXLR8_ERR_ALIGN;
  EXLR8_TIMED(EXLR8_KERNEL_EP_RETURN, as_stream(stream),
              launch_ep_return(values, x_dtype, hidden, ranks, rank, static_cast<int>(tokens * 8), max_capacity, peers,
                               region, status, as_stream(stream)));
  return EXLR8_OK;
}

// ---- owner's half of an expert-parallel layer -----------------------------

constexpr int64_t kFusedSharedMaxRows = 4096;  // stream path with dense units up to this many rows

size_t exlr8_expert_mlp_shared_workspace(int64_t rows, int hidden, int intermediate, int64_t experts,
                                         int64_t shared_tokens) {
  if (!sizes_ok(rows, 1, hidden, intermediate, experts) || !sizes_ok(shared_tokens, 1, hidden, intermediate, 0))
    return kBadSize;
  if (rows <= kFusedSharedMaxRows)
    return mlp_layout(rows, hidden, intermediate, experts).total() +
           dense_layout(shared_tokens, hidden, intermediate).total();
  return align_up(exlr8_expert_mlp_workspace(rows, 1, hidden, intermediate, experts)) +
         exlr8_shared_expert_workspace(shared_tokens, hidden, intermediate);
}

int exlr8_expert_mlp_shared(const void* x, int x_dtype, const uint32_t* indices, int64_t rows,
                            const exlr8_trellis_experts* ex, const void* shared_x, int64_t shared_tokens,
                            const exlr8_dense_expert* shared, void* out, void* shared_out, void* workspace,
                            size_t workspace_bytes, void* stream) {
  int64_t experts = 0;
  EXLR8_CHECK(check_experts(ex, &experts));
  if (!valid_act(x_dtype)) return EXLR8_ERR_DTYPE;
  if (!shared) return EXLR8_ERR_ARG;
  EXLR8_CHECK(check_dense(shared, x_dtype, ex->hidden, ex->intermediate));
  if (rows < 0 || shared_tokens < 0) return EXLR8_ERR_ROWS;
  if ((rows > 0 && (!x || !indices || !out)) || (shared_tokens > 0 && (!shared_x || !shared_out)))
    return EXLR8_ERR_ARG;
  if ((x && !aligned16(x)) || (shared_x && !aligned16(shared_x))) return EXLR8_ERR_ALIGN;
  if (rows > (1 << 20) || shared_tokens > (1 << 20)) return EXLR8_ERR_UNSUPPORTED;
  if (!workspace ||
      workspace_bytes < exlr8_expert_mlp_shared_workspace(rows, ex->hidden, ex->intermediate, experts, shared_tokens))
    return EXLR8_ERR_WORKSPACE;
  cudaStream_t s = as_stream(stream);
  const int h = ex->hidden, m = ex->intermediate;
  if (rows > kFusedSharedMaxRows) {
    const size_t mlp_bytes = align_up(exlr8_expert_mlp_workspace(rows, 1, h, m, experts));
    EXLR8_CHECK(exlr8_expert_mlp(x, x_dtype, 1, indices, rows, 1, ex, out, workspace, mlp_bytes, stream));
    if (shared_tokens == 0) return EXLR8_OK;
    return exlr8_shared_expert(shared_x, x_dtype, shared_tokens, h, m, shared, shared_out,
                               static_cast<char*>(workspace) + mlp_bytes, workspace_bytes - mlp_bytes, stream);
  }
  if (rows == 0 && shared_tokens == 0) return EXLR8_OK;
  const MlpLayout l = mlp_layout(rows, h, m, experts);
  Carver c(workspace);
  const MlpBuffers b = carve_mlp(l, rows, experts, true, shared_tokens, h, m, c);
  const int n = static_cast<int>(rows), e = static_cast<int>(experts);
  EXLR8_TIMED(EXLR8_KERNEL_PLAN, s, launch_plan(indices, n, e, 1, -1, b.plan, s));
  // An owner's rows: fixed capacity per source, mostly empty at decode sizes.
  EXLR8_CHECK(run_mlp_after_plan(x, x_dtype, 1, 1, indices, rows, ex, experts, shared_tokens > 0 ? shared : nullptr,
                                 shared_x, shared_tokens, l, b, s, nullptr, 1));
  if (rows > 0) {
    ProfileScope scope(EXLR8_KERNEL_FINISH, s);
    EXLR8_TRY(launch_finish(b.dpart, l.s2.count, nullptr, indices, n, ex->out_scale[2], ex->scale_dtype, h, e,
                            x_dtype, out, s));
  }
  if (shared_tokens == 0) return EXLR8_OK;
  return cuda_status(launch_sum_cast(b.ddown, dense_down_splits(m), shared_tokens * h, x_dtype, shared_out, s));
}

size_t exlr8_shared_expert_workspace(int64_t tokens, int hidden, int intermediate) {
  if (!sizes_ok(tokens, 1, hidden, intermediate, 0)) return kBadSize;
  if (tokens <= 0) return 0;
  if (tokens < kPrefillMinTokens)
    return dense_layout(tokens, hidden, intermediate).total();
  const int t = static_cast<int>(tokens);
  const size_t sgu = bf16_gemm_splits(t, hidden, intermediate), sd = bf16_gemm_splits(t, intermediate, hidden);
  return 2 * align_up(sgu * tokens * intermediate * sizeof(float)) + align_up(tokens * intermediate * 2) +
         align_up(sd * tokens * hidden * sizeof(float)) + align_up(16);
}

// T(down(SwiGLU(T(x Wg^T), T(x Wu^T)))) of the dense bf16 shared expert for
// every token: the typed slot-8 value of the combine (model.py:415-418).
int exlr8_shared_expert(const void* x, int x_dtype, int64_t tokens, int hidden, int intermediate,
                        const exlr8_dense_expert* shared, void* out, void* workspace, size_t workspace_bytes,
                        void* stream) {
  if (!shared) return EXLR8_ERR_ARG;
  EXLR8_CHECK(check_dense(shared, x_dtype, hidden, intermediate));
  if (tokens < 0) return EXLR8_ERR_ROWS;
  if (tokens == 0) return EXLR8_OK;
  if (!x || !out) return EXLR8_ERR_ARG;
  if (!aligned16(x)) return EXLR8_ERR_ALIGN;
  if (tokens > (int64_t(1) << 20)) return EXLR8_ERR_UNSUPPORTED;
  if (!workspace || workspace_bytes < exlr8_shared_expert_workspace(tokens, hidden, intermediate))
    return EXLR8_ERR_WORKSPACE;
  cudaStream_t s = as_stream(stream);
  const int t = static_cast<int>(tokens);
  const uint16_t* xb = static_cast<const uint16_t*>(x);
  Carver c(workspace);
  if (tokens < kPrefillMinTokens) {
    const DenseLayout dl = dense_layout(tokens, hidden, intermediate);
    float* dg = c.take<float>(dl.gate);
    float* du = c.take<float>(dl.up);
    void* dh = c.take<void>(dl.h);
    float* dd = c.take<float>(dl.down);
    int32_t* counters = c.take<int32_t>(dl.counters);
    EXLR8_CHECK(launch_dense_decode(x, x_dtype, tokens, shared, hidden, intermediate, dg, du, dh, dd, counters, s));
    return cuda_status(launch_sum_cast(dd, kDenseDownSplits, tokens * hidden, x_dtype, out, s));
  }
  const int sgu = bf16_gemm_splits(t, hidden, intermediate), sd = bf16_gemm_splits(t, intermediate, hidden);
  float* dg = c.take<float>(static_cast<size_t>(sgu) * tokens * intermediate * sizeof(float));
  float* du = c.take<float>(static_cast<size_t>(sgu) * tokens * intermediate * sizeof(float));
  void* dh = c.take<void>(static_cast<size_t>(tokens) * intermediate * 2);
  float* dd = c.take<float>(static_cast<size_t>(sd) * tokens * hidden * sizeof(float));
  int32_t* err = c.take<int32_t>(16);
  EXLR8_TRY(cudaMemsetAsync(err, 0, sizeof(int32_t), s));
  EXLR8_TIMED(EXLR8_KERNEL_DENSE, s,
              launch_dense_gemm(xb, t, hidden, static_cast<const uint16_t*>(shared->gate), intermediate, sgu, dg, err,
                                s));
  EXLR8_TIMED(EXLR8_KERNEL_DENSE, s,
              launch_dense_gemm(xb, t, hidden, static_cast<const uint16_t*>(shared->up), intermediate, sgu, du, err,
                                s));
  EXLR8_TIMED(EXLR8_KERNEL_DENSE, s, launch_dense_swiglu(dg, du, sgu, tokens * intermediate, x_dtype, dh, s));
  EXLR8_TIMED(EXLR8_KERNEL_DENSE, s,
              launch_dense_gemm(static_cast<const uint16_t*>(dh), t, intermediate,
                                static_cast<const uint16_t*>(shared->down), hidden, sd, dd, err, s));
  return cuda_status(launch_sum_cast(dd, sd, tokens * hidden, x_dtype, out, s));
}

int exlr8_prefill_status(const void* workspace, int64_t tokens, int slots, int intermediate, int64_t experts,
                         int32_t* header_out, void* stream) {
  if (!workspace || !header_out || tokens <= 0 || slots <= 0 || intermediate <= 0) return EXLR8_ERR_ARG;
  Carver c(const_cast<void*>(workspace));
  const PrefillBuffers b = carve_prefill(tokens, slots, 128, intermediate, experts, false, c);
  EXLR8_TRY(cudaMemcpyAsync(header_out, b.chunks.header, 8 * sizeof(int32_t), cudaMemcpyDeviceToHost,
                            as_stream(stream)));
  return cuda_status(cudaStreamSynchronize(as_stream(stream)));
}

int exlr8_workspace_bad_ids(const void* workspace, int64_t* bad_ids, void* stream) {
  if (!workspace || !bad_ids) return EXLR8_ERR_ARG;
  int32_t header[16];
  EXLR8_TRY(cudaMemcpyAsync(header, workspace, sizeof(header), cudaMemcpyDeviceToHost, as_stream(stream)));
  EXLR8_TRY(cudaStreamSynchronize(as_stream(stream)));
  *bad_ids = header[8];
  return EXLR8_OK;
}

int exlr8_gemm_pair(int enable) { return set_gemm_pair(enable); }

}  // extern "C"
