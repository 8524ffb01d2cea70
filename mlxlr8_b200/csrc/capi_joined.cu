// extern "C" entry points of the joined MXFP4 path (exlr8 joined_mxfp4.py
// JoinedMXFP4.slots / .finish and the prefill MoE layer around them).
//
// Sequence of one call (all on the caller's stream, no allocation):
//   plan (expert sort) -> segments/row maps -> prep (H(x * unit), E4M3 hi/lo)
//   -> grouped tcgen05 gate+up GEMM -> gate finish (SwiGLU, down input
//   quantised) -> grouped tcgen05 down GEMM -> finish (per slot, or fused
//   with the routing-weighted combine, the shared slot and the residual).

#include "capi_util.cuh"
#include "common.cuh"
#include "joined.cuh"
#include "joined_stream.cuh"
#include "mx_gemm.cuh"
#include "router.cuh"
#include "router_gemm.cuh"
#include "stream.cuh"
#include "trellis_gemv.cuh"

using namespace exlr8;

namespace {

struct JoinedLayout {
  int64_t rows, padded, max_chunks;
};

JoinedLayout joined_layout(int64_t tokens, int slots, int64_t experts) {
  JoinedLayout l;
  l.rows = tokens * slots;
  l.padded = mx_padded_rows(l.rows, experts);
  l.max_chunks = mx_max_chunks(l.rows, experts);
  return l;
}

struct JoinedBuffers {
  PlanView plan;
  MxChunks chunks;
  uint8_t *x_hi, *x_lo, *x_scales;
  float* gu;
  uint8_t *h_hi, *h_lo, *h_scales;
  float* v;
};

JoinedBuffers carve_joined(const JoinedLayout& l, int hidden, int inter, int64_t experts, Carver& c) {
  JoinedBuffers b;
  void* plan_base = c.take<char>(plan_bytes(static_cast<int>(l.rows), static_cast<int>(experts)));
  b.plan = plan_view(plan_base, static_cast<int>(l.rows), static_cast<int>(experts));
  b.chunks.header = c.take<int32_t>(16 * sizeof(int32_t));
  b.chunks.chunk_start = c.take<int32_t>(l.max_chunks * sizeof(int32_t));
  b.chunks.chunk_rows = c.take<int32_t>(l.max_chunks * sizeof(int32_t));
  b.chunks.chunk_expert = c.take<int32_t>(l.max_chunks * sizeof(int32_t));
  b.chunks.padded_start = c.take<int32_t>((experts + 1) * sizeof(int32_t));
  b.chunks.row_slot = c.take<int32_t>(l.padded * sizeof(int32_t));
  b.chunks.slot_row = c.take<int32_t>(l.rows * sizeof(int32_t));
  b.x_hi = c.take<uint8_t>(l.padded * hidden);
  b.x_lo = c.take<uint8_t>(l.padded * hidden);
  b.x_scales = c.take<uint8_t>(l.padded * hidden / 32);
  b.gu = c.take<float>(l.padded * 2 * inter * sizeof(float));
  b.h_hi = c.take<uint8_t>(l.padded * inter);
  b.h_lo = c.take<uint8_t>(l.padded * inter);
  b.h_scales = c.take<uint8_t>(l.padded * inter / 32);
  b.v = c.take<float>(l.padded * hidden * sizeof(float));
  return b;
}

inline bool aligned32(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 31u) == 0; }

int check_joined(const exlr8_joined_mxfp4* w) {
  if (!w) return EXLR8_ERR_ARG;
  if (w->experts <= 0 || w->hidden <= 0 || w->intermediate <= 0) return EXLR8_ERR_DIMS;
  if (w->hidden % 256 || w->intermediate % 128) return EXLR8_ERR_DIMS;
  if (w->experts * 2 * w->intermediate >= (int64_t(1) << 31) || w->experts * w->hidden >= (int64_t(1) << 31))
    return EXLR8_ERR_UNSUPPORTED;
  if (!valid_scale(w->scale_dtype)) return EXLR8_ERR_DTYPE;
  if (!w->gate_up || !w->gate_up_scales || !w->down || !w->down_scales || !w->unit || !w->gate_out || !w->up_out ||
      !w->down_in || !w->down_out)
    return EXLR8_ERR_ARG;
  if (!aligned32(w->gate_up) || !aligned32(w->down) || !aligned16(w->gate_up_scales) || !aligned16(w->down_scales))
    return EXLR8_ERR_ALIGN;
  return EXLR8_OK;
}

// ---- decode batches: the MXFP4 streaming GEMV -----------------------------
//
// Up to kJoinedStreamMaxTokens token rows the joined products run as the
// streaming GEMV of joined_stream.cu (the reference's ordered-gather GEMV and
// small-batch gather_qmm roles): plan (expert groups of <= 8 slots) ->
// activation records of H(x * unit) -> gate/up stream (one joined [2m]
// matrix, written as gate and up planes) -> gate finish (Hadamard, output
// scales, typed SwiGLU, down input scale, Hadamard -> records) -> down stream
// -> the trellis path's finish kernels (the finishing arithmetic is the same).
constexpr int64_t kJoinedStreamMaxTokens = 16;
constexpr int64_t kJoinedStreamCtasHint = 296;  // persistent stream CTAs on a B200 (2 per SM)

struct JoinedSplits {
  int kb, count;
};

// K splits of a stream: enough units for >= 4 per persistent CTA, an even
// number of 128-wide K blocks per split (a stream stage holds two).
inline JoinedSplits joined_splits(int in_features, int64_t units_per_split, int cap) {
  const int kblocks = in_features / 128;
  int64_t want = (4 * kJoinedStreamCtasHint + units_per_split - 1) / (units_per_split > 0 ? units_per_split : 1);
  if (want < 1) want = 1;
  if (want > cap) want = cap;
  if (want > kblocks) want = kblocks;
  JoinedSplits sp;
  sp.kb = (kblocks + static_cast<int>(want) - 1) / static_cast<int>(want);
  sp.kb += sp.kb & 1;  // whole stages (two blocks each) per split
  sp.count = (kblocks + sp.kb - 1) / sp.kb;
  return sp;
}

struct JoinedDecodeLayout {
  JoinedSplits s1, s2;
  size_t plan, frag_gu, gu, frag_d, dpart;
  size_t total() const { return plan + frag_gu + gu + frag_d + dpart; }
};

JoinedDecodeLayout joined_decode_layout(int64_t rows, int h, int m, int64_t experts) {
  JoinedDecodeLayout l;
  l.s1 = joined_splits(h, rows * (2 * m / 128), 16);
  l.s2 = joined_splits(m, rows * (h / 128), 8);
  l.plan = align_up(plan_bytes(static_cast<int>(rows), static_cast<int>(experts)));
  l.frag_gu = align_up(frag_bytes(rows, h, 1));
  l.gu = align_up(2 * static_cast<size_t>(rows) * l.s1.count * m * sizeof(float));
  l.frag_d = align_up(frag_bytes(rows, m, 1));
  l.dpart = align_up(static_cast<size_t>(rows) * l.s2.count * h * sizeof(float));
  return l;
}

struct JoinedDecodeBuffers {
  PlanView plan;
  unsigned char *frag_gu, *frag_d;
  float *gu, *dpart;
};

JoinedDecodeBuffers carve_joined_decode(const JoinedDecodeLayout& l, int64_t rows, int64_t experts, Carver& c) {
  JoinedDecodeBuffers b;
  b.plan = plan_view(c.take<int32_t>(l.plan), static_cast<int>(rows), static_cast<int>(experts));
  b.frag_gu = c.take<unsigned char>(l.frag_gu);
  b.gu = c.take<float>(l.gu);
  b.frag_d = c.take<unsigned char>(l.frag_d);
  b.dpart = c.take<float>(l.dpart);
  return b;
}

inline bool use_joined_stream(int64_t tokens) { return tokens <= kJoinedStreamMaxTokens; }

// Everything after the plan up to the float32 down partials in b.dpart.
int joined_decode_products(const void* x, int x_dtype, int per_slot, int slots, const uint32_t* ids, int64_t rows,
                           const exlr8_joined_mxfp4* w, const JoinedDecodeLayout& l, const JoinedDecodeBuffers& b,
                           cudaStream_t s) {
  const int h = w->hidden, m = w->intermediate;
  const int n = static_cast<int>(rows), e = static_cast<int>(w->experts);
  EXLR8_TIMED(EXLR8_KERNEL_PREP, s,
              launch_prep_frag(x, x_dtype, per_slot, slots, ids, n, w->unit, w->unit, w->scale_dtype, h, e, 1,
                               b.frag_gu, s, 0, 1));
  JoinedStreamParams gp;
  memset(&gp, 0, sizeof(gp));
  if (!joined_code_map(&gp.codes, w->gate_up, w->experts * 2 * m, h)) return EXLR8_ERR_CUDA;
  gp.scales = static_cast<const uint8_t*>(w->gate_up_scales);
  gp.frag = b.frag_gu;
  gp.partial = b.gu;
  gp.plan = b.plan;
  gp.counter = 2;
  gp.in_features = h;
  gp.out_features = 2 * m;
  gp.plane_rows = m;
  gp.kb_per_split = l.s1.kb;
  gp.splits = l.s1.count;
  gp.nslots = n;
  EXLR8_TIMED(EXLR8_KERNEL_GATE_UP, s, launch_joined_stream(gp, s));
  EXLR8_TIMED(EXLR8_KERNEL_GATE_FINISH, s,
              launch_gate_finish_frag(b.gu, l.s1.count, ids, n, w->gate_out, w->up_out, w->down_in, w->scale_dtype, m,
                                      e, x_dtype, b.frag_d, nullptr, nullptr, 0, 0, nullptr, s, 1));
  JoinedStreamParams dp;
  memset(&dp, 0, sizeof(dp));
  if (!joined_code_map(&dp.codes, w->down, w->experts * h, m)) return EXLR8_ERR_CUDA;
  dp.scales = static_cast<const uint8_t*>(w->down_scales);
  dp.frag = b.frag_d;
  dp.partial = b.dpart;
  dp.plan = b.plan;
  dp.counter = 3;
  dp.in_features = m;
  dp.out_features = h;
  dp.plane_rows = h;
  dp.kb_per_split = l.s2.kb;
  dp.splits = l.s2.count;
  dp.nslots = n;
  EXLR8_TIMED(EXLR8_KERNEL_DOWN, s, launch_joined_stream(dp, s));
  return EXLR8_OK;
}

// Shared body: everything up to the float32 down products in b.v.
int joined_products(const void* x, int x_dtype, const uint32_t* ids, int64_t tokens, int slots,
                    const exlr8_joined_mxfp4* w, const JoinedLayout& l, const JoinedBuffers& b, cudaStream_t s) {
  const int experts = static_cast<int>(w->experts);
  const int h = w->hidden, m = w->intermediate;
  EXLR8_TIMED(EXLR8_KERNEL_PLAN, s,
              launch_plan(ids, static_cast<int>(l.rows), experts, slots, -1, b.plan, s));
  EXLR8_TIMED(EXLR8_KERNEL_PLAN, s, launch_joined_segments(b.plan, experts, static_cast<int>(l.rows), b.chunks, s));
  EXLR8_TIMED(EXLR8_KERNEL_PREP, s,
              launch_joined_prep(x, x_dtype, w->unit, w->scale_dtype, slots, static_cast<int>(tokens), b.chunks, h,
                                 b.x_hi, b.x_lo, b.x_scales, s));
  ExpertGemmArgs g = {};
  g.weights[0] = w->gate_up;
  g.weight_scales[0] = static_cast<const uint8_t*>(w->gate_up_scales);
  g.x_hi[0] = b.x_hi;
  g.x_lo[0] = b.x_lo;
  g.x_scales[0] = b.x_scales;
  g.chunks = b.chunks;
  g.counter_index = 2;
  g.experts = w->experts;
  g.padded_rows = l.padded;
  g.in_features = h;
  g.out_features = 2 * m;
  g.projections = 1;
  g.paired = 1;
  g.trellis_k = 0;
  g.out = b.gu;
  g.out_stride = 2 * m;
  EXLR8_TIMED(EXLR8_KERNEL_GATE_UP, s, launch_expert_gemm(g, s));
  EXLR8_TIMED(EXLR8_KERNEL_GATE_FINISH, s,
              launch_joined_gate_finish(b.gu, ids, static_cast<int>(l.rows), b.chunks, w->gate_out, w->up_out,
                                        w->down_in, w->scale_dtype, m, x_dtype, b.h_hi, b.h_lo, b.h_scales, s));
  g.weights[0] = w->down;
  g.weight_scales[0] = static_cast<const uint8_t*>(w->down_scales);
  g.x_hi[0] = b.h_hi;
  g.x_lo[0] = b.h_lo;
  g.x_scales[0] = b.h_scales;
  g.counter_index = 3;
  g.in_features = m;
  g.out_features = h;
  g.paired = 0;
  g.out = b.v;
  g.out_stride = h;
  EXLR8_TIMED(EXLR8_KERNEL_DOWN, s, launch_expert_gemm(g, s));
  return EXLR8_OK;
}

}  // namespace

extern "C" {

size_t exlr8_mxfp4_prepared_scales_bytes(int64_t rows, int in_features) {
  if (rows <= 0 || in_features <= 0) return 0;
  return static_cast<size_t>(rows) * static_cast<size_t>(in_features / 32);
}

int exlr8_mxfp4_prepare_scales(const uint8_t* scales, int64_t rows, int in_features, uint8_t* prepared, void* stream) {
  if (rows < 0 || in_features <= 0 || rows % 128 || in_features % 128) return EXLR8_ERR_DIMS;
  if (rows == 0) return EXLR8_OK;
  if (!scales || !prepared) return EXLR8_ERR_ARG;
  return cuda_status(launch_mx_prepare_scales(scales, rows, in_features / 32, prepared, as_stream(stream)));
}

size_t exlr8_joined_workspace(int64_t tokens, int slots, int hidden, int intermediate, int64_t experts) {
  if (!sizes_ok(tokens, slots, hidden, intermediate, experts)) return kBadSize;
  if (tokens <= 0) return 0;
  if (use_joined_stream(tokens)) return joined_decode_layout(tokens * slots, hidden, intermediate, experts).total();
  Carver c(nullptr);
  carve_joined(joined_layout(tokens, slots, experts), hidden, intermediate, experts, c);
  return c.used;
}

int exlr8_joined_slots(const void* x, int x_dtype, const uint32_t* indices, int64_t tokens, int slots,
                       const exlr8_joined_mxfp4* w, void* out, void* workspace, size_t workspace_bytes,
                       void* stream) {
  EXLR8_CHECK(check_joined(w));
  if (!valid_act(x_dtype)) return EXLR8_ERR_DTYPE;
  if (tokens < 0 || slots <= 0) return EXLR8_ERR_ROWS;
  if (tokens == 0) return EXLR8_OK;
  if (slots > 32 || tokens * slots > (int64_t(1) << 24)) return EXLR8_ERR_UNSUPPORTED;
  if (!x || !indices || !out) return EXLR8_ERR_ARG;
  if (!workspace || workspace_bytes < exlr8_joined_workspace(tokens, slots, w->hidden, w->intermediate, w->experts))
    return EXLR8_ERR_WORKSPACE;
  cudaStream_t s = as_stream(stream);
  if (use_joined_stream(tokens)) {
    const int64_t rows = tokens * slots;
    const JoinedDecodeLayout dl = joined_decode_layout(rows, w->hidden, w->intermediate, w->experts);
    Carver dc(workspace);
    const JoinedDecodeBuffers db = carve_joined_decode(dl, rows, w->experts, dc);
    EXLR8_TIMED(EXLR8_KERNEL_PLAN, s,
                launch_plan(indices, static_cast<int>(rows), static_cast<int>(w->experts), slots, -1, db.plan, s));
    EXLR8_CHECK(joined_decode_products(x, x_dtype, 0, slots, indices, rows, w, dl, db, s));
    EXLR8_TIMED(EXLR8_KERNEL_FINISH, s,
                launch_finish(db.dpart, dl.s2.count, nullptr, indices, static_cast<int>(rows), w->down_out,
                              w->scale_dtype, w->hidden, static_cast<int>(w->experts), x_dtype, out, s));
    return EXLR8_OK;
  }
  const JoinedLayout l = joined_layout(tokens, slots, w->experts);
  Carver c(workspace);
  const JoinedBuffers b = carve_joined(l, w->hidden, w->intermediate, w->experts, c);
  EXLR8_CHECK(joined_products(x, x_dtype, indices, tokens, slots, w, l, b, s));
  EXLR8_TIMED(EXLR8_KERNEL_FINISH, s,
              launch_finish(b.v, 1, b.chunks.slot_row, indices, static_cast<int>(l.rows), w->down_out,
                            w->scale_dtype, w->hidden, static_cast<int>(w->experts), x_dtype, out, s));
  return EXLR8_OK;
}

int exlr8_joined_finish(const void* x, int x_dtype, const uint32_t* indices, const float* scores,
                        const void* residual, int64_t tokens, const exlr8_joined_mxfp4* w, void* out,
                        void* workspace, size_t workspace_bytes, void* stream) {
  EXLR8_CHECK(check_joined(w));
  if (!valid_act(x_dtype)) return EXLR8_ERR_DTYPE;
  if (tokens < 0) return EXLR8_ERR_ROWS;
  if (tokens == 0) return EXLR8_OK;
  if (tokens * 9 > (int64_t(1) << 24)) return EXLR8_ERR_UNSUPPORTED;
  if (!x || !indices || !scores || !residual || !out) return EXLR8_ERR_ARG;
  if (!workspace || workspace_bytes < exlr8_joined_workspace(tokens, 9, w->hidden, w->intermediate, w->experts))
    return EXLR8_ERR_WORKSPACE;
  cudaStream_t s = as_stream(stream);
  if (use_joined_stream(tokens)) {
    const int64_t rows = tokens * 9;
    const JoinedDecodeLayout dl = joined_decode_layout(rows, w->hidden, w->intermediate, w->experts);
    Carver dc(workspace);
    const JoinedDecodeBuffers db = carve_joined_decode(dl, rows, w->experts, dc);
    EXLR8_TIMED(EXLR8_KERNEL_PLAN, s,
                launch_plan(indices, static_cast<int>(rows), static_cast<int>(w->experts), 9, -1, db.plan, s));
    EXLR8_CHECK(joined_decode_products(x, x_dtype, 0, 9, indices, rows, w, dl, db, s));
    EXLR8_TIMED(EXLR8_KERNEL_FINISH, s,
                launch_finish_fused(db.dpart, dl.s2.count, nullptr, indices, static_cast<int>(tokens), w->down_out,
                                    w->scale_dtype, w->hidden, static_cast<int>(w->experts), scores, residual,
                                    nullptr, 0, x_dtype, out, s));
    return EXLR8_OK;
  }
  const JoinedLayout l = joined_layout(tokens, 9, w->experts);
  Carver c(workspace);
  const JoinedBuffers b = carve_joined(l, w->hidden, w->intermediate, w->experts, c);
  EXLR8_CHECK(joined_products(x, x_dtype, indices, tokens, 9, w, l, b, s));
  EXLR8_TIMED(EXLR8_KERNEL_FINISH, s,
              launch_joined_finish(b.v, b.chunks.slot_row, indices, static_cast<int>(tokens), w->hidden,
                                   static_cast<int>(w->experts), w->down_out, w->scale_dtype, scores, residual, nullptr,
                                   0, x_dtype, out, s));
  return EXLR8_OK;
}

// Router outputs of the fused layer, carved after the expert buffers.
struct RouterBuffers {
  float* logits;
  uint32_t* ids;
  float* scores;
  void* gemm;
};

size_t router_buffers_bytes(int64_t tokens, int hidden) {
  return align_up(tokens * 256 * sizeof(float)) + align_up(tokens * 9 * sizeof(uint32_t)) +
         align_up(tokens * 8 * sizeof(float)) + align_up(router_gemm_workspace(static_cast<int>(tokens), hidden, EXLR8_DTYPE_F32));
}

RouterBuffers carve_router(int64_t tokens, int hidden, Carver& c) {
  RouterBuffers r;
  r.logits = c.take<float>(tokens * 256 * sizeof(float));
  r.ids = c.take<uint32_t>(tokens * 9 * sizeof(uint32_t));
  r.scores = c.take<float>(tokens * 8 * sizeof(float));
  r.gemm = c.take<char>(router_gemm_workspace(static_cast<int>(tokens), hidden, EXLR8_DTYPE_F32));
  return r;
}

size_t exlr8_joined_moe_layer_workspace(int64_t tokens, int hidden, int intermediate, int64_t experts) {
  if (!sizes_ok(tokens, 9, hidden, intermediate, experts)) return kBadSize;
  if (tokens <= 0) return 0;
  return exlr8_joined_workspace(tokens, 9, hidden, intermediate, experts) + router_buffers_bytes(tokens, hidden);
}

int exlr8_joined_moe_layer(const void* x, int x_dtype, const void* residual, int64_t tokens, const float* gate_weight,
                           const float* bias, const exlr8_joined_mxfp4* w, void* out, uint32_t* indices,
                           float* scores, void* workspace, size_t workspace_bytes, void* stream) {
  EXLR8_CHECK(check_joined(w));
  if (!valid_act(x_dtype)) return EXLR8_ERR_DTYPE;
  if (w->experts < 257) return EXLR8_ERR_ID_RANGE;  // slot 8 routes to expert 256 (the shared expert)
  if (tokens < 0) return EXLR8_ERR_ROWS;
  if (tokens == 0) return EXLR8_OK;
  if (tokens * 9 > (int64_t(1) << 24)) return EXLR8_ERR_UNSUPPORTED;
  if (!x || !residual || !gate_weight || !bias || !out) return EXLR8_ERR_ARG;
  if (!aligned16(gate_weight) || !aligned16(x)) return EXLR8_ERR_ALIGN;
  if (!workspace ||
      workspace_bytes < exlr8_joined_moe_layer_workspace(tokens, w->hidden, w->intermediate, w->experts))
    return EXLR8_ERR_WORKSPACE;
  cudaStream_t s = as_stream(stream);
  if (use_joined_stream(tokens)) {
    // Gate product, then top-8 and the plan, then the decode chain.
    const int64_t rows = tokens * 9;
    const JoinedDecodeLayout dl = joined_decode_layout(rows, w->hidden, w->intermediate, w->experts);
    Carver dc(workspace);
    const JoinedDecodeBuffers db = carve_joined_decode(dl, rows, w->experts, dc);
    const RouterBuffers rb = carve_router(tokens, w->hidden, dc);
    uint32_t* ids = indices ? indices : rb.ids;
    float* sc = scores ? scores : rb.scores;
    EXLR8_TIMED(EXLR8_KERNEL_ROUTER, s,
                launch_gate_logits(x, x_dtype, static_cast<int>(tokens), w->hidden, gate_weight, rb.logits, 256, s));
    EXLR8_TIMED(EXLR8_KERNEL_PLAN, s,
                launch_route_plan(rb.logits, bias, static_cast<int>(tokens), ids, sc, static_cast<int>(w->experts), -1,
                                  db.plan, s));
    EXLR8_CHECK(joined_decode_products(x, x_dtype, 0, 9, ids, rows, w, dl, db, s));
    EXLR8_TIMED(EXLR8_KERNEL_FINISH, s,
                launch_finish_fused(db.dpart, dl.s2.count, nullptr, ids, static_cast<int>(tokens), w->down_out,
                                    w->scale_dtype, w->hidden, static_cast<int>(w->experts), sc, residual, nullptr, 0,
                                    x_dtype, out, s));
    return EXLR8_OK;
  }
  const JoinedLayout l = joined_layout(tokens, 9, w->experts);
  Carver c(workspace);
  const JoinedBuffers b = carve_joined(l, w->hidden, w->intermediate, w->experts, c);
  const RouterBuffers rb = carve_router(tokens, w->hidden, c);
  uint32_t* ids = indices ? indices : rb.ids;
  float* sc = scores ? scores : rb.scores;
  if (tokens >= kRouterGemmMinTokens) {
    EXLR8_TIMED(EXLR8_KERNEL_ROUTER, s,
                launch_router_gemm(x, x_dtype, static_cast<int>(tokens), w->hidden, gate_weight, rb.logits, rb.gemm,
                                   s));
  } else {
    EXLR8_TIMED(EXLR8_KERNEL_ROUTER, s,
                launch_gate_logits(x, x_dtype, static_cast<int>(tokens), w->hidden, gate_weight, rb.logits, 256, s));
  }
  EXLR8_TIMED(EXLR8_KERNEL_ROUTER, s, launch_route(rb.logits, bias, static_cast<int>(tokens), ids, sc, 2.5f, 256u, s));
  EXLR8_CHECK(joined_products(x, x_dtype, ids, tokens, 9, w, l, b, s));
  EXLR8_TIMED(EXLR8_KERNEL_FINISH, s,
              launch_joined_finish(b.v, b.chunks.slot_row, ids, static_cast<int>(tokens), w->hidden,
                                   static_cast<int>(w->experts), w->down_out, w->scale_dtype, sc, residual, nullptr, 0,
                                   x_dtype, out, s));
  return EXLR8_OK;
}

size_t exlr8_router_logits_workspace(int64_t tokens, int hidden, int x_dtype) {
  if (tokens <= 0 || hidden <= 0) return 0;
  return router_gemm_workspace(static_cast<int>(tokens), hidden, x_dtype);
}

int exlr8_router_logits(const void* x, int x_dtype, int64_t tokens, int hidden, const float* gate_weight,
                        float* logits, void* workspace, size_t workspace_bytes, void* stream) {
  if (!valid_act(x_dtype)) return EXLR8_ERR_DTYPE;
  if (tokens < 0 || hidden <= 0 || hidden % 64) return EXLR8_ERR_ARG;
  if (tokens == 0) return EXLR8_OK;
  if (tokens > (int64_t(1) << 24)) return EXLR8_ERR_UNSUPPORTED;
  if (!x || !gate_weight || !logits) return EXLR8_ERR_ARG;
  if (!aligned16(x) || !aligned16(gate_weight) || !aligned16(logits)) return EXLR8_ERR_ALIGN;
  if (!workspace || workspace_bytes < router_gemm_workspace(static_cast<int>(tokens), hidden, x_dtype))
    return EXLR8_ERR_WORKSPACE;
  return cuda_status(launch_router_gemm(x, x_dtype, static_cast<int>(tokens), hidden, gate_weight, logits, workspace,
                                        as_stream(stream)));
}

int exlr8_joined_status(const void* workspace, int64_t tokens, int slots, int64_t experts, int32_t* header_out,
                        void* stream) {
  if (!workspace || !header_out || tokens <= 0 || slots <= 0) return EXLR8_ERR_ARG;
  if (use_joined_stream(tokens)) {
    // Decode chain: no GEMM chunks; [2..3] the stream unit counters, [4] the
    // bounded-wait error bits of the stream kernels (plan header[9]).
    int32_t plan_header[16];
    EXLR8_TRY(cudaMemcpyAsync(plan_header, workspace, sizeof(plan_header), cudaMemcpyDeviceToHost,
                              as_stream(stream)));
    EXLR8_TRY(cudaStreamSynchronize(as_stream(stream)));
    const int32_t out[8] = {0, 0, plan_header[2], plan_header[3], plan_header[9], 0, 0, 0};
    memcpy(header_out, out, sizeof(out));
    return EXLR8_OK;
  }
  const JoinedLayout l = joined_layout(tokens, slots, experts);
  Carver c(const_cast<void*>(workspace));
  // Only the carve offsets are used; hidden/intermediate do not move the header.
  const JoinedBuffers b = carve_joined(l, 128, 128, experts, c);
  EXLR8_TRY(cudaMemcpyAsync(header_out, b.chunks.header, 8 * sizeof(int32_t), cudaMemcpyDeviceToHost,
                            as_stream(stream)));
  return cuda_status(cudaStreamSynchronize(as_stream(stream)));
}

}  // extern "C"
