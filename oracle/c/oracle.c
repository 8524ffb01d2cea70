/*
 * C restatement of the exlr8 routed-MoE layer (TEST INFRASTRUCTURE ONLY).
 *
 * Used by the tests (as a fast checker, itself pinned to the NumPy oracle),
 * by bench.py's cpu_baseline leg and by `bench.py --impl reference` (the
 * reference's operators are Metal-only, so this port is the CPU arm).  The
 * product library never links it.
 *
 * Arithmetic follows, per function, the reference lines cited there
 * (package exlr8 v0.1.21).  The codebook table (the value of every 16-bit
 * trellis state, exlr8/trellis.py:43-50) is passed in by the caller, which
 * takes it from the NumPy oracle.
 *
 * Build: make -C oracle/c   (gcc -O3 -march=x86-64-v3 -fopenmp -shared)
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- typed rounding --------------------------------------------------- */

static inline float f32_from_bits(uint32_t b) {
  float f;
  memcpy(&f, &b, 4);
  return f;
}
static inline uint32_t bits_from_f32(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  return b;
}

/* float -> bfloat16 -> float, nearest even (NaN kept). */
static inline float round_bf16(float v) {
  uint32_t b = bits_from_f32(v);
  if ((b & 0x7f800000u) == 0x7f800000u && (b & 0x007fffffu)) return v;
  b = (b + 0x7fffu + ((b >> 16) & 1u)) & 0xffff0000u;
  return f32_from_bits(b);
}

/* float -> float16 -> float, nearest even (finite range). */
static inline float round_f16(float v) {
  _Float16 h = (_Float16)v;
  return (float)h;
}

/* dtype: 0 = float32, 1 = float16, 2 = bfloat16 */
static inline float round_to(int dtype, float v) {
  if (dtype == 2) return round_bf16(v);
  if (dtype == 1) return round_f16(v);
  return v;
}

/* ---- Hadamard-128 (exlr8/trellis.py:67-75; stage order 1,2,...,64) ----- */

static void hadamard128(float* x) {
  for (int bit = 1; bit < 128; bit <<= 1) {
    for (int i = 0; i < 128; ++i) {
      if (i & bit) continue;
      float a = x[i], b = x[i | bit];
      x[i] = a + b;
      x[i | bit] = a - b;
    }
  }
  const float s = (float)(1.0 / sqrt(128.0));
  for (int i = 0; i < 128; ++i) x[i] *= s;
}

static void hadamard_rows(float* x, int64_t n) {
  for (int64_t b = 0; b < n / 128; ++b) hadamard128(x + b * 128);
}

/* ---- trellis geometry (exlr8/trellis.py:78-102) ------------------------- */

typedef struct {
  int left[256], right[256], shift[256], pos[256]; /* pos = row*16 + col */
} Geometry;

static void make_geometry(int k, Geometry* g) {
  const int words = 8 * k;
  for (int i = 0; i < 256; ++i) {
    int end = (i + 1) * k + 256 * k;
    int last = (end - 1) / 32;
    g->left[i] = (last - 1) % words;
    g->right[i] = last % words;
    g->shift[i] = (last + 1) * 32 - end;
    int lane = i / 8, slot = i % 8;
    int row = (lane % 4) * 2 + (slot & 1) + (slot & 2) * 4;
    int col = lane / 4 + (slot & 4) * 2;
    g->pos[i] = row * 16 + col;
  }
}

static inline int64_t tile_index(int64_t e, int tk, int tn, int it, int ot, int side) {
  if (side == 2) return ((((e * (it / 8) + tk / 8) * (ot / 8) + tn / 8) * 8 + tk % 8) * 8) + tn % 8;
  return ((e * (ot / 8) + tn / 8) * it + tk) * 8 + tn % 8;
}

static inline void decode_tile(const uint32_t* words, const Geometry* g, const float* codebook, float* tile) {
  for (int i = 0; i < 256; ++i) {
    uint64_t merged = ((uint64_t)words[g->left[i]] << 32) | words[g->right[i]];
    tile[g->pos[i]] = codebook[(merged >> g->shift[i]) & 0xffffu];
  }
}

/* inner[rows][out] = xh[rows][in] @ W_e (float32), one expert, rows share it.
 * Output columns are split across threads in 128-wide blocks. */
/* Dot products may use fused multiply-add; every typed step elsewhere
 * rounds exactly as written (the file builds with -ffp-contract=off). */
__attribute__((optimize("fp-contract=fast"))) static void trellis_gemv(const float* xh, int rows, const uint32_t* packed, int64_t expert, int k, int in_f, int out_f,
                         int side, const float* codebook, const Geometry* g, float* inner) {
  const int it = in_f / 16, ot = out_f / 16;
  const int words = 8 * k;
#pragma omp parallel for schedule(static)
  for (int nb = 0; nb < ot / 8; ++nb) {
    float tile[256];
    float acc[8][128];
    for (int r = 0; r < rows; ++r)
      for (int c = 0; c < 128; ++c) acc[r][c] = 0.f;
    for (int tk = 0; tk < it; ++tk) {
      for (int t = 0; t < 8; ++t) {
        const int tn = nb * 8 + t;
        decode_tile(packed + tile_index(expert, tk, tn, it, ot, side) * words, g, codebook, tile);
        for (int r = 0; r < rows; ++r) {
          const float* x = xh + (int64_t)r * in_f + tk * 16;
          float* a = acc[r] + t * 16;
          for (int kr = 0; kr < 16; ++kr) {
            const float xv = x[kr];
            const float* w = tile + kr * 16;
            for (int c = 0; c < 16; ++c) a[c] += xv * w[c];
          }
        }
      }
    }
    for (int r = 0; r < rows; ++r) memcpy(inner + (int64_t)r * out_f + nb * 128, acc[r], 128 * sizeof(float));
  }
}

/* Typed SwiGLU T(T(g*sigmoid(g))*u) (metal/fast_decode_common.metal:40-49). */
static inline float swiglu_typed(int dtype, float gate, float up) {
  float g = round_to(dtype, gate), u = round_to(dtype, up);
  float e = round_to(dtype, expf(fabsf(g)));
  float tail = round_to(dtype, 1.0f / round_to(dtype, 1.0f + e));
  float sig = g < 0.0f ? tail : round_to(dtype, 1.0f - tail);
  return round_to(dtype, round_to(dtype, g * sig) * u);
}

static inline float load_scale(const void* s, int scale_dtype, int64_t i) {
  if (scale_dtype == 0) return ((const float*)s)[i];
  return (float)((const _Float16*)s)[i];
}

/*
 * Fused expert MLP for `rows` rows that all use expert `e` (fast_decode.py:168-205):
 * xh = H(x*in_gate), H(x*in_up); gate/up trellis products; H, out scales,
 * typed SwiGLU, * in_down, H; down product; H, out scale, cast.
 * x: [rows][hidden] floats (already typed values); out: [rows][hidden].
 */
int oracle_expert_mlp_rows(const float* x, int rows, int64_t e, const uint32_t* gate, const uint32_t* up,
                           const uint32_t* down, const void* const* in_scale, const void* const* out_scale,
                           int scale_dtype, int k, int hidden, int inter, int dtype, const float* codebook,
                           float* out) {
  if (rows > 8) return -1;
  Geometry g;
  make_geometry(k, &g);
  float* xg = malloc(sizeof(float) * rows * hidden);
  float* xu = malloc(sizeof(float) * rows * hidden);
  float* gi = malloc(sizeof(float) * rows * inter);
  float* ui = malloc(sizeof(float) * rows * inter);
  float* dx = malloc(sizeof(float) * rows * inter);
  float* di = malloc(sizeof(float) * rows * hidden);
  for (int r = 0; r < rows; ++r) {
    for (int c = 0; c < hidden; ++c) {
      xg[r * hidden + c] = x[(int64_t)r * hidden + c] * load_scale(in_scale[0], scale_dtype, e * hidden + c);
      xu[r * hidden + c] = x[(int64_t)r * hidden + c] * load_scale(in_scale[1], scale_dtype, e * hidden + c);
    }
  }
  hadamard_rows(xg, (int64_t)rows * hidden);
  hadamard_rows(xu, (int64_t)rows * hidden);
  trellis_gemv(xg, rows, gate, e, k, hidden, inter, 1, codebook, &g, gi);
  trellis_gemv(xu, rows, up, e, k, hidden, inter, 1, codebook, &g, ui);
  hadamard_rows(gi, (int64_t)rows * inter);
  hadamard_rows(ui, (int64_t)rows * inter);
  for (int r = 0; r < rows; ++r) {
    for (int c = 0; c < inter; ++c) {
      int64_t si = e * inter + c;
      float gv = gi[r * inter + c] * load_scale(out_scale[0], scale_dtype, si);
      float uv = ui[r * inter + c] * load_scale(out_scale[1], scale_dtype, si);
      dx[r * inter + c] = swiglu_typed(dtype, gv, uv) * load_scale(in_scale[2], scale_dtype, si);
    }
  }
  hadamard_rows(dx, (int64_t)rows * inter);
  trellis_gemv(dx, rows, down, e, k, inter, hidden, 2, codebook, &g, di);
  hadamard_rows(di, (int64_t)rows * hidden);
  for (int r = 0; r < rows; ++r)
    for (int c = 0; c < hidden; ++c)
      out[(int64_t)r * hidden + c] =
          round_to(dtype, di[r * hidden + c] * load_scale(out_scale[2], scale_dtype, e * hidden + c));
  free(xg);
  free(xu);
  free(gi);
  free(ui);
  free(dx);
  free(di);
  return 0;
}

/* Fused router (metal/fast_router.metal:1-42) on float32 logits [rows][256]. */
void oracle_route(const float* logits, const float* bias, int rows, uint32_t* ids, float* scores) {
  for (int r = 0; r < rows; ++r) {
    float original[256], choice[256];
    for (int e = 0; e < 256; ++e) {
      float v = logits[r * 256 + e];
      float y = 1.0f / (1.0f + expf(fabsf(v)));
      original[e] = v < 0 ? y : 1.0f - y;
      choice[e] = original[e] + bias[e];
    }
    float sel[8];
    for (int rank = 0; rank < 8; ++rank) {
      int best = 0;
      for (int e = 1; e < 256; ++e)
        if (choice[e] > choice[best]) best = e;
      ids[r * 9 + rank] = (uint32_t)best;
      sel[rank] = original[best];
      choice[best] = -INFINITY;
    }
    float total = 1e-20f;
    for (int i = 0; i < 8; ++i) total += sel[i];
    for (int i = 0; i < 8; ++i) scores[r * 8 + i] = (sel[i] / total) * 2.5f;
    ids[r * 9 + 8] = 256u;
  }
}

/* x [tokens][hidden] typed values; logits = x @ Wg^T in float32. */
__attribute__((optimize("fp-contract=fast"))) void oracle_router_logits(const float* x, int tokens, int hidden, const float* wg, float* logits) {
#pragma omp parallel for schedule(static)
  for (int e = 0; e < 256; ++e) {
    for (int t = 0; t < tokens; ++t) {
      float acc = 0.f;
      for (int c = 0; c < hidden; ++c) acc += x[(int64_t)t * hidden + c] * wg[(int64_t)e * hidden + c];
      logits[t * 256 + e] = acc;
    }
  }
}

static inline float bf16_to_f32(uint16_t b) { return f32_from_bits((uint32_t)b << 16); }

/* y[t][n] = x[t][:] . W[n][:] with W bf16 [n][kdim], float32 accumulation. */
__attribute__((optimize("fp-contract=fast"))) static void dense_bf16(const float* x, int tokens, const uint16_t* w, int n, int kdim, float* y) {
#pragma omp parallel for schedule(static)
  for (int o = 0; o < n; ++o) {
    for (int t = 0; t < tokens; ++t) {
      float acc = 0.f;
      const uint16_t* row = w + (int64_t)o * kdim;
      const float* xr = x + (int64_t)t * kdim;
      for (int c = 0; c < kdim; ++c) acc += xr[c] * bf16_to_f32(row[c]);
      y[(int64_t)t * n + o] = acc;
    }
  }
}

/* bf16 shared expert: T(T(swiglu(T(x Wg^T), T(x Wu^T))) Wd^T). */
void oracle_shared_bf16(const float* x, int tokens, const uint16_t* wg, const uint16_t* wu, const uint16_t* wd,
                        int hidden, int inter, int dtype, float* out) {
  float* g = malloc(sizeof(float) * tokens * inter);
  float* u = malloc(sizeof(float) * tokens * inter);
  float* h = malloc(sizeof(float) * tokens * inter);
  dense_bf16(x, tokens, wg, inter, hidden, g);
  dense_bf16(x, tokens, wu, inter, hidden, u);
  for (int64_t i = 0; i < (int64_t)tokens * inter; ++i) h[i] = swiglu_typed(dtype, round_to(dtype, g[i]), round_to(dtype, u[i]));
  dense_bf16(h, tokens, wd, hidden, inter, out);
  for (int64_t i = 0; i < (int64_t)tokens * hidden; ++i) out[i] = round_to(dtype, out[i]);
  free(g);
  free(u);
  free(h);
}

/*
 * One MoE layer (model.py:385-418 MoE branch): router, routed experts,
 * shared expert (bf16 when shared_gate != NULL, else trellis matrix 256),
 * combine in the fused-finish order (fast_decode_finish_fused.metal:52-62).
 * out [tokens][hidden]; ids/scores outputs as exlr8_route.
 */
int oracle_moe_layer(const float* x, const float* residual, int tokens, const float* wg, const float* bias,
                     const uint32_t* gate, const uint32_t* up, const uint32_t* down, const void* const* in_scale,
                     const void* const* out_scale, int scale_dtype, int k, int hidden, int inter,
                     const uint16_t* shared_gate, const uint16_t* shared_up, const uint16_t* shared_down, int dtype,
                     const float* codebook, float* out, uint32_t* ids, float* scores, const float* logits_in) {
  /* logits_in (optional, [tokens][256]) replaces the float32 gate product,
   * so that a checker can route from another implementation's logits. */
  float* logits = malloc(sizeof(float) * tokens * 256);
  if (logits_in) memcpy(logits, logits_in, sizeof(float) * tokens * 256);
  else oracle_router_logits(x, tokens, hidden, wg, logits);
  oracle_route(logits, bias, tokens, ids, scores);
  free(logits);
  float* values = malloc(sizeof(float) * (int64_t)tokens * 9 * hidden);
  for (int t = 0; t < tokens; ++t) {
    const int slots = shared_gate ? 8 : 9;
    for (int s = 0; s < slots; ++s) {
      int st = oracle_expert_mlp_rows(x + (int64_t)t * hidden, 1, ids[t * 9 + s], gate, up, down, in_scale, out_scale,
                                      scale_dtype, k, hidden, inter, dtype, codebook,
                                      values + ((int64_t)t * 9 + s) * hidden);
      if (st) return st;
    }
  }
  if (shared_gate) {
    float* sh = malloc(sizeof(float) * (int64_t)tokens * hidden);
    oracle_shared_bf16(x, tokens, shared_gate, shared_up, shared_down, hidden, inter, dtype, sh);
    for (int t = 0; t < tokens; ++t) memcpy(values + ((int64_t)t * 9 + 8) * hidden, sh + (int64_t)t * hidden, sizeof(float) * hidden);
    free(sh);
  }
  for (int t = 0; t < tokens; ++t) {
    for (int c = 0; c < hidden; ++c) {
      float prod[8];
      for (int s = 0; s < 8; ++s) prod[s] = values[((int64_t)t * 9 + s) * hidden + c] * scores[t * 8 + s];
      float total = prod[0] + 0.0f;
      for (int s = 1; s < 8; ++s) total = (prod[s] + 0.0f) + total;
      float routed = round_to(dtype, total);
      float combined = round_to(dtype, routed + round_to(dtype, values[((int64_t)t * 9 + 8) * hidden + c]));
      out[(int64_t)t * hidden + c] = round_to(dtype, residual[(int64_t)t * hidden + c] + combined);
    }
  }
  free(values);
  return 0;
}

int oracle_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
