/*
 * exlr8_b200 -- C ABI of the B200 (sm_100a) routed mixture-of-experts path.
 *
 * Drop-in boundary for the expert-operator surface of the reference package
 * exlr8 (GordoAR/MLXLR8 v0.1.21): exlr8/trellis.py, exlr8/fast_router.py,
 * exlr8/fast_decode.py, exlr8/fast_prefill.py, exlr8/joined_mxfp4.py and the
 * MoE branch of exlr8/model.py (DecoderLayer.__call__).  Every entry point
 * below names the reference function it replaces.
 *
 * Conventions
 *  - All tensor pointers are device pointers owned by the caller.  Nothing
 *    here allocates device memory: calls that need scratch take a caller
 *    workspace whose size comes from the matching *_workspace() query.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream).  Every call
 *    is ordered on that stream and returns without synchronising it.
 *  - Activations are float32, float16 or bfloat16 (EXLR8_DTYPE_*), row-major.
 *    Side-scale vectors are float16 (as in EXLR8 checkpoints) or float32.
 *  - Trellis weights are the EXLR8 "grouped128" packed bytes exactly as
 *    stored in the checkpoint (K*in*out/8 bytes per matrix, matrices
 *    concatenated), 16-byte aligned.
 *  - Return value: EXLR8_OK or a status code; exlr8_status_string() gives
 *    the reference's error message for it.
 */
#ifndef EXLR8_B200_H
#define EXLR8_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EXLR8_ABI_VERSION 1

#define EXLR8_DTYPE_F32 0
#define EXLR8_DTYPE_F16 1
#define EXLR8_DTYPE_BF16 2

enum exlr8_status {
  EXLR8_OK = 0,
  EXLR8_ERR_WIDTH = 1,      /* "EXLR8 trellis width must be 2, 3, or 4"            trellis.py:54-55 */
  EXLR8_ERR_DIMS = 2,       /* "trellis dimensions must be positive multiples of 128" trellis.py:56-57 */
  EXLR8_ERR_SIDE = 3,       /* "sharded_side must be 0, 1, or 2"                    trellis.py:58-59 */
  EXLR8_ERR_BYTES = 4,      /* "packed byte count does not match the trellis dimensions" trellis.py:61-63 */
  EXLR8_ERR_SCALES = 5,     /* "expert side vectors must contain full signed channel scales" trellis.py:183-184 */
  EXLR8_ERR_ROWS = 6,       /* "activation rows do not match the expert indices"   trellis.py:189-190 */
  EXLR8_ERR_WIDTH_X = 7,    /* "activation width does not match in_features"       trellis.py:181-182 */
  EXLR8_ERR_DTYPE = 8,      /* unsupported activation or scale type */
  EXLR8_ERR_ALIGN = 9,      /* a pointer is not 16-byte aligned */
  EXLR8_ERR_WORKSPACE = 10, /* workspace missing or smaller than the *_workspace() size */
  EXLR8_ERR_ARG = 11,       /* null pointer or out-of-range argument */
  EXLR8_ERR_CUDA = 12,      /* a CUDA runtime call failed (see exlr8_last_cuda_error) */
  EXLR8_ERR_ID_RANGE = 13,  /* "Expert IDs must be in 0..256"                       experts.py:158-159 */
  EXLR8_ERR_UNSUPPORTED = 14,
  EXLR8_ERR_STATIC_LIMIT = 15 /* needs more scratch than EXLR8_NOALLOC_SCRATCH_BYTES */
};

/* Library ABI version (EXLR8_ABI_VERSION). */
int exlr8_abi_version(void);

/* Message for a status code (the reference's ValueError text where one exists). */
const char* exlr8_status_string(int status);

/* Text of the last CUDA error seen by this thread ("" if none). */
const char* exlr8_last_cuda_error(void);

/*
 * Trellis expert weights: the `packed` and `scales` dictionaries of
 * exlr8.experts.ExpertLayer (experts.py:97-124).  Index 0/1/2 = gate/up/down.
 * Gate/up matrices are [hidden -> intermediate] stored side 1, down is
 * [intermediate -> hidden] stored side 2.  in_scale[p] is [experts][in],
 * out_scale[p] is [experts][out] (signed channel scales, fp16 or fp32).
 */
typedef struct exlr8_trellis_experts {
  const void* packed[3];
  int64_t packed_bytes[3];
  const void* in_scale[3];
  const void* out_scale[3];
  int scale_dtype;
  int64_t scale_experts; /* rows of every scale matrix */
  int k;                 /* 2, 3 or 4 bits per weight */
  int hidden;
  int intermediate;
} exlr8_trellis_experts;

/*
 * Dense bf16 shared expert (row-major bf16 weights; the reference keeps the
 * shared expert as trellis matrix 256, experts.py:116-124, which
 * exlr8_trellis_experts also supports).  Row-major [out][in] bf16 matrices:
 * gate/up [intermediate][hidden], down [hidden][intermediate].
 */
typedef struct exlr8_dense_expert {
  const void* gate;
  const void* up;
  const void* down;
} exlr8_dense_expert;

/* ---- codec ------------------------------------------------------------ */

/* Value of each 16-bit trellis state (exlr8/trellis.py:43-50 mcg_codebook;
 * metal/fast_decode_common.metal:4-26 exlr8_decode / exlr8_decode2).
 * paired != 0 uses the two-state vector form. values: float32[count]. */
int exlr8_codebook(const uint32_t* states, float* values, int64_t count, int paired, void* stream);

/* Host-only format check (exlr8/trellis.py:53-64 _check_format); writes the
 * matrix count. */
int exlr8_check_format(int64_t packed_bytes, int k, int in_features, int out_features, int sharded_side,
                       int64_t* matrices);

/* Decode matrix `matrix` of a packed buffer to inner weights float32
 * [in][out] (metal/decode.metal; first stage of trellis.py:199-214). */
int exlr8_decode_trellis(const void* packed, int64_t packed_bytes, int64_t matrix, int k, int in_features,
                         int out_features, int sharded_side, float* inner, void* stream);

/* Static hot-expert cache (exlr8/static_cache.py:29-42 expand_static_trellis):
 * the exact E4M3 bytes of every stored tile of a packed buffer, tile order
 * kept, 256 bytes per 16x16 tile (in_features * out_features bytes per
 * matrix); byte p of a tile is the E4M3 code of its codeword p (codeword j
 * of lane l at p = 8 l + j).  packed and out 4-byte aligned. */
int exlr8_expand_static_trellis(const void* packed, int64_t packed_bytes, int k, int in_features, int out_features,
                                int sharded_side, uint8_t* out, void* stream);

/* Public dense matrix float32 [out][in] of a single-matrix buffer
 * (exlr8/trellis.py:199-214 dequantize_trellis). */
size_t exlr8_dequantize_trellis_workspace(int in_features, int out_features);
int exlr8_dequantize_trellis(const void* packed, int64_t packed_bytes, const void* suh, const void* svh,
                             int scale_dtype, int k, int in_features, int out_features, int sharded_side,
                             float* weight, void* workspace, size_t workspace_bytes, void* stream);

/* Normalised Hadamard transform in independent 128-value blocks of each row
 * (exlr8/trellis.py:134-137 _hadamard, mx.hadamard_transform scale
 * 1/sqrt(128); the reference transform hadamard_reference, trellis.py:67-75).
 * x, out: float32 [rows][features], features a multiple of 128; out may be x. */
int exlr8_hadamard128(const float* x, int64_t rows, int features, float* out, void* stream);

/* ---- MXFP4 encode (load time) ------------------------------------------ */

/* MLX quantize(w, mode="mxfp4") (group 32) of float32 rows w [rows][in]:
 * codes uint32 [rows][in / 8] (eight E2M1 codes, low nibble first) and E8M0
 * scales uint8 [rows][in / 32].  Per block of 32: e = round(log2(amax / 6))
 * clamped to [-127, 127], scale code e + 127 (0 for an all-zero block);
 * elements rounded to the nearest E2M1 value of v / 2^e, ties to even,
 * saturating at 6.  The quantisation of dense_trellis.py:97-101
 * encode_mxfp4 and of joined_mxfp4.py:32.  w and codes 16-byte aligned. */
int exlr8_mxfp4_quantize(const float* w, int64_t rows, int in_features, uint32_t* codes, uint8_t* scales,
                         void* stream);

/* JoinedMXFP4 load-time re-encode of one projection of every matrix in a
 * trellis buffer (joined_mxfp4.py:12-47 encode): matrix e decoded to inner
 * [in][out] (decode.metal), rows multiplied by in_scale[e][i] * unit[i] when
 * in_scale is given (the gate/up fold, joined_mxfp4.py:22,30-31: the product
 * formed in the scale dtype, then widened to float32; unit may be NULL for no
 * sign vector), quantised as W^T [out][in] as
 * exlr8_mxfp4_quantize.  Row o of matrix e is written at row
 * e * rows_per_matrix + row_offset + o of codes [.][in / 8] and scales
 * [.][in / 32], so gate (row_offset 0) and up (row_offset = out_features,
 * rows_per_matrix 2 * out_features) land in the joined [E][2m] layout of
 * joined_mxfp4.py:41-45.  packed and codes 16-byte aligned, scales 4-byte
 * aligned. */
int exlr8_mxfp4_encode_trellis(const void* packed, int64_t packed_bytes, int k, int in_features, int out_features,
                               int sharded_side, const void* in_scale, const void* unit, int scale_dtype,
                               uint32_t* codes, uint8_t* scales, int64_t rows_per_matrix, int64_t row_offset,
                               void* stream);

/* ---- router ----------------------------------------------------------- */

/* exlr8/fast_router.py:17-24 route(logits, bias): logits float32 [rows][256],
 * bias float32 [256] -> indices uint32 [rows][9] (slot 8 = 256, the shared
 * expert), scores float32 [rows][8]. */
int exlr8_route(const float* logits, const float* bias, int64_t rows, uint32_t* indices, float* scores,
                void* stream);

/* Gate GEMV + route (model.py:366-371 gate in float32, fast_router.py:34):
 * logits float32 [tokens][256] = x @ gate_weight^T with gate_weight float32
 * [256][hidden]; then exlr8_route. */
int exlr8_router(const void* x, int x_dtype, int64_t tokens, int hidden, const float* gate_weight,
                 const float* bias, float* logits, uint32_t* indices, float* scores, void* stream);

/* ---- dispatch and combine --------------------------------------------- */

/* exlr8/fast_prefill.py:38-46 _plan(indices, experts, block_rows) with the
 * block table of :19-35 _segment_table: ids uint32 [rows] (flattened slot
 * ids) -> order uint32 [rows] (slots sorted by id, stable), sorted_ids uint32
 * [rows] = ids[order], and table uint32 [3][table_capacity]: for each expert
 * e in order, ceil(count_e / block_rows) columns (e, first sorted row,
 * length <= block_rows); *count (device int32) = the number of columns.
 * table_capacity >= min(rows, rows / block_rows + experts), the reference's
 * width; columns past *count are not written.  Ids >= experts follow every
 * valid id in row order and are left out of the table (the reference's
 * argsort orders them by value; they are outside its contract).
 * 1 <= experts <= 1024.  Workspace: exlr8_dispatch_plan_workspace. */
size_t exlr8_dispatch_plan_workspace(int64_t rows, int experts);
int exlr8_dispatch_plan(const uint32_t* ids, int64_t rows, int experts, int block_rows, uint32_t* order,
                        uint32_t* sorted_ids, uint32_t* table, int64_t table_capacity, int32_t* count,
                        void* workspace, size_t workspace_bytes, void* stream);

/* exlr8/model.py:415-418 combine of per-slot expert outputs: values [tokens]
 * [9][hidden] in `dtype` (slot 8 = the shared expert), scores float32
 * [tokens][8], residual and out [tokens][hidden] in `dtype`:
 * out = T(residual + T(T(sum_r values[r] * scores[r]) + values[8])), the
 * routed sum in float32 in the order of
 * metal/fast_decode_finish_fused.metal:52-57 (slot 0, then
 * (slot r + 0) + total for r = 1..7). */
int exlr8_combine(const void* values, const float* scores, const void* residual, int64_t tokens, int hidden,
                  int dtype, void* out, void* stream);

/* ---- trellis expert operators ----------------------------------------- */

/* exlr8/trellis.py:172-196 expert_linear and fast_decode.py:153-165
 * fast_expert_linear: out[t][s] = T(H(H(x*in_s[e]) @ W_e) * out_s[e]) for
 * e = indices[t][s].  x is [tokens][in] (per_slot = 0) or
 * [tokens][slots][in] (per_slot = 1); out is [tokens][slots][out] in x_dtype. */
size_t exlr8_expert_linear_workspace(int64_t tokens, int slots, int in_features, int out_features,
                                     int64_t experts);
int exlr8_expert_linear(const void* x, int x_dtype, int per_slot, const uint32_t* indices, int64_t tokens,
                        int slots, const void* packed, int64_t packed_bytes, const void* in_scale,
                        const void* out_scale, int scale_dtype, int64_t scale_experts, int k, int in_features,
                        int out_features, int sharded_side, void* out, void* workspace, size_t workspace_bytes,
                        void* stream);

/* exlr8/fast_decode.py:208-221 fast_expert_mlp (and experts.py:150-188
 * ExpertLayer.__call__): gate/up, typed SwiGLU, down for every selected
 * slot; out [tokens][slots][hidden] in x_dtype. */
size_t exlr8_expert_mlp_workspace(int64_t tokens, int slots, int hidden, int intermediate, int64_t experts);
int exlr8_expert_mlp(const void* x, int x_dtype, int per_slot, const uint32_t* indices, int64_t tokens, int slots,
                     const exlr8_trellis_experts* experts, void* out, void* workspace, size_t workspace_bytes,
                     void* stream);

/* Static hot-expert cache (exlr8/static_cache.py:91-134 StaticExpertCache,
 * the fp8 / expert_to_slot arguments of fast_expert_mlp): fp8[p] holds the
 * exact E4M3 bytes of the cached experts of projection p (gate, up, down) as
 * exlr8_expand_static_trellis writes them, in_features * out_features bytes
 * per slot, 16-byte aligned; expert_to_slot[e] is the slot of expert e or -1
 * (the uint32 0xFFFFFFFF of the reference). */
typedef struct exlr8_static_cache {
  const uint8_t* fp8[3];
  const int32_t* expert_to_slot;
  int64_t slots;
} exlr8_static_cache;

/* exlr8_expert_mlp with a static cache: the streaming decode reads the cached
 * experts' bytes instead of decoding their codes; outputs are bit-equal to
 * exlr8_expert_mlp (the bytes are the same weights, taken in the same order).
 * Batches on the tensor-core prefill path decode the codes as before. */
int exlr8_expert_mlp_cached(const void* x, int x_dtype, int per_slot, const uint32_t* indices, int64_t tokens,
                            int slots, const exlr8_trellis_experts* experts, const exlr8_static_cache* cache,
                            void* out, void* workspace, size_t workspace_bytes, void* stream);

/* exlr8/fast_decode.py:224-244 compiled_expert_mlp_finish: nine slots per
 * token (eight routed, slot 8 shared), scores float32 [tokens][8], residual
 * [tokens][hidden]; out = residual + T(T(sum_r v_r*score_r) + v_shared).
 * With `shared` non-null the shared expert is the dense bf16 expert and
 * indices[t][8] is ignored. */
size_t exlr8_expert_mlp_finish_workspace(int64_t tokens, int hidden, int intermediate, int64_t experts);
int exlr8_expert_mlp_finish(const void* x, int x_dtype, const uint32_t* indices, const float* scores,
                            const void* residual, int64_t tokens, const exlr8_trellis_experts* experts,
                            const exlr8_dense_expert* shared, void* out, void* workspace, size_t workspace_bytes,
                            void* stream);

/* Whole routed-MoE layer: exlr8/fast_router.py:27-37 compiled_finish and the
 * MoE branch of DecoderLayer.__call__ (model.py:385-418): router gate,
 * route, experts, shared expert, combine with the residual.  indices/scores
 * outputs are optional (may be NULL). */
size_t exlr8_moe_layer_workspace(int64_t tokens, int hidden, int intermediate, int64_t experts);
int exlr8_moe_layer(const void* x, int x_dtype, const void* residual, int64_t tokens, const float* gate_weight,
                    const float* bias, const exlr8_trellis_experts* experts, const exlr8_dense_expert* shared,
                    void* out, uint32_t* indices, float* scores, void* workspace, size_t workspace_bytes,
                    void* stream);

/* ---- pinned host buffers ------------------------------------------------ */

/* Device-accessible address of a buffer the layer's kernels may read or
 * write: device (or managed) memory as is, page-locked host memory
 * (cudaHostAlloc / cudaHostRegister, e.g. torch pin_memory) at its mapped
 * address.  Pageable host memory is refused (EXLR8_ERR_ARG): no kernel ever
 * dereferences it.  Passing a page-locked `out` this way to exlr8_moe_layer
 * makes its finishing kernel write the result to the host directly.  No
 * counterpart in the reference (MLX's unified memory needs no transfer). */
int exlr8_host_device_pointer(const void* ptr, void** device_ptr);

/* A step's two inputs from page-locked host (or device) memory into device
 * buffers, dst0 <- src0 and dst1 <- src1, `bytes` each, by one kernel at the
 * head of the layer's launch chain instead of copy-engine transfers.  Every
 * pointer 16-byte aligned and accepted by exlr8_host_device_pointer (host
 * pointers are translated here); bytes a multiple of 16. */
int exlr8_stage_in(const void* src0, void* dst0, const void* src1, void* dst1, int64_t bytes, void* stream);

/* ---- kernel timing ----------------------------------------------------- */

/* Kernel kinds reported by exlr8_profile_read. */
enum exlr8_kernel_kind {
  EXLR8_KERNEL_ROUTER = 0,       /* gate GEMV + top-8 selection */
  EXLR8_KERNEL_PLAN = 1,         /* expert sort / group table */
  EXLR8_KERNEL_PREP = 2,         /* input transform -> activation fragments */
  EXLR8_KERNEL_GATE_UP = 3,      /* trellis gate/up streaming GEMV */
  EXLR8_KERNEL_GATE_FINISH = 4,  /* gate/up finish -> down fragments */
  EXLR8_KERNEL_DOWN = 5,         /* trellis down streaming GEMV */
  EXLR8_KERNEL_FINISH = 6,       /* output finish / combine */
  EXLR8_KERNEL_DENSE = 7,        /* bf16 shared expert */
  EXLR8_KERNEL_EP_SEND = 8,      /* expert-parallel dispatch over peer memory (includes the wait for peers) */
  EXLR8_KERNEL_EP_RETURN = 9,    /* expert-parallel return over peer memory (includes the wait for owners) */
  EXLR8_KERNEL_EP_COMBINE = 10,  /* expert-parallel weighted combine */
  EXLR8_KERNEL_NORM = 11,        /* residual add + RMS norm */
  EXLR8_KERNEL_KINDS = 12
};

/* Opt-in per-launch timing (the reference prints per-layer seconds with
 * --trace, cli.py:51-63; this times every kernel): while enabled on the
 * calling thread, each launch is bracketed by CUDA events on its stream, up
 * to `capacity` launches.  exlr8_profile_read synchronises the recorded
 * events and returns the launch count and total milliseconds of one kind. */
int exlr8_profile_enable(int enable, int capacity);
int exlr8_profile_read(int kind, int64_t* launches, double* total_ms);

/* ---- tuning ---------------------------------------------------------------- */

/* Block-scaled (MXFP4) grouped GEMMs whose shape allows it (one projection,
 * out_features a multiple of 512) run on SM pairs: a two-CTA cluster issuing
 * M = 256 tcgen05 MMAs (cta_group::2) with the activation tile split between
 * the two SMs.  The one-SM kernel issues the same MMAs in the same order per
 * accumulator.  exlr8_gemm_pair(0 or 1) selects the form for later calls and
 * returns the previous setting; a negative argument only reads it.  Default
 * 1.  No counterpart in the reference. */
int exlr8_gemm_pair(int enable);

/* ---- measurement ---------------------------------------------------------- */

/* Tensor-core peak probe, no counterpart in the reference: the throughput
 * of tcgen05.mma issued back to back on every SM from zero-filled shared
 * tiles (M = 128, N = n, n a multiple of 16 up to 256), timed with CUDA
 * events on `stream` (synchronises it).  kind 0: kind::f16 (bf16 x bf16,
 * float32 accumulation); kind 1: kind::mxf8f6f4.block_scale (E4M3 x E4M3,
 * E8M0 scales), the kind the block-scaled GEMMs issue.  Writes dense
 * TFLOP/s; status (device int32) is non-zero if the bounded wait for the
 * tensor pipe timed out. */
int exlr8_tensor_peak(int kind, int n, int iters, double* tflops, int32_t* status, void* stream);

/* Trellis decode compute probe, no counterpart in the reference: the decode
 * GEMV's inner loop (exact K4 codec + mma.sync) over codes held in shared
 * memory, at the streaming kernel's occupancy, timed with CUDA events on
 * `stream` (synchronises it).  Writes decoded weights per second: the
 * decode's compute ceiling on this GPU, whatever HBM delivers.  `sink` is a
 * device float the kernel writes so that the work is kept. */
int exlr8_codec_peak(int iters, double* weights_per_s, float* sink, void* stream);

/* ---- no-allocation variant ------------------------------------------------ */

/* Size of the fixed device scratch used by exlr8_moe_layer_noalloc. */
#define EXLR8_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)

/* exlr8_moe_layer without a caller workspace.  No counterpart in the
 * reference (exlr8 runs on MLX, which owns all of its memory); it serves
 * hosts that hold device pointers but cannot allocate device memory, such as
 * an FFI caller whose tensors come from another runtime or a server whose
 * memory pool is fixed at start-up.  Scratch is one static device array of
 * EXLR8_NOALLOC_SCRATCH_BYTES inside the library (held on every GPU that
 * loads it until exit); nothing is allocated.  Requests whose
 * exlr8_moe_layer_workspace() exceeds that size return
 * EXLR8_ERR_STATIC_LIMIT: at GLM-5 size up to 5 tokens fit, and the
 * grouped-GEMM path (more than 16 tokens) never fits, so calls through this
 * entry point always take the streaming decode path.  The first call on
 * a device looks up the array's device address; make it before any stream
 * capture.  All calls share the array: calls that overlap on the GPU race
 * and must be serialised by the caller. */
int exlr8_moe_layer_noalloc(const void* x, int x_dtype, const void* residual, int64_t tokens,
                            const float* gate_weight, const float* bias, const exlr8_trellis_experts* experts,
                            const exlr8_dense_expert* shared, void* out, uint32_t* indices, float* scores,
                            void* stream);

/* Device-side id check of the last call that used `workspace`: writes the
 * number of expert ids that were out of range (those slots produce zeros).
 * Synchronises `stream`. */
int exlr8_workspace_bad_ids(const void* workspace, int64_t* bad_ids, void* stream);

/* Dispatch header of the last trellis prefill call (more than 16 tokens)
 * that used `workspace` (sizes as given to that call; slots = 9 for the
 * finish and layer entries): [0] chunks, [1] padded rows, [2..3] GEMM unit
 * counters, [4] GEMM error code (0 = none; non-zero = a bounded wait timed
 * out).  Synchronises `stream`. */
int exlr8_prefill_status(const void* workspace, int64_t tokens, int slots, int intermediate, int64_t experts,
                         int32_t* header, void* stream);

/* ---- expert parallelism ------------------------------------------------------ */

/*
 * The routed experts sharded over `ranks` devices (rank r owns experts
 * [r * experts_per_rank, (r + 1) * experts_per_rank)), each rank holding its
 * own tokens.  One layer on one rank:
 *   exlr8_router                         ids [tokens][9], scores [tokens][8]
 *   exlr8_ep_dispatch                    per-destination rows (below)
 *   all-to-all of send_x and send_meta   (NCCL; the caller's collective)
 *   exlr8_expert_mlp on the received rows (slots = 1, ids = received meta;
 *                                         empty rows carry id -1 -> zeros)
 *   all-to-all of the slot values back
 *   exlr8_shared_expert (or the shared trellis expert) on the local tokens
 *   exlr8_ep_combine                     routed sum + shared + residual
 * The reference runs all experts on one device (model.py:385-418); this
 * split keeps its arithmetic: each slot value is computed exactly as in
 * exlr8_expert_mlp and combined in the same order.
 *
 * exlr8_ep_dispatch: send_x [ranks][capacity][hidden] (x dtype),
 * send_meta int32 [ranks][capacity] (local expert id, -1 = empty row),
 * slot_pos int32 [tokens * 8] (destination * capacity + row, -1 for ids
 * outside [0, ranks * experts_per_rank)), counts int32 [ranks], status int32
 * [1] (slots lost to overflow; capacity = tokens * 8 never overflows).  Rows
 * keep slot order per destination.  hidden * element size % 16 == 0.
 */
int exlr8_ep_dispatch(const uint32_t* indices, int64_t tokens, const void* x, int x_dtype, int hidden, int ranks,
                      int experts_per_rank, int capacity, void* send_x, int32_t* send_meta, int32_t* slot_pos,
                      int32_t* counts, int32_t* status, void* stream);

/* values [ranks * capacity][hidden] (the returned slot values, x dtype),
 * shared [tokens][hidden] typed shared-expert output, residual and out
 * [tokens][hidden]. */
int exlr8_ep_combine(const void* values, int x_dtype, const int32_t* slot_pos, const float* scores, const void* shared,
                     const void* residual, int64_t tokens, int hidden, void* out, void* stream);

/*
 * Peer-memory exchange for the expert-parallel layer (in place of the
 * dispatch + NCCL all-to-all + all-to-all back).  Each rank creates one
 * region (exlr8_ep_peer_create: the one entry point here that allocates
 * device memory, once per layer), publishes its 64-byte CUDA IPC handle to
 * the other ranks (the caller's collective) and opens theirs
 * (exlr8_ep_peer_open).  `peers` is a device array of `ranks` uint64 region
 * addresses as seen from this rank (its own region at [rank]).  Per layer
 * call, on every rank with the same token count:
 *   exlr8_ep_send    routed rows -> owners' regions; waits for the rows
 *                    addressed to this rank (received rows at offset `rows`
 *                    [ranks][C][hidden], local expert ids at `meta` [ranks][C])
 *   exlr8_expert_mlp_shared on those rows (ids -1 = empty)
 *   exlr8_ep_return  values [ranks * C][hidden] -> sources' regions; waits
 *                    for this rank's values (offset `back`), then advances
 *                    the region's epoch
 *   exlr8_ep_combine with values = region + back
 * C = tokens * 8 <= max_capacity <= 4096; ranks <= 64; hidden * element size
 * a multiple of 16.  status int32 [2]: [0] slots lost to overflow, [1] bit 0
 * / bit 1 when a wait for a peer timed out (about 1 s; the call's outputs are
 * then invalid).  Regions start zeroed; all ranks must make the same calls.
 */
size_t exlr8_ep_peer_bytes(int ranks, int max_capacity, int hidden, int x_dtype);
int exlr8_ep_peer_offsets(int ranks, int max_capacity, int hidden, int x_dtype, size_t* meta, size_t* rows,
                          size_t* back);
int exlr8_ep_peer_create(size_t bytes, void** region, void* ipc_handle);
int exlr8_ep_peer_open(const void* ipc_handle, void** region);
int exlr8_ep_peer_close(void* region);
int exlr8_ep_peer_destroy(void* region);
int exlr8_ep_send(const uint32_t* indices, int64_t tokens, const void* x, int x_dtype, int hidden, int ranks, int rank,
                  int experts_per_rank, int max_capacity, const uint64_t* peers, void* region, int32_t* slot_pos,
                  int32_t* status, void* stream);
int exlr8_ep_return(const void* values, int x_dtype, int hidden, int ranks, int rank, int64_t tokens,
                    int max_capacity, const uint64_t* peers, void* region, int32_t* status, void* stream);

/* Measurement helper, no counterpart in the reference: copies `bytes` (a
 * multiple of 16) from local device memory to `dst` with the 16-byte SM
 * stores the exchange kernels use; `dst` may be another GPU's memory mapped
 * through exlr8_ep_peer_open.  Timing it gives the per-direction NVLink
 * store bandwidth that bounds the exchange. */
int exlr8_peer_write(void* dst, const void* src, int64_t bytes, void* stream);

/* Typed output of the dense bf16 shared expert for every token (slot 8 of
 * the combine): T(down(SwiGLU(T(x Wg^T), T(x Wu^T)))). */
/* The owner's half of an expert-parallel layer in one call: the trellis
 * expert MLP over `rows` received rows (x [rows][hidden], one expert id per
 * row in indices [rows]; ids outside [0, experts) give zeros), written to
 * out [rows][hidden] as exlr8_expert_mlp with slots = 1 would, and the bf16
 * shared expert over the rank's own tokens (shared_x [shared_tokens][hidden])
 * written typed to shared_out [shared_tokens][hidden] as exlr8_shared_expert
 * would.  Up to 4096 rows the shared expert's rows stream inside the trellis
 * kernels (bound by their decode arithmetic, not by HBM); beyond that the two
 * run one after the other.  bf16 activations; x, shared_x 16-byte aligned. */
size_t exlr8_expert_mlp_shared_workspace(int64_t rows, int hidden, int intermediate, int64_t experts,
                                         int64_t shared_tokens);
int exlr8_expert_mlp_shared(const void* x, int x_dtype, const uint32_t* indices, int64_t rows,
                            const exlr8_trellis_experts* experts, const void* shared_x, int64_t shared_tokens,
                            const exlr8_dense_expert* shared, void* out, void* shared_out, void* workspace,
                            size_t workspace_bytes, void* stream);

size_t exlr8_shared_expert_workspace(int64_t tokens, int hidden, int intermediate);
int exlr8_shared_expert(const void* x, int x_dtype, int64_t tokens, int hidden, int intermediate,
                        const exlr8_dense_expert* shared, void* out, void* workspace, size_t workspace_bytes,
                        void* stream);

/* ---- joined MXFP4 experts (prefill) -------------------------------------- */

/*
 * Resident four-bit experts of exlr8.joined_mxfp4.JoinedMXFP4
 * (joined_mxfp4.py:137-165): gate and up concatenated per expert as
 * [2 * intermediate][hidden] (gate rows first, joined_mxfp4.py:41-45), down
 * as [hidden][intermediate]; E2M1 values, eight per uint32 word with the low
 * nibble first, and one E8M0 scale per 32 values along the input.  Scales are
 * passed in the layout written by exlr8_mxfp4_prepare_scales.  `unit` is the
 * sign vector folded into the gate/up input (joined_mxfp4.py:13);
 * gate_out/up_out/down_in/down_out are the remaining signed channel scales
 * (scales["gate"][1], scales["up"][1], scales["down"][0], scales["down"][1]).
 * Requirements: hidden % 256 == 0, intermediate % 128 == 0, code buffers
 * 32-byte aligned, scale buffers 16-byte aligned.
 */
typedef struct exlr8_joined_mxfp4 {
  const void* gate_up;        /* uint32 [experts][2 * intermediate][hidden / 8] */
  const void* gate_up_scales; /* prepared E8M0 of [experts * 2 * intermediate][hidden / 32] */
  const void* down;           /* uint32 [experts][hidden][intermediate / 8] */
  const void* down_scales;    /* prepared E8M0 of [experts * hidden][intermediate / 32] */
  const void* unit;           /* [hidden] */
  const void* gate_out;       /* [experts][intermediate] */
  const void* up_out;         /* [experts][intermediate] */
  const void* down_in;        /* [experts][intermediate] */
  const void* down_out;       /* [experts][hidden] */
  int scale_dtype;            /* EXLR8_DTYPE_F16 or EXLR8_DTYPE_F32 (unit and channel scales) */
  int64_t experts;
  int hidden;
  int intermediate;
} exlr8_joined_mxfp4;

/* Re-lay E8M0 scales uint8 [rows][in_features / 32] (MLX quantize output,
 * joined_mxfp4.py:32) for the tensor-core GEMM: 512-byte blocks of 128 rows x
 * 4 scales, byte (r % 32) * 16 + (r % 128 / 32) * 4 + k % 4 of block
 * [r / 128][k / 4].  rows and in_features must be multiples of 128. */
size_t exlr8_mxfp4_prepared_scales_bytes(int64_t rows, int in_features);
int exlr8_mxfp4_prepare_scales(const uint8_t* scales, int64_t rows, int in_features, uint8_t* prepared, void* stream);

/* The joined calls below pick their path by batch size, as the reference's
 * _inner does (joined_mxfp4.py:90-134): up to 16 token rows a streaming
 * MXFP4 GEMV over the selected experts (float16 hi/lo activations, float32
 * accumulation, E8M0 scales applied per 32-block), above it the grouped
 * block-scaled tensor-core GEMM (E4M3 hi/lo activations).  Both read the
 * prepared scales; the stream also reads gate_up / down through 2-D tensor
 * maps (rows of in_features / 2 bytes). */

/* JoinedMXFP4.slots(x, ids) (joined_mxfp4.py:147-150): x [tokens][hidden],
 * indices uint32 [tokens][slots] -> out [tokens][slots][hidden] in x's dtype,
 * each slot T(H(v) * down_out[e]).  Ids outside [0, experts) give zeros.
 * slots <= 32. */
size_t exlr8_joined_workspace(int64_t tokens, int slots, int hidden, int intermediate, int64_t experts);
int exlr8_joined_slots(const void* x, int x_dtype, const uint32_t* indices, int64_t tokens, int slots,
                       const exlr8_joined_mxfp4* weights, void* out, void* workspace, size_t workspace_bytes,
                       void* stream);

/* JoinedMXFP4.finish(x, ids, scores, residual) (joined_mxfp4.py:152-163):
 * nine slots per token (slot 8 = shared expert), routing-weighted combine in
 * the order of metal/fast_decode_finish_fused.metal plus the residual.
 * Workspace: exlr8_joined_workspace(tokens, 9, ...). */
int exlr8_joined_finish(const void* x, int x_dtype, const uint32_t* indices, const float* scores,
                        const void* residual, int64_t tokens, const exlr8_joined_mxfp4* weights, void* out,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Router + JoinedMXFP4.finish: the MoE branch of DecoderLayer
 * (model.py:385-418) on the joined path.  experts must be >= 257 (expert 256
 * is the shared expert).  indices/scores may be null. */
size_t exlr8_joined_moe_layer_workspace(int64_t tokens, int hidden, int intermediate, int64_t experts);
int exlr8_joined_moe_layer(const void* x, int x_dtype, const void* residual, int64_t tokens, const float* gate_weight,
                           const float* bias, const exlr8_joined_mxfp4* weights, void* out, uint32_t* indices,
                           float* scores, void* workspace, size_t workspace_bytes, void* stream);

/* Router gate product on the tensor cores for prefill batches:
 * logits [tokens][256] float32 = x . gate_weight^T (model.py:366-371), as
 * bf16 piece products that sum to the float32 product (the weight split into
 * three bf16 pieces; float16 / float32 x into two / three).  hidden % 64 == 0;
 * x, gate_weight and logits 16-byte aligned.  exlr8_joined_moe_layer uses it
 * from 64 tokens up. */
size_t exlr8_router_logits_workspace(int64_t tokens, int hidden, int x_dtype);
int exlr8_router_logits(const void* x, int x_dtype, int64_t tokens, int hidden, const float* gate_weight,
                        float* logits, void* workspace, size_t workspace_bytes, void* stream);

/* Residual add + RMS norm in front of each MoE block (model.py:373-384,
 * the fused form of exlr8/fast_norm.py residual_rms_pair): per row,
 *   h   = T(x + residual)                      (h = x when residual is null)
 *   out = T(w * T(h * rsqrt(sum(h * h) / hidden + eps)))
 * with the sum of squares in float32; h_out (nullable) receives h.  x,
 * residual, h_out and out [rows][hidden] in x_dtype; w [hidden] in x_dtype. */
int exlr8_residual_rms_norm(const void* x, const void* residual, const void* weight, int x_dtype, int64_t rows,
                            int hidden, float eps, void* h_out, void* out, void* stream);

/* Dispatch header of the last joined call that used `workspace` (sizes as
 * given to that call): [0] chunks, [1] padded rows, [2..3] GEMM unit counters,
 * [4] GEMM error code (0 = none; non-zero = a bounded wait timed out).
 * Synchronises `stream`. */
int exlr8_joined_status(const void* workspace, int64_t tokens, int slots, int64_t experts, int32_t* header,
                        void* stream);

#ifdef __cplusplus
}
#endif

#endif /* EXLR8_B200_H */
