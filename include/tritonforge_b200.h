/*
 * tritonforge_b200 -- C ABI of the B200 (sm_100a) int4 decode/prefill kernels.
 *
 * Every entry point takes caller-owned device pointers, plain sizes and a CUDA
 * stream (passed as `void*`, a `cudaStream_t`), launches asynchronously on that
 * stream, never allocates and never synchronises. Each returns a tf_status
 * code; the text of the last failure on the calling thread is available from
 * tf_last_error_message().
 *
 * Weight format (identical to the reference's `src/tritonforge/quant.py`):
 *   packed  uint8 [K_pad/2, N]   packed[j, n] = code(2j, n) | code(2j+1, n) << 4
 *   scales  half  [K_pad/g, N]   fp16 or bf16 (`param_dtype`)
 *   zeros   half  [K_pad/g, N]   integral values 0..15, same dtype as scales
 *   W[k, n] = (code(k, n) - zeros[k/g, n]) * scales[k/g, n]
 * All 2-D arrays are row-major and contiguous unless a leading dimension is
 * passed.
 */
#ifndef TRITONFORGE_B200_H
#define TRITONFORGE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes and element types ---------------------------------- */
typedef enum tf_status {
  TF_OK = 0,
  TF_ERR_BAD_SHAPE = 1,   /* shapes inconsistent (reference raises ValueError) */
  TF_ERR_BAD_DTYPE = 2,   /* unsupported element type (reference: ValueError)  */
  TF_ERR_UNALIGNED = 3,   /* pointer/stride alignment the kernel needs is missing */
  TF_ERR_CUDA = 4,        /* a CUDA runtime call or launch failed              */
  TF_ERR_TIMEOUT = 5,     /* a bounded device-side wait expired                 */
  TF_ERR_WORKSPACE = 6,   /* workspace missing or smaller than required         */
  TF_ERR_BAD_ARG = 7,     /* other invalid argument (null pointer, bad group)   */
  TF_ERR_UNSUPPORTED = 8  /* valid request that this build cannot run           */
} tf_status;

typedef enum tf_dtype { TF_F16 = 0, TF_BF16 = 1, TF_F32 = 2, TF_U8 = 3 } tf_dtype;

/* Regime selector for tf_qlinear_ex. */
typedef enum tf_regime {
  TF_REGIME_AUTO = 0,  /* pick by M and shape (what tf_qlinear does)            */
  TF_REGIME_GEMV = 1,  /* decode: TMA-streamed split-K int4 GEMV, M <= 32       */
  TF_REGIME_GEMM = 2,  /* prefill: TMA + tcgen05/TMEM GEMM, dequant once in smem */
  TF_REGIME_SIMT = 3   /* any shape/alignment: CUDA-core kernel                  */
} tf_regime;

/* ABI version of this header (bumped on any signature change). */
int tf_abi_version(void);
/* Static text for a status code. */
const char* tf_status_string(int status);
/* Thread-local detail of the last failure reported by this library. */
const char* tf_last_error_message(void);

/* ---- quantized_linear -------------------------------------------------
 * Replaces `tritonforge.kernels.quantized_linear`
 * (reference src/tritonforge/kernels/dequant_gemm.py:151-210, validation
 * :121-148, Triton kernel :39-113):
 *   out[M, N] = x[M, K] @ dequant(packed)[:K] (+ bias)
 * x holds M rows of K values with row stride `ldx` elements; columns
 * K..K_pad-1 are treated as zero (the reference zero-pads x, :166-167).
 * Weights are dequantised and rounded to the activation dtype, products are
 * accumulated in fp32, the result is rounded to the activation dtype and the
 * bias (any of fp16/bf16/fp32, or NULL) is added and rounded again -- the
 * rounding points of the reference oracle (reference.py:21-36).
 * `workspace` must hold at least 256 bytes and be zeroed once before its
 * first use; tf_qlinear_workspace_bytes(...) is the size for the fastest
 * schedule (above 128 rows the tcgen05 GEMM splits tiles between CTAs when
 * its tiles would leave SMs idle, and keeps partial tiles there; with less
 * it runs one tile per CTA). Word 0 is the error word of the kernels' bounded
 * waits: a wait that gives up (1 s) sets a bit there and the call still
 * returns TF_OK, so read it with tf_workspace_error; it stays set until the
 * caller clears it. Calls that share a workspace must be ordered on one
 * stream.
 */
size_t tf_qlinear_workspace_bytes(int64_t M, int64_t N, int64_t K_pad, int32_t group_size);

/* The tcgen05 GEMM's schedule for an M x N x K problem given a workspace of
 * tf_qlinear_workspace_bytes: the number of CTAs of its stream-K schedule
 * (contiguous ranges of (tile, 64-k chunk) units, a split tile finished by
 * the last CTA to arrive, which adds the pieces in k order), or 0 when it
 * runs one 256 x 256 tile per CTA. No reference counterpart (the reference
 * launches one Triton program per output tile, dequant_gemm.py:174-175). */
int tf_qlinear_gemm_stream_k_grid(int64_t M, int64_t N, int64_t K);

int tf_qlinear(const void* x, int64_t ldx, int x_dtype,
               const uint8_t* packed, const void* scales, const void* zeros, int param_dtype,
               const void* bias, int bias_dtype,
               void* out, int64_t ldo,
               int64_t M, int64_t N, int64_t K, int64_t K_pad, int32_t group_size,
               void* workspace, size_t workspace_bytes, void* stream);

/* Same as tf_qlinear with an explicit regime (tf_regime); used by tests and
 * benchmarks to exercise each kernel. AUTO behaves exactly like tf_qlinear. */
int tf_qlinear_ex(const void* x, int64_t ldx, int x_dtype,
                  const uint8_t* packed, const void* scales, const void* zeros, int param_dtype,
                  const void* bias, int bias_dtype,
                  void* out, int64_t ldo,
                  int64_t M, int64_t N, int64_t K, int64_t K_pad, int32_t group_size,
                  void* workspace, size_t workspace_bytes, int regime, void* stream);

/* tf_qlinear for callers that cannot allocate device memory (for example a
 * plugin inside a framework whose allocator owns all device memory, or a host
 * runtime behind an FFI with no CUDA allocator). No counterpart in the
 * reference. The scratch comes from a 4 KiB array built into the library
 * instead of a caller workspace; problems that need more are rejected with
 * TF_ERR_WORKSPACE. The first call on each device sets the array up (looks up
 * its device address, clears it on `stream`), so make it before any stream
 * capture. All calls share the array: calls that can overlap on the GPU race,
 * order them on one stream. Allocates nothing. A bounded device wait that
 * gives up does not change the return code: read it with
 * tf_qlinear_noalloc_error. */
int tf_qlinear_noalloc(const void* x, int64_t ldx, int x_dtype,
                       const uint8_t* packed, const void* scales, const void* zeros, int param_dtype,
                       const void* bias, int bias_dtype,
                       void* out, int64_t ldo,
                       int64_t M, int64_t N, int64_t K, int64_t K_pad, int32_t group_size,
                       void* stream);

/* The error word of tf_qlinear_noalloc's built-in scratch on the current
 * device (no counterpart in the reference): a bounded device-side wait of any
 * tf_qlinear_noalloc call that gave up set a bit there, while that call still
 * returned TF_OK. Copies the word to *error_out (blocking on `stream`), clears
 * it on the device when `clear` is non-zero and the word was set, and returns
 * TF_ERR_TIMEOUT when it was set, TF_OK otherwise. Order it after the calls it
 * should cover (same stream). Allocates nothing. */
int tf_qlinear_noalloc_error(int* error_out, int clear, void* stream);

/* Reads the device-side error word of a workspace (blocking copy on `stream`):
 * 0 when every kernel that used it completed its bounded waits. */
int tf_workspace_error(const void* workspace, int* error_out, void* stream);

/* ---- rmsnorm_residual / rmsnorm ---------------------------------------
 * Replaces `tritonforge.kernels.rmsnorm_residual` and `.rmsnorm`
 * (reference src/tritonforge/kernels/rmsnorm_residual.py:141-161, launch
 * :85-138, kernel :26-79; oracle reference.py:39-50):
 *   summed = x + residual                     (rounded to dtype)
 *   normed = (summed * rsqrt(mean(summed^2) + eps)) -> dtype, * weight -> dtype
 * `residual == NULL` gives plain RMSNorm (then `summed` must be NULL);
 * `summed == NULL` skips writing the sum. x, residual, normed and summed are
 * [M, N] contiguous of `dtype`; weight is [N] of `w_dtype`.
 */
int tf_rmsnorm_residual(const void* x, const void* residual, const void* weight, int w_dtype,
                        void* normed, void* summed, int64_t M, int64_t N, float eps,
                        int dtype, void* stream);

/* ---- swiglu -------------------------------------------------------------
 * Replaces `tritonforge.kernels.swiglu` (reference src/tritonforge/kernels/
 * swiglu.py:36-57, kernel :21-30; oracle reference.py:53-57):
 *   out = (gate * sigmoid(gate)) * up, in fp32, rounded once to dtype,
 * over `numel` contiguous elements.
 */
int tf_swiglu(const void* gate, const void* up, void* out, int64_t numel, int dtype,
              void* stream);

/* ---- quantizer and format helpers ---------------------------------------
 * tf_quantize_int4 replaces `tritonforge.quant.quantize_int4_group`
 * (reference src/tritonforge/quant.py:29-63), bit-exact: w is the fp32
 * [N, K] weight (nn.Linear layout); outputs are packed [K_pad/2, N] and
 * scales/zeros [K_pad/g, N] of `param_dtype`, K_pad = ceil(K/g)*g.
 * tf_dequantize_int4 replaces `quant.dequantize_int4` (quant.py:90-105):
 * out [K_pad, N] of `out_dtype` = ((code - zero) * scale) in fp32, rounded.
 * tf_unpack_int4 replaces `quant.unpack_int4` (quant.py:66-74): codes
 * uint8 [K_pad, N].
 */
int tf_quantize_int4(const float* w, int64_t N, int64_t K, int32_t group_size,
                     uint8_t* packed, void* scales, void* zeros, int param_dtype,
                     void* stream);

int tf_dequantize_int4(const uint8_t* packed, const void* scales, const void* zeros,
                       int param_dtype, void* out, int out_dtype,
                       int64_t K_pad, int64_t N, int32_t group_size, void* stream);

int tf_unpack_int4(const uint8_t* packed, uint8_t* codes, int64_t K_pad, int64_t N,
                   void* stream);

/* ---- decode-loop support (Qwen2-shaped engine) ---------------------------
 * No reference counterpart as kernels: the reference runs these steps through
 * transformers' Qwen2 code (rotary embedding, SDPA attention, DynamicCache;
 * reference src/tritonforge/integration/qwen.py:124-152 calls into them).
 * They exist so a whole decode step, with positions and lengths read from
 * device memory, can be captured in one CUDA graph.
 *
 * tf_rope_kv_append: qkv rows [B, (hq + 2*hkv) * D] (row stride ld_qkv
 * elements) -> q_out [B, hq, D] rotated; k rotated and v appended to the
 * caches [B, hkv, t_max, D] at position *pos (device int). cos/sin tables are
 * [t_max, D] in the model dtype; rounding as transformers' apply_rotary_pos_emb.
 */
int tf_rope_kv_append(const void* qkv, int64_t ld_qkv, void* q_out, const void* cos_table,
                      const void* sin_table, void* k_cache, void* v_cache, const int* pos,
                      int64_t B, int32_t hq, int32_t hkv, int32_t head_dim, int64_t t_max, int dtype,
                      void* stream);

/* ---- prompt prefill support ---------------------------------------------
 * No reference counterpart as kernels: the reference's prefill runs through
 * transformers (rotary embedding, DynamicCache, and `_mlp_forward`'s swiglu
 * on separate gate/up outputs; reference integration/qwen.py:118-144).
 *
 * tf_rope_kv_prefill: t0 rows of the fused q|k|v projection [t0, (hq +
 * 2*hkv) * D] (row stride ld_qkv elements) -> q_out rows [t0, hq * D] (row
 * stride ld_q) rotated, in place when q_out == qkv and ld_q == ld_qkv; k
 * rotated and v copied into positions 0..t0-1 of one sequence's caches
 * [hkv, t_max, D]. cos/sin tables [>= t0, D] in the model dtype; rounding as
 * tf_rope_kv_append. D a multiple of 16; pointers and rows 16-byte aligned.
 */
int tf_rope_kv_prefill(const void* qkv, int64_t ld_qkv, void* q_out, int64_t ld_q, const void* cos_table,
                       const void* sin_table, void* k_cache, void* v_cache, int64_t t0, int32_t hq,
                       int32_t hkv, int32_t head_dim, int64_t t_max, int dtype, void* stream);

/* tf_swiglu_gu: act [M, inter] = silu(gate) * up from the fused gate|up
 * projection [M, 2*inter] (row stride ld_gu) whose columns interleave gate
 * and up per 64 (gate j at 128 (j / 64) + j % 64, up 64 further); rounding
 * as tf_swiglu. inter a multiple of 64; pointers and rows 16-byte aligned. */
int tf_swiglu_gu(const void* gu, int64_t ld_gu, void* act, int64_t ld_act, int64_t M, int64_t inter,
                 int dtype, void* stream);

/* tf_decode_attention: out [B, hq, D] = softmax(q k^T * scale) v over the
 * first *len (device int) cached positions; grouped-query (hq % hkv == 0),
 * D in {64, 128}; fp32 scores/softmax/accumulation, one rounding. */
int tf_decode_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                        const int* len, int64_t B, int32_t hq, int32_t hkv, int32_t head_dim,
                        int64_t t_max, float scale, int dtype, void* stream);

/* tf_decode_attention_rope: tf_rope_kv_append and tf_decode_attention in one
 * launch (same results bit for bit): q and the new key are rotated from the
 * q|k|v projection rows qkv [B, ld_qkv] at position pos[0], the key and value
 * are appended to the caches at pos[0], and attention runs over pos[1]
 * (= pos[0] + 1) cached positions. */
int tf_decode_attention_rope(const void* qkv, int64_t ld_qkv, const void* cos_table, const void* sin_table,
                             void* k_cache, void* v_cache, const int* pos, void* out, int64_t B, int32_t hq,
                             int32_t hkv, int32_t head_dim, int64_t t_max, float scale, int dtype, void* stream);

/* tf_swiglu_strided: SwiGLU over row-strided gate/up views (e.g. the two
 * halves of a fused gate|up projection), same math as tf_swiglu. */
int tf_swiglu_strided(const void* gate, const void* up, void* out, int64_t M, int64_t N, int64_t ldg,
                      int64_t ldu, int64_t ldo, int dtype, void* stream);

/* tf_qlinear_swiglu: the gate and up projections of a SwiGLU MLP in one
 * int4 linear (no reference counterpart: the reference runs quantized_linear
 * twice and then swiglu, integration/qwen.py:118-121). The N = 2 I weight
 * columns are interleaved per 128-column block as [gate 64 | up 64]; out
 * [M, I] (row stride ldo) = round(silu(g) * u) with g = round(x @ Wg),
 * u = round(x @ Wu) in x's dtype (no bias). The regimes of tf_qlinear: the
 * decode GEMV up to 32 rows, 32-row chunks of it up to 128, above that the
 * tcgen05 GEMM with the SwiGLU in its epilogue (the [M, N] projection is
 * never written). N % 128 == 0. Workspace as tf_qlinear. */
int tf_qlinear_swiglu(const void* x, int64_t ldx, int x_dtype, const uint8_t* packed, const void* scales,
                      const void* zeros, int param_dtype, void* out, int64_t ldo, int64_t M, int64_t N, int64_t K,
                      int64_t K_pad, int32_t group_size, void* workspace, size_t workspace_bytes, void* stream);

/* tf_repack_int4_cm: the reference's packed int4 weights [K_pad/2, N]
 * (K-major, low nibble = even k; reference src/tritonforge/quant.py:25-63)
 * -> the tiled column-major layout of the decode kernels: 16 KiB tiles
 * [ceil(N/256)][K_pad/128][256 columns][64 B]. In a tile row (one output
 * column, 128 k) 32-bit word w holds k = 8w..8w+7 with nibble p = k 8w+2p and
 * nibble p+4 = k 8w+2p+1 (p = 0..3), and 16-byte chunk c is stored at position
 * c ^ ((row / 2) & 3). Columns >= N are zero. Same codes, another order: a
 * decode engine converts its weights once (no reference counterpart).
 * K_pad % 128 == 0; packed_cm holds tf_int4_cm_bytes(N, K_pad) bytes and is
 * 16-byte aligned. */
size_t tf_int4_cm_bytes(int64_t N, int64_t K_pad);
int tf_repack_int4_cm(const uint8_t* packed, uint8_t* packed_cm, int64_t N, int64_t K_pad, void* stream);

/* tf_qlinear_cm: tf_qlinear on tiled column-major weights (tf_repack_int4_cm),
 * decode regime: any M >= 1 (one launch per 64 rows, each streaming the
 * weights once), x and scales/zeros of the same 16-bit type,
 * K % 64 == 0, group_size % 128 == 0, N % 16 == 0, 16-byte aligned operands.
 * Same outputs as tf_qlinear within the floating-point contract (weights
 * dequantised bit-exactly, fp32 accumulation, the same roundings); computed
 * on the tcgen05 tensor cores (weights on the MMA's N = 256). Replaces
 * quantized_linear (reference src/tritonforge/kernels/dequant_gemm.py:121-210)
 * inside the decode engine. Long k ranges are split over a thread-block
 * cluster whose CTAs add their partial tiles through distributed shared
 * memory in rank order (results do not depend on timing). `workspace` holds
 * tf_qlinear_cm_workspace_bytes(M, N, K_pad) bytes (the error word of the
 * bounded waits), zeroed before its first use. */
size_t tf_qlinear_cm_workspace_bytes(int64_t M, int64_t N, int64_t K_pad);
int tf_qlinear_cm(const void* x, int64_t ldx, int x_dtype, const uint8_t* packed_cm, const void* scales,
                  const void* zeros, int param_dtype, const void* bias, int bias_dtype, void* out, int64_t ldo,
                  int64_t M, int64_t N, int64_t K, int64_t K_pad, int32_t group_size, void* workspace,
                  size_t workspace_bytes, void* stream);

/* tf_qlinear_cm_swiglu: tf_qlinear_swiglu on tiled column-major weights
 * (gate/up interleaved per 64 columns before the repack); constraints and
 * workspace of tf_qlinear_cm, N % 128 == 0. */
int tf_qlinear_cm_swiglu(const void* x, int64_t ldx, int x_dtype, const uint8_t* packed_cm, const void* scales,
                         const void* zeros, int param_dtype, void* out, int64_t ldo, int64_t M, int64_t N, int64_t K,
                         int64_t K_pad, int32_t group_size, void* workspace, size_t workspace_bytes, void* stream);

/* tf_qlinear_partial / tf_qlinear_cm_partial: the int4 linear of a
 * row-parallel tensor-parallel projection (o_proj, down_proj sharded on K):
 * out[M, N] (fp32, row stride ldo) = x @ W with the fp32 sums stored
 * unrounded and no bias. Each rank's partial is then added across ranks in
 * fp32 and rounded once (tf_allreduce_rmsnorm_residual with TF_F32 partials),
 * so a tensor-parallel layer rounds where the single-GPU layer rounds (no
 * reference counterpart: the reference is single-GPU; replaces the sharded
 * half of quantized_linear, reference src/tritonforge/kernels/
 * dequant_gemm.py:151-210). tf_qlinear_partial takes the reference's packed
 * layout (any regime), tf_qlinear_cm_partial the tiled column-major layout
 * (constraints of tf_qlinear_cm). Workspace as tf_qlinear. */
int tf_qlinear_partial(const void* x, int64_t ldx, int x_dtype, const uint8_t* packed, const void* scales,
                       const void* zeros, int param_dtype, float* out, int64_t ldo, int64_t M, int64_t N, int64_t K,
                       int64_t K_pad, int32_t group_size, void* workspace, size_t workspace_bytes, void* stream);
int tf_qlinear_cm_partial(const void* x, int64_t ldx, int x_dtype, const uint8_t* packed_cm, const void* scales,
                          const void* zeros, int param_dtype, float* out, int64_t ldo, int64_t M, int64_t N,
                          int64_t K, int64_t K_pad, int32_t group_size, void* workspace, size_t workspace_bytes,
                          void* stream);

/* tf_allreduce_rmsnorm_residual: tensor-parallel all-reduce of row-parallel
 * partial sums fused with residual-add + RMSNorm (no reference counterpart:
 * the reference is single-GPU; it replaces an all-reduce followed by
 * rmsnorm_residual, reference integration/qwen.py:145-150 / kernels
 * rmsnorm_residual.py:141-151).
 *   peer_buffers[r]      device address of rank r's symmetric buffer (device array)
 *   peer_signal_pads[r]  device address of rank r's signal pad of u32 slots (device array)
 *   offset_bytes         this call's partial tile [M, N] inside every buffer
 *   pad_slot             first signal-pad slot used (pad_slot .. pad_slot + world - 1)
 *   counters             this rank's device u32[2], zeroed once before the first call
 *   partial_dtype        TF_F32 (the unrounded sums of tf_qlinear_partial;
 *                        offset_bytes % 32 == 0) or `dtype`
 * Computes o = round(sum_r partial_r) (fp32 sum in rank order, identical on
 * every rank), summed = round(o + residual), normed = round(round(summed *
 * rstd) * weight). Waits for the peers' signals at most 1 s; on expiry sets
 * bit 16 of *error_word and still returns TF_OK (read the word to check).
 * N % 8 == 0, N <= 16384. */
int tf_allreduce_rmsnorm_residual(const uint64_t* peer_buffers, const uint64_t* peer_signal_pads,
                                  int64_t offset_bytes, int32_t pad_slot, int32_t rank, int32_t world,
                                  uint32_t* counters, const void* residual, const void* weight, int w_dtype,
                                  void* normed, void* summed, int64_t M, int64_t N, float eps, int dtype,
                                  int partial_dtype, int* error_word, void* stream);

/* The decode step's head (no reference counterpart: the reference patches only
 * the decoder layers, integration/qwen.py:155-185, and leaves the embedding
 * lookup, the lm_head matmul and the greedy argmax to transformers).
 *
 * tf_embed_gather: x[b, :] = embed[tokens[b], :] for b < B, and the same rows
 * into `res` when it is not null (the residual stream starts as the
 * embedding). tokens are int64; a token outside [0, V) gives a zero row. Rows
 * are whole 16-byte chunks, pointers 16-byte aligned; dtype TF_F16, TF_BF16
 * or TF_F32. */
int tf_embed_gather(const void* embed, int64_t lde, const int64_t* tokens, void* x, int64_t ldx, void* res,
                    int64_t ldr, int64_t V, int64_t H, int64_t B, int32_t dtype, void* stream);

/* tf_lm_head_argmax: logits[b, v] = round(sum_k x[b, k] * w[v, k]) for a
 * [V, H] weight (ldw elements per row), B <= 64 rows of x, fp32 accumulation
 * and one rounding to `dtype` (TF_F16 or TF_BF16), and the greedy argmax over
 * the rounded logits with ties to the smallest id (torch.argmax's first
 * maximum). Outputs, each optional (at least one given): `logits` [B, ldl];
 * `tokens` [B] int64 ids; `best` [B, 2] fp32 (best logit, global id) for a
 * vocabulary slice whose ids start at v0 (vocabulary-parallel tensor
 * parallelism, then tf_best_of_ranks); ids are reported as id + v0. `pos`
 * (n_pos int32 counters, may be null) is advanced by one once the tokens are
 * written. H % 128 == 0; ldx, ldw multiples of 8; x, w 16-byte aligned.
 * `workspace` holds tf_lm_head_workspace_bytes(B) zeroed bytes (the error
 * word, as tf_qlinear, then a counter the kernel leaves zeroed and per-CTA
 * partial results). */
size_t tf_lm_head_workspace_bytes(int64_t B);
int tf_lm_head_argmax(const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t V, int64_t H, int64_t B,
                      int32_t dtype, void* logits, int64_t ldl, int64_t* tokens, float* best, int64_t v0,
                      int32_t* pos, int32_t n_pos, void* workspace, size_t workspace_bytes, void* stream);

/* tf_best_of_ranks: greedy ids [B] (int64) from every rank's (best logit,
 * global id) pairs [world][B][2] (fp32), ranks holding consecutive vocabulary
 * slices in rank order: the largest logit wins, ties to the lowest rank. */
int tf_best_of_ranks(const float* all_best, int64_t* tokens, int32_t world, int64_t B, void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* TRITONFORGE_B200_H */
