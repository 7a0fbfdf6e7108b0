/*
 * b200dec.h -- C ABI of the B200 (sm_100a) decode-step hot path.
 *
 * The reference project (ios_kernels, a Metal/Swift LLM runtime) has no in-process operator
 * API: its decode kernels are private to the Swift Engine and bound through Metal buffer
 * slots.  Each entry point below replaces one of those kernels or host helpers; the comment
 * above it names the reference lines it stands in for (LK = ios_kernels/kernels/
 * unsloth__Llama-3.2-1B-Instruct/kernel_metal_f16_20261024-1620, GK = ios_kernels/kernels/
 * google__gemma-4-E2B-it/kernel_metal_f16_20261025-1225).
 *
 * Conventions
 *  - Every pointer argument is DEVICE memory unless the comment says "host".  The caller owns
 *    all memory; no entry point allocates, except b2d_decoder_create (explicit handle).
 *  - Every call is stream-ordered on `stream` (a cudaStream_t; NULL = legacy default stream)
 *    and returns an int status: 0 = B2D_OK, otherwise a B2D_ERR_* code.  Nothing aborts or
 *    traps; b2d_status_string() names the code.  A CUDA launch error is returned as
 *    B2D_ERR_CUDA and its cudaError_t is kept in b2d_last_cuda_error().
 *  - Matrices are row-major [M, K] (out_features x in_features), like the reference's weights
 *    file (LK/convert_weights.py:60-72).  Activations are [batch, K] with a row stride.
 *  - Vector loads are 16 bytes wide: weight rows and activation rows must start on 16-byte
 *    boundaries (B2D_ERR_ALIGN otherwise).
 *
 * Extension formats (no reference code exists; BASELINE config 3/4):
 *  - Q8_32: int8 q[M, K] in [-127, 127] + fp16 scales[M, K/32];  w = float(s) * q  (exact).
 *  - Q4_32: uint8 q[M, K/2], element 2j in the low nibble of byte j, 2j+1 in the high nibble,
 *           nibble n -> ((n ^ 8) - 8) in [-8, 7]; fp16 scales[M, K/32].
 *  - Paged KV cache: per layer, K and V pages of [n_blocks][Hkv][16][HD] fp16; a block table
 *    int32[batch][max_blocks] maps token j of sequence b to page table[b][j/16], slot j%16.
 */
#ifndef B200DEC_H
#define B200DEC_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B2D_API __attribute__((visibility("default")))
#else
#define B2D_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* b2d_stream_t; /* same type as cudaStream_t */

enum b2d_status {
  B2D_OK = 0,
  B2D_ERR_NULL = 1,        /* a required pointer is NULL */
  B2D_ERR_SHAPE = 2,       /* sizes out of range or not supported by the kernel */
  B2D_ERR_ALIGN = 3,       /* pointer or row stride not 16-byte aligned */
  B2D_ERR_UNSUPPORTED = 4, /* dtype / epilogue / head_dim combination not built */
  B2D_ERR_WORKSPACE = 5,   /* workspace missing or smaller than the *_workspace_bytes query */
  B2D_ERR_CUDA = 6,        /* a CUDA runtime call failed (see b2d_last_cuda_error) */
  B2D_ERR_NCCL = 7,        /* an NCCL call failed */
  B2D_ERR_TIMEOUT = 8,     /* a bounded device-side wait gave up */
  B2D_ERR_STATE = 9        /* handle used out of order (e.g. step before weights are set) */
};

/* B2D_F16X2: an fp32 value carried as two fp16 planes, hi = fp16(v) and lo = fp16(v - hi)
 * (~22 significant bits), the tensor-core operand form of fp32 activations.  A [rows, cols]
 * array of this type with row stride ld is the hi plane [rows, ld] followed by the lo plane,
 * which starts rows * ld elements after the first.  (Extension: the reference keeps its
 * activations in fp32, LK/kernels.metal:106-131; this is how they reach fp16 tensor cores.) */
enum b2d_dtype { B2D_F32 = 0, B2D_F16 = 1, B2D_Q8_32 = 2, B2D_Q4_32 = 3, B2D_F16X2 = 4 };

/* GEMV epilogues (GK/kernels.metal:151-198 EPI 0/1/2; LK/kernels.metal:139-173; :307-345). */
enum b2d_epilogue {
  B2D_EPI_STORE = 0,    /* y = W x                                */
  B2D_EPI_ADD = 1,      /* y += W x          (residual add)       */
  B2D_EPI_GELU_MUL = 2, /* y = gelu_tanh(W x) * aux                */
  B2D_EPI_SWIGLU = 3,   /* y = silu(W x) * (W_up x)                */
  B2D_EPI_ARGMAX = 4,   /* logits = W x (optional), token = argmax */
  B2D_EPI_SILU_MUL = 5  /* y = silu(W x) * aux: the gate half of a SwiGLU whose up half was
                           computed separately (tensor-core GEMMs only) */
};

B2D_API const char* b2d_status_string(int status);
B2D_API int b2d_last_cuda_error(void);
B2D_API int b2d_version(void);
/* Kernel launches the library has enqueued from the calling thread so far (launches made
 * while a stream is being captured into a CUDA graph count once, at capture). */
B2D_API long long b2d_launch_counter(void);

/* ---------------------------------------------------------------------------------------
 * GEMV family (decode matrix-vector products on CUDA cores; 16-byte streaming loads)
 * ------------------------------------------------------------------------------------- */

/* Config 1: y[M] = W[M,K] x[K], all fp32, fp32 accumulation.
 * Replaces matvec_f16 (LK/kernels.metal:106-137; host Engine.matvec LK/main.swift:248-259)
 * for fp32 weights.  K % 4 == 0. */
B2D_API int b2d_gemv_f32(const float* W, const float* x, float* y, int M, int K, b2d_stream_t stream);

/* The fused decode GEMV.  For each of `batch` activation rows x_b (row stride ldx elements):
 *   prologue  if gamma != NULL:  x_b <- x_b * rsqrt(mean(x_b^2) + eps) * gamma
 *             (rmsnorm LK/kernels.metal:71-89 fused in front of the matvec, LK/main.swift:333-334)
 *   product   acc_b = W x_b   with W of w_dtype (F32, F16, Q8_32, Q4_32; scales for Q*)
 *   epilogue  per `epilogue` into y (row stride ldy, y_dtype F32 or F16):
 *             STORE / ADD (matvec_f16<ADD> LK/kernels.metal:106-137),
 *             GELU_MUL with aux[batch, M] (stride ldy) (GK/kernels.metal:159-198),
 *             SWIGLU with the second matrix W_up/W_up_scales (matvec_gate_up_silu
 *             LK/kernels.metal:144-173).
 * x_dtype is F32 or F16.  K must be a multiple of 32 for Q*, 8 for F16, 4 for F32.
 * batch >= 1 (rows are processed in groups; batch <= 8 streams W once).
 * ARGMAX is served by b2d_lm_head_argmax.
 * F16, Q8_32 and Q4_32 weights (the formats enabled with b2d_gemv_mma_formats) whose row is a
 * multiple of 128 bytes, with scales 8-byte (Q8) / 16-byte (Q4) aligned, run on the tensor-core
 * GEMV: weights as exact fp16 on mma.sync (integers dequantized exactly), the block scale
 * applied to each block's fp32 result, up to 16 fp16 tokens (8 when x is fp32 or normalized:
 * hi + lo fp16 columns) per pass over W.  Everything else (F32 weights) runs on CUDA cores. */
/* Weight dtypes that b2d_gemv sends to the tensor-core GEMV: bit d set for dtype d (F16, Q8_32,
 * Q4_32; F32 is ignored); bit 4 (B2D_GEMV_MMA_INT8_B1): a quantized GEMV of one token runs on the
 * integer tensor cores (the token as 3 int8 digits of a 21-bit fixed-point value, exact int32
 * block sums).  Default (1 << B2D_F16) | (1 << B2D_Q8_32) | (1 << B2D_Q4_32).  mask < 0 only
 * queries.  Returns the previous mask.  Process-wide; set it before capturing graphs. */
#define B2D_GEMV_MMA_INT8_B1 16
B2D_API int b2d_gemv_mma_formats(int mask);

B2D_API int b2d_gemv(int w_dtype, const void* W, const void* W_scales, const void* W_up,
             const void* W_up_scales, int x_dtype, const void* x, int ldx, const float* gamma,
             float eps, int epilogue, int y_dtype, void* y, int ldy, const float* aux, int M,
             int K, int batch, b2d_stream_t stream);

/* Config 2 shorthand: fp16 W, fp32 x and y, fused RMSNorm (gamma may be NULL), batch rows. */
B2D_API int b2d_rmsnorm_gemv_f16(const uint16_t* W, const float* x, const float* gamma, float eps,
                         float* y, int M, int K, int batch, int epilogue, const float* aux,
                         const uint16_t* W_up, b2d_stream_t stream);

/* Config 3 shorthands: 32-block quantized weights, fp16 activations x[batch,K], fp32 y[batch,M]. */
B2D_API int b2d_gemv_q8_32(const int8_t* q, const uint16_t* scales, const uint16_t* x, float* y, int M,
                   int K, int batch, b2d_stream_t stream);
B2D_API int b2d_gemv_q4_32(const uint8_t* q, const uint16_t* scales, const uint16_t* x, float* y, int M,
                   int K, int batch, b2d_stream_t stream);

/* Dequantize to fp32 w[M,K] = float(scale) * q, exact (bit-exact test target). */
B2D_API int b2d_dequant_q8_32(const int8_t* q, const uint16_t* scales, float* w, int M, int K,
                      b2d_stream_t stream);
B2D_API int b2d_dequant_q4_32(const uint8_t* q, const uint16_t* scales, float* w, int M, int K,
                      b2d_stream_t stream);

/* LM head + greedy sampling fused: logits_b = W (rmsnorm(x_b) if gamma) with fp16 W [V, K],
 * fp32 x; tokens[b] = argmax (ties -> lowest index) + index_offset; optional outputs
 * logits[batch, V] (fp32, NULL to skip) and max_vals[batch] (the winning logit, NULL to skip).
 * Replaces lmHeadAndArgmax (LK/main.swift:305-315) + argmax (LK/kernels.metal:310-345).
 * Needs workspace of b2d_lm_head_argmax_workspace_bytes(V, batch) bytes, zero-filled before
 * its first use; every call leaves its arrival counter at zero again for the next call. */
B2D_API size_t b2d_lm_head_argmax_workspace_bytes(int V, int batch);
B2D_API int b2d_lm_head_argmax(const uint16_t* W, const float* x, int ldx, const float* gamma, float eps,
                       int V, int K, int batch, int index_offset, float* logits,
                       int* tokens, float* max_vals, void* workspace, size_t workspace_bytes,
                       b2d_stream_t stream);

/* Batched decode GEMM on the tensor cores (tcgen05.mma with TMEM accumulators, operands staged
 * by TMA) for 1 <= batch <= 32 -- the batch >= 16 path of matvec_f16 / matvec_gate_up_silu
 * (LK/kernels.metal:106-173) and lmHeadAndArgmax (LK/main.swift:305-315):
 *   Y[b, m] = epilogue(sum_k W[m, k] X[b, k]),  W fp16 [M, K] row-major, X fp16 [batch, K]
 *   (row stride ldx, a multiple of 8), K a multiple of 8.
 * Epilogues: STORE / ADD (y fp32 or fp16, row stride ldy), GELU_MUL (aux), SWIGLU (W_up: both
 * matrices share each X tile), ARGMAX (tokens[b] = argmax + index_offset, ties -> lowest index;
 * logits[batch, M] and max_vals[batch] optional, y unused).  Split-K partial sums are reduced
 * in a fixed order (deterministic).  Workspace: b2d_gemm_tc_workspace_bytes(M, K, batch,
 * epilogue) bytes, zero-filled before first use; its first int is an error word (non-zero after
 * a bounded device-side wait gave up); calls leave its counters at zero. */
B2D_API size_t b2d_gemm_tc_workspace_bytes(int M, int K, int batch, int epilogue);
B2D_API int b2d_gemm_tc(const uint16_t* W, const uint16_t* W_up, const uint16_t* X, int ldx,
                        int epilogue, int y_dtype, void* y, int ldy, const float* aux, int M, int K,
                        int batch, float* logits, int* tokens, float* max_vals, int index_offset,
                        void* workspace, size_t workspace_bytes, b2d_stream_t stream);
/* b2d_gemm_tc with the activation type explicit: x_dtype B2D_F16 (as above) or B2D_F16X2 --
 * fp32-precision activations as hi + lo fp16 planes (X, and X + batch * ldx), multiplied in one
 * tcgen05.mma of twice the N (the reference's fp16 W x fp32 x, LK/kernels.metal:106-131).
 * y_dtype may be B2D_F16X2 too (lo plane at y + batch * ldy): the SwiGLU output that feeds the
 * down projection. */
B2D_API int b2d_gemm_tc_ex(int x_dtype, const uint16_t* W, const uint16_t* W_up,
                           const uint16_t* X, int ldx, int epilogue, int y_dtype, void* y, int ldy,
                           const float* aux, int M, int K, int batch, float* logits, int* tokens,
                           float* max_vals, int index_offset, void* workspace,
                           size_t workspace_bytes, b2d_stream_t stream);

/* Packed weight layout for the tensor-core GEMV (an HBM layout choice of this library; the
 * reference's weights file is row-major, LK/convert_weights.py:60-72): W [M, K] fp16 becomes
 * ceil(M/128) x ceil(K/64) tiles of 16 KB, tile (mt, kt) at byte ((mt * ceil(K/64)) + kt) *
 * 16384, each the 128 x 64 block of rows mt*128.. and columns kt*64.. in the MMA's shared-memory
 * image (row r at (r/8)*1024 + (r%8)*128, 16-byte chunk c of the row at ((c ^ (r%8)) * 16));
 * rows / columns past M / K are zero.  Each CTA then streams contiguous HBM instead of 128-byte
 * row pieces.  b2d_tc_pack_f16 writes it (out: b2d_tc_packed_bytes(M, K) bytes, 16-byte
 * aligned; K % 8 == 0), and b2d_gemm_tc_packed is b2d_gemm_tc with Wp / Wp_up in this layout. */
B2D_API size_t b2d_tc_packed_bytes(int M, int K);
B2D_API int b2d_tc_pack_f16(const uint16_t* W, int ldw, int M, int K, void* out,
                            b2d_stream_t stream);
B2D_API int b2d_gemm_tc_packed(const void* Wp, const void* Wp_up, const uint16_t* X, int ldx,
                               int epilogue, int y_dtype, void* y, int ldy, const float* aux,
                               int M, int K, int batch, float* logits, int* tokens,
                               float* max_vals, int index_offset, void* workspace,
                               size_t workspace_bytes, b2d_stream_t stream);

/* The tensor-core batched GEMV for 32-block quantized weights (w_dtype B2D_Q8_32 or B2D_Q4_32,
 * layouts above; scales fp16 [M, K/32]): TMA streams the raw weight tiles through a deep
 * shared-memory ring and dequantizer warps expand them to fp16(scale * q) -- the MMA operand --
 * so the batch reads every weight byte once.  X fp16 [batch <= 32, K], K a multiple of 32;
 * epilogues STORE / ADD / GELU_MUL into y (fp32 or fp16, row stride ldy).  Workspace as
 * b2d_gemm_tc_workspace_bytes(M, K, batch, epilogue).  (Extension: the reference has no
 * quantized weights, ios_kernels/PLAN.md:175,256.) */
B2D_API int b2d_gemm_tc_q(int w_dtype, const void* q, const uint16_t* scales, const uint16_t* X,
                          int ldx, int epilogue, int y_dtype, void* y, int ldy, const float* aux,
                          int M, int K, int batch, void* workspace, size_t workspace_bytes,
                          b2d_stream_t stream);
/* b2d_gemm_tc_q with x_dtype B2D_F16 or B2D_F16X2 (hi + lo planes, as b2d_gemm_tc_ex). */
B2D_API int b2d_gemm_tc_q_ex(int x_dtype, int w_dtype, const void* q, const uint16_t* scales,
                             const uint16_t* X, int ldx, int epilogue, int y_dtype, void* y,
                             int ldy, const float* aux, int M, int K, int batch, void* workspace,
                             size_t workspace_bytes, b2d_stream_t stream);

/* ---------------------------------------------------------------------------------------
 * Small ops of the decode step
 * ------------------------------------------------------------------------------------- */

/* y[r] = x[r] * rsqrt(mean(x[r]^2) + eps) * w, rows of length D, fp32 (LK/kernels.metal:71-89). */
B2D_API int b2d_rmsnorm(const float* x, const float* w, float* y, int rows, int D, float eps,
                b2d_stream_t stream);

/* x[b, :] = float(E[tokens[b], :]), fp16 E [V, D] (embed LK/kernels.metal:31-39). */
B2D_API int b2d_embed_f16(const uint16_t* E, const int* tokens, float* x, int D, int batch,
                  b2d_stream_t stream);

/* tokens[b] = argmax(logits[b, :N]) + index_offset, ties -> lowest (LK/kernels.metal:310-345). */
B2D_API int b2d_argmax_f32(const float* logits, int N, int batch, int* tokens, int index_offset,
                   b2d_stream_t stream);

/* Combine per-rank (value, index) candidates [n_parts][batch] -> tokens[batch] (ties ->
 * lowest index).  Used after the vocab-parallel LM head's all-gather. */
B2D_API int b2d_argmax_combine(const float* vals, const int* idxs, int n_parts, int batch, int* tokens,
                       b2d_stream_t stream);

/* Residual add + RMSNorm to fp16 (the tensor-core GEMM operand), rows of length D:
 * if p != NULL: x += p (x updated in place); out = fp16(x * rsqrt(mean(x^2) + eps) * gamma).
 * (rmsnorm LK/kernels.metal:71-89.) */
B2D_API int b2d_add_rmsnorm_f16(float* x, const float* p, const float* gamma, float eps,
                                uint16_t* out, int rows, int D, b2d_stream_t stream);
/* The same with the output type explicit: out_dtype B2D_F16 (as above) or B2D_F16X2 (hi plane
 * out[rows, D], lo plane at out + rows * D): the fp32-precision operand of the tensor-core
 * projections. */
B2D_API int b2d_add_rmsnorm(float* x, const float* p, const float* gamma, float eps, int out_dtype,
                            void* out, int rows, int D, b2d_stream_t stream);

/* Embedding + RMSNorm: x[b] = float(E[tokens[b]]); out[b] = fp16(rmsnorm(x[b]) * gamma)
 * (embed LK/kernels.metal:31-39 fused with the first rmsnorm). */
B2D_API int b2d_embed_rmsnorm_f16(const uint16_t* E, const int* tokens, float* x,
                                  const float* gamma, float eps, uint16_t* out, int D, int batch,
                                  b2d_stream_t stream);

/* x[i] += p[i], fp32, n elements (residual add after a tensor-parallel all-reduce). */
B2D_API int b2d_add_f32(float* x, const float* p, size_t n, b2d_stream_t stream);

/* RoPE inverse frequencies, computed in double and rounded to fp32 (LK/main.swift:90-94);
 * out is HOST memory of head_dim/2 floats. */
B2D_API int b2d_inv_freq(int head_dim, double theta, float* out_host);

/* ---------------------------------------------------------------------------------------
 * Paged decode attention (ragged batch, GQA, RoPE, KV append, split-K)
 * ------------------------------------------------------------------------------------- */

/* RoPE + KV append only (rope_kv LK/kernels.metal:182-224, paged): for each sequence b with
 * pos = ctx_lens[b], rotate q heads in place in qkv (row stride ldqkv elements, layout
 * [q Hq*HD | k Hkv*HD | v Hkv*HD], qkv_dtype F32 or F16), rotate k and write k, v as fp16
 * into the pages at pos (not written if the page id is outside [0, n_blocks)). */
B2D_API int b2d_rope_kv_append(void* qkv, int qkv_dtype, int ldqkv, uint16_t* k_pages,
                       uint16_t* v_pages, const int* block_table, int max_blocks,
                       int n_blocks, const int* ctx_lens, const float* inv_freq, int n_heads, int n_kv_heads,
                       int head_dim, int batch, b2d_stream_t stream);

/* Single-query attention for each sequence b of the batch over tokens [start, pos] of its
 * paged cache, pos = ctx_lens[b], start = max(0, pos + 1 - window) (window 0 = full).
 * Replaces attention (LK/kernels.metal:235-305; window GK/kernels.metal:343) and, when
 * `append` != 0, rope_kv (LK/kernels.metal:182-224): q and the new k are rotated at pos, and
 * k, v are written into the pages at pos before use.  With append == 0 the caller has already
 * rotated q and stored the token at pos (e.g. b2d_rope_kv_append).
 * Split-K: keys are cut into chunks of b2d_attn_chunk_tokens(batch, n_kv_heads, max_ctx)
 * keys; each (sequence, KV head, chunk) is one CTA whose GQA query heads share every K/V
 * load; partial softmax states go to `workspace` and the last CTA of each (sequence, KV head)
 * merges them.  The workspace must be zero-filled before its first use; every call leaves its
 * arrival counters at zero again, so it can be reused by later calls on the same stream.
 * out[b, Hq*HD] (row stride ldout, out_dtype F32, F16 or F16X2 -- lo plane at out + batch *
 * ldout).  head_dim 64, 128 or 256; n_heads /
 * n_kv_heads in {1, 2, 4, 8}.  scale <= 0 means 1/sqrt(head_dim) (LK/main.swift:293).
 * max_ctx bounds every ctx_lens[b] + 1 and sizes the workspace; n_blocks is the page-pool
 * size: a block-table entry outside [0, n_blocks) is never dereferenced (its keys are
 * skipped). */
B2D_API int b2d_attn_chunk_tokens(int batch, int n_kv_heads, int max_ctx);
B2D_API size_t b2d_paged_attn_workspace_bytes(int batch, int n_heads, int n_kv_heads, int head_dim,
                                      int max_ctx);
B2D_API int b2d_paged_decode_attn(void* qkv, int qkv_dtype, int ldqkv, uint16_t* k_pages,
                          uint16_t* v_pages, const int* block_table, int max_blocks,
                          int n_blocks, const int* ctx_lens, const float* inv_freq,
                          int n_heads, int n_kv_heads, int head_dim, int batch, int max_ctx,
                          float scale, int window, int append, void* out, int out_dtype,
                          int ldout, void* workspace, size_t workspace_bytes,
                          b2d_stream_t stream);

/* Allocation-free variant of b2d_paged_decode_attn (no counterpart in the reference, which
 * has no allocator constraints).  For callers that cannot allocate device memory -- code
 * living inside another framework's memory pool, plugins whose host forbids cudaMalloc after
 * start-up -- it takes no workspace: the split-K scratch is a fixed 16 MiB device array
 * inside this library (held on every GPU that loads it until exit).  Sizes whose
 * b2d_paged_attn_workspace_bytes exceed b2d_paged_decode_attn_noalloc_max_scratch_bytes()
 * return B2D_ERR_WORKSPACE.  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress), so make that first call before any stream capture.  Each call
 * clears the array's header (error word, arrival counters) on `stream` before its kernel.
 * All calls share the array: calls whose kernels overlap on the GPU race on it.  Never calls
 * cudaMalloc / cudaFree.  Other arguments and results as b2d_paged_decode_attn.
 * b2d_paged_decode_attn_noalloc_error waits for the device (cudaDeviceSynchronize) and returns
 * B2D_ERR_TIMEOUT if a bounded device-side wait of the most recent call on the current device
 * gave up (its output is then incomplete), else B2D_OK; the next call clears the word. */
B2D_API size_t b2d_paged_decode_attn_noalloc_max_scratch_bytes(void);
B2D_API int b2d_paged_decode_attn_noalloc_error(void);
B2D_API int b2d_paged_decode_attn_noalloc(void* qkv, int qkv_dtype, int ldqkv, uint16_t* k_pages,
                                          uint16_t* v_pages, const int* block_table,
                                          int max_blocks, int n_blocks, const int* ctx_lens,
                                          const float* inv_freq, int n_heads, int n_kv_heads,
                                          int head_dim, int batch, int max_ctx, float scale,
                                          int window, int append, void* out, int out_dtype,
                                          int ldout, b2d_stream_t stream);

/* ---------------------------------------------------------------------------------------
 * Decode step of a Llama-style model (Engine.encodeDecode LK/main.swift:321-347), ragged
 * batch over a paged cache, optionally tensor-parallel over NCCL.
 * ------------------------------------------------------------------------------------- */

typedef struct b2d_decoder b2d_decoder;

typedef struct {
  int dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, vocab;
  float eps;
  double rope_theta;
  int max_batch;      /* largest batch a step may use */
  int max_ctx;        /* every ctx_lens[b] + 1 <= max_ctx */
  int max_blocks;     /* block-table row length (>= ceil(max_ctx / 16)) */
  int n_blocks;       /* pages in each layer's K (and V) page pool */
} b2d_model_config;

/* NCCL unique id (128 bytes) for tensor parallelism; call on rank 0 and share the bytes. */
B2D_API int b2d_nccl_unique_id_bytes(void);
B2D_API int b2d_nccl_get_unique_id(void* out_host);

/* Create a decoder for rank `tp_rank` of `tp_size` (<= 8) on the current CUDA device.  With
 * tp_size > 1, nccl_id (host, 128 bytes from rank 0) sets up the communicator, and the ranks
 * map each other's partial-sum buffers (CUDA IPC) so the row-parallel sums and the LM-head
 * gather run over NVLink peer memory; where any rank cannot map them, or the environment sets
 * B2D_TP_COLLECTIVE=nccl, all ranks use ncclAllReduce / ncclAllGather instead.  The handle
 * allocates its activation buffers once; weights and KV pages stay owned by the caller.
 * b2d_decoder_destroy is collective when tp_size > 1 (every rank calls it). */
B2D_API int b2d_decoder_create(const b2d_model_config* cfg, int tp_rank, int tp_size,
                       const void* nccl_id, b2d_decoder** out);
B2D_API int b2d_decoder_destroy(b2d_decoder* h);
/* Prefill: run the n prompt tokens (device array) of one sequence at positions start_pos ..
 * start_pos + n - 1 through the model, writing their K/V into the pages of the sequence's
 * block-table row seq_table [max_blocks] (device), and set next_token (device int) to the greedy
 * token after the last one; logits (device [lm_rows], optional) receives the last position's
 * logits.  The tokens go through the decode step in chunks of max_batch consecutive positions
 * (LK/main.swift:357-372 prefills in chunks of rows too): each chunk's K/V is written first,
 * then every row attends to the positions up to its own, so a chunk costs one step (tcgen05
 * projections from 9 rows up) instead of one step per token.  Not graph-captured; collective
 * across tensor-parallel ranks (every rank calls it with the same arguments). */
B2D_API int b2d_decoder_prefill(b2d_decoder* h, const int* tokens, int n, const int* seq_table,
                                int start_pos, int* next_token, float* logits, b2d_stream_t stream);

/* Device-resident greedy decode loop: n_steps decode steps back to back with no host round trip.
 * After each step the next tokens replace tokens[b], ctx_lens[b] grows by one, and the tokens
 * are written to ring row (*ring_count % ring_steps), ring [ring_steps][batch] int32, after which
 * *ring_count grows by one (all device memory; tokens and ctx_lens are updated in place).  The
 * caller keeps ctx_lens + n_steps within max_ctx and the block table covering them.  The step
 * and the advance are captured into one CUDA graph (per pointer set) and launched n_steps times
 * (the reference's pipelined decode loop, LK/main.swift:473-491, with sampling kept on the GPU). */
B2D_API int b2d_decoder_generate(b2d_decoder* h, int* tokens, int* ctx_lens, const int* block_table,
                                 int batch, int n_steps, int* ring, int ring_steps, int* ring_count,
                                 b2d_stream_t stream);
/* Replace the RoPE inverse frequencies (host, head_dim / 2 floats; default: theta^(-2i/HD) from
 * rope_theta), e.g. with Llama-3 frequency scaling (LK/main.swift:89-108). */
B2D_API int b2d_decoder_set_inv_freq(b2d_decoder* h, const float* inv_freq_host, int n);
/* 1 if the steps so far use the peer-memory collectives, 0 for NCCL (or tp_size == 1). */
B2D_API int b2d_decoder_peer_collectives(const b2d_decoder* h);
/* Device-side status of the steps enqueued so far (cudaDeviceSynchronize, then reads the error
 * words): 0, or B2D_ERR_TIMEOUT if a bounded device-side wait gave up -- a peer barrier waiting
 * for another rank (10 s), or a TMA / mbarrier wait inside the attention or a tensor-core GEMM
 * (about 2 s); the outputs of that step are then incomplete.  Reading clears the error words
 * and resets the split-K arrival counters, so later steps start clean. */
B2D_API int b2d_decoder_error(b2d_decoder* h);

/* Weights of this rank's shard (fp16 matrices, fp32 norms), as b2d_shard_* in the Python
 * host lays them out: wqkv [(Hq+2Hkv)/tp*HD, D] rows [q | k | v] of the local heads;
 * wo [D, Hq/tp*HD]; wgate, wup [F/tp, D]; wdown [D, F/tp]. */
B2D_API int b2d_decoder_set_layer(b2d_decoder* h, int layer, const float* attn_norm,
                          const uint16_t* wqkv, const uint16_t* wo, const float* ffn_norm,
                          const uint16_t* wgate, const uint16_t* wup, const uint16_t* wdown,
                          uint16_t* k_pages, uint16_t* v_pages);
/* b2d_decoder_set_layer with the five projections in one weight type: w_dtype B2D_F16 (as
 * b2d_decoder_set_layer; scales ignored) or B2D_Q8_32 / B2D_Q4_32 (layouts at the top of this
 * file; each matrix with its fp16 scales [rows, K/32]), streamed as stored -- 1.06 / 0.56 bytes
 * per weight instead of 2.  Batches below 9 run them on the tensor-core GEMV (integers exact in
 * fp16, the block scale applied to each block's fp32 result: exact dequantization); batches of
 * 9 and more on the tcgen05 GEMM, whose MMA operand is fp16(scale * q) (one fp16 rounding of
 * the dequantized weight), the gate/up SwiGLU as an up GEMM and a gate GEMM with the SILU_MUL
 * epilogue.  Every projection's K (D, local heads * HD, local FFN rows) must be a multiple of
 * 32.  (Extension: the reference's quantized weights are roadmap only,
 * ios_kernels/PLAN.md:175-176,256.) */
B2D_API int b2d_decoder_set_layer_q(b2d_decoder* h, int layer, int w_dtype, const float* attn_norm,
                                    const void* wqkv, const uint16_t* wqkv_scales, const void* wo,
                                    const uint16_t* wo_scales, const float* ffn_norm,
                                    const void* wgate, const uint16_t* wgate_scales,
                                    const void* wup, const uint16_t* wup_scales, const void* wdown,
                                    const uint16_t* wdown_scales, uint16_t* k_pages,
                                    uint16_t* v_pages);
/* embed [V, D] fp16 (replicated); lm_head [ceil(V/tp), D] fp16 rows of this rank's vocab
 * shard (the tied embedding's rows); final_norm [D]. */
B2D_API int b2d_decoder_set_head(b2d_decoder* h, const uint16_t* embed, const uint16_t* lm_head,
                         int lm_rows, const float* final_norm);

/* One decode step: tokens[b] at position ctx_lens[b] for b < batch.  Writes next_tokens[b]
 * (greedy) and, if logits != NULL, this rank's vocab-shard logits [batch, lm_rows].  The KV
 * pages receive the new token.  use_graph != 0 captures the step into a CUDA graph on first
 * use (per batch size and pointer set) and replays it afterwards. */
B2D_API int b2d_decoder_step(b2d_decoder* h, const int* tokens, const int* ctx_lens,
                     const int* block_table, int batch, int* next_tokens, float* logits,
                     int use_graph, b2d_stream_t stream);

/* ---------------------------------------------------------------------------------------
 * Tensor-parallel collectives over NVLink peer memory (what the decoder runs between the
 * row-parallel projections; no reference counterpart: the reference runs on one device).
 * ------------------------------------------------------------------------------------- */

/* x[b] += parts[0][b] + parts[1][b] + ... + parts[tp-1][b]  (rank order, so every rank computes
 * bit-identical sums), then, if gamma != NULL, out16[b] = fp16(rmsnorm(x[b]) * gamma), for
 * b < rows; D % 4 == 0.  parts (host array of tp device pointers) are the ranks' partial sums
 * [rows, D] fp32, mapped into this process; sigs (host array of tp device pointers) are the
 * ranks' signal arrays of (slot0 + rows) * 8 uint32 each, zero-initialised once; epochs
 * (this rank's, slot0 + rows uint32, zero-initialised once) count the barrier uses per slot.
 * Row b waits, bounded by timeout_ns, until every rank has announced its partial of row b;
 * on timeout *err (device int) becomes B2D_ERR_TIMEOUT and that row is left unchanged. */
B2D_API int b2d_tp_allreduce_add_rmsnorm(const float* const* parts, uint32_t* const* sigs,
                                         uint32_t* epochs, int rank, int tp, int slot0, float* x,
                                         const float* gamma, float eps, uint16_t* out16, int D,
                                         int rows, long long timeout_ns, int* err,
                                         b2d_stream_t stream);
/* tokens[b] = the index of the best (value, index) pair over the ranks' vals[r][b], idxs[r][b]
 * (larger value, ties -> lower index), after the same bounded barrier on signal slot `slot`. */
B2D_API int b2d_tp_argmax_gather(const float* const* vals, const int* const* idxs,
                                 uint32_t* const* sigs, uint32_t* epochs, int rank, int tp,
                                 int slot, int B, int* tokens, long long timeout_ns, int* err,
                                 b2d_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* B200DEC_H */
