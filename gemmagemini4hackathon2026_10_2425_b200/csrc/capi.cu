// extern "C" entry points of libb200dec.so (declared in include/b200dec.h) and the shared
// host plumbing: status strings, the last CUDA error, the per-device SM count.
#include <cmath>
#include <mutex>

#include "common.cuh"

namespace b2d {

static thread_local int g_last_cuda_error = 0;
static thread_local long long g_launches = 0;
void set_cuda_error(cudaError_t e) { g_last_cuda_error = (int)e; }
void count_launch(int n) { g_launches += n; }

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

// implemented in gemv.cu / gemv_mma.cu / ops.cu / attention.cu
int gemv_mma_formats(int mask);
int gemv_dispatch(int, const void*, const void*, const void*, const void*, int, const void*, int,
                  const float*, float, int, int, void*, int, const float*, int, int, int,
                  cudaStream_t);
size_t lm_head_argmax_workspace_bytes(int V, int batch);
int lm_head_argmax(const uint16_t*, const float*, int, const float*, float, int, int, int, int,
                   float*, int*, float*, void*, size_t, cudaStream_t);
int dequant(bool q4, const void* q, const uint16_t* scales, float* w, int M, int K, cudaStream_t);
int rmsnorm(const float*, const float*, float*, int, int, float, cudaStream_t);
int embed_f16(const uint16_t*, const int*, float*, int, int, cudaStream_t);
int argmax_f32(const float*, int, int, int*, int, cudaStream_t);
int argmax_combine(const float*, const int*, int, int, int*, cudaStream_t);
int add_f32(float*, const float*, size_t, cudaStream_t);
int rope_kv_append(void*, int, int, uint16_t*, uint16_t*, const int*, int, int, const int*,
                   const float*, int, int, int, int, cudaStream_t);
int attn_chunk_tokens(int, int, int);
int add_rmsnorm_f16(float*, const float*, const float*, float, uint16_t*, uint16_t*, int, int,
                    cudaStream_t);
int embed_rmsnorm_f16(const uint16_t*, const int*, float*, const float*, float, uint16_t*,
                      uint16_t*, float*, int, int, cudaStream_t);
size_t tc_gemm_workspace_bytes(int M, int K, int batch, int epilogue);
int tc_gemm(int, const uint16_t*, const uint16_t*, const uint16_t*, int, int, int, void*, int,
            const float*, int, int, int, float*, int*, float*, int, void*, size_t, cudaStream_t,
            const void*, size_t);
int tc_gemm_q(int, int, const void*, const uint16_t*, const uint16_t*, int, int, int, void*, int,
              const float*, int, int, int, void*, size_t, cudaStream_t, float* const*, int,
              const void*, size_t);
int tc_gemm_packed(const uint8_t*, const uint8_t*, const uint16_t*, int, int, int, void*, int,
                   const float*, int, int, int, float*, int*, float*, int, void*, size_t,
                   cudaStream_t);
size_t tc_packed_bytes(int, int);
int tc_pack_f16(const uint16_t*, int, int, int, void*, cudaStream_t);
int tp_allreduce_add_rmsnorm(const float* const*, uint32_t* const*, uint32_t*, int, int, int,
                             float*, const float*, float, uint16_t*, uint16_t*, int, int,
                             long long, int*, cudaStream_t);
int tp_argmax_gather(const float* const*, const int* const*, uint32_t* const*, uint32_t*, int,
                     int, int, int, int*, long long, int*, cudaStream_t);
size_t paged_attn_workspace_bytes(int, int, int, int, int);
int paged_decode_attn(void*, int, int, uint16_t*, uint16_t*, const int*, int, int, const int*,
                      const float*, int, int, int, int, int, float, int, int, void*, int, int,
                      void*, size_t, cudaStream_t);

}  // namespace b2d

using namespace b2d;

static inline cudaStream_t S(b2d_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

extern "C" {

const char* b2d_status_string(int status) {
  switch (status) {
    case B2D_OK: return "ok";
    case B2D_ERR_NULL: return "a required pointer is NULL";
    case B2D_ERR_SHAPE: return "sizes out of range or not supported";
    case B2D_ERR_ALIGN: return "pointer or row stride not 16-byte aligned";
    case B2D_ERR_UNSUPPORTED: return "dtype / epilogue / head_dim combination not supported";
    case B2D_ERR_WORKSPACE: return "workspace missing or too small";
    case B2D_ERR_CUDA: return "CUDA runtime error";
    case B2D_ERR_NCCL: return "NCCL error";
    case B2D_ERR_TIMEOUT: return "bounded device wait timed out";
    case B2D_ERR_STATE: return "handle used out of order";
    default: return "unknown status";
  }
}

int b2d_last_cuda_error(void) { return g_last_cuda_error; }
int b2d_version(void) { return 1; }
long long b2d_launch_counter(void) { return g_launches; }

int b2d_gemv_f32(const float* W, const float* x, float* y, int M, int K, b2d_stream_t stream) {
  return gemv_dispatch(B2D_F32, W, nullptr, nullptr, nullptr, B2D_F32, x, K, nullptr, 0.f,
                       B2D_EPI_STORE, B2D_F32, y, M, nullptr, M, K, 1, S(stream));
}

int b2d_gemv_mma_formats(int mask) { return gemv_mma_formats(mask); }

int b2d_gemv(int w_dtype, const void* W, const void* W_scales, const void* W_up,
             const void* W_up_scales, int x_dtype, const void* x, int ldx, const float* gamma,
             float eps, int epilogue, int y_dtype, void* y, int ldy, const float* aux, int M,
             int K, int batch, b2d_stream_t stream) {
  return gemv_dispatch(w_dtype, W, W_scales, W_up, W_up_scales, x_dtype, x, ldx, gamma, eps,
                       epilogue, y_dtype, y, ldy, aux, M, K, batch, S(stream));
}

int b2d_rmsnorm_gemv_f16(const uint16_t* W, const float* x, const float* gamma, float eps,
                         float* y, int M, int K, int batch, int epilogue, const float* aux,
                         const uint16_t* W_up, b2d_stream_t stream) {
  return gemv_dispatch(B2D_F16, W, nullptr, W_up, nullptr, B2D_F32, x, K, gamma, eps, epilogue,
                       B2D_F32, y, M, aux, M, K, batch, S(stream));
}

int b2d_gemv_q8_32(const int8_t* q, const uint16_t* scales, const uint16_t* x, float* y, int M,
                   int K, int batch, b2d_stream_t stream) {
  return gemv_dispatch(B2D_Q8_32, q, scales, nullptr, nullptr, B2D_F16, x, K, nullptr, 0.f,
                       B2D_EPI_STORE, B2D_F32, y, M, nullptr, M, K, batch, S(stream));
}

int b2d_gemv_q4_32(const uint8_t* q, const uint16_t* scales, const uint16_t* x, float* y, int M,
                   int K, int batch, b2d_stream_t stream) {
  return gemv_dispatch(B2D_Q4_32, q, scales, nullptr, nullptr, B2D_F16, x, K, nullptr, 0.f,
                       B2D_EPI_STORE, B2D_F32, y, M, nullptr, M, K, batch, S(stream));
}

int b2d_dequant_q8_32(const int8_t* q, const uint16_t* scales, float* w, int M, int K,
                      b2d_stream_t stream) {
  return dequant(false, q, scales, w, M, K, S(stream));
}

int b2d_dequant_q4_32(const uint8_t* q, const uint16_t* scales, float* w, int M, int K,
                      b2d_stream_t stream) {
  return dequant(true, q, scales, w, M, K, S(stream));
}

size_t b2d_lm_head_argmax_workspace_bytes(int V, int batch) {
  return lm_head_argmax_workspace_bytes(V, batch);
}

int b2d_lm_head_argmax(const uint16_t* W, const float* x, int ldx, const float* gamma, float eps,
                       int V, int K, int batch, int index_offset, float* logits, int* tokens,
                       float* max_vals, void* workspace, size_t workspace_bytes,
                       b2d_stream_t stream) {
  return lm_head_argmax(W, x, ldx, gamma, eps, V, K, batch, index_offset, logits, tokens,
                        max_vals, workspace, workspace_bytes, S(stream));
}

int b2d_rmsnorm(const float* x, const float* w, float* y, int rows, int D, float eps,
                b2d_stream_t stream) {
  return rmsnorm(x, w, y, rows, D, eps, S(stream));
}

int b2d_embed_f16(const uint16_t* E, const int* tokens, float* x, int D, int batch,
                  b2d_stream_t stream) {
  return embed_f16(E, tokens, x, D, batch, S(stream));
}

int b2d_argmax_f32(const float* logits, int N, int batch, int* tokens, int index_offset,
                   b2d_stream_t stream) {
  return argmax_f32(logits, N, batch, tokens, index_offset, S(stream));
}

int b2d_argmax_combine(const float* vals, const int* idxs, int n_parts, int batch, int* tokens,
                       b2d_stream_t stream) {
  return argmax_combine(vals, idxs, n_parts, batch, tokens, S(stream));
}

int b2d_add_f32(float* x, const float* p, size_t n, b2d_stream_t stream) {
  return add_f32(x, p, n, S(stream));
}

int b2d_add_rmsnorm_f16(float* x, const float* p, const float* gamma, float eps, uint16_t* out,
                        int rows, int D, b2d_stream_t stream) {
  return add_rmsnorm_f16(x, p, gamma, eps, out, nullptr, rows, D, S(stream));
}

int b2d_add_rmsnorm(float* x, const float* p, const float* gamma, float eps, int out_dtype,
                    void* out, int rows, int D, b2d_stream_t stream) {
  if (out_dtype != B2D_F16 && out_dtype != B2D_F16X2) return B2D_ERR_UNSUPPORTED;
  uint16_t* o = static_cast<uint16_t*>(out);
  return add_rmsnorm_f16(x, p, gamma, eps, o,
                         (out_dtype == B2D_F16X2 && o) ? o + (size_t)rows * D : nullptr, rows, D,
                         S(stream));
}

int b2d_embed_rmsnorm_f16(const uint16_t* E, const int* tokens, float* x, const float* gamma,
                          float eps, uint16_t* out, int D, int batch, b2d_stream_t stream) {
  return embed_rmsnorm_f16(E, tokens, x, gamma, eps, out, nullptr, nullptr, D, batch, S(stream));
}

size_t b2d_gemm_tc_workspace_bytes(int M, int K, int batch, int epilogue) {
  return tc_gemm_workspace_bytes(M, K, batch, epilogue);
}

int b2d_gemm_tc(const uint16_t* W, const uint16_t* W_up, const uint16_t* X, int ldx, int epilogue,
                int y_dtype, void* y, int ldy, const float* aux, int M, int K, int batch,
                float* logits, int* tokens, float* max_vals, int index_offset, void* workspace,
                size_t workspace_bytes, b2d_stream_t stream) {
  return tc_gemm(B2D_F16, W, W_up, X, ldx, epilogue, y_dtype, y, ldy, aux, M, K, batch, logits,
                 tokens, max_vals, index_offset, workspace, workspace_bytes, S(stream), nullptr, 0);
}

int b2d_gemm_tc_ex(int x_dtype, const uint16_t* W, const uint16_t* W_up, const uint16_t* X,
                   int ldx, int epilogue, int y_dtype, void* y, int ldy, const float* aux, int M,
                   int K, int batch, float* logits, int* tokens, float* max_vals,
                   int index_offset, void* workspace, size_t workspace_bytes,
                   b2d_stream_t stream) {
  return tc_gemm(x_dtype, W, W_up, X, ldx, epilogue, y_dtype, y, ldy, aux, M, K, batch, logits,
                 tokens, max_vals, index_offset, workspace, workspace_bytes, S(stream), nullptr, 0);
}

size_t b2d_tc_packed_bytes(int M, int K) { return tc_packed_bytes(M, K); }

int b2d_tc_pack_f16(const uint16_t* W, int ldw, int M, int K, void* out, b2d_stream_t stream) {
  return tc_pack_f16(W, ldw, M, K, out, S(stream));
}

int b2d_gemm_tc_packed(const void* Wp, const void* Wp_up, const uint16_t* X, int ldx,
                       int epilogue, int y_dtype, void* y, int ldy, const float* aux, int M,
                       int K, int batch, float* logits, int* tokens, float* max_vals,
                       int index_offset, void* workspace, size_t workspace_bytes,
                       b2d_stream_t stream) {
  return tc_gemm_packed(static_cast<const uint8_t*>(Wp), static_cast<const uint8_t*>(Wp_up), X,
                        ldx, epilogue, y_dtype, y, ldy, aux, M, K, batch, logits, tokens,
                        max_vals, index_offset, workspace, workspace_bytes, S(stream));
}

int b2d_gemm_tc_q(int w_dtype, const void* q, const uint16_t* scales, const uint16_t* X, int ldx,
                  int epilogue, int y_dtype, void* y, int ldy, const float* aux, int M, int K,
                  int batch, void* workspace, size_t workspace_bytes, b2d_stream_t stream) {
  return tc_gemm_q(B2D_F16, w_dtype, q, scales, X, ldx, epilogue, y_dtype, y, ldy, aux, M, K,
                   batch, workspace, workspace_bytes, S(stream), nullptr, 0, nullptr, 0);
}

int b2d_gemm_tc_q_ex(int x_dtype, int w_dtype, const void* q, const uint16_t* scales,
                     const uint16_t* X, int ldx, int epilogue, int y_dtype, void* y, int ldy,
                     const float* aux, int M, int K, int batch, void* workspace,
                     size_t workspace_bytes, b2d_stream_t stream) {
  return tc_gemm_q(x_dtype, w_dtype, q, scales, X, ldx, epilogue, y_dtype, y, ldy, aux, M, K,
                   batch, workspace, workspace_bytes, S(stream), nullptr, 0, nullptr, 0);
}

int b2d_tp_allreduce_add_rmsnorm(const float* const* parts, uint32_t* const* sigs,
                                 uint32_t* epochs, int rank, int tp, int slot0, float* x,
                                 const float* gamma, float eps, uint16_t* out16, int D, int rows,
                                 long long timeout_ns, int* err, b2d_stream_t stream) {
  return tp_allreduce_add_rmsnorm(parts, sigs, epochs, rank, tp, slot0, x, gamma, eps, out16,
                                  nullptr, D, rows, timeout_ns, err, S(stream));
}

int b2d_tp_argmax_gather(const float* const* vals, const int* const* idxs, uint32_t* const* sigs,
                         uint32_t* epochs, int rank, int tp, int slot, int B, int* tokens,
                         long long timeout_ns, int* err, b2d_stream_t stream) {
  return tp_argmax_gather(vals, idxs, sigs, epochs, rank, tp, slot, B, tokens, timeout_ns, err,
                          S(stream));
}

int b2d_inv_freq(int head_dim, double theta, float* out_host) {
  if (!out_host) return B2D_ERR_NULL;
  if (head_dim <= 0 || head_dim % 2 || !(theta > 0.0)) return B2D_ERR_SHAPE;
  for (int i = 0; i < head_dim / 2; ++i)
    out_host[i] = (float)(1.0 / std::pow(theta, (double)(2 * i) / (double)head_dim));
  return B2D_OK;
}

int b2d_rope_kv_append(void* qkv, int qkv_dtype, int ldqkv, uint16_t* k_pages,
                       uint16_t* v_pages, const int* block_table, int max_blocks, int n_blocks,
                       const int* ctx_lens, const float* inv_freq, int n_heads, int n_kv_heads,
                       int head_dim, int batch, b2d_stream_t stream) {
  return rope_kv_append(qkv, qkv_dtype, ldqkv, k_pages, v_pages, block_table, max_blocks,
                        n_blocks, ctx_lens, inv_freq, n_heads, n_kv_heads, head_dim, batch,
                        S(stream));
}

int b2d_attn_chunk_tokens(int batch, int n_kv_heads, int max_ctx) {
  return attn_chunk_tokens(batch, n_kv_heads, max_ctx);
}

size_t b2d_paged_attn_workspace_bytes(int batch, int n_heads, int n_kv_heads, int head_dim,
                                      int max_ctx) {
  return paged_attn_workspace_bytes(batch, n_heads, n_kv_heads, head_dim, max_ctx);
}

int b2d_paged_decode_attn(void* qkv, int qkv_dtype, int ldqkv, uint16_t* k_pages,
                          uint16_t* v_pages, const int* block_table, int max_blocks,
                          int n_blocks, const int* ctx_lens, const float* inv_freq, int n_heads,
                          int n_kv_heads, int head_dim, int batch, int max_ctx, float scale,
                          int window, int append, void* out, int out_dtype, int ldout,
                          void* workspace, size_t workspace_bytes, b2d_stream_t stream) {
  return paged_decode_attn(qkv, qkv_dtype, ldqkv, k_pages, v_pages, block_table, max_blocks,
                           n_blocks, ctx_lens, inv_freq, n_heads, n_kv_heads, head_dim, batch,
                           max_ctx, scale, window, append, out, out_dtype, ldout, workspace,
                           workspace_bytes, S(stream));
}

}  // extern "C"
