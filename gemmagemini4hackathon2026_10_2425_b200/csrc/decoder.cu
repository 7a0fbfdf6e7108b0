// Decode step of a Llama-style model over a ragged paged batch, optionally tensor-parallel.
//
// Replaces Engine.encodeDecode (LK/main.swift:321-347): embed -> per layer [RMSNorm + QKV
// matvec, RoPE + KV write, attention, O matvec + residual, RMSNorm + gate/up SwiGLU, down +
// residual] -> final norm + LM head + argmax.  The reference encodes ~115 dispatches per token
// for one sequence; here one step serves a whole batch and every RMSNorm, the RoPE, the KV
// append and the argmax are fused into the kernel that consumes them:
//
//   embed                                   (1 launch)
//   per layer: rmsnorm+QKV GEMV -> rope+append+split-K attention -> O GEMV (+residual)
//              -> rmsnorm+gate/up SwiGLU GEMV -> down GEMV (+residual)        (5 launches)
//   rmsnorm + LM-head GEMV + argmax         (1 launch)
//
// Tensor parallelism (tp > 1, one process per GPU): QKV and gate/up are column-parallel (this
// rank's heads / FFN rows), O and down are row-parallel and their partial sums are summed
// before the residual add; the LM head is vocab-parallel and each rank's (max, index) pair is
// gathered and combined (ties -> lowest index).  The sums and the gather run over NVLink peer
// memory (tp_peer.cu: one kernel = all-reduce + residual add + next RMSNorm), with NCCL
// (ncclAllReduce / ncclAllGather) as the path where the ranks cannot map each other's memory
// or B2D_TP_COLLECTIVE=nccl asks for it.  The whole step can be captured once into a CUDA
// graph and replayed.
#include <nccl.h>

#include <cmath>
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "common.cuh"

namespace b2d {
int gemv_dispatch(int, const void*, const void*, const void*, const void*, int, const void*, int,
                  const float*, float, int, int, void*, int, const float*, int, int, int,
                  cudaStream_t);
size_t lm_head_argmax_workspace_bytes(int V, int batch);
int lm_head_argmax(const uint16_t*, const float*, int, const float*, float, int, int, int, int,
                   float*, int*, float*, void*, size_t, cudaStream_t);
int embed_f16(const uint16_t*, const int*, float*, int, int, cudaStream_t);
int argmax_combine(const float*, const int*, int, int, int*, cudaStream_t);
int add_f32(float*, const float*, size_t, cudaStream_t);
size_t paged_attn_workspace_bytes(int, int, int, int, int);
size_t attn_ws_header_bytes(int batch, int n_kv_heads);
int paged_decode_attn(void*, int, int, uint16_t*, uint16_t*, const int*, int, int, const int*,
                      const float*, int, int, int, int, int, float, int, int, void*, int, int,
                      void*, size_t, cudaStream_t);
int rope_kv_append(void*, int, int, uint16_t*, uint16_t*, const int*, int, int, const int*,
                   const float*, int, int, int, int, cudaStream_t);
int add_rmsnorm_f16(float*, const float*, const float*, float, uint16_t*, uint16_t*, int, int,
                    cudaStream_t);
int embed_rmsnorm_f16(const uint16_t*, const int*, float*, const float*, float, uint16_t*,
                      uint16_t*, float*, int, int, cudaStream_t);
size_t tc_gemm_workspace_bytes(int M, int K, int batch, int epilogue);
int tc_gemm(int, const uint16_t*, const uint16_t*, const uint16_t*, int, int, int, void*, int,
            const float*, int, int, int, float*, int*, float*, int, void*, size_t, cudaStream_t,
            const void* pf, size_t pf_bytes);
int tc_gemm_norm(int, const uint16_t*, const uint16_t*, const uint16_t*, int, int, int, void*, int,
                 const float*, int, int, int, float*, int*, void*, size_t, cudaStream_t,
                 const void* pf, size_t pf_bytes, const TcNorm& nrm);
int tc_gemm_multi_store(int, const uint16_t*, const uint16_t*, int, float* const*, int, int, int,
                        int, int, void*, size_t, cudaStream_t, const void* pf, size_t pf_bytes);
int tc_gemm_q(int, int, const void*, const uint16_t*, const uint16_t*, int, int, int, void*, int,
              const float*, int, int, int, void*, size_t, cudaStream_t, float* const*, int,
              const void* pf, size_t pf_bytes);
int tp_allreduce_add_rmsnorm(const float* const*, uint32_t* const*, uint32_t*, int, int, int,
                             float*, const float*, float, uint16_t*, uint16_t*, int, int,
                             long long, int*, cudaStream_t);
int tp_argmax_gather(const float* const*, const int* const*, uint32_t* const*, uint32_t*, int,
                     int, int, int, int*, long long, int*, cudaStream_t);
}  // namespace b2d

// Batches of at least this many sequences run their projections on the tensor cores.
static constexpr int kTcMinBatch = 9;
static constexpr int kMaxTp = 8;
// Bound on a peer-barrier wait (a rank that never arrives turns into B2D_ERR_TIMEOUT).
static constexpr long long kPeerTimeoutNs = 10000000000LL;

using namespace b2d;

struct Layer {
  const float* attn_norm = nullptr;
  const uint16_t* wqkv = nullptr;  // fp16 weights, or the raw q8_32 / q4_32 integers
  const uint16_t* wo = nullptr;
  const float* ffn_norm = nullptr;
  const uint16_t* wgate = nullptr;
  const uint16_t* wup = nullptr;
  const uint16_t* wdown = nullptr;
  uint16_t* k_pages = nullptr;
  uint16_t* v_pages = nullptr;
  int wdt = B2D_F16;  // B2D_F16, B2D_Q8_32 or B2D_Q4_32 (all five projections)
  // fp16 block scales [rows, K/32] of the quantized projections (nullptr for fp16 weights)
  const uint16_t* sqkv = nullptr;
  const uint16_t* so = nullptr;
  const uint16_t* sgate = nullptr;
  const uint16_t* sup = nullptr;
  const uint16_t* sdown = nullptr;
};

struct GraphKey {
  int batch = -1;
  const void* ptrs[6] = {};
  cudaStream_t stream = nullptr;
  bool operator==(const GraphKey& o) const {
    if (batch != o.batch || stream != o.stream) return false;
    for (int i = 0; i < 6; ++i)
      if (ptrs[i] != o.ptrs[i]) return false;
    return true;
  }
};

struct b2d_decoder {
  b2d_model_config cfg{};
  int rank = 0, tp = 1, device = 0;
  ncclComm_t comm = nullptr;
  int hq = 0, hk = 0, fl = 0, qkv_l = 0, lm_rows = 0, lm_stride = 0;
  std::vector<Layer> layers;
  const uint16_t* embed = nullptr;
  const uint16_t* lm_head = nullptr;
  const float* final_norm = nullptr;
  // handle-owned device buffers (one allocation)
  void* arena = nullptr;
  float* x = nullptr;       // [B, D] residual stream, fp32
  float* qkv = nullptr;     // [B, qkv_l]
  float* att = nullptr;     // [B, hq*HD]
  float* hid = nullptr;     // [B, fl]
  float* invf = nullptr;    // [HD/2]
  float* cand_val = nullptr;  // [tp, B]
  int* cand_idx = nullptr;    // [tp, B]
  void* attn_ws = nullptr;
  size_t attn_ws_bytes = 0;
  void* am_ws = nullptr;
  size_t am_ws_bytes = 0;
  // tensor-core path (batch >= kTcMinBatch): activation operands as B2D_F16X2 hi + lo fp16
  // planes (a step of batch B keeps the lo plane B rows after the hi plane) + GEMM workspace
  uint16_t* xn16 = nullptr;   // [2][B, D]   rmsnorm(x) * gamma
  uint16_t* att16 = nullptr;  // [2][B, hq*HD]  attention output
  uint16_t* h16 = nullptr;    // [2][B, fl]  SwiGLU output
  // single-GPU tensor-core step with the RMSNorms folded into the GEMMs (TcNorm): two
  // slice-sum blocks (after the O and the down projection) and the last norm factor per token
  float* nrm_part = nullptr;  // [2][tc_norm_part_floats(D)]
  float* nrm_r = nullptr;     // [B]
  void* tc_ws = nullptr;
  size_t tc_ws_bytes = 0;
  // tensor parallelism: buffers the peers read (one IPC-shared allocation per rank)
  bool peer = false;                   // peer-memory collectives (else NCCL)
  void* peer_arena = nullptr;          // this rank's shared buffers
  void* peer_open[kMaxTp] = {};        // peers' arenas mapped here (nullptr for this rank)
  // row-parallel partial sums [B, D], two alternating buffers: recv[buf][owner][src] is the
  // slot in rank `owner`'s memory that holds rank `src`'s partial (mapped here over IPC)
  float* recv[2][kMaxTp][kMaxTp] = {};
  float* am_val[kMaxTp] = {};          // LM-head (max, index) per token [B]
  int* am_idx[kMaxTp] = {};
  uint32_t* sigs[kMaxTp] = {};         // signal arrays [(B + 1) slots][kMaxTp]
  uint32_t* epochs = nullptr;          // this rank's barrier epochs [(B + 1) slots]
  int* err = nullptr;                  // device error word of the peer kernels
  // graph cache
  cudaGraphExec_t gexec = nullptr;
  GraphKey gkey;
  // device-resident decode loop (b2d_decoder_generate): step + advance, captured once
  int* gen_next = nullptr;  // [B] next tokens of the loop's step (also prefill's last chunk)
  // chunked prefill: positions [2][B] and block-table rows [2][B][max_blocks] of a chunk
  int* pf_ctx = nullptr;
  int* pf_table = nullptr;
  cudaGraphExec_t gen_exec = nullptr;
  GraphKey gen_key;
};

static int nccl_status(ncclResult_t r) { return r == ncclSuccess ? B2D_OK : B2D_ERR_NCCL; }

// Cross-kernel weight prefetch: each projection (and the attention) pulls the leading bytes of
// the next weight-bearing kernel's matrices into L2 at its tail, so HBM keeps streaming through
// the epilogue / launch gap between two kernels.  B2D_L2_PREFETCH_MB caps the bytes per kernel
// (default 16 MB; 0 turns it off), read once.
struct Pf {
  const void* p = nullptr;
  size_t n = 0;
};

static size_t prefetch_cap() {
  static const size_t cap = [] {
    const char* e = std::getenv("B2D_L2_PREFETCH_MB");
    const long v = e ? std::atol(e) : 16;
    return (size_t)(v > 0 ? v : 0) << 20;
  }();
  return cap;
}

// The first min(cap, size) bytes of a [rows, K] matrix stored as wdt (fp16 or 32-block integers).
static Pf pf_mat(const void* W, size_t rows, size_t K, int wdt) {
  const size_t bytes = wdt == B2D_F16 ? rows * K * 2 : (wdt == B2D_Q8_32 ? rows * K : rows * K / 2);
  return Pf{W, std::min(bytes, prefetch_cap()) & ~size_t(15)};
}

static int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return B2D_OK;
  set_cuda_error(e);
  return B2D_ERR_CUDA;
}

static size_t align256(size_t n) { return (n + 255) / 256 * 256; }

// Row-parallel projection (tensor cores) of this rank into buffer `buf`: with peer memory the
// epilogue stores the partial straight into every rank's receive slot for this rank (the data
// crosses NVLink while the GEMM finishes), else into the local slot for NCCL.
static int tp_partial(b2d_decoder* h, int buf, int wdt, const uint16_t* W, const uint16_t* scales,
                      const uint16_t* X, int K, int B, cudaStream_t s, Pf pf) {
  const int D = h->cfg.dim;
  float* ys[kMaxTp];
  int n_ys = 0;
  if (h->peer)
    for (int r = 0; r < h->tp; ++r) ys[n_ys++] = h->recv[buf][r][h->rank];
  float* mine = h->peer ? nullptr : h->recv[buf][h->rank][h->rank];
  if (wdt != B2D_F16)
    return tc_gemm_q(B2D_F16X2, wdt, W, scales, X, K, B2D_EPI_STORE, B2D_F32, mine, D, nullptr, D,
                     K, B, h->tc_ws, h->tc_ws_bytes, s, ys, n_ys, pf.p, pf.n);
  if (h->peer)
    return tc_gemm_multi_store(B2D_F16X2, W, X, K, ys, n_ys, D, D, K, B, h->tc_ws,
                               h->tc_ws_bytes, s, pf.p, pf.n);
  return tc_gemm(B2D_F16X2, W, nullptr, X, K, B2D_EPI_STORE, B2D_F32, mine, D, nullptr, D, K, B,
                 nullptr, nullptr, nullptr, 0, h->tc_ws, h->tc_ws_bytes, s, pf.p, pf.n);
}

// One projection of the tensor-core step: y = epilogue(W x) with x as B2D_F16X2 planes, on the
// fp16 or the quantized tcgen05 GEMM by the layer's weight type.
static int tc_proj(b2d_decoder* h, int wdt, const uint16_t* W, const uint16_t* scales,
                   const uint16_t* X, int K, int epi, int y_dtype, void* y, int ldy, int M,
                   const float* aux, int B, cudaStream_t s, Pf pf) {
  if (wdt != B2D_F16)
    return tc_gemm_q(B2D_F16X2, wdt, W, scales, X, K, epi, y_dtype, y, ldy, aux, M, K, B, h->tc_ws,
                     h->tc_ws_bytes, s, nullptr, 0, pf.p, pf.n);
  return tc_gemm(B2D_F16X2, W, nullptr, X, K, epi, y_dtype, y, ldy, aux, M, K, B, nullptr,
                 nullptr, nullptr, 0, h->tc_ws, h->tc_ws_bytes, s, pf.p, pf.n);
}

// Sum the ranks' row-parallel partials (buffer `buf`) into the residual x; with gamma, also
// write rmsnorm(x) * gamma to out16 as B2D_F16X2 planes of B rows.  `pushed`: every rank's producer already stored its
// partial into this rank's receive slots (the tensor-core path), so the sum reads local memory;
// otherwise each rank's partial sits in its own slot and the sum reads it over NVLink.
static int tp_reduce(b2d_decoder* h, int buf, const float* gamma, uint16_t* out16, int B,
                     bool pushed, cudaStream_t s) {
  const int D = h->cfg.dim;
  if (h->peer) {
    float* parts[kMaxTp];
    for (int r = 0; r < h->tp; ++r) parts[r] = pushed ? h->recv[buf][h->rank][r] : h->recv[buf][r][r];
    return tp_allreduce_add_rmsnorm(parts, h->sigs, h->epochs, h->rank, h->tp, 0, h->x, gamma,
                                    h->cfg.eps, out16, out16 ? out16 + (size_t)B * D : nullptr, D,
                                    B, kPeerTimeoutNs, h->err, s);
  }
  float* mine = h->recv[buf][h->rank][h->rank];
  B2D_TRY(nccl_status(ncclAllReduce(mine, mine, (size_t)B * D, ncclFloat, ncclSum, h->comm, s)));
  return gamma ? add_rmsnorm_f16(h->x, mine, gamma, h->cfg.eps, out16, out16 + (size_t)B * D, B,
                                 D, s)
               : add_f32(h->x, mine, (size_t)B * D, s);
}

// Combine the ranks' LM-head (max, index) pairs into next_tokens.
static int tp_argmax(b2d_decoder* h, int B, int* next_tokens, cudaStream_t s) {
  if (h->peer)
    return tp_argmax_gather(h->am_val, h->am_idx, h->sigs, h->epochs, h->rank, h->tp,
                            h->cfg.max_batch, B, next_tokens, kPeerTimeoutNs, h->err, s);
  B2D_TRY(nccl_status(ncclGroupStart()));
  B2D_TRY(nccl_status(ncclAllGather(h->am_val[h->rank], h->cand_val, B, ncclFloat, h->comm, s)));
  B2D_TRY(nccl_status(ncclAllGather(h->am_idx[h->rank], h->cand_idx, B, ncclInt32, h->comm, s)));
  B2D_TRY(nccl_status(ncclGroupEnd()));
  return argmax_combine(h->cand_val, h->cand_idx, h->tp, B, next_tokens, s);
}

// RoPE + KV append and attention of one layer.  In a decode step each token's K/V is appended by
// the attention kernel itself.  In a prefill chunk the tokens are consecutive positions of one
// sequence and each attends to the ones before it, so the whole chunk's K/V is written first
// (rope_kv_append, a plain launch: it starts after the QKV projection has completed) and the
// attention then only reads the pages.
static int layer_attention(b2d_decoder* h, const Layer& L, const int* ctx_lens,
                           const int* block_table, int B, bool prefill, void* out, int out_dtype,
                           cudaStream_t s) {
  const b2d_model_config& c = h->cfg;
  const int HD = c.head_dim;
  if (prefill)
    B2D_TRY(rope_kv_append(h->qkv, B2D_F32, h->qkv_l, L.k_pages, L.v_pages, block_table,
                           c.max_blocks, c.n_blocks, ctx_lens, h->invf, h->hq, h->hk, HD, B, s));
  return paged_decode_attn(h->qkv, B2D_F32, h->qkv_l, L.k_pages, L.v_pages, block_table,
                           c.max_blocks, c.n_blocks, ctx_lens, h->invf, h->hq, h->hk, HD, B,
                           c.max_ctx, 0.f, 0, prefill ? 0 : 1, out, out_dtype, h->hq * HD,
                           h->attn_ws, h->attn_ws_bytes, s);
}

// Tensor-core step (batch >= kTcMinBatch): every projection's activation operand enters as
// B2D_F16X2 hi + lo fp16 planes (fp32 precision, like the reference's fp32 activations), with
// RMSNorm fused into the producer of the operand; weights are read once per step.
// next_tokens == nullptr skips the LM head (a prefill chunk whose outputs nobody reads).
static int enqueue_step_tc(b2d_decoder* h, const int* tokens, const int* ctx_lens,
                           const int* block_table, int B, int* next_tokens, float* logits,
                           cudaStream_t s, bool prefill) {
  const b2d_model_config& c = h->cfg;
  const int D = c.dim, HQD = h->hq * c.head_dim;
  const bool tpar = h->tp > 1;
  void* ws = h->tc_ws;
  const size_t wsb = h->tc_ws_bytes;
  constexpr int X2 = B2D_F16X2;
  uint16_t* const xn_lo = h->xn16 + (size_t)B * D;  // lo planes of this batch's operands
  // Single GPU, fp16 weights: the RMSNorms after the O and the down projection are folded into
  // the GEMMs (TcNorm) -- the projection emits x * gamma and slice sums of x^2, the next GEMM
  // scales its product by the norm factor -- instead of a separate add_rmsnorm launch.
  // B2D_NORM_FOLD=0 keeps the separate launches (read once).
  static const bool fold_env = [] {
    const char* e = std::getenv("B2D_NORM_FOLD");
    return !(e && std::atoi(e) == 0);
  }();
  const bool fold = fold_env && !tpar && D % 128 == 0;
  auto fold_into = [&](int l) {  // may the GEMMs of layer l (n_layers: the LM head) consume one
    return fold && (l >= c.n_layers || h->layers[l].wdt == B2D_F16);
  };
  float* const part_o = h->nrm_part;  // slice sums after O (read by gate/up)
  float* const part_down = h->nrm_part + align256(tc_norm_part_floats(D) * 4) / 4;  // after down
  const float* pending = nullptr;  // slice sums the next QKV / LM head consumes (else normalized)
  bool r_ok = fold;                // h->nrm_r holds this step's last norm factor per token
  B2D_TRY(embed_rmsnorm_f16(h->embed, tokens, h->x, h->layers[0].attn_norm, c.eps, h->xn16, xn_lo,
                            fold ? h->nrm_r : nullptr, D, B, s));
  for (int l = 0; l < c.n_layers; ++l) {
    const Layer& L = h->layers[l];
    const float* next_norm = l + 1 < c.n_layers ? h->layers[l + 1].attn_norm : h->final_norm;
    const int wd = L.wdt;
    const bool f = fold_into(l);
    // what each kernel prefetches into L2: the next weight-bearing kernel's matrices
    const Pf pf_o = pf_mat(L.wo, D, HQD, wd);
    const Pf pf_up = pf_mat(L.wup, h->fl, D, wd);
    const Pf pf_gate = pf_mat(L.wgate, h->fl, D, wd);
    const Pf pf_down = pf_mat(L.wdown, D, h->fl, wd);
    const Pf pf_next = l + 1 < c.n_layers
                           ? pf_mat(h->layers[l + 1].wqkv, h->qkv_l, D, h->layers[l + 1].wdt)
                           : (next_tokens ? pf_mat(h->lm_head, h->lm_rows, D, B2D_F16) : Pf{});
    // QKV (column-parallel)
    if (pending) {
      TcNorm n;
      n.part_in = pending;
      n.r_out = h->nrm_r;
      n.eps = c.eps;
      B2D_TRY(tc_gemm_norm(X2, L.wqkv, nullptr, h->xn16, D, B2D_EPI_STORE, B2D_F32, h->qkv,
                           h->qkv_l, nullptr, h->qkv_l, D, B, nullptr, nullptr, ws, wsb, s,
                           pf_o.p, pf_o.n, n));
      r_ok = true;
    } else {
      B2D_TRY(tc_proj(h, wd, L.wqkv, L.sqkv, h->xn16, D, B2D_EPI_STORE, B2D_F32, h->qkv, h->qkv_l,
                      h->qkv_l, nullptr, B, s, pf_o));
      if (l > 0) r_ok = false;
    }
    // RoPE + KV append + split-K attention -> hi/lo operand of the O projection
    B2D_TRY(layer_attention(h, L, ctx_lens, block_table, B, prefill, h->att16, X2, s));
    // O projection (row-parallel) + residual, then RMSNorm(ffn) -> hi/lo
    if (f) {
      TcNorm n;
      n.gamma = L.ffn_norm;
      n.planes = h->xn16;
      n.part_out = part_o;
      n.r_prev = r_ok ? h->nrm_r : nullptr;
      B2D_TRY(tc_gemm_norm(X2, L.wo, nullptr, h->att16, HQD, B2D_EPI_ADD, B2D_F32, h->x, D,
                           nullptr, D, HQD, B, nullptr, nullptr, ws, wsb, s, pf_up.p, pf_up.n, n));
    } else if (!tpar) {
      B2D_TRY(tc_proj(h, wd, L.wo, L.so, h->att16, HQD, B2D_EPI_ADD, B2D_F32, h->x, D, D,
                      nullptr, B, s, pf_up));
      B2D_TRY(add_rmsnorm_f16(h->x, nullptr, L.ffn_norm, c.eps, h->xn16, xn_lo, B, D, s));
    } else {
      B2D_TRY(tp_partial(h, 0, wd, L.wo, L.so, h->att16, HQD, B, s, pf_up));
      B2D_TRY(tp_reduce(h, 0, L.ffn_norm, h->xn16, B, h->peer, s));
    }
    // gate/up SwiGLU (column-parallel) -> hi/lo.  fp16 weights: one dual-matrix GEMM; quantized
    // weights: the up projection into hid (fp32), then the gate projection times it.
    if (f) {
      TcNorm n;
      n.part_in = part_o;
      n.r_out = h->nrm_r;
      n.eps = c.eps;
      B2D_TRY(tc_gemm_norm(X2, L.wgate, L.wup, h->xn16, D, B2D_EPI_SWIGLU, X2, h->h16, h->fl,
                           nullptr, h->fl, D, B, nullptr, nullptr, ws, wsb, s, pf_down.p,
                           pf_down.n, n));
      r_ok = true;
    } else if (wd == B2D_F16) {
      B2D_TRY(tc_gemm(X2, L.wgate, L.wup, h->xn16, D, B2D_EPI_SWIGLU, X2, h->h16, h->fl, nullptr,
                      h->fl, D, B, nullptr, nullptr, nullptr, 0, ws, wsb, s, pf_down.p, pf_down.n));
      r_ok = false;
    } else {
      B2D_TRY(tc_proj(h, wd, L.wup, L.sup, h->xn16, D, B2D_EPI_STORE, B2D_F32, h->hid, h->fl,
                      h->fl, nullptr, B, s, pf_gate));
      B2D_TRY(tc_proj(h, wd, L.wgate, L.sgate, h->xn16, D, B2D_EPI_SILU_MUL, X2, h->h16, h->fl,
                      h->fl, h->hid, B, s, pf_down));
      r_ok = false;
    }
    // down (row-parallel) + residual, then the next RMSNorm -> hi/lo
    pending = nullptr;
    if (f && fold_into(l + 1)) {
      TcNorm n;
      n.gamma = next_norm;
      n.planes = h->xn16;
      n.part_out = part_down;
      n.r_prev = h->nrm_r;  // the gate/up GEMM's factor
      B2D_TRY(tc_gemm_norm(X2, L.wdown, nullptr, h->h16, h->fl, B2D_EPI_ADD, B2D_F32, h->x, D,
                           nullptr, D, h->fl, B, nullptr, nullptr, ws, wsb, s, pf_next.p,
                           pf_next.n, n));
      pending = part_down;
    } else if (!tpar) {
      B2D_TRY(tc_proj(h, wd, L.wdown, L.sdown, h->h16, h->fl, B2D_EPI_ADD, B2D_F32, h->x, D, D,
                      nullptr, B, s, pf_next));
      B2D_TRY(add_rmsnorm_f16(h->x, nullptr, next_norm, c.eps, h->xn16, xn_lo, B, D, s));
    } else {
      B2D_TRY(tp_partial(h, 1, wd, L.wdown, L.sdown, h->h16, h->fl, B, s, pf_next));
      B2D_TRY(tp_reduce(h, 1, next_norm, h->xn16, B, h->peer, s));
    }
  }
  // LM head (vocab-parallel) + argmax
  if (!next_tokens) return B2D_OK;
  const int offset = h->rank * h->lm_stride;
  if (pending) {
    TcNorm n;
    n.part_in = pending;
    n.eps = c.eps;
    B2D_TRY(tc_gemm_norm(X2, h->lm_head, nullptr, h->xn16, D, B2D_EPI_ARGMAX, B2D_F32, nullptr, 0,
                         nullptr, h->lm_rows, D, B, logits, next_tokens, ws, wsb, s, nullptr, 0,
                         n));
  } else if (!tpar) {
    B2D_TRY(tc_gemm(X2, h->lm_head, nullptr, h->xn16, D, B2D_EPI_ARGMAX, B2D_F32, nullptr, 0,
                    nullptr, h->lm_rows, D, B, logits, next_tokens, nullptr, 0, ws, wsb, s,
                    nullptr, 0));
  } else {
    B2D_TRY(tc_gemm(X2, h->lm_head, nullptr, h->xn16, D, B2D_EPI_ARGMAX, B2D_F32, nullptr, 0,
                    nullptr, h->lm_rows, D, B, logits, h->am_idx[h->rank], h->am_val[h->rank],
                    offset, ws, wsb, s, nullptr, 0));
    B2D_TRY(tp_argmax(h, B, next_tokens, s));
  }
  return B2D_OK;
}

// A prefill chunk's per-row inputs: row b is position pos0 + b of the sequence whose block-table
// row is seq_table (every row of the chunk reads and writes the same pages).
__global__ void prefill_chunk_kernel(const int* seq_table, int max_blocks, int pos0, int nb,
                                     int* ctx, int* table) {
  const int b = blockIdx.x;
  if (b >= nb) return;
  if (threadIdx.x == 0) ctx[b] = pos0 + b;
  for (int j = threadIdx.x; j < max_blocks; j += blockDim.x)
    table[(size_t)b * max_blocks + j] = seq_table[j];
}

// Device-resident loop: after a step, the next tokens become the inputs of the following step,
// every position advances by one, and the tokens are appended to a ring the host reads later.
__global__ void advance_kernel(int* tokens, int* ctx_lens, const int* next, int* ring,
                               int* ring_count, int ring_steps, int B) {
  const int row = *ring_count % ring_steps;
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const int t = next[b];
    tokens[b] = t;
    ctx_lens[b] += 1;
    ring[(size_t)row * B + b] = t;
  }
  __syncthreads();
  if (threadIdx.x == 0) *ring_count += 1;
}

// Enqueue one decode step on `s` (no synchronization, graph-capturable).
static int enqueue_step(b2d_decoder* h, const int* tokens, const int* ctx_lens,
                        const int* block_table, int B, int* next_tokens, float* logits,
                        cudaStream_t s, bool prefill = false) {
  if (B >= kTcMinBatch)
    return enqueue_step_tc(h, tokens, ctx_lens, block_table, B, next_tokens, logits, s, prefill);
  const b2d_model_config& c = h->cfg;
  const int D = c.dim, HD = c.head_dim;
  const bool tpar = h->tp > 1;
  B2D_TRY(embed_f16(h->embed, tokens, h->x, D, B, s));
  for (int l = 0; l < c.n_layers; ++l) {
    const Layer& L = h->layers[l];
    const int wd = L.wdt;
    // RMSNorm + QKV (column-parallel: this rank's heads)
    B2D_TRY(gemv_dispatch(wd, L.wqkv, L.sqkv, nullptr, nullptr, B2D_F32, h->x, D, L.attn_norm,
                          c.eps, B2D_EPI_STORE, B2D_F32, h->qkv, h->qkv_l, nullptr, h->qkv_l, D, B,
                          s));
    // RoPE + KV append + split-K GQA attention over the paged cache
    B2D_TRY(layer_attention(h, L, ctx_lens, block_table, B, prefill, h->att, B2D_F32, s));
    // O projection (row-parallel) + residual
    if (!tpar) {
      B2D_TRY(gemv_dispatch(wd, L.wo, L.so, nullptr, nullptr, B2D_F32, h->att, h->hq * HD, nullptr,
                            0.f, B2D_EPI_ADD, B2D_F32, h->x, D, nullptr, D, h->hq * HD, B, s));
    } else {
      B2D_TRY(gemv_dispatch(wd, L.wo, L.so, nullptr, nullptr, B2D_F32, h->att, h->hq * HD, nullptr,
                            0.f, B2D_EPI_STORE, B2D_F32, h->recv[0][h->rank][h->rank], D, nullptr,
                            D, h->hq * HD, B, s));
      B2D_TRY(tp_reduce(h, 0, nullptr, nullptr, B, false, s));
    }
    // RMSNorm + gate/up SwiGLU (column-parallel: this rank's FFN rows)
    B2D_TRY(gemv_dispatch(wd, L.wgate, L.sgate, L.wup, L.sup, B2D_F32, h->x, D, L.ffn_norm, c.eps,
                          B2D_EPI_SWIGLU, B2D_F32, h->hid, h->fl, nullptr, h->fl, D, B, s));
    // down projection (row-parallel) + residual
    if (!tpar) {
      B2D_TRY(gemv_dispatch(wd, L.wdown, L.sdown, nullptr, nullptr, B2D_F32, h->hid, h->fl, nullptr,
                            0.f, B2D_EPI_ADD, B2D_F32, h->x, D, nullptr, D, h->fl, B, s));
    } else {
      B2D_TRY(gemv_dispatch(wd, L.wdown, L.sdown, nullptr, nullptr, B2D_F32, h->hid, h->fl,
                            nullptr, 0.f, B2D_EPI_STORE, B2D_F32, h->recv[1][h->rank][h->rank], D,
                            nullptr, D, h->fl, B, s));
      B2D_TRY(tp_reduce(h, 1, nullptr, nullptr, B, false, s));
    }
  }
  // final RMSNorm + LM head (vocab-parallel) + argmax
  if (!next_tokens) return B2D_OK;
  const int offset = h->rank * h->lm_stride;  // first vocab row of this rank
  if (!tpar) {
    B2D_TRY(lm_head_argmax(h->lm_head, h->x, D, h->final_norm, c.eps, h->lm_rows, D, B, 0,
                           logits, next_tokens, nullptr, h->am_ws, h->am_ws_bytes, s));
  } else {
    B2D_TRY(lm_head_argmax(h->lm_head, h->x, D, h->final_norm, c.eps, h->lm_rows, D, B, offset,
                           logits, h->am_idx[h->rank], h->am_val[h->rank], h->am_ws,
                           h->am_ws_bytes, s));
    B2D_TRY(tp_argmax(h, B, next_tokens, s));
  }
  return B2D_OK;
}

// Tensor-parallel buffers shared with the peers: receive slots for every rank's partial sums
// (2 x tp x [B, D] fp32), LM-head (max, index) [B] and the signal array.  With CUDA IPC every rank maps every peer's allocation (handles are
// exchanged with one ncclAllGather); if any rank cannot, or B2D_TP_COLLECTIVE=nccl, all ranks
// keep their buffers local and use NCCL collectives instead (decided together: ncclMin).
static int setup_peers(b2d_decoder* h) {
  const int B = h->cfg.max_batch, D = h->cfg.dim, tp = h->tp;
  const size_t part_b = align256((size_t)B * D * 4), am_b = align256((size_t)B * 4);
  const size_t sig_b = align256((size_t)(B + 1) * kMaxTp * 4);
  const size_t recv_b = 2 * (size_t)tp * part_b;
  const size_t total = recv_b + 2 * am_b + sig_b;
  B2D_TRY(cuda_status(cudaMalloc(&h->peer_arena, total)));
  B2D_TRY(cuda_status(cudaMemset(h->peer_arena, 0, total)));
  B2D_TRY(cuda_status(cudaDeviceSynchronize()));  // signals are zero before any peer can write
  char* base[kMaxTp] = {};
  base[h->rank] = static_cast<char*>(h->peer_arena);
  const char* env = std::getenv("B2D_TP_COLLECTIVE");
  int ok = !(env && std::strcmp(env, "nccl") == 0);
  cudaIpcMemHandle_t mine;
  if (ok && cudaIpcGetMemHandle(&mine, h->peer_arena) != cudaSuccess) ok = 0;
  cudaGetLastError();
  // exchange the handles (and whether this rank can take part) over the communicator
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  std::vector<char> all(hb * tp, 0);
  char* dev = nullptr;
  B2D_TRY(cuda_status(cudaMalloc(&dev, hb * tp + 16)));
  int* dok = reinterpret_cast<int*>(dev + hb * tp);
  int st = B2D_OK;
  if (ok) cudaMemcpy(dev + hb * h->rank, &mine, hb, cudaMemcpyHostToDevice);
  if (ncclAllGather(dev + hb * h->rank, dev, hb, ncclChar, h->comm, nullptr) != ncclSuccess)
    st = B2D_ERR_NCCL;
  if (st == B2D_OK) st = cuda_status(cudaMemcpy(all.data(), dev, hb * tp, cudaMemcpyDeviceToHost));
  for (int r = 0; st == B2D_OK && ok && r < tp; ++r) {
    if (r == h->rank) continue;
    cudaIpcMemHandle_t hr;
    memcpy(&hr, all.data() + hb * r, hb);
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, hr, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      ok = 0;
      break;
    }
    h->peer_open[r] = p;
    base[r] = static_cast<char*>(p);
  }
  if (st == B2D_OK) {
    cudaMemcpy(dok, &ok, sizeof(int), cudaMemcpyHostToDevice);
    if (ncclAllReduce(dok, dok, 1, ncclInt32, ncclMin, h->comm, nullptr) != ncclSuccess)
      st = B2D_ERR_NCCL;
    else
      st = cuda_status(cudaMemcpy(&ok, dok, sizeof(int), cudaMemcpyDeviceToHost));
  }
  cudaFree(dev);
  B2D_TRY(st);
  h->peer = ok != 0;
  for (int r = 0; r < tp; ++r) {
    char* b = h->peer ? base[r] : (r == h->rank ? base[r] : nullptr);
    if (!b) continue;
    for (int buf = 0; buf < 2; ++buf)
      for (int src = 0; src < tp; ++src)
        h->recv[buf][r][src] = reinterpret_cast<float*>(b + ((size_t)buf * tp + src) * part_b);
    h->am_val[r] = reinterpret_cast<float*>(b + recv_b);
    h->am_idx[r] = reinterpret_cast<int*>(b + recv_b + am_b);
    h->sigs[r] = reinterpret_cast<uint32_t*>(b + recv_b + 2 * am_b);
  }
  if (!h->peer)
    for (int r = 0; r < kMaxTp; ++r)
      if (h->peer_open[r]) {
        cudaIpcCloseMemHandle(h->peer_open[r]);
        h->peer_open[r] = nullptr;
      }
  return B2D_OK;
}

extern "C" {

int b2d_nccl_unique_id_bytes(void) { return (int)sizeof(ncclUniqueId); }

int b2d_nccl_get_unique_id(void* out_host) {
  if (!out_host) return B2D_ERR_NULL;
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return B2D_ERR_NCCL;
  memcpy(out_host, &id, sizeof(id));
  return B2D_OK;
}

int b2d_decoder_create(const b2d_model_config* cfg, int tp_rank, int tp_size,
                       const void* nccl_id, b2d_decoder** out) {
  if (!cfg || !out) return B2D_ERR_NULL;
  *out = nullptr;
  const b2d_model_config& c = *cfg;
  if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size) return B2D_ERR_SHAPE;
  if (c.dim <= 0 || c.n_layers <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.head_dim <= 0 ||
      c.ffn_dim <= 0 || c.vocab <= 0 || c.max_batch <= 0 || c.max_ctx <= 0 ||
      c.max_blocks * 16 < c.max_ctx || c.n_blocks <= 0)
    return B2D_ERR_SHAPE;
  if (c.n_kv_heads % tp_size || c.n_heads % c.n_kv_heads || c.ffn_dim % tp_size)
    return B2D_ERR_SHAPE;
  if (tp_size > 1 && !nccl_id) return B2D_ERR_NULL;
  b2d_decoder* h = new b2d_decoder();
  h->cfg = c;
  h->rank = tp_rank;
  h->tp = tp_size;
  cudaGetDevice(&h->device);
  h->hq = c.n_heads / tp_size;
  h->hk = c.n_kv_heads / tp_size;
  h->fl = c.ffn_dim / tp_size;
  h->qkv_l = (h->hq + 2 * h->hk) * c.head_dim;
  h->lm_stride = (c.vocab + tp_size - 1) / tp_size;
  h->lm_rows = std::min(h->lm_stride, c.vocab - tp_rank * h->lm_stride);
  if (h->lm_rows <= 0) {
    delete h;
    return B2D_ERR_SHAPE;
  }
  h->layers.resize(c.n_layers);
  const int B = c.max_batch, D = c.dim;
  // the split-K chunk size depends on the batch, so size for the worst batch of any step
  h->attn_ws_bytes = 0;
  for (int b = 1; b <= B; ++b)
    h->attn_ws_bytes = std::max(h->attn_ws_bytes,
                                paged_attn_workspace_bytes(b, h->hq, h->hk, c.head_dim, c.max_ctx));
  h->am_ws_bytes = lm_head_argmax_workspace_bytes(h->lm_rows, B);
  // tensor-core GEMM workspace: the largest of the step's call sites, for both N tiles
  h->tc_ws_bytes = 0;
  if (B >= kTcMinBatch) {
    const int HQD = h->hq * c.head_dim;
    const int shapes[5][3] = {{h->qkv_l, D, B2D_EPI_STORE},
                              {D, HQD, B2D_EPI_ADD},
                              {h->fl, D, B2D_EPI_SWIGLU},
                              {D, h->fl, B2D_EPI_ADD},
                              {h->lm_rows, D, B2D_EPI_ARGMAX}};
    for (int b : {std::min(B, 16), B})
      for (auto& sh : shapes)
        h->tc_ws_bytes = std::max(h->tc_ws_bytes, tc_gemm_workspace_bytes(sh[0], sh[1], b, sh[2]));
  }
  size_t sizes[] = {
      (size_t)B * D * 4,          (size_t)B * h->qkv_l * 4, (size_t)B * h->hq * c.head_dim * 4,
      (size_t)B * h->fl * 4,      (size_t)(B + 1) * 4,      (size_t)c.head_dim / 2 * 4,
      (size_t)tp_size * B * 4,    (size_t)tp_size * B * 4,  (size_t)4,  (size_t)B * 4,
      (size_t)2 * B * 4,          (size_t)2 * B * c.max_blocks * 4,
      h->attn_ws_bytes,           h->am_ws_bytes,
      (size_t)2 * B * D * 2,      (size_t)2 * B * h->hq * c.head_dim * 2, (size_t)2 * B * h->fl * 2,
      2 * align256(tc_norm_part_floats(D) * 4), (size_t)B * 4,
      h->tc_ws_bytes};
  size_t total = 0;
  for (size_t s : sizes) total += align256(s);
  int st = cuda_status(cudaMalloc(&h->arena, total));
  if (st != B2D_OK) {
    delete h;
    return st;
  }
  cudaMemset(h->arena, 0, total);
  char* p = static_cast<char*>(h->arena);
  void** slots[] = {(void**)&h->x,        (void**)&h->qkv,      (void**)&h->att,
                    (void**)&h->hid,      (void**)&h->epochs,   (void**)&h->invf,
                    (void**)&h->cand_val, (void**)&h->cand_idx, (void**)&h->err,
                    (void**)&h->gen_next,
                    (void**)&h->pf_ctx,   (void**)&h->pf_table,
                    (void**)&h->attn_ws,  (void**)&h->am_ws,
                    (void**)&h->xn16,     (void**)&h->att16,    (void**)&h->h16,
                    (void**)&h->nrm_part, (void**)&h->nrm_r,
                    (void**)&h->tc_ws};
  static_assert(sizeof(slots) / sizeof(slots[0]) == sizeof(sizes) / sizeof(sizes[0]),
                "one slot per buffer size");
  for (size_t i = 0; i < sizeof(sizes) / sizeof(sizes[0]); ++i) {
    *slots[i] = p;
    p += align256(sizes[i]);
  }
  std::vector<float> invf(c.head_dim / 2);
  for (int i = 0; i < c.head_dim / 2; ++i)
    invf[i] = (float)(1.0 / std::pow(c.rope_theta, (double)(2 * i) / (double)c.head_dim));
  st = cuda_status(cudaMemcpy(h->invf, invf.data(), invf.size() * 4, cudaMemcpyHostToDevice));
  if (st == B2D_OK && tp_size > 1) {
    if (tp_size > kMaxTp) st = B2D_ERR_SHAPE;
    ncclUniqueId id;
    memcpy(&id, nccl_id, sizeof(id));
    if (st == B2D_OK && ncclCommInitRank(&h->comm, tp_size, id, tp_rank) != ncclSuccess)
      st = B2D_ERR_NCCL;
    if (st == B2D_OK) st = setup_peers(h);
  }
  if (st != B2D_OK) {
    b2d_decoder_destroy(h);
    return st;
  }
  *out = h;
  return B2D_OK;
}

int b2d_decoder_destroy(b2d_decoder* h) {
  if (!h) return B2D_OK;
  if (h->gexec) cudaGraphExecDestroy(h->gexec);
  if (h->gen_exec) cudaGraphExecDestroy(h->gen_exec);
  if (h->comm && h->peer) {
    // every rank stops reading its peers' buffers before any rank frees its own
    cudaDeviceSynchronize();
    ncclAllReduce(h->err, h->err, 1, ncclInt32, ncclMax, h->comm, nullptr);
    cudaDeviceSynchronize();
  }
  for (int r = 0; r < kMaxTp; ++r)
    if (h->peer_open[r]) cudaIpcCloseMemHandle(h->peer_open[r]);
  if (h->comm) ncclCommDestroy(h->comm);
  if (h->peer_arena) cudaFree(h->peer_arena);
  if (h->arena) cudaFree(h->arena);
  delete h;
  return B2D_OK;
}

int b2d_decoder_set_inv_freq(b2d_decoder* h, const float* inv_freq_host, int n) {
  if (!h || !inv_freq_host) return B2D_ERR_NULL;
  if (n != h->cfg.head_dim / 2) return B2D_ERR_SHAPE;
  // same device buffer: a captured step graph picks the new values up
  return cuda_status(cudaMemcpy(h->invf, inv_freq_host, (size_t)n * 4, cudaMemcpyHostToDevice));
}

int b2d_decoder_peer_collectives(const b2d_decoder* h) { return h && h->peer ? 1 : 0; }

int b2d_decoder_error(b2d_decoder* h) {
  if (!h) return B2D_ERR_NULL;
  // the steps may have run on any stream of this device (engine streams do not wait for the
  // legacy default stream): wait for all of them before reading the error words
  B2D_TRY(cuda_status(cudaDeviceSynchronize()));
  // error words: the peer barriers' (h->err), the attention's and the tensor-core GEMMs'
  // (first int of their workspaces; each of their bounded waits sets it when it gives up)
  int words[3] = {0, 0, 0};
  B2D_TRY(cuda_status(cudaMemcpy(&words[0], h->err, sizeof(int), cudaMemcpyDeviceToHost)));
  B2D_TRY(cuda_status(cudaMemcpy(&words[1], h->attn_ws, sizeof(int), cudaMemcpyDeviceToHost)));
  if (h->tc_ws_bytes)  // only decoders whose batch reaches the tensor-core path have one
    B2D_TRY(cuda_status(cudaMemcpy(&words[2], h->tc_ws, sizeof(int), cudaMemcpyDeviceToHost)));
  if (!(words[0] | words[1] | words[2])) return B2D_OK;
  // A CTA whose wait gave up returned before its arrival on the split-K / argmax counters, so
  // besides the error words the counters are reset too: later steps start from zero again.
  B2D_TRY(cuda_status(cudaMemset(h->err, 0, sizeof(int))));
  B2D_TRY(cuda_status(
      cudaMemset(h->attn_ws, 0, attn_ws_header_bytes(h->cfg.max_batch, h->hk))));
  if (h->tc_ws_bytes)
    B2D_TRY(cuda_status(cudaMemset(h->tc_ws, 0, std::min<size_t>(h->tc_ws_bytes, 512))));
  B2D_TRY(cuda_status(cudaDeviceSynchronize()));
  return words[0] ? words[0] : B2D_ERR_TIMEOUT;
}

int b2d_decoder_set_layer(b2d_decoder* h, int layer, const float* attn_norm,
                          const uint16_t* wqkv, const uint16_t* wo, const float* ffn_norm,
                          const uint16_t* wgate, const uint16_t* wup, const uint16_t* wdown,
                          uint16_t* k_pages, uint16_t* v_pages) {
  if (!h) return B2D_ERR_NULL;
  if (layer < 0 || layer >= h->cfg.n_layers) return B2D_ERR_SHAPE;
  if (!attn_norm || !wqkv || !wo || !ffn_norm || !wgate || !wup || !wdown || !k_pages || !v_pages)
    return B2D_ERR_NULL;
  Layer& L = h->layers[layer];
  L = Layer{attn_norm, wqkv, wo, ffn_norm, wgate, wup, wdown, k_pages, v_pages};
  if (h->gexec) {  // pointers changed: the captured graph is stale
    cudaGraphExecDestroy(h->gexec);
    h->gexec = nullptr;
    h->gkey = GraphKey();
  }
  if (h->gen_exec) {
    cudaGraphExecDestroy(h->gen_exec);
    h->gen_exec = nullptr;
    h->gen_key = GraphKey();
  }
  return B2D_OK;
}

int b2d_decoder_set_layer_q(b2d_decoder* h, int layer, int w_dtype, const float* attn_norm,
                            const void* wqkv, const uint16_t* wqkv_scales, const void* wo,
                            const uint16_t* wo_scales, const float* ffn_norm, const void* wgate,
                            const uint16_t* wgate_scales, const void* wup,
                            const uint16_t* wup_scales, const void* wdown,
                            const uint16_t* wdown_scales, uint16_t* k_pages, uint16_t* v_pages) {
  if (!h) return B2D_ERR_NULL;
  if (w_dtype == B2D_F16)
    return b2d_decoder_set_layer(h, layer, attn_norm, static_cast<const uint16_t*>(wqkv),
                                 static_cast<const uint16_t*>(wo), ffn_norm,
                                 static_cast<const uint16_t*>(wgate),
                                 static_cast<const uint16_t*>(wup),
                                 static_cast<const uint16_t*>(wdown), k_pages, v_pages);
  if (w_dtype != B2D_Q8_32 && w_dtype != B2D_Q4_32) return B2D_ERR_UNSUPPORTED;
  if (!wqkv_scales || !wo_scales || !wgate_scales || !wup_scales || !wdown_scales)
    return B2D_ERR_NULL;
  // every projection's K must hold whole 32-element blocks (the row-parallel shards included)
  const b2d_model_config& c = h->cfg;
  if (c.dim % 32 || (h->hq * c.head_dim) % 32 || h->fl % 32) return B2D_ERR_SHAPE;
  B2D_TRY(b2d_decoder_set_layer(h, layer, attn_norm, static_cast<const uint16_t*>(wqkv),
                                static_cast<const uint16_t*>(wo), ffn_norm,
                                static_cast<const uint16_t*>(wgate),
                                static_cast<const uint16_t*>(wup),
                                static_cast<const uint16_t*>(wdown), k_pages, v_pages));
  Layer& L = h->layers[layer];
  L.wdt = w_dtype;
  L.sqkv = wqkv_scales;
  L.so = wo_scales;
  L.sgate = wgate_scales;
  L.sup = wup_scales;
  L.sdown = wdown_scales;
  return B2D_OK;
}

int b2d_decoder_set_head(b2d_decoder* h, const uint16_t* embed, const uint16_t* lm_head,
                         int lm_rows, const float* final_norm) {
  if (!h) return B2D_ERR_NULL;
  if (!embed || !lm_head || !final_norm) return B2D_ERR_NULL;
  if (lm_rows != h->lm_rows) return B2D_ERR_SHAPE;
  h->embed = embed;
  h->lm_head = lm_head;
  h->final_norm = final_norm;
  if (h->gexec) {
    cudaGraphExecDestroy(h->gexec);
    h->gexec = nullptr;
    h->gkey = GraphKey();
  }
  if (h->gen_exec) {
    cudaGraphExecDestroy(h->gen_exec);
    h->gen_exec = nullptr;
    h->gen_key = GraphKey();
  }
  return B2D_OK;
}

int b2d_decoder_step(b2d_decoder* h, const int* tokens, const int* ctx_lens,
                     const int* block_table, int batch, int* next_tokens, float* logits,
                     int use_graph, b2d_stream_t stream) {
  if (!h) return B2D_ERR_NULL;
  if (!tokens || !ctx_lens || !block_table || !next_tokens) return B2D_ERR_NULL;
  if (batch <= 0 || batch > h->cfg.max_batch) return B2D_ERR_SHAPE;
  if (!h->embed) return B2D_ERR_STATE;
  for (const Layer& L : h->layers)
    if (!L.wqkv) return B2D_ERR_STATE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (!use_graph) return enqueue_step(h, tokens, ctx_lens, block_table, batch, next_tokens, logits, s);
  if (s == nullptr) return B2D_ERR_STATE;  // the legacy default stream cannot be captured
  GraphKey key;
  key.batch = batch;
  key.stream = s;
  const void* ptrs[6] = {tokens, ctx_lens, block_table, next_tokens, logits, nullptr};
  for (int i = 0; i < 6; ++i) key.ptrs[i] = ptrs[i];
  if (!h->gexec || !(key == h->gkey)) {
    if (h->gexec) {
      cudaGraphExecDestroy(h->gexec);
      h->gexec = nullptr;
    }
    B2D_TRY(cuda_status(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal)));
    int st = enqueue_step(h, tokens, ctx_lens, block_table, batch, next_tokens, logits, s);
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamEndCapture(s, &graph);
    if (st != B2D_OK) {
      if (graph) cudaGraphDestroy(graph);
      return st;
    }
    B2D_TRY(cuda_status(e));
    e = cudaGraphInstantiate(&h->gexec, graph, 0);
    cudaGraphDestroy(graph);
    B2D_TRY(cuda_status(e));
    h->gkey = key;
  }
  return cuda_status(cudaGraphLaunch(h->gexec, s));
}

int b2d_decoder_prefill(b2d_decoder* h, const int* tokens, int n, const int* seq_table,
                        int start_pos, int* next_token, float* logits, b2d_stream_t stream) {
  if (!h) return B2D_ERR_NULL;
  if (!tokens || !seq_table || !next_token) return B2D_ERR_NULL;
  if (n <= 0 || start_pos < 0 || start_pos + n > h->cfg.max_ctx) return B2D_ERR_SHAPE;
  if (!h->embed) return B2D_ERR_STATE;
  for (const Layer& L : h->layers)
    if (!L.wqkv) return B2D_ERR_STATE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int chunk = h->cfg.max_batch, mb = h->cfg.max_blocks;
  // with logits, the last token runs as its own step (its logits row is the caller's buffer)
  const int n_chunked = logits ? n - 1 : n;
  int parity = 0;
  auto run = [&](int c0, int nb, bool last_out, float* lg) -> int {
    int* ctx = h->pf_ctx + (size_t)parity * chunk;
    int* table = h->pf_table + (size_t)parity * chunk * mb;
    parity ^= 1;  // the previous chunk's kernels may still read the other pair
    prefill_chunk_kernel<<<nb, 128, 0, s>>>(seq_table, mb, start_pos + c0, nb, ctx, table);
    B2D_TRY(launch_status());
    return enqueue_step(h, tokens + c0, ctx, table, nb, last_out ? h->gen_next : nullptr, lg, s,
                        true);
  };
  for (int c0 = 0; c0 < n_chunked; c0 += chunk) {
    const int nb = std::min(chunk, n_chunked - c0);
    const bool last = !logits && c0 + nb == n;
    B2D_TRY(run(c0, nb, last, nullptr));
    if (last)
      return cuda_status(cudaMemcpyAsync(next_token, h->gen_next + nb - 1, sizeof(int),
                                         cudaMemcpyDeviceToDevice, s));
  }
  B2D_TRY(run(n - 1, 1, true, logits));
  return cuda_status(
      cudaMemcpyAsync(next_token, h->gen_next, sizeof(int), cudaMemcpyDeviceToDevice, s));
}

int b2d_decoder_generate(b2d_decoder* h, int* tokens, int* ctx_lens, const int* block_table,
                         int batch, int n_steps, int* ring, int ring_steps, int* ring_count,
                         b2d_stream_t stream) {
  if (!h) return B2D_ERR_NULL;
  if (!tokens || !ctx_lens || !block_table || !ring || !ring_count) return B2D_ERR_NULL;
  if (batch <= 0 || batch > h->cfg.max_batch || n_steps < 0 || ring_steps <= 0)
    return B2D_ERR_SHAPE;
  if (!h->embed) return B2D_ERR_STATE;
  for (const Layer& L : h->layers)
    if (!L.wqkv) return B2D_ERR_STATE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (s == nullptr) return B2D_ERR_STATE;  // the legacy default stream cannot be captured
  GraphKey key;
  key.batch = batch * 65536 + ring_steps;
  key.stream = s;
  const void* ptrs[6] = {tokens, ctx_lens, block_table, ring, ring_count, nullptr};
  for (int i = 0; i < 6; ++i) key.ptrs[i] = ptrs[i];
  if (!h->gen_exec || !(key == h->gen_key)) {
    if (h->gen_exec) {
      cudaGraphExecDestroy(h->gen_exec);
      h->gen_exec = nullptr;
    }
    B2D_TRY(cuda_status(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal)));
    int st = enqueue_step(h, tokens, ctx_lens, block_table, batch, h->gen_next, nullptr, s);
    if (st == B2D_OK) {
      advance_kernel<<<1, 256, 0, s>>>(tokens, ctx_lens, h->gen_next, ring, ring_count,
                                       ring_steps, batch);
      st = launch_status();
    }
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamEndCapture(s, &graph);
    if (st != B2D_OK) {
      if (graph) cudaGraphDestroy(graph);
      return st;
    }
    B2D_TRY(cuda_status(e));
    e = cudaGraphInstantiate(&h->gen_exec, graph, 0);
    cudaGraphDestroy(graph);
    B2D_TRY(cuda_status(e));
    h->gen_key = key;
  }
  for (int i = 0; i < n_steps; ++i) B2D_TRY(cuda_status(cudaGraphLaunch(h->gen_exec, s)));
  return B2D_OK;
}

}  // extern "C"
