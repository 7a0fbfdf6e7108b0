// Paged single-query decode attention for a ragged batch: RoPE + KV append + split-K GQA
// attention with an online-softmax merge.
//
// Reference: attention (LK/kernels.metal:235-305) keeps all scores of one (head, query) in
// threadgroup memory, which caps the context at 4096, and re-reads K/V once per query head.
// rope_kv (LK/kernels.metal:182-224) rotates q/k and writes the contiguous fp16 cache.
// Sliding window: GK/kernels.metal:343.
//
// B200 design (HBM-bound: ~4 flops per KV byte):
//  * one CTA per (chunk of keys, KV head, sequence): all G = Hq/Hkv query heads of the KV head
//    share every K/V load, so the cache is read exactly once;
//  * a sub-warp of HD/8 lanes owns one key at a time (16-byte loads, 8 dims per lane), U keys
//    in flight per sub-warp, online softmax (running max / sum / weighted V) in registers;
//  * the CTA merges its sub-warps through shared memory; if the sequence spans several
//    chunks, it writes (max, sum, unnormalized output) to the workspace and the last CTA of
//    the (sequence, KV head) -- found with an arrival counter -- merges them (log-sum-exp
//    weights) and writes the output, then resets the counter for the next call;
//  * with `append`, the CTA that owns the chunk holding position pos rotates q and the new k,
//    writes k and v to their page slot, and uses the fp16-rounded values it just wrote.
#include <algorithm>

#include "common.cuh"

namespace b2d {

constexpr int kAttnThreads = 128;

struct AttnParams {
  const void* qkv;
  int qkv_f16;
  int ldqkv;
  uint16_t* k_pages;
  uint16_t* v_pages;
  const int* block_table;
  int max_blocks;
  int n_blocks;
  const int* ctx_lens;
  const float* inv_freq;
  int n_heads, n_kv_heads;
  float scale;
  int window;
  int append;
  void* out;
  int out_f16;
  int ldout;
  int max_ctx;     // every ctx_lens[b] + 1 must be <= max_ctx
  int chunk;       // keys per CTA (multiple of 16)
  int max_chunks;  // chunks per sequence covered by the workspace
  unsigned int* counters;  // [B][Hkv]
  float* partials;         // [B][Hkv][max_chunks][G][HD + 2]
};

__device__ __forceinline__ float load_qkv(const AttnParams& p, size_t i) {
  return p.qkv_f16 ? h2f(reinterpret_cast<const uint16_t*>(p.qkv)[i])
                   : reinterpret_cast<const float*>(p.qkv)[i];
}

template <int HD, int G>
struct AttnCfg {
  static constexpr int L = HD / 8;                 // lanes per key
  static constexpr int TPW = 32 / L;               // keys per warp per sub-step
  static constexpr int NSUB = (kAttnThreads / 32) * TPW;  // sub-warps per CTA
  static constexpr int U = (HD <= 128) ? 4 : 2;    // keys in flight per sub-warp
  static constexpr int STEP = NSUB * U;            // keys per CTA iteration
  static constexpr size_t smem_bytes() {
    return sizeof(float) * ((size_t)G * HD        // rotated, scaled q
                            + 2 * HD               // new k / v (fp16-rounded)
                            + (size_t)NSUB * G * (HD + 2)  // sub-warp states
                            + 64);                 // block ids of the chunk
  }
};

template <int HD, int G>
__global__ void __launch_bounds__(kAttnThreads) paged_attn_kernel(const AttnParams p) {
  using C = AttnCfg<HD, G>;
  constexpr int L = C::L, TPW = C::TPW, NSUB = C::NSUB, U = C::U;
  extern __shared__ __align__(16) float sm[];
  float* qs = sm;                         // [G][HD]
  float* kn = qs + G * HD;                // [HD]
  float* vn = kn + HD;                    // [HD]
  float* st = vn + HD;                    // [NSUB][G][HD + 2]
  int* blk_s = reinterpret_cast<int*>(st + NSUB * G * (HD + 2));  // [<= 64]

  const int c = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  pdl_wait();
  const int pos = p.ctx_lens[b];
  if (pos < 0 || pos >= p.max_ctx) return;  // outside the caller's contract: output untouched
  const int n = pos + 1;
  const int start = (p.window > 0 && n > p.window) ? n - p.window : 0;
  const int first_c = start / p.chunk, last_c = (n - 1) / p.chunk;
  if (c < first_c || c > last_c) return;
  const int tok_lo = max(c * p.chunk, start);
  const int tok_hi = min((c + 1) * p.chunk, n);
  const int nact = last_c - first_c + 1;
  const bool owns_new = p.append && c == last_c;
  const int tid = threadIdx.x;
  const int hd2 = HD / 2;

  // ---- prologue: block ids of the chunk, rotated q (and new k / v) in shared memory
  const int* bt = p.block_table + (size_t)b * p.max_blocks;
  for (int i = tid; i < p.chunk / 16; i += kAttnThreads) {
    const int lb = (c * p.chunk) / 16 + i;
    blk_s[i] = lb < p.max_blocks ? bt[lb] : -1;
  }
  const size_t row = (size_t)b * p.ldqkv;
  for (int i = tid; i < G * hd2; i += kAttnThreads) {
    const int g = i / hd2, d = i % hd2;
    const size_t qo = row + (size_t)(kvh * G + g) * HD;
    float a = load_qkv(p, qo + d), bq = load_qkv(p, qo + d + hd2);
    if (p.append) {
      float sn, cs;
      sincosf((float)pos * p.inv_freq[d], &sn, &cs);
      const float ra = a * cs - bq * sn;
      const float rb = bq * cs + a * sn;
      a = ra;
      bq = rb;
    }
    qs[g * HD + d] = a * p.scale;
    qs[g * HD + d + hd2] = bq * p.scale;
  }
  if (owns_new) {
    const size_t ko = row + (size_t)(p.n_heads + kvh) * HD;
    const size_t vo = row + (size_t)(p.n_heads + p.n_kv_heads + kvh) * HD;
    const int blk = bt[pos / 16];
    const bool ok = blk >= 0 && blk < p.n_blocks;
    const size_t slot = (((size_t)blk * p.n_kv_heads + kvh) * 16 + (pos % 16)) * HD;
    for (int d = tid; d < hd2; d += kAttnThreads) {
      float sn, cs;
      sincosf((float)pos * p.inv_freq[d], &sn, &cs);
      const float a = load_qkv(p, ko + d), bk = load_qkv(p, ko + d + hd2);
      const uint16_t ra = f2h(a * cs - bk * sn), rb = f2h(bk * cs + a * sn);
      const uint16_t va = f2h(load_qkv(p, vo + d)), vb = f2h(load_qkv(p, vo + d + hd2));
      kn[d] = h2f(ra);
      kn[d + hd2] = h2f(rb);
      vn[d] = h2f(va);
      vn[d + hd2] = h2f(vb);
      if (ok) {
        p.k_pages[slot + d] = ra;
        p.k_pages[slot + d + hd2] = rb;
        p.v_pages[slot + d] = va;
        p.v_pages[slot + d + hd2] = vb;
      }
    }
  }
  __syncthreads();
  pdl_launch_dependents();

  // ---- main loop: each sub-warp streams keys, online softmax in registers
  const int warp = tid >> 5, lane = tid & 31;
  const int sub = lane / L, li = lane % L;
  const int sw = warp * TPW + sub;  // sub-warp id in the CTA
  float qv[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int i = 0; i < 8; ++i) qv[g][i] = qs[g * HD + li * 8 + i];
  float m[G], l[G], acc[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[g][i] = 0.f;
  }
  const int c0 = c * p.chunk;
  const size_t head_off = (size_t)kvh * 16 * HD + (size_t)li * 8;
  for (int base = tok_lo + warp * TPW * U; base < tok_hi; base += C::STEP) {
    uint4 kr[U], vr[U];
    bool valid[U];
    bool from_smem[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = base + u * TPW + sub;
      valid[u] = j < tok_hi;
      from_smem[u] = owns_new && j == pos;
      kr[u] = make_uint4(0, 0, 0, 0);
      vr[u] = make_uint4(0, 0, 0, 0);
      if (valid[u] && !from_smem[u]) {
        const int blk = blk_s[(j - c0) >> 4];
        if (blk >= 0 && blk < p.n_blocks) {
          const size_t off = (size_t)blk * p.n_kv_heads * 16 * HD + head_off + (size_t)(j & 15) * HD;
          kr[u] = ld_stream16(p.k_pages + off);
          vr[u] = ld_stream16(p.v_pages + off);
        } else {
          valid[u] = false;  // block id outside the pool: the key is skipped
        }
      }
    }
    float s[U][G];
    float kf[U][8];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (from_smem[u]) {
#pragma unroll
        for (int i = 0; i < 8; ++i) kf[u][i] = kn[li * 8 + i];
      } else {
        const uint32_t w[4] = {kr[u].x, kr[u].y, kr[u].z, kr[u].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = h2f2(w[i]);
          kf[u][2 * i] = f.x;
          kf[u][2 * i + 1] = f.y;
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) a = fmaf(qv[g][i], kf[u][i], a);
        s[u][g] = a;
      }
    }
#pragma unroll
    for (int o = L / 2; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int g = 0; g < G; ++g) s[u][g] += __shfl_xor_sync(0xffffffffu, s[u][g], o);

    float vf[U][8];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (from_smem[u]) {
#pragma unroll
        for (int i = 0; i < 8; ++i) vf[u][i] = vn[li * 8 + i];
      } else {
        const uint32_t w[4] = {vr[u].x, vr[u].y, vr[u].z, vr[u].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = h2f2(w[i]);
          vf[u][2 * i] = f.x;
          vf[u][2 * i + 1] = f.y;
        }
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mx = m[g];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (valid[u]) mx = fmaxf(mx, s[u][g]);
      if (mx == -INFINITY) continue;
      const float corr = __expf(m[g] - mx);
      m[g] = mx;
      l[g] *= corr;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[g][i] *= corr;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (!valid[u]) continue;
        const float pu = __expf(s[u][g] - mx);
        l[g] += pu;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[g][i] = fmaf(pu, vf[u][i], acc[g][i]);
      }
    }
  }

  // ---- merge the sub-warps of this CTA
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float* sp = st + ((size_t)sw * G + g) * (HD + 2);
#pragma unroll
    for (int i = 0; i < 8; ++i) sp[li * 8 + i] = acc[g][i];
    if (li == 0) {
      sp[HD] = m[g];
      sp[HD + 1] = l[g];
    }
  }
  __syncthreads();

  const bool single = nact == 1;
  float* part = p.partials + (((size_t)b * p.n_kv_heads + kvh) * p.max_chunks + (c - first_c)) *
                                 G * (HD + 2);
  for (int i = tid; i < G * HD; i += kAttnThreads) {
    const int g = i / HD, d = i % HD;
    float M = -INFINITY;
    for (int w = 0; w < NSUB; ++w) M = fmaxf(M, st[((size_t)w * G + g) * (HD + 2) + HD]);
    float o = 0.f, lsum = 0.f;
    for (int w = 0; w < NSUB; ++w) {
      const float* sp = st + ((size_t)w * G + g) * (HD + 2);
      const float e = sp[HD] == -INFINITY ? 0.f : __expf(sp[HD] - M);
      o = fmaf(e, sp[d], o);
      lsum = fmaf(e, sp[HD + 1], lsum);
    }
    if (single) {
      const float r = o / lsum;
      const size_t oi = (size_t)b * p.ldout + (size_t)(kvh * G + g) * HD + d;
      if (p.out_f16)
        reinterpret_cast<uint16_t*>(p.out)[oi] = f2h(r);
      else
        reinterpret_cast<float*>(p.out)[oi] = r;
    } else {
      part[(size_t)g * (HD + 2) + d] = o;
      if (d == 0) {
        part[(size_t)g * (HD + 2) + HD] = M;
        part[(size_t)g * (HD + 2) + HD + 1] = lsum;
      }
    }
  }
  if (single) return;

  // ---- cross-chunk merge by the last arriving CTA of this (sequence, KV head)
  __shared__ bool is_last;
  __threadfence();
  __syncthreads();
  unsigned int* cnt = p.counters + (size_t)b * p.n_kv_heads + kvh;
  if (tid == 0) is_last = atomicAdd(cnt, 1u) == (unsigned)(nact - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const float* base_part =
      p.partials + (((size_t)b * p.n_kv_heads + kvh) * p.max_chunks) * G * (HD + 2);
  for (int i = tid; i < G * HD; i += kAttnThreads) {
    const int g = i / HD, d = i % HD;
    float M = -INFINITY;
    for (int k = 0; k < nact; ++k)
      M = fmaxf(M, __ldcg(base_part + ((size_t)k * G + g) * (HD + 2) + HD));
    float o = 0.f, lsum = 0.f;
    for (int k = 0; k < nact; ++k) {
      const float* pp = base_part + ((size_t)k * G + g) * (HD + 2);
      const float e = __expf(__ldcg(pp + HD) - M);
      o = fmaf(e, __ldcg(pp + d), o);
      lsum = fmaf(e, __ldcg(pp + HD + 1), lsum);
    }
    const float r = o / lsum;
    const size_t oi = (size_t)b * p.ldout + (size_t)(kvh * G + g) * HD + d;
    if (p.out_f16)
      reinterpret_cast<uint16_t*>(p.out)[oi] = f2h(r);
    else
      reinterpret_cast<float*>(p.out)[oi] = r;
  }
  if (tid == 0) *cnt = 0u;
}

// ------------------------------------------------------------------------------------------
// Standalone RoPE + append (rope_kv, LK/kernels.metal:182-224, with a paged destination).
// One CTA per sequence; threads walk (head, pair) items over q and k heads.
// ------------------------------------------------------------------------------------------
__global__ void rope_kv_append_kernel(void* qkv, int qkv_f16, int ldqkv, uint16_t* k_pages,
                                      uint16_t* v_pages, const int* block_table, int max_blocks,
                                      int n_blocks, const int* ctx_lens, const float* inv_freq, int n_heads,
                                      int n_kv, int HD) {
  const int b = blockIdx.x;
  const int pos = ctx_lens[b];
  if (pos < 0 || pos / 16 >= max_blocks) return;
  const int hd2 = HD / 2;
  const int blk = block_table[(size_t)b * max_blocks + pos / 16];
  const size_t row = (size_t)b * ldqkv;
  float* qf = reinterpret_cast<float*>(qkv);
  uint16_t* qh = reinterpret_cast<uint16_t*>(qkv);
  for (int it = threadIdx.x; it < (n_heads + n_kv) * hd2; it += blockDim.x) {
    const int h = it / hd2, i = it % hd2;
    const size_t o = row + (size_t)h * HD;
    const float a = qkv_f16 ? h2f(qh[o + i]) : qf[o + i];
    const float bb = qkv_f16 ? h2f(qh[o + i + hd2]) : qf[o + i + hd2];
    float sn, cs;
    sincosf((float)pos * inv_freq[i], &sn, &cs);
    const float ra = a * cs - bb * sn, rb = bb * cs + a * sn;
    if (h < n_heads) {
      if (qkv_f16) {
        qh[o + i] = f2h(ra);
        qh[o + i + hd2] = f2h(rb);
      } else {
        qf[o + i] = ra;
        qf[o + i + hd2] = rb;
      }
    } else if (blk >= 0 && blk < n_blocks) {
      const int kvh = h - n_heads;
      const size_t slot = (((size_t)blk * n_kv + kvh) * 16 + (pos % 16)) * HD;
      const size_t vo = row + (size_t)(n_heads + n_kv + kvh) * HD;
      k_pages[slot + i] = f2h(ra);
      k_pages[slot + i + hd2] = f2h(rb);
      v_pages[slot + i] = f2h(qkv_f16 ? h2f(qh[vo + i]) : qf[vo + i]);
      v_pages[slot + i + hd2] = f2h(qkv_f16 ? h2f(qh[vo + i + hd2]) : qf[vo + i + hd2]);
    }
  }
}

int rope_kv_append(void* qkv, int qkv_dtype, int ldqkv, uint16_t* k_pages, uint16_t* v_pages,
                   const int* block_table, int max_blocks, int n_blocks, const int* ctx_lens,
                   const float* inv_freq, int n_heads, int n_kv_heads, int head_dim, int batch,
                   cudaStream_t stream) {
  if (!qkv || !k_pages || !v_pages || !block_table || !ctx_lens || !inv_freq) return B2D_ERR_NULL;
  if (batch <= 0 || head_dim <= 0 || head_dim % 2 || n_heads <= 0 || n_kv_heads <= 0 ||
      max_blocks <= 0 || n_blocks <= 0)
    return B2D_ERR_SHAPE;
  if (qkv_dtype != B2D_F32 && qkv_dtype != B2D_F16) return B2D_ERR_UNSUPPORTED;
  if (ldqkv < (n_heads + 2 * n_kv_heads) * head_dim) return B2D_ERR_SHAPE;
  rope_kv_append_kernel<<<batch, 256, 0, stream>>>(qkv, qkv_dtype == B2D_F16, ldqkv, k_pages,
                                                   v_pages, block_table, max_blocks, n_blocks,
                                                   ctx_lens,
                                                   inv_freq, n_heads, n_kv_heads, head_dim);
  return launch_status();
}

// ------------------------------------------------------------------------------------------
// host side of the split-K kernel
// ------------------------------------------------------------------------------------------

// Keys per CTA: the largest of {512, 256, 128, 64} that still gives >= 4 CTAs per SM when
// every sequence is half of max_ctx long (a graph-stable choice: no device data is read).
int attn_chunk_tokens(int batch, int n_kv_heads, int max_ctx) {
  const long target = 4L * num_sms();
  const long half_ctx = std::max(1, max_ctx / 2);
  for (int ch = 512; ch > 64; ch >>= 1)
    if ((long)batch * n_kv_heads * ((half_ctx + ch - 1) / ch) >= target) return ch;
  return 64;
}

static size_t ws_header_bytes(int batch, int n_kv_heads) {
  return ((size_t)batch * n_kv_heads * sizeof(unsigned int) + 255) / 256 * 256;
}

size_t paged_attn_workspace_bytes(int batch, int n_heads, int n_kv_heads, int head_dim,
                                  int max_ctx) {
  if (batch <= 0 || n_kv_heads <= 0 || n_heads <= 0 || max_ctx <= 0) return 0;
  const int ch = attn_chunk_tokens(batch, n_kv_heads, max_ctx);
  const size_t max_chunks = (size_t)(max_ctx + ch - 1) / ch;
  const int G = n_heads / n_kv_heads;
  return ws_header_bytes(batch, n_kv_heads) +
         (size_t)batch * n_kv_heads * max_chunks * G * (head_dim + 2) * sizeof(float);
}

template <int HD, int G>
static int launch_attn(AttnParams& prm, int batch, cudaStream_t stream) {
  using C = AttnCfg<HD, G>;
  const size_t smem = C::smem_bytes();
  auto kern = paged_attn_kernel<HD, G>;
  static int cached_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != cached_dev) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return launch_status();
    cached_dev = dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(prm.max_chunks, prm.n_kv_heads, batch);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, prm);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return B2D_ERR_CUDA;
  }
  count_launch();
  return B2D_OK;
}

template <int HD>
static int launch_attn_g(AttnParams& prm, int G, int batch, cudaStream_t stream) {
  switch (G) {
    case 1: return launch_attn<HD, 1>(prm, batch, stream);
    case 2: return launch_attn<HD, 2>(prm, batch, stream);
    case 4: return launch_attn<HD, 4>(prm, batch, stream);
    case 8: return launch_attn<HD, 8>(prm, batch, stream);
    default: return B2D_ERR_UNSUPPORTED;
  }
}

int paged_decode_attn(void* qkv, int qkv_dtype, int ldqkv, uint16_t* k_pages, uint16_t* v_pages,
                      const int* block_table, int max_blocks, int n_blocks, const int* ctx_lens,
                      const float* inv_freq, int n_heads, int n_kv_heads, int head_dim,
                      int batch, int max_ctx, float scale, int window, int append, void* out,
                      int out_dtype, int ldout, void* workspace, size_t workspace_bytes,
                      cudaStream_t stream) {
  if (!qkv || !k_pages || !v_pages || !block_table || !ctx_lens || !out) return B2D_ERR_NULL;
  if (append && !inv_freq) return B2D_ERR_NULL;
  if (batch <= 0 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || max_ctx <= 0 ||
      max_blocks * 16 < max_ctx || n_blocks <= 0 || window < 0)
    return B2D_ERR_SHAPE;
  if (head_dim != 64 && head_dim != 128 && head_dim != 256) return B2D_ERR_UNSUPPORTED;
  if (qkv_dtype != B2D_F32 && qkv_dtype != B2D_F16) return B2D_ERR_UNSUPPORTED;
  if (out_dtype != B2D_F32 && out_dtype != B2D_F16) return B2D_ERR_UNSUPPORTED;
  if (ldqkv < (n_heads + 2 * n_kv_heads) * head_dim || ldout < n_heads * head_dim)
    return B2D_ERR_SHAPE;
  if (!aligned16(k_pages) || !aligned16(v_pages)) return B2D_ERR_ALIGN;
  const size_t need = paged_attn_workspace_bytes(batch, n_heads, n_kv_heads, head_dim, max_ctx);
  if (!workspace || workspace_bytes < need) return B2D_ERR_WORKSPACE;
  if (!aligned16(workspace)) return B2D_ERR_ALIGN;
  AttnParams prm = {};
  prm.qkv = qkv;
  prm.qkv_f16 = qkv_dtype == B2D_F16;
  prm.ldqkv = ldqkv;
  prm.k_pages = k_pages;
  prm.v_pages = v_pages;
  prm.block_table = block_table;
  prm.max_blocks = max_blocks;
  prm.n_blocks = n_blocks;
  prm.ctx_lens = ctx_lens;
  prm.inv_freq = inv_freq;
  prm.n_heads = n_heads;
  prm.n_kv_heads = n_kv_heads;
  prm.scale = scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim);
  prm.window = window;
  prm.append = append;
  prm.out = out;
  prm.out_f16 = out_dtype == B2D_F16;
  prm.ldout = ldout;
  prm.max_ctx = max_ctx;
  prm.chunk = attn_chunk_tokens(batch, n_kv_heads, max_ctx);
  prm.max_chunks = (max_ctx + prm.chunk - 1) / prm.chunk;
  char* ws = static_cast<char*>(workspace);
  prm.counters = reinterpret_cast<unsigned int*>(ws);
  prm.partials = reinterpret_cast<float*>(ws + ws_header_bytes(batch, n_kv_heads));
  const int G = n_heads / n_kv_heads;
  switch (head_dim) {
    case 64: return launch_attn_g<64>(prm, G, batch, stream);
    case 128: return launch_attn_g<128>(prm, G, batch, stream);
    default: return launch_attn_g<256>(prm, G, batch, stream);
  }
}

}  // namespace b2d
