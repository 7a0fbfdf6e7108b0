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

#include "async.cuh"
#include "common.cuh"

namespace b2d {

constexpr int kAttnThreads = 128;

struct AttnParams {
  CUtensorMap tmK;  // K page pool as [n_blocks * Hkv * 16, HD] fp16, box {64, 16}, 128B swizzle
  CUtensorMap tmV;  // V page pool, same geometry (tensor-core kernel only)
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
  uint16_t* out_lo;  // B2D_F16X2 output: the lo plane (nullptr otherwise)
  int ldout;
  int max_ctx;     // every ctx_lens[b] + 1 must be <= max_ctx
  int chunk;       // keys per CTA (multiple of 16)
  int max_chunks;  // chunks per sequence covered by the workspace
  unsigned int* counters;  // [B][Hkv]
  float* partials;         // [B][Hkv][max_chunks][G][HD + 2]
  int* err;                // error word (a bounded wait gave up)
};

__device__ __forceinline__ float load_qkv(const AttnParams& p, size_t i) {
  return p.qkv_f16 ? h2f(reinterpret_cast<const uint16_t*>(p.qkv)[i])
                   : reinterpret_cast<const float*>(p.qkv)[i];
}

// Combine the CTA's NSUB partial softmax states st[NSUB][G][HD + 2] (unnormalized output, max,
// sum) into this chunk's result: the output itself when the sequence has one chunk, otherwise a
// partial in the workspace; the last CTA of the (sequence, KV head) then merges all chunks with
// log-sum-exp weights and re-zeroes its arrival counter.  Called by all threads after a barrier.
template <int HD, int G, int NSUB>
__device__ void chunk_finish(const AttnParams& p, const float* st, int b, int kvh, int c,
                             int first_c, int nact) {
  const int tid = threadIdx.x;
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
        store_f16_split(reinterpret_cast<uint16_t*>(p.out), p.out_lo, oi, r);
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
  __shared__ float chunk_w[64 * 8];  // per (chunk, head) weight exp(M_k - M), up to 64 chunks
  __shared__ float head_inv[8];
  __threadfence();
  __syncthreads();
  unsigned int* cnt = p.counters + (size_t)b * p.n_kv_heads + kvh;
  if (tid == 0) is_last = atomicAdd(cnt, 1u) == (unsigned)(nact - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const float* base_part =
      p.partials + (((size_t)b * p.n_kv_heads + kvh) * p.max_chunks) * G * (HD + 2);
  const bool fits = nact <= 64 && G <= 8;
  if (fits) {
    // weights once per (chunk, head): one warp per head, lanes over chunks
    const int warp = tid >> 5, lane = tid & 31;
    for (int g = warp; g < G; g += kAttnThreads / 32) {
      float M = -INFINITY;
      for (int k = lane; k < nact; k += 32)
        M = fmaxf(M, __ldcg(base_part + ((size_t)k * G + g) * (HD + 2) + HD));
      M = warp_max(M);
      float lsum = 0.f;
      for (int k = lane; k < nact; k += 32) {
        const float* pp = base_part + ((size_t)k * G + g) * (HD + 2);
        const float e = __expf(__ldcg(pp + HD) - M);
        chunk_w[k * 8 + g] = e;
        lsum = fmaf(e, __ldcg(pp + HD + 1), lsum);
      }
      lsum = warp_sum(lsum);
      if (lane == 0) head_inv[g] = 1.0f / lsum;
    }
    __syncthreads();
  }
  for (int i = tid; i < G * HD; i += kAttnThreads) {
    const int g = i / HD, d = i % HD;
    float r;
    if (fits) {
      float o = 0.f;
      for (int k = 0; k < nact; ++k)
        o = fmaf(chunk_w[k * 8 + g], __ldcg(base_part + ((size_t)k * G + g) * (HD + 2) + d), o);
      r = o * head_inv[g];
    } else {
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
      r = o / lsum;
    }
    const size_t oi = (size_t)b * p.ldout + (size_t)(kvh * G + g) * HD + d;
    if (p.out_f16)
      store_f16_split(reinterpret_cast<uint16_t*>(p.out), p.out_lo, oi, r);
    else
      reinterpret_cast<float*>(p.out)[oi] = r;
  }
  if (tid == 0) *cnt = 0u;
}

template <int HD, int G>
struct AttnCfg {
  static constexpr int L = HD / 8;                        // lanes per key (8 dims each)
  static constexpr int NSUB = kAttnThreads / L;           // sub-warps per CTA
  static constexpr int TPP = 16 / NSUB;                   // keys per sub-warp per page
  static constexpr int PAGE_BYTES = 16 * HD * 2;          // one KV head's slice of a page
  static constexpr int STAGES = HD == 64 ? 8 : (HD == 128 ? 6 : 4);
  static constexpr int RING_BYTES = STAGES * 2 * PAGE_BYTES;
  static constexpr int STATE_BYTES = NSUB * G * (HD + 2) * 4;  // sub-warp merge (aliases ring)
  static constexpr int REGION0 = RING_BYTES > STATE_BYTES ? RING_BYTES : STATE_BYTES;
  static constexpr size_t smem_bytes() {
    return REGION0 + sizeof(float) * ((size_t)G * HD + 2 * HD + 64);
  }
};

template <int HD, int G>
__global__ void __launch_bounds__(kAttnThreads) paged_attn_kernel(const __grid_constant__ AttnParams p) {
  using C = AttnCfg<HD, G>;
  constexpr int L = C::L, NSUB = C::NSUB, TPP = C::TPP, STAGES = C::STAGES;
  extern __shared__ __align__(128) uint8_t sm_raw[];
  uint8_t* ring = sm_raw;                                        // [STAGES][K page | V page]
  float* st = reinterpret_cast<float*>(sm_raw);                  // [NSUB][G][HD + 2] after the loop
  float* qs = reinterpret_cast<float*>(sm_raw + C::REGION0);     // [G][HD]
  float* kn = qs + G * HD;                                       // [HD]
  float* vn = kn + HD;                                           // [HD]
  int* blk_s = reinterpret_cast<int*>(vn + HD);                  // [<= 64]
  __shared__ __align__(8) uint64_t full_bar[STAGES];

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
  const int pg0 = (c * p.chunk) / 16;             // first page of the chunk
  const int pg_lo = tok_lo / 16, pg_hi = (tok_hi + 15) / 16;
  const int npg = pg_hi - pg_lo;

  // ---- prologue: block ids of the chunk, barriers, first ring of page copies
  const int* bt = p.block_table + (size_t)b * p.max_blocks;
  for (int i = tid; i < p.chunk / 16; i += kAttnThreads) {
    const int lb = pg0 + i;
    const int v = lb < p.max_blocks ? bt[lb] : -1;
    blk_s[i] = (v >= 0 && v < p.n_blocks) ? v : -1;  // ids outside the pool are never read
  }
  if (tid == 0) {
    for (int s2 = 0; s2 < STAGES; ++s2) mbar_init(&full_bar[s2], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const size_t kv_head_off = (size_t)kvh * 16 * HD;  // elements
  const size_t blk_stride = (size_t)p.n_kv_heads * 16 * HD;
  auto issue = [&](int i) {  // page pg_lo + i into stage i % STAGES (thread 0 only)
    const int s2 = i % STAGES;
    uint64_t* bar = &full_bar[s2];
    const int blk = blk_s[pg_lo + i - pg0];
    if (blk >= 0) {
      uint8_t* dst = ring + (size_t)s2 * 2 * C::PAGE_BYTES;
      mbar_expect_tx(bar, 2 * C::PAGE_BYTES);
      const uint64_t pol = l2_evict_first();  // KV pages are read once per step
      bulk_load_hint(dst, p.k_pages + (size_t)blk * blk_stride + kv_head_off, C::PAGE_BYTES, bar,
                     pol);
      bulk_load_hint(dst + C::PAGE_BYTES, p.v_pages + (size_t)blk * blk_stride + kv_head_off,
                     C::PAGE_BYTES, bar, pol);
    } else {
      mbar_arrive(bar);  // nothing to load: complete the phase, the page is masked
    }
  };
  if (tid == 0)
    for (int i = 0; i < min(npg, STAGES); ++i) issue(i);

  // rotated, pre-scaled q (and the new token's k / v) in shared memory
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
    const int blk = blk_s[pos / 16 - pg0];
    const size_t slot = ((size_t)blk * p.n_kv_heads * 16 + (size_t)kvh * 16 + (pos % 16)) * HD;
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
      if (blk >= 0) {
        p.k_pages[slot + d] = ra;
        p.k_pages[slot + d + hd2] = rb;
        p.v_pages[slot + d] = va;
        p.v_pages[slot + d + hd2] = vb;
      }
    }
  }
  __syncthreads();
  pdl_launch_dependents();

  // ---- main loop over pages: sub-warps own TPP keys of each page, online softmax in registers
  const int warp = tid >> 5, lane = tid & 31;
  const int sub = lane / L, li = lane % L;
  const int sw = warp * (32 / L) + sub;  // sub-warp id in the CTA
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
  int issued = min(npg, STAGES);  // meaningful in thread 0 only
  for (int i = 0; i < npg; ++i) {
    const int s2 = i % STAGES;
    const bool arrived = mbar_wait(&full_bar[s2], (i / STAGES) & 1, p.err, 1);
    const int pg = pg_lo + i;
    const bool page_ok = arrived && blk_s[pg - pg0] >= 0;
    const uint8_t* kpage = ring + (size_t)s2 * 2 * C::PAGE_BYTES;
    const uint8_t* vpage = kpage + C::PAGE_BYTES;
    float s[TPP][G];
    bool valid[TPP];
    float vf[TPP][8];
#pragma unroll
    for (int u = 0; u < TPP; ++u) {
      const int t = sw * TPP + u;
      const int j = pg * 16 + t;
      valid[u] = page_ok && j >= tok_lo && j < tok_hi;
      const bool mine_new = owns_new && j == pos;
      float kf[8];
      if (mine_new) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          kf[e] = kn[li * 8 + e];
          vf[u][e] = vn[li * 8 + e];
        }
        valid[u] = j >= tok_lo && j < tok_hi;
      } else {
        const uint4 kr = *reinterpret_cast<const uint4*>(kpage + (size_t)t * HD * 2 + li * 16);
        const uint4 vr = *reinterpret_cast<const uint4*>(vpage + (size_t)t * HD * 2 + li * 16);
        const uint32_t kw[4] = {kr.x, kr.y, kr.z, kr.w};
        const uint32_t vw[4] = {vr.x, vr.y, vr.z, vr.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 fk = h2f2(kw[e]);
          const float2 fv = h2f2(vw[e]);
          kf[2 * e] = fk.x;
          kf[2 * e + 1] = fk.y;
          vf[u][2 * e] = fv.x;
          vf[u][2 * e + 1] = fv.y;
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float a = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) a = fmaf(qv[g][e], kf[e], a);
        s[u][g] = a;
      }
    }
#pragma unroll
    for (int o = L / 2; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < TPP; ++u)
#pragma unroll
        for (int g = 0; g < G; ++g) s[u][g] += __shfl_xor_sync(0xffffffffu, s[u][g], o);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mx = m[g];
#pragma unroll
      for (int u = 0; u < TPP; ++u)
        if (valid[u]) mx = fmaxf(mx, s[u][g]);
      if (mx == -INFINITY) continue;
      const float corr = __expf(m[g] - mx);
      m[g] = mx;
      l[g] *= corr;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[g][e] *= corr;
#pragma unroll
      for (int u = 0; u < TPP; ++u) {
        if (!valid[u]) continue;
        const float pu = __expf(s[u][g] - mx);
        l[g] += pu;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] = fmaf(pu, vf[u][e], acc[g][e]);
      }
    }
    // every thread is done with stage s2; a timed-out wait anywhere stops the whole CTA
    if (__syncthreads_or(arrived ? 0 : 1)) {
      if (tid == 0)  // let the copies already in flight land before the CTA exits
        for (int j = i; j < issued; ++j) mbar_wait(&full_bar[j % STAGES], (j / STAGES) & 1, p.err, 1);
      return;
    }
    if (tid == 0 && i + STAGES < npg) {
      issue(i + STAGES);
      ++issued;
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
  chunk_finish<HD, G, NSUB>(p, st, b, kvh, c, first_c, nact);
}

// ------------------------------------------------------------------------------------------
// Tensor-core variant (head_dim 64 / 128): every warp owns a private ring of pages loaded by
// TMA (tiled, 128-byte swizzle) and treats one page as one warp-level MMA tile:
//   S[h, j] = q_h . k_j  as  m16n8k16 with the G query heads as rows, tokens as columns;
//   P = exp(S - m) in registers; O[h, :] += P V with P re-packed from the S accumulators as
//   the A operand and V read with ldmatrix.trans.
// q and p enter each MMA as hi + lo fp16 pairs -- hi parts in rows 0..7, lo parts in rows
// 8..15 of the same 16-row tile (mma_hilo) -- so scores and weights keep ~22-bit precision at
// one MMA per tile (K and V are exactly their stored fp16 values).  No CTA-wide barrier runs
// inside the main loop; warps merge at the end like the sub-warps of the CUDA-core kernel.
// ------------------------------------------------------------------------------------------

// Pages in flight per warp of the tensor-core kernel.  Fewer stages mean less shared memory per
// CTA and more CTAs (warps) per SM, which beat deeper rings on B200: head_dim 64 at 2 stages
// (6 CTAs per SM) 34.2 us for the config-5 layer vs 36.9 at 3 and 41.0 at 4; head_dim 128 at 2
// stages (3 CTAs per SM) 203 us for config 4 vs 217 at 1 and 229 at 3.
#ifndef B2D_ATTN_STAGES_HD64
#define B2D_ATTN_STAGES_HD64 2
#endif
#ifndef B2D_ATTN_STAGES_HD128
#define B2D_ATTN_STAGES_HD128 2
#endif

template <int HD>
struct TcAttnCfg {
  static constexpr int WARPS = kAttnThreads / 32;     // 4
  static constexpr int BOXES = HD / 64;               // 64-column TMA boxes per page slice
  static constexpr int PAGE_BYTES = 16 * HD * 2;      // one KV head's K (or V) page slice
  static constexpr int SW = HD == 64 ? B2D_ATTN_STAGES_HD64 : B2D_ATTN_STAGES_HD128;  // per warp
  static constexpr int STAGE_BYTES = 2 * PAGE_BYTES;  // K slice, then V slice
  static constexpr int WARP_RING = SW * STAGE_BYTES;
  static constexpr int RING = WARPS * WARP_RING;
  static constexpr int STATE = WARPS * 8 * (HD + 2) * 4;  // merge buffer (G <= 8), aliases ring
  static constexpr int REGION0 = RING > STATE ? RING : STATE;
  static constexpr size_t smem_bytes(int G) {
    return 1024 + REGION0 + sizeof(float) * ((size_t)G * HD + 2 * HD + 64);
  }
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D += A(16x16) * B(16x8) with the hi parts of the G <= 8 live rows in rows 0..7 and their lo
// parts (x - fp16(x)) in rows 8..15: d[0], d[1] accumulate the hi products and d[2], d[3] the
// lo products of the same (row, column) pairs, so d[0] + d[2] and d[1] + d[3] carry ~22-bit
// operand precision from one fp16 MMA (the reference computes q.k and p.v in fp32).
__device__ __forceinline__ void mma_hilo(float* d, uint32_t hi0, uint32_t lo0, uint32_t hi2,
                                         uint32_t lo2, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(hi0), "r"(lo0), "r"(hi2), "r"(lo2), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// hi/lo fp16 split of two floats: hi = fp16(x), lo = fp16(x - hi)
__device__ __forceinline__ void split_h2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
  const __half l0 = __float2half_rn(x0 - __half2float(h0));
  const __half l1 = __float2half_rn(x1 - __half2float(h1));
  __half2 H = __halves2half2(h0, h1), L = __halves2half2(l0, l1);
  hi = *reinterpret_cast<uint32_t*>(&H);
  lo = *reinterpret_cast<uint32_t*>(&L);
}

template <int HD, int G>
__global__ void __launch_bounds__(kAttnThreads) paged_attn_tc_kernel(const __grid_constant__ AttnParams p) {
  static_assert(G <= 8, "query heads per KV head must fit the MMA's 8 live rows");
  using C = TcAttnCfg<HD>;
  constexpr int SW = C::SW, KS = HD / 16, ND = HD / 8;
  extern __shared__ uint8_t sm_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) &
                                             ~uintptr_t(1023));
  float* st = reinterpret_cast<float*>(base);                 // [WARPS][G][HD + 2] after the loop
  float* qs = reinterpret_cast<float*>(base + C::REGION0);     // [G][HD]
  float* kn = qs + G * HD;
  float* vn = kn + HD;
  int* blk_s = reinterpret_cast<int*>(vn + HD);
  __shared__ __align__(8) uint64_t full_bar[C::WARPS][SW];
  __shared__ int cta_failed;

  const int c = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  // Context lengths, the block table and the cached pages are inputs of the step that no kernel
  // of the step writes before this one, so everything up to the first ring of page copies runs
  // before griddepcontrol.wait, overlapping the tail of the QKV projection.
  const int pos = p.ctx_lens[b];
  const int n = pos + 1;
  const int start = (p.window > 0 && n > p.window) ? n - p.window : 0;
  const int first_c = start / p.chunk, last_c = (n - 1) / p.chunk;
  // no keys here (or outside the caller's contract: output untouched)
  if (pos < 0 || pos >= p.max_ctx || c < first_c || c > last_c) return;
  const int tok_lo = max(c * p.chunk, start);
  const int tok_hi = min((c + 1) * p.chunk, n);
  const int nact = last_c - first_c + 1;
  const bool owns_new = p.append && c == last_c;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hd2 = HD / 2;
  const int pg0 = (c * p.chunk) / 16;
  const int pg_lo = tok_lo / 16, pg_hi = (tok_hi + 15) / 16;
  const int npg = pg_hi - pg_lo;

  const int* bt = p.block_table + (size_t)b * p.max_blocks;
  for (int i = tid; i < p.chunk / 16; i += kAttnThreads) {
    const int lb = pg0 + i;
    const int v = lb < p.max_blocks ? bt[lb] : -1;
    blk_s[i] = (v >= 0 && v < p.n_blocks) ? v : -1;  // ids outside the pool are never read
  }
  if (tid == 0) {
    for (int w = 0; w < C::WARPS; ++w)
      for (int s2 = 0; s2 < SW; ++s2) mbar_init(&full_bar[w][s2], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    cta_failed = 0;
  }
  __syncthreads();

  // this warp's pages: i = warp, warp + 4, ... ; local index k, ring stage k % SW
  const int my_n = npg > warp ? (npg - warp + C::WARPS - 1) / C::WARPS : 0;
  uint8_t* my_ring = base + warp * C::WARP_RING;
  auto issue = [&](int k) {  // lane 0 only
    const int i = warp + k * C::WARPS;
    uint64_t* bar = &full_bar[warp][k % SW];
    const int blk = blk_s[pg_lo + i - pg0];
    if (blk >= 0) {
      uint8_t* dst = my_ring + (k % SW) * C::STAGE_BYTES;
      const int row0 = (blk * p.n_kv_heads + kvh) * 16;
      const uint64_t pol = l2_evict_first();  // KV pages are read once per step
      mbar_expect_tx(bar, C::STAGE_BYTES);
#pragma unroll
      for (int bx = 0; bx < C::BOXES; ++bx) {
        tma_load_2d_hint(dst + bx * 2048, &p.tmK, bx * 64, row0, bar, pol);
        tma_load_2d_hint(dst + C::PAGE_BYTES + bx * 2048, &p.tmV, bx * 64, row0, bar, pol);
      }
    } else {
      mbar_arrive(bar);  // nothing to load: the page is masked
    }
  };
  if (lane == 0)
    for (int k = 0; k < min(my_n, SW); ++k) issue(k);
  pdl_wait();  // q, k, v of the new token come from the previous kernel

  // rotated, pre-scaled q and the new token's k / v (as in the CUDA-core kernel)
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
    const int blk = blk_s[pos / 16 - pg0];
    const size_t slot = ((size_t)blk * p.n_kv_heads * 16 + (size_t)kvh * 16 + (pos % 16)) * HD;
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
      if (blk >= 0) {
        p.k_pages[slot + d] = ra;
        p.k_pages[slot + d + hd2] = rb;
        p.v_pages[slot + d] = va;
        p.v_pages[slot + d + hd2] = vb;
      }
    }
  }
  __syncthreads();
  pdl_launch_dependents();

  // q as the A operand, hi/lo fp16 (rows = heads g < G; rows >= G and 8..15 are zero)
  const int g = lane >> 2, t4 = lane & 3;
  uint32_t qa[KS][2], qb[KS][2];  // qa: hi (a0, a2), qb: lo (a0, a2)
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
    if (g < G) {
      const float* qr = qs + g * HD + 16 * ks + 2 * t4;
      split_h2(qr[0], qr[1], qa[ks][0], qb[ks][0]);
      split_h2(qr[8], qr[9], qa[ks][1], qb[ks][1]);
    } else {
      qa[ks][0] = qa[ks][1] = qb[ks][0] = qb[ks][1] = 0u;
    }
  }
  float o[ND][4];
#pragma unroll
  for (int nd = 0; nd < ND; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.f;
  float m = -INFINITY, l = 0.f;
  bool failed = false;
  int issued = min(my_n, SW);
  const int r8 = lane & 7, mat = lane >> 3;

  for (int k = 0; k < my_n; ++k) {
    const int s2 = k % SW;
    const bool arrived = __all_sync(0xffffffffu, mbar_wait(&full_bar[warp][s2], (k / SW) & 1, p.err, 1));
    if (!arrived) {
      failed = true;
      break;
    }
    const int i = warp + k * C::WARPS;
    const int pg = pg_lo + i;
    const bool page_ok = blk_s[pg - pg0] >= 0;
    uint8_t* Kt = my_ring + s2 * C::STAGE_BYTES;
    uint8_t* Vt = Kt + C::PAGE_BYTES;
    if (owns_new && page_ok && pos / 16 == pg) {
      // the page copy raced with this CTA's own append: use the values it wrote
      const int rr = pos % 16;
      for (int ch = lane; ch < HD / 8; ch += 32) {
        const int off = (ch / 8) * 2048 + rr * 128 + (((ch % 8) ^ (rr & 7)) * 16);
        uint4 kv, vv;
        kv.x = pack_h2(kn[ch * 8 + 0], kn[ch * 8 + 1]);
        kv.y = pack_h2(kn[ch * 8 + 2], kn[ch * 8 + 3]);
        kv.z = pack_h2(kn[ch * 8 + 4], kn[ch * 8 + 5]);
        kv.w = pack_h2(kn[ch * 8 + 6], kn[ch * 8 + 7]);
        vv.x = pack_h2(vn[ch * 8 + 0], vn[ch * 8 + 1]);
        vv.y = pack_h2(vn[ch * 8 + 2], vn[ch * 8 + 3]);
        vv.z = pack_h2(vn[ch * 8 + 4], vn[ch * 8 + 5]);
        vv.w = pack_h2(vn[ch * 8 + 6], vn[ch * 8 + 7]);
        *reinterpret_cast<uint4*>(Kt + off) = kv;
        *reinterpret_cast<uint4*>(Vt + off) = vv;
      }
      __syncwarp();
    }
    // S = Q K^T for the page's two 8-token column tiles
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t kbase = smem_u32(Kt);
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const int trow = 8 * (mat >> 1) + r8;
      const int ch = 2 * ks + (mat & 1);
      const uint32_t addr = kbase + (ch / 8) * 2048 + trow * 128 + (((ch % 8) ^ (trow & 7)) << 4);
      uint32_t b00, b01, b10, b11;
      ldsm_x4(addr, b00, b01, b10, b11);
      mma_hilo(s0, qa[ks][0], qb[ks][0], qa[ks][1], qb[ks][1], b00, b01);
      mma_hilo(s1, qa[ks][0], qb[ks][0], qa[ks][1], qb[ks][1], b10, b11);
    }
    // online softmax for row g over this page's 16 tokens (4 per thread, quad of lanes)
    const int j0 = pg * 16 + 2 * t4;
    float sv[4] = {s0[0] + s0[2], s0[1] + s0[3], s1[0] + s1[2], s1[1] + s1[3]};
    const int jj[4] = {j0, j0 + 1, j0 + 8, j0 + 9};
    float mx = -INFINITY;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const bool ok = page_ok && jj[e] >= tok_lo && jj[e] < tok_hi;
      sv[e] = ok ? sv[e] : -INFINITY;
      mx = fmaxf(mx, sv[e]);
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m, mx);
    float pe[4];
    float corr = 1.f;
    if (m_new == -INFINITY) {
      pe[0] = pe[1] = pe[2] = pe[3] = 0.f;
    } else {
      corr = __expf(m - m_new);
#pragma unroll
      for (int e = 0; e < 4; ++e) pe[e] = sv[e] == -INFINITY ? 0.f : __expf(sv[e] - m_new);
      m = m_new;
    }
    l = fmaf(l, corr, pe[0] + pe[1] + pe[2] + pe[3]);
#pragma unroll
    for (int nd = 0; nd < ND; ++nd) {
      o[nd][0] *= corr;
      o[nd][1] *= corr;
      o[nd][2] *= corr;
      o[nd][3] *= corr;
    }
    uint32_t ph0, pl0, ph2, pl2;
    split_h2(pe[0], pe[1], ph0, pl0);
    split_h2(pe[2], pe[3], ph2, pl2);
    // O += P V
    const uint32_t vbase = smem_u32(Vt);
#pragma unroll
    for (int nd = 0; nd < ND; nd += 2) {
      const int tok = 8 * (mat & 1) + r8;
      const int ch = nd + (mat >> 1);
      const uint32_t addr = vbase + (ch / 8) * 2048 + tok * 128 + (((ch % 8) ^ (tok & 7)) << 4);
      uint32_t v0, v1, v2, v3;
      ldsm_x4_t(addr, v0, v1, v2, v3);
      mma_hilo(o[nd], ph0, pl0, ph2, pl2, v0, v1);
      mma_hilo(o[nd + 1], ph0, pl0, ph2, pl2, v2, v3);
    }
    __syncwarp();
    if (lane == 0 && k + SW < my_n) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // our reads before the refill
      issue(k + SW);
      ++issued;
    }
  }
  if (failed) {
    if (lane == 0)  // let this warp's copies in flight land before the CTA exits
      for (int k = 0; k < issued; ++k) mbar_wait(&full_bar[warp][k % SW], (k / SW) & 1, p.err, 1);
    cta_failed = 1;
  }
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);
  __syncthreads();  // all rings drained: the merge buffer may alias them
  if (cta_failed) return;
  if (g < G) {
    float* sp = st + ((size_t)warp * G + g) * (HD + 2);
#pragma unroll
    for (int nd = 0; nd < ND; ++nd) {
      sp[8 * nd + 2 * t4] = o[nd][0] + o[nd][2];
      sp[8 * nd + 2 * t4 + 1] = o[nd][1] + o[nd][3];
    }
    if (t4 == 0) {
      sp[HD] = m;
      sp[HD + 1] = l;
    }
  }
  __syncthreads();
  chunk_finish<HD, G, C::WARPS>(p, st, b, kvh, c, first_c, nact);
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

// Keys per CTA: the largest of {1024, 512, 256, 128, 64} (1024 measured best on B200: config 4
// 203 -> 193 us, config 5 unchanged; 256 is slower) that still gives >= 4 CTAs per SM when
// every sequence is half of max_ctx long (a graph-stable choice: no device data is read).
#ifndef B2D_ATTN_MAX_CHUNK
#define B2D_ATTN_MAX_CHUNK 1024
#endif

// CTAs per SM the chunking aims for when every sequence is half of max_ctx long (3 measured
// best on B200: the config-5 layer 34.0 -> 32.8 us against 4, which split it into 512-key chunks).
#ifndef B2D_ATTN_CTAS_PER_SM
#define B2D_ATTN_CTAS_PER_SM 3
#endif
int attn_chunk_tokens(int batch, int n_kv_heads, int max_ctx) {
  const long target = (long)B2D_ATTN_CTAS_PER_SM * num_sms();
  const long half_ctx = std::max(1, max_ctx / 2);
  for (int ch = B2D_ATTN_MAX_CHUNK; ch > 64; ch >>= 1)
    if ((long)batch * n_kv_heads * ((half_ctx + ch - 1) / ch) >= target) return ch;
  return 64;
}

// Workspace layout, identical for every call so that a workspace shared by calls of different
// shapes never has one call's partials where another call's counters live:
// [0] error word, [256, 256 + 4*kMaxSeqHeads) arrival counters [B][Hkv], then the partials.
constexpr int kMaxSeqHeads = 65536;  // batch * n_kv_heads per call
constexpr size_t kAttnHeaderBytes = 256 + (size_t)kMaxSeqHeads * sizeof(unsigned int);

// Bytes at the start of the workspace that must be zero before a call with this batch
// (error word + this call's counters).
size_t attn_ws_header_bytes(int batch, int n_kv_heads) {
  return 256 + (size_t)batch * n_kv_heads * sizeof(unsigned int);
}
static size_t ws_header_bytes(int, int) { return kAttnHeaderBytes; }

size_t paged_attn_workspace_bytes(int batch, int n_heads, int n_kv_heads, int head_dim,
                                  int max_ctx) {
  if (batch <= 0 || n_kv_heads <= 0 || n_heads <= 0 || max_ctx <= 0) return 0;
  if ((long long)batch * n_kv_heads > kMaxSeqHeads) return 0;
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

int make_tmap_f16(CUtensorMap* m, const void* base, uint64_t rows, int cols, int ld,
                  int box_rows);

template <int HD, int G>
static int launch_attn_tc(AttnParams& prm, int batch, cudaStream_t stream) {
  using C = TcAttnCfg<HD>;
  const size_t smem = C::smem_bytes(G);
  auto kern = paged_attn_tc_kernel<HD, G>;
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
  if constexpr (HD <= 128) {  // tensor-core kernel (head_dim 64 / 128)
    switch (G) {
      case 1: return launch_attn_tc<HD, 1>(prm, batch, stream);
      case 2: return launch_attn_tc<HD, 2>(prm, batch, stream);
      case 4: return launch_attn_tc<HD, 4>(prm, batch, stream);
      case 8: return launch_attn_tc<HD, 8>(prm, batch, stream);
      default: return B2D_ERR_UNSUPPORTED;
    }
  } else {  // CUDA-core kernel (head_dim 256)
  switch (G) {
    case 1: return launch_attn<HD, 1>(prm, batch, stream);
    case 2: return launch_attn<HD, 2>(prm, batch, stream);
    case 4: return launch_attn<HD, 4>(prm, batch, stream);
    case 8: return launch_attn<HD, 8>(prm, batch, stream);
    default: return B2D_ERR_UNSUPPORTED;
  }
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
  if (out_dtype != B2D_F32 && out_dtype != B2D_F16 && out_dtype != B2D_F16X2)
    return B2D_ERR_UNSUPPORTED;
  if (ldqkv < (n_heads + 2 * n_kv_heads) * head_dim || ldout < n_heads * head_dim)
    return B2D_ERR_SHAPE;
  if (!aligned16(k_pages) || !aligned16(v_pages)) return B2D_ERR_ALIGN;
  if ((long long)batch * n_kv_heads > kMaxSeqHeads) return B2D_ERR_SHAPE;
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
  prm.out_f16 = out_dtype != B2D_F32;
  prm.out_lo = out_dtype == B2D_F16X2 ? static_cast<uint16_t*>(out) + (size_t)batch * ldout : nullptr;
  prm.ldout = ldout;
  prm.max_ctx = max_ctx;
  prm.chunk = attn_chunk_tokens(batch, n_kv_heads, max_ctx);
  prm.max_chunks = (max_ctx + prm.chunk - 1) / prm.chunk;
  char* ws = static_cast<char*>(workspace);
  prm.err = reinterpret_cast<int*>(ws);
  prm.counters = reinterpret_cast<unsigned int*>(ws + 256);
  prm.partials = reinterpret_cast<float*>(ws + ws_header_bytes(batch, n_kv_heads));
  const int G = n_heads / n_kv_heads;
  if (head_dim <= 128) {  // page pools as 2D tensors for the TMA loads of the tensor-core kernel
    const uint64_t rows = (uint64_t)n_blocks * n_kv_heads * 16;
    B2D_TRY(make_tmap_f16(&prm.tmK, k_pages, rows, head_dim, head_dim, 16));
    B2D_TRY(make_tmap_f16(&prm.tmV, v_pages, rows, head_dim, head_dim, 16));
  }
  switch (head_dim) {
    case 64: return launch_attn_g<64>(prm, G, batch, stream);
    case 128: return launch_attn_g<128>(prm, G, batch, stream);
    default: return launch_attn_g<256>(prm, G, batch, stream);
  }
}

}  // namespace b2d
