// Decode GEMV with tensor-core dot products, for 32-block quantized (int8 / 4-bit) and fp16
// weights:  y[b, r] = epilogue(sum_k W[r, k] * xhat[b, k]),  up to 16 tokens per pass over W.
//
// Same operation and epilogues as the CUDA-core GEMV (gemv.cu; the reference's matvec kernels,
// LK/kernels.metal:106-173, with the RMSNorm of :71-89 fused).  What changes is how a weight is
// consumed.  The CUDA-core loop spends ~3.5 instructions per 4-bit or 8-bit weight (unpack,
// int -> float, FMA), as much issue time as HBM needs to deliver the weight.  Here:
//
//  * weights are never converted to fp32.  A 32-block of a 16-row tile becomes exact fp16
//    integers in registers (the byte or nibble is placed under the exponent of 1024 and the bias
//    subtracted: ~1.1 instructions per weight, two weights per instruction) and is multiplied on
//    the tensor cores with mma.sync m16n8k16 (fp32 accumulation);
//  * the block's fp16 scale multiplies the block's 16x8 result in fp32 (one FMA per output), so
//    sum_k (s * q_k) * x_k is evaluated as s * sum_k q_k * x_k with every q_k exact;
//  * activations sit in shared memory as fp16 columns of the MMA's B operand.  fp16 activations
//    without a norm are exact.  Otherwise (fp32 input, or the fused RMSNorm) each token is split
//    into a hi and a lo fp16 column (x = hi + lo to ~22 bits, after a per-token power-of-two
//    scale that keeps both in fp16's normal range): the MMA's N dimension has room for them;
//  * the MMA may sum the K dimension in any order, so each lane fetches the bytes that are
//    contiguous for it (whole 32-byte sectors per warp) and the activation columns are stored in
//    the matching order (4-bit: pairs (0,4)(1,5)(2,6)(3,7) of every 8 elements; 4-bit rows are
//    fetched 8 bytes per lane over two blocks and exchanged with one shuffle);
//  * a CTA of NW warps (8 or 16) splits K into KW slices and owns 16 * (NW / KW) rows at a time.
//    Each warp streams its slices through its own ring of D shared-memory slots (cp.async, no
//    register staging): D batches of 128 bytes x 16 rows are in flight per warp, so an SM keeps
//    64-128 KB of weight loads outstanding, which HBM latency needs.  The ring runs ahead across
//    row groups, and the first batches are requested before the kernel waits for the previous
//    kernel (weights do not depend on it).  K slices are summed in a fixed order.
#include <algorithm>

#include "async.cuh"
#include "common.cuh"

namespace b2d {

namespace {

constexpr int kMaxWarps = 16;
constexpr int kXPad = 32;       // halves of padding per activation column: conflict-free B loads
constexpr int kMaxTok = 16;
constexpr int kBatchBytes = 128;          // weight bytes per row in one batch of a warp
constexpr int kSlotW = 16 * kBatchBytes;  // weight bytes of one ring slot (16 rows)

enum { MW_F16 = 1, MW_Q8 = 2, MW_Q4 = 3 };  // same values as gemv.cu's weight types

template <int WT>
struct MmaFmt;
template <>
struct MmaFmt<MW_F16> {
  static constexpr int BLK_BYTES = 64;  // bytes of one 32-element block of a row
  static constexpr bool Q = false;
};
template <>
struct MmaFmt<MW_Q8> {
  static constexpr int BLK_BYTES = 32;
  static constexpr bool Q = true;
};
template <>
struct MmaFmt<MW_Q4> {
  static constexpr int BLK_BYTES = 16;
  static constexpr bool Q = true;
};

// Blocks per batch, and the scale bytes of a slot (16 rows x BPB fp16 scales).
template <int WT>
struct Slot {
  static constexpr int BPB = kBatchBytes / MmaFmt<WT>::BLK_BYTES;
  static constexpr int SCALE_BYTES = MmaFmt<WT>::Q ? 16 * BPB * 2 : 0;
  static constexpr int MAT_BYTES = kSlotW + SCALE_BYTES;  // one matrix's share of a slot
};

struct MmaGemvParams {
  const void* W;
  const uint16_t* Ws;
  const void* W2;  // up matrix (SWIGLU)
  const uint16_t* W2s;
  const void* x;
  int x_f16;
  int ldx;
  const float* gamma;
  float eps;
  int epi;
  void* y;
  int y_f16;
  int ldy;
  const float* aux;
  int M, K, nb, ncols, lo;
  size_t row_bytes;
  int kw;        // K slices per row tile (power of two <= warps per CTA)
  int depth;     // ring slots per warp (2..4)
  int n_groups;  // row groups of 16 * (warps / kw) rows
};

__device__ __forceinline__ uint32_t hsub2_u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// d = A(16x16, row) * B(16x8, col) + c, fp16 operands, fp32 accumulation.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1,
                                          const float (&c)[4]) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
        "f"(c[3]));
}

// int8 x4 -> fp16 pairs (e0, e1), (e2, e3), exact: 0x64uu is 1024 + u, u = q + 128.
__device__ __forceinline__ void q8_pairs(uint32_t w, uint32_t& p01, uint32_t& p23) {
  const uint32_t u = w ^ 0x80808080u;
  p01 = hsub2_u(__byte_perm(u, 0x64646464u, 0x4140), 0x64806480u);  // - 1152
  p23 = hsub2_u(__byte_perm(u, 0x64646464u, 0x4342), 0x64806480u);
}

// 8 nibbles (byte j = e_{2j} | e_{2j+1} << 4, value = (n ^ 8) - 8) -> fp16 pairs
// (e0, e4), (e1, e5), (e2, e6), (e3, e7), exact.
__device__ __forceinline__ void q4_pairs(uint32_t w, uint32_t (&p)[4]) {
  const uint32_t w8 = w >> 8;
  p[0] = hsub2_u((w & 0x000F000Fu) ^ 0x64086408u, 0x64086408u);               // 1024+m - 1032
  p[1] = hfma2_u((w & 0x00F000F0u) ^ 0x64806480u, 0x2C002C00u, 0xD480D480u);  // (1024+16m)/16-72
  p[2] = hsub2_u((w8 & 0x000F000Fu) ^ 0x64086408u, 0x64086408u);
  p[3] = hfma2_u((w8 & 0x00F000F0u) ^ 0x64806480u, 0x2C002C00u, 0xD480D480u);
}

// ---- cp.async (global -> shared, no register staging) ------------------------------------
// The lanes of a row ask for 32-64 B at a time; the L2::256B prefetch size makes each miss fetch
// the whole aligned 256 B of the row from HBM, which the next copies then find in L2.

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint.L2::256B [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "l"(pol)
               : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src, uint64_t pol) {
  asm volatile("cp.async.ca.shared.global.L2::cache_hint.L2::256B [%0], [%1], 8, %2;" ::"r"(dst), "l"(src),
               "l"(pol)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Wait until at most depth - 1 of this thread's groups are pending (depth is warp-uniform).
__device__ __forceinline__ void cp_async_wait_ring(int depth) {
  switch (depth) {
    case 2: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
  }
}

// A lane's 64 weight bytes of a slot are 4 chunks of 16 B; chunk c of every lane lies in plane c
// (512 B, lane-major), so the warp's copies into a plane and its LDS.128 reads of it are
// contiguous (8-byte copies: two wavefronts per 256 B; reads: conflict-free).
__device__ __forceinline__ int chunk_off(int lane, int c) { return c * 512 + lane * 16; }

// This lane's share of one batch: rows g and g + 8 of the tile (w0, w1: their first byte plus
// the lane's offset), 128 bytes per row from byte bat * 128; the scales of the tile's 16 rows
// (lanes 0-15, one row each, from ws).
template <int WT, bool IM8>
__device__ __forceinline__ void issue_matrix(uint32_t slot, const char* w0, const char* w1,
                                             const uint16_t* ws, int bat, int lane, uint64_t pol) {
  const char* rows[2] = {w0, w1};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const char* base = rows[h] + (size_t)bat * kBatchBytes;
    if constexpr (WT == MW_F16 || (IM8 && WT == MW_Q8)) {
      // fp16: chunk 2h + j = block j, bytes [64j + 16t, +16); int8 digits path: block pair j,
      // bytes [64j + 16t, +16) (lanes 0-1 hold the pair's first block, lanes 2-3 its second)
#pragma unroll
      for (int j = 0; j < 2; ++j) cp_async16(slot + chunk_off(lane, 2 * h + j), base + 64 * j, pol);
    } else {  // piece 4h + j (q8: block j; q4: block pair j): bytes [32j + 8t, +8)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        cp_async8(slot + chunk_off(lane, 2 * h + (j >> 1)) + 8 * (j & 1), base + 32 * j, pol);
    }
  }
  if constexpr (MmaFmt<WT>::Q) {
    constexpr int BPB = Slot<WT>::BPB;
    if (lane < 16) {
      const uint16_t* sp = ws + (size_t)bat * BPB;
      const uint32_t d = slot + kSlotW + lane * BPB * 2;
      if constexpr (BPB == 4)
        cp_async8(d, sp, pol);
      else
        cp_async16(d, sp, pol);
    }
  }
}

// Registers of one batch of one matrix: the lane's 16 words (two rows) and the two rows' scales.
template <int WT>
struct Raw {
  uint32_t w[2][8];
  uint32_t s[2][MmaFmt<WT>::Q ? Slot<WT>::BPB / 2 : 1];
};

template <int WT>
__device__ __forceinline__ void read_matrix(Raw<WT>& r, const char* slot, int lane, int g) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 v = *reinterpret_cast<const uint4*>(slot + chunk_off(lane, c));
    r.w[c >> 1][4 * (c & 1)] = v.x;
    r.w[c >> 1][4 * (c & 1) + 1] = v.y;
    r.w[c >> 1][4 * (c & 1) + 2] = v.z;
    r.w[c >> 1][4 * (c & 1) + 3] = v.w;
  }
  if constexpr (MmaFmt<WT>::Q) {
    constexpr int BPB = Slot<WT>::BPB;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const char* sp = slot + kSlotW + (g + 8 * h) * BPB * 2;
      if constexpr (BPB == 4) {
        const uint2 v = *reinterpret_cast<const uint2*>(sp);
        r.s[h][0] = v.x;
        r.s[h][1] = v.y;
      } else {
        const uint4 v = *reinterpret_cast<const uint4*>(sp);
        r.s[h][0] = v.x;
        r.s[h][1] = v.y;
        r.s[h][2] = v.z;
        r.s[h][3] = v.w;
      }
    }
  }
}

__device__ __forceinline__ float scale_of(const uint32_t* s, int j) {
  const uint32_t w = s[j >> 1];
  return h2f((uint16_t)((j & 1) ? (w >> 16) : (w & 0xFFFFu)));
}

// Multiply one batch into acc[NT][4].  xs: activation columns; bat: batch index along K.
template <int WT, int NT>
__device__ __forceinline__ void compute_batch(const Raw<WT>& r, float (&acc)[NT][4],
                                              const uint16_t* xs, int XS, int ncols, int bat,
                                              int g, int t) {
  constexpr int BPB = Slot<WT>::BPB;
  uint32_t wq[2][8];  // q4: per row, the word of each block of this lane after the exchange
  if constexpr (WT == MW_Q4) {
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t recv = __shfl_xor_sync(0xffffffffu, r.w[h][2 * j + 1], 2);
        const bool low = t < 2;
        wq[h][2 * j] = low ? r.w[h][2 * j] : recv;      // block 2j (even)
        wq[h][2 * j + 1] = low ? recv : r.w[h][2 * j];  // block 2j + 1 (odd)
      }
  }
  const int brt = ((t & 1) << 1) | (t >> 1);
#pragma unroll
  for (int j = 0; j < BPB; ++j) {
    // A operands of the two k16 steps: {row g pair0, row g+8 pair0, row g pair1, row g+8 pair1}
    uint32_t a[2][4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if constexpr (WT == MW_F16) {
        a[0][h] = r.w[h][4 * j];
        a[0][h + 2] = r.w[h][4 * j + 1];
        a[1][h] = r.w[h][4 * j + 2];
        a[1][h + 2] = r.w[h][4 * j + 3];
      } else if constexpr (WT == MW_Q8) {
        q8_pairs(r.w[h][2 * j], a[0][h], a[0][h + 2]);
        q8_pairs(r.w[h][2 * j + 1], a[1][h], a[1][h + 2]);
      } else {
        uint32_t pr[4];
        q4_pairs(wq[h][j], pr);
        a[0][h] = pr[0];
        a[0][h + 2] = pr[1];
        a[1][h] = pr[2];
        a[1][h + 2] = pr[3];
      }
    }
    // element offset of this lane's 8 activations in the block
    const int blk = bat * BPB + j;
    const int koff = 32 * blk + 8 * (WT == MW_Q4 ? (brt ^ (j & 1)) : t);
    float s0 = 1.f, s1 = 1.f;
    if constexpr (MmaFmt<WT>::Q) {
      s0 = scale_of(r.s[0], j);
      s1 = scale_of(r.s[1], j);
    }
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int c = 8 * n + g;
      uint4 b = make_uint4(0u, 0u, 0u, 0u);
      if (c < ncols) b = *reinterpret_cast<const uint4*>(xs + (size_t)c * XS + koff);
      // Every block starts from zero and is added in fp32: chaining the MMA accumulator over
      // a whole K slice loses accuracy (the tensor core's internal accumulation is not an fp32
      // add; measured on the decode step: 2.4x the error of fp32 FMAs, 1.4e-2 on a token).
      const float z[4] = {0.f, 0.f, 0.f, 0.f};
      float d[4];
      mma_16816(d, a[0][0], a[0][1], a[0][2], a[0][3], b.x, b.y, z);
      mma_16816(d, a[1][0], a[1][1], a[1][2], a[1][3], b.z, b.w, d);
      if constexpr (MmaFmt<WT>::Q) {
        acc[n][0] = fmaf(s0, d[0], acc[n][0]);
        acc[n][1] = fmaf(s0, d[1], acc[n][1]);
        acc[n][2] = fmaf(s1, d[2], acc[n][2]);
        acc[n][3] = fmaf(s1, d[3], acc[n][3]);
      } else {
        acc[n][0] += d[0];
        acc[n][1] += d[1];
        acc[n][2] += d[2];
        acc[n][3] += d[3];
      }
    }
  }
}

// 8 activations of token tok starting at element 8i, as floats.
__device__ __forceinline__ void load_x8(const MmaGemvParams& p, int tok, int i, float (&v)[8]) {
  if (p.x_f16) {
    const uint4 u = *reinterpret_cast<const uint4*>(
        reinterpret_cast<const uint16_t*>(p.x) + (size_t)tok * p.ldx + 8 * i);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = h2f2(w[q]);
      v[2 * q] = f.x;
      v[2 * q + 1] = f.y;
    }
  } else {
    const float4* xp =
        reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.x) + (size_t)tok * p.ldx) +
        2 * i;
    const float4 a = xp[0], b = xp[1];
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w;
    v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  }
}

// gamma[8i .. 8i + 8), eight independent loads (all ones without gamma: multiplying by them is
// exact).
__device__ __forceinline__ void load_gamma8(const MmaGemvParams& p, int i, float (&g)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) g[e] = p.gamma ? __ldg(p.gamma + 8 * i + e) : 1.f;
}

// One 8-element group of a token as hi and lo fp16 columns: x * ns * gamma * f, in the staged
// element order (natural, or (0,4)(1,5)(2,6)(3,7) for 4-bit weights).
template <bool P4>
__device__ __forceinline__ void store_hilo8(uint16_t* xs, int XS, int tok, int i, const float (&v)[8],
                                            const float (&g)[8], float ns, float f) {
  constexpr int perm[8] = {0, P4 ? 4 : 1, P4 ? 1 : 2, P4 ? 5 : 3, P4 ? 2 : 4, P4 ? 6 : 5, P4 ? 3 : 6, 7};
  uint32_t hi[4], lo[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint16_t h[2], l[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int e = perm[2 * q + u];
      float xv = v[e] * ns;
      xv *= g[e];
      xv *= f;
      h[u] = f2h(xv);
      l[u] = f2h(xv - h2f(h[u]));
    }
    hi[q] = (uint32_t)h[0] | ((uint32_t)h[1] << 16);
    lo[q] = (uint32_t)l[0] | ((uint32_t)l[1] << 16);
  }
  *reinterpret_cast<uint4*>(xs + (size_t)(2 * tok) * XS + 8 * i) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  *reinterpret_cast<uint4*>(xs + (size_t)(2 * tok + 1) * XS + 8 * i) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

// Stage the activation columns (see the file comment).  tok_inv[t] undoes the token's scale.
// Staging reads what the previous kernel wrote, so it is on the critical path: loads of
// several tokens of a group are issued before the first is used.
template <int WT>
__device__ void stage_columns(const MmaGemvParams& p, uint16_t* xs, int XS, float* tok_inv) {
  __shared__ float st_ss[kMaxWarps][kMaxTok], st_mx[kMaxWarps][kMaxTok];
  __shared__ float tok_norm[kMaxTok], tok_pow[kMaxTok];
  const int tid = threadIdx.x, nthr = blockDim.x, warp = tid >> 5, lane = tid & 31;
  const int n8 = p.K / 8, nb = p.nb;
  if (p.lo) {
    // per token: the sum of squares and the largest |x * gamma|; two tokens per pass over the
    // thread's groups, their loads (and gamma's) issued together
    for (int t0 = 0; t0 < nb; t0 += 2) {
      const bool two = t0 + 1 < nb;
      float ss0 = 0.f, mx0 = 0.f, ss1 = 0.f, mx1 = 0.f;
      for (int i = tid; i < n8; i += nthr) {
        float v0[8], v1[8], g[8];
        load_x8(p, t0, i, v0);
        if (two) load_x8(p, t0 + 1, i, v1);
        load_gamma8(p, i, g);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          ss0 = fmaf(v0[e], v0[e], ss0);
          mx0 = fmaxf(mx0, fabsf(v0[e] * g[e]));
        }
        if (two) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            ss1 = fmaf(v1[e], v1[e], ss1);
            mx1 = fmaxf(mx1, fabsf(v1[e] * g[e]));
          }
        }
      }
      ss0 = warp_sum(ss0);
      mx0 = warp_max(mx0);
      ss1 = warp_sum(ss1);
      mx1 = warp_max(mx1);
      if (lane == 0) {
        st_ss[warp][t0] = ss0;
        st_mx[warp][t0] = mx0;
        if (two) {
          st_ss[warp][t0 + 1] = ss1;
          st_mx[warp][t0 + 1] = mx1;
        }
      }
    }
    __syncthreads();
    if (tid < nb) {
      float ss = 0.f, mx = 0.f;
      for (int w = 0; w < (nthr >> 5); ++w) {
        ss += st_ss[w][tid];
        mx = fmaxf(mx, st_mx[w][tid]);
      }
      const float ns = p.gamma ? rsqrtf(ss / (float)p.K + p.eps) : 1.f;
      const float amax = ns * mx;
      float f = 1.f, inv = 1.f;
      if (amax > 0.f && amax <= 3.0e38f) {  // scale the token's largest value into [2^13, 2^14)
        int ex;
        frexpf(amax, &ex);
        ex = max(ex, -100);
        f = ldexpf(1.f, 14 - ex);
        inv = ldexpf(1.f, ex - 14);
      }
      tok_norm[tid] = ns;
      tok_pow[tid] = f;
      tok_inv[tid] = inv;
    }
    __syncthreads();
  } else if (tid < nb) {
    tok_inv[tid] = 1.f;
  }
  // element order of a staged group of 8: natural, or (0,4)(1,5)(2,6)(3,7) for 4-bit weights
  constexpr bool P4 = WT == MW_Q4;
  if (!p.lo) {
    // fp16 activations, no norm: copied (reordered for 4-bit weights).  Staging reads what the
    // previous kernel wrote, so it is on the critical path: each thread issues the loads of TC
    // tokens of one 8-element group before storing any of them (one memory latency per batch
    // of tokens, not one per token).
    constexpr int TC = 4;
    for (int i = tid; i < n8; i += nthr) {
#pragma unroll
      for (int t0 = 0; t0 < kMaxTok; t0 += TC) {
        if (t0 >= nb) break;
        uint4 x[TC];
#pragma unroll
        for (int u = 0; u < TC; ++u)
          if (t0 + u < nb)
            x[u] = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.x) +
                                                   (size_t)(t0 + u) * p.ldx + 8 * i);
#pragma unroll
        for (int u = 0; u < TC; ++u) {
          if (t0 + u >= nb) break;
          uint32_t hi[4];
          if constexpr (P4) {
            hi[0] = __byte_perm(x[u].x, x[u].z, 0x5410);  // (x0, x4)
            hi[1] = __byte_perm(x[u].x, x[u].z, 0x7632);  // (x1, x5)
            hi[2] = __byte_perm(x[u].y, x[u].w, 0x5410);  // (x2, x6)
            hi[3] = __byte_perm(x[u].y, x[u].w, 0x7632);  // (x3, x7)
          } else {
            hi[0] = x[u].x, hi[1] = x[u].y, hi[2] = x[u].z, hi[3] = x[u].w;
          }
          *reinterpret_cast<uint4*>(xs + (size_t)(t0 + u) * XS + 8 * i) =
              make_uint4(hi[0], hi[1], hi[2], hi[3]);
        }
      }
    }
    __syncthreads();
    return;
  }
  // hi + lo columns of x * norm * gamma * 2^e, two tokens per pass as above
  for (int t0 = 0; t0 < nb; t0 += 2) {
    const bool two = t0 + 1 < nb;
    for (int i = tid; i < n8; i += nthr) {
      float v0[8], v1[8], g[8];
      load_x8(p, t0, i, v0);
      if (two) load_x8(p, t0 + 1, i, v1);
      load_gamma8(p, i, g);
      store_hilo8<P4>(xs, XS, t0, i, v0, g, tok_norm[t0], tok_pow[t0]);
      if (two) store_hilo8<P4>(xs, XS, t0 + 1, i, v1, g, tok_norm[t0 + 1], tok_pow[t0 + 1]);
    }
  }
  __syncthreads();
}

// ---- batch 1 on the integer tensor cores ------------------------------------------------
//
// The token is scaled by a power of two into a 21-bit integer x_int (|x_int| <= 2^20: 2^-20 of
// the token's largest value) and split into three balanced base-128 digits, x_int = d0 + 128 d1 +
// 16384 d2 with |d| <= 65, stored as three int8 columns.  Weights enter mma.sync m16n8k32 as
// they are (int8; 4-bit nibbles as unsigned n ^ 8 = q + 8, corrected by 8 * the block's digit
// sum), the int32 block results are exact, and each is scaled in fp32.  Two blocks share an MMA:
// lanes t = 0, 1 carry the first block's k values and columns 0-2 its digits, lanes 2, 3 the
// second block's and columns 3-5, so one MMA pair yields (block, digit) sums for two blocks.

__device__ __forceinline__ void imma_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                           uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void immau_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                            uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Exact int -> float for |v| < 2^22 (the integer is added under the exponent of 1.5 * 2^23).
__device__ __forceinline__ float small_int_to_float(int v) {
  return __int_as_float(v + 0x4B400000) - 12582912.0f;
}

// acc[e]: rows (g, g, g+8, g+8) x columns (2t, 2t+1, 2t, 2t+1); column c = (block c / 3 of the
// pair, digit c % 3); columns 6, 7 are unused.
template <int WT>
__device__ __forceinline__ void compute_batch_im8(const Raw<WT>& r, float (&acc)[4],
                                                  const int8_t* xd, int XD, const int* dsum,
                                                  int bat, int g, int t) {
  constexpr int BPB = Slot<WT>::BPB;
  constexpr int NP = BPB / 2;  // block pairs per batch
  const bool active = g < 6 && g / 3 == (t >> 1);  // this lane's k values meet column g
  const int8_t* xcol = xd + (size_t)(g % 3) * XD;
  const int c0 = 2 * t, c1 = 2 * t + 1;
#pragma unroll
  for (int P = 0; P < NP; ++P) {
    const int blk_l = bat * BPB + 2 * P + (t >> 1);  // the block of this lane's k values
    int d[4] = {0, 0, 0, 0};
#pragma unroll
    for (int st = 0; st < 2; ++st) {
      uint32_t a0, a1, a2, a3;
      if constexpr (WT == MW_Q8) {  // 16 bytes per row per pair: words 4P..4P+3
        a0 = r.w[0][4 * P + 2 * st];
        a2 = r.w[0][4 * P + 2 * st + 1];
        a1 = r.w[1][4 * P + 2 * st];
        a3 = r.w[1][4 * P + 2 * st + 1];
      } else {  // 8 bytes per row per pair: word 2P + st, nibbles widened to bytes u = n ^ 8
        const uint32_t w0 = r.w[0][2 * P + st], w1 = r.w[1][2 * P + st];
        a0 = (w0 & 0x0F0F0F0Fu) ^ 0x08080808u;         // elements 0, 2, 4, 6
        a2 = ((w0 >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;  // elements 1, 3, 5, 7
        a1 = (w1 & 0x0F0F0F0Fu) ^ 0x08080808u;
        a3 = ((w1 >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
      }
      uint2 b = make_uint2(0u, 0u);
      if (active)
        b = *reinterpret_cast<const uint2*>(xcol + 32 * blk_l + 16 * (t & 1) + 8 * st);
      if constexpr (WT == MW_Q8)
        imma_16832(d, a0, a1, a2, a3, b.x, b.y);
      else
        immau_16832(d, a0, a1, a2, a3, b.x, b.y);
    }
    const int bc0 = bat * BPB + 2 * P + c0 / 3, bc1 = bat * BPB + 2 * P + c1 / 3;
    if constexpr (WT == MW_Q4) {  // q = u - 8: subtract 8 * the block's digit sum
      if (c0 < 6) {
        d[0] -= 8 * dsum[4 * bc0 + c0 % 3];
        d[2] -= 8 * dsum[4 * bc0 + c0 % 3];
      }
      if (c1 < 6) {
        d[1] -= 8 * dsum[4 * bc1 + c1 % 3];
        d[3] -= 8 * dsum[4 * bc1 + c1 % 3];
      }
    }
    const int j0 = 2 * P + min(c0 / 3, 1), j1 = 2 * P + min(c1 / 3, 1);
    acc[0] = fmaf(small_int_to_float(d[0]), scale_of(r.s[0], j0), acc[0]);
    acc[1] = fmaf(small_int_to_float(d[1]), scale_of(r.s[0], j1), acc[1]);
    acc[2] = fmaf(small_int_to_float(d[2]), scale_of(r.s[1], j0), acc[2]);
    acc[3] = fmaf(small_int_to_float(d[3]), scale_of(r.s[1], j1), acc[3]);
  }
}

// Stage the single token as 3 int8 digit columns (4-bit weights: each 8 elements stored as
// 0,2,4,6,1,3,5,7, and the blocks' digit sums).  tok_inv[0] undoes the power-of-two scale.
template <int WT>
__device__ void stage_digits(const MmaGemvParams& p, int8_t* xd, int XD, int* dsum, float* tok_inv) {
  __shared__ float st_ss[kMaxWarps], st_mx[kMaxWarps];
  __shared__ float tok_mul;
  const int tid = threadIdx.x, nthr = blockDim.x, warp = tid >> 5, lane = tid & 31;
  const int n8 = p.K / 8;
  float ss = 0.f, mx = 0.f;
  for (int i = tid; i < n8; i += nthr) {
    float v[8];
    load_x8(p, 0, i, v);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      ss = fmaf(v[e], v[e], ss);
      mx = fmaxf(mx, fabsf(p.gamma ? v[e] * __ldg(p.gamma + 8 * i + e) : v[e]));
    }
  }
  ss = warp_sum(ss);
  mx = warp_max(mx);
  if (lane == 0) {
    st_ss[warp] = ss;
    st_mx[warp] = mx;
  }
  __syncthreads();
  if (tid == 0) {
    float s = 0.f, m = 0.f;
    for (int w = 0; w < (nthr >> 5); ++w) {
      s += st_ss[w];
      m = fmaxf(m, st_mx[w]);
    }
    const float ns = p.gamma ? rsqrtf(s / (float)p.K + p.eps) : 1.f;
    const float amax = ns * m;
    float f = 0.f, inv = 0.f;  // an all-zero token stays zero
    if (amax > 0.f && amax <= 3.0e38f) {  // largest |x_int| <= 2^20
      int ex;
      frexpf(amax, &ex);
      ex = max(ex, -100);
      f = ldexpf(1.f, 20 - ex);
      inv = ldexpf(1.f, ex - 20);
    }
    tok_mul = ns * f;  // one rounding; the result is then rounded to an integer anyway
    tok_inv[0] = inv;
  }
  __syncthreads();
  const float mul = tok_mul;
  constexpr bool P4 = WT == MW_Q4;
  constexpr int perm[8] = {0, P4 ? 2 : 1, P4 ? 4 : 2, P4 ? 6 : 3, P4 ? 1 : 4, P4 ? 3 : 5, P4 ? 5 : 6, 7};
  for (int i = tid; i < n8; i += nthr) {  // n8 is a multiple of 32: whole warps
    float v[8];
    load_x8(p, 0, i, v);
    uint32_t dw[3][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}};
    int sum[3] = {0, 0, 0};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int src = perm[e];
      float xv = v[src];
      if (p.gamma) xv *= __ldg(p.gamma + 8 * i + src);
      const int xi = __float2int_rn(xv * mul);
      const int d0 = ((xi + 64) & 127) - 64;
      const int r1 = (xi - d0) >> 7;
      const int d1 = ((r1 + 64) & 127) - 64;
      const int d2 = (r1 - d1) >> 7;
      const int dd[3] = {d0, d1, d2};
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        dw[k][e >> 2] |= ((uint32_t)dd[k] & 0xFFu) << (8 * (e & 3));
        sum[k] += dd[k];
      }
    }
#pragma unroll
    for (int k = 0; k < 3; ++k)
      *reinterpret_cast<uint2*>(xd + (size_t)k * XD + 8 * i) = make_uint2(dw[k][0], dw[k][1]);
    if constexpr (P4) {  // a block is 4 consecutive groups: lanes 4m .. 4m + 3
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        sum[k] += __shfl_xor_sync(0xffffffffu, sum[k], 1);
        sum[k] += __shfl_xor_sync(0xffffffffu, sum[k], 2);
      }
      if ((i & 3) == 0) *reinterpret_cast<int4*>(dsum + 4 * (i >> 2)) = make_int4(sum[0], sum[1], sum[2], 0);
    }
  }
  __syncthreads();
}

// Floats per row of a warp's partial tile: the columns (even) plus 2, so that the reduction's
// reads of consecutive rows spread over the banks.
__host__ __device__ inline int red_stride(int ncols) { return ((ncols + 1) & ~1) + 2; }

// Dynamic shared memory: [activation columns][partial tiles of every warp, two buffers (x2 more
// for SWIGLU)][ring: warps x depth x slot].
template <int WT, bool DUAL, bool IM8>
struct Layout {
  // fp16 path: ncols fp16 columns.  int8 digits path: 3 int8 columns (+ 4-bit: the blocks' digit
  // sums, int32 [K/32][4]).
  __host__ __device__ static size_t xs_bytes(int ncols, int K) {
    if (IM8) return (size_t)3 * (K + kXPad) + (WT == MW_Q4 ? (size_t)(K / 32) * 16 : 0);
    return (size_t)ncols * (K + kXPad) * 2;
  }
  __host__ __device__ static size_t red_floats(int nw, int ncols) { return (size_t)nw * 16 * red_stride(ncols); }
  __host__ __device__ static size_t red_bytes(int nw, int ncols) {
    return red_floats(nw, ncols) * 4 * 2 * (DUAL ? 2 : 1);
  }
  static constexpr int SLOT = Slot<WT>::MAT_BYTES * (DUAL ? 2 : 1);
  __host__ __device__ static size_t total(int ncols, int K, int nw, int depth) {
    return xs_bytes(ncols, K) + red_bytes(nw, ncols) + (size_t)nw * depth * SLOT;
  }
};

// One row group of 16 * mw rows: its first row, and this lane's row pointers into W (and W2).
struct RowPtrs {
  const char* w0;
  const char* w1;
  const uint16_t* ws;
};

template <int WT, int NT, bool DUAL, int MINB, bool IM8>
__global__ void __launch_bounds__(kMaxWarps * 32, MINB) gemv_mma_kernel(const __grid_constant__ MmaGemvParams p) {
  using L = Layout<WT, DUAL, IM8>;
  constexpr int MAT = Slot<WT>::MAT_BYTES;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ float tok_inv[kMaxTok];

  const int nw = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int K = p.K, XS = K + kXPad, M = p.M, depth = p.depth;
  const int kw = p.kw, mw = nw / kw, rg = warp / kw, ks = warp % kw;
  const int nbt = (int)(p.row_bytes / kBatchBytes);  // batches per row
  const int b0 = ks * nbt / kw, nbw = (ks + 1) * nbt / kw - b0;
  const int nscale = K / 32;
  const int RS = red_stride(p.ncols);
  const size_t red_n = L::red_floats(nw, p.ncols);

  uint16_t* xs = reinterpret_cast<uint16_t*>(smem);
  float* red_base = reinterpret_cast<float*>(smem + L::xs_bytes(p.ncols, K));
  unsigned char* ring =
      smem + L::xs_bytes(p.ncols, K) + L::red_bytes(nw, p.ncols) + (size_t)warp * depth * L::SLOT;
  const uint32_t ring_s = smem_u32(ring);

  // this CTA's row groups: blockIdx.x, + gridDim.x, ...; this warp's batches of each: nbw
  const int n_mine =
      (int)blockIdx.x < p.n_groups ? (p.n_groups - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const uint64_t pol = l2_evict_first();
  // lane offsets inside a row's batch: fp16 (and int8 on the integer path) 16 B per lane at 16t,
  // otherwise 8 B per lane at 8t
  const size_t lane_off =
      (size_t)(WT == MW_F16 || (IM8 && WT == MW_Q8) ? 16 * t : 8 * t) + (size_t)b0 * kBatchBytes;
  auto rows_of = [&](int gi, const char* W, const uint16_t* Ws) {
    const int row0 = (((int)blockIdx.x + gi * (int)gridDim.x) * mw + rg) * 16;
    RowPtrs r;
    r.w0 = W + (size_t)min(row0 + g, M - 1) * p.row_bytes + lane_off;
    r.w1 = W + (size_t)min(row0 + g + 8, M - 1) * p.row_bytes + lane_off;
    r.ws = Ws ? Ws + (size_t)min(row0 + (lane & 15), M - 1) * nscale + (size_t)b0 * Slot<WT>::BPB : nullptr;
    return r;
  };

  // producer state: the next batch to request (group igi, batch ij of the slice) and its slot
  int igi = 0, ij = 0, islot = 0;
  RowPtrs ip = rows_of(0, static_cast<const char*>(p.W), p.Ws), ip2{};
  if constexpr (DUAL) ip2 = rows_of(0, static_cast<const char*>(p.W2), p.W2s);
  auto issue = [&]() {  // one group of copies per call, empty past the end
    if (igi < n_mine) {
      const uint32_t slot = ring_s + (uint32_t)(islot * L::SLOT);
      issue_matrix<WT, IM8>(slot, ip.w0, ip.w1, ip.ws, ij, lane, pol);
      if constexpr (DUAL) issue_matrix<WT, IM8>(slot + MAT, ip2.w0, ip2.w1, ip2.ws, ij, lane, pol);
      if (++ij == nbw) {
        ij = 0;
        ++igi;
        ip = rows_of(igi, static_cast<const char*>(p.W), p.Ws);
        if constexpr (DUAL) ip2 = rows_of(igi, static_cast<const char*>(p.W2), p.W2s);
      }
    }
    islot = islot + 1 == depth ? 0 : islot + 1;
    cp_async_commit();
  };

  for (int d = 0; d < depth; ++d) issue();  // weights do not depend on the previous kernel
  pdl_wait();
  int8_t* xd = reinterpret_cast<int8_t*>(smem);  // integer path: 3 digit columns, then digit sums
  int* dsum = reinterpret_cast<int*>(smem + (size_t)3 * XS);
  if constexpr (IM8)
    stage_digits<WT>(p, xd, XS, dsum, tok_inv);
  else
    stage_columns<WT>(p, xs, XS, tok_inv);
  pdl_launch_dependents();

  int rslot = 0;
  for (int gi = 0; gi < n_mine; ++gi) {
    const int grp = (int)blockIdx.x + gi * (int)gridDim.x;
    float acc[NT][4], acc2[DUAL ? NT : 1][4];
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc[n][e] = 0.f;
        if constexpr (DUAL) acc2[n][e] = 0.f;
      }
    for (int j = 0; j < nbw; ++j) {
      cp_async_wait_ring(depth);
      __syncwarp();  // the scale rows were fetched by other lanes
      const char* slot = reinterpret_cast<const char*>(ring) + rslot * L::SLOT;
      Raw<WT> r, r2;
      read_matrix<WT>(r, slot, lane, g);
      if constexpr (DUAL) read_matrix<WT>(r2, slot + MAT, lane, g);
      __syncwarp();  // every lane has read the slot before it is refilled
      rslot = rslot + 1 == depth ? 0 : rslot + 1;
      issue();
      if constexpr (IM8) {
        compute_batch_im8<WT>(r, acc[0], xd, XS, dsum, b0 + j, g, t);
        if constexpr (DUAL) compute_batch_im8<WT>(r2, acc2[0], xd, XS, dsum, b0 + j, g, t);
      } else {
        compute_batch<WT, NT>(r, acc, xs, XS, p.ncols, b0 + j, g, t);
        if constexpr (DUAL) compute_batch<WT, NT>(r2, acc2, xs, XS, p.ncols, b0 + j, g, t);
      }
    }

    // partial tiles -> shared memory (two buffers: one barrier per group); then sum the K
    // slices in order and apply the epilogue
    float* red = red_base + (size_t)(gi & 1) * red_n * (DUAL ? 2 : 1);
    float* red2 = red + red_n;
    float* rw = red + warp * 16 * RS;
    float* rw2 = red2 + warp * 16 * RS;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      if (8 * n + 2 * t < p.ncols) {
        *reinterpret_cast<float2*>(rw + g * RS + 8 * n + 2 * t) = make_float2(acc[n][0], acc[n][1]);
        *reinterpret_cast<float2*>(rw + (g + 8) * RS + 8 * n + 2 * t) = make_float2(acc[n][2], acc[n][3]);
        if constexpr (DUAL) {
          *reinterpret_cast<float2*>(rw2 + g * RS + 8 * n + 2 * t) = make_float2(acc2[n][0], acc2[n][1]);
          *reinterpret_cast<float2*>(rw2 + (g + 8) * RS + 8 * n + 2 * t) =
              make_float2(acc2[n][2], acc2[n][3]);
        }
      }
    }
    __syncthreads();
    const int rows_grp = 16 * mw;
    for (int o = threadIdx.x; o < rows_grp * p.nb; o += blockDim.x) {
      const int r = o % rows_grp, tok = o / rows_grp, rt = r >> 4, rr = r & 15;
      const int row = grp * rows_grp + r;
      const int c = p.lo ? 2 * tok : tok;
      float s = 0.f, s2 = 0.f;
      for (int k = 0; k < kw; ++k) {
        const int off = ((rt * kw + k) * 16 + rr) * RS + c;
        if constexpr (IM8) {  // columns (block of the pair, digit): weights 1, 128, 16384
          s += (red[off] + red[off + 3]) +
               ((red[off + 1] + red[off + 4]) * 128.f + (red[off + 2] + red[off + 5]) * 16384.f);
          if constexpr (DUAL)
            s2 += (red2[off] + red2[off + 3]) +
                  ((red2[off + 1] + red2[off + 4]) * 128.f + (red2[off + 2] + red2[off + 5]) * 16384.f);
        } else {
          s += p.lo ? red[off] + red[off + 1] : red[off];
          if constexpr (DUAL) s2 += p.lo ? red2[off] + red2[off + 1] : red2[off];
        }
      }
      if (row >= M) continue;
      s *= tok_inv[tok];
      const size_t yi = (size_t)tok * p.ldy + row;
      float v;
      if constexpr (DUAL) {
        v = silu(s) * (s2 * tok_inv[tok]);
      } else {
        v = s;
        if (p.epi == B2D_EPI_ADD) {
          v += p.y_f16 ? h2f(static_cast<const uint16_t*>(p.y)[yi]) : static_cast<const float*>(p.y)[yi];
        } else if (p.epi == B2D_EPI_GELU_MUL) {
          v = gelu_tanh(v) * p.aux[yi];
        }
      }
      if (p.y_f16)
        static_cast<uint16_t*>(p.y)[yi] = f2h(v);
      else
        static_cast<float*>(p.y)[yi] = v;
    }
    // no second barrier: the next group writes the other buffer, and this one again only after
    // the next group's barrier, which every thread reaches after finishing the loop above
  }
  asm volatile("cp.async.wait_all;" ::: "memory");  // no copy outlives the CTA
}

// Largest dynamic shared memory a CTA may use (the static part is < 2.5 KB).
constexpr size_t kMaxDynSmem = 220 * 1024;

// Warps per CTA and ring depth.  First choice: two CTAs of 16 warps per SM (more warps hide the
// dequant -> MMA -> FMA latencies) with 2 slots each -- not for two matrices, which need more
// than 64 registers; then one CTA of 16 warps with 4 or 3 slots; then 8 warps with 4 down to 2.
// False if none fits next to the activation columns.
#ifndef B2D_MMA_TWO_CTAS
#define B2D_MMA_TWO_CTAS 1
#endif
template <int WT, bool DUAL, bool IM8 = false>
bool pick_shape(int ncols, int K, int& nw, int& depth, int& per_sm) {
  using L = Layout<WT, DUAL, IM8>;
  if (B2D_MMA_TWO_CTAS && !DUAL && L::total(ncols, K, 16, 2) <= kMaxDynSmem / 2 - 4096) {
    nw = 16, depth = 2, per_sm = 2;
    return true;
  }
  for (int w = 16; w >= 8; w -= 8) {
    for (int d = 4; d >= (w == 16 ? 3 : 2); --d) {
      if (L::total(ncols, K, w, d) <= kMaxDynSmem) {
        nw = w, depth = d, per_sm = 1;
        return true;
      }
    }
  }
  return false;
}

template <int WT, int NT, bool DUAL, int MINB, bool IM8>
int launch_shape(MmaGemvParams& p, int nw, int depth, cudaStream_t stream) {
  auto kern = gemv_mma_kernel<WT, NT, DUAL, MINB, IM8>;
  const size_t smem = Layout<WT, DUAL, IM8>::total(p.ncols, p.K, nw, depth);
  static int cached_dev = -1;
  static size_t cached_smem = 0;
  static int cached_nw = 0;
  static int occ = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != cached_dev || smem != cached_smem || nw != cached_nw) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxDynSmem) !=
        cudaSuccess)
      return launch_status();
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, nw * 32, smem) != cudaSuccess)
      return launch_status();
    cached_dev = dev;
    cached_smem = smem;
    cached_nw = nw;
  }
  const int nbt = (int)(p.row_bytes / kBatchBytes);
  p.kw = 1;
  while (p.kw < nw && p.kw * 2 <= nbt) p.kw *= 2;
  p.depth = depth;
  const int rows_grp = 16 * (nw / p.kw);
  p.n_groups = (p.M + rows_grp - 1) / rows_grp;
  const int grid = std::min(p.n_groups, std::max(1, occ) * num_sms());
  return launch_pdl(kern, dim3(grid), dim3(nw * 32), smem, stream, p);
}

template <int WT, int NT, bool DUAL, bool IM8 = false>
int launch_mma(MmaGemvParams& p, cudaStream_t stream) {
  int nw = 0, depth = 0, per_sm = 0;
  if (!pick_shape<WT, DUAL, IM8>(p.ncols, p.K, nw, depth, per_sm)) return B2D_ERR_SHAPE;
  // two resident CTAs need <= 64 registers per thread
  if constexpr (!DUAL)
    if (per_sm == 2) return launch_shape<WT, NT, DUAL, 2, IM8>(p, nw, depth, stream);
  return launch_shape<WT, NT, DUAL, 1, IM8>(p, nw, depth, stream);
}

template <int WT, bool DUAL>
int launch_nt(MmaGemvParams& p, cudaStream_t stream) {
  return p.ncols <= 8 ? launch_mma<WT, 1, DUAL>(p, stream) : launch_mma<WT, 2, DUAL>(p, stream);
}

// Tokens per pass over W: the most (<= 16 columns) whose activation columns leave room for the
// warps' rings.
template <int WT, bool DUAL>
int max_tokens(int K, bool lo) {
  const int per = lo ? 2 : 1;
  int nw, depth, per_sm;
  for (int n = kMaxTok / per; n >= 1; --n)
    if (pick_shape<WT, DUAL>(n * per, K, nw, depth, per_sm)) return n;
  return 0;
}

}  // namespace

// Which weight formats take the tensor-core GEMV (bit d set: dtype d; fp32 weights never do:
// their products are not exact in fp16), and bit 4: quantized single tokens on the integer
// tensor cores (3 int8 digit columns) instead of fp16 operands -- off by default: measured on
// B200 it is no faster than the fp16-operand path (config 3 q8 4096x14336: 17.5 vs 18.3 us,
// 4096x4096: 8.1 vs 7.2 us; q4: 17.9 vs 16.3 and 8.2 vs 6.5 us).
constexpr int kMmaInt8B1 = 1 << 4;
#ifndef B2D_GEMV_MMA_MASK
#define B2D_GEMV_MMA_MASK ((1 << B2D_F16) | (1 << B2D_Q8_32) | (1 << B2D_Q4_32))
#endif
constexpr int kMmaFormats = (1 << B2D_F16) | (1 << B2D_Q8_32) | (1 << B2D_Q4_32) | kMmaInt8B1;

static int g_mma_mask = B2D_GEMV_MMA_MASK & kMmaFormats;

int gemv_mma_formats(int mask) {
  const int prev = __atomic_load_n(&g_mma_mask, __ATOMIC_RELAXED);
  if (mask >= 0) __atomic_store_n(&g_mma_mask, mask & kMmaFormats, __ATOMIC_RELAXED);
  return prev;
}

static int group_tokens(int w_dtype, bool dual, int K, bool lo) {
  switch (w_dtype) {
    case B2D_F16: return dual ? max_tokens<MW_F16, true>(K, lo) : max_tokens<MW_F16, false>(K, lo);
    case B2D_Q8_32: return dual ? max_tokens<MW_Q8, true>(K, lo) : max_tokens<MW_Q8, false>(K, lo);
    default: return dual ? max_tokens<MW_Q4, true>(K, lo) : max_tokens<MW_Q4, false>(K, lo);
  }
}

bool gemv_mma_eligible(int w_dtype, const void* W_scales, const void* W_up_scales, int K,
                       int epilogue) {
  const int mask = __atomic_load_n(&g_mma_mask, __ATOMIC_RELAXED);
  if (w_dtype < B2D_F16 || w_dtype > B2D_Q4_32 || !((mask >> w_dtype) & 1)) return false;
  const int blk_bytes = w_dtype == B2D_F16 ? 64 : (w_dtype == B2D_Q8_32 ? 32 : 16);
  const size_t row_bytes = (size_t)K * blk_bytes / 32;
  if (K % 32 || row_bytes % kBatchBytes) return false;
  const uintptr_t salign = (uintptr_t)(kBatchBytes / blk_bytes) * 2 - 1;  // a batch's scales: one copy
  if (w_dtype != B2D_F16 && ((reinterpret_cast<uintptr_t>(W_scales) & salign) ||
                             (W_up_scales && (reinterpret_cast<uintptr_t>(W_up_scales) & salign))))
    return false;
  return group_tokens(w_dtype, epilogue == B2D_EPI_SWIGLU, K, true) >= 1;
}

// Caller has validated pointers, shapes and alignment (gemv_dispatch) and gemv_mma_eligible.
int gemv_mma_dispatch(int w_dtype, const void* W, const void* W_scales, const void* W_up,
                      const void* W_up_scales, int x_dtype, const void* x, int ldx,
                      const float* gamma, float eps, int epilogue, int y_dtype, void* y, int ldy,
                      const float* aux, int M, int K, int batch, cudaStream_t stream) {
  const bool lo = !(x_dtype == B2D_F16 && gamma == nullptr);
  const bool dual = epilogue == B2D_EPI_SWIGLU;
  const int group = group_tokens(w_dtype, dual, K, lo);
  if (group < 1) return B2D_ERR_SHAPE;
  const int blk_bytes = w_dtype == B2D_F16 ? 64 : (w_dtype == B2D_Q8_32 ? 32 : 16);
  MmaGemvParams p = {};
  p.W = W;
  p.Ws = static_cast<const uint16_t*>(W_scales);
  p.W2 = W_up;
  p.W2s = static_cast<const uint16_t*>(W_up_scales);
  p.x_f16 = x_dtype == B2D_F16;
  p.ldx = ldx;
  p.gamma = gamma;
  p.eps = eps;
  p.epi = epilogue;
  p.y_f16 = y_dtype == B2D_F16;
  p.ldy = ldy;
  p.M = M;
  p.K = K;
  p.lo = lo;
  p.row_bytes = (size_t)K * blk_bytes / 32;
  const size_t xsz = p.x_f16 ? 2 : 4, ysz = p.y_f16 ? 2 : 4;
  const bool int8_b1 = w_dtype != B2D_F16 && (__atomic_load_n(&g_mma_mask, __ATOMIC_RELAXED) & kMmaInt8B1);
  for (int b0 = 0; b0 < batch; b0 += group) {
    p.nb = std::min(group, batch - b0);
    p.ncols = p.nb * (lo ? 2 : 1);
    p.x = static_cast<const char*>(x) + (size_t)b0 * ldx * xsz;
    p.y = static_cast<char*>(y) + (size_t)b0 * ldy * ysz;
    p.aux = aux ? aux + (size_t)b0 * ldy : nullptr;
    int st;
    if (p.nb == 1 && int8_b1) {  // one token: int8 weights x 3 int8 digit columns
      MmaGemvParams q = p;
      q.ncols = 6;
      q.lo = 0;
      if (w_dtype == B2D_Q8_32)
        st = dual ? launch_mma<MW_Q8, 1, true, true>(q, stream) : launch_mma<MW_Q8, 1, false, true>(q, stream);
      else
        st = dual ? launch_mma<MW_Q4, 1, true, true>(q, stream) : launch_mma<MW_Q4, 1, false, true>(q, stream);
      if (st != B2D_OK) return st;
      continue;
    }
    switch (w_dtype) {
      case B2D_F16:
        st = dual ? launch_nt<MW_F16, true>(p, stream) : launch_nt<MW_F16, false>(p, stream);
        break;
      case B2D_Q8_32:
        st = dual ? launch_nt<MW_Q8, true>(p, stream) : launch_nt<MW_Q8, false>(p, stream);
        break;
      default:
        st = dual ? launch_nt<MW_Q4, true>(p, stream) : launch_nt<MW_Q4, false>(p, stream);
        break;
    }
    if (st != B2D_OK) return st;
  }
  return B2D_OK;
}

}  // namespace b2d
