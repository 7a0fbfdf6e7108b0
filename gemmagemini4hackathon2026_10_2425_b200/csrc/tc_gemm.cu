// Batched decode GEMM on the 5th-generation tensor cores (sm_100a tcgen05 + TMEM + TMA).
//
//   Y[b, m] = epilogue( sum_k W[m, k] * X[b, k] ),  b < batch <= 32,  W fp16 [M, K], X fp16 [batch, K]
//
// Activations at fp32 precision (XS = 2): the reference multiplies fp16 weights by fp32
// activations (LK/kernels.metal:106-131).  An fp32 activation x is carried as two fp16 planes,
// hi = fp16(x) and lo = fp16(x - hi) (~22 significant bits); both planes are loaded into one B
// tile of 2N rows, so a single tcgen05.mma with N doubled produces W*hi and W*lo side by side in
// TMEM, and the epilogue adds the two columns of each token.  fp16 x fp16 products are exact
// and accumulate in fp32, so the result is the fp32-activation product.  The extra MMA columns
// cost no weight bytes (the tensor pipe is a few percent busy at decode batch sizes).
//
// Why tensor cores here: at batch 16-32 a decode GEMV does 32-64 flops per weight byte; keeping
// up with ~6.5 TB/s of HBM needs 200-400 TFLOP/s, beyond the CUDA cores' fp32 FMA rate.  The
// reference runs these projections as matvec_f16 / matvec_gate_up_silu (LK/kernels.metal:106-173)
// once per sequence; this kernel serves the whole ragged batch in one pass over the weights.
//
// Structure ("swap AB": weights are the MMA's M side, tokens its N side):
//  * one CTA per (128-row tile of W, K split); 128 threads;
//  * warp 0 / lane 0 streams W tiles [128 x 64] (and W_up tiles for SwiGLU) and X tiles [N x 64]
//    with TMA (cp.async.bulk.tensor, 128-byte swizzle) through a STAGES-deep shared-memory ring
//    guarded by mbarriers.  Weight tiles do not depend on the previous kernel, so the first ring
//    of them is issued before griddepcontrol.wait (programmatic dependent launch);
//  * warp 1 / lane 0 issues tcgen05.mma.cta_group::1.kind::f16 (M=128, N=16|32, K=16, fp32
//    accumulate) into TMEM and frees each ring slot with tcgen05.commit;
//  * all four warps read the accumulator tile back with tcgen05.ld (warp w owns TMEM lanes
//    32w..32w+31 = W rows), then finish the epilogue (store / residual add / SwiGLU / argmax);
//  * split-K: the K splits of a row tile run as one thread-block cluster (<= 8 CTAs); partial
//    tiles meet in distributed shared memory and each CTA reduces a slice of rows over its
//    peers in a fixed order (deterministic, no global round trip).
//  * every mbarrier wait is bounded by a clock64 budget; on timeout the CTA records an error
//    word in the workspace, skips the rest and still releases its TMEM.
#include <cooperative_groups.h>
#include <cuda.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "async.cuh"
#include "common.cuh"

namespace b2d {

namespace tc {

constexpr int BM = 128;        // W rows per tile (MMA M)
constexpr int BK = 64;         // K elements per stage (128 bytes of fp16 = one swizzle row)
constexpr int THREADS = 128;

enum { ERR_TIMEOUT_FULL = 1, ERR_TIMEOUT_EMPTY = 2, ERR_TIMEOUT_DONE = 3 };
constexpr int kMaxSplits = 8;  // K splits of a row tile = CTAs of one (portable) cluster

struct Params {
  CUtensorMap tmA;   // W      [M, K] fp16, box {64, 128}, 128B swizzle
  CUtensorMap tmA2;  // W_up   (SwiGLU only)
  CUtensorMap tmB;   // X      [batch, K] fp16, box {64, N}, 128B swizzle (the hi plane for XS=2)
  CUtensorMap tmB2;  // X lo plane [batch, K] (XS = 2 only)
  int M, K, batch;
  int k_tiles, k_splits, m_tiles;
  int epi;           // B2D_EPI_*
  void* y;
  int y_f16;
  void* y_lo;        // fp16 output as hi/lo planes: lo = fp16(v - hi) here (nullptr: hi only)
  int ldy;
  const float* aux;
  int* err;                  // error word
  // argmax
  float* logits;             // optional [batch][M] (ld = ldy)
  int* tokens;
  float* max_vals;
  int index_offset;
  unsigned long long* am_key;  // [N] running best (value, row) key per token, zero between calls
  unsigned int* am_counter;
  const uint16_t* scales;    // quantized weights: fp16 [M, K/32]
  // fp16 weights pre-packed into 16 KB tiles (tc_pack_f16), read with 1D bulk copies instead
  // of the tensor maps tmA / tmA2 (nullptr: row-major weights through the tensor maps)
  const uint8_t* pA;
  const uint8_t* pA2;
  // STORE epilogue into several fp32 copies of y (n_ys > 0, then y is unused): tensor-parallel
  // partial sums pushed straight into every rank's receive buffer over NVLink
  float* ys[8];
  int n_ys;
  // the next kernel's weights, pulled into L2 by this kernel's tail (nullptr: none)
  const void* pf;
  unsigned long long pf_bytes;
  // accumulation chains per CTA (1..kMaxChains): k-tile i accumulates into TMEM accumulator
  // i % chains, and the epilogue adds the chains in fp32 in a fixed order.  Tensor-core
  // accumulation over a long run of MMAs is measurably less exact than round-to-nearest fp32
  // adds; short chains keep each run to a few k-tiles.
  int chains;
  uint32_t tmem_cols;  // TMEM columns the CTA allocates (power of two >= 32)
  // RMSNorm folded into a residual-add producer and the GEMM that consumes its output:
  //   rmsnorm(x)[t] * gamma = r[t] * (x[t] * gamma),  r[t] = rsqrt(mean(x[t]^2) + eps)
  // so W (rmsnorm(x) * gamma) = r[t] / e[t] * (W (x * gamma * e[t])) for any power of two e[t].
  // Producer (ADD epilogue, nrm_gamma set): besides the new residual y it writes the hi / lo
  // fp16 planes of y * gamma * e[t] to nrm_planes (lo at + batch * ldy), and to nrm_part_out
  // the sum of y^2 over each 16-row slice, [32 tokens][M / 16], then e[32].  e[t] is the power
  // of two at or below the last norm factor of token t (nrm_r_prev; 1 without it), which keeps
  // the planes near unit scale.  Consumer (nrm_part_in set, fp16 weights): adds the slice sums
  // in a fixed order, scales its product by r[t] / e[t] and, with nrm_r_out, records r[t].
  const float* nrm_gamma;
  uint16_t* nrm_planes;
  float* nrm_part_out;
  const float* nrm_r_prev;
  const float* nrm_part_in;
  float* nrm_r_out;
  float nrm_eps;
};
constexpr int kMaxChains = 4;

// The power of two at or below a positive normal float (1 for anything else).
__device__ __forceinline__ float pow2_floor(float v) {
  const float e = __int_as_float(__float_as_int(v) & 0x7f800000);
  return v > 0.f && e > 0.f && e < INFINITY ? e : 1.f;
}

// Barrier among the four epilogue warps (128 threads), leaving the other warps free.
__device__ __forceinline__ void epi_bar_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Folded RMSNorm, producer: once the epilogue threads have put y^2 of their owned rows into
// sq ([token][owned row], zero for rows past M), each 16-row slice's sum per token, added in
// row order, goes to nrm_part_out[t][slice]; owned slice ls is slice gs0 + ls * gs_step of M.
// One CTA (write_e) also records e[t] after the sums.
__device__ __forceinline__ void nrm_slice_sums(const Params& p, const float* sq,
                                               const float* nrm_e, int own_rows, int gs0,
                                               int gs_step, int etid, bool write_e) {
  epi_bar_sync();
  const int nsl = own_rows / 16, S = p.M / 16;
  for (int i = etid; i < nsl * p.batch; i += THREADS) {
    const int t = i / nsl, ls = i - t * nsl;
    const int gs = gs0 + ls * gs_step;
    if (gs >= S) continue;
    const float4* src = reinterpret_cast<const float4*>(sq + t * own_rows + ls * 16);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 u = src[j];
      sum += u.x;
      sum += u.y;
      sum += u.z;
      sum += u.w;
    }
    p.nrm_part_out[(size_t)t * S + gs] = sum;
  }
  if (write_e && etid < p.batch) p.nrm_part_out[(size_t)32 * S + etid] = nrm_e[etid];
}

// y[yi] = v into y, or into every copy in p.ys
template <typename P>
__device__ __forceinline__ void store_y(const P& p, size_t yi, float v) {
  if (p.n_ys > 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < p.n_ys) p.ys[i][yi] = v;
  } else if (p.y_f16) {
    const uint16_t hi = f2h(v);
    reinterpret_cast<uint16_t*>(p.y)[yi] = hi;
    if (p.y_lo) reinterpret_cast<uint16_t*>(p.y_lo)[yi] = f2h(v - h2f(hi));
  } else {
    reinterpret_cast<float*>(p.y)[yi] = v;
  }
}

// Previous value of y[yi] (ADD epilogue): fp32, fp16, or the hi + lo fp16 planes.
template <typename P>
__device__ __forceinline__ float load_y(const P& p, size_t yi) {
  if (!p.y_f16) return reinterpret_cast<const float*>(p.y)[yi];
  float v = h2f(reinterpret_cast<const uint16_t*>(p.y)[yi]);
  if (p.y_lo) v += h2f(reinterpret_cast<const uint16_t*>(p.y_lo)[yi]);
  return v;
}

// (value, row) -> 64-bit key whose unsigned order is "larger value, then lower row": the high
// word is the float's bits made monotone, the low word is ~row.  NaN maps below -inf.
__device__ __forceinline__ unsigned long long argmax_key(float v, int row) {
  uint32_t u = __float_as_uint(v);
  u = (v != v) ? 0u : ((u & 0x80000000u) ? ~u : (u | 0x80000000u));
  return ((unsigned long long)u << 32) | (uint32_t)(~(uint32_t)row);
}
__device__ __forceinline__ int argmax_key_row(unsigned long long k) {
  return (int)(~(uint32_t)(k & 0xffffffffull));
}
__device__ __forceinline__ float argmax_key_value(unsigned long long k) {
  const uint32_t u = (uint32_t)(k >> 32);
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

// One 128 x 64 fp16 weight tile: row-major [M, K] through its tensor map (128-byte rows, one
// per weight row), or the packed tile (16 KB contiguous, already in the 128-byte-swizzled
// shared-memory image).
__device__ __forceinline__ void load_a_tile(void* dst, const CUtensorMap* tm, const uint8_t* packed,
                                            int m_tile, int k_tiles, int kt, uint64_t* bar) {
  const uint64_t pol = l2_evict_first();  // weights are read once per step
  if (packed)
    bulk_load_hint(dst, packed + ((size_t)m_tile * k_tiles + kt) * (BM * BK * 2), BM * BK * 2, bar,
                   pol);
  else
    tma_load_2d_hint(dst, tm, kt * BK, m_tile * BM, bar, pol);
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* tm) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}

// K-major operand, 128-byte swizzle: rows of 128 B, 8-row groups 1024 B apart (SBO), LBO = 1
// (unused for swizzled K-major), descriptor version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t smem_desc_sw128(const void* tile) {
  const uint64_t addr = smem_u32(tile);
  return ((addr & 0x3FFFFull) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: D fp32, A/B fp16, both K-major, M = 128, N.
template <int N>
__device__ __forceinline__ uint32_t idesc_f16() {
  return (1u << 4) | (uint32_t(N >> 3) << 17) | (uint32_t(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 lanes x N columns of fp32 from TMEM: thread = lane, N registers = N columns.
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float* v);

template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <>
__device__ __forceinline__ void tmem_ld<32>(uint32_t taddr, float* v) {
  tmem_ld<16>(taddr, v);
  tmem_ld<16>(taddr + 16, v + 16);
}

// Weight-ring depth (stages of 64 K-columns) of the fp16 kernels.  With hi/lo activation planes
// (XS = 2) a single-matrix stage is 24 KB instead of 20 KB: 3 stages keep two CTAs per SM.
#ifndef B2D_TC_STAGES
#define B2D_TC_STAGES 4
#endif
#ifndef B2D_TC_STAGES_X2
#define B2D_TC_STAGES_X2 3
#endif
#ifndef B2D_TC_STAGES_DUAL
#define B2D_TC_STAGES_DUAL 4
#endif

// QUANT: 0 = fp16 weights (TMA straight into the MMA operand), 1 = q8_32, 2 = q4_32 (TMA
// streams the raw tiles; four dequant warps expand them into the fp16 operand).
constexpr int threads_for(int quant) { return quant ? 192 : 128; }

template <int N, bool DUAL, int QUANT = 0, int XS = 1>
struct Cfg {
  static constexpr int NB = N * XS;                    // MMA N: tokens x activation planes
  static constexpr int A_BYTES = BM * BK * 2;          // 16 KB
  static constexpr int B_BYTES = NB * BK * 2;          // 2 / 4 KB per plane
  static constexpr int B_OFF = A_BYTES * (DUAL ? 2 : 1);
  // fp16 weights: one ring of STAGES x [A | (A_up) | B], filled by TMA
  static constexpr int STAGE_BYTES = B_OFF + B_BYTES;
  // non-dual: 4 stages (~100 KB) so two CTAs share an SM and one streams while the other
  // runs its prologue or epilogue; dual (gate/up, 36 KB stages): one CTA per SM
  static constexpr int STAGES =
      DUAL ? B2D_TC_STAGES_DUAL : (XS == 2 ? B2D_TC_STAGES_X2 : B2D_TC_STAGES);
  // quantized weights: a deep ring of RS raw tiles (the HBM stream) and a shallow ring of AS
  // operand stages [A fp16 | B] that the dequant warps fill
  static constexpr int RAW_ROW = QUANT == 1 ? BK : (QUANT == 2 ? BK / 2 : 0);  // bytes per row
  static constexpr int RAW_BYTES = BM * RAW_ROW;  // 8 KB (q8) / 4 KB (q4)
  static constexpr int RS = QUANT == 1 ? 12 : (QUANT == 2 ? 24 : 1);
  static constexpr int AS = 3;
  static constexpr int RAW_RING_OFF = AS * STAGE_BYTES;
  static constexpr int RING_BYTES = QUANT ? RAW_RING_OFF + RS * RAW_BYTES : STAGES * STAGE_BYTES;
  static constexpr int NACC = DUAL ? 2 : 1;
  // split-K receive buffer (not aliased with the ring: peers write into it while this CTA may
  // still be streaming): [source rank][acc][token][owned rows + pad], owned rows = BM / splits
  // split-K receive buffer: [source rank][accumulator][owned row][N + 4] (padded rows: the
  // 16-byte reads of consecutive rows fall in distinct banks); ks x (BM / ks) = BM rows in all
  static constexpr int RED_FLOATS = NACC * BM * (N + 4);
  static constexpr int SMEM = RING_BYTES + RED_FLOATS * 4 + 1024;  // + alignment slack
  static constexpr int ACC_COLS = NB * NACC;  // TMEM columns of one accumulation chain
  // CTAs of this kernel one SM holds (228 KB of shared memory per SM, ~1 KB reserved per CTA,
  // plus the kernel's static shared memory)
  static constexpr int CTAS_PER_SM = 2 * (SMEM + 4096) <= 228 * 1024 ? 2 : 1;
};

template <int N, bool DUAL, bool ARGMAX, int QUANT = 0, int XS = 1>
__global__ void __launch_bounds__(threads_for(QUANT), 1)
    tc_gemm_kernel(const __grid_constant__ Params p) {
  using C = Cfg<N, DUAL, QUANT, XS>;
  constexpr int EPI0 = QUANT ? 2 : 0;  // first epilogue warp (epilogue warps hold TMEM quarters)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[C::STAGES];
  __shared__ __align__(8) uint64_t empty_bar[C::STAGES];
  // quantized pipeline: raw ring (TMA -> dequant) and operand ring (dequant + TMA(B) -> MMA)
  __shared__ __align__(8) uint64_t raw_full[QUANT ? C::RS : 1];
  __shared__ __align__(8) uint64_t raw_empty[QUANT ? C::RS : 1];
  __shared__ __align__(8) uint64_t a_full[QUANT ? C::AS : 1];
  __shared__ __align__(8) uint64_t a_empty[QUANT ? C::AS : 1];
  __shared__ __align__(8) uint64_t done_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  __shared__ bool is_last;
  __shared__ float am_v[4][N];
  __shared__ int am_i[4][N];
  __shared__ float nrm_s[N];  // folded RMSNorm, consumer: r[t] / e[t]
  __shared__ float nrm_e[N];  // folded RMSNorm, producer: e[t]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m_tile = blockIdx.x, split = blockIdx.y;
  const int m0 = m_tile * BM;
  const int kt_begin = (int)((long long)split * p.k_tiles / p.k_splits);
  const int kt_end = (int)((long long)(split + 1) * p.k_tiles / p.k_splits);
  const int nkt = kt_end - kt_begin;

  const int first = min(nkt, C::STAGES);
  if (tid == 0) {
    if constexpr (QUANT) {
      for (int s = 0; s < C::RS; ++s) {
        mbar_init(&raw_full[s], 1);
        mbar_init(&raw_empty[s], 4);  // one arrival per dequant warp
      }
      for (int s = 0; s < C::AS; ++s) {
        mbar_init(&a_full[s], 5);  // 4 dequant warps + the producer's B copy
        mbar_init(&a_empty[s], 1);
      }
    } else {
      for (int s = 0; s < C::STAGES; ++s) {
        mbar_init(&full_bar[s], 1);
        mbar_init(&empty_bar[s], 1);
      }
    }
    mbar_init(&done_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    abort_flag = 0;
    // weight tiles do not depend on the previous kernel: start streaming them at once
    if constexpr (QUANT) {
      for (int i = 0; i < min(nkt, C::RS); ++i) {
        mbar_expect_tx(&raw_full[i], C::RAW_BYTES);
        tma_load_2d_hint(smem + C::RAW_RING_OFF + i * C::RAW_BYTES, &p.tmA,
                         (kt_begin + i) * C::RAW_ROW, m0, &raw_full[i], l2_evict_first());
      }
    } else {
      for (int i = 0; i < first; ++i) {
        uint8_t* st = smem + i * C::STAGE_BYTES;
        mbar_expect_tx(&full_bar[i], C::STAGE_BYTES);
        load_a_tile(st, &p.tmA, p.pA, m_tile, p.k_tiles, kt_begin + i, &full_bar[i]);
        if (DUAL)
          load_a_tile(st + C::A_BYTES, &p.tmA2, p.pA2, m_tile, p.k_tiles, kt_begin + i, &full_bar[i]);
      }
    }
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_slot)),
                 "r"(p.tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  const int chains = min(p.chains, max(nkt, 1));  // chains this CTA writes (each at least once)
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  // split-K clusters: announce that this CTA runs (peers write into its shared memory later)
  if (p.k_splits > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    pdl_wait();  // activations come from the previous kernel
    if constexpr (QUANT) {
      for (int i = 0; i < nkt; ++i) {
        const int as = i % C::AS;
        if (i >= C::AS &&
            !mbar_wait(&a_empty[as], ((i / C::AS) - 1) & 1, p.err, ERR_TIMEOUT_EMPTY)) {
          abort_flag = 1;
          break;
        }
        mbar_expect_tx(&a_full[as], C::B_BYTES);
        tma_load_2d(smem + as * C::STAGE_BYTES + C::B_OFF, &p.tmB, (kt_begin + i) * BK, 0,
                    &a_full[as]);
        if constexpr (XS == 2)  // lo plane: rows N..2N-1 of the B tile
          tma_load_2d(smem + as * C::STAGE_BYTES + C::B_OFF + N * BK * 2, &p.tmB2,
                      (kt_begin + i) * BK, 0, &a_full[as]);
        const int j = i + C::RS;  // raw tile that reuses the slot k-tile i is draining
        if (j < nkt) {
          const int rs = i % C::RS;
          if (!mbar_wait(&raw_empty[rs], (i / C::RS) & 1, p.err, ERR_TIMEOUT_EMPTY)) {
            abort_flag = 1;
            break;
          }
          mbar_expect_tx(&raw_full[rs], C::RAW_BYTES);
          tma_load_2d_hint(smem + C::RAW_RING_OFF + rs * C::RAW_BYTES, &p.tmA,
                           (kt_begin + j) * C::RAW_ROW, m0, &raw_full[rs], l2_evict_first());
        }
      }
    } else {
      for (int i = 0; i < first; ++i) {
        uint8_t* st = smem + i * C::STAGE_BYTES;
        tma_load_2d(st + C::B_OFF, &p.tmB, (kt_begin + i) * BK, 0, &full_bar[i]);
        if constexpr (XS == 2)
          tma_load_2d(st + C::B_OFF + N * BK * 2, &p.tmB2, (kt_begin + i) * BK, 0, &full_bar[i]);
      }
      for (int i = first; i < nkt; ++i) {
        const int s = i % C::STAGES;
        if (!mbar_wait(&empty_bar[s], ((i / C::STAGES) - 1) & 1, p.err, ERR_TIMEOUT_EMPTY)) {
          abort_flag = 1;
          break;
        }
        uint8_t* st = smem + s * C::STAGE_BYTES;
        mbar_expect_tx(&full_bar[s], C::STAGE_BYTES);
        load_a_tile(st, &p.tmA, p.pA, m_tile, p.k_tiles, kt_begin + i, &full_bar[s]);
        if (DUAL)
          load_a_tile(st + C::A_BYTES, &p.tmA2, p.pA2, m_tile, p.k_tiles, kt_begin + i, &full_bar[s]);
        tma_load_2d(st + C::B_OFF, &p.tmB, (kt_begin + i) * BK, 0, &full_bar[s]);
        if constexpr (XS == 2)
          tma_load_2d(st + C::B_OFF + N * BK * 2, &p.tmB2, (kt_begin + i) * BK, 0, &full_bar[s]);
      }
    }
    // this CTA's weights are all requested: start pulling the next kernel's into L2, so HBM
    // stays busy through this kernel's epilogue and the next one's launch
    if (!abort_flag) l2_prefetch_share(p.pf, p.pf_bytes);
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = idesc_f16<C::NB>();
    bool ok = true;
    int chain = 0;
    for (int i = 0; i < nkt; ++i) {
      const int s = QUANT ? i % C::AS : i % C::STAGES;
      const int ph = QUANT ? (i / C::AS) & 1 : (i / C::STAGES) & 1;
      uint64_t* ready = QUANT ? &a_full[s] : &full_bar[s];
      if (!mbar_wait(ready, ph, p.err, ERR_TIMEOUT_FULL)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint8_t* st = smem + s * C::STAGE_BYTES;
      const uint64_t a = smem_desc_sw128(st);
      const uint64_t b = smem_desc_sw128(st + C::B_OFF);
      const uint32_t dacc = tmem + (uint32_t)(chain * C::ACC_COLS);  // this k-tile's chain
#pragma unroll
      for (int k = 0; k < BK / 16; ++k) {  // 32 bytes of K per MMA: +2 in the 16-byte address field
        const uint32_t acc = (i >= chains || k > 0) ? 1u : 0u;
        mma_f16(dacc, a + 2 * k, b + 2 * k, idesc, acc);
        if (DUAL) {
          const uint64_t a2 = smem_desc_sw128(st + C::A_BYTES);
          mma_f16(dacc + C::NB, a2 + 2 * k, b + 2 * k, idesc, acc);
        }
      }
      chain = chain + 1 == chains ? 0 : chain + 1;
      mma_commit(QUANT ? &a_empty[s] : &empty_bar[s]);  // slot free once these MMAs read it
    }
    if (ok) mma_commit(&done_bar);
    else abort_flag = 1;
  } else if (QUANT && warp >= 2) {
    // ---------------- dequantizers: one thread per weight row of the tile ----------------
    const int dr = (warp - 2) * 32 + lane;
    const int grow = m0 + dr;
    const int nsb = p.K / 32;  // scale blocks per row
    const uint16_t* srow = p.scales + (size_t)min(grow, p.M - 1) * nsb;
    auto scale_pair = [&](int kt) -> uint32_t {  // fp16 scales of blocks 2kt, 2kt+1 (0 outside)
      if (grow >= p.M) return 0u;
      const uint32_t s0 = 2 * kt < nsb ? (uint32_t)__ldg(srow + 2 * kt) : 0u;
      const uint32_t s1 = 2 * kt + 1 < nsb ? (uint32_t)__ldg(srow + 2 * kt + 1) : 0u;
      return s0 | (s1 << 16);
    };
    // The row's scales come from HBM: fetching them one k-tile ahead put a memory latency on
    // every k-tile.  When the rows hold whole 16-byte groups (K % 256 == 0), each 16-byte load
    // brings 4 k-tiles' scales and a ring of three such loads runs 8-12 k-tiles ahead.
    const bool vec_sc = (p.K % 256) == 0 && (reinterpret_cast<uintptr_t>(p.scales) & 15) == 0;
    auto scale_group = [&](int g) -> uint4 {  // scales of k-tiles 4g .. 4g + 3
      if (grow >= p.M || 4 * g >= p.k_tiles) return make_uint4(0u, 0u, 0u, 0u);
      return __ldg(reinterpret_cast<const uint4*>(srow) + g);
    };
    int g0 = kt_begin >> 2;
    uint4 sg0 = make_uint4(0u, 0u, 0u, 0u), sg1 = sg0, sg2 = sg0;
    if (vec_sc) {
      sg0 = scale_group(g0);
      sg1 = scale_group(g0 + 1);
      sg2 = scale_group(g0 + 2);
    }
    uint32_t sc_next = vec_sc ? 0u : scale_pair(kt_begin);
    for (int i = 0; i < nkt; ++i) {
      const int rs = i % C::RS, as = i % C::AS;
      uint32_t sc;
      if (vec_sc) {
        const int kt = kt_begin + i;
        if ((kt >> 2) > g0) {  // next group: rotate the ring and fetch three groups ahead
          sg0 = sg1;
          sg1 = sg2;
          sg2 = scale_group(g0 + 3);
          ++g0;
        }
        const int w = kt & 3;
        sc = w == 0 ? sg0.x : (w == 1 ? sg0.y : (w == 2 ? sg0.z : sg0.w));
      } else {
        sc = sc_next;
        if (i + 1 < nkt) sc_next = scale_pair(kt_begin + i + 1);
      }
      if (!mbar_wait(&raw_full[rs], (i / C::RS) & 1, p.err, ERR_TIMEOUT_FULL) ||
          (i >= C::AS &&
           !mbar_wait(&a_empty[as], ((i / C::AS) - 1) & 1, p.err, ERR_TIMEOUT_EMPTY))) {
        abort_flag = 1;
        break;
      }
      const uint8_t* raw = smem + C::RAW_RING_OFF + rs * C::RAW_BYTES + dr * C::RAW_ROW;
      uint8_t* arow = smem + as * C::STAGE_BYTES + (dr >> 3) * 1024 + (dr & 7) * 128;  // SW128
      const __half2 s_lo = __half2half2(__ushort_as_half((uint16_t)(sc & 0xFFFF)));
      const __half2 s_hi = __half2half2(__ushort_as_half((uint16_t)(sc >> 16)));
      if (QUANT == 1) {
        const __half2 bias = __float2half2_rn(1152.0f);  // 1024 + 128
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {  // 16-byte raw chunks, rotated by row (bank spread)
          const int c = (cc + dr) & 3;
          const uint4 w = *reinterpret_cast<const uint4*>(raw + c * 16);
          const __half2 sc2 = c < 2 ? s_lo : s_hi;
          const uint32_t wv[4] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u, w.z ^ 0x80808080u,
                                  w.w ^ 0x80808080u};
          uint32_t out[8];
#pragma unroll
          for (int j = 0; j < 4; ++j) {  // byte b -> fp16 (1024 + b) - 1152 = q, then * scale
            uint32_t lo = __byte_perm(wv[j], 0x64646464u, 0x4140);
            uint32_t hi = __byte_perm(wv[j], 0x64646464u, 0x4342);
            __half2 hl = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&lo), bias), sc2);
            __half2 hh = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&hi), bias), sc2);
            out[2 * j] = *reinterpret_cast<uint32_t*>(&hl);
            out[2 * j + 1] = *reinterpret_cast<uint32_t*>(&hh);
          }
          const int o0 = 2 * c, o1 = 2 * c + 1;  // output 8-element chunks
          *reinterpret_cast<uint4*>(arow + ((o0 ^ (dr & 7)) << 4)) =
              make_uint4(out[0], out[1], out[2], out[3]);
          *reinterpret_cast<uint4*>(arow + ((o1 ^ (dr & 7)) << 4)) =
              make_uint4(out[4], out[5], out[6], out[7]);
        }
      } else {
        const __half2 bias = __float2half2_rn(1032.0f);  // 1024 + 8
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {  // 16-byte raw chunks = 32 nibbles = one scale block
          const int c = (cc + dr) & 1;
          const uint4 w = *reinterpret_cast<const uint4*>(raw + c * 16);
          const __half2 sc2 = c == 0 ? s_lo : s_hi;
          const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
          uint32_t out[16];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t lo = (wv[j] & 0x0F0F0F0Fu) ^ 0x08080808u;        // even elements
            const uint32_t hi = ((wv[j] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;  // odd elements
            const uint32_t e03 = __byte_perm(lo, hi, 0x5140);  // bytes e0 e1 e2 e3
            const uint32_t e47 = __byte_perm(lo, hi, 0x7362);  // bytes e4 e5 e6 e7
            uint32_t p0 = __byte_perm(e03, 0x64646464u, 0x4140);
            uint32_t p1 = __byte_perm(e03, 0x64646464u, 0x4342);
            uint32_t p2 = __byte_perm(e47, 0x64646464u, 0x4140);
            uint32_t p3 = __byte_perm(e47, 0x64646464u, 0x4342);
            __half2 h0 = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&p0), bias), sc2);
            __half2 h1 = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&p1), bias), sc2);
            __half2 h2 = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&p2), bias), sc2);
            __half2 h3 = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&p3), bias), sc2);
            out[4 * j] = *reinterpret_cast<uint32_t*>(&h0);
            out[4 * j + 1] = *reinterpret_cast<uint32_t*>(&h1);
            out[4 * j + 2] = *reinterpret_cast<uint32_t*>(&h2);
            out[4 * j + 3] = *reinterpret_cast<uint32_t*>(&h3);
          }
#pragma unroll
          for (int o = 0; o < 4; ++o) {
            const int oc = 4 * c + o;
            *reinterpret_cast<uint4*>(arow + ((oc ^ (dr & 7)) << 4)) =
                make_uint4(out[4 * o], out[4 * o + 1], out[4 * o + 2], out[4 * o + 3]);
          }
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to tcgen05.mma
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&a_full[as]);
        mbar_arrive(&raw_empty[rs]);
      }
    }
  } else if (!QUANT && (warp == 2 || warp == 3) && p.nrm_part_in) {
    // ---------------- folded RMSNorm: the per-token factor, during the main loop ----------------
    // Two threads per token each add half of the producer's slice sums (four interleaved fp32
    // sums, combined in a fixed order), then r = rsqrt(sum / K + eps).
    pdl_wait();  // the slice sums come from the previous kernel
    const int q = tid - 64, t = q >> 1, half = q & 1;
    const int S = p.K / 16;
    float ssum = 0.f;
    if (t < p.batch) {
      const float4* src =
          reinterpret_cast<const float4*>(p.nrm_part_in + (size_t)t * S) + half * (S / 8);
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll 8
      for (int i = 0; i < S / 8; ++i) {
        const float4 u = src[i];
        a0 += u.x;
        a1 += u.y;
        a2 += u.z;
        a3 += u.w;
      }
      ssum = (a0 + a1) + (a2 + a3);
    }
    ssum += __shfl_xor_sync(0xffffffffu, ssum, 1);  // both halves: the same sum
    if (half == 0 && t < N) {
      float sc = 1.f;
      if (t < p.batch) {
        const float rn = rsqrtf(ssum / (float)p.K + p.nrm_eps);
        sc = rn / p.nrm_part_in[(size_t)32 * S + t];
        if (p.nrm_r_out && m_tile == 0 && split == 0) p.nrm_r_out[t] = rn;
      }
      nrm_s[t] = sc;
    }
  }
  __syncwarp();

  // ---------------- epilogue (all 4 warps) ----------------
  // CTA-uniform: tcgen05.ld below is warp-collective
  const bool have =
      __syncthreads_and(mbar_wait(&done_bar, 0, p.err, ERR_TIMEOUT_DONE) ? 1 : 0) != 0 && nkt > 0;
  tc_fence_after();
  float acc[N], acc2[DUAL ? N : 1];
  const bool epi_warp = warp >= EPI0 && warp < EPI0 + 4;
  if (have && epi_warp) {
    // sum of the chains (and of the hi / lo plane columns of each token), in a fixed order
    const uint32_t taddr = tmem + (uint32_t((warp & 3) * 32) << 16);
    tmem_ld<N>(taddr, acc);
    if (DUAL) tmem_ld<N>(taddr + C::NB, acc2);
    float part[N];
    for (int ch = 0; ch < chains; ++ch) {
      const uint32_t ca = taddr + (uint32_t)(ch * C::ACC_COLS);
#pragma unroll
      for (int pl = 0; pl < XS; ++pl) {
        if (ch == 0 && pl == 0) continue;  // loaded above
        tmem_ld<N>(ca + pl * N, part);
#pragma unroll
        for (int t = 0; t < N; ++t) acc[t] += part[t];
        if constexpr (DUAL) {
          tmem_ld<N>(ca + C::NB + pl * N, part);
#pragma unroll
          for (int t = 0; t < N; ++t) acc2[t] += part[t];
        }
      }
    }
    if (!QUANT && p.nrm_part_in) {  // folded RMSNorm: the product times r[t] / e[t]
#pragma unroll
      for (int t = 0; t < N; ++t) {
        acc[t] *= nrm_s[t];
        if constexpr (DUAL) acc2[t] *= nrm_s[t];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(p.tmem_cols));
  }
  const bool ok = have && !abort_flag;  // CTA-uniform
  const int r = (warp & 3) * 32 + lane;       // row within the tile (epilogue warps)
  const int etid = (warp - EPI0) * 32 + lane;  // 0..127 on epilogue warps
  const int row = m0 + r;
  // folded RMSNorm, producer side (ADD epilogue): CTA-uniform; y^2 per (token, owned row) is
  // staged in the operand ring, idle once the accumulator is complete
  constexpr bool EMIT = !DUAL && !ARGMAX;
  const bool emit = EMIT && p.nrm_gamma != nullptr && p.epi == B2D_EPI_ADD;
  float* sq = reinterpret_cast<float*>(smem);

  if (p.k_splits > 1) {
    // Split-K through the thread-block cluster: the k_splits CTAs of this row tile form one
    // cluster.  Rows are owned in 16-row slices (slice s by rank s % k_splits).  Each CTA
    // stores its partial rows straight into the owners' receive buffers (distributed shared
    // memory), one cluster barrier publishes them, and every owner sums its rows over the
    // sources in rank order (deterministic) from local shared memory, then runs the epilogue.
    // No CTA touches a peer's memory after the barrier, so one barrier suffices.
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    const int ks = p.k_splits;
    const int rank = (int)cl.block_rank();
    const int own_rows = BM / ks;
    constexpr int NP = N + 4;  // padded row of the receive buffer (floats)
    float* red = reinterpret_cast<float*>(smem + C::RING_BYTES);
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // every peer has started
    if (ok && epi_warp) {
      // this thread's row of partial sums (N tokens) goes to its owner as N/4 16-byte stores
      const int sl = r / 16, owner = sl % ks;
      const int lr = (sl / ks) * 16 + (r % 16);
      float* dst = cl.map_shared_rank(red, owner);
      float4* d0 = reinterpret_cast<float4*>(dst + ((rank * C::NACC + 0) * own_rows + lr) * NP);
#pragma unroll
      for (int t = 0; t < N; t += 4) d0[t / 4] = make_float4(acc[t], acc[t + 1], acc[t + 2], acc[t + 3]);
      if constexpr (DUAL) {
        float4* d1 = reinterpret_cast<float4*>(dst + ((rank * C::NACC + 1) * own_rows + lr) * NP);
#pragma unroll
        for (int t = 0; t < N; t += 4)
          d1[t / 4] = make_float4(acc2[t], acc2[t + 1], acc2[t + 2], acc2[t + 3]);
      }
    }
    // each owner thread then finishes items of (one owned row, 4 consecutive tokens); prefetch
    // what those items read from global memory while the barrier completes
    constexpr int MAXQ = N / 8;  // items per thread (k_splits >= 2)
    float yv[DUAL ? 1 : MAXQ][4];
    float gv[EMIT ? MAXQ : 1];  // folded RMSNorm: gamma of each item's row
    pdl_wait();
    pdl_launch_dependents();
    const int nq = own_rows * (N / 4);
    if (!DUAL && ok && epi_warp &&
        (p.epi == B2D_EPI_ADD || p.epi == B2D_EPI_GELU_MUL || p.epi == B2D_EPI_SILU_MUL)) {
#pragma unroll
      for (int k = 0; k < MAXQ; ++k) {
        const int v = etid + k * THREADS;
        const int lr = v % own_rows, t0 = 4 * (v / own_rows);
        const int grow = m0 + ((lr / 16) * ks + rank) * 16 + (lr % 16);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          yv[k][j] = 0.f;
          if (v < nq && t0 + j < p.batch && grow < p.M) {
            const size_t yi = (size_t)(t0 + j) * p.ldy + grow;
            yv[k][j] = p.epi == B2D_EPI_ADD ? load_y(p, yi) : p.aux[yi];
          }
        }
        if constexpr (EMIT) gv[k] = emit && v < nq && grow < p.M ? p.nrm_gamma[grow] : 0.f;
      }
    }
    if (emit && ok && epi_warp && etid < N)
      nrm_e[etid] = etid < p.batch && p.nrm_r_prev ? pow2_floor(p.nrm_r_prev[etid]) : 1.f;
    cl.sync();  // every partial row has reached its owner (and nrm_e is visible)
    if (ok && epi_warp) {
#pragma unroll
      for (int k = 0; k < MAXQ; ++k) {
        const int v = etid + k * THREADS;
        if (v >= nq) break;
        const int lr = v % own_rows, t0 = 4 * (v / own_rows);
        const int grow = m0 + ((lr / 16) * ks + rank) * 16 + (lr % 16);
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f), a2 = a;
        for (int q = 0; q < ks; ++q) {  // fixed source order: deterministic sums
          const float4 u = *reinterpret_cast<const float4*>(red + ((q * C::NACC + 0) * own_rows + lr) * NP + t0);
          a.x += u.x;
          a.y += u.y;
          a.z += u.z;
          a.w += u.w;
          if constexpr (DUAL) {
            const float4 u2 = *reinterpret_cast<const float4*>(red + ((q * C::NACC + 1) * own_rows + lr) * NP + t0);
            a2.x += u2.x;
            a2.y += u2.y;
            a2.z += u2.z;
            a2.w += u2.w;
          }
        }
        if (grow >= p.M) {
          if (emit) {  // rows past M add nothing to their slice's sum
#pragma unroll
            for (int j = 0; j < 4; ++j) sq[(t0 + j) * own_rows + lr] = 0.f;
          }
          continue;
        }
        const float av[4] = {a.x, a.y, a.z, a.w}, a2v[4] = {a2.x, a2.y, a2.z, a2.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int t = t0 + j;
          if (t >= p.batch) break;
          const size_t yi = (size_t)t * p.ldy + grow;
          float y;
          if constexpr (DUAL) {
            y = silu(av[j]) * a2v[j];
          } else {
            y = av[j];
            if (p.epi == B2D_EPI_ADD) y += yv[k][j];
            else if (p.epi == B2D_EPI_GELU_MUL) y = gelu_tanh(y) * yv[k][j];
            else if (p.epi == B2D_EPI_SILU_MUL) y = silu(y) * yv[k][j];
          }
          store_y(p, yi, y);
          if constexpr (EMIT) {
            if (emit) {
              store_f16_split(p.nrm_planes, p.nrm_planes + (size_t)p.batch * p.ldy, yi,
                              y * gv[k] * nrm_e[t]);
              sq[t * own_rows + lr] = y * y;
            }
          }
        }
      }
      if (emit)
        nrm_slice_sums(p, sq, nrm_e, own_rows, m_tile * (BM / 16) + rank, ks, etid,
                       m_tile == 0 && rank == 0);
    }
    return;
  }

  if (!ok || !epi_warp) return;
  pdl_wait();  // epilogue reads / writes buffers the previous kernel may touch
  pdl_launch_dependents();

  if constexpr (ARGMAX) {
    // logits (optional), then per-token (max, row) over this tile
#pragma unroll
    for (int t = 0; t < N; ++t) {
      float v = (row < p.M && t < p.batch) ? acc[t] : -INFINITY;
      int idx = row < p.M ? row : 0x7fffffff;
      if (p.logits && row < p.M && t < p.batch) p.logits[(size_t)t * p.ldy + row] = acc[t];
      warp_argmax(v, idx);
      if (lane == 0) {
        am_v[warp][t] = v;
        am_i[warp][t] = idx;
      }
    }
    __syncthreads();
    // the tile's winner per token joins the grid-wide maximum of (value, -row) keys: one 64-bit
    // atomicMax per token and tile, order-independent (deterministic), no serial merge at the end
    if (tid < N && tid < p.batch) {
      float bv = am_v[0][tid];
      int bi = am_i[0][tid];
      for (int w = 1; w < 4; ++w)
        if (better(am_v[w][tid], am_i[w][tid], bv, bi)) {
          bv = am_v[w][tid];
          bi = am_i[w][tid];
        }
      if (bi != 0x7fffffff) atomicMax(p.am_key + tid, argmax_key(bv, bi));
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = atomicAdd(p.am_counter, 1u) == (unsigned)(gridDim.x * gridDim.y - 1);
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    if (tid < p.batch) {
      const unsigned long long key = atomicExch(p.am_key + tid, 0ull);  // read, and reset
      p.tokens[tid] = argmax_key_row(key) + p.index_offset;
      if (p.max_vals) p.max_vals[tid] = argmax_key_value(key);
    }
    if (tid == 0) *p.am_counter = 0u;
  } else {
    if constexpr (EMIT) {
      if (emit) {
        if (etid < N)
          nrm_e[etid] = etid < p.batch && p.nrm_r_prev ? pow2_floor(p.nrm_r_prev[etid]) : 1.f;
        epi_bar_sync();
        const float g = row < p.M ? p.nrm_gamma[row] : 0.f;
#pragma unroll
        for (int t = 0; t < N; ++t) {
          if (t >= p.batch) break;
          float sqv = 0.f;
          if (row < p.M) {
            const size_t yi = (size_t)t * p.ldy + row;
            const float v = acc[t] + load_y(p, yi);
            store_y(p, yi, v);
            store_f16_split(p.nrm_planes, p.nrm_planes + (size_t)p.batch * p.ldy, yi,
                            v * g * nrm_e[t]);
            sqv = v * v;
          }
          sq[t * BM + r] = sqv;
        }
        nrm_slice_sums(p, sq, nrm_e, BM, m_tile * (BM / 16), 1, etid, m_tile == 0);
        return;
      }
    }
    if (row >= p.M) return;
#pragma unroll
    for (int t = 0; t < N; ++t) {
      if (t >= p.batch) break;
      const size_t yi = (size_t)t * p.ldy + row;
      float v;
      if (DUAL) {
        v = silu(acc[t]) * acc2[t];
      } else {
        v = acc[t];
        if (p.epi == B2D_EPI_ADD)
          v += load_y(p, yi);
        else if (p.epi == B2D_EPI_GELU_MUL)
          v = gelu_tanh(v) * p.aux[yi];
        else if (p.epi == B2D_EPI_SILU_MUL)
          v = silu(v) * p.aux[yi];
      }
      store_y(p, yi, v);
    }
  }
}

}  // namespace tc

// ------------------------------------------------------------------------------------------
// host
// ------------------------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2D fp16 tensor [rows, cols] with row stride ld (elements), box {64, box_rows}, 128B swizzle.
int make_tmap_f16(CUtensorMap* m, const void* base, uint64_t rows, int cols, int ld,
                  int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return B2D_ERR_CUDA;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)tc::BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B2D_OK : B2D_ERR_ALIGN;
}

// 2D uint8 tensor [rows, cols] (bytes), box {box_cols, box_rows}, no swizzle: the raw tiles of
// quantized weights, which the dequant warps read with plain shared-memory loads.
static int make_tmap_u8(CUtensorMap* m, const void* base, uint64_t rows, int cols, int box_cols,
                        int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return B2D_ERR_CUDA;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B2D_OK : B2D_ERR_ALIGN;
}

constexpr int kMaxTiles = 4096;  // row tiles per call: M <= 4096 * 128

struct TcPlan {
  int n_tile, m_tiles, k_tiles, k_splits, nacc;
  size_t off_key, total;
};

static TcPlan tc_plan(int M, int K, int batch, int epilogue) {
  TcPlan pl{};
  pl.n_tile = batch <= 16 ? 16 : 32;
  pl.m_tiles = (M + tc::BM - 1) / tc::BM;
  pl.k_tiles = (K + tc::BK - 1) / tc::BK;
  pl.nacc = epilogue == B2D_EPI_SWIGLU ? 2 : 1;
  pl.k_splits = 1;  // chosen at launch (tc_pick_splits): it depends on cluster residency
  auto a256 = [](size_t n) { return (n + 255) / 256 * 256; };
  // [0] error word, [64] argmax arrival counter, [256, 512) argmax keys (one u64 per token)
  size_t o = 256;
  pl.off_key = o;
  if (epilogue == B2D_EPI_ARGMAX) o += a256((size_t)32 * 8);
  pl.total = o;
  return pl;
}

size_t tc_gemm_workspace_bytes(int M, int K, int batch, int epilogue) {
  if (M <= 0 || K <= 0 || batch <= 0 || batch > 32 || M > kMaxTiles * tc::BM) return 0;
  return tc_plan(M, K, batch, epilogue).total;
}

template <int N, bool DUAL, bool ARGMAX, int QUANT = 0, int XS = 1>
static int launch_tc(const tc::Params& prm, dim3 grid, cudaStream_t stream) {
  using C = tc::Cfg<N, DUAL, QUANT, XS>;
  auto kern = tc::tc_gemm_kernel<N, DUAL, ARGMAX, QUANT, XS>;
  static int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) {
      set_cuda_error(e);
      return B2D_ERR_CUDA;
    }
    configured_dev = dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(tc::threads_for(QUANT));
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int na = 1;
  if (grid.y > 1) {  // the K splits of a row tile run as one thread-block cluster
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = grid.y;
    attr[1].val.clusterDim.z = 1;
    na = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, prm);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return B2D_ERR_CUDA;
  }
  count_launch();
  return B2D_OK;
}

// K splits (= cluster size) for a row-tile count: the largest power of two <= 8 whose clusters
// all fit on the GPU in one wave (cudaOccupancyMaxActiveClusters for this kernel), without
// more CTAs than SMs and without splitting K below one 64-wide tile.
template <int N, bool DUAL, int QUANT = 0, int XS = 1>
static int tc_pick_splits(int m_tiles, int k_tiles) {
  // The largest power-of-two split (<= 8, the portable cluster size) whose CTAs all fit on the
  // SMs at once: two per SM for the single-matrix fp16 kernel (about 100 KB of shared memory;
  // QKV 6.9 -> 6.3 us with 8-way splits), one for the others.  An earlier rule that
  // also asked cudaOccupancyMaxActiveClusters for a full wave of clusters picked 4-way splits
  // for the down and O projections (64 CTAs on 148 SMs): 14.6 -> 10.3 us and 7.5 -> 6.1 us
  // measured on B200 with the split that fills the SMs.
#ifndef B2D_TC_SPLIT_CTAS_PER_SM
#define B2D_TC_SPLIT_CTAS_PER_SM 2
#endif
  using C = tc::Cfg<N, DUAL, QUANT, XS>;
  const int per_sm = !DUAL && !QUANT ? std::min(B2D_TC_SPLIT_CTAS_PER_SM, C::CTAS_PER_SM) : 1;
  const int slots = per_sm * num_sms();
  // B2D_TC_MAX_SPLITS caps the split count (a tuning knob, read once; default 8)
  static const int max_ks = [] {
    const char* e = std::getenv("B2D_TC_MAX_SPLITS");
    const int v = e ? std::atoi(e) : tc::kMaxSplits;
    return v >= 1 && v <= tc::kMaxSplits ? v : tc::kMaxSplits;
  }();
  for (int ks = max_ks; ks >= 2; ks >>= 1)
    if (ks <= k_tiles && m_tiles * ks <= slots) return ks;
  return 1;
}

// A prepared call: tensor maps encoded once, reusable (and graph-capturable) while the
// pointers stay the same.
struct TcCall {
  tc::Params prm;
  dim3 grid;
  int n_tile;
  bool dual, argmax;
  int quant = 0;  // 0 fp16, 1 q8_32, 2 q4_32
  int xs = 1;     // activation planes: 1 fp16, 2 hi + lo fp16
};

// Accumulation chains and the TMEM allocation for a call: one chain per 8 k-tiles of a CTA's
// K range (at most kMaxChains), within the TMEM its co-resident CTAs leave (512 columns per SM).
// B2D_TC_CHAIN_KTILES overrides the 8 (a tuning knob, read once).
static void pick_chains(tc::Params& p, int acc_cols, int ctas_per_sm) {
  static const int ktiles_per_chain = [] {
    const char* e = std::getenv("B2D_TC_CHAIN_KTILES");
    const int v = e ? std::atoi(e) : 8;
    return v > 0 ? v : 8;
  }();
  const int nkt = (p.k_tiles + p.k_splits - 1) / p.k_splits;
  int c = std::min(tc::kMaxChains, std::max(1, (nkt + ktiles_per_chain - 1) / ktiles_per_chain));
  auto cols = [&](int ch) {
    uint32_t n = 32;
    while (n < (uint32_t)(ch * acc_cols)) n <<= 1;
    return n;
  };
  while (c > 1 && cols(c) * ctas_per_sm > 512) --c;
  p.chains = c;
  p.tmem_cols = cols(c);
}

template <int N, bool DUAL, int QUANT, int XS>
static void pick_chains_t(tc::Params& p) {
  using C = tc::Cfg<N, DUAL, QUANT, XS>;
  pick_chains(p, C::ACC_COLS, C::CTAS_PER_SM);
}

static void pick_chains_for(tc::Params& p, int n_tile, bool dual, int quant, int xs) {
#define B2D_CH(NT, DU, QU, X)                                 \
  if (n_tile == NT && dual == DU && quant == QU && xs == X) { \
    pick_chains_t<NT, DU, QU, X>(p);                          \
    return;                                                   \
  }
#define B2D_CH_Q(NT, DU, X) B2D_CH(NT, DU, 0, X) B2D_CH(NT, DU, 1, X) B2D_CH(NT, DU, 2, X)
  B2D_CH_Q(16, false, 1)
  B2D_CH_Q(16, false, 2)
  B2D_CH_Q(32, false, 1)
  B2D_CH_Q(32, false, 2)
  B2D_CH(16, true, 0, 1)
  B2D_CH(16, true, 0, 2)
  B2D_CH(32, true, 0, 1)
  B2D_CH(32, true, 0, 2)
#undef B2D_CH_Q
#undef B2D_CH
  p.chains = 1;
  p.tmem_cols = 128;
}

// Split count for a call's kernel variant.
static int pick_splits(int n_tile, bool dual, int quant, int xs, int m_tiles, int k_tiles) {
#define B2D_PICK(NT, DU, QU, X)                          \
  if (n_tile == NT && dual == DU && quant == QU && xs == X) \
    return tc_pick_splits<NT, DU, QU, X>(m_tiles, k_tiles);
#define B2D_PICK_Q(NT, DU, X) B2D_PICK(NT, DU, 0, X) B2D_PICK(NT, DU, 1, X) B2D_PICK(NT, DU, 2, X)
  B2D_PICK_Q(16, false, 1)
  B2D_PICK_Q(16, false, 2)
  B2D_PICK_Q(32, false, 1)
  B2D_PICK_Q(32, false, 2)
  B2D_PICK(16, true, 0, 1)
  B2D_PICK(16, true, 0, 2)
  B2D_PICK(32, true, 0, 1)
  B2D_PICK(32, true, 0, 2)
#undef B2D_PICK_Q
#undef B2D_PICK
  return 1;
}

// x_dtype B2D_F16 (X fp16 [batch, ldx]) or B2D_F16X2 (hi plane X, lo plane X + batch * ldx);
// y_dtype B2D_F32, B2D_F16 or B2D_F16X2 (lo plane y + batch * ldy).
int tc_gemm_prepare(TcCall* call, int x_dtype, const uint16_t* W, const uint16_t* W_up,
                    const uint16_t* X, int ldx, int epilogue, int y_dtype, void* y, int ldy,
                    const float* aux, int M, int K, int batch, float* logits, int* tokens,
                    float* max_vals, int index_offset, void* workspace, size_t workspace_bytes,
                    bool packed = false, float* const* ys = nullptr, int n_ys = 0) {
  if (!call || !W || !X) return B2D_ERR_NULL;
  if (x_dtype != B2D_F16 && x_dtype != B2D_F16X2) return B2D_ERR_UNSUPPORTED;
  if (M <= 0 || K <= 0 || batch <= 0 || batch > 32 || K % 8 || ldx < K || ldx % 8 ||
      M > kMaxTiles * tc::BM)
    return B2D_ERR_SHAPE;
  if (epilogue < B2D_EPI_STORE || epilogue > B2D_EPI_SILU_MUL) return B2D_ERR_UNSUPPORTED;
  if (y_dtype != B2D_F32 && y_dtype != B2D_F16 && y_dtype != B2D_F16X2) return B2D_ERR_UNSUPPORTED;
  if (epilogue == B2D_EPI_SWIGLU && !W_up) return B2D_ERR_NULL;
  if ((epilogue == B2D_EPI_GELU_MUL || epilogue == B2D_EPI_SILU_MUL) && !aux) return B2D_ERR_NULL;
  if (epilogue == B2D_EPI_ARGMAX && !tokens) return B2D_ERR_NULL;
  if (epilogue != B2D_EPI_ARGMAX && !y && n_ys == 0) return B2D_ERR_NULL;
  if (n_ys < 0 || n_ys > 8 || (n_ys > 0 && (!ys || epilogue != B2D_EPI_STORE || y_dtype != B2D_F32)))
    return B2D_ERR_UNSUPPORTED;
  if (epilogue != B2D_EPI_ARGMAX && ldy < M) return B2D_ERR_SHAPE;
  if (!aligned16(W) || !aligned16(X) || (W_up && !aligned16(W_up))) return B2D_ERR_ALIGN;
  const TcPlan pl = tc_plan(M, K, batch, epilogue);
  if (!workspace || workspace_bytes < pl.total) return B2D_ERR_WORKSPACE;
  if (!aligned16(workspace)) return B2D_ERR_ALIGN;
  tc::Params& p = call->prm;
  p = tc::Params{};
  if (packed) {
    p.pA = reinterpret_cast<const uint8_t*>(W);
    p.pA2 = reinterpret_cast<const uint8_t*>(W_up);
  } else {
    B2D_TRY(make_tmap_f16(&p.tmA, W, M, K, K, tc::BM));
    if (W_up) B2D_TRY(make_tmap_f16(&p.tmA2, W_up, M, K, K, tc::BM));
  }
  const int xs = x_dtype == B2D_F16X2 ? 2 : 1;
  B2D_TRY(make_tmap_f16(&p.tmB, X, batch, K, ldx, pl.n_tile));
  if (xs == 2) B2D_TRY(make_tmap_f16(&p.tmB2, X + (size_t)batch * ldx, batch, K, ldx, pl.n_tile));
  char* ws = static_cast<char*>(workspace);
  p.M = M;
  p.K = K;
  p.batch = batch;
  p.k_tiles = pl.k_tiles;
  p.k_splits = pl.k_splits;
  p.m_tiles = pl.m_tiles;
  p.epi = epilogue;
  p.y = y;
  p.y_f16 = y_dtype != B2D_F32;
  p.y_lo = (y_dtype == B2D_F16X2 && y) ? static_cast<uint16_t*>(y) + (size_t)batch * ldy : nullptr;
  p.ldy = epilogue == B2D_EPI_ARGMAX ? M : ldy;
  p.aux = aux;
  p.err = reinterpret_cast<int*>(ws);
  p.am_counter = reinterpret_cast<unsigned int*>(ws + 64);
  p.logits = logits;
  p.tokens = tokens;
  p.max_vals = max_vals;
  p.index_offset = index_offset;
  p.am_key = reinterpret_cast<unsigned long long*>(ws + pl.off_key);
  p.n_ys = n_ys;
  for (int i = 0; i < n_ys; ++i) {
    if (!ys[i]) return B2D_ERR_NULL;
    p.ys[i] = ys[i];
  }
  if (epilogue != B2D_EPI_ARGMAX)
    p.k_splits = pick_splits(pl.n_tile, epilogue == B2D_EPI_SWIGLU, 0, xs, pl.m_tiles, pl.k_tiles);
  pick_chains_for(p, pl.n_tile, epilogue == B2D_EPI_SWIGLU, 0, xs);
  call->grid = dim3(pl.m_tiles, p.k_splits);
  call->n_tile = pl.n_tile;
  call->dual = epilogue == B2D_EPI_SWIGLU;
  call->argmax = epilogue == B2D_EPI_ARGMAX;
  call->quant = 0;
  call->xs = xs;
  return B2D_OK;
}

template <int XS>
static int tc_gemm_launch_xs(const TcCall& c, cudaStream_t stream) {
  if (c.quant == 1)
    return c.n_tile == 16 ? launch_tc<16, false, false, 1, XS>(c.prm, c.grid, stream)
                          : launch_tc<32, false, false, 1, XS>(c.prm, c.grid, stream);
  if (c.quant == 2)
    return c.n_tile == 16 ? launch_tc<16, false, false, 2, XS>(c.prm, c.grid, stream)
                          : launch_tc<32, false, false, 2, XS>(c.prm, c.grid, stream);
  if (c.n_tile == 16) {
    if (c.argmax) return launch_tc<16, false, true, 0, XS>(c.prm, c.grid, stream);
    if (c.dual) return launch_tc<16, true, false, 0, XS>(c.prm, c.grid, stream);
    return launch_tc<16, false, false, 0, XS>(c.prm, c.grid, stream);
  }
  if (c.argmax) return launch_tc<32, false, true, 0, XS>(c.prm, c.grid, stream);
  if (c.dual) return launch_tc<32, true, false, 0, XS>(c.prm, c.grid, stream);
  return launch_tc<32, false, false, 0, XS>(c.prm, c.grid, stream);
}

int tc_gemm_launch(const TcCall& c, cudaStream_t stream) {
  return c.xs == 2 ? tc_gemm_launch_xs<2>(c, stream) : tc_gemm_launch_xs<1>(c, stream);
}

int tc_gemm(int x_dtype, const uint16_t* W, const uint16_t* W_up, const uint16_t* X, int ldx,
            int epilogue, int y_dtype, void* y, int ldy, const float* aux, int M, int K,
            int batch, float* logits, int* tokens, float* max_vals, int index_offset,
            void* workspace, size_t workspace_bytes, cudaStream_t stream,
            const void* pf = nullptr, size_t pf_bytes = 0) {
  TcCall c;
  B2D_TRY(tc_gemm_prepare(&c, x_dtype, W, W_up, X, ldx, epilogue, y_dtype, y, ldy, aux, M, K,
                          batch, logits, tokens, max_vals, index_offset, workspace,
                          workspace_bytes));
  c.prm.pf = pf;
  c.prm.pf_bytes = pf_bytes;
  return tc_gemm_launch(c, stream);
}

// tc_gemm with the RMSNorm of its input and / or of its output folded in (TcNorm).  fp16 weights
// only.  Producer: ADD epilogue into fp32 y, M % 16 == 0.  Consumer: K % 128 == 0, part_in
// 16-byte aligned.
int tc_gemm_norm(int x_dtype, const uint16_t* W, const uint16_t* W_up, const uint16_t* X,
                 int ldx, int epilogue, int y_dtype, void* y, int ldy, const float* aux, int M,
                 int K, int batch, float* logits, int* tokens, void* workspace,
                 size_t workspace_bytes, cudaStream_t stream, const void* pf, size_t pf_bytes,
                 const TcNorm& nrm) {
  if (nrm.gamma) {
    if (!nrm.planes || !nrm.part_out) return B2D_ERR_NULL;
    if (epilogue != B2D_EPI_ADD || y_dtype != B2D_F32) return B2D_ERR_UNSUPPORTED;
    if (M % 16) return B2D_ERR_SHAPE;
  }
  if (nrm.part_in) {
    if (K % 128) return B2D_ERR_SHAPE;
    if (!aligned16(nrm.part_in)) return B2D_ERR_ALIGN;
  }
  TcCall c;
  B2D_TRY(tc_gemm_prepare(&c, x_dtype, W, W_up, X, ldx, epilogue, y_dtype, y, ldy, aux, M, K,
                          batch, logits, tokens, nullptr, 0, workspace, workspace_bytes));
  tc::Params& p = c.prm;
  p.pf = pf;
  p.pf_bytes = pf_bytes;
  p.nrm_gamma = nrm.gamma;
  p.nrm_planes = nrm.planes;
  p.nrm_part_out = nrm.part_out;
  p.nrm_r_prev = nrm.r_prev;
  p.nrm_part_in = nrm.part_in;
  p.nrm_r_out = nrm.r_out;
  p.nrm_eps = nrm.eps;
  return tc_gemm_launch(c, stream);
}

// STORE of the fp32 product into n_ys copies (row stride ldy each), e.g. every tensor-parallel
// rank's receive buffer.
int tc_gemm_multi_store(int x_dtype, const uint16_t* W, const uint16_t* X, int ldx,
                        float* const* ys, int n_ys, int ldy, int M, int K, int batch,
                        void* workspace, size_t workspace_bytes, cudaStream_t stream,
                        const void* pf = nullptr, size_t pf_bytes = 0) {
  TcCall c;
  B2D_TRY(tc_gemm_prepare(&c, x_dtype, W, nullptr, X, ldx, B2D_EPI_STORE, B2D_F32, nullptr, ldy,
                          nullptr, M, K, batch, nullptr, nullptr, nullptr, 0, workspace,
                          workspace_bytes, false, ys, n_ys));
  c.prm.pf = pf;
  c.prm.pf_bytes = pf_bytes;
  return tc_gemm_launch(c, stream);
}

// Same product with the weights in the packed tile layout (tc_pack_f16).
int tc_gemm_packed(const uint8_t* Wp, const uint8_t* Wp_up, const uint16_t* X, int ldx,
                   int epilogue, int y_dtype, void* y, int ldy, const float* aux, int M, int K,
                   int batch, float* logits, int* tokens, float* max_vals, int index_offset,
                   void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  TcCall c;
  B2D_TRY(tc_gemm_prepare(&c, B2D_F16, reinterpret_cast<const uint16_t*>(Wp),
                          reinterpret_cast<const uint16_t*>(Wp_up), X, ldx, epilogue, y_dtype, y,
                          ldy, aux, M, K, batch, logits, tokens, max_vals, index_offset,
                          workspace, workspace_bytes, true));
  return tc_gemm_launch(c, stream);
}

// ---------------------------------------------------------------------------------------------
// Packed weight layout for the tensor-core GEMV: W [M, K] fp16 (row stride ldw) becomes
// ceil(M/128) x ceil(K/64) tiles of 16 KB, tile (mt, kt) at ((mt * k_tiles) + kt) * 16 KB, each
// holding rows mt*128.. and columns kt*64.. exactly as the MMA reads them from shared memory
// (K-major, 128-byte swizzle: row r at (r/8)*1024 + (r%8)*128, 16-byte chunk c at c ^ (r%8));
// rows / columns past M / K are zero.  A CTA's k-range of one row tile is one contiguous run
// of HBM, where the row-major layout gives it 128-byte pieces of rows K*2 bytes apart.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128) tc_pack_f16_kernel(const uint16_t* __restrict__ W, int M,
                                                          int K, int ldw, int k_tiles,
                                                          uint8_t* __restrict__ out) {
  const int mt = blockIdx.y, kt = blockIdx.x, r = threadIdx.x;
  const int row = mt * tc::BM + r;
  uint8_t* tile = out + ((size_t)mt * k_tiles + kt) * (tc::BM * tc::BK * 2);
  uint8_t* dst = tile + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int col = kt * tc::BK + c * 8;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (row < M && col < K) v = *reinterpret_cast<const uint4*>(W + (size_t)row * ldw + col);
    *reinterpret_cast<uint4*>(dst + ((c ^ (r & 7)) << 4)) = v;
  }
}

size_t tc_packed_bytes(int M, int K) {
  if (M <= 0 || K <= 0) return 0;
  return (size_t)((M + tc::BM - 1) / tc::BM) * ((K + tc::BK - 1) / tc::BK) * (tc::BM * tc::BK * 2);
}

int tc_pack_f16(const uint16_t* W, int ldw, int M, int K, void* out, cudaStream_t stream) {
  if (!W || !out) return B2D_ERR_NULL;
  if (M <= 0 || K <= 0 || K % 8 || ldw < K || ldw % 8 || M > kMaxTiles * tc::BM)
    return B2D_ERR_SHAPE;
  if (!aligned16(W) || !aligned16(out)) return B2D_ERR_ALIGN;
  const int k_tiles = (K + tc::BK - 1) / tc::BK, m_tiles = (M + tc::BM - 1) / tc::BM;
  tc_pack_f16_kernel<<<dim3(k_tiles, m_tiles), 128, 0, stream>>>(W, M, K, ldw, k_tiles,
                                                                  static_cast<uint8_t*>(out));
  return launch_status();
}

// Quantized weights (q8_32 / q4_32) on the tensor cores: STORE / ADD / GELU_MUL epilogues.
int tc_gemm_q(int x_dtype, int w_dtype, const void* q, const uint16_t* scales, const uint16_t* X,
              int ldx, int epilogue, int y_dtype, void* y, int ldy, const float* aux, int M,
              int K, int batch, void* workspace, size_t workspace_bytes, cudaStream_t stream,
              float* const* ys, int n_ys, const void* pf = nullptr, size_t pf_bytes = 0) {
  if (!q || !scales || !X || (!y && n_ys == 0)) return B2D_ERR_NULL;
  if (w_dtype != B2D_Q8_32 && w_dtype != B2D_Q4_32) return B2D_ERR_UNSUPPORTED;
  if (x_dtype != B2D_F16 && x_dtype != B2D_F16X2) return B2D_ERR_UNSUPPORTED;
  if (n_ys < 0 || n_ys > 8 || (n_ys > 0 && (!ys || epilogue != B2D_EPI_STORE || y_dtype != B2D_F32)))
    return B2D_ERR_UNSUPPORTED;
  if (epilogue != B2D_EPI_STORE && epilogue != B2D_EPI_ADD && epilogue != B2D_EPI_GELU_MUL &&
      epilogue != B2D_EPI_SILU_MUL)
    return B2D_ERR_UNSUPPORTED;
  if (y_dtype != B2D_F32 && y_dtype != B2D_F16 && y_dtype != B2D_F16X2) return B2D_ERR_UNSUPPORTED;
  if ((epilogue == B2D_EPI_GELU_MUL || epilogue == B2D_EPI_SILU_MUL) && !aux) return B2D_ERR_NULL;
  if (M <= 0 || K <= 0 || batch <= 0 || batch > 32 || K % 32 || ldx < K || ldx % 8 || ldy < M ||
      M > kMaxTiles * tc::BM)
    return B2D_ERR_SHAPE;
  if (!aligned16(q) || !aligned16(X) || (reinterpret_cast<uintptr_t>(scales) & 1))
    return B2D_ERR_ALIGN;
  const TcPlan pl = tc_plan(M, K, batch, epilogue);
  if (!workspace || workspace_bytes < pl.total) return B2D_ERR_WORKSPACE;
  if (!aligned16(workspace)) return B2D_ERR_ALIGN;
  const int quant = w_dtype == B2D_Q8_32 ? 1 : 2;
  TcCall c;
  tc::Params& p = c.prm;
  p = tc::Params{};
  const int row_bytes = quant == 1 ? K : K / 2;
  const int xs = x_dtype == B2D_F16X2 ? 2 : 1;
  B2D_TRY(make_tmap_u8(&p.tmA, q, M, row_bytes, quant == 1 ? tc::BK : tc::BK / 2, tc::BM));
  B2D_TRY(make_tmap_f16(&p.tmB, X, batch, K, ldx, pl.n_tile));
  if (xs == 2) B2D_TRY(make_tmap_f16(&p.tmB2, X + (size_t)batch * ldx, batch, K, ldx, pl.n_tile));
  char* ws = static_cast<char*>(workspace);
  p.M = M;
  p.K = K;
  p.batch = batch;
  p.k_tiles = pl.k_tiles;
  p.m_tiles = pl.m_tiles;
  p.epi = epilogue;
  p.y = y;
  p.y_f16 = y_dtype != B2D_F32;
  p.y_lo = (y_dtype == B2D_F16X2 && y) ? static_cast<uint16_t*>(y) + (size_t)batch * ldy : nullptr;
  p.ldy = ldy;
  p.aux = aux;
  p.err = reinterpret_cast<int*>(ws);
  p.am_counter = reinterpret_cast<unsigned int*>(ws + 64);
  p.scales = scales;
  p.n_ys = n_ys;
  for (int i = 0; i < n_ys; ++i) {
    if (!ys[i]) return B2D_ERR_NULL;
    p.ys[i] = ys[i];
  }
  p.pf = pf;
  p.pf_bytes = pf_bytes;
  p.k_splits = pick_splits(pl.n_tile, false, quant, xs, pl.m_tiles, pl.k_tiles);
  pick_chains_for(p, pl.n_tile, false, quant, xs);
  c.grid = dim3(pl.m_tiles, p.k_splits);
  c.n_tile = pl.n_tile;
  c.dual = false;
  c.argmax = false;
  c.quant = quant;
  c.xs = xs;
  return tc_gemm_launch(c, stream);
}

}  // namespace b2d
