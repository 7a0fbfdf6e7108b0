// Decode GEMV on CUDA cores: y[b, r] = epilogue(sum_k W[r, k] * xhat[b, k]).
//
// Replaces the reference's matvec_f16 / matvec_f16_add / matvec_gate_up_silu / argmax Metal
// kernels (LK/kernels.metal:106-173, :307-345; epilogue set of GK/kernels.metal:151-198) and
// fuses the RMSNorm dispatch that precedes them (LK/kernels.metal:71-89, LK/main.swift:333).
//
// Design (batch <= 8, HBM-bound: ~2 flops per weight byte):
//  * persistent grid of 256-thread CTAs, sized to fill all SMs once; each warp owns R
//    consecutive rows of a row tile, lanes stride the row in 16-byte chunks, so one warp
//    instruction moves 512 contiguous bytes of a row;
//  * every CTA first stages the (normalized) activations for its batch in shared memory as
//    fp32, computing the RMSNorm scale from the raw rows itself (no separate norm launch);
//  * weights stream with ld.global.nc.L1::no_allocate 16-byte loads, U*R of them in flight
//    per lane, dequantized in registers (int8 / int4 -> fp32 via exponent tricks, one scale
//    multiply per 32-block), accumulated in fp32 and reduced with warp shuffles;
//  * the epilogue (store / residual add / gelu*aux / swiglu / argmax) runs on the reduced sums.
#include <algorithm>

#include "common.cuh"

namespace b2d {

enum { WT_F32 = 0, WT_F16 = 1, WT_Q8 = 2, WT_Q4 = 3 };

template <int WT>
struct WFmt;
template <>
struct WFmt<WT_F32> {
  static constexpr int VEC = 4;  // elements per 16-byte chunk
  static constexpr bool Q = false;
};
template <>
struct WFmt<WT_F16> {
  static constexpr int VEC = 8;
  static constexpr bool Q = false;
};
template <>
struct WFmt<WT_Q8> {
  static constexpr int VEC = 16;
  static constexpr bool Q = true;
};
template <>
struct WFmt<WT_Q4> {
  static constexpr int VEC = 32;
  static constexpr bool Q = true;
};

struct GemvParams {
  const void* W;
  const uint16_t* Ws;   // scales (Q formats)
  const void* W2;       // up matrix (SWIGLU)
  const uint16_t* W2s;  // up scales
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
  int M, K, nb;          // nb = tokens in this launch (<= NB)
  size_t row_bytes;      // bytes per weight row
  int n_tiles;           // row tiles
  int kw;                // warps sharing one row group, each streaming a K slice (1, 2, 4, 8)
  // argmax
  float* logits;         // optional [nb, M]
  int ld_logits;
  int* tokens;
  float* max_vals;
  int index_offset;
  float* part_val;       // [gridDim.x][NB]
  int* part_idx;
  unsigned int* counter;
};

// dot(16-byte weight chunk, VEC fp32 activations); Q formats return the unscaled sum.
template <int WT>
__device__ __forceinline__ float chunk_dot(const uint4& w, const float* xv) {
  float s = 0.f;
  if constexpr (WT == WT_F32) {
    s = fmaf(__uint_as_float(w.x), xv[0], s);
    s = fmaf(__uint_as_float(w.y), xv[1], s);
    s = fmaf(__uint_as_float(w.z), xv[2], s);
    s = fmaf(__uint_as_float(w.w), xv[3], s);
  } else if constexpr (WT == WT_F16) {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = h2f2(u[i]);
      s = fmaf(f.x, xv[2 * i], s);
      s = fmaf(f.y, xv[2 * i + 1], s);
    }
  } else if constexpr (WT == WT_Q8) {
    const uint32_t u[4] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u, w.z ^ 0x80808080u,
                           w.w ^ 0x80808080u};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float q = __uint_as_float(__byte_perm(u[i], 0x4B000000u, 0x7650 + j)) - 8388736.0f;
        s = fmaf(q, xv[4 * i + j], s);
      }
    }
  } else {  // Q4: byte j of the chunk holds elements 2j (low nibble) and 2j+1 (high nibble)
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t lo = (u[i] & 0x0F0F0F0Fu) ^ 0x08080808u;
      uint32_t hi = ((u[i] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float ql = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7650 + j)) - 8388616.0f;
        float qh = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7650 + j)) - 8388616.0f;
        s = fmaf(ql, xv[8 * i + 2 * j], s);
        s = fmaf(qh, xv[8 * i + 2 * j + 1], s);
      }
    }
  }
  return s;
}

// Stage x (optionally RMS-normalized and gamma-scaled) into shared memory as fp32 [NB][K].
// Rows t >= nb are zero.  Also serves as the RMSNorm of LK/kernels.metal:71-89.
template <int NB>
__device__ void stage_x(const GemvParams& p, float* xs, float* red) {
  const int K = p.K;
  const int tid = threadIdx.x;
  float ss[NB];
#pragma unroll
  for (int t = 0; t < NB; ++t) ss[t] = 0.f;
#pragma unroll
  for (int t = 0; t < NB; ++t) {
    if (t < p.nb) {
      if (p.x_f16) {
        const uint16_t* xr = reinterpret_cast<const uint16_t*>(p.x) + (size_t)t * p.ldx;
        for (int k = tid * 8; k < K; k += 256 * 8) {
          uint4 v = *reinterpret_cast<const uint4*>(xr + k);
          const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float2 f = h2f2(u[i]);
            xs[t * K + k + 2 * i] = f.x;
            xs[t * K + k + 2 * i + 1] = f.y;
            ss[t] = fmaf(f.x, f.x, ss[t]);
            ss[t] = fmaf(f.y, f.y, ss[t]);
          }
        }
      } else {
        const float* xr = reinterpret_cast<const float*>(p.x) + (size_t)t * p.ldx;
        for (int k = tid * 4; k < K; k += 256 * 4) {
          float4 v = *reinterpret_cast<const float4*>(xr + k);
          *reinterpret_cast<float4*>(xs + t * K + k) = v;
          ss[t] = fmaf(v.x, v.x, ss[t]);
          ss[t] = fmaf(v.y, v.y, ss[t]);
          ss[t] = fmaf(v.z, v.z, ss[t]);
          ss[t] = fmaf(v.w, v.w, ss[t]);
        }
      }
    } else {
      for (int k = tid; k < K; k += 256) xs[t * K + k] = 0.f;
    }
  }
  if (p.gamma == nullptr) {
    __syncthreads();
    return;
  }
  const int warp = tid >> 5, lane = tid & 31;
#pragma unroll
  for (int t = 0; t < NB; ++t) {
    float v = warp_sum(ss[t]);
    if (lane == 0) red[warp * NB + t] = v;
  }
  __syncthreads();
  float scale[NB];
#pragma unroll
  for (int t = 0; t < NB; ++t) {
    float tot = 0.f;
    for (int w = 0; w < 8; ++w) tot += red[w * NB + t];
    scale[t] = rsqrtf(tot / (float)K + p.eps);
  }
  for (int k = tid; k < K; k += 256) {
    const float g = __ldg(p.gamma + k);
#pragma unroll
    for (int t = 0; t < NB; ++t) xs[t * K + k] = xs[t * K + k] * scale[t] * g;
  }
  __syncthreads();
}

#ifndef B2D_GEMV_TILES_PER_SM
#define B2D_GEMV_TILES_PER_SM 2
#endif

template <int WT, int NB, bool DUAL>
struct GemvCfg {
  static constexpr int R = DUAL ? 2 : (NB >= 4 ? 2 : 4);  // rows per warp
  static constexpr int U = 2;                              // chunk iterations in flight
  static constexpr int ROWS_PER_CTA = 8 * R;               // with kw = 1 (R * 8 / kw in general)
};

template <int WT, int NB, bool DUAL, bool ARGMAX, bool KSPLIT>
__global__ void __launch_bounds__(256) gemv_kernel(const GemvParams p) {
  using F = WFmt<WT>;
  constexpr int VEC = F::VEC;
  constexpr int R = GemvCfg<WT, NB, DUAL>::R;
  constexpr int U = GemvCfg<WT, NB, DUAL>::U;
  extern __shared__ __align__(16) float xs[];  // [NB][K]
  __shared__ float red[8 * 8 * 2];
  __shared__ int redi[8 * 8];
  // K-split partial sums of the warps of a row group: [warp][R][NB] (and the up matrix's)
  __shared__ float kpart[8][R][NB];
  __shared__ float kpart2[DUAL ? 8 : 1][R][NB];

  pdl_wait();
  stage_x<NB>(p, xs, red);
  pdl_launch_dependents();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Short, wide matrices (few row tiles, long rows) let kw warps share a row group, each
  // streaming an interleaved slice of K, so that every SM has enough loads in flight.
  const int kw = KSPLIT ? p.kw : 1, groups = 8 / kw, grp = warp / kw, kslice = warp % kw;
  const int K = p.K, M = p.M;
  const int nchunks = K / VEC;
  const int nscale = K / 32;
  const char* Wb = reinterpret_cast<const char*>(p.W);
  const char* W2b = reinterpret_cast<const char*>(p.W2);

  float best_v[NB];
  int best_i[NB];
  if constexpr (ARGMAX) {
#pragma unroll
    for (int t = 0; t < NB; ++t) {
      best_v[t] = -INFINITY;
      best_i[t] = 0x7fffffff;
    }
  }

  for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
    const int row0 = (tile * groups + grp) * R;
    const bool active = row0 < M;  // no early exit: the K-split reduce below is CTA-wide
    int rows[R];
#pragma unroll
    for (int r = 0; r < R; ++r) rows[r] = min(row0 + r, M - 1);

    float acc[R][NB];
    float acc2[DUAL ? R : 1][NB];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int t = 0; t < NB; ++t) {
        acc[r][t] = 0.f;
        if constexpr (DUAL) acc2[r][t] = 0.f;
      }

    for (int c0 = kslice * 32 + lane; active && c0 < nchunks; c0 += 32 * U * kw) {
      uint4 wv[U][R];
      uint4 wv2[DUAL ? U : 1][R];
      float sc[U][R], sc2[DUAL ? U : 1][R];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + 32 * kw * u;
        const int cc = c < nchunks ? c : c0;  // clamp: re-read a valid chunk, discarded below
#pragma unroll
        for (int r = 0; r < R; ++r) {
          wv[u][r] = ld_stream16(Wb + (size_t)rows[r] * p.row_bytes + (size_t)cc * 16);
          if constexpr (DUAL)
            wv2[u][r] = ld_stream16(W2b + (size_t)rows[r] * p.row_bytes + (size_t)cc * 16);
          if constexpr (F::Q) {
            const int si = (cc * VEC) / 32;
            sc[u][r] = h2f(__ldg(p.Ws + (size_t)rows[r] * nscale + si));
            if constexpr (DUAL) sc2[u][r] = h2f(__ldg(p.W2s + (size_t)rows[r] * nscale + si));
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + 32 * kw * u;
        if (c >= nchunks) break;
#pragma unroll
        for (int t = 0; t < NB; ++t) {
          float xv[VEC];
          const float4* xp = reinterpret_cast<const float4*>(xs + t * K + c * VEC);
#pragma unroll
          for (int i = 0; i < VEC / 4; ++i) {
            float4 f = xp[i];
            xv[4 * i] = f.x;
            xv[4 * i + 1] = f.y;
            xv[4 * i + 2] = f.z;
            xv[4 * i + 3] = f.w;
          }
#pragma unroll
          for (int r = 0; r < R; ++r) {
            float d = chunk_dot<WT>(wv[u][r], xv);
            if constexpr (F::Q) d *= sc[u][r];
            acc[r][t] += d;
            if constexpr (DUAL) {
              float d2 = chunk_dot<WT>(wv2[u][r], xv);
              if constexpr (F::Q) d2 *= sc2[u][r];
              acc2[r][t] += d2;
            }
          }
        }
      }
    }

    // reduce (warp, then across the kw warps of the group in a fixed order) + epilogue
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int t = 0; t < NB; ++t) {
        acc[r][t] = warp_sum(acc[r][t]);
        if constexpr (DUAL) acc2[r][t] = warp_sum(acc2[r][t]);
      }
    if (KSPLIT && kw > 1) {
      if (lane == 0)
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int t = 0; t < NB; ++t) {
            kpart[warp][r][t] = acc[r][t];
            if constexpr (DUAL) kpart2[warp][r][t] = acc2[r][t];
          }
      __syncthreads();
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < NB; ++t) {
          float a = 0.f, a2 = 0.f;
          for (int j = 0; j < kw; ++j) {
            a += kpart[grp * kw + j][r][t];
            if constexpr (DUAL) a2 += kpart2[grp * kw + j][r][t];
          }
          acc[r][t] = a;
          if constexpr (DUAL) acc2[r][t] = a2;
        }
      __syncthreads();  // kpart is rewritten by the next tile
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int row = row0 + r;
#pragma unroll
      for (int t = 0; t < NB; ++t) {
        const float s = acc[r][t];
        float s2 = 0.f;
        if constexpr (DUAL) s2 = acc2[r][t];
        if (active && kslice == 0 && row < M && t < p.nb) {
          if constexpr (ARGMAX) {
            if (lane == 0 && p.logits) p.logits[(size_t)t * p.ld_logits + row] = s;
            if (better(s, row, best_v[t], best_i[t])) {
              best_v[t] = s;
              best_i[t] = row;
            }
          } else if (lane == 0) {
            float v;
            const size_t yi = (size_t)t * p.ldy + row;
            if constexpr (DUAL) {
              v = silu(s) * s2;
            } else {
              v = s;
              if (p.epi == B2D_EPI_ADD) {
                v += p.y_f16 ? h2f(reinterpret_cast<const uint16_t*>(p.y)[yi])
                             : reinterpret_cast<const float*>(p.y)[yi];
              } else if (p.epi == B2D_EPI_GELU_MUL) {
                v = gelu_tanh(v) * p.aux[yi];
              }
            }
            if (p.y_f16)
              reinterpret_cast<uint16_t*>(p.y)[yi] = f2h(v);
            else
              reinterpret_cast<float*>(p.y)[yi] = v;
          }
        }
      }
    }
  }

  if constexpr (ARGMAX) {
    // CTA-level reduce (all lanes of a warp hold the same best), then one partial per CTA.
    __syncthreads();
    if (lane == 0) {
#pragma unroll
      for (int t = 0; t < NB; ++t) {
        red[warp * NB + t] = best_v[t];
        redi[warp * NB + t] = best_i[t];
      }
    }
    __syncthreads();
    __shared__ bool is_last;
    if (threadIdx.x < NB) {
      const int t = threadIdx.x;
      float bv = red[t];
      int bi = redi[t];
      for (int w = 1; w < 8; ++w)
        if (better(red[w * NB + t], redi[w * NB + t], bv, bi)) {
          bv = red[w * NB + t];
          bi = redi[w * NB + t];
        }
      p.part_val[blockIdx.x * NB + t] = bv;
      p.part_idx[blockIdx.x * NB + t] = bi;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = (atomicAdd(p.counter, 1u) == gridDim.x - 1);
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // last CTA: warp t reduces token t over all CTA partials
    for (int t = warp; t < p.nb; t += 8) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int b = lane; b < (int)gridDim.x; b += 32) {
        float v = __ldcg(p.part_val + b * NB + t);
        int i = __ldcg(p.part_idx + b * NB + t);
        if (better(v, i, bv, bi)) {
          bv = v;
          bi = i;
        }
      }
      warp_argmax(bv, bi);
      if (lane == 0) {
        p.tokens[t] = bi + p.index_offset;
        if (p.max_vals) p.max_vals[t] = bv;
      }
    }
    if (threadIdx.x == 0) *p.counter = 0u;  // ready for the next launch
  }
}

// ------------------------------------------------------------------------------------------
// host
// ------------------------------------------------------------------------------------------

struct LaunchInfo {
  int grid_cap = 0;
};

template <int WT, int NB, bool DUAL, bool ARGMAX, bool KSPLIT>
static int launch_gemv_k(GemvParams& p, cudaStream_t stream, int max_grid) {
  constexpr int ROWS = GemvCfg<WT, NB, DUAL>::ROWS_PER_CTA;
  const size_t smem = (size_t)NB * p.K * sizeof(float);
  static int cached_dev = -1;
  static size_t cached_smem = 0;
  static int occ = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  auto kern = gemv_kernel<WT, NB, DUAL, ARGMAX, KSPLIT>;
  if (dev != cached_dev || smem != cached_smem) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return launch_status();
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, 256, smem) != cudaSuccess)
      return launch_status();
    cached_dev = dev;
    cached_smem = smem;
  }
  const int rows_per_tile = ROWS / p.kw;
  p.n_tiles = (p.M + rows_per_tile - 1) / rows_per_tile;
  int grid = std::min(p.n_tiles, std::max(1, occ) * num_sms());
  if (max_grid > 0) grid = std::min(grid, max_grid);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return B2D_ERR_CUDA;
  }
  count_launch();
  return B2D_OK;
}

// kw: the fewest warps per row group that still give every SM B2D_GEMV_TILES_PER_SM row tiles;
// matrices with enough rows keep the plain kernel (one warp per row group).
template <int WT, int NB, bool DUAL, bool ARGMAX>
static int launch_gemv(GemvParams& p, cudaStream_t stream, int max_grid = 0) {
  constexpr int ROWS = GemvCfg<WT, NB, DUAL>::ROWS_PER_CTA;
  p.kw = 1;
  while (p.kw < 8 && (p.M + ROWS / p.kw - 1) / (ROWS / p.kw) < B2D_GEMV_TILES_PER_SM * num_sms())
    p.kw *= 2;
  return p.kw > 1 ? launch_gemv_k<WT, NB, DUAL, ARGMAX, true>(p, stream, max_grid)
                  : launch_gemv_k<WT, NB, DUAL, ARGMAX, false>(p, stream, max_grid);
}

// Largest fp32 activation staging per CTA (bytes): NB * K * 4 must fit.
static constexpr size_t kMaxStageBytes = 160 * 1024;

template <int WT, bool DUAL, bool ARGMAX>
static int dispatch_nb(GemvParams& p, int nb, cudaStream_t stream, int max_grid = 0) {
  p.nb = nb;
  if (nb == 1) return launch_gemv<WT, 1, DUAL, ARGMAX>(p, stream, max_grid);
  if (nb == 2) return launch_gemv<WT, 2, DUAL, ARGMAX>(p, stream, max_grid);
  if (nb <= 4) return launch_gemv<WT, 4, DUAL, ARGMAX>(p, stream, max_grid);
  return launch_gemv<WT, 8, DUAL, ARGMAX>(p, stream, max_grid);
}

// Largest token group whose fp32 staging fits in shared memory.
static int max_group(int K) {
  int g = 8;
  while (g > 1 && (size_t)g * K * 4 > kMaxStageBytes) g >>= 1;
  return g;
}

template <int WT, bool DUAL>
static int run_groups(GemvParams p, int batch, cudaStream_t stream) {
  const int g = max_group(p.K);
  const size_t xsz = p.x_f16 ? 2 : 4;
  const size_t ysz = p.y_f16 ? 2 : 4;
  const void* x0 = p.x;
  void* y0 = p.y;
  const float* aux0 = p.aux;
  for (int b0 = 0; b0 < batch; b0 += g) {
    const int nb = std::min(g, batch - b0);
    p.x = static_cast<const char*>(x0) + (size_t)b0 * p.ldx * xsz;
    p.y = static_cast<char*>(y0) + (size_t)b0 * p.ldy * ysz;
    p.aux = aux0 ? aux0 + (size_t)b0 * p.ldy : nullptr;
    B2D_TRY((dispatch_nb<WT, DUAL, false>(p, nb, stream)));
  }
  return B2D_OK;
}

// Tensor-core GEMV for quantized (and optionally fp16) weights, gemv_mma.cu.
bool gemv_mma_eligible(int w_dtype, const void* W_scales, const void* W_up_scales, int K,
                       int epilogue);
int gemv_mma_dispatch(int w_dtype, const void* W, const void* W_scales, const void* W_up,
                      const void* W_up_scales, int x_dtype, const void* x, int ldx,
                      const float* gamma, float eps, int epilogue, int y_dtype, void* y, int ldy,
                      const float* aux, int M, int K, int batch, cudaStream_t stream);

static size_t elem_row_bytes(int w_dtype, int K) {
  switch (w_dtype) {
    case B2D_F32: return (size_t)K * 4;
    case B2D_F16: return (size_t)K * 2;
    case B2D_Q8_32: return (size_t)K;
    default: return (size_t)K / 2;
  }
}

int gemv_dispatch(int w_dtype, const void* W, const void* W_scales, const void* W_up,
                  const void* W_up_scales, int x_dtype, const void* x, int ldx,
                  const float* gamma, float eps, int epilogue, int y_dtype, void* y, int ldy,
                  const float* aux, int M, int K, int batch, cudaStream_t stream) {
  if (!W || !x || !y) return B2D_ERR_NULL;
  if (M <= 0 || K <= 0 || batch <= 0) return B2D_ERR_SHAPE;
  if (epilogue < B2D_EPI_STORE || epilogue > B2D_EPI_SWIGLU) return B2D_ERR_UNSUPPORTED;
  if (x_dtype != B2D_F32 && x_dtype != B2D_F16) return B2D_ERR_UNSUPPORTED;
  if (y_dtype != B2D_F32 && y_dtype != B2D_F16) return B2D_ERR_UNSUPPORTED;
  const bool quant = (w_dtype == B2D_Q8_32 || w_dtype == B2D_Q4_32);
  if (w_dtype < B2D_F32 || w_dtype > B2D_Q4_32) return B2D_ERR_UNSUPPORTED;
  const int kmul = quant ? 32 : (w_dtype == B2D_F16 ? 8 : 4);
  if (K % kmul) return B2D_ERR_SHAPE;
  if (x_dtype == B2D_F16 && K % 8) return B2D_ERR_SHAPE;  // fp16 rows are staged 8 at a time
  if (quant && (!W_scales || (epilogue == B2D_EPI_SWIGLU && !W_up_scales)))
    return B2D_ERR_NULL;
  if (epilogue == B2D_EPI_SWIGLU && !W_up) return B2D_ERR_NULL;
  if (epilogue == B2D_EPI_GELU_MUL && !aux) return B2D_ERR_NULL;
  if ((size_t)K * 4 > kMaxStageBytes) return B2D_ERR_SHAPE;
  if (ldx < K || ldy < M) return B2D_ERR_SHAPE;
  const size_t xsz = x_dtype == B2D_F16 ? 2 : 4;
  if (!aligned16(W) || !aligned16(x) || ((size_t)ldx * xsz) % 16 || (W_up && !aligned16(W_up)))
    return B2D_ERR_ALIGN;
  if (gemv_mma_eligible(w_dtype, W_scales, W_up_scales, K, epilogue))
    return gemv_mma_dispatch(w_dtype, W, W_scales, W_up, W_up_scales, x_dtype, x, ldx, gamma, eps,
                             epilogue, y_dtype, y, ldy, aux, M, K, batch, stream);
  GemvParams p = {};
  p.W = W;
  p.Ws = static_cast<const uint16_t*>(W_scales);
  p.W2 = W_up;
  p.W2s = static_cast<const uint16_t*>(W_up_scales);
  p.x = x;
  p.x_f16 = x_dtype == B2D_F16;
  p.ldx = ldx;
  p.gamma = gamma;
  p.eps = eps;
  p.epi = epilogue;
  p.y = y;
  p.y_f16 = y_dtype == B2D_F16;
  p.ldy = ldy;
  p.aux = aux;
  p.M = M;
  p.K = K;
  p.row_bytes = elem_row_bytes(w_dtype, K);
  const bool dual = epilogue == B2D_EPI_SWIGLU;
  switch (w_dtype) {
    case B2D_F32:
      if (dual) return B2D_ERR_UNSUPPORTED;
      return run_groups<WT_F32, false>(p, batch, stream);
    case B2D_F16:
      return dual ? run_groups<WT_F16, true>(p, batch, stream)
                  : run_groups<WT_F16, false>(p, batch, stream);
    case B2D_Q8_32:
      return dual ? run_groups<WT_Q8, true>(p, batch, stream)
                  : run_groups<WT_Q8, false>(p, batch, stream);
    default:
      return dual ? run_groups<WT_Q4, true>(p, batch, stream)
                  : run_groups<WT_Q4, false>(p, batch, stream);
  }
}

// LM head + argmax.  Workspace: [grid cap][8] (value, index) partials + one counter.
static int argmax_grid_cap() { return 8 * num_sms(); }

size_t lm_head_argmax_workspace_bytes(int V, int batch) {
  (void)V;
  (void)batch;
  const size_t parts = (size_t)argmax_grid_cap() * 8;
  return 256 + parts * (sizeof(float) + sizeof(int));
}

int lm_head_argmax(const uint16_t* W, const float* x, int ldx, const float* gamma, float eps,
                   int V, int K, int batch, int index_offset, float* logits, int* tokens,
                   float* max_vals, void* workspace, size_t workspace_bytes,
                   cudaStream_t stream) {
  if (!W || !x || !tokens) return B2D_ERR_NULL;
  if (V <= 0 || K <= 0 || batch <= 0 || K % 8 || ldx < K) return B2D_ERR_SHAPE;
  if ((size_t)K * 4 > kMaxStageBytes) return B2D_ERR_SHAPE;
  if (!aligned16(W) || !aligned16(x) || ((size_t)ldx * 4) % 16) return B2D_ERR_ALIGN;
  if (!workspace || workspace_bytes < lm_head_argmax_workspace_bytes(V, batch))
    return B2D_ERR_WORKSPACE;
  if (!aligned16(workspace)) return B2D_ERR_ALIGN;
  GemvParams p = {};
  p.W = W;
  p.x = x;
  p.x_f16 = 0;
  p.ldx = ldx;
  p.gamma = gamma;
  p.eps = eps;
  p.epi = B2D_EPI_ARGMAX;
  p.M = V;
  p.K = K;
  p.row_bytes = (size_t)K * 2;
  p.index_offset = index_offset;
  char* ws = static_cast<char*>(workspace);
  p.counter = reinterpret_cast<unsigned int*>(ws);
  const size_t parts = (size_t)argmax_grid_cap() * 8;
  p.part_val = reinterpret_cast<float*>(ws + 256);
  p.part_idx = reinterpret_cast<int*>(ws + 256 + parts * sizeof(float));
  const int g = max_group(K);
  for (int b0 = 0; b0 < batch; b0 += g) {
    const int nb = std::min(g, batch - b0);
    p.x = x + (size_t)b0 * ldx;
    p.logits = logits ? logits + (size_t)b0 * V : nullptr;
    p.ld_logits = V;
    p.tokens = tokens + b0;
    p.max_vals = max_vals ? max_vals + b0 : nullptr;
    B2D_TRY((dispatch_nb<WT_F16, false, true>(p, nb, stream, argmax_grid_cap())));
  }
  return B2D_OK;
}

// ------------------------------------------------------------------------------------------
// Dequantization to fp32 (exact): one thread per 16-byte chunk of q.
// ------------------------------------------------------------------------------------------
template <bool Q4>
__global__ void dequant_kernel(const uint8_t* q, const uint16_t* scales, float* w, int M, int K) {
  const int per_row = Q4 ? K / 32 : K / 16;  // 16-byte chunks per row
  const size_t n = (size_t)M * per_row;
  for (size_t c = blockIdx.x * (size_t)blockDim.x + threadIdx.x; c < n;
       c += (size_t)gridDim.x * blockDim.x) {
    const int row = (int)(c / per_row), ci = (int)(c % per_row);
    const uint4 v = *reinterpret_cast<const uint4*>(q + (size_t)row * (Q4 ? K / 2 : K) + ci * 16);
    const int k0 = ci * (Q4 ? 32 : 16);
    const float s = h2f(scales[(size_t)row * (K / 32) + k0 / 32]);
    float* out = w + (size_t)row * K + k0;
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (Q4) {
        uint32_t lo = (u[i] & 0x0F0F0F0Fu) ^ 0x08080808u;
        uint32_t hi = ((u[i] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          out[8 * i + 2 * j] =
              s * (__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7650 + j)) - 8388616.0f);
          out[8 * i + 2 * j + 1] =
              s * (__uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7650 + j)) - 8388616.0f);
        }
      } else {
        const uint32_t b = u[i] ^ 0x80808080u;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          out[4 * i + j] =
              s * (__uint_as_float(__byte_perm(b, 0x4B000000u, 0x7650 + j)) - 8388736.0f);
      }
    }
  }
}

int dequant(bool q4, const void* q, const uint16_t* scales, float* w, int M, int K,
            cudaStream_t stream) {
  if (!q || !scales || !w) return B2D_ERR_NULL;
  if (M <= 0 || K <= 0 || K % 32) return B2D_ERR_SHAPE;
  if (!aligned16(q)) return B2D_ERR_ALIGN;
  const size_t chunks = (size_t)M * (q4 ? K / 32 : K / 16);
  const int grid = (int)std::min<size_t>((chunks + 255) / 256, (size_t)num_sms() * 16);
  if (q4)
    dequant_kernel<true><<<grid, 256, 0, stream>>>(static_cast<const uint8_t*>(q), scales, w, M, K);
  else
    dequant_kernel<false><<<grid, 256, 0, stream>>>(static_cast<const uint8_t*>(q), scales, w, M, K);
  return launch_status();
}

}  // namespace b2d
