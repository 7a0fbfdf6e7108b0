// Small ops of the decode step: RMSNorm, embedding gather, argmax, residual add.
// Each replaces one reference Metal kernel (cited per kernel).
#include <algorithm>

#include "common.cuh"

namespace b2d {

// One CTA per row: y = x * rsqrt(mean(x^2) + eps) * w   (LK/kernels.metal:71-89)
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* x, const float* w, float* y,
                                                      int D, float eps) {
  __shared__ float red[8];
  const float* xr = x + (size_t)blockIdx.x * D;
  float* yr = y + (size_t)blockIdx.x * D;
  float ss = 0.f;
  for (int i = threadIdx.x; i < D; i += 256) ss = fmaf(xr[i], xr[i], ss);
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float scale = rsqrtf(tot / (float)D + eps);
  for (int i = threadIdx.x; i < D; i += 256) yr[i] = xr[i] * scale * w[i];
}

int rmsnorm(const float* x, const float* w, float* y, int rows, int D, float eps,
            cudaStream_t stream) {
  if (!x || !w || !y) return B2D_ERR_NULL;
  if (rows <= 0 || D <= 0) return B2D_ERR_SHAPE;
  rmsnorm_kernel<<<rows, 256, 0, stream>>>(x, w, y, D, eps);
  return launch_status();
}

// x[b, i] = float(E[tokens[b], i])   (LK/kernels.metal:31-39)
__global__ void embed_kernel(const uint16_t* E, const int* tokens, float* x, int D) {
  const int b = blockIdx.y;
  const size_t tok = (size_t)tokens[b];
  const uint16_t* er = E + tok * D;
  float* xr = x + (size_t)b * D;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < D; i += gridDim.x * blockDim.x)
    xr[i] = h2f(er[i]);
}

int embed_f16(const uint16_t* E, const int* tokens, float* x, int D, int batch,
              cudaStream_t stream) {
  if (!E || !tokens || !x) return B2D_ERR_NULL;
  if (D <= 0 || batch <= 0) return B2D_ERR_SHAPE;
  dim3 grid((D + 255) / 256, batch);
  embed_kernel<<<grid, 256, 0, stream>>>(E, tokens, x, D);
  return launch_status();
}

// tokens[b] = argmax(logits[b]) + offset, ties -> lowest index (LK/kernels.metal:310-345).
// One 1024-thread CTA per row, like the reference's single threadgroup.
__global__ void __launch_bounds__(1024) argmax_kernel(const float* logits, int N, int* tokens,
                                                      int offset) {
  __shared__ float bvs[32];
  __shared__ int bis[32];
  const float* row = logits + (size_t)blockIdx.x * N;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < N; i += 1024) {
    const float v = row[i];
    if (better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
  warp_argmax(bv, bi);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    bvs[warp] = bv;
    bis[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    bv = bvs[lane];
    bi = bis[lane];
    warp_argmax(bv, bi);
    if (lane == 0) tokens[blockIdx.x] = (bi == 0x7fffffff ? 0 : bi) + offset;
  }
}

int argmax_f32(const float* logits, int N, int batch, int* tokens, int offset,
               cudaStream_t stream) {
  if (!logits || !tokens) return B2D_ERR_NULL;
  if (N <= 0 || batch <= 0) return B2D_ERR_SHAPE;
  argmax_kernel<<<batch, 1024, 0, stream>>>(logits, N, tokens, offset);
  return launch_status();
}

// Combine [n_parts][batch] (value, global index) candidates; ties -> lowest index.
__global__ void argmax_combine_kernel(const float* vals, const int* idxs, int n_parts, int batch,
                                      int* tokens) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  float bv = vals[b];
  int bi = idxs[b];
  for (int r = 1; r < n_parts; ++r) {
    const float v = vals[(size_t)r * batch + b];
    const int i = idxs[(size_t)r * batch + b];
    if (better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
  tokens[b] = bi;
}

int argmax_combine(const float* vals, const int* idxs, int n_parts, int batch, int* tokens,
                   cudaStream_t stream) {
  if (!vals || !idxs || !tokens) return B2D_ERR_NULL;
  if (n_parts <= 0 || batch <= 0) return B2D_ERR_SHAPE;
  argmax_combine_kernel<<<(batch + 127) / 128, 128, 0, stream>>>(vals, idxs, n_parts, batch,
                                                                 tokens);
  return launch_status();
}

__global__ void add_kernel(float* x, const float* p, size_t n) {
  const size_t n4 = n / 4;
  float4* x4 = reinterpret_cast<float4*>(x);
  const float4* p4 = reinterpret_cast<const float4*>(p);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4;
       i += (size_t)gridDim.x * blockDim.x) {
    float4 a = x4[i];
    const float4 b = p4[i];
    a.x += b.x;
    a.y += b.y;
    a.z += b.z;
    a.w += b.w;
    x4[i] = a;
  }
  for (size_t i = n4 * 4 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    x[i] += p[i];
}

int add_f32(float* x, const float* p, size_t n, cudaStream_t stream) {
  if (!x || !p) return B2D_ERR_NULL;
  if (n == 0) return B2D_OK;
  if (!aligned16(x) || !aligned16(p)) return B2D_ERR_ALIGN;
  const int grid = (int)std::min<size_t>((n / 4 + 255) / 256 + 1, (size_t)num_sms() * 4);
  add_kernel<<<grid, 256, 0, stream>>>(x, p, n);
  return launch_status();
}

// Residual add + RMSNorm to fp16 (the tensor-core GEMMs' activation operand), one CTA per row:
//   if p: x += p (written back);   out = fp16(x * rsqrt(mean(x^2) + eps) * gamma)
// and, with out_lo, the remainder fp16(v - out) into out_lo (the B2D_F16X2 lo plane).
// (rmsnorm LK/kernels.metal:71-89; the add is the residual update after a tensor-parallel
// all-reduce).  Launched with programmatic dependent launch.
// Row width handled from registers: up to kNormVec float4 per thread (D <= 4096 at 256 threads);
// wider or unaligned rows take the scalar loop.
constexpr int kNormVec = 4;

__device__ __forceinline__ float block_sum_256(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) t += red[i];
  return t;
}

__global__ void __launch_bounds__(256) add_rmsnorm_f16_kernel(float* x, const float* p,
                                                              const float* gamma, float eps,
                                                              uint16_t* out, uint16_t* out_lo,
                                                              int D) {
  __shared__ float red[8];
  pdl_wait();
  float* xr = x + (size_t)blockIdx.x * D;
  const float* pr = p ? p + (size_t)blockIdx.x * D : nullptr;
  uint16_t* orow = out + (size_t)blockIdx.x * D;
  uint16_t* lrow = out_lo ? out_lo + (size_t)blockIdx.x * D : nullptr;
  const bool vec = (D & 3) == 0 && D <= kNormVec * 4 * 256 &&
                   ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(gamma) |
                     reinterpret_cast<uintptr_t>(p)) & 15) == 0 &&
                   ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(out_lo)) & 7) == 0;
  if (vec) {
    // all loads of the row issued before the first use: one memory latency, not D/256 of them
    float4 v[kNormVec];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < kNormVec; ++k) {
      const int i = threadIdx.x + k * 256;
      if (4 * i < D) {
        v[k] = reinterpret_cast<const float4*>(xr)[i];
        if (pr) {
          const float4 a = reinterpret_cast<const float4*>(pr)[i];
          v[k].x += a.x;
          v[k].y += a.y;
          v[k].z += a.z;
          v[k].w += a.w;
        }
      }
    }
#pragma unroll
    for (int k = 0; k < kNormVec; ++k) {
      const int i = threadIdx.x + k * 256;
      if (4 * i < D) {
        if (pr) reinterpret_cast<float4*>(xr)[i] = v[k];
        ss = fmaf(v[k].x, v[k].x, fmaf(v[k].y, v[k].y, fmaf(v[k].z, v[k].z, fmaf(v[k].w, v[k].w, ss))));
      }
    }
    const float scale = rsqrtf(block_sum_256(ss, red) / (float)D + eps);
    pdl_launch_dependents();
#pragma unroll
    for (int k = 0; k < kNormVec; ++k) {
      const int i = threadIdx.x + k * 256;
      if (4 * i < D) {
        const float4 g = reinterpret_cast<const float4*>(gamma)[i];
        uint2 lo;
        reinterpret_cast<uint2*>(orow)[i] = split4_f16(v[k].x * scale * g.x, v[k].y * scale * g.y,
                                                       v[k].z * scale * g.z, v[k].w * scale * g.w, &lo);
        if (lrow) reinterpret_cast<uint2*>(lrow)[i] = lo;
      }
    }
    return;
  }
  float ss = 0.f;
  for (int i = threadIdx.x; i < D; i += 256) {
    float v = xr[i];
    if (pr) {
      v += pr[i];
      xr[i] = v;
    }
    ss = fmaf(v, v, ss);
  }
  const float scale = rsqrtf(block_sum_256(ss, red) / (float)D + eps);
  pdl_launch_dependents();
  for (int i = threadIdx.x; i < D; i += 256) store_f16_split(orow, lrow, i, xr[i] * scale * gamma[i]);
}

int add_rmsnorm_f16(float* x, const float* p, const float* gamma, float eps, uint16_t* out,
                    uint16_t* out_lo, int rows, int D, cudaStream_t stream) {
  if (!x || !gamma || !out) return B2D_ERR_NULL;
  if (rows <= 0 || D <= 0) return B2D_ERR_SHAPE;
  return launch_pdl(add_rmsnorm_f16_kernel, dim3(rows), dim3(256), 0, stream, x, p, gamma, eps,
                    out, out_lo, D);
}

// Embedding gather + RMSNorm to fp16: x[b] = float(E[tokens[b]]); out[b] = fp16(norm(x[b])*gamma)
// (embed LK/kernels.metal:31-39 fused with the first layer's rmsnorm); with out_lo, also the
// B2D_F16X2 lo plane.
__global__ void __launch_bounds__(256) embed_rmsnorm_f16_kernel(const uint16_t* E,
                                                                const int* tokens, float* x,
                                                                const float* gamma, float eps,
                                                                uint16_t* out, uint16_t* out_lo,
                                                                float* r_out, int D) {
  __shared__ float red[8];
  pdl_wait();
  const size_t tok = (size_t)tokens[blockIdx.x];
  const uint16_t* er = E + tok * D;
  float* xr = x + (size_t)blockIdx.x * D;
  uint16_t* orow = out + (size_t)blockIdx.x * D;
  uint16_t* lrow = out_lo ? out_lo + (size_t)blockIdx.x * D : nullptr;
  float ss = 0.f;
  for (int i = threadIdx.x; i < D; i += 256) {
    const float v = h2f(er[i]);
    xr[i] = v;
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float scale = rsqrtf(tot / (float)D + eps);
  if (r_out && threadIdx.x == 0) r_out[blockIdx.x] = scale;
  pdl_launch_dependents();
  for (int i = threadIdx.x; i < D; i += 256) store_f16_split(orow, lrow, i, xr[i] * scale * gamma[i]);
}

// r_out (optional): each row's norm factor rsqrt(mean(x^2) + eps).
int embed_rmsnorm_f16(const uint16_t* E, const int* tokens, float* x, const float* gamma,
                      float eps, uint16_t* out, uint16_t* out_lo, float* r_out, int D, int batch,
                      cudaStream_t stream) {
  if (!E || !tokens || !x || !gamma || !out) return B2D_ERR_NULL;
  if (D <= 0 || batch <= 0) return B2D_ERR_SHAPE;
  return launch_pdl(embed_rmsnorm_f16_kernel, dim3(batch), dim3(256), 0, stream, E, tokens, x,
                    gamma, eps, out, out_lo, r_out, D);
}

}  // namespace b2d
