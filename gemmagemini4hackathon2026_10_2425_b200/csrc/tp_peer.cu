// Tensor-parallel collectives of the decode step over NVLink peer memory.
//
// The row-parallel O and down projections leave each rank with a partial sum of the residual
// update; the reference runs one GPU and has no such step (ios_kernels/kernels/*/main.swift
// encodeDecode adds the projection straight into the residual).  Here the partials of all
// ranks are summed with one kernel that also does what follows the sum in the decode step:
//
//   x[b] += part_0[b] + part_1[b] + ... + part_{tp-1}[b]        (rank order: every rank gets
//   out16[b] = fp16(rmsnorm(x[b]) * gamma)                        bit-identical results)
//
// One CTA per token row.  The partials live in buffers every rank has mapped (CUDA IPC).  With
// the tensor-core projections each rank's GEMM epilogue has already stored its partial into
// every rank's receive slot (remote stores overlap the GEMM's tail), so the sum reads local
// memory; otherwise each rank's partial sits in its own memory and is read over NVLink.  A CTA
// announces "my partial of row b is complete" by writing an epoch number into every peer's
// signal array, waits (bounded) until all peers' epochs for row b have arrived in its own
// array, then sums.  Per-row barriers, no grid-wide synchronization, no NCCL launch, and the
// residual add + RMSNorm kernel that would follow the all-reduce is gone.
//
// The vocab-parallel LM head ends the same way: each rank's (max logit, index) per token is
// gathered from the peers and combined (ties -> lowest index), replacing two all-gathers and a
// combine kernel.
//
// Buffer reuse: the decoder alternates two sets of partial buffers (O -> 0, down -> 1).  A rank
// writes set k again (locally or into a peer's receive slots) only after it has passed the
// barrier of the use in between, which every peer reaches only after finishing its reads of set
// k (each kernel waits for its predecessor with griddepcontrol.wait before doing anything that
// depends on it).
#include <cstdint>

#include "common.cuh"

namespace b2d {

constexpr int kMaxTp = 8;
constexpr int kSigStride = kMaxTp;  // signal words per slot: one per source rank

struct PeerSet {
  const float* part[kMaxTp];  // each rank's partial [rows, D] (this use's buffer)
  uint32_t* sig[kMaxTp];      // each rank's signal array [slots][kMaxTp]
};

struct PeerGather {
  const float* val[kMaxTp];  // each rank's best logit per token
  const int* idx[kMaxTp];    // and its (global) vocab index
  uint32_t* sig[kMaxTp];
};

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Per-slot barrier among the tp ranks.  Thread r < tp announces this rank to rank r and then
// waits for rank r's announcement.
//  * Writer: the data a rank announces was written by the previous kernel on that rank (its
//    partial in its own memory, or pushed into the peers' receive slots over NVLink).  This
//    kernel stores the flag only after griddepcontrol.wait, which returns once that grid has
//    completed and its memory operations are performed -- the pushed partials have reached the
//    peers' memory before the flag store is even issued.  The flag is therefore a relaxed
//    system-scope store: a release store (or fence) at system scope would add a full
//    system-scope memory barrier per flag, which measured 15.6 instead of ~5 us per all-reduce
//    kernel at TP8 on B200s (per-kernel timeline of the graph-replayed step).
//  * Reader: polls with acquire loads at system scope, so nothing after the poll (the sums below,
//    L1-bypassing loads) is performed before the flag value is observed; the CTA barrier that
//    follows carries that order to every thread of the CTA.
// Returns false (CTA-uniform) if some peer did not arrive within timeout_ns; *err then holds
// B2D_ERR_TIMEOUT.
__device__ bool peer_barrier(uint32_t* const* sig, int rank, int tp, int slot, uint32_t* epochs,
                             long long timeout_ns, int* err) {
  __shared__ uint32_t epoch_s;
  if (threadIdx.x == 0) {
    const uint32_t e = epochs[slot] + 1u;
    epochs[slot] = e;
    epoch_s = e;
  }
  __syncthreads();
  const uint32_t e = epoch_s;
  bool ok = true;
  if (threadIdx.x < tp) {
    const int r = threadIdx.x;
    st_relaxed_sys(sig[r] + slot * kSigStride + rank, e);
    const uint32_t* mine = sig[rank] + slot * kSigStride + r;
    if ((int)(ld_acquire_sys(mine) - e) < 0) {
      const uint64_t t0 = global_ns();
      while ((int)(ld_acquire_sys(mine) - e) < 0) {
        if ((long long)(global_ns() - t0) > timeout_ns) {
          ok = false;
          atomicExch(err, B2D_ERR_TIMEOUT);
          break;
        }
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

// x[b] += sum_r part_r[b]; out16[b] = fp16(rmsnorm(x[b]) * gamma) if gamma (else x only).
__global__ void __launch_bounds__(256) tp_allreduce_add_rmsnorm_kernel(
    const __grid_constant__ PeerSet ps, uint32_t* epochs, int rank, int tp, int slot0, float* x,
    const float* gamma, float eps, uint16_t* out16, uint16_t* out_lo, int D,
    long long timeout_ns, int* err) {
  __shared__ float red[8];
  pdl_wait();  // this rank's partial and residual are complete
  const int b = blockIdx.x;
  if (!peer_barrier(ps.sig, rank, tp, slot0 + b, epochs, timeout_ns, err)) return;
  float4* xr = reinterpret_cast<float4*>(x + (size_t)b * D);
  const int n4 = D / 4;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n4; i += blockDim.x) {
    float4 v[kMaxTp];
#pragma unroll
    for (int r = 0; r < kMaxTp; ++r)  // all loads in flight before the sums
      if (r < tp) v[r] = __ldcv(reinterpret_cast<const float4*>(ps.part[r] + (size_t)b * D) + i);
    float4 s = v[0];
#pragma unroll
    for (int r = 1; r < kMaxTp; ++r)
      if (r < tp) {
        s.x += v[r].x;
        s.y += v[r].y;
        s.z += v[r].z;
        s.w += v[r].w;
      }
    float4 xv = xr[i];
    xv.x += s.x;
    xv.y += s.y;
    xv.z += s.z;
    xv.w += s.w;
    xr[i] = xv;
    ss = fmaf(xv.x, xv.x, fmaf(xv.y, xv.y, fmaf(xv.z, xv.z, fmaf(xv.w, xv.w, ss))));
  }
  pdl_launch_dependents();
  if (!gamma) return;
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
  const float scale = rsqrtf(tot / (float)D + eps);
  uint2* orow = reinterpret_cast<uint2*>(out16 + (size_t)b * D);
  uint2* lrow = out_lo ? reinterpret_cast<uint2*>(out_lo + (size_t)b * D) : nullptr;
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  for (int i = threadIdx.x; i < n4; i += blockDim.x) {
    const float4 xv = xr[i], g = g4[i];
    uint2 lo;
    orow[i] = split4_f16(xv.x * scale * g.x, xv.y * scale * g.y, xv.z * scale * g.z,
                         xv.w * scale * g.w, &lo);
    if (lrow) lrow[i] = lo;  // B2D_F16X2 lo plane
  }
}

// tokens[b] = index of the best (value, index) over the ranks' candidates (ties -> lowest).
__global__ void __launch_bounds__(128) tp_argmax_gather_kernel(
    const __grid_constant__ PeerGather pg, uint32_t* epochs, int rank, int tp, int slot, int B,
    int* tokens, long long timeout_ns, int* err) {
  pdl_wait();
  if (!peer_barrier(pg.sig, rank, tp, slot, epochs, timeout_ns, err)) return;
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    float bv = __ldcv(pg.val[0] + b);
    int bi = __ldcv(pg.idx[0] + b);
    for (int r = 1; r < tp; ++r) {
      const float v = __ldcv(pg.val[r] + b);
      const int i = __ldcv(pg.idx[r] + b);
      if (better(v, i, bv, bi)) {
        bv = v;
        bi = i;
      }
    }
    tokens[b] = bi;
  }
  pdl_launch_dependents();
}

int tp_allreduce_add_rmsnorm(const float* const* parts, uint32_t* const* sigs, uint32_t* epochs,
                             int rank, int tp, int slot0, float* x, const float* gamma,
                             float eps, uint16_t* out16, uint16_t* out_lo, int D, int rows,
                             long long timeout_ns, int* err, cudaStream_t stream) {
  if (!parts || !sigs || !epochs || !x || !err) return B2D_ERR_NULL;
  if (tp < 1 || tp > kMaxTp || rank < 0 || rank >= tp || rows <= 0 || D <= 0 || D % 4 ||
      slot0 < 0 || timeout_ns <= 0)
    return B2D_ERR_SHAPE;
  if (gamma && !out16) return B2D_ERR_NULL;
  PeerSet ps = {};
  for (int r = 0; r < tp; ++r) {
    if (!parts[r] || !sigs[r]) return B2D_ERR_NULL;
    if (!aligned16(parts[r]) || (reinterpret_cast<uintptr_t>(sigs[r]) & 3)) return B2D_ERR_ALIGN;
    ps.part[r] = parts[r];
    ps.sig[r] = sigs[r];
  }
  if (!aligned16(x) ||
      (gamma && (!aligned16(gamma) ||
                 ((reinterpret_cast<uintptr_t>(out16) | reinterpret_cast<uintptr_t>(out_lo)) & 7))))
    return B2D_ERR_ALIGN;
  return launch_pdl(tp_allreduce_add_rmsnorm_kernel, dim3(rows), dim3(256), 0, stream, ps,
                    epochs, rank, tp, slot0, x, gamma, eps, out16, out_lo, D, timeout_ns, err);
}

int tp_argmax_gather(const float* const* vals, const int* const* idxs, uint32_t* const* sigs,
                     uint32_t* epochs, int rank, int tp, int slot, int B, int* tokens,
                     long long timeout_ns, int* err, cudaStream_t stream) {
  if (!vals || !idxs || !sigs || !epochs || !tokens || !err) return B2D_ERR_NULL;
  if (tp < 1 || tp > kMaxTp || rank < 0 || rank >= tp || B <= 0 || slot < 0 || timeout_ns <= 0)
    return B2D_ERR_SHAPE;
  PeerGather pg = {};
  for (int r = 0; r < tp; ++r) {
    if (!vals[r] || !idxs[r] || !sigs[r]) return B2D_ERR_NULL;
    pg.val[r] = vals[r];
    pg.idx[r] = idxs[r];
    pg.sig[r] = sigs[r];
  }
  return launch_pdl(tp_argmax_gather_kernel, dim3(1), dim3(128), 0, stream, pg, epochs, rank, tp,
                    slot, B, tokens, timeout_ns, err);
}

}  // namespace b2d
