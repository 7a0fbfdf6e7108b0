// Shared device helpers and host-side status plumbing for the decode-step library.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/b200dec.h"

namespace b2d {

// ------------------------------------------------------------------------------------------
// host: status handling
// ------------------------------------------------------------------------------------------
void set_cuda_error(cudaError_t e);

// Kernel launches this library has enqueued on the calling thread (captured ones included).
void count_launch(int n = 1);

// Checks the launch that was just issued; returns B2D_OK or B2D_ERR_CUDA.
inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return B2D_ERR_CUDA;
  }
  count_launch();
  return B2D_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int num_sms();  // cached per device

#define B2D_TRY(expr)              \
  do {                             \
    int _st = (expr);              \
    if (_st != B2D_OK) return _st; \
  } while (0)

// ------------------------------------------------------------------------------------------
// device: loads
// ------------------------------------------------------------------------------------------

// 16-byte streaming load of read-only data, not kept in L1 (weights, KV pages).
// Streaming 16-byte load of data read once per step (weights): no L1 allocation, and evicted
// from L2 first so it does not displace the step's small hot data.
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint64_t pol;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}

__device__ __forceinline__ float2 h2f2(uint32_t u) {
  __half2 h = *reinterpret_cast<__half2*>(&u);
  return __half22float2(h);
}

__device__ __forceinline__ float h2f(uint16_t u) { return __half2float(__ushort_as_half(u)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// Four fp32 values as fp16 hi + lo planes (B2D_F16X2): hi = fp16(v), lo = fp16(v - hi).
// Returns the hi plane's 8 bytes; the lo plane's go to *lo.
__device__ __forceinline__ uint2 split4_f16(float a, float b, float c, float d, uint2* lo) {
  const __half2 h01 = __floats2half2_rn(a, b), h23 = __floats2half2_rn(c, d);
  const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
  const __half2 l01 = __floats2half2_rn(a - f01.x, b - f01.y);
  const __half2 l23 = __floats2half2_rn(c - f23.x, d - f23.y);
  *lo = make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
  return make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
}

// Store v as fp16 at out[i] and, if out_lo, its remainder fp16(v - hi) at out_lo[i].
__device__ __forceinline__ void store_f16_split(uint16_t* out, uint16_t* out_lo, size_t i, float v) {
  const uint16_t hi = f2h(v);
  out[i] = hi;
  if (out_lo) out_lo[i] = f2h(v - h2f(hi));
}

// Signed bytes -> floats without I2F: place byte^0x80 under the exponent of 2^23 and subtract
// (2^23 + 128).  Exact for every int8 value.
__device__ __forceinline__ float byte_to_float(uint32_t biased_word, int i) {
  // biased_word already holds (word ^ 0x80808080); byte i goes to the low 8 bits
  uint32_t f = __byte_perm(biased_word, 0x4B000000u, 0x7650 + i) ;
  return __uint_as_float(f) - 8388736.0f;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// (value, index) max with ties to the lowest index (LK/kernels.metal:326).
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, v, o);
    int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (better(ov, oi, v, i)) {
      v = ov;
      i = oi;
    }
  }
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

__device__ __forceinline__ float gelu_tanh(float x) {
  return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}

// Programmatic dependent launch: wait for the preceding kernel's writes / let the next kernel
// start its prologue.  Both are no-ops when the launch did not opt in.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;");
}

// Launch with programmatic dependent launch allowed (the kernel must call pdl_wait() before it
// touches data written by the previous kernel on the stream).
template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                      cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return B2D_ERR_CUDA;
  }
  count_launch();
  return B2D_OK;
}

// RMSNorm folded into a tensor-core GEMM pair (tc_gemm_norm): a residual-add producer emits
// the un-normalized operand and per-slice sums of squares, its consumer scales its product by
// the norm factor.  Producer fields (gamma set): gamma of the next norm [M], planes (hi / lo
// fp16 of y * gamma * e[t], lo at + batch * ldy), part_out ([32][M / 16] slice sums, then
// e[32]), r_prev (the last norm factor per token, for e[t]; nullptr: e = 1).  Consumer fields
// (part_in set): a producer's part_out, r_out (the norm factor per token, optional), eps.
struct TcNorm {
  const float* gamma = nullptr;
  uint16_t* planes = nullptr;
  float* part_out = nullptr;
  const float* r_prev = nullptr;
  const float* part_in = nullptr;
  float* r_out = nullptr;
  float eps = 0.f;
};

// Floats of one TcNorm slice-sum block for M rows: [32][M / 16] sums, then e[32].
inline size_t tc_norm_part_floats(int M) { return (size_t)32 * (M / 16) + 32; }

}  // namespace b2d
