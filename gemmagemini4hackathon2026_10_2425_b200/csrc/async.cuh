// mbarrier, bulk-copy and TMA helpers shared by the asynchronous-copy kernels (sm_100a).
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace b2d {

// Bounded waits: ~2 s at 1.9 GHz before a wait gives up and reports an error.
constexpr long long kAsyncWaitCycles = 4000000000LL;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

// Bounded wait: false (and the error word set) if the phase did not complete in time.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase, int* err, int code) {
  if (mbar_try_wait(bar, phase)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, phase)) {
    if (clock64() - t0 > kAsyncWaitCycles) {
      atomicCAS(err, 0, code);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int c0, int c1,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// L2 policy for data that is read once per step (weights, KV pages): evict it first, so the
// streams do not push the step's small hot data out of L2 (activations, partial sums, block
// tables -- and the kernels' own code, which every SM otherwise re-fetches from HBM).
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t pol;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* tm, int c0, int c1,
                                                 uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void bulk_load_hint(void* dst, const void* src, uint32_t bytes,
                                               uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// 1D bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16), completing
// bytes on an mbarrier.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Prefetch of [src, src + bytes) into L2 (no shared memory, no completion to wait for): the
// next kernel's weights, pulled from HBM while this kernel's own stream winds down.  src 16-byte
// aligned, bytes a multiple of 16.
__device__ __forceinline__ void l2_prefetch_bulk(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)),
               "r"(bytes)
               : "memory");
}

// This CTA's share of an L2 prefetch of [base, base + bytes): the range is cut into 16-byte
// aligned slices, one per CTA of the grid, issued in pieces of at most 64 KB.
__device__ __forceinline__ void l2_prefetch_share(const void* base, size_t bytes) {
  if (!base || bytes < 16) return;
  const size_t ctas = (size_t)gridDim.x * gridDim.y * gridDim.z;
  const size_t cta = ((size_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
  const size_t per = ((bytes / ctas) + 15) & ~size_t(15);
  const size_t lo = cta * per, hi = lo + per < bytes ? lo + per : bytes;
  const char* b = static_cast<const char*>(base);
  for (size_t o = lo; o + 16 <= hi; o += 65536) {
    const size_t n = (hi - o < 65536 ? hi - o : 65536) & ~size_t(15);
    if (n) l2_prefetch_bulk(b + o, (uint32_t)n);
  }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

}  // namespace b2d
