// Allocation-free variant of the paged decode attention entry point.
//
// Some callers cannot allocate device memory at all: code that runs inside another
// framework's memory pool or under a strict allocator (a serving process that has handed all
// free HBM to its cache allocator), plugins loaded into a host that forbids cudaMalloc after
// start-up, and processes that must not allocate while other work is being captured.  For
// them, b2d_paged_decode_attn_noalloc takes no workspace argument: its split-K scratch lives
// in a fixed file-scope device array of kNoAllocScratchBytes, which every GPU that loads this
// library holds until the process exits.
//
// The array's name, used in host code, is only a host-side stand-in for the symbol, not a
// device address.  So on the first call on each device, with that device current, this file
// looks up the device address once with cudaGetSymbolAddress and caches it; kernels then get
// that address.  Make that first call before any stream capture on the device.  A __device__
// array starts zero-filled when the module loads, and nothing here fills it in bulk: before
// every launch the call clears the scratch's header (error word and arrival counters) with a
// cudaMemsetAsync on the caller's own stream, so the clear is ordered with the kernel whatever
// kind of stream the caller uses; the partials behind the header are always written before
// they are read.  Every call shares the one array: calls whose kernels overlap on the GPU
// (different streams running concurrently on the same device) race on the scratch and must be
// serialized by the caller.  A bounded device-side wait that gives up leaves a non-zero error
// word, which b2d_paged_decode_attn_noalloc_error reports until the next call clears it.
#include <mutex>

#include "common.cuh"

namespace b2d {
size_t paged_attn_workspace_bytes(int, int, int, int, int);
size_t attn_ws_header_bytes(int batch, int n_kv_heads);
int paged_decode_attn(void*, int, int, uint16_t*, uint16_t*, const int*, int, int, const int*,
                      const float*, int, int, int, int, int, float, int, int, void*, int, int,
                      void*, size_t, cudaStream_t);
}  // namespace b2d

using namespace b2d;

// 16 MiB: enough for 64 sequences x 8 KV heads x 8192-token contexts at head_dim 128.
static constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) unsigned char g_noalloc_attn_scratch[kNoAllocScratchBytes];

static constexpr int kMaxDevices = 64;
static void* g_scratch_ptr[kMaxDevices] = {};
static std::mutex g_scratch_mu;

// Device address of the scratch array on the current device (looked up on first use).
static int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return B2D_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) return B2D_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_attn_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_cuda_error(e == cudaSuccess ? cudaErrorInvalidSymbol : e);
      return B2D_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return B2D_OK;
}

extern "C" {

size_t b2d_paged_decode_attn_noalloc_max_scratch_bytes(void) { return kNoAllocScratchBytes; }

int b2d_paged_decode_attn_noalloc(void* qkv, int qkv_dtype, int ldqkv, uint16_t* k_pages,
                                  uint16_t* v_pages, const int* block_table, int max_blocks,
                                  int n_blocks, const int* ctx_lens, const float* inv_freq,
                                  int n_heads, int n_kv_heads, int head_dim, int batch,
                                  int max_ctx, float scale, int window, int append, void* out,
                                  int out_dtype, int ldout, b2d_stream_t stream) {
  if (batch <= 0 || n_heads <= 0 || n_kv_heads <= 0 || max_ctx <= 0) return B2D_ERR_SHAPE;
  const size_t need = paged_attn_workspace_bytes(batch, n_heads, n_kv_heads, head_dim, max_ctx);
  if (need == 0) return B2D_ERR_SHAPE;
  if (need > kNoAllocScratchBytes) return B2D_ERR_WORKSPACE;  // beyond the fixed scratch
  void* scratch = nullptr;
  B2D_TRY(scratch_for_current_device(&scratch));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // the arrival counters and the error word (the scratch's header) must start at zero
  const size_t counter_bytes = attn_ws_header_bytes(batch, n_kv_heads);
  cudaError_t e = cudaMemsetAsync(scratch, 0, counter_bytes, s);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return B2D_ERR_CUDA;
  }
  return paged_decode_attn(qkv, qkv_dtype, ldqkv, k_pages, v_pages, block_table, max_blocks,
                           n_blocks, ctx_lens, inv_freq, n_heads, n_kv_heads, head_dim, batch,
                           max_ctx, scale, window, append, out, out_dtype, ldout, scratch,
                           kNoAllocScratchBytes, s);
}

int b2d_paged_decode_attn_noalloc_error(void) {
  void* scratch = nullptr;
  B2D_TRY(scratch_for_current_device(&scratch));
  // the last call may run on any stream of this device: wait for all of them
  cudaError_t e = cudaDeviceSynchronize();
  int word = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&word, scratch, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return B2D_ERR_CUDA;
  }
  return word ? B2D_ERR_TIMEOUT : B2D_OK;
}

}  // extern "C"
