// Decode attention (K2 + K3) for callers that cannot allocate device memory.
//
// lf_decode_partial / lf_decode_merge exchange their split partials through a
// workspace the caller allocates.  Some callers cannot allocate: code running
// where the allocator must not be entered (inside a custom memory pool's own
// callbacks, or a runtime that pre-plans every device allocation up front and
// forbids any later cudaMalloc), or a host that links only this library and
// has no allocator of its own.  lf_decode_noalloc gives them the same
// attention with the partials kept in a fixed array that is part of the
// library's device image instead.
//
// The array is a file-scope __device__ variable of kNoAllocScratchBytes (8 MiB):
// every GPU on which the library's device code is loaded holds it until the
// process exits.  Host code cannot use the variable's name as a device
// address, so the first call on each device (with that device current) looks
// the address up with cudaGetSymbolAddress and caches it; make that first
// call before any stream capture.  All calls share the array: two calls whose
// kernels overlap on the GPU (different streams, or different host threads
// without ordering) race on it and must be serialised by the caller.  Nothing
// in the array needs to start at zero: every partial the merge reads is
// written earlier in the same call, so the contents left by the previous call
// are never read.
#include <mutex>

#include "lf_common.cuh"

namespace lf {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

static std::mutex g_noalloc_mutex;
static float* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once).
static int noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("lf_decode_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    return LF_ERR_LAUNCH;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("lf_decode_noalloc: device %d beyond the %d supported", dev, kMaxDevices);
    return LF_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr) {
      set_error("lf_decode_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return LF_ERR_LAUNCH;
    }
    g_noalloc_ptr[dev] = static_cast<float*>(ptr);
  }
  *out = g_noalloc_ptr[dev];
  return LF_OK;
}

}  // namespace lf

extern "C" int lf_decode_noalloc(const lf_layout* layout, const int32_t* rows, const uint16_t* kmeta,
                                 const int32_t* slot_chan, const int32_t* hist_tokens, const void* tail_k,
                                 const void* tail_v, int64_t tail_seq_stride, int64_t tail_head_stride,
                                 const int32_t* tail_len, int resid_dtype, const void* k_new,
                                 const void* v_new, int64_t new_seq_stride, int64_t new_head_stride,
                                 const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
                                 int batch, int n_q, float scaling, int pages_per_split, int max_splits,
                                 void* out, int out_dtype, int64_t out_seq_stride, int64_t out_head_stride,
                                 int32_t* status, lf_stream_t stream) {
  LF_CHECK_ARG(layout != nullptr, "lf_decode_noalloc: null layout");
  const size_t need = lf_decode_workspace_bytes(batch, layout->kv_heads, n_q, layout->head_dim, max_splits);
  LF_CHECK_ARG(need > 0, "lf_decode_noalloc: batch %d, n_q %d, max_splits %d give no partials", batch, n_q,
               max_splits);
  LF_CHECK_ARG(need <= lf::kNoAllocScratchBytes,
               "lf_decode_noalloc: %zu bytes of split partials (batch %d x %d KV heads x %d splits) exceed the "
               "fixed %zu-byte scratch; use lf_decode_partial/lf_decode_merge with a caller workspace",
               need, batch, layout->kv_heads, max_splits, lf::kNoAllocScratchBytes);
  float* scratch = nullptr;
  int st = lf::noalloc_scratch(&scratch);
  if (st != LF_OK) return st;
  st = lf_decode_partial(layout, rows, kmeta, slot_chan, hist_tokens, tail_k, tail_v, tail_seq_stride,
                         tail_head_stride, tail_len, resid_dtype, k_new, v_new, new_seq_stride, new_head_stride, q,
                         q_dtype, q_seq_stride, q_head_stride, batch, n_q, scaling, pages_per_split, max_splits,
                         scratch, status, stream);
  if (st != LF_OK) return st;
  return lf_decode_merge(scratch, hist_tokens, batch, layout->kv_heads, n_q, layout->head_dim, layout->page_size,
                         pages_per_split, max_splits, out, out_dtype, out_seq_stride, out_head_stride, stream);
}
