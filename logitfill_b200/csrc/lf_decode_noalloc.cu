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
// address, so the address is looked up with cudaGetSymbolAddress, with the
// device current, the first time a call runs in a CUDA context, and cached
// per context: a context created later (cudaDeviceReset, a driver-API
// context made current by the host) loads the module again, possibly at
// another address, and gets its own lookup.  Make the first call in each
// context before any stream capture.  All calls share the array: two calls
// whose kernels overlap on the GPU (different streams, or different host
// threads without ordering) race on it and must be serialised by the caller.
// Nothing in the array needs to start at zero: every partial the merge reads
// is written earlier in the same call, so the contents left by the previous
// call are never read.
#include <cuda.h>

#include <mutex>

#include "lf_common.cuh"

namespace lf {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

struct NoAllocSlot {
  unsigned long long ctx_id;  // unique over the process lifetime; 0 = empty
  float* ptr;
};

static std::mutex g_noalloc_mutex;
static NoAllocSlot g_noalloc_slot[kMaxDevices] = {};
static CtxGetCurrentFn g_ctx_get_current = nullptr;
static CtxGetIdFn g_ctx_get_id = nullptr;

// Driver entry points through the runtime (the library does not link libcuda).
static int driver_entry_points() {
  if (g_ctx_get_current != nullptr && g_ctx_get_id != nullptr) return LF_OK;
  void* cur = nullptr;
  void* id = nullptr;
  cudaDriverEntryPointQueryResult q1 = cudaDriverEntryPointSymbolNotFound, q2 = cudaDriverEntryPointSymbolNotFound;
  if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &cur, cudaEnableDefault, &q1) != cudaSuccess ||
      cudaGetDriverEntryPoint("cuCtxGetId", &id, cudaEnableDefault, &q2) != cudaSuccess ||
      q1 != cudaDriverEntryPointSuccess || q2 != cudaDriverEntryPointSuccess || cur == nullptr || id == nullptr) {
    cudaGetLastError();
    set_error("lf_decode_noalloc: driver entry points cuCtxGetCurrent / cuCtxGetId unavailable");
    return LF_ERR_LAUNCH;
  }
  g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(cur);
  g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(id);
  return LF_OK;
}

// Device address of the scratch array in the current context (looked up once
// per context, with its device current).
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
  int st = driver_entry_points();
  if (st != LF_OK) return st;
  auto lookup = [](void** ptr) -> int {
    const cudaError_t err = cudaGetSymbolAddress(ptr, g_noalloc_scratch);
    if (err != cudaSuccess || *ptr == nullptr) {
      cudaGetLastError();
      set_error("lf_decode_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(err));
      return LF_ERR_LAUNCH;
    }
    return LF_OK;
  };
  CUcontext ctx = nullptr;
  void* fresh = nullptr;
  if (g_ctx_get_current(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  if (ctx == nullptr) {
    // No context on this thread yet: the runtime binds the device's primary
    // context on the lookup, which is then this context's.
    st = lookup(&fresh);
    if (st != LF_OK) return st;
    if (g_ctx_get_current(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  }
  unsigned long long ctx_id = 0;
  if (ctx == nullptr || g_ctx_get_id(ctx, &ctx_id) != CUDA_SUCCESS || ctx_id == 0) {
    set_error("lf_decode_noalloc: cannot identify the current CUDA context");
    return LF_ERR_LAUNCH;
  }
  NoAllocSlot& slot = g_noalloc_slot[dev];
  if (slot.ctx_id != ctx_id || slot.ptr == nullptr) {
    if (fresh == nullptr) {
      st = lookup(&fresh);
      if (st != LF_OK) return st;
    }
    slot.ctx_id = ctx_id;
    slot.ptr = static_cast<float*>(fresh);
  }
  *out = slot.ptr;
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
  // Output checks before anything is launched (lf_decode repeats them).
  LF_CHECK_ARG(out != nullptr, "lf_decode_noalloc: null output");
  LF_CHECK_ARG(out_dtype == LF_F32 || out_dtype == LF_F16 || out_dtype == LF_BF16,
               "lf_decode_noalloc: out dtype %d", out_dtype);
  LF_CHECK_ARG(layout->head_dim % 2 == 0, "lf_decode_noalloc: head_dim %d must be even", layout->head_dim);
  const size_t need = lf_decode_workspace_bytes(batch, layout->kv_heads, n_q, layout->head_dim, max_splits);
  LF_CHECK_ARG(need > 0, "lf_decode_noalloc: batch %d, n_q %d, max_splits %d give no partials", batch, n_q,
               max_splits);
  LF_CHECK_ARG(need <= lf::kNoAllocScratchBytes,
               "lf_decode_noalloc: %zu bytes of split partials (batch %d x %d KV heads x %d splits) exceed the "
               "fixed %zu-byte scratch; use lf_decode_partial/lf_decode_merge with a caller workspace",
               need, batch, layout->kv_heads, max_splits, lf::kNoAllocScratchBytes);
  float* scratch = nullptr;
  const int st = lf::noalloc_scratch(&scratch);
  if (st != LF_OK) return st;
  // lf_decode validates every input before it launches K2, then launches K3.
  return lf_decode(layout, rows, kmeta, slot_chan, hist_tokens, tail_k, tail_v, tail_seq_stride, tail_head_stride,
                   tail_len, resid_dtype, k_new, v_new, new_seq_stride, new_head_stride, q, q_dtype, q_seq_stride,
                   q_head_stride, batch, n_q, scaling, pages_per_split, max_splits, scratch, out, out_dtype,
                   out_seq_stride, out_head_stride, status, stream);
}
