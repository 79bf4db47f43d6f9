// Host side of the C ABI: history layout, status text, error capture.
#include <stdarg.h>
#include <stdio.h>

#include <map>
#include <mutex>
#include <utility>

#include "lf_common.cuh"

namespace lf {

static thread_local char g_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

cudaError_t raise_smem_limit(const void* kern, int bytes, bool max_carveout) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> limit;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  int& cur = limit[std::make_pair(kern, dev)];
  if (bytes <= cur) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && max_carveout)
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess) cur = bytes;
  return e;
}

cudaError_t launch_programmatic(const void* kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                void** args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, kern, args);
}

int launch_status(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(err));
    return LF_ERR_LAUNCH;
  }
  return LF_OK;
}

}  // namespace lf

static int round_up(int x, int m) { return (x + m - 1) / m * m; }

extern "C" int lf_layout_init(lf_layout* out, int kv_heads, int head_dim, int page_size,
                              int k_group, int v_group, int bit_v, const int32_t* tier_counts,
                              int64_t row_cap, int64_t group_cap) {
  LF_CHECK_ARG(out != nullptr && tier_counts != nullptr, "lf_layout_init: null pointer");
  LF_CHECK_ARG(kv_heads > 0 && head_dim > 0 && page_size > 0 && k_group > 0 && v_group > 0,
               "lf_layout_init: sizes must be positive");
  LF_CHECK_ARG(page_size % k_group == 0, "page_size %d is not a multiple of k_group %d", page_size,
               k_group);
  LF_CHECK_ARG(head_dim % v_group == 0, "head_dim %d is not divisible by v_group %d", head_dim,
               v_group);
  LF_CHECK_SUPPORTED(bit_v == 2 || bit_v == 4 || bit_v == 8, "bit_v %d is not packed (2, 4, 8)",
                     bit_v);
  LF_CHECK_ARG(row_cap >= 0 && row_cap % page_size == 0,
               "row_cap %lld is not a non-negative multiple of page_size", (long long)row_cap);
  LF_CHECK_ARG(group_cap >= row_cap / k_group, "group_cap %lld < row_cap / k_group",
               (long long)group_cap);
  lf_layout L{};
  L.kv_heads = kv_heads;
  L.head_dim = head_dim;
  L.page_size = page_size;
  L.k_group = k_group;
  L.v_group = v_group;
  L.bit_v = bit_v;
  for (int t = 0; t < 4; ++t) {
    int w = 0;
    for (int h = 0; h < kv_heads; ++h) {
      const int c = tier_counts[t * kv_heads + h];
      LF_CHECK_ARG(c >= 0 && c <= head_dim, "tier %d count %d out of range", t, c);
      w = c > w ? c : w;
    }
    L.width[t] = w;
  }
  int sum = 0;
  for (int h = 0; h < kv_heads; ++h) {
    int s = 0;
    for (int t = 0; t < 4; ++t) s += tier_counts[t * kv_heads + h];
    LF_CHECK_ARG(s == head_dim, "head %d tier counts sum to %d, not head_dim %d", h, s, head_dim);
    sum += s;
  }
  (void)sum;
  const int bits[3] = {2, 4, 8};
  int off = 0;
  for (int t = 0; t < 3; ++t) {
    const int per = 32 / bits[t];
    L.words[t] = (L.width[t] + per - 1) / per;  // layout.py:82
    L.code_off[t] = off;
    off += L.words[t];
  }
  L.vcode_off = off;
  const int vper = 32 / bit_v;
  L.vcode_words = (head_dim + vper - 1) / vper;  // pack_ints pads to a whole word
  off += L.vcode_words;
  L.half_off = off;
  const int halves = L.width[3] + 2 * (head_dim / v_group);
  off += (halves + 1) / 2;
  // Odd row length: the 32 rows a warp reads at one word offset fall in 32
  // different shared-memory banks.  A page block (page_size rows) stays a
  // multiple of 16 bytes for the 1-D bulk copies.
  L.row_words = off | 1;
  int hoff = 0;
  for (int t = 0; t < 3; ++t) {
    L.scale_off[t] = hoff;
    hoff += L.width[t];
    L.min_off[t] = hoff;
    hoff += L.width[t];
  }
  // The Key group's largest tier scale (written by lf_pack_pages): the
  // decoder's fixed-point exponent for the page, readable without a reduction.
  L.kmax_off = hoff;
  hoff += 1;
  L.meta_halves = round_up(hoff, 8);
  L.row_cap = row_cap;
  L.group_cap = group_cap;
  *out = L;
  return LF_OK;
}

extern "C" const char* lf_status_string(int status) {
  switch (status) {
    case LF_OK: return "ok";
    case LF_ERR_INVALID_ARGUMENT: return "invalid argument";
    case LF_ERR_UNSUPPORTED: return "unsupported geometry";
    case LF_ERR_LAUNCH: return "CUDA launch failed";
    case LF_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case LF_ERR_OUT_OF_RANGE: return "device-side bounds check rejected a job";
    case LF_ERR_CUDA: return "CUDA runtime call failed";
    default: return "unknown status";
  }
}

extern "C" const char* lf_last_error(void) { return lf::g_error; }
