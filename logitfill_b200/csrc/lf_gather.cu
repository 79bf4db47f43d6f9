// KV-head sharding over NVLink: the split merge (K3) fused with the output
// all-gather.  Rank r of N holds KV heads [r H/N, (r+1) H/N) and their q-heads;
// every layer's output [B, n_q/N, D] must reach every rank as block r of the
// gathered buffer [N, B, n_q/N, D] (the head-sharded layout the reference
// expands with repeat_kv, reference.py:10-15).
//
// lf_decode_merge_gather computes the merge exactly as lf_decode_merge and
// stores each output row into the gathered buffer of every rank (peer memory
// opened with CUDA IPC, plain stores over NVLink, no multicast).  Each CTA then
// makes its stores visible system-wide and adds 1 to the layer's counter on
// every rank (a release add at system scope).  lf_gather_wait, on the consumer
// rank, polls its own counter until all N ranks' CTAs have signalled, bounded
// by a time limit, and takes the count back so the counter serves the next
// step.  No kernel waits on another kernel of its own GPU.
#include <cstring>

#include "lf_common.cuh"
#include "lf_decode_common.cuh"

namespace lf {

constexpr int kGatherWarps = 4;
constexpr int kMaxRanks = 8;

__device__ __forceinline__ void red_release_sys_add(uint32_t* addr, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Output of one (sequence, q-head) of this rank, one warp: the merge of
// decode_merge_kernel (lf_decode.cu) for one query token and one head chunk
// per KV head, then the row stored into every rank's gathered block `rank`.
template <typename OT>
__global__ void __launch_bounds__(kGatherWarps * 32)
merge_gather_kernel(const float* __restrict__ ws, const int32_t* __restrict__ hist_tokens, int batch,
                    int kv_heads, int n_q, int D, int P, int pps, int max_splits, const uint64_t* peer_out,
                    const uint64_t* peer_flags, int layer, int rank, int world) {
  const int lane = threadIdx.x & 31;
  const int task = blockIdx.x * kGatherWarps + (threadIdx.x >> 5);
  grid_dep_wait();
  grid_dep_trigger();
  if (task < batch * n_q) {
    const int b = task / n_q, qh = task - b * n_q;
    const int gq = n_q / kv_heads, h = qh / gq, jj = qh - h * gq;
    const int pages = hist_tokens[b] / P;
    const int n_s = min((pages + pps - 1) / pps + residual_splits(P, 1), max_splits);
    const int64_t item = static_cast<int64_t>(gq) * (D + 2);
    const float* base = ws + (static_cast<int64_t>(b) * kv_heads + h) * max_splits * item;
    const float* mstat = base + static_cast<int64_t>(gq) * D + jj;
    const float* vals = base + static_cast<int64_t>(jj) * D;
    const int d0 = 2 * lane, d1 = 2 * lane + 64;
    float M = -INFINITY;
    for (int s = lane; s < n_s; s += 32) M = fmaxf(M, mstat[s * item]);
#pragma unroll
    for (int sh = 16; sh > 0; sh >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, sh));
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f, Lsum = 0.f;
    for (int s0 = 0; s0 < n_s; s0 += 32) {
      float wl = 0.f;
      if (s0 + lane < n_s) {
        const float ms = mstat[(s0 + lane) * item];
        if (ms != -INFINITY) {
          wl = expf(ms - M);
          Lsum = fmaf(wl, mstat[(s0 + lane) * item + gq], Lsum);
        }
      }
      const int cnt = min(32, n_s - s0);
      for (int k = 0; k < cnt; ++k) {
        const float w = __shfl_sync(0xffffffffu, wl, k);
        const float* row = vals + static_cast<int64_t>(s0 + k) * item;
        if (d0 < D) {
          const float2 v = *reinterpret_cast<const float2*>(row + d0);
          fma2_acc(w, v, a0, a1);
        }
        if (d1 < D) {
          const float2 v = *reinterpret_cast<const float2*>(row + d1);
          fma2_acc(w, v, a2, a3);
        }
      }
    }
#pragma unroll
    for (int sh = 16; sh > 0; sh >>= 1) Lsum += __shfl_xor_sync(0xffffffffu, Lsum, sh);
    const float inv = Lsum > 0.f ? 1.0f / Lsum : 0.f;
    // Block `rank` of layer `layer` in every rank's gathered buffer
    // [layers][world][batch][n_q][D].
    const int64_t off = ((static_cast<int64_t>(layer) * world + rank) * batch + b) * n_q * D +
                        static_cast<int64_t>(qh) * D;
    for (int r = 0; r < world; ++r) {
      OT* o = reinterpret_cast<OT*>(peer_out[r]) + off;
      if (d0 < D) {
        Scalar<OT>::store(o + d0, a0 * inv);
        Scalar<OT>::store(o + d0 + 1, a1 * inv);
      }
      if (d1 < D) {
        Scalar<OT>::store(o + d1, a2 * inv);
        Scalar<OT>::store(o + d1 + 1, a3 * inv);
      }
    }
  }
  // Every thread's stores become visible system-wide before the CTA's
  // signal (the barrier orders them before the release add).
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < world)
    red_release_sys_add(reinterpret_cast<uint32_t*>(peer_flags[threadIdx.x]) + layer, 1u);
}

// One thread: wait until `expected` signals reached counter `layer`, then
// take them back.  Gives up after limit_ns, recording LF_ERR_DEVICE_TIMEOUT.
__global__ void gather_wait_kernel(uint32_t* flags, int layer, uint32_t expected, uint64_t limit_ns, int* status) {
  uint32_t* f = flags + layer;
  const uint64_t t0 = global_ns();
  for (uint32_t n = 0;; ++n) {
    if (ld_acquire_sys(f) >= expected) break;
    if ((n & 255u) == 255u && global_ns() - t0 > limit_ns) {
      if (status != nullptr) atomicExch(status, LF_ERR_DEVICE_TIMEOUT);
      return;
    }
  }
  atomicSub(f, expected);
}

}  // namespace lf

// ------------------------------------------------------------------ C ABI --
extern "C" int lf_ipc_alloc(size_t bytes, void** ptr) {
  LF_CHECK_ARG(ptr != nullptr && bytes > 0, "lf_ipc_alloc: null pointer or zero size");
  *ptr = nullptr;
  const cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) {
    lf::set_error("lf_ipc_alloc: %zu B: %s", bytes, cudaGetErrorString(e));
    return LF_ERR_CUDA;
  }
  const cudaError_t z = cudaMemset(*ptr, 0, bytes);
  if (z != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    lf::set_error("lf_ipc_alloc: clearing %zu B: %s", bytes, cudaGetErrorString(z));
    return LF_ERR_CUDA;
  }
  return LF_OK;
}

extern "C" int lf_ipc_free(void* ptr) {
  if (ptr == nullptr) return LF_OK;
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) {
    lf::set_error("lf_ipc_free: %s", cudaGetErrorString(e));
    return LF_ERR_CUDA;
  }
  return LF_OK;
}

extern "C" int lf_ipc_handle(const void* ptr, void* handle) {
  LF_CHECK_ARG(ptr != nullptr && handle != nullptr, "lf_ipc_handle: null pointer");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) {
    lf::set_error("lf_ipc_handle: %s", cudaGetErrorString(e));
    return LF_ERR_CUDA;
  }
  memcpy(handle, &h, sizeof(h));
  return LF_OK;
}

extern "C" int lf_ipc_open(const void* handle, void** ptr) {
  LF_CHECK_ARG(ptr != nullptr && handle != nullptr, "lf_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    lf::set_error("lf_ipc_open: %s", cudaGetErrorString(e));
    return LF_ERR_CUDA;
  }
  return LF_OK;
}

extern "C" int lf_ipc_close(void* ptr) {
  if (ptr == nullptr) return LF_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) {
    lf::set_error("lf_ipc_close: %s", cudaGetErrorString(e));
    return LF_ERR_CUDA;
  }
  return LF_OK;
}

extern "C" int lf_decode_merge_gather(const float* workspace, const int32_t* hist_tokens, int batch, int kv_heads,
                                      int n_q, int head_dim, int page_size, int pages_per_split, int max_splits,
                                      const uint64_t* peer_out, const uint64_t* peer_flags, int layer, int rank,
                                      int world, int out_dtype, lf_stream_t stream) {
  LF_CHECK_ARG(workspace && hist_tokens && peer_out && peer_flags, "lf_decode_merge_gather: null pointer");
  LF_CHECK_ARG(batch > 0 && kv_heads > 0 && n_q > 0 && n_q % kv_heads == 0 && n_q / kv_heads <= lf::kGQ,
               "lf_decode_merge_gather: batch %d n_q %d kv_heads %d", batch, n_q, kv_heads);
  LF_CHECK_ARG(head_dim > 0 && head_dim <= 128 && head_dim % 2 == 0 && page_size > 0 && pages_per_split > 0 &&
                   max_splits > 0,
               "lf_decode_merge_gather: bad sizes");
  LF_CHECK_ARG(world >= 1 && world <= lf::kMaxRanks && rank >= 0 && rank < world && layer >= 0,
               "lf_decode_merge_gather: rank %d of %d, layer %d", rank, world, layer);
  const void* kern = nullptr;
  switch (out_dtype) {
    case LF_F32: kern = reinterpret_cast<const void*>(lf::merge_gather_kernel<float>); break;
    case LF_F16: kern = reinterpret_cast<const void*>(lf::merge_gather_kernel<__half>); break;
    case LF_BF16: kern = reinterpret_cast<const void*>(lf::merge_gather_kernel<__nv_bfloat16>); break;
    default:
      lf::set_error("lf_decode_merge_gather: out dtype %d", out_dtype);
      return LF_ERR_INVALID_ARGUMENT;
  }
  const int64_t tasks = static_cast<int64_t>(batch) * n_q;
  const dim3 grid(static_cast<unsigned>((tasks + lf::kGatherWarps - 1) / lf::kGatherWarps));
  void* args[] = {&workspace, &hist_tokens, &batch, &kv_heads, &n_q, &head_dim, &page_size, &pages_per_split,
                  &max_splits, &peer_out, &peer_flags, &layer, &rank, &world};
  const cudaError_t e = lf::launch_programmatic(kern, grid, dim3(lf::kGatherWarps * 32), 0,
                                                static_cast<cudaStream_t>(stream), args);
  if (e != cudaSuccess) {
    lf::set_error("lf_decode_merge_gather: %s", cudaGetErrorString(e));
    return LF_ERR_LAUNCH;
  }
  return lf::launch_status("lf_decode_merge_gather");
}

extern "C" int lf_gather_signals(int batch, int n_q, int world) {
  if (batch <= 0 || n_q <= 0 || world <= 0) return 0;
  const int64_t tasks = static_cast<int64_t>(batch) * n_q;
  return static_cast<int>((tasks + lf::kGatherWarps - 1) / lf::kGatherWarps) * world;
}

extern "C" int lf_gather_wait(uint32_t* flags, int layer, uint32_t expected, uint64_t limit_ns, int32_t* status,
                              lf_stream_t stream) {
  LF_CHECK_ARG(flags != nullptr && layer >= 0 && expected > 0, "lf_gather_wait: bad arguments");
  lf::gather_wait_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(flags, layer, expected, limit_ns, status);
  return lf::launch_status("lf_gather_wait");
}
