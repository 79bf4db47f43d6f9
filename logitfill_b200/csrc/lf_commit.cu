// Device-side commit of one decode token per sequence, so that a whole decode
// step (attention, then commit) can be captured in a CUDA graph and replayed:
// every position is read from the device lengths, none from the host.
//
// The order of the reference's page-delayed store (cache.py:48-62, one
// token): append the token to the original-dtype residual page; when the page
// is full, quantize and pack it into the next history slot (K1) and start an
// empty residual page.  Three launches on the caller's stream:
//   1. append: the token's Key/Value rows at tail_len[b]; the job row for K1
//      (the full page, or an empty job when the page is not full yet);
//   2. K1 over the job rows (empty jobs return at once);
//   3. lengths: tail_len[b] + 1, or 0 with hist_tokens[b] + page_size.

#include "lf_common.cuh"

namespace lf {

constexpr int kCommitInvalid = -2;  // job row of a sequence whose lengths were out of range

// Launches K1 (lf_pack.cu) on device-built job rows.
int launch_pack_rows(const lf_layout& L, const void* k, const void* v, int dtype, int64_t s_seq, int64_t s_head,
                     int64_t s_tok, const int32_t* jobs, int n_jobs, int dst_batch, const int32_t* chan_code,
                     int32_t* rows, uint16_t* kmeta, int32_t* status, cudaStream_t stream);

template <typename T>
__global__ void append_token_kernel(T* tail_k, T* tail_v, int64_t tail_seq, int64_t tail_head, const T* k_new,
                                    const T* v_new, int64_t new_seq, int64_t new_head, const int32_t* hist,
                                    const int32_t* tail, int H, int D, int P, int64_t row_cap, int32_t* jobs,
                                    int32_t* status) {
  const int b = blockIdx.x;
  const int t = tail[b];
  if (t < 0 || t >= P) {  // lengths out of range: touch nothing, advance nothing
    if (threadIdx.x == 0) {
      jobs[4 * b] = kCommitInvalid;
      if (status != nullptr) atomicExch(status, LF_ERR_OUT_OF_RANGE);
    }
    return;
  }
  for (int i = threadIdx.x; i < H * D; i += blockDim.x) {
    const int h = i / D, d = i - h * D;
    tail_k[b * tail_seq + h * tail_head + static_cast<int64_t>(t) * D + d] = k_new[b * new_seq + h * new_head + d];
    tail_v[b * tail_seq + h * tail_head + static_cast<int64_t>(t) * D + d] = v_new[b * new_seq + h * new_head + d];
  }
  if (threadIdx.x == 0) {
    const bool full = t + 1 == P;
    const bool fits = hist[b] + P <= row_cap;
    if (full && !fits && status != nullptr) atomicExch(status, LF_ERR_OUT_OF_RANGE);
    jobs[4 * b + 0] = full && fits ? b : -1;
    jobs[4 * b + 1] = 0;
    jobs[4 * b + 2] = b;
    jobs[4 * b + 3] = full && fits ? hist[b] / P : 0;
  }
}

__global__ void advance_lengths_kernel(int32_t* hist, int32_t* tail, const int32_t* jobs, int batch, int P) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch || jobs[4 * b] == kCommitInvalid) return;
  const int t = tail[b] + 1;
  if (t == P && jobs[4 * b] == b) {
    hist[b] += P;
    tail[b] = 0;
  } else if (t < P) {
    tail[b] = t;
  }
}

}  // namespace lf

extern "C" int lf_commit_token(const lf_layout* layout, int32_t* rows, uint16_t* kmeta, const int32_t* chan_code,
                               void* tail_k, void* tail_v, int64_t tail_seq_stride, int64_t tail_head_stride,
                               int32_t* hist_tokens, int32_t* tail_len, int dtype, const void* k_new,
                               const void* v_new, int64_t new_seq_stride, int64_t new_head_stride, int batch,
                               int32_t* jobs, int32_t* status, lf_stream_t stream) {
  LF_CHECK_ARG(layout != nullptr, "lf_commit_token: null layout");
  const lf_layout& L = *layout;
  LF_CHECK_ARG(rows && chan_code && tail_k && tail_v && hist_tokens && tail_len && k_new && v_new && jobs,
               "lf_commit_token: null pointer");
  LF_CHECK_ARG(L.meta_halves == 0 || kmeta, "lf_commit_token: null kmeta");
  LF_CHECK_ARG(batch > 0 && batch <= 65535, "lf_commit_token: batch %d", batch);
  LF_CHECK_ARG(dtype == LF_F32 || dtype == LF_F16 || dtype == LF_BF16, "lf_commit_token: dtype %d", dtype);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int threads = 256;
  switch (dtype) {
    case LF_F32:
      lf::append_token_kernel<float><<<batch, threads, 0, s>>>(
          static_cast<float*>(tail_k), static_cast<float*>(tail_v), tail_seq_stride, tail_head_stride,
          static_cast<const float*>(k_new), static_cast<const float*>(v_new), new_seq_stride, new_head_stride,
          hist_tokens, tail_len, L.kv_heads, L.head_dim, L.page_size, L.row_cap, jobs, status);
      break;
    case LF_F16:
      lf::append_token_kernel<__half><<<batch, threads, 0, s>>>(
          static_cast<__half*>(tail_k), static_cast<__half*>(tail_v), tail_seq_stride, tail_head_stride,
          static_cast<const __half*>(k_new), static_cast<const __half*>(v_new), new_seq_stride, new_head_stride,
          hist_tokens, tail_len, L.kv_heads, L.head_dim, L.page_size, L.row_cap, jobs, status);
      break;
    default:
      lf::append_token_kernel<__nv_bfloat16><<<batch, threads, 0, s>>>(
          static_cast<__nv_bfloat16*>(tail_k), static_cast<__nv_bfloat16*>(tail_v), tail_seq_stride,
          tail_head_stride, static_cast<const __nv_bfloat16*>(k_new), static_cast<const __nv_bfloat16*>(v_new),
          new_seq_stride, new_head_stride, hist_tokens, tail_len, L.kv_heads, L.head_dim, L.page_size, L.row_cap,
          jobs, status);
  }
  int st = lf::launch_status("lf_commit_token (append)");
  if (st != LF_OK) return st;
  st = lf::launch_pack_rows(L, tail_k, tail_v, dtype, tail_seq_stride, tail_head_stride, L.head_dim, jobs, batch,
                            batch, chan_code, rows, kmeta, status, s);
  if (st != LF_OK) return st;
  lf::advance_lengths_kernel<<<(batch + 127) / 128, 128, 0, s>>>(hist_tokens, tail_len, jobs, batch, L.page_size);
  return lf::launch_status("lf_commit_token (lengths)");
}
