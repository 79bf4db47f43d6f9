/*
 * logitfill_b200 -- C ABI of the B200 packed KV-cache hot path.
 *
 * Drop-in replacement for the device side of LogitFill's `packed` backend
 * (GASSFY/Logitfill, src/logitfill/packed/).  Every entry point takes plain
 * device pointers, sizes and a cudaStream_t, allocates nothing, launches on
 * the given stream and returns an lf_status (0 = success).  No torch types.
 *
 * History layout in HBM (one layer):
 *   rows   int32 [batch][kv_heads][row_cap][row_words]   one row per token:
 *            INT2 | INT4 | INT8 Key codes (packed along tier channels, slot 0
 *            in the low bits, as layout.py:21-35 packs them), Value codes
 *            (packed along head_dim), then an fp16 region holding the FP16
 *            Key tier, the Value scales and the Value mins.
 *   kmeta  fp16  [batch][kv_heads][group_cap][meta_halves]  one row per Key
 *            group (k_group tokens): scale and min of every INT2/INT4/INT8
 *            tier channel.
 * Every per-sequence array of the reference (layout.py:71-129, stored as
 * cache.py:64-81 concatenates it) is a strided view of these two buffers, so
 * the reference's shapes and bytes are recovered without copying.
 *
 * Thread safety: entry points are reentrant; kernels on one stream run in
 * order.  Calls that share an output buffer must be ordered by the caller.
 */
#ifndef LOGITFILL_B200_H
#define LOGITFILL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define LF_API __attribute__((visibility("default")))
#else
#define LF_API
#endif

typedef struct CUstream_st* lf_stream_t; /* == cudaStream_t */

enum lf_status {
  LF_OK = 0,
  LF_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, inconsistent layout  */
  LF_ERR_UNSUPPORTED = 2,      /* geometry this build does not implement           */
  LF_ERR_LAUNCH = 3,           /* the CUDA launch failed (see lf_last_error)       */
  LF_ERR_DEVICE_TIMEOUT = 4,   /* a bounded device-side wait gave up               */
  LF_ERR_OUT_OF_RANGE = 5,     /* a device-side bounds check rejected a job        */
  LF_ERR_CUDA = 6              /* a CUDA runtime call failed (see lf_last_error)   */
};

enum lf_dtype { LF_F32 = 0, LF_F16 = 1, LF_BF16 = 2 };

typedef struct lf_layout {
  int32_t kv_heads;     /* H                                                     */
  int32_t head_dim;     /* D                                                     */
  int32_t page_size;    /* tokens per packed page (flush unit)                   */
  int32_t k_group;      /* Key scale/min group along tokens, divides page_size   */
  int32_t v_group;      /* Value scale/min group along channels, divides D       */
  int32_t bit_v;        /* Value code bits                                       */
  int32_t width[4];     /* channels per tier, max over heads: INT2 INT4 INT8 FP16 */
  int32_t words[3];     /* int32 words per token of the INT2 INT4 INT8 codes     */
  int32_t code_off[3];  /* word offset of each tier's codes in a row             */
  int32_t vcode_off;    /* word offset of the Value codes                        */
  int32_t vcode_words;  /* D * bit_v / 32                                        */
  int32_t half_off;     /* word offset of the fp16 region                        */
  int32_t row_words;    /* words per row, odd (bank-conflict-free row reads)     */
  int32_t meta_halves;  /* fp16 per Key-group meta row, multiple of 8            */
  int32_t scale_off[3]; /* fp16 offset of each tier's scales in a meta row       */
  int32_t min_off[3];   /* fp16 offset of each tier's mins in a meta row         */
  int32_t kmax_off;     /* fp16 offset of the group's largest INT2/4/8 Key scale */
  int64_t row_cap;      /* rows reserved per (sequence, head), multiple of page  */
  int64_t group_cap;    /* meta rows reserved per (sequence, head)               */
} lf_layout;

/*
 * Channel tables (device int32, built once per layer from the [H][D] level
 * map of layout.py:49-68):
 *   chan_code [H][D]    (tier << 16) | position of the channel inside its tier
 *   slot_chan [4][H][D] channel held by tier slot i, -1 past the head's count
 */

/* Fill *out from the per-head tier channel counts (host int32 [4][H]:
 * INT2, INT4, INT8, FP16).  Replaces the width bookkeeping of
 * layout.py:57,82-85 and the concatenation layout of cache.py:64-81. */
LF_API int lf_layout_init(lf_layout* out, int kv_heads, int head_dim, int page_size, int k_group,
                   int v_group, int bit_v, const int32_t* tier_counts, int64_t row_cap,
                   int64_t group_cap);

/*
 * K1: quantize and pack whole pages (layout.py:71-129 quantize_key_page +
 * quantize_value_page, written where cache.py:64-81 would concatenate them).
 * Bit-exact with the reference: IEEE fp32 divide, round-half-even, fp16 RNE.
 * src_k/src_v: [seq][head][token][D] with the given element strides (channel
 * stride 1), dtype src_dtype.  jobs (device int32 [n_jobs][4]):
 * {src_seq, src_token0, dst_seq, dst_page}; a job with src_seq = -1 packs
 * nothing.  dst_batch bounds dst_seq; any other job outside [0, dst_batch) x
 * [0, row_cap/page_size) is skipped and LF_ERR_OUT_OF_RANGE is written to
 * *status (device int32, may be NULL).
 */
LF_API int lf_pack_pages(const lf_layout* layout, const void* src_k, const void* src_v, int src_dtype,
                  int64_t src_seq_stride, int64_t src_head_stride, int64_t src_tok_stride,
                  const int32_t* jobs, int n_jobs, int dst_batch, const int32_t* chan_code,
                  int32_t* rows, uint16_t* kmeta, int32_t* status, lf_stream_t stream);

/*
 * Dequantize tokens [0, tokens) of one sequence to fp32 [H][tokens][D]
 * (layout.py:132-182; code * scale + min as separately rounded multiply and
 * add, so the round trip is bit-exact with the reference).
 */
LF_API int lf_dequantize(const lf_layout* layout, const int32_t* rows, const uint16_t* kmeta,
                  const int32_t* chan_code, int seq, int64_t tokens, float* out_k, float* out_v,
                  lf_stream_t stream);

/*
 * One decode token per sequence committed on the device (no counterpart in
 * the reference, whose commit runs on the host, cache.py:48-62): the token's
 * Key/Value (k_new/v_new [batch][H][D], strides new_seq_stride /
 * new_head_stride, dtype = the residual page's) is appended to the residual
 * page at tail_len[b]; a page that becomes full is quantized and packed into
 * history page hist_tokens[b] / page_size (K1, bit-exact) and the residual
 * page starts empty; then tail_len / hist_tokens are advanced on the device.
 * Every position comes from the device lengths, so the call can be captured in
 * a CUDA graph and replayed step after step.  jobs: device int32 scratch
 * [batch][4].  A page that would pass row_cap is not packed and
 * LF_ERR_OUT_OF_RANGE is written to *status.
 */
LF_API int lf_commit_token(const lf_layout* layout, int32_t* rows, uint16_t* kmeta, const int32_t* chan_code,
                           void* tail_k, void* tail_v, int64_t tail_seq_stride, int64_t tail_head_stride,
                           int32_t* hist_tokens, int32_t* tail_len, int dtype, const void* k_new,
                           const void* v_new, int64_t new_seq_stride, int64_t new_head_stride, int batch,
                           int32_t* jobs, int32_t* status, lf_stream_t stream);

/* Resident K2 CTAs per SM for this layer and split size (occupancy of the
 * kernel lf_decode_partial would launch, capped by tensor-memory columns);
 * <= 0 on error.  Needs a current CUDA device. */
LF_API int lf_decode_occupancy(const lf_layout* layout, int n_q, int pages_per_split);

/* Bytes of fp32 split partials K2 writes and K3 reads. */
LF_API size_t lf_decode_workspace_bytes(int batch, int kv_heads, int n_q, int head_dim, int max_splits);

/* Number of work-item splits per (sequence, KV head): page splits for a
 * history of up to max_pages pages cut into pages_per_split, plus the
 * residual splits (32 residual tokens each, ceil(page_size / 32)). */
LF_API int lf_decode_max_splits(int64_t max_pages, int pages_per_split, int page_size);

/* As lf_decode_max_splits for calls with q_len query tokens per sequence:
 * the residual (tail rows + q_len new tokens) takes
 * ceil((page_size - 1 + q_len) / 32) splits. */
LF_API int lf_decode_max_splits_multi(int64_t max_pages, int pages_per_split, int page_size, int q_len);

/*
 * K2: split-K GQA decode attention over the packed history plus the
 * original-dtype residual page and the new token (replaces kernel.cu:112-190
 * launched from reference.py:59-109).  One work item per (sequence, KV head,
 * split); split s < n = ceil(pages/pages_per_split) covers pages
 * [s*pps, min((s+1)*pps, pages)); splits n .. n + ceil(page_size/32) - 1
 * cover 32 residual tokens each (tail_len[b] tail rows followed by the new
 * token when k_new is not NULL; rows 16-byte aligned).
 * Writes an unnormalised partial (running max m, sum l, accumulator) per
 * (item, q-head) into workspace.
 *   hist_tokens [batch] device int32, multiple of page_size
 *   tail_k/tail_v [batch][H][page_size][D] (strides tail_seq_stride,
 *     tail_head_stride elements; token stride D), dtype resid_dtype
 *   tail_len [batch] device int32 in [0, page_size)
 *   k_new/v_new [batch][H][D] (strides new_seq_stride, new_head_stride), resid_dtype, or NULL
 *   q [batch][n_q][D] (strides q_seq_stride, q_head_stride), dtype q_dtype
 * q-head j of KV head h is h * (n_q / H) + j (repeat_kv, reference.py:10-15).
 * GQA groups above 8 are split over several CTAs per KV head.
 * status (device int32, may be NULL) is set to LF_ERR_DEVICE_TIMEOUT if a
 * bounded device-side wait expires; the kernel then returns without hanging.
 * Geometry head_dim 128 / page 128 / k_group 128 / v_group 128
 * runs on the tensor cores (tcgen05.mma kind::i8); other supported
 * geometries (head_dim <= 128, page <= 128, k_group == page, v_group ==
 * head_dim) on a CUDA-core kernel.
 */
LF_API int lf_decode_partial(const lf_layout* layout, const int32_t* rows, const uint16_t* kmeta,
                      const int32_t* slot_chan, const int32_t* hist_tokens, const void* tail_k,
                      const void* tail_v, int64_t tail_seq_stride, int64_t tail_head_stride,
                      const int32_t* tail_len, int resid_dtype, const void* k_new,
                      const void* v_new, int64_t new_seq_stride, int64_t new_head_stride,
                      const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
                      int batch, int n_q, float scaling, int pages_per_split, int max_splits,
                      float* workspace, int32_t* status, lf_stream_t stream);

/*
 * K3: merge the split partials into the attention output
 * out [batch][n_q][D] (strides out_seq_stride, out_head_stride), dtype out_dtype.
 * Softmax-exact: out = sum_s e^(m_s - M) acc_s / sum_s e^(m_s - M) l_s.
 * head_dim must be even (the partials are read two channels at a time).
 */
LF_API int lf_decode_merge(const float* workspace, const int32_t* hist_tokens, int batch, int kv_heads,
                    int n_q, int head_dim, int page_size, int pages_per_split, int max_splits,
                    void* out, int out_dtype, int64_t out_seq_stride, int64_t out_head_stride,
                    lf_stream_t stream);

/*
 * K2 then K3 in one call (the reference's single decode op, logitfill_decode,
 * kernel.cu:198-284): same inputs as lf_decode_partial (workspace of
 * lf_decode_workspace_bytes bytes), same output as lf_decode_merge.
 */
LF_API int lf_decode(const lf_layout* layout, const int32_t* rows, const uint16_t* kmeta,
                     const int32_t* slot_chan, const int32_t* hist_tokens, const void* tail_k,
                     const void* tail_v, int64_t tail_seq_stride, int64_t tail_head_stride,
                     const int32_t* tail_len, int resid_dtype, const void* k_new, const void* v_new,
                     int64_t new_seq_stride, int64_t new_head_stride, const void* q, int q_dtype,
                     int64_t q_seq_stride, int64_t q_head_stride, int batch, int n_q, float scaling,
                     int pages_per_split, int max_splits, float* workspace, void* out, int out_dtype,
                     int64_t out_seq_stride, int64_t out_head_stride, int32_t* status, lf_stream_t stream);

/*
 * K2 then K3 for q_len query tokens per sequence (a chunked prefill over the
 * packed history, or a decode step when q_len is 1): the dense attention the
 * reference runs for a multi-token call with history, reference.py:30-56
 * with the right-aligned causal mask of reference.py:18-27 (it has no kernel
 * for it).  Every query token sees the packed history and the tail rows;
 * query token i sees new tokens 0..i.
 *   k_new/v_new [batch][H][q_len][D] (strides new_seq_stride, new_head_stride,
 *     new_tok_stride; rows 16-byte aligned), resid_dtype, or NULL
 *   q [batch][n_q][q_len][D] (strides q_seq_stride, q_head_stride, q_tok_stride)
 *   out [batch][n_q][q_len][D] (strides out_seq_stride, out_head_stride, out_tok_stride)
 *   workspace: lf_decode_workspace_bytes(batch, H, n_q * q_len, D, max_splits)
 *   max_splits >= lf_decode_max_splits_multi(row_cap / page_size, pps, page_size, q_len)
 * The other arguments are those of lf_decode.  One CTA per split computes up
 * to 8 (q-head, query token) pairs, so every page is read once per 8 pairs.
 */
LF_API int lf_decode_multi(const lf_layout* layout, const int32_t* rows, const uint16_t* kmeta,
                           const int32_t* slot_chan, const int32_t* hist_tokens, const void* tail_k,
                           const void* tail_v, int64_t tail_seq_stride, int64_t tail_head_stride,
                           const int32_t* tail_len, int resid_dtype, const void* k_new, const void* v_new,
                           int64_t new_seq_stride, int64_t new_head_stride, int64_t new_tok_stride,
                           const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
                           int64_t q_tok_stride, int q_len, int batch, int n_q, float scaling,
                           int pages_per_split, int max_splits, float* workspace, void* out, int out_dtype,
                           int64_t out_seq_stride, int64_t out_head_stride, int64_t out_tok_stride,
                           int32_t* status, lf_stream_t stream);

/*
 * K2 + K3 without a caller workspace, for callers that cannot allocate
 * device memory (allocator callbacks, runtimes that plan every allocation up
 * front, hosts that link only this library).  No counterpart in the
 * reference: its decode op allocates its output on every call.
 * Same inputs as lf_decode_partial, same output as lf_decode_merge; the split
 * partials live in a fixed 8 MiB __device__ array inside the library, held
 * on every GPU that loads it.  Rejects (LF_ERR_INVALID_ARGUMENT) a call whose
 * partials, lf_decode_workspace_bytes(batch, H, n_q, D, max_splits), exceed
 * 8 MiB.  Allocates nothing.  The first call on a device looks up the array's
 * address (cudaGetSymbolAddress); make it before any stream capture.  Calls
 * share the array: calls that overlap on the GPU race and must be ordered by
 * the caller.
 */
LF_API int lf_decode_noalloc(const lf_layout* layout, const int32_t* rows, const uint16_t* kmeta,
                             const int32_t* slot_chan, const int32_t* hist_tokens, const void* tail_k,
                             const void* tail_v, int64_t tail_seq_stride, int64_t tail_head_stride,
                             const int32_t* tail_len, int resid_dtype, const void* k_new, const void* v_new,
                             int64_t new_seq_stride, int64_t new_head_stride, const void* q, int q_dtype,
                             int64_t q_seq_stride, int64_t q_head_stride, int batch, int n_q, float scaling,
                             int pages_per_split, int max_splits, void* out, int out_dtype,
                             int64_t out_seq_stride, int64_t out_head_stride, int32_t* status,
                             lf_stream_t stream);

/*
 * Self-test of the bounded device-side wait used on every mbarrier of the
 * decode kernels (no counterpart in the reference).  One thread waits, with
 * limit_ns, for a barrier phase that completes only when arrive != 0; it
 * writes LF_OK, or LF_ERR_DEVICE_TIMEOUT once the limit runs out, to *status
 * (device int32) and returns.  No fault, trap or hang in either case.
 */
LF_API int lf_selftest_wait(int32_t* status, int64_t limit_ns, int arrive, lf_stream_t stream);

/*
 * Self-test of K1's per-element arithmetic (no counterpart in the reference;
 * it checks the restatement of layout.py:12-18).  For i < n (device arrays):
 * quotient[i] = (x[i] - lo[i]) / scale[i] as K1 computes it (IEEE subtract,
 * Markstein division with RN(1 / scale)) and code[i] =
 * clamp(round_half_even(quotient[i]), 0, 2^bits - 1).  A test compares both
 * with IEEE division bit for bit.
 */
LF_API int lf_selftest_divide(const float* x, const float* lo, const float* scale, int64_t n, int bits,
                              float* quotient, uint32_t* code, lf_stream_t stream);

/*
 * KV-head sharding over NVLink: the split merge fused with the output
 * all-gather.  The reference decodes all KV heads on one device
 * (reference.py:45-47 expands them with repeat_kv, kernel.cu:234 launches one
 * CTA per q-head); when the KV heads are split over N GPUs, rank r owns heads
 * [r H/N, (r+1) H/N) and every layer's output must reach every rank.
 *
 * Buffers shared between the ranks' processes come from lf_ipc_alloc (device
 * memory, zero-filled) and travel as 64-byte CUDA IPC handles (lf_ipc_handle,
 * lf_ipc_open with peer access enabled, lf_ipc_close; lf_ipc_free on the
 * owner after every peer has closed it).
 *
 * lf_decode_merge_gather is lf_decode_merge for one query token per sequence
 * (n_q / kv_heads <= 8 q-heads per KV head; same workspace, same result bit
 * for bit), storing this rank's output [batch, n_q, head_dim] (n_q = the
 * rank's q-heads) as block `rank` of layer `layer` of every rank's gathered
 * buffer [layers][world][batch][n_q][head_dim] (dtype out_dtype): peer_out
 * holds the world buffer addresses (device array of uint64).  Each CTA then
 * adds 1 to uint32 counter `layer` of every rank's flag array (peer_flags,
 * device array of uint64), after making its stores visible to all GPUs.
 * lf_gather_signals(batch, n_q, world) is the number of adds a rank receives
 * per layer.
 *
 * lf_gather_wait launches one thread on `stream` that waits until counter
 * `layer` of this rank's flags reaches `expected`, then subtracts `expected`,
 * so the counter serves the next step.  It gives up after limit_ns and
 * writes LF_ERR_DEVICE_TIMEOUT to *status (device int32, may be NULL).
 * Kernels after it on the stream see every rank's block of that layer.
 */
LF_API int lf_ipc_alloc(size_t bytes, void** ptr);
LF_API int lf_ipc_free(void* ptr);
LF_API int lf_ipc_handle(const void* ptr, void* handle);
LF_API int lf_ipc_open(const void* handle, void** ptr);
LF_API int lf_ipc_close(void* ptr);
LF_API int lf_decode_merge_gather(const float* workspace, const int32_t* hist_tokens, int batch, int kv_heads,
                                  int n_q, int head_dim, int page_size, int pages_per_split, int max_splits,
                                  const uint64_t* peer_out, const uint64_t* peer_flags, int layer, int rank,
                                  int world, int out_dtype, lf_stream_t stream);
LF_API int lf_gather_signals(int batch, int n_q, int world);
LF_API int lf_gather_wait(uint32_t* flags, int layer, uint32_t expected, uint64_t limit_ns, int32_t* status,
                          lf_stream_t stream);

/* Human-readable text of a status code; detail of the last failure on this thread. */
LF_API const char* lf_status_string(int status);
LF_API const char* lf_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* LOGITFILL_B200_H */
