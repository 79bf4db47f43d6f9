// Pieces shared by the decode kernels: launch parameters, CTA reductions,
// the residual split (original-dtype tail rows + new tokens) and the partial
// writer read by the merge kernel.
//
// Query tokens.  A call attends q_len query tokens per sequence (1 for a
// decode step, more for a chunked prefill over the packed history).  The
// kernels see "virtual heads": KV head h owns gq * q_len of them, v = j * q_len
// + i for q-head h * gq + j and query token i, and one CTA takes cg of them
// (chunk c = v / cg, n_chunks = gq * q_len / cg chunks per KV head).  Every
// virtual head sees the whole packed history and residual page; of the q_len
// new tokens, query token i sees tokens 0..i (the causal mask aligned to the
// right edge, reference.py:18-27).
#pragma once

#include "lf_common.cuh"

namespace lf {

constexpr int kDecThreads = 128;
constexpr int kGQ = 8;         // q-heads per KV head handled by one CTA
constexpr int kResChunk = 32;  // residual tokens per chunk

struct DecodeParams {
  lf_layout L;
  const int32_t* rows;
  const uint16_t* kmeta;
  const int32_t* slot_chan;
  const int32_t* hist_tokens;
  const void* tail_k;
  const void* tail_v;
  int64_t tail_seq_stride, tail_head_stride;
  const int32_t* tail_len;
  const void* k_new;
  const void* v_new;
  int64_t new_seq_stride, new_head_stride, new_tok_stride;
  const void* q;
  int64_t q_seq_stride, q_head_stride, q_tok_stride;
  int batch, n_q, gq, pps, max_splits, n_slots;
  int q_len, cg, n_chunks;  // query tokens; virtual heads per CTA; CTAs per KV head and split
  float scaling;
  float* ws;
  int32_t* status;  // device status word (LF_ERR_DEVICE_TIMEOUT on a timed-out wait), may be null
  int q_dtype, resid_dtype;  // lf_dtype of q and of the residual rows
};

// Sum (or max) of kGQ values over the CTA; every thread receives the result.
template <bool kMax>
__device__ __forceinline__ void block_reduce8(float (&v)[kGQ], float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int j = 0; j < kGQ; ++j) {
    float x = v[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float y = __shfl_xor_sync(0xffffffffu, x, o);
      x = kMax ? fmaxf(x, y) : x + y;
    }
    v[j] = x;
  }
  if (lane == 0) {
#pragma unroll
    for (int j = 0; j < kGQ; ++j) red[warp * kGQ + j] = v[j];
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kGQ; ++j) {
    float x = red[j];
#pragma unroll
    for (int w = 1; w < kDecThreads / 32; ++w)
      x = kMax ? fmaxf(x, red[w * kGQ + j]) : x + red[w * kGQ + j];
    v[j] = x;
  }
  __syncthreads();
}

// Element offset of virtual head v of KV head h in sequence b's query
// (q-head h * gq + v / q_len, the repeat_kv order of reference.py:10-15;
// query token v % q_len).
__device__ __forceinline__ int64_t vhead_q_offset(const DecodeParams& p, int b, int h, int v) {
  const int j = v / p.q_len, i = v - j * p.q_len;
  return b * p.q_seq_stride + static_cast<int64_t>(h * p.gq + j) * p.q_head_stride +
         static_cast<int64_t>(i) * p.q_tok_stride;
}
// Index of the partial record of (sequence b, KV head h, chunk c, split s).
__device__ __forceinline__ int64_t item_index(const DecodeParams& p, int b, int h, int c, int s) {
  return ((static_cast<int64_t>(b) * p.L.kv_heads + h) * p.n_chunks + c) * p.max_splits + s;
}

// Virtual heads c*cg .. c*cg+cg-1 of KV head h into q_s [kGQ][D] fp32,
// zero-padded to kGQ heads; thread d < D loads channel d of every head (all
// loads issued before the stores).  The virtual heads are stepped in order
// (q-head jh, query token ii), so no division is needed per head.
template <typename LOAD>
__device__ __forceinline__ void gather_query_group(const DecodeParams& p, int b, int h, int c, float* q_s,
                                                   LOAD load) {
  const int D = p.L.head_dim, d = threadIdx.x, v0 = c * p.cg;
  int jh = v0 / p.q_len, ii = v0 - jh * p.q_len;
  const int64_t base = b * p.q_seq_stride + static_cast<int64_t>(h) * p.gq * p.q_head_stride + d;
  float vals[kGQ];
#pragma unroll
  for (int j = 0; j < kGQ; ++j) {
    vals[j] = (j < p.cg && d < D) ? load(base + jh * p.q_head_stride + ii * p.q_tok_stride) : 0.0f;
    if (++ii == p.q_len) {
      ii = 0;
      ++jh;
    }
  }
  if (d < D) {
#pragma unroll
    for (int j = 0; j < kGQ; ++j) q_s[j * D + d] = vals[j];
  }
}

template <typename QT>
__device__ __forceinline__ void load_query_group(const DecodeParams& p, int b, int h, int c, float* q_s) {
  const QT* q = static_cast<const QT*>(p.q);
  gather_query_group(p, b, h, c, q_s, [&](int64_t o) { return Scalar<QT>::load(q + o); });
}

// Query group as load_query_group, dtype chosen at run time (p.q_dtype).
// Called by the first 128 threads (head_dim <= 128).
__device__ __forceinline__ void load_query_group_rt(const DecodeParams& p, int b, int h, int c, float* q_s) {
  switch (p.q_dtype) {
    case LF_F32: {
      const float* q = static_cast<const float*>(p.q);
      gather_query_group(p, b, h, c, q_s, [&](int64_t o) { return q[o]; });
      break;
    }
    case LF_F16: {
      const __half* q = static_cast<const __half*>(p.q);
      gather_query_group(p, b, h, c, q_s, [&](int64_t o) { return __half2float(q[o]); });
      break;
    }
    default: {
      const __nv_bfloat16* q = static_cast<const __nv_bfloat16*>(p.q);
      gather_query_group(p, b, h, c, q_s, [&](int64_t o) { return __bfloat162float(q[o]); });
    }
  }
}

// Named barrier over the first `count` threads of the CTA (id >= 1).
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Sum of N values over the first 128 threads only, synchronised on barrier `bar_id`.
template <int N>
__device__ __forceinline__ void group_sum(float (&v)[N], float* red, int bar_id) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    float x = v[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    v[j] = x;
  }
  if (lane == 0) {
#pragma unroll
    for (int j = 0; j < N; ++j) red[warp * kGQ + j] = v[j];
  }
  named_sync(bar_id, kDecThreads);
#pragma unroll
  for (int j = 0; j < N; ++j) v[j] = (red[j] + red[kGQ + j]) + (red[2 * kGQ + j] + red[3 * kGQ + j]);
  named_sync(bar_id, kDecThreads);
}

// Residual splits: chunk c of the original-dtype residual (tail_len[b] tail
// rows followed by the q_len new tokens; reference.py:38-42) covers tokens
// [kResChunk*c, kResChunk*(c+1)).  Up to ceil((page - 1 + q_len)/kResChunk)
// chunks, one work item each, so the residual is spread over several CTAs.
__host__ __device__ inline int residual_splits(int page_size, int q_len) {
  return (page_size - 1 + q_len + kResChunk - 1) / kResChunk;
}

struct ResidSmem {
  int k, v, part, p, stat, total;  // byte offsets from the region base
};
__host__ __device__ inline ResidSmem resid_smem(int D) {
  ResidSmem r;
  int off = 0;
  r.k = off; off += kResChunk * (D + 1) * 4;     // K rows, stride D+1 (conflict-free columns)
  r.v = off; off += kResChunk * D * 4;           // V rows
  r.part = off; off += 4 * kResChunk * kGQ * 4;  // per-warp partial scores
  r.p = off; off += kResChunk * kGQ * 4;         // probabilities
  r.stat = off; off += 3 * kGQ * 4;              // new max, alpha, chunk sum
  r.total = off;
  return r;
}

template <typename RT>
__device__ __forceinline__ void load_vec_to_float(const RT* src, float* dst);
template <>
__device__ __forceinline__ void load_vec_to_float<__nv_bfloat16>(const __nv_bfloat16* src, float* dst) {
  const uint4 u = *reinterpret_cast<const uint4*>(src);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    dst[2 * i] = __uint_as_float(w[i] << 16);
    dst[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
template <>
__device__ __forceinline__ void load_vec_to_float<__half>(const __half* src, float* dst) {
  const uint4 u = *reinterpret_cast<const uint4*>(src);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    dst[2 * i] = f.x;
    dst[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load_vec_to_float<float>(const float* src, float* dst) {
  const float4 a = *reinterpret_cast<const float4*>(src);
  const float4 b = *reinterpret_cast<const float4*>(src + 4);
  dst[0] = a.x; dst[1] = a.y; dst[2] = a.z; dst[3] = a.w;
  dst[4] = b.x; dst[5] = b.y; dst[6] = b.z; dst[7] = b.w;
}

// One residual chunk: attention of the query group (q_s [kGQ][D]) over up to
// kResChunk tokens in fp32.  Thread d < D accumulates channel d in acc; the
// chunk's probability sum is added to lt of thread 0 only (lt is summed over
// the CTA afterwards).  Rows are read 8 elements per load (16 B for bf16/fp16;
// the residual page and the new-token rows are contiguous, D a multiple of 8).
// 8 consecutive elements of dtype `dtype` (16-byte aligned rows) as fp32.
__device__ __forceinline__ void load_vec_to_float_rt(const void* src, int dtype, float* dst) {
  switch (dtype) {
    case LF_F32: load_vec_to_float<float>(static_cast<const float*>(src), dst); break;
    case LF_F16: load_vec_to_float<__half>(static_cast<const __half*>(src), dst); break;
    default: load_vec_to_float<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(src), dst); break;
  }
}

// One residual chunk: attention of the query group (q_s [kGQ][D]) over up to
// kResChunk tokens in fp32, first 128 threads, barrier 1.  Thread d < D
// accumulates channel d in acc; the chunk's probability sum is added to lt of
// thread 0 only.  When load_q is set the query group is fetched here, after
// the row loads are issued, so the two global-memory latencies overlap.
static __device__ __forceinline__ void residual_chunk(const DecodeParams& p, int b, int h, int vc, int chunk,
                                                      float* q_s, bool load_q, unsigned char* region,
                                                      float (&m)[kGQ], float (&acc)[kGQ], float (&lt)[kGQ]) {
  const int RS_ = p.resid_dtype == LF_F32 ? 4 : 2;  // element size
  const int D = p.L.head_dim, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, GQ = p.cg;
  const ResidSmem RS = resid_smem(D);
  float* k_s = reinterpret_cast<float*>(region + RS.k);
  float* v_s = reinterpret_cast<float*>(region + RS.v);
  float* part = reinterpret_cast<float*>(region + RS.part);
  float* p_s = reinterpret_cast<float*>(region + RS.p);
  float* stat = reinterpret_cast<float*>(region + RS.stat);
  const int tl = p.tail_len[b];
  const int total = tl + (p.k_new != nullptr ? p.q_len : 0);
  const int t0 = chunk * kResChunk;
  const int ntok = min(kResChunk, total - t0);
  if (ntok <= 0) {
    if (load_q) load_query_group_rt(p, b, h, vc, q_s);
    return;
  }
  const char* tk = static_cast<const char*>(p.tail_k) + (b * p.tail_seq_stride + h * p.tail_head_stride) * RS_;
  const char* tv = static_cast<const char*>(p.tail_v) + (b * p.tail_seq_stride + h * p.tail_head_stride) * RS_;
  const char* nk = p.k_new != nullptr
                       ? static_cast<const char*>(p.k_new) + (b * p.new_seq_stride + h * p.new_head_stride) * RS_
                       : nullptr;
  const char* nv = p.v_new != nullptr
                       ? static_cast<const char*>(p.v_new) + (b * p.new_seq_stride + h * p.new_head_stride) * RS_
                       : nullptr;
  // 1. Rows -> fp32 in shared memory; every thread issues all its loads first.
  const int vec_per_row = D / 8;
  const int nvec = kResChunk * vec_per_row;  // <= 512
  constexpr int kMaxVec = kResChunk * 128 / 8 / kDecThreads;  // 4
  float kv[kMaxVec][8], vv[kMaxVec][8];
#pragma unroll
  for (int r = 0; r < kMaxVec; ++r) {
    const int i = tid + r * kDecThreads;
    const int t = i / vec_per_row, c = i - t * vec_per_row;
    const int tok = t0 + t;
    if (i < nvec && t < ntok) {
      const char* ks = tok < tl ? tk + static_cast<int64_t>(tok) * D * RS_ : nk + (tok - tl) * p.new_tok_stride * RS_;
      const char* vs = tok < tl ? tv + static_cast<int64_t>(tok) * D * RS_ : nv + (tok - tl) * p.new_tok_stride * RS_;
      load_vec_to_float_rt(ks + c * 8 * RS_, p.resid_dtype, kv[r]);
      load_vec_to_float_rt(vs + c * 8 * RS_, p.resid_dtype, vv[r]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) kv[r][e] = vv[r][e] = 0.f;
    }
  }
  if (load_q) load_query_group_rt(p, b, h, vc, q_s);
#pragma unroll
  for (int r = 0; r < kMaxVec; ++r) {
    const int i = tid + r * kDecThreads;
    if (i >= nvec) break;
    const int t = i / vec_per_row, c = i - t * vec_per_row;
#pragma unroll
    for (int e = 0; e < 8; ++e) k_s[t * (D + 1) + c * 8 + e] = kv[r][e];
    *reinterpret_cast<float4*>(v_s + t * D + c * 8) = make_float4(vv[r][0], vv[r][1], vv[r][2], vv[r][3]);
    *reinterpret_cast<float4*>(v_s + t * D + c * 8 + 4) = make_float4(vv[r][4], vv[r][5], vv[r][6], vv[r][7]);
  }
  named_sync(1, kDecThreads);
  // 2. Partial scores: lane = token, warp = quarter of the head dim; four
  // channels per step, the query read as float4 (broadcast).
  {
    const int dq = D / 4, d0 = warp * dq;
    float ps[kGQ];
#pragma unroll
    for (int j = 0; j < kGQ; ++j) ps[j] = 0.f;
    const float* kr = k_s + lane * (D + 1);
#pragma unroll 2
    for (int d = d0; d < d0 + dq; d += 4) {
      const float k0 = kr[d], k1 = kr[d + 1], k2 = kr[d + 2], k3 = kr[d + 3];
#pragma unroll
      for (int j = 0; j < kGQ; ++j) {
        const float4 qv = *reinterpret_cast<const float4*>(q_s + j * D + d);
        ps[j] = fmaf(qv.x, k0, fmaf(qv.y, k1, fmaf(qv.z, k2, fmaf(qv.w, k3, ps[j]))));
      }
    }
    float* dst = part + (warp * kResChunk + lane) * kGQ;
    *reinterpret_cast<float4*>(dst) = make_float4(ps[0], ps[1], ps[2], ps[3]);
    *reinterpret_cast<float4*>(dst + 4) = make_float4(ps[4], ps[5], ps[6], ps[7]);
  }
  named_sync(1, kDecThreads);
  // 3. Softmax statistics of the chunk (lane = token): warp w takes heads
  // 2w and 2w + 1.  New token r (row tl + r) is visible to virtual heads of
  // query token i >= r.
  {
    const int rnew = t0 + lane - tl;  // new-token index of this row, < 0 for a tail row
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int j = 2 * warp + jj;
      const int vt = (vc * GQ + j) % p.q_len;  // query token of virtual head j
      float sj = -INFINITY;
      if (lane < ntok && j < GQ && rnew <= vt) {
        sj = (part[(0 * kResChunk + lane) * kGQ + j] + part[(1 * kResChunk + lane) * kGQ + j]) +
             (part[(2 * kResChunk + lane) * kGQ + j] + part[(3 * kResChunk + lane) * kGQ + j]);
        sj *= p.scaling;
      }
      float mx = sj;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float mj = m[0];  // running max of head j (the same in every thread); selected without dynamic indexing
#pragma unroll
      for (int t = 1; t < kGQ; ++t)
        if (t == j) mj = m[t];
      const float mnew = fmaxf(mj, mx);
      const float pj = (sj == -INFINITY) ? 0.f : expf(sj - mnew);
      p_s[lane * kGQ + j] = pj;
      float sum = pj;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (lane == 0) {
        stat[j] = mnew;
        stat[kGQ + j] = (mj == -INFINITY || mnew == -INFINITY) ? 0.f : expf(mj - mnew);
        stat[2 * kGQ + j] = sum;
      }
    }
  }
  named_sync(1, kDecThreads);
  // 4. Rescale and accumulate.
#pragma unroll
  for (int j = 0; j < kGQ; ++j) {
    if (j >= GQ) continue;
    const float alpha = stat[kGQ + j];
    m[j] = stat[j];
    lt[j] = lt[j] * alpha + (tid == 0 ? stat[2 * kGQ + j] : 0.f);
    acc[j] *= alpha;
  }
  if (tid < D) {
#pragma unroll 4
    for (int t = 0; t < ntok; ++t) {
      const float v = v_s[t * D + tid];
      const float4 a = *reinterpret_cast<const float4*>(p_s + t * kGQ);
      const float4 c = *reinterpret_cast<const float4*>(p_s + t * kGQ + 4);
      acc[0] = fmaf(a.x, v, acc[0]);
      acc[1] = fmaf(a.y, v, acc[1]);
      acc[2] = fmaf(a.z, v, acc[2]);
      acc[3] = fmaf(a.w, v, acc[3]);
      acc[4] = fmaf(c.x, v, acc[4]);
      acc[5] = fmaf(c.y, v, acc[5]);
      acc[6] = fmaf(c.z, v, acc[6]);
      acc[7] = fmaf(c.w, v, acc[7]);
    }
  }
}

// Partial of a residual item, whose statistics need no reduction: m is the
// same in every thread, the probability sum lives in thread 0 and there is
// no Value-min term.  Thread d < D writes channel d.
__device__ __forceinline__ void write_partial_resid(const DecodeParams& p, int64_t index, const float (&acc)[kGQ],
                                                    const float (&m)[kGQ], const float (&lt)[kGQ]) {
  const int D = p.L.head_dim, GQ = p.cg, d = threadIdx.x;
  float* item = p.ws + index * (GQ * (D + 2));
  if (d < D) {
#pragma unroll
    for (int j = 0; j < kGQ; ++j)
      if (j < GQ) item[j * D + d] = acc[j];
  }
  if (d == 0) {
#pragma unroll
    for (int j = 0; j < kGQ; ++j) {
      if (j < GQ) {
        item[GQ * D + j] = m[j];
        item[GQ * D + GQ + j] = lt[j];
      }
    }
  }
}

// Partial writer for the first 128 threads only (barrier `bar_id`), N >= p.cg.
template <int N>
__device__ __forceinline__ void write_partial_group(const DecodeParams& p, int64_t index, int channel,
                                                    const float (&acc)[N], const float (&m)[N],
                                                    float (&lt)[N], float (&lvt)[N], float* red, int bar_id) {
  const int D = p.L.head_dim, GQ = p.cg;
  group_sum<N>(lt, red, bar_id);
  group_sum<N>(lvt, red, bar_id);
  float* item = p.ws + index * (GQ * (D + 2));
  if (channel >= 0 && channel < D) {
#pragma unroll
    for (int j = 0; j < N; ++j)
      if (j < GQ) item[j * D + channel] = acc[j] + lvt[j];
  }
  if (threadIdx.x == 0) {
#pragma unroll
    for (int j = 0; j < N; ++j) {
      if (j < GQ) {
        item[GQ * D + j] = m[j];
        item[GQ * D + GQ + j] = lt[j];
      }
    }
  }
}

// Write one work item's partial: acc[j][d] + lv[j], m[j] (natural-log units), l[j].
// lt/lvt are per-thread partial sums, reduced here over the CTA.
__device__ __forceinline__ void write_partial(const DecodeParams& p, int64_t index, int channel,
                                              const float (&acc)[kGQ], const float (&m)[kGQ],
                                              float (&lt)[kGQ], float (&lvt)[kGQ], float* red) {
  const int D = p.L.head_dim, GQ = p.cg;
  block_reduce8<false>(lt, red);
  block_reduce8<false>(lvt, red);
  float* item = p.ws + index * (GQ * (D + 2));
  if (channel >= 0 && channel < D) {
#pragma unroll
    for (int j = 0; j < kGQ; ++j)
      if (j < GQ) item[j * D + channel] = acc[j] + lvt[j];
  }
  if (threadIdx.x == 0) {
#pragma unroll
    for (int j = 0; j < kGQ; ++j) {
      if (j < GQ) {
        item[GQ * D + j] = m[j];
        item[GQ * D + GQ + j] = lt[j];
      }
    }
  }
}

}  // namespace lf
