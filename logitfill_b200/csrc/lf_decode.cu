// K2 (split-K GQA decode over packed pages + residual) and K3 (split merge).
//
// Work item = (split s, KV head h and virtual-head chunk c, sequence b); one
// 128-thread CTA each.  All q-heads of the GQA group are computed together
// (one chunk for a decode step), so each packed page is read from HBM once
// per KV head (the reference kernel re-reads it once per q-head,
// kernel.cu:112-190).
//
// The packed history is affine per page: a Key channel's scale/min is
// constant over its k_group tokens and a token's Value scale/min is constant
// over its v_group channels.  So
//   q.k_t = sum_c (q_c s_c) code_tc + sum_c q_c m_c        (per-page q' and bias)
//   sum_t p_t v_t = sum_t (p_t s_t) code_t + (sum_t p_t m_t) 1
// and the inner loops multiply raw integer codes by precomputed fp32 factors.

#include <cstdlib>
#include <cstring>

#include "lf_decode_common.cuh"

namespace lf {

// Tensor-core decode (lf_decode_tc.cu).
bool tc_supported(const lf_layout& L, int gq, int pps);
int launch_partial_tc(const DecodeParams& p, int resid_dtype, int q_dtype, cudaStream_t stream);
int occupancy_tc(const lf_layout& L, int gq, int pps);
bool tc_allowed();

struct DecodeSmem {
  int q, qp, p, red, slot, slot16, region, rows_bytes, total;
};

__host__ __device__ inline DecodeSmem decode_smem(const lf_layout& L, int n_slots) {
  const int D = L.head_dim, P = L.page_size;
  DecodeSmem s;
  int off = 0;
  s.q = off; off += kGQ * D * 4;
  s.qp = off; off += ((n_slots + 3) / 4 * 4) * kGQ * 4;
  s.p = off; off += (P > kResChunk ? P : kResChunk) * kGQ * 4;
  s.red = off; off += 2 * (kDecThreads / 32) * kGQ * 4;
  s.slot = off; off += ((n_slots + 3) / 4 * 4) * 4;
  s.slot16 = off; off += ((L.width[3] + 3) / 4 * 4) * 4;
  off = (off + 15) / 16 * 16;
  s.region = off;
  const int page_bytes = P * L.row_words * 4 + (L.meta_halves * 2 + 15) / 16 * 16;
  const int resid_bytes = resid_smem(D).total;
  s.rows_bytes = page_bytes;
  off += page_bytes > resid_bytes ? page_bytes : resid_bytes;
  s.total = (off + 15) / 16 * 16;
  return s;
}

template <typename RT, typename QT>
__global__ void __launch_bounds__(kDecThreads)
decode_partial_simt(DecodeParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const lf_layout& L = p.L;
  const DecodeSmem S = decode_smem(L, p.n_slots);
  float* q_s = reinterpret_cast<float*>(smem + S.q);
  float* qp_s = reinterpret_cast<float*>(smem + S.qp);
  float* p_s = reinterpret_cast<float*>(smem + S.p);
  float* red = reinterpret_cast<float*>(smem + S.red);
  int* slot_s = reinterpret_cast<int*>(smem + S.slot);
  int* slot16_s = reinterpret_cast<int*>(smem + S.slot16);
  unsigned char* region = smem + S.region;

  const int s = blockIdx.x, h = blockIdx.y / p.n_chunks, c = blockIdx.y % p.n_chunks, b = blockIdx.z;
  const int tid = threadIdx.x;
  const int P = L.page_size, D = L.head_dim, R = L.row_words, H = L.kv_heads;
  const int GQ = p.cg;
  grid_dep_wait();
  grid_dep_trigger();
  const int pages = p.hist_tokens[b] / P;
  const int n_page_splits = (pages + p.pps - 1) / p.pps;
  if (s >= n_page_splits + residual_splits(P, p.q_len)) return;

  load_query_group<QT>(p, b, h, c, q_s);
  // Tier slot -> channel, in history-row order.
  for (int i = tid; i < p.n_slots; i += kDecThreads) {
    int tier = 0, base = 0;
    while (tier < 2 && i >= base + (32 / (2 << tier)) * L.words[tier]) {
      base += (32 / (2 << tier)) * L.words[tier];
      ++tier;
    }
    const int local = i - base;
    const int ch = local < L.width[tier] ? p.slot_chan[(tier * H + h) * D + local] : -1;
    // channel | tier << 16 | position << 18, or -1 for a padding slot (code 0).
    slot_s[i] = ch < 0 ? -1 : (ch | (tier << 16) | (local << 18));
  }
  for (int i = tid; i < L.width[3]; i += kDecThreads) slot16_s[i] = p.slot_chan[(3 * H + h) * D + i];

  float m[kGQ], acc[kGQ], lt[kGQ], lvt[kGQ];
#pragma unroll
  for (int j = 0; j < kGQ; ++j) {
    m[j] = -INFINITY;
    acc[j] = 0.f;
    lt[j] = 0.f;
    lvt[j] = 0.f;
  }

  if (s < n_page_splits) {
    int32_t* row_s = reinterpret_cast<int32_t*>(region);
    uint16_t* meta_s = reinterpret_cast<uint16_t*>(region + P * R * 4);
    const uint16_t* row16_s = reinterpret_cast<const uint16_t*>(row_s);
    const int pg0 = s * p.pps;
    const int pg1 = min(pages, pg0 + p.pps);
    const int64_t head_row = (static_cast<int64_t>(b) * H + h) * L.row_cap;
    const int64_t head_meta = (static_cast<int64_t>(b) * H + h) * L.group_cap;
    for (int pg = pg0; pg < pg1; ++pg) {
      __syncthreads();
      const int4* src = reinterpret_cast<const int4*>(p.rows + (head_row + static_cast<int64_t>(pg) * P) * R);
      int4* dst = reinterpret_cast<int4*>(row_s);
      for (int i = tid; i < P * R / 4; i += kDecThreads) dst[i] = __ldg(src + i);
      const int4* msrc = reinterpret_cast<const int4*>(p.kmeta + (head_meta + pg) * L.meta_halves);
      for (int i = tid; i < L.meta_halves / 8; i += kDecThreads)
        reinterpret_cast<int4*>(meta_s)[i] = __ldg(msrc + i);
      __syncthreads();

      // Per-page q' = q * scale (per slot) and bias = sum_c q_c * min_c.
      float bias[kGQ];
#pragma unroll
      for (int j = 0; j < kGQ; ++j) bias[j] = 0.f;
      for (int i = tid; i < p.n_slots; i += kDecThreads) {
        const int e = slot_s[i];
        float* dstq = qp_s + i * kGQ;
        if (e < 0) {
#pragma unroll
          for (int j = 0; j < kGQ; ++j) dstq[j] = 0.f;
          continue;
        }
        const int ch = e & 0xFFFF, tier = (e >> 16) & 3, local = (e >> 18) & 0x1FFF;
        const float sc = half_bits_to_float(meta_s[L.scale_off[tier] + local]);
        const float mn = half_bits_to_float(meta_s[L.min_off[tier] + local]);
#pragma unroll
        for (int j = 0; j < kGQ; ++j) {
          const float qv = q_s[j * D + ch];
          dstq[j] = qv * sc;
          bias[j] = fmaf(qv, mn, bias[j]);
        }
      }
      block_reduce8<false>(bias, red);

      float sc_t[kGQ];
      if (tid < P) {
#pragma unroll
        for (int j = 0; j < kGQ; ++j) sc_t[j] = bias[j];
        const uint32_t* row = reinterpret_cast<const uint32_t*>(row_s + tid * R);
        int slot = 0;
#pragma unroll
        for (int tier = 0; tier < 3; ++tier) {
          const int bits = 2 << tier, per = 32 / bits;
          const uint32_t mask = (1u << bits) - 1u;
          for (int w = 0; w < L.words[tier]; ++w) {
            const uint32_t x = row[L.code_off[tier] + w];
            for (int k = 0; k < per; ++k, ++slot) {
              const float c = static_cast<float>((x >> (k * bits)) & mask);
              const float4 a = *reinterpret_cast<const float4*>(qp_s + slot * kGQ);
              const float4 bq = *reinterpret_cast<const float4*>(qp_s + slot * kGQ + 4);
              sc_t[0] = fmaf(a.x, c, sc_t[0]);
              sc_t[1] = fmaf(a.y, c, sc_t[1]);
              sc_t[2] = fmaf(a.z, c, sc_t[2]);
              sc_t[3] = fmaf(a.w, c, sc_t[3]);
              sc_t[4] = fmaf(bq.x, c, sc_t[4]);
              sc_t[5] = fmaf(bq.y, c, sc_t[5]);
              sc_t[6] = fmaf(bq.z, c, sc_t[6]);
              sc_t[7] = fmaf(bq.w, c, sc_t[7]);
            }
          }
        }
        const uint16_t* r16 = row16_s + tid * 2 * R + 2 * L.half_off;
        for (int i = 0; i < L.width[3]; ++i) {
          const int ch = slot16_s[i];
          if (ch < 0) continue;
          const float kv = half_bits_to_float(r16[i]);
#pragma unroll
          for (int j = 0; j < kGQ; ++j) sc_t[j] = fmaf(q_s[j * D + ch], kv, sc_t[j]);
        }
#pragma unroll
        for (int j = 0; j < kGQ; ++j) sc_t[j] = j < GQ ? sc_t[j] * p.scaling : -INFINITY;
      } else {
#pragma unroll
        for (int j = 0; j < kGQ; ++j) sc_t[j] = -INFINITY;
      }
      float pm[kGQ];
#pragma unroll
      for (int j = 0; j < kGQ; ++j) pm[j] = sc_t[j];
      block_reduce8<true>(pm, red);
      float alpha[kGQ];
#pragma unroll
      for (int j = 0; j < kGQ; ++j) {
        const float mn = fmaxf(m[j], pm[j]);
        alpha[j] = m[j] == -INFINITY ? 0.f : expf(m[j] - mn);
        m[j] = mn;
      }
      if (tid < P) {
        const uint16_t* r16 = row16_s + tid * 2 * R + 2 * L.half_off + L.width[3];
        const float vs = half_bits_to_float(r16[0]);
        const float vm = half_bits_to_float(r16[1]);
#pragma unroll
        for (int j = 0; j < kGQ; ++j) {
          const float pj = m[j] == -INFINITY ? 0.f : expf(sc_t[j] - m[j]);
          lt[j] = fmaf(lt[j], alpha[j], pj);
          lvt[j] = fmaf(lvt[j], alpha[j], pj * vm);
          p_s[tid * kGQ + j] = pj * vs;
        }
      } else {
#pragma unroll
        for (int j = 0; j < kGQ; ++j) {
          lt[j] *= alpha[j];
          lvt[j] *= alpha[j];
        }
      }
      __syncthreads();
      if (tid < D) {
#pragma unroll
        for (int j = 0; j < kGQ; ++j) acc[j] *= alpha[j];
        const int wd = L.vcode_off + tid / 16, sh = 2 * (tid % 16);
        for (int t = 0; t < P; ++t) {
          const float c = static_cast<float>((static_cast<uint32_t>(row_s[t * R + wd]) >> sh) & 3u);
          const float4 a = *reinterpret_cast<const float4*>(p_s + t * kGQ);
          const float4 bq = *reinterpret_cast<const float4*>(p_s + t * kGQ + 4);
          acc[0] = fmaf(a.x, c, acc[0]);
          acc[1] = fmaf(a.y, c, acc[1]);
          acc[2] = fmaf(a.z, c, acc[2]);
          acc[3] = fmaf(a.w, c, acc[3]);
          acc[4] = fmaf(bq.x, c, acc[4]);
          acc[5] = fmaf(bq.y, c, acc[5]);
          acc[6] = fmaf(bq.z, c, acc[6]);
          acc[7] = fmaf(bq.w, c, acc[7]);
        }
      }
    }
  } else {
    residual_chunk(p, b, h, c, s - n_page_splits, q_s, false, region, m, acc, lt);
  }

  write_partial(p, item_index(p, b, h, c, s), tid, acc, m, lt, lvt, red);
}

// K3: one warp per (sequence, virtual head).  Lane s (mod 32) reads split s's max
// and sum; the global max, the weights exp(m_s - M) and the normaliser are
// warp reductions; then every lane accumulates its four channels over all
// splits, the weight of split s broadcast from the lane that computed it.
// The partial records (GQ x (D + 2) floats) are 8-byte aligned, so the
// values are read as float2.
constexpr int kMergeWarps = 4;

template <typename OT, int kFew>
__global__ void __launch_bounds__(kMergeWarps * 32)
decode_merge_kernel(const float* __restrict__ ws, const int32_t* __restrict__ hist_tokens, int batch,
                    int kv_heads, int n_q, int q_len, int cg, int D, int P, int pps, int max_splits,
                    OT* __restrict__ out, int64_t out_seq_stride, int64_t out_head_stride,
                    int64_t out_tok_stride) {
  const int lane = threadIdx.x & 31;
  const int task = blockIdx.x * kMergeWarps + (threadIdx.x >> 5);
  const int nv = n_q * q_len;  // virtual heads per sequence
  grid_dep_wait();
  grid_dep_trigger();
  if (task >= batch * nv) return;
  const int b = task / nv, vh = task - b * nv;
  const int VG = nv / kv_heads, h = vh / VG, v = vh - h * VG;  // virtual head v of KV head h
  int c = 0, jj = v, qh = vh, qi = 0;  // one query token: one chunk per KV head, v is the q-head's slot
  if (q_len > 1 || cg != VG) {
    c = v / cg;  // its chunk and slot in the chunk
    jj = v - c * cg;
    qh = h * (n_q / kv_heads) + v / q_len;
    qi = v % q_len;
  }
  const int pages = hist_tokens[b] / P;
  const int n_s = min((pages + pps - 1) / pps + residual_splits(P, q_len), max_splits);
  const int64_t item = static_cast<int64_t>(cg) * (D + 2);
  const float* base = ws + ((static_cast<int64_t>(b) * kv_heads + h) * (VG / cg) + c) * max_splits * item;
  const float* mstat = base + static_cast<int64_t>(cg) * D + jj;  // split s: mstat[s * item], lstat[s * item]
  OT* o = out + b * out_seq_stride + qh * out_head_stride + qi * out_tok_stride;
  const float* vals = base + static_cast<int64_t>(jj) * D;
  // Lane d covers channels (2d, 2d + 1) and (2d + 64, 2d + 65).
  const int d0 = 2 * lane, d1 = 2 * lane + 64;
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f, Lsum = 0.f;
  // Accumulates splits [s0, s0 + cnt) with weight wl of lane k for split s0 + k;
  // eight splits' loads are issued before any of them is used.
  auto accumulate = [&](int s0, int cnt, float wl) {
    int k = 0;
    for (; k + 8 <= cnt; k += 8) {
      float2 v0[8], v1[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float* row = vals + static_cast<int64_t>(s0 + k + u) * item;
        v0[u] = d0 < D ? *reinterpret_cast<const float2*>(row + d0) : make_float2(0.f, 0.f);
        v1[u] = d1 < D ? *reinterpret_cast<const float2*>(row + d1) : make_float2(0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float w = __shfl_sync(0xffffffffu, wl, k + u);
        fma2_acc(w, v0[u], a0, a1);
        fma2_acc(w, v1[u], a2, a3);
      }
    }
    for (; k < cnt; ++k) {
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
  };
  if (kFew > 0) {
    // At most kFew splits and head_dim 128 (the host's choice of this
    // instantiation): the values are loaded together with the statistics (one
    // round of loads instead of two), then summed in split order.  A separate
    // instantiation, so the general path keeps its smaller register footprint.
    float2 v0[kFew > 0 ? kFew : 1], v1[kFew > 0 ? kFew : 1];
#pragma unroll
    for (int u = 0; u < kFew; ++u) {
      if (u < n_s) {
        const float* row = vals + static_cast<int64_t>(u) * item;
        v0[u] = *reinterpret_cast<const float2*>(row + d0);
        v1[u] = *reinterpret_cast<const float2*>(row + d1);
      }
    }
    const float ms = lane < n_s ? mstat[lane * item] : -INFINITY;
    const float ls = lane < n_s ? mstat[lane * item + cg] : 0.f;
    float M = ms;
#pragma unroll
    for (int sh = 16; sh > 0; sh >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, sh));
    const float wl = ms == -INFINITY ? 0.f : expf(ms - M);
    Lsum = wl * ls;
#pragma unroll
    for (int u = 0; u < kFew; ++u) {
      if (u < n_s) {
        const float w = __shfl_sync(0xffffffffu, wl, u);
        fma2_acc(w, v0[u], a0, a1);
        fma2_acc(w, v1[u], a2, a3);
      }
    }
  } else if (n_s <= 32) {
    // Every split's statistics in one lane, read once.
    const float ms = lane < n_s ? mstat[lane * item] : -INFINITY;
    const float ls = lane < n_s ? mstat[lane * item + cg] : 0.f;
    float M = ms;
#pragma unroll
    for (int sh = 16; sh > 0; sh >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, sh));
    const float wl = ms == -INFINITY ? 0.f : expf(ms - M);
    Lsum = wl * ls;
    accumulate(0, n_s, wl);
  } else {
    float M = -INFINITY;
    for (int s = lane; s < n_s; s += 32) M = fmaxf(M, mstat[s * item]);
#pragma unroll
    for (int sh = 16; sh > 0; sh >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, sh));
    for (int s0 = 0; s0 < n_s; s0 += 32) {
      float wl = 0.f;
      if (s0 + lane < n_s) {
        const float ms = mstat[(s0 + lane) * item];
        if (ms != -INFINITY) {
          wl = expf(ms - M);
          Lsum = fmaf(wl, mstat[(s0 + lane) * item + cg], Lsum);
        }
      }
      accumulate(s0, min(32, n_s - s0), wl);
    }
  }
#pragma unroll
  for (int sh = 16; sh > 0; sh >>= 1) Lsum += __shfl_xor_sync(0xffffffffu, Lsum, sh);
  const float inv = Lsum > 0.f ? 1.0f / Lsum : 0.f;
  if (d0 < D) {
    Scalar<OT>::store(o + d0, a0 * inv);
    Scalar<OT>::store(o + d0 + 1, a1 * inv);
  }
  if (d1 < D) {
    Scalar<OT>::store(o + d1, a2 * inv);
    Scalar<OT>::store(o + d1 + 1, a3 * inv);
  }
}

static int n_slots_of(const lf_layout& L) { return 16 * L.words[0] + 8 * L.words[1] + 4 * L.words[2]; }

template <typename RT, typename QT>
static int launch_partial(const DecodeParams& p, cudaStream_t stream) {
  const DecodeSmem S = decode_smem(p.L, p.n_slots);
  auto kern = decode_partial_simt<RT, QT>;
  // The limit is raised once per size, outside any later stream capture of
  // the launch.
  cudaError_t e = raise_smem_limit(reinterpret_cast<const void*>(kern), S.total, false);
  if (e != cudaSuccess) {
    set_error("lf_decode_partial: shared memory %d B: %s", S.total, cudaGetErrorString(e));
    return LF_ERR_UNSUPPORTED;
  }
  dim3 grid(p.max_splits, p.L.kv_heads * p.n_chunks, p.batch);
  DecodeParams q = p;
  void* args[] = {&q};
  e = launch_programmatic(reinterpret_cast<const void*>(kern), grid, dim3(kDecThreads), S.total, stream, args);
  if (e != cudaSuccess) {
    set_error("lf_decode_partial: %s", cudaGetErrorString(e));
    return LF_ERR_LAUNCH;
  }
  return launch_status("lf_decode_partial");
}

template <typename RT>
static int dispatch_q(const DecodeParams& p, int q_dtype, cudaStream_t stream) {
  switch (q_dtype) {
    case LF_F32: return launch_partial<RT, float>(p, stream);
    case LF_F16: return launch_partial<RT, __half>(p, stream);
    case LF_BF16: return launch_partial<RT, __nv_bfloat16>(p, stream);
  }
  set_error("lf_decode_partial: q dtype %d", q_dtype);
  return LF_ERR_INVALID_ARGUMENT;
}

// Virtual heads per CTA: the largest divisor of gq * q_len that is at most kGQ
// (the whole GQA group for a decode step with gq <= 8).
static int chunk_heads(int gq, int q_len) {
  const int nv = gq * q_len;
  for (int c = kGQ; c > 1; --c)
    if (nv % c == 0) return c;
  return 1;
}

// K3 over the partials of a call with q_len query tokens per sequence.
static int launch_merge(const float* workspace, const int32_t* hist_tokens, int batch, int kv_heads, int n_q,
                        int q_len, int head_dim, int page_size, int pages_per_split, int max_splits, void* out,
                        int out_dtype, int64_t out_seq_stride, int64_t out_head_stride, int64_t out_tok_stride,
                        cudaStream_t s) {
  int cg = chunk_heads(n_q / kv_heads, q_len);
  // Every item has at most 16 (32) splits: the one-round-of-loads instantiation.
  const int few = head_dim != 128 ? 0 : max_splits <= 16 ? 16 : max_splits <= 32 ? 32 : 0;
  const int64_t tasks = static_cast<int64_t>(batch) * n_q * q_len;
  const dim3 grid(static_cast<unsigned>((tasks + kMergeWarps - 1) / kMergeWarps));
  const dim3 block(kMergeWarps * 32);
  const void* kern = nullptr;
  switch (out_dtype) {
    case LF_F32:
      kern = few == 16   ? reinterpret_cast<const void*>(decode_merge_kernel<float, 16>)
             : few == 32 ? reinterpret_cast<const void*>(decode_merge_kernel<float, 32>)
                         : reinterpret_cast<const void*>(decode_merge_kernel<float, 0>);
      break;
    case LF_F16:
      kern = few == 16   ? reinterpret_cast<const void*>(decode_merge_kernel<__half, 16>)
             : few == 32 ? reinterpret_cast<const void*>(decode_merge_kernel<__half, 32>)
                         : reinterpret_cast<const void*>(decode_merge_kernel<__half, 0>);
      break;
    case LF_BF16:
      kern = few == 16   ? reinterpret_cast<const void*>(decode_merge_kernel<__nv_bfloat16, 16>)
             : few == 32 ? reinterpret_cast<const void*>(decode_merge_kernel<__nv_bfloat16, 32>)
                         : reinterpret_cast<const void*>(decode_merge_kernel<__nv_bfloat16, 0>);
      break;
    default:
      set_error("lf_decode_merge: out dtype %d", out_dtype);
      return LF_ERR_INVALID_ARGUMENT;
  }
  void* args[] = {&workspace, &hist_tokens, &batch, &kv_heads, &n_q, &q_len, &cg,
                  &head_dim, &page_size, &pages_per_split, &max_splits, &out, &out_seq_stride,
                  &out_head_stride, &out_tok_stride};
  const cudaError_t e = launch_programmatic(kern, grid, block, 0, s, args);
  if (e != cudaSuccess) {
    set_error("lf_decode_merge: %s", cudaGetErrorString(e));
    return LF_ERR_LAUNCH;
  }
  return launch_status("lf_decode_merge");
}

}  // namespace lf

extern "C" int lf_decode_occupancy(const lf_layout* layout, int n_q, int pages_per_split) {
  if (layout == nullptr || n_q <= 0 || pages_per_split <= 0 || n_q % layout->kv_heads) return 0;
  const int gq = lf::chunk_heads(n_q / layout->kv_heads, 1);
  if (lf::tc_allowed() && lf::tc_supported(*layout, gq, pages_per_split))
    return lf::occupancy_tc(*layout, gq, pages_per_split);
  const lf::DecodeSmem S = lf::decode_smem(*layout, lf::n_slots_of(*layout));
  if (S.total > 227 * 1024) return 0;
  auto kern = lf::decode_partial_simt<__nv_bfloat16, __nv_bfloat16>;
  int blocks = 0;
  if (lf::raise_smem_limit(reinterpret_cast<const void*>(kern), S.total, false) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kern, lf::kDecThreads, S.total) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  return blocks;
}

extern "C" size_t lf_decode_workspace_bytes(int batch, int kv_heads, int n_q, int head_dim,
                                            int max_splits) {
  if (batch <= 0 || kv_heads <= 0 || n_q <= 0 || head_dim <= 0 || max_splits <= 0) return 0;
  const size_t gq = static_cast<size_t>(n_q / kv_heads);
  return static_cast<size_t>(batch) * kv_heads * max_splits * gq * (head_dim + 2) * sizeof(float);
}

extern "C" int lf_decode_max_splits_multi(int64_t max_pages, int pages_per_split, int page_size, int q_len) {
  if (max_pages < 0 || pages_per_split <= 0 || page_size <= 0 || q_len <= 0) return 0;
  return static_cast<int>((max_pages + pages_per_split - 1) / pages_per_split) +
         lf::residual_splits(page_size, q_len);
}

extern "C" int lf_decode_max_splits(int64_t max_pages, int pages_per_split, int page_size) {
  return lf_decode_max_splits_multi(max_pages, pages_per_split, page_size, 1);
}

namespace lf {

// Validated launch parameters of K2 (shared by lf_decode_partial and lf_decode).
static int prepare_decode(const char* who, const lf_layout* layout, const int32_t* rows, const uint16_t* kmeta,
                          const int32_t* slot_chan, const int32_t* hist_tokens, const void* tail_k,
                          const void* tail_v, int64_t tail_seq_stride, int64_t tail_head_stride,
                          const int32_t* tail_len, int resid_dtype, const void* k_new, const void* v_new,
                          int64_t new_seq_stride, int64_t new_head_stride, int64_t new_tok_stride, const void* q,
                          int q_dtype, int64_t q_seq_stride, int64_t q_head_stride, int64_t q_tok_stride,
                          int q_len, int batch, int n_q, float scaling, int pages_per_split, int max_splits,
                          float* workspace, int32_t* status, DecodeParams& p) {
  LF_CHECK_ARG(layout != nullptr, "%s: null layout", who);
  const lf_layout& L = *layout;
  LF_CHECK_ARG(rows && slot_chan && hist_tokens && tail_k && tail_v && tail_len && q && workspace,
               "%s: null pointer", who);
  LF_CHECK_ARG((k_new == nullptr) == (v_new == nullptr), "%s: k_new/v_new mismatch", who);
  LF_CHECK_ARG(batch > 0 && batch <= 65535 && n_q > 0 && n_q % L.kv_heads == 0,
               "%s: batch %d, n_q %d, kv_heads %d", who, batch, n_q, L.kv_heads);
  LF_CHECK_ARG(pages_per_split > 0 && max_splits >= 1 && max_splits <= 65535,
               "%s: pages_per_split %d, max_splits %d", who, pages_per_split, max_splits);
  LF_CHECK_ARG(q_len >= 1 && q_len <= 65535, "%s: q_len %d", who, q_len);
  LF_CHECK_ARG(max_splits >= lf_decode_max_splits_multi(L.row_cap / L.page_size, pages_per_split, L.page_size, q_len),
               "%s: max_splits %d cannot cover row_cap %lld with %d query tokens", who, max_splits,
               (long long)L.row_cap, q_len);
  {
    const int esz = resid_dtype == LF_F32 ? 4 : 2;
    const bool aligned = (reinterpret_cast<uintptr_t>(tail_k) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(tail_v) % 16 == 0) &&
                         (tail_seq_stride * esz) % 16 == 0 && (tail_head_stride * esz) % 16 == 0 &&
                         (k_new == nullptr || ((reinterpret_cast<uintptr_t>(k_new) % 16 == 0) &&
                                               (reinterpret_cast<uintptr_t>(v_new) % 16 == 0) &&
                                               (new_seq_stride * esz) % 16 == 0 && (new_head_stride * esz) % 16 == 0 &&
                                               (new_tok_stride * esz) % 16 == 0));
    LF_CHECK_ARG(aligned, "%s: residual / new-token rows must be 16-byte aligned", who);
  }
  LF_CHECK_ARG(resid_dtype == LF_F32 || resid_dtype == LF_F16 || resid_dtype == LF_BF16, "%s: residual dtype %d",
               who, resid_dtype);
  LF_CHECK_ARG(q_dtype == LF_F32 || q_dtype == LF_F16 || q_dtype == LF_BF16, "%s: q dtype %d", who, q_dtype);
  LF_CHECK_SUPPORTED(L.head_dim % 8 == 0, "decode head_dim %d must be a multiple of 8", L.head_dim);
  LF_CHECK_SUPPORTED(L.bit_v == 2, "decode supports bit_v 2, got %d", L.bit_v);
  LF_CHECK_SUPPORTED(L.k_group == L.page_size, "decode needs k_group == page_size (%d vs %d)",
                     L.k_group, L.page_size);
  LF_CHECK_SUPPORTED(L.v_group == L.head_dim, "decode needs v_group == head_dim (%d vs %d)",
                     L.v_group, L.head_dim);
  LF_CHECK_SUPPORTED(L.head_dim % 16 == 0 && L.head_dim <= kDecThreads,
                     "decode head_dim %d not supported", L.head_dim);
  LF_CHECK_SUPPORTED(L.page_size <= kDecThreads && L.page_size % 4 == 0,
                     "decode page_size %d must be a multiple of 4 and at most %d", L.page_size, kDecThreads);
  const int gq = n_q / L.kv_heads, cg = chunk_heads(gq, q_len), n_chunks = gq * q_len / cg;
  LF_CHECK_SUPPORTED(static_cast<int64_t>(L.kv_heads) * n_chunks <= 65535, "%s: %d KV heads x %d head chunks",
                     who, L.kv_heads, n_chunks);
  p = DecodeParams{};
  p.L = L;
  p.rows = rows;
  p.kmeta = kmeta;
  p.slot_chan = slot_chan;
  p.hist_tokens = hist_tokens;
  p.tail_k = tail_k;
  p.tail_v = tail_v;
  p.tail_seq_stride = tail_seq_stride;
  p.tail_head_stride = tail_head_stride;
  p.tail_len = tail_len;
  p.k_new = k_new;
  p.v_new = v_new;
  p.new_seq_stride = new_seq_stride;
  p.new_head_stride = new_head_stride;
  p.new_tok_stride = new_tok_stride;
  p.q = q;
  p.q_seq_stride = q_seq_stride;
  p.q_head_stride = q_head_stride;
  p.q_tok_stride = q_tok_stride;
  p.q_len = q_len;
  p.cg = cg;
  p.n_chunks = n_chunks;
  p.batch = batch;
  p.n_q = n_q;
  p.gq = gq;
  p.pps = pages_per_split;
  p.max_splits = max_splits;
  p.n_slots = n_slots_of(L);
  p.scaling = scaling;
  p.ws = workspace;
  p.status = status;
  p.resid_dtype = resid_dtype;
  p.q_dtype = q_dtype;
  return LF_OK;
}

// Whether the tensor-core kernel may serve the geometries it supports: yes,
// unless the environment variable LF_K2_KERNEL is "simt" (read once), which
// sends every call to the CUDA-core kernel for an A/B measurement of the two.
bool tc_allowed() {
  static const bool allowed = [] {
    const char* e = getenv("LF_K2_KERNEL");
    return !(e != nullptr && strcmp(e, "simt") == 0);
  }();
  return allowed;
}

// K2 on the kernel the geometry selects.
static int launch_decode(const DecodeParams& p, cudaStream_t s) {
  if (tc_allowed() && tc_supported(p.L, p.cg, p.pps)) return launch_partial_tc(p, p.resid_dtype, p.q_dtype, s);
  LF_CHECK_SUPPORTED(decode_smem(p.L, p.n_slots).total <= 227 * 1024, "decode shared memory %d B too large",
                     decode_smem(p.L, p.n_slots).total);
  switch (p.resid_dtype) {
    case LF_F32: return dispatch_q<float>(p, p.q_dtype, s);
    case LF_F16: return dispatch_q<__half>(p, p.q_dtype, s);
    default: return dispatch_q<__nv_bfloat16>(p, p.q_dtype, s);
  }
}

}  // namespace lf

extern "C" int lf_decode_partial(const lf_layout* layout, const int32_t* rows, const uint16_t* kmeta,
                                 const int32_t* slot_chan, const int32_t* hist_tokens,
                                 const void* tail_k, const void* tail_v, int64_t tail_seq_stride,
                                 int64_t tail_head_stride, const int32_t* tail_len, int resid_dtype,
                                 const void* k_new, const void* v_new, int64_t new_seq_stride,
                                 int64_t new_head_stride, const void* q, int q_dtype,
                                 int64_t q_seq_stride, int64_t q_head_stride, int batch, int n_q,
                                 float scaling, int pages_per_split, int max_splits,
                                 float* workspace, int32_t* status, lf_stream_t stream) {
  lf::DecodeParams p;
  const int st = lf::prepare_decode("lf_decode_partial", layout, rows, kmeta, slot_chan, hist_tokens, tail_k, tail_v,
                                    tail_seq_stride, tail_head_stride, tail_len, resid_dtype, k_new, v_new,
                                    new_seq_stride, new_head_stride, 0, q, q_dtype, q_seq_stride, q_head_stride, 0, 1,
                                    batch, n_q, scaling, pages_per_split, max_splits, workspace, status, p);
  if (st != LF_OK) return st;
  return lf::launch_decode(p, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int lf_decode(const lf_layout* layout, const int32_t* rows, const uint16_t* kmeta,
                         const int32_t* slot_chan, const int32_t* hist_tokens, const void* tail_k,
                         const void* tail_v, int64_t tail_seq_stride, int64_t tail_head_stride,
                         const int32_t* tail_len, int resid_dtype, const void* k_new, const void* v_new,
                         int64_t new_seq_stride, int64_t new_head_stride, const void* q, int q_dtype,
                         int64_t q_seq_stride, int64_t q_head_stride, int batch, int n_q, float scaling,
                         int pages_per_split, int max_splits, float* workspace, void* out, int out_dtype,
                         int64_t out_seq_stride, int64_t out_head_stride, int32_t* status, lf_stream_t stream) {
  return lf_decode_multi(layout, rows, kmeta, slot_chan, hist_tokens, tail_k, tail_v, tail_seq_stride,
                         tail_head_stride, tail_len, resid_dtype, k_new, v_new, new_seq_stride, new_head_stride, 0, q,
                         q_dtype, q_seq_stride, q_head_stride, 0, 1, batch, n_q, scaling, pages_per_split,
                         max_splits, workspace, out, out_dtype, out_seq_stride, out_head_stride, 0, status, stream);
}

extern "C" int lf_decode_multi(const lf_layout* layout, const int32_t* rows, const uint16_t* kmeta,
                               const int32_t* slot_chan, const int32_t* hist_tokens, const void* tail_k,
                               const void* tail_v, int64_t tail_seq_stride, int64_t tail_head_stride,
                               const int32_t* tail_len, int resid_dtype, const void* k_new, const void* v_new,
                               int64_t new_seq_stride, int64_t new_head_stride, int64_t new_tok_stride,
                               const void* q, int q_dtype, int64_t q_seq_stride, int64_t q_head_stride,
                               int64_t q_tok_stride, int q_len, int batch, int n_q, float scaling,
                               int pages_per_split, int max_splits, float* workspace, void* out, int out_dtype,
                               int64_t out_seq_stride, int64_t out_head_stride, int64_t out_tok_stride,
                               int32_t* status, lf_stream_t stream) {
  lf::DecodeParams p;
  const int st = lf::prepare_decode("lf_decode", layout, rows, kmeta, slot_chan, hist_tokens, tail_k, tail_v,
                                    tail_seq_stride, tail_head_stride, tail_len, resid_dtype, k_new, v_new,
                                    new_seq_stride, new_head_stride, new_tok_stride, q, q_dtype, q_seq_stride,
                                    q_head_stride, q_tok_stride, q_len, batch, n_q, scaling, pages_per_split,
                                    max_splits, workspace, status, p);
  if (st != LF_OK) return st;
  LF_CHECK_ARG(out != nullptr, "lf_decode: null output");
  LF_CHECK_ARG(out_dtype == LF_F32 || out_dtype == LF_F16 || out_dtype == LF_BF16, "lf_decode: out dtype %d",
               out_dtype);
  LF_CHECK_ARG(layout->head_dim % 2 == 0, "lf_decode: head_dim %d must be even", layout->head_dim);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int k2 = lf::launch_decode(p, s);
  if (k2 != LF_OK) return k2;
  return lf::launch_merge(workspace, hist_tokens, batch, layout->kv_heads, n_q, q_len, layout->head_dim,
                          layout->page_size, pages_per_split, max_splits, out, out_dtype, out_seq_stride,
                          out_head_stride, out_tok_stride, s);
}

extern "C" int lf_decode_merge(const float* workspace, const int32_t* hist_tokens, int batch,
                               int kv_heads, int n_q, int head_dim, int page_size,
                               int pages_per_split, int max_splits, void* out, int out_dtype,
                               int64_t out_seq_stride, int64_t out_head_stride,
                               lf_stream_t stream) {
  LF_CHECK_ARG(workspace && hist_tokens && out, "lf_decode_merge: null pointer");
  LF_CHECK_ARG(batch > 0 && batch <= 65535 && kv_heads > 0 && n_q % kv_heads == 0 && n_q <= 65535,
               "lf_decode_merge: batch %d n_q %d kv_heads %d", batch, n_q, kv_heads);
  LF_CHECK_ARG(page_size > 0 && pages_per_split > 0 && max_splits > 0 && head_dim > 0 && head_dim % 2 == 0,
               "lf_decode_merge: bad sizes");
  LF_CHECK_SUPPORTED(head_dim <= lf::kDecThreads, "lf_decode_merge: head_dim %d > %d", head_dim, lf::kDecThreads);
  return lf::launch_merge(workspace, hist_tokens, batch, kv_heads, n_q, 1, head_dim, page_size, pages_per_split,
                          max_splits, out, out_dtype, out_seq_stride, out_head_stride, 0,
                          reinterpret_cast<cudaStream_t>(stream));
}
