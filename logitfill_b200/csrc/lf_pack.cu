// K1: page quantize + pack, and the history dequantizer.
//
// One CTA per (job, KV head).  The page's Key and Value tiles are staged in
// shared memory as fp32 (exact for bf16/fp16/fp32 inputs), the per-channel
// Key statistics (one min/max per k_group tokens, layout.py:86-99) and the
// per-token Value statistics (layout.py:122-129) are computed once, and every
// output word of the history rows is then assembled by one thread and written
// with coalesced stores.  Arithmetic is the reference's, bit for bit:
// fp32 max/min, IEEE subtract and divide, clamp to [1e-5, 1e5], round half to
// even, fp16 round-to-nearest-even of the stored scale/min (layout.py:12-18,98-99).

#include "lf_common.cuh"

namespace lf {

constexpr int kPackThreads = 256;

struct PackSmem {
  // Byte offsets into dynamic shared memory.
  int xk, xv, ksc, klo, vsc, vlo, slotmap, meta, total;
};

__host__ __device__ inline PackSmem pack_smem(const lf_layout& L) {
  const int P = L.page_size, D = L.head_dim;
  const int G = P / L.k_group, NV = D / L.v_group;
  PackSmem s;
  int off = 0;
  s.xk = off; off += P * D * 4;
  s.xv = off; off += P * D * 4;
  s.ksc = off; off += G * D * 4;
  s.klo = off; off += G * D * 4;
  s.vsc = off; off += P * NV * 4;
  s.vlo = off; off += P * NV * 4;
  s.slotmap = off; off += 4 * D * 4;
  s.meta = off; off += G * L.meta_halves * 2;
  s.total = (off + 15) / 16 * 16;
  return s;
}

template <typename T>
__global__ void __launch_bounds__(kPackThreads)
pack_pages_kernel(lf_layout L, const T* __restrict__ src_k, const T* __restrict__ src_v,
                  int64_t s_seq, int64_t s_head, int64_t s_tok, const int32_t* __restrict__ jobs,
                  int dst_batch, const int32_t* __restrict__ chan_code, int32_t* __restrict__ rows,
                  uint16_t* __restrict__ kmeta, int32_t* status) {
  extern __shared__ __align__(16) unsigned char smem[];
  const PackSmem S = pack_smem(L);
  float* xk = reinterpret_cast<float*>(smem + S.xk);
  float* xv = reinterpret_cast<float*>(smem + S.xv);
  float* ksc = reinterpret_cast<float*>(smem + S.ksc);
  float* klo = reinterpret_cast<float*>(smem + S.klo);
  float* vsc = reinterpret_cast<float*>(smem + S.vsc);
  float* vlo = reinterpret_cast<float*>(smem + S.vlo);
  int* slotmap = reinterpret_cast<int*>(smem + S.slotmap);
  uint16_t* meta = reinterpret_cast<uint16_t*>(smem + S.meta);

  const int job = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int P = L.page_size, D = L.head_dim, R = L.row_words, M = L.meta_halves;
  const int G = P / L.k_group, NV = D / L.v_group, H = L.kv_heads;
  const int src_seq = jobs[4 * job + 0], tok0 = jobs[4 * job + 1];
  const int dst_seq = jobs[4 * job + 2], dst_page = jobs[4 * job + 3];
  if (dst_seq < 0 || dst_seq >= dst_batch || dst_page < 0 ||
      static_cast<int64_t>(dst_page + 1) * P > L.row_cap ||
      static_cast<int64_t>(dst_page + 1) * G > L.group_cap || src_seq < 0 || tok0 < 0) {
    if (tid == 0 && status != nullptr) atomicExch(status, LF_ERR_OUT_OF_RANGE);
    return;
  }

  // Stage the page (fp32, exact) and initialise the channel map and meta rows.
  const T* ksrc = src_k + src_seq * s_seq + h * s_head + static_cast<int64_t>(tok0) * s_tok;
  const T* vsrc = src_v + src_seq * s_seq + h * s_head + static_cast<int64_t>(tok0) * s_tok;
  for (int i = tid; i < P * D; i += kPackThreads) {
    const int t = i / D, c = i - t * D;
    xk[i] = Scalar<T>::load(ksrc + t * s_tok + c);
    xv[i] = Scalar<T>::load(vsrc + t * s_tok + c);
  }
  for (int i = tid; i < 4 * D; i += kPackThreads) slotmap[i] = -1;
  for (int i = tid; i < G * M; i += kPackThreads) {
    const int e = i % M;
    // Padding channels of a tier keep scale 1.0 and min 0 (layout.py:84-85).
    bool is_scale = false;
    for (int b = 0; b < 3; ++b)
      is_scale |= (e >= L.scale_off[b] && e < L.scale_off[b] + L.width[b]);
    meta[i] = is_scale ? 0x3C00 : 0;
  }
  __syncthreads();
  for (int c = tid; c < D; c += kPackThreads) {
    const int code = chan_code[h * D + c];
    const int tier = code >> 16, local = code & 0xFFFF;
    if (tier >= 0 && tier < 4 && local < L.width[tier]) slotmap[tier * D + local] = c;
  }
  // Key statistics: one (max, min) per channel per k_group tokens.
  for (int i = tid; i < G * D; i += kPackThreads) {
    const int g = i / D, c = i - g * D;
    const int code = chan_code[h * D + c];
    const int tier = code >> 16, local = code & 0xFFFF;
    if (tier < 0 || tier > 2) continue;
    const int bits = 2 << tier;
    float hi = -INFINITY, lo = INFINITY;
    for (int t = g * L.k_group; t < (g + 1) * L.k_group; ++t) {
      const float x = xk[t * D + c];
      hi = fmaxf(hi, x);
      lo = fminf(lo, x);
    }
    const float sc = asym_scale(hi, lo, bits);
    ksc[i] = sc;
    klo[i] = lo;
    if (local < L.width[tier]) {
      meta[g * M + L.scale_off[tier] + local] = float_to_half_bits(sc);
      meta[g * M + L.min_off[tier] + local] = float_to_half_bits(lo);
    }
  }
  // Value statistics: one (max, min) per token per v_group channels.
  for (int i = tid; i < P * NV; i += kPackThreads) {
    const int t = i / NV, g = i - t * NV;
    float hi = -INFINITY, lo = INFINITY;
    for (int c = g * L.v_group; c < (g + 1) * L.v_group; ++c) {
      const float x = xv[t * D + c];
      hi = fmaxf(hi, x);
      lo = fminf(lo, x);
    }
    vsc[i] = asym_scale(hi, lo, L.bit_v);
    vlo[i] = lo;
  }
  __syncthreads();
  // Largest stored Key scale of each group over the head's INT2/INT4/INT8
  // channels (positive fp16 values order as their bit patterns).
  for (int g = tid; g < G; g += kPackThreads) {
    uint16_t mx = 0;
    for (int b = 0; b < 3; ++b)
      for (int slot = 0; slot < L.width[b]; ++slot)
        if (slotmap[b * D + slot] >= 0) mx = max(mx, meta[g * M + L.scale_off[b] + slot]);
    meta[g * M + L.kmax_off] = mx;
  }

  // Assemble every word of the page's rows.
  int32_t* out_rows = rows + ((static_cast<int64_t>(dst_seq) * H + h) * L.row_cap +
                              static_cast<int64_t>(dst_page) * P) * R;
  for (int i = tid; i < P * R; i += kPackThreads) {
    const int t = i / R, w = i - t * R;
    uint32_t word = 0;
    if (w < L.vcode_off) {
      int b = 0;
      while (b < 2 && w >= L.code_off[b] + L.words[b]) ++b;
      const int bits = 2 << b, per = 32 / bits, wi = w - L.code_off[b];
      const int g = t / L.k_group;
      for (int k = 0; k < per; ++k) {
        const int slot = wi * per + k;
        if (slot >= L.width[b]) break;
        const int c = slotmap[b * D + slot];
        if (c < 0) continue;  // padding slot: code 0 (layout.py:95-97)
        const uint32_t q = asym_code(xk[t * D + c], klo[g * D + c], ksc[g * D + c], bits);
        word |= q << (k * bits);
      }
    } else if (w < L.half_off) {
      const int per = 32 / L.bit_v, wi = w - L.vcode_off;
      for (int k = 0; k < per; ++k) {
        const int d = wi * per + k;
        if (d >= D) break;
        const int g = d / L.v_group;
        const uint32_t q = asym_code(xv[t * D + d], vlo[t * NV + g], vsc[t * NV + g], L.bit_v);
        word |= q << (k * L.bit_v);
      }
    } else {
      for (int e = 0; e < 2; ++e) {
        const int hx = 2 * (w - L.half_off) + e;
        uint32_t hv = 0;
        if (hx < L.width[3]) {
          const int c = slotmap[3 * D + hx];
          if (c >= 0) hv = float_to_half_bits(xk[t * D + c]);  // layout.py:110
        } else if (hx < L.width[3] + NV) {
          hv = float_to_half_bits(vsc[t * NV + (hx - L.width[3])]);
        } else if (hx < L.width[3] + 2 * NV) {
          hv = float_to_half_bits(vlo[t * NV + (hx - L.width[3] - NV)]);
        }
        word |= hv << (16 * e);
      }
    }
    out_rows[i] = static_cast<int32_t>(word);
  }
  __syncthreads();  // the group maxima
  uint16_t* out_meta = kmeta + ((static_cast<int64_t>(dst_seq) * H + h) * L.group_cap +
                                static_cast<int64_t>(dst_page) * G) * M;
  for (int i = tid; i < G * M; i += kPackThreads) out_meta[i] = meta[i];
}

__global__ void dequantize_kernel(lf_layout L, const int32_t* __restrict__ rows,
                                  const uint16_t* __restrict__ kmeta,
                                  const int32_t* __restrict__ chan_code, int seq, int64_t tokens,
                                  float* __restrict__ out_k, float* __restrict__ out_v) {
  const int h = blockIdx.y, D = L.head_dim, R = L.row_words, M = L.meta_halves;
  const int NV = D / L.v_group;
  const int64_t base_row = (static_cast<int64_t>(seq) * L.kv_heads + h) * L.row_cap;
  const int64_t base_meta = (static_cast<int64_t>(seq) * L.kv_heads + h) * L.group_cap;
  const int64_t n = tokens * D;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / D;
    const int c = static_cast<int>(i - t * D);
    const uint32_t* row = reinterpret_cast<const uint32_t*>(rows + (base_row + t) * R);
    const uint16_t* row16 = reinterpret_cast<const uint16_t*>(row);
    const int code = chan_code[h * D + c];
    const int tier = code >> 16, local = code & 0xFFFF;
    float kv;
    if (tier < 3) {
      const int bits = 2 << tier, per = 32 / bits;
      const uint32_t q = (row[L.code_off[tier] + local / per] >> ((local % per) * bits)) &
                         ((1u << bits) - 1u);
      const uint16_t* meta = kmeta + (base_meta + t / L.k_group) * M;
      const float sc = half_bits_to_float(meta[L.scale_off[tier] + local]);
      const float mn = half_bits_to_float(meta[L.min_off[tier] + local]);
      kv = __fadd_rn(__fmul_rn(static_cast<float>(q), sc), mn);  // layout.py:157, no FMA
    } else {
      kv = half_bits_to_float(row16[2 * L.half_off + local]);
    }
    const int vper = 32 / L.bit_v, g = c / L.v_group;
    const uint32_t vq = (row[L.vcode_off + c / vper] >> ((c % vper) * L.bit_v)) &
                        ((1u << L.bit_v) - 1u);
    const float vs = half_bits_to_float(row16[2 * L.half_off + L.width[3] + g]);
    const float vm = half_bits_to_float(row16[2 * L.half_off + L.width[3] + NV + g]);
    const int64_t o = (static_cast<int64_t>(h) * tokens + t) * D + c;
    out_k[o] = kv;
    out_v[o] = __fadd_rn(__fmul_rn(static_cast<float>(vq), vs), vm);  // layout.py:181
  }
}

template <typename T>
static int launch_pack(const lf_layout& L, const void* k, const void* v, int64_t s_seq,
                       int64_t s_head, int64_t s_tok, const int32_t* jobs, int n_jobs,
                       int dst_batch, const int32_t* chan_code, int32_t* rows, uint16_t* kmeta,
                       int32_t* status, cudaStream_t stream) {
  const PackSmem S = pack_smem(L);
  auto kern = pack_pages_kernel<T>;
  // The limit is raised once per size, outside any later stream capture of
  // the launch.
  cudaError_t e = raise_smem_limit(reinterpret_cast<const void*>(kern), S.total, false);
  if (e != cudaSuccess) {
    set_error("lf_pack_pages: shared memory %d B: %s", S.total, cudaGetErrorString(e));
    return LF_ERR_UNSUPPORTED;
  }
  dim3 grid(n_jobs, L.kv_heads);
  kern<<<grid, kPackThreads, S.total, stream>>>(L, static_cast<const T*>(k), static_cast<const T*>(v),
                                                 s_seq, s_head, s_tok, jobs, dst_batch, chan_code,
                                                 rows, kmeta, status);
  return launch_status("lf_pack_pages");
}

}  // namespace lf

extern "C" int lf_pack_pages(const lf_layout* layout, const void* src_k, const void* src_v,
                             int src_dtype, int64_t src_seq_stride, int64_t src_head_stride,
                             int64_t src_tok_stride, const int32_t* jobs, int n_jobs,
                             int dst_batch, const int32_t* chan_code, int32_t* rows,
                             uint16_t* kmeta, int32_t* status, lf_stream_t stream) {
  LF_CHECK_ARG(layout != nullptr, "lf_pack_pages: null layout");
  if (n_jobs == 0) return LF_OK;
  LF_CHECK_ARG(n_jobs > 0 && n_jobs <= 65535 * 64, "lf_pack_pages: n_jobs %d", n_jobs);
  LF_CHECK_ARG(src_k && src_v && jobs && chan_code && rows, "lf_pack_pages: null pointer");
  LF_CHECK_ARG(layout->meta_halves == 0 || kmeta, "lf_pack_pages: null kmeta");
  const lf_layout& L = *layout;
  LF_CHECK_SUPPORTED(lf::pack_smem(L).total <= 227 * 1024,
                     "lf_pack_pages: page %d x head_dim %d does not fit shared memory", L.page_size,
                     L.head_dim);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (src_dtype) {
    case LF_F32:
      return lf::launch_pack<float>(L, src_k, src_v, src_seq_stride, src_head_stride,
                                    src_tok_stride, jobs, n_jobs, dst_batch, chan_code, rows, kmeta,
                                    status, s);
    case LF_F16:
      return lf::launch_pack<__half>(L, src_k, src_v, src_seq_stride, src_head_stride,
                                     src_tok_stride, jobs, n_jobs, dst_batch, chan_code, rows,
                                     kmeta, status, s);
    case LF_BF16:
      return lf::launch_pack<__nv_bfloat16>(L, src_k, src_v, src_seq_stride, src_head_stride,
                                            src_tok_stride, jobs, n_jobs, dst_batch, chan_code,
                                            rows, kmeta, status, s);
    default:
      lf::set_error("lf_pack_pages: dtype %d", src_dtype);
      return LF_ERR_INVALID_ARGUMENT;
  }
}

extern "C" int lf_dequantize(const lf_layout* layout, const int32_t* rows, const uint16_t* kmeta,
                             const int32_t* chan_code, int seq, int64_t tokens, float* out_k,
                             float* out_v, lf_stream_t stream) {
  LF_CHECK_ARG(layout != nullptr, "lf_dequantize: null layout");
  if (tokens == 0) return LF_OK;
  LF_CHECK_ARG(tokens > 0 && tokens <= layout->row_cap, "lf_dequantize: tokens %lld",
               (long long)tokens);
  LF_CHECK_ARG(rows && chan_code && out_k && out_v && seq >= 0, "lf_dequantize: bad argument");
  const int64_t n = tokens * layout->head_dim;
  int blocks = static_cast<int>((n + 255) / 256);
  if (blocks > 4096) blocks = 4096;
  dim3 grid(blocks, layout->kv_heads);
  lf::dequantize_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      *layout, rows, kmeta, chan_code, seq, tokens, out_k, out_v);
  return lf::launch_status("lf_dequantize");
}
