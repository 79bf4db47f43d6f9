// K1: page quantize + pack, and the history dequantizer.
//
// One CTA per (job, KV head).  The page's Key and Value tiles are staged in
// shared memory in their own dtype (16-byte streaming loads), the per-channel
// Key statistics (one min/max per k_group tokens, layout.py:86-99) and the
// per-token Value statistics (layout.py:122-129) are computed once, every
// element is replaced in place by its code (uniform work over the CTA), and
// every output word of the history rows is then assembled from the codes by
// one thread and written with coalesced stores.  Arithmetic is the reference's, bit for bit:
// fp32 max/min, IEEE subtract and divide, clamp to [1e-5, 1e5], round half to
// even, fp16 round-to-nearest-even of the stored scale/min (layout.py:12-18,98-99).

#include <type_traits>

#include "lf_common.cuh"

namespace lf {

constexpr int kPackThreads = 256;
constexpr int kPackSkip = -1;  // src_seq of a job that packs nothing

struct PackSmem {
  // Byte offsets into dynamic shared memory.
  int xk, xv, ksc, klo, krc, vsc, vlo, vrc, slotmap, wdesc, meta, total;
};

// The page's Key and Value tiles are staged in their own dtype (esz bytes per
// element): 64 KB for a bf16 128 x 128 page pair, so three CTAs fit on an SM.
__host__ __device__ inline PackSmem pack_smem(const lf_layout& L, int esz) {
  const int P = L.page_size, D = L.head_dim;
  const int G = P / L.k_group, NV = D / L.v_group;
  PackSmem s;
  int off = 0;
  s.xk = off; off += (P * D * esz + 15) / 16 * 16;
  s.xv = off; off += (P * D * esz + 15) / 16 * 16;
  s.ksc = off; off += G * D * 4;
  s.klo = off; off += G * D * 4;
  s.krc = off; off += G * D * 4;
  s.vsc = off; off += P * NV * 4;
  s.vlo = off; off += P * NV * 4;
  s.vrc = off; off += P * NV * 4;
  s.slotmap = off; off += 4 * D * 4;
  s.wdesc = off; off += L.row_words * 4;
  s.meta = off; off += G * L.meta_halves * 2;
  s.total = (off + 15) / 16 * 16;
  return s;
}

// Row-word descriptors: kind (0-2 Key tier, 3 Value codes, 4 fp16 halves) | index << 3.
enum { kWordValue = 3, kWordHalf = 4 };

template <typename T>
__global__ void __launch_bounds__(kPackThreads)
pack_pages_kernel(lf_layout L, const T* __restrict__ src_k, const T* __restrict__ src_v,
                  int64_t s_seq, int64_t s_head, int64_t s_tok, const int32_t* __restrict__ jobs,
                  int dst_batch, const int32_t* __restrict__ chan_code, int32_t* __restrict__ rows,
                  uint16_t* __restrict__ kmeta, int32_t* status) {
  extern __shared__ __align__(16) unsigned char smem[];
  const PackSmem S = pack_smem(L, sizeof(T));
  T* xk = reinterpret_cast<T*>(smem + S.xk);
  T* xv = reinterpret_cast<T*>(smem + S.xv);
  float* ksc = reinterpret_cast<float*>(smem + S.ksc);
  float* klo = reinterpret_cast<float*>(smem + S.klo);
  float* krc = reinterpret_cast<float*>(smem + S.krc);  // RN(1 / scale)
  float* vsc = reinterpret_cast<float*>(smem + S.vsc);
  float* vlo = reinterpret_cast<float*>(smem + S.vlo);
  float* vrc = reinterpret_cast<float*>(smem + S.vrc);
  int* slotmap = reinterpret_cast<int*>(smem + S.slotmap);
  int* wdesc = reinterpret_cast<int*>(smem + S.wdesc);
  uint16_t* meta = reinterpret_cast<uint16_t*>(smem + S.meta);

  const int job = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int P = L.page_size, D = L.head_dim, R = L.row_words, M = L.meta_halves;
  const int G = P / L.k_group, NV = D / L.v_group, H = L.kv_heads;
  const int src_seq = jobs[4 * job + 0], tok0 = jobs[4 * job + 1];
  const int dst_seq = jobs[4 * job + 2], dst_page = jobs[4 * job + 3];
  if (src_seq == kPackSkip) return;  // a job slot left empty by the device-side commit
  if (dst_seq < 0 || dst_seq >= dst_batch || dst_page < 0 ||
      static_cast<int64_t>(dst_page + 1) * P > L.row_cap ||
      static_cast<int64_t>(dst_page + 1) * G > L.group_cap || src_seq < 0 || tok0 < 0) {
    if (tid == 0 && status != nullptr) atomicExch(status, LF_ERR_OUT_OF_RANGE);
    return;
  }

  // 1. Stage the page in its dtype: 16-byte streaming loads (all of a
  // thread's loads issued before its stores) when the rows are aligned.
  const T* ksrc = src_k + src_seq * s_seq + h * s_head + static_cast<int64_t>(tok0) * s_tok;
  const T* vsrc = src_v + src_seq * s_seq + h * s_head + static_cast<int64_t>(tok0) * s_tok;
  constexpr int kVec = 16 / sizeof(T);
  const bool vec = (reinterpret_cast<uintptr_t>(ksrc) % 16 == 0) && (reinterpret_cast<uintptr_t>(vsrc) % 16 == 0) &&
                   (s_tok * static_cast<int64_t>(sizeof(T))) % 16 == 0 && D % kVec == 0;
  if (vec) {
    const int vpr = D / kVec, nvec = P * vpr;
    const bool pow2 = (vpr & (vpr - 1)) == 0;
    const int vshift = 31 - __clz(vpr);
    constexpr int kBatch = 8;
    for (int base = tid; base < nvec; base += kPackThreads * kBatch) {
      uint4 a[kBatch], c[kBatch];
#pragma unroll
      for (int r = 0; r < kBatch; ++r) {
        const int i = base + r * kPackThreads;
        if (i < nvec) {
          const int t = pow2 ? i >> vshift : i / vpr, e = (i - t * vpr) * kVec;
          a[r] = __ldcs(reinterpret_cast<const uint4*>(ksrc + t * s_tok + e));
          c[r] = __ldcs(reinterpret_cast<const uint4*>(vsrc + t * s_tok + e));
        }
      }
#pragma unroll
      for (int r = 0; r < kBatch; ++r) {
        const int i = base + r * kPackThreads;
        if (i < nvec) {
          reinterpret_cast<uint4*>(xk)[i] = a[r];
          reinterpret_cast<uint4*>(xv)[i] = c[r];
        }
      }
    }
  } else {
    for (int i = tid; i < P * D; i += kPackThreads) {
      const int t = i / D, e = i - t * D;
      xk[i] = ksrc[t * s_tok + e];
      xv[i] = vsrc[t * s_tok + e];
    }
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
  for (int w = tid; w < R; w += kPackThreads) {
    int d;
    if (w < L.vcode_off) {
      int b = 0;
      while (b < 2 && w >= L.code_off[b] + L.words[b]) ++b;
      d = b | ((w - L.code_off[b]) << 3);
    } else if (w < L.half_off) {
      d = kWordValue | ((w - L.vcode_off) << 3);
    } else {
      d = kWordHalf | ((w - L.half_off) << 3);
    }
    wdesc[w] = d;
  }
  __syncthreads();
  for (int c = tid; c < D; c += kPackThreads) {
    const int code = chan_code[h * D + c];
    const int tier = code >> 16, local = code & 0xFFFF;
    if (tier >= 0 && tier < 4 && local < L.width[tier]) slotmap[tier * D + local] = c;
  }
  // 2. Statistics, one work item per thread: (max, min) of a Key channel over
  // k_group tokens (layout.py:86-99), or of a token over v_group Value
  // channels (layout.py:122-129).
  for (int i = tid; i < G * D + P * NV; i += kPackThreads) {
    if (i < G * D) {
      const int g = i / D, c = i - g * D;
      const int code = chan_code[h * D + c];
      const int tier = code >> 16, local = code & 0xFFFF;
      if (tier < 0 || tier > 2) continue;
      float hi = -INFINITY, lo = INFINITY;
      const T* col = xk + g * L.k_group * D + c;
#pragma unroll 8
      for (int t = 0; t < L.k_group; ++t) {
        const float x = Scalar<T>::load(col + t * D);
        hi = fmaxf(hi, x);
        lo = fminf(lo, x);
      }
      const float sc = asym_scale(hi, lo, 2 << tier);
      ksc[i] = sc;
      klo[i] = lo;
      krc[i] = __frcp_rn(sc);
      if (local < L.width[tier]) {
        meta[g * M + L.scale_off[tier] + local] = float_to_half_bits(sc);
        meta[g * M + L.min_off[tier] + local] = float_to_half_bits(lo);
      }
    } else {
      const int j = i - G * D, t = j / NV, g = j - t * NV;
      float hi = -INFINITY, lo = INFINITY;
      const T* row = xv + t * D + g * L.v_group;
      // Neighbouring threads take neighbouring tokens (rows D elements apart,
      // the same bank): each starts at its own column so a warp's reads spread
      // over the banks.  Max and min do not depend on the order.
      int cc = t % L.v_group;
#pragma unroll 8
      for (int c = 0; c < L.v_group; ++c) {
        const float x = Scalar<T>::load(row + cc);
        hi = fmaxf(hi, x);
        lo = fminf(lo, x);
        if (++cc == L.v_group) cc = 0;
      }
      const float sc = asym_scale(hi, lo, L.bit_v);
      vsc[j] = sc;
      vlo[j] = lo;
      vrc[j] = __frcp_rn(sc);
    }
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

  // 3. Codes, in place: every staged Key element of an INT2/INT4/INT8
  // channel and every Value element is replaced by its code (same thread
  // reads and writes an element; uniform work across the CTA).
  using U = typename std::conditional<sizeof(T) == 4, uint32_t, uint16_t>::type;
  U* ck = reinterpret_cast<U*>(xk);
  U* cv = reinterpret_cast<U*>(xv);
  // Channel-major split of the threads: thread (c, r0) takes channel c of
  // tokens r0, r0 + rows_step, ... (no division per element).
  const int rows_step = D <= kPackThreads ? kPackThreads / D : 1;
  const int r0 = D <= kPackThreads ? tid / D : 0;
  for (int c = D <= kPackThreads ? tid % D : tid; c < D && r0 < rows_step; c += kPackThreads) {
    const int tier = __ldg(chan_code + h * D + c) >> 16;
    const bool keyed = tier >= 0 && tier <= 2;
    const int bits = keyed ? 2 << tier : 2;
    const int vg = c / L.v_group;
    int g = 0, g_end = L.k_group;  // Key group of token t, stepped as t advances
    float g_lo = klo[c], g_sc = ksc[c], g_rc = krc[c];  // that group's statistics, in registers
    for (int t = r0; t < P; t += rows_step) {
      if (t >= g_end) {
        while (t >= g_end) {
          ++g;
          g_end += L.k_group;
        }
        g_lo = klo[g * D + c];
        g_sc = ksc[g * D + c];
        g_rc = krc[g * D + c];
      }
      const int e = t * D + c;
      if (keyed) ck[e] = static_cast<U>(asym_code_rcp(Scalar<T>::load(xk + e), g_lo, g_sc, g_rc, bits));
      const int vi = t * NV + vg;
      cv[e] = static_cast<U>(asym_code_rcp(Scalar<T>::load(xv + e), vlo[vi], vsc[vi], vrc[vi], L.bit_v));
    }
  }
  __syncthreads();
  // 4. Assemble every word of the page's rows from the codes (consecutive
  // threads write consecutive words of a token row).
  int32_t* out_rows = rows + ((static_cast<int64_t>(dst_seq) * H + h) * L.row_cap +
                              static_cast<int64_t>(dst_page) * P) * R;
  const int warp = tid >> 5, lane = tid & 31;
  for (int t = warp; t < P; t += kPackThreads / 32)  // a warp per token row, lanes over its words
  for (int w = lane; w < R; w += 32) {
    const int i = t * R + w;
    const int desc = wdesc[w], kind = desc & 7, wi = desc >> 3;
    uint32_t word = 0;
    if (kind < kWordValue) {
      const int bits = 2 << kind, per = 32 / bits;
      const U* cr = ck + t * D;
      const int* sm = slotmap + kind * D + wi * per;
      const int nslot = min(per, L.width[kind] - wi * per);
      for (int k = 0; k < nslot; ++k) {
        const int c = sm[k];
        if (c >= 0) word |= static_cast<uint32_t>(cr[c]) << (k * bits);  // padding slot: code 0 (layout.py:95-97)
      }
    } else if (kind == kWordValue) {
      const int per = 32 / L.bit_v, d0 = wi * per, nd = min(per, D - d0);
      const U* cr = cv + t * D + d0;
      if (sizeof(U) == 2 && L.bit_v == 2 && nd == 16 && D % 8 == 0) {  // 16-byte aligned rows
        // 16 two-bit codes held as u16: two 16-byte reads, two codes per u32.
        const uint4 a = *reinterpret_cast<const uint4*>(cr);
        const uint4 b = *reinterpret_cast<const uint4*>(cr + 8);
        const uint32_t u[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) word |= ((u[k] & 3u) | ((u[k] >> 14) & 0xCu)) << (4 * k);
      } else {
        for (int k = 0; k < nd; ++k) word |= static_cast<uint32_t>(cr[k]) << (k * L.bit_v);
      }
    } else {
      for (int e = 0; e < 2; ++e) {
        const int hx = 2 * wi + e;
        uint32_t hv = 0;
        if (hx < L.width[3]) {
          const int c = slotmap[3 * D + hx];
          if (c >= 0) hv = float_to_half_bits(Scalar<T>::load(xk + t * D + c));  // layout.py:110
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
  const PackSmem S = pack_smem(L, sizeof(T));
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

int launch_pack_rows(const lf_layout& L, const void* k, const void* v, int dtype, int64_t s_seq, int64_t s_head,
                     int64_t s_tok, const int32_t* jobs, int n_jobs, int dst_batch, const int32_t* chan_code,
                     int32_t* rows, uint16_t* kmeta, int32_t* status, cudaStream_t stream) {
  LF_CHECK_SUPPORTED(pack_smem(L, dtype == LF_F32 ? 4 : 2).total <= 227 * 1024,
                     "K1: page %d x head_dim %d does not fit shared memory", L.page_size, L.head_dim);
  switch (dtype) {
    case LF_F32:
      return launch_pack<float>(L, k, v, s_seq, s_head, s_tok, jobs, n_jobs, dst_batch, chan_code, rows, kmeta,
                                status, stream);
    case LF_F16:
      return launch_pack<__half>(L, k, v, s_seq, s_head, s_tok, jobs, n_jobs, dst_batch, chan_code, rows, kmeta,
                                 status, stream);
    default:
      return launch_pack<__nv_bfloat16>(L, k, v, s_seq, s_head, s_tok, jobs, n_jobs, dst_batch, chan_code, rows,
                                        kmeta, status, stream);
  }
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
  LF_CHECK_SUPPORTED(lf::pack_smem(L, src_dtype == LF_F32 ? 4 : 2).total <= 227 * 1024,
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
