// K1: page quantize + pack, and the history dequantizer.
//
// One CTA of 256 threads per (job, KV head).  The page's Key and Value tiles
// are staged in shared memory in their own dtype (16-byte streaming loads,
// rows padded to an odd number of 32-bit words so a warp reading one column
// of 32 rows touches 32 banks).  Statistics: each Key channel's max / min over
// its k_group tokens (layout.py:86-99) and each token's over its v_group Value
// channels (layout.py:122-129), on packed 16-bit pairs.  Each Key tier slot
// then gets a record {scale, RN(1/scale), min, channel offset}; codes and
// words are formed one thread per token row and role (128 threads build the
// Key tier words and the fp16 words of their rows, 128 the Value code words),
// written to a staged copy of the page's rows and stored coalesced.
// Arithmetic is the reference's, bit for bit: fp32 max/min, IEEE subtract and
// divide, clamp to [1e-5, 1e5], round half to even, fp16 round-to-nearest-even
// of the stored scale/min (layout.py:12-18,98-99); the per-element division is
// Markstein's (lf_common.cuh) and the rounding a magic-number add (pack_code).

#include <type_traits>

#include "lf_common.cuh"

namespace lf {

constexpr int kPackThreads = 256;
constexpr int kPackRole = kPackThreads / 2;  // threads per role: Key words / Value words
constexpr int kPackRows = 128;               // token rows one pass of a role covers
constexpr int kPackParts = kPackRole / kPackRows;  // threads of a role per token row
constexpr int kPackSkip = -1;                 // src_seq of a job that packs nothing

// Shared memory of one (job, KV head).  The page's Key and Value tiles are
// staged in their own dtype with a row stride of `sw` 32-bit words: odd, so
// the 32 rows a warp reads at one column lie in 32 banks, and at least one
// word longer than the row, so every row ends in a zero word (`pad_off`,
// the element a padding slot reads).
struct PackSmem {
  int xk, xv, chan, kslot, vstat, h16, out, meta, kmax, total;
  int sw;      // staged row stride, 32-bit words
  int pad_off; // byte offset of the zero word in a staged row
  int nslot;   // Key tier slots the row words hold: 16 words0 + 8 words1 + 4 words2
  int tbase1, tbase2;  // first slot of the INT4 / INT8 tiers
};

__host__ __device__ inline int round16(int x) { return (x + 15) / 16 * 16; }

__host__ __device__ inline PackSmem pack_smem(const lf_layout& L, int esz) {
  const int P = L.page_size, D = L.head_dim, G = P / L.k_group, NV = D / L.v_group;
  PackSmem s;
  const int data_words = (D * esz + 3) / 4;
  s.sw = data_words + ((data_words & 1) ? 2 : 1);
  s.pad_off = data_words * 4;
  s.tbase1 = 16 * L.words[0];
  s.tbase2 = s.tbase1 + 8 * L.words[1];
  s.nslot = s.tbase2 + 4 * L.words[2];
  int off = 0;
  s.xk = off; off += round16(P * s.sw * 4);
  s.xv = off; off += round16(P * s.sw * 4);
  s.chan = off; off += round16(D * 4);
  s.kslot = off; off += G * (s.nslot > 0 ? s.nslot : 2) * 16;
  s.vstat = off; off += P * NV * 16;
  s.h16 = off; off += round16((L.width[3] > 0 ? L.width[3] : 1) * 4);
  s.out = off; off += round16(P * L.row_words * 4);
  s.meta = off; off += round16(G * L.meta_halves * 2);
  s.kmax = off; off += round16(G * 4);
  s.total = off;
  return s;
}

// Records of two adjacent Key tier slots (group g, tier slots 2i and 2i+1),
// lane e for slot 2i + e, laid out so each field pair is one fp32x2 operand:
// -scale, RN(1/scale), min, and the byte offset of the slot's channel in a
// staged row.  A padding slot (past the head's channel count, or past the
// tier width) reads the zero word of the row with scale 1, min 0: its code
// is 0 (layout.py:95-97).  Every tier starts at an even slot.
struct __align__(16) SlotPair {
  float nscale[2], rcp[2];
  float lo[2];
  int off[2];
};

template <typename T>
__device__ __forceinline__ float load_elem(const unsigned char* p) {
  return Scalar<T>::load(reinterpret_cast<const T*>(p));
}

// Running max / min of two adjacent 16-bit elements (exact: the max of two
// bf16 or fp16 values is the max of their fp32 values).
template <typename T> struct Pair;
template <> struct Pair<__nv_bfloat16> {
  using V = __nv_bfloat162;
  static __device__ __forceinline__ V lowest() { return __nv_bfloat162(__ushort_as_bfloat16(0xFF80), __ushort_as_bfloat16(0xFF80)); }
  static __device__ __forceinline__ V highest() { return __nv_bfloat162(__ushort_as_bfloat16(0x7F80), __ushort_as_bfloat16(0x7F80)); }
  static __device__ __forceinline__ V max(V a, V b) { return __hmax2(a, b); }
  static __device__ __forceinline__ V min(V a, V b) { return __hmin2(a, b); }
  static __device__ __forceinline__ float lo(V a) { return __low2float(a); }
  static __device__ __forceinline__ float hi(V a) { return __high2float(a); }
};
template <> struct Pair<__half> {
  using V = __half2;
  static __device__ __forceinline__ V lowest() { return __half2(__ushort_as_half(0xFC00), __ushort_as_half(0xFC00)); }
  static __device__ __forceinline__ V highest() { return __half2(__ushort_as_half(0x7C00), __ushort_as_half(0x7C00)); }
  static __device__ __forceinline__ V max(V a, V b) { return __hmax2(a, b); }
  static __device__ __forceinline__ V min(V a, V b) { return __hmin2(a, b); }
  static __device__ __forceinline__ float lo(V a) { return __low2float(a); }
  static __device__ __forceinline__ float hi(V a) { return __high2float(a); }
};

// Key statistics of channels c0 .. c0+n-1 (n = 2 for a 16-bit pair, 1 otherwise)
// of group g over tokens [g kg, (g+1) kg), split over SPLIT consecutive lanes
// of full warps.  With SPLIT > 1 (kg a multiple of 32), part h takes tokens
// 32 b + (32 / SPLIT) h + i of every 32-token block b, i < 32 / SPLIT: at each
// step the parts of one warp are 32 / SPLIT rows apart, so (rows being an odd
// number of words) they read different banks, and every part runs the same
// loop.  Every lane of the split returns the combined max / min.
template <typename T, int SPLIT>
__device__ __forceinline__ void key_stats(const unsigned char* xk, int sw, int g, int kg, int c0, int h,
                                          float (&hi)[2], float (&lo)[2]) {
  constexpr int kSub = 32 / SPLIT;
  const int stride = sw * 4;
  const int t0 = g * kg + (SPLIT > 1 ? kSub * h : 0);
  // visit(offset): the element of token t0 + offset
  auto scan = [&](auto visit) {
    if (SPLIT > 1) {
      for (int b = 0; b < kg; b += 32) {
#pragma unroll
        for (int i = 0; i < kSub; ++i) visit(b + i);
      }
    } else {
#pragma unroll 8
      for (int j = 0; j < kg; ++j) visit(j);
    }
  };
  if constexpr (sizeof(T) == 2) {
    using PR = Pair<T>;
    typename PR::V mx = PR::lowest(), mn = PR::highest();
    const unsigned char* col = xk + c0 * 2 + t0 * stride;
    scan([&](int j) {
      const typename PR::V v = *reinterpret_cast<const typename PR::V*>(col + j * stride);
      mx = PR::max(mx, v);
      mn = PR::min(mn, v);
    });
    hi[0] = PR::lo(mx); hi[1] = PR::hi(mx);
    lo[0] = PR::lo(mn); lo[1] = PR::hi(mn);
  } else {
    float mx = -INFINITY, mn = INFINITY;
    const unsigned char* col = xk + c0 * 4 + t0 * stride;
    scan([&](int j) {
      const float v = *reinterpret_cast<const float*>(col + j * stride);
      mx = fmaxf(mx, v);
      mn = fminf(mn, v);
    });
    hi[0] = hi[1] = mx;
    lo[0] = lo[1] = mn;
  }
#pragma unroll
  for (int o = 1; o < SPLIT; o <<= 1) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      hi[e] = fmaxf(hi[e], __shfl_xor_sync(0xffffffffu, hi[e], o));
      lo[e] = fminf(lo[e], __shfl_xor_sync(0xffffffffu, lo[e], o));
    }
  }
}

// Two adjacent 16-bit elements (one 32-bit shared load) as fp32.
template <typename T>
__device__ __forceinline__ float2 load_pair(const unsigned char* p);
template <>
__device__ __forceinline__ float2 load_pair<__nv_bfloat16>(const unsigned char* p) {
  const uint32_t u = *reinterpret_cast<const uint32_t*>(p);
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
}
template <>
__device__ __forceinline__ float2 load_pair<__half>(const unsigned char* p) {
  return __half22float2(*reinterpret_cast<const __half2*>(p));
}
template <>
__device__ __forceinline__ float2 load_pair<float>(const unsigned char* p) {
  return make_float2(*reinterpret_cast<const float*>(p), *reinterpret_cast<const float*>(p + 4));
}

// A Key word of token row `row`: BITS-bit codes of the slots of the pairs
// rec[0 .. 16 / BITS), two codes per packed fp32x2 evaluation.
template <typename T, int BITS>
__device__ __forceinline__ uint32_t key_word(const unsigned char* row, const SlotPair* rec) {
  constexpr int kPer = 32 / BITS;
  constexpr uint32_t kQmax = (1u << BITS) - 1u;
  uint32_t word = 0, bias = 0;
#pragma unroll
  for (int k = 0; k < kPer; k += 2) {
    const float4 a = *reinterpret_cast<const float4*>(rec[k / 2].nscale);  // -scale x2, rcp x2
    const int4 b = *reinterpret_cast<const int4*>(rec[k / 2].lo);          // min x2, offset x2
    const float2 x = make_float2(load_elem<T>(row + b.z), load_elem<T>(row + b.w));
    const uint2 c = pack_bits2(x, make_float2(__int_as_float(b.x), __int_as_float(b.y)), make_float2(a.x, a.y),
                               make_float2(a.z, a.w), kQmax);
    // the fields are disjoint: adding is OR-ing (one shift-add); each sum
    // carries kMagicBits, taken off once at the end (mod 2^32)
    word += c.x << (k * BITS);
    word += c.y << ((k + 1) * BITS);
    bias += (kMagicBits << (k * BITS)) + (kMagicBits << ((k + 1) * BITS));
  }
  return word - bias;
}

template <typename T>
__global__ void __launch_bounds__(kPackThreads, 2)
pack_pages_kernel(const __grid_constant__ lf_layout L, const T* __restrict__ src_k, const T* __restrict__ src_v,
                  int64_t s_seq, int64_t s_head, int64_t s_tok, const int32_t* __restrict__ jobs,
                  int dst_batch, const int32_t* __restrict__ chan_code, int32_t* __restrict__ rows,
                  uint16_t* __restrict__ kmeta, int32_t* status) {
  extern __shared__ __align__(16) unsigned char smem[];
  const PackSmem S = pack_smem(L, sizeof(T));
  unsigned char* xk = smem + S.xk;
  unsigned char* xv = smem + S.xv;
  int* chan = reinterpret_cast<int*>(smem + S.chan);        // chan_code of the head
  SlotPair* kslot = reinterpret_cast<SlotPair*>(smem + S.kslot);
  float4* vstat = reinterpret_cast<float4*>(smem + S.vstat);  // [token][v group]: scale, rcp, min
  int* h16 = reinterpret_cast<int*>(smem + S.h16);          // FP16 slot -> byte offset in a row
  uint32_t* out = reinterpret_cast<uint32_t*>(smem + S.out);
  uint16_t* meta = reinterpret_cast<uint16_t*>(smem + S.meta);
  // Per group: the largest stored INT2/INT4/INT8 Key scale as fp16 bits
  // (positive fp16 values order as their bit patterns), raised by every record.
  unsigned int* kmax_s = reinterpret_cast<unsigned int*>(smem + S.kmax);

  const int job = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int P = L.page_size, D = L.head_dim, R = L.row_words, M = L.meta_halves;
  const int kg = L.k_group, G = P / kg, NV = D / L.v_group, H = L.kv_heads;
  const int src_seq = jobs[4 * job + 0], tok0 = jobs[4 * job + 1];
  const int dst_seq = jobs[4 * job + 2], dst_page = jobs[4 * job + 3];
  if (src_seq == kPackSkip) return;  // a job slot left empty by the device-side commit
  if (dst_seq < 0 || dst_seq >= dst_batch || dst_page < 0 ||
      static_cast<int64_t>(dst_page + 1) * P > L.row_cap ||
      static_cast<int64_t>(dst_page + 1) * G > L.group_cap || src_seq < 0 || tok0 < 0) {
    if (tid == 0 && status != nullptr) atomicExch(status, LF_ERR_OUT_OF_RANGE);
    return;
  }
  const int sw = S.sw, sw4 = S.sw * 4;

  // 1. Stage the page in its dtype, rows sw words apart: 16-byte streaming
  // loads (all of a thread's loads issued before its stores) when the rows
  // are aligned, 32-bit shared stores; the zero word after every row.
  const T* ksrc = src_k + src_seq * s_seq + h * s_head + static_cast<int64_t>(tok0) * s_tok;
  const T* vsrc = src_v + src_seq * s_seq + h * s_head + static_cast<int64_t>(tok0) * s_tok;
  constexpr int kVec = 16 / sizeof(T);
  const bool vec = (reinterpret_cast<uintptr_t>(ksrc) % 16 == 0) && (reinterpret_cast<uintptr_t>(vsrc) % 16 == 0) &&
                   (s_tok * static_cast<int64_t>(sizeof(T))) % 16 == 0 && D % kVec == 0;
  // The head's channel codes are loaded first and stored after the staging,
  // and the tables that need no input are filled while the page's loads are
  // in flight.
  const int chv = tid < D ? chan_code[h * D + tid] : 0;
  auto init_tables = [&]() {
    for (int i = tid; i < L.width[3]; i += kPackThreads) h16[i] = S.pad_off;  // padding slots read 0
    for (int i = tid; i < G * M; i += kPackThreads) {
      const int e = i % M;
      // Padding channels of a tier keep scale 1.0 and min 0 (layout.py:84-85).
      bool is_scale = false;
      for (int b = 0; b < 3; ++b)
        is_scale |= (e >= L.scale_off[b] && e < L.scale_off[b] + L.width[b]);
      meta[i] = is_scale ? 0x3C00 : 0;
    }
    for (int i = tid; i < G * S.nslot / 2; i += kPackThreads)
      kslot[i] = SlotPair{{-1.0f, -1.0f}, {1.0f, 1.0f}, {0.0f, 0.0f}, {S.pad_off, S.pad_off}};
    for (int g = tid; g < G; g += kPackThreads) kmax_s[g] = 0u;
  };
  bool tables_done = false;
  if (vec && kPackThreads % (D / kVec) == 0) {
    // Each thread keeps one 16-byte column of the rows: no division per vector.
    const int vpr = D / kVec, rstep = kPackThreads / vpr;
    const int tr = tid / vpr, ec = (tid - tr * vpr) * kVec;
    constexpr int kBatch = 8;
    for (int t0 = tr; t0 < P; t0 += rstep * kBatch) {
      uint4 a[kBatch], c[kBatch];
#pragma unroll
      for (int r = 0; r < kBatch; ++r) {
        const int t = t0 + r * rstep;
        if (t < P) {
          a[r] = __ldcs(reinterpret_cast<const uint4*>(ksrc + t * s_tok + ec));
          c[r] = __ldcs(reinterpret_cast<const uint4*>(vsrc + t * s_tok + ec));
        }
      }
      if (!tables_done) {
        init_tables();
        tables_done = true;
      }
#pragma unroll
      for (int r = 0; r < kBatch; ++r) {
        const int t = t0 + r * rstep;
        if (t < P) {
          const int wo = t * sw + ec * static_cast<int>(sizeof(T)) / 4;
          uint32_t* dk = reinterpret_cast<uint32_t*>(xk) + wo;
          uint32_t* dv = reinterpret_cast<uint32_t*>(xv) + wo;
          dk[0] = a[r].x; dk[1] = a[r].y; dk[2] = a[r].z; dk[3] = a[r].w;
          dv[0] = c[r].x; dv[1] = c[r].y; dv[2] = c[r].z; dv[3] = c[r].w;
        }
      }
    }
  } else if (vec) {
    const int vpr = D / kVec, nvec = P * vpr;
    for (int i = tid; i < nvec; i += kPackThreads) {
      const int t = i / vpr, e = (i - t * vpr) * kVec;
      const uint4 a = __ldcs(reinterpret_cast<const uint4*>(ksrc + t * s_tok + e));
      const uint4 c = __ldcs(reinterpret_cast<const uint4*>(vsrc + t * s_tok + e));
      const int wo = t * sw + e * static_cast<int>(sizeof(T)) / 4;
      uint32_t* dk = reinterpret_cast<uint32_t*>(xk) + wo;
      uint32_t* dv = reinterpret_cast<uint32_t*>(xv) + wo;
      dk[0] = a.x; dk[1] = a.y; dk[2] = a.z; dk[3] = a.w;
      dv[0] = c.x; dv[1] = c.y; dv[2] = c.z; dv[3] = c.w;
    }
  } else {
    for (int i = tid; i < P * D; i += kPackThreads) {
      const int t = i / D, e = i - t * D;
      reinterpret_cast<T*>(xk + t * sw4)[e] = ksrc[t * s_tok + e];
      reinterpret_cast<T*>(xv + t * sw4)[e] = vsrc[t * s_tok + e];
    }
  }
  {
    const int data_words = S.pad_off / 4;
    for (int t = tid; t < P; t += kPackThreads) {
      for (int w = data_words; w < sw; ++w) {
        reinterpret_cast<uint32_t*>(xk)[t * sw + w] = 0u;
        reinterpret_cast<uint32_t*>(xv)[t * sw + w] = 0u;
      }
    }
    // A 16-bit tile whose row has an odd number of elements: the half word
    // after the last element is zeroed with the rest of the row's tail.
    if (sizeof(T) == 2 && (D & 1)) {
      for (int t = tid; t < P; t += kPackThreads) {
        reinterpret_cast<uint16_t*>(xk + t * sw4)[D] = 0;
        reinterpret_cast<uint16_t*>(xv + t * sw4)[D] = 0;
      }
    }
  }
  if (!tables_done) init_tables();
  if (tid < D) chan[tid] = chv;
  for (int c = tid + kPackThreads; c < D; c += kPackThreads) chan[c] = chan_code[h * D + c];
  __syncthreads();
  // FP16 tier slot -> byte offset of its channel in a staged row (read by the
  // code phase, after the statistics' barrier).
  for (int c = tid; c < D; c += kPackThreads) {
    const int code = chan[c];
    const int local = code & 0xFFFF;
    if ((code >> 16) == 3 && local < L.width[3]) h16[local] = c * static_cast<int>(sizeof(T));
  }

  // 2. Statistics.  Threads 0..127: Key channel (pairs of 16-bit elements)
  // over each group of k_group tokens (layout.py:86-99); threads 128..255:
  // Value token over each group of v_group channels (layout.py:122-129).
  if (tid < kPackRole) {
    const int cw = sizeof(T) == 2 ? 2 : 1;  // channels per task
    const int tasks = G * ((D + cw - 1) / cw);
    // Split a channel's tokens over 2 or 4 lanes when the tasks leave threads
    // idle; a split runs on whole warps (its lanes shuffle) and leaves every
    // part at least 32 tokens.
    int split = 1;
    for (int s2 = 4; s2 > 1; s2 >>= 1) {
      if (tasks * s2 <= kPackRole && (tasks * s2) % 32 == 0 && kg % 32 == 0 && kg / s2 >= 32) {
        split = s2;
        break;
      }
    }
    for (int i = tid; i < tasks * split; i += kPackRole) {
      const int task = i / split, part = i - task * split;
      const int g = task / ((D + cw - 1) / cw), c0 = (task - g * ((D + cw - 1) / cw)) * cw;
      float hi[2], lo[2];
      if (split == 4) key_stats<T, 4>(xk, sw, g, kg, c0, part, hi, lo);
      else if (split == 2) key_stats<T, 2>(xk, sw, g, kg, c0, part, hi, lo);
      else key_stats<T, 1>(xk, sw, g, kg, c0, part, hi, lo);
      // Slot record and meta entries of channel c0 + e.
      auto record = [&](int e, float hv, float lv) {
        if (e >= cw || c0 + e >= D) return;
        const int code = chan[c0 + e];
        const int tier = code >> 16, local = code & 0xFFFF;
        if (tier < 0 || tier > 2 || local >= L.width[tier]) return;
        const float sc = asym_scale(hv, lv, 2 << tier);
        const int base = tier == 0 ? 0 : tier == 1 ? S.tbase1 : S.tbase2;
        const int si = g * S.nslot + base + local;
        SlotPair& sp = kslot[si >> 1];
        sp.nscale[si & 1] = -sc;
        sp.rcp[si & 1] = __frcp_rn(sc);
        sp.lo[si & 1] = lv;
        sp.off[si & 1] = (c0 + e) * static_cast<int>(sizeof(T));
        const uint16_t sb = float_to_half_bits(sc);
        meta[g * M + L.scale_off[tier] + local] = sb;
        meta[g * M + L.min_off[tier] + local] = float_to_half_bits(lv);
        atomicMax(kmax_s + g, static_cast<unsigned int>(sb));
      };
      if (split > 1) {
        // Every lane of the split holds both channels' statistics: parts 0
        // and 1 each take one channel's record, in one converged pass.
        if (part < 2) record(part, part ? hi[1] : hi[0], part ? lo[1] : lo[0]);
      } else {
#pragma unroll
        for (int e = 0; e < 2; ++e) record(e, hi[e], lo[e]);
      }
    }
  } else {
    // Two lanes per (token, v group) when every lane has a partner: each
    // scans half of the group's channel pairs, the second half starting 16
    // words in, so the two lanes of a token read different banks.
    const int vg = L.v_group, tasks = P * NV;
    const bool pairs = sizeof(T) == 2 && vg % 4 == 0;
    const int split = (pairs && tasks * 2 <= kPackRole && (tasks * 2) % 32 == 0) ? 2 : 1;
    for (int i = tid - kPackRole; i < tasks * split; i += kPackRole) {
      const int j = i / split, h = i - j * split;
      const int t = j / NV, g = j - t * NV;
      const unsigned char* row = xv + t * sw4 + g * vg * static_cast<int>(sizeof(T));
      float hi = -INFINITY, lo = INFINITY;
      if constexpr (sizeof(T) == 2) {
        if (pairs) {
          using PR = Pair<T>;
          typename PR::V mx = PR::lowest(), mn = PR::highest();
          const int nw = vg / 2 / split;                 // 32-bit words of this lane's part
          const unsigned char* base = row + h * nw * 4;
          const int rot = (h == 1 && nw >= 32) ? 16 : 0;
          auto scan = [&](int k0, int k1) {
#pragma unroll 8
            for (int k = k0; k < k1; ++k) {
              const typename PR::V v = *reinterpret_cast<const typename PR::V*>(base + k * 4);
              mx = PR::max(mx, v);
              mn = PR::min(mn, v);
            }
          };
          scan(rot, nw);
          scan(0, rot);
          hi = fmaxf(PR::lo(mx), PR::hi(mx));
          lo = fminf(PR::lo(mn), PR::hi(mn));
        } else {
          for (int c = 0; c < vg; ++c) {
            const float x = load_elem<T>(row + c * 2);
            hi = fmaxf(hi, x);
            lo = fminf(lo, x);
          }
        }
      } else {
#pragma unroll 8
        for (int c = 0; c < vg; ++c) {
          const float x = load_elem<T>(row + c * 4);
          hi = fmaxf(hi, x);
          lo = fminf(lo, x);
        }
      }
      if (split == 2) {
        hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, 1));
        lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, 1));
      }
      if (h == 0) {
        const float sc = asym_scale(hi, lo, L.bit_v);
        vstat[j] = make_float4(sc, __frcp_rn(sc), lo, 0.f);
      }
    }
  }
  __syncthreads();
  // Largest stored Key scale of each group over the head's INT2/INT4/INT8
  // channels, gathered by the records' atomic maxima (0 with no such channel).
  for (int g = tid; g < G; g += kPackThreads) meta[g * M + L.kmax_off] = static_cast<uint16_t>(kmax_s[g]);

  // 3. Codes and words, kPackParts threads per token row and role (every
  // kPackParts-th word each): the first kPackRole threads the Key tier words
  // [0, ksplit) and (last part of a row) the fp16 words (FP16 Key tier, Value
  // scale and min), the others the Value code words and, on the pair-wise
  // Value path, the Key words [ksplit, nk).  ksplit balances the two roles (a
  // Key code costs about twice a Value code: a record and a gathered element
  // each).  Lanes are consecutive rows, so a warp reads one column of 32 rows
  // (32 banks).  Each word goes to the row staged in `out`.
  const int nk0 = L.words[0], nk1 = L.words[1], nk = nk0 + nk1 + L.words[2];
  const bool v_pairs = D % 16 == 0 && L.v_group % 16 == 0;
  int ksplit = nk;
  if (v_pairs) {
    const int cost_k = 2 * (16 * nk0 + 8 * nk1 + 4 * L.words[2]);
    const int target = (cost_k + 16 * L.vcode_words) / 2;
    int acc = 0;
    ksplit = 0;
    while (ksplit < nk) {
      const int c = 2 * (ksplit < nk0 ? 16 : ksplit < nk0 + nk1 ? 8 : 4);
      if (acc + c / 2 > target) break;  // the word goes where more than half of it falls
      acc += c;
      ++ksplit;
    }
  }
  // Key words [w0, w1) of row t (this thread's part, every kPackParts-th
  // word), one loop per tier so each runs with its code width fixed.
  auto key_words = [&](int t, int w0, int w1) {
    const unsigned char* row = xk + t * sw4;
    const SlotPair* rec = kslot + (t / kg) * (S.nslot / 2);
    uint32_t* orow = out + t * R;
    int w = w0;
    for (const int e = min(w1, nk0); w < e; w += kPackParts) orow[L.code_off[0] + w] = key_word<T, 2>(row, rec + 8 * w);
    for (const int e = min(w1, nk0 + nk1); w < e; w += kPackParts)
      orow[L.code_off[1] + w - nk0] = key_word<T, 4>(row, rec + S.tbase1 / 2 + 4 * (w - nk0));
    for (; w < w1; w += kPackParts)
      orow[L.code_off[2] + w - nk0 - nk1] = key_word<T, 8>(row, rec + S.tbase2 / 2 + 2 * (w - nk0 - nk1));
  };
  if (tid < kPackRole) {
    const int part = tid / kPackRows;
    const int half_part = kPackParts - 1;  // the part that also writes the fp16 words
    for (int t = tid % kPackRows; t < P; t += kPackRows) {
      const unsigned char* row = xk + t * sw4;
      uint32_t* orow = out + t * R;
      key_words(t, part, ksplit);
      if (part != half_part) continue;
      const int w3 = L.width[3];
      for (int w = L.half_off; w < R; ++w) {
        uint32_t word = 0;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int hx = 2 * (w - L.half_off) + e;
          uint32_t hv = 0;
          if (hx < w3) {
            hv = float_to_half_bits(load_elem<T>(row + h16[hx]));  // layout.py:110; padding reads 0
          } else if (hx < w3 + NV) {
            hv = float_to_half_bits(vstat[t * NV + hx - w3].x);
          } else if (hx < w3 + 2 * NV) {
            hv = float_to_half_bits(vstat[t * NV + hx - w3 - NV].z);
          }
          word |= hv << (16 * e);
        }
        orow[w] = word;
      }
    }
  } else if (D % 16 == 0 && L.v_group % 16 == 0) {
    // Value words, 16 channels each inside one v_group: the token's group
    // statistics change at word boundaries only; elements read in pairs.
    const int part = (tid - kPackRole) / kPackRows;
    const int wpg = L.v_group / 16;  // words per Value group
    for (int t = tid % kPackRows; t < P; t += kPackRows) {
      const unsigned char* row = xv + t * sw4;
      uint32_t* orow = out + t * R + L.vcode_off;
      int gi = 0, wg = part;  // group of word w and w's position in it
      while (wg >= wpg) {
        wg -= wpg;
        ++gi;
      }
      for (int w = part; w < L.vcode_words; w += kPackParts) {
        const float4 st = vstat[t * NV + gi];
        const float2 lo2 = make_float2(st.z, st.z), ns2 = make_float2(-st.x, -st.x), rc2 = make_float2(st.y, st.y);
        const unsigned char* src = row + 16 * w * static_cast<int>(sizeof(T));
        uint32_t word = 0, bias = 0;
#pragma unroll
        for (int k = 0; k < 16; k += 2) {
          const uint2 c = pack_bits2(load_pair<T>(src + k * static_cast<int>(sizeof(T))), lo2, ns2, rc2, 3u);
          word += c.x << (2 * k);
          word += c.y << (2 * k + 2);
          bias += (kMagicBits << (2 * k)) + (kMagicBits << (2 * k + 2));
        }
        orow[w] = word - bias;
        wg += kPackParts;
        while (wg >= wpg) {
          wg -= wpg;
          ++gi;
        }
      }
      key_words(t, ksplit + part, nk);
    }
  } else {
    const int vg = L.v_group;
    for (int t = tid - kPackRole; t < P; t += kPackRole) {
      const unsigned char* row = xv + t * sw4;
      uint32_t* orow = out + t * R + L.vcode_off;
      int g = 0, g_end = vg;
      float4 st = vstat[t * NV];
      for (int w = 0; w < L.vcode_words; ++w) {
        uint32_t word = 0;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const int d = 16 * w + k;
          if (d < D) {
            if (d >= g_end) {
              ++g;
              g_end += vg;
              st = vstat[t * NV + g];
            }
            word |= pack_code(load_elem<T>(row + d * static_cast<int>(sizeof(T))), st.z, st.x, st.y, 3u) << (2 * k);
          }
        }
        orow[w] = word;
      }
    }
  }
  __syncthreads();

  // 4. The page's rows (contiguous in the history) and meta rows, coalesced.
  const int64_t row0 = (static_cast<int64_t>(dst_seq) * H + h) * L.row_cap + static_cast<int64_t>(dst_page) * P;
  int32_t* out_rows = rows + row0 * R;
  const int nw = P * R;
  if ((reinterpret_cast<uintptr_t>(out_rows) % 16) == 0 && nw % 4 == 0) {
    for (int i = tid; i < nw / 4; i += kPackThreads)
      reinterpret_cast<uint4*>(out_rows)[i] = reinterpret_cast<const uint4*>(out)[i];
  } else {
    for (int i = tid; i < nw; i += kPackThreads) out_rows[i] = static_cast<int32_t>(out[i]);
  }
  uint16_t* out_meta = kmeta + ((static_cast<int64_t>(dst_seq) * H + h) * L.group_cap +
                                static_cast<int64_t>(dst_page) * G) * M;
  for (int i = tid; i < G * M; i += kPackThreads) out_meta[i] = meta[i];
}

__global__ void dequantize_kernel(const __grid_constant__ lf_layout L, const int32_t* __restrict__ rows,
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
