// K2 on the 5th-generation tensor cores (sm_100a, tcgen05.mma kind::i8).
//
// Geometry: head_dim 128, page 128 = Key group 128, Value group 128, bit_v 2
// (the LogitFill defaults, deepseek_qwen.py:24-46).  One 128-thread CTA per
// (split, KV head, sequence) work item; thread t owns token t of the current
// page, TMEM lane t and, for the PV result, head-dim position t.
//
// Per page (128 tokens) of packed history:
//   [A] the row block (all tiers' Key codes, Value codes, FP16 Key tier,
//       Value scale/min of 128 tokens) arrives by one 1-D bulk copy;
//       each thread unpacks its token's Key codes to u8 straight into TMEM
//       (A operand of QK, K-major) and its Value codes to u8 into shared memory
//       (A operand of PV, MN-major), and writes the B row of QK for its tier
//       slots: 24-bit fixed point X = q_j * scale_c * 2^-E_j offset by 2^23,
//       three unsigned limbs, plus a column of ones.
//   QK = codes . B  (5 x M128 N32 K32 MMAs for 160 slots)
//       score_tj = 2^E_j (acc0 + 256 acc1 + 65536 (acc2 - 128 ones))
//                  + sum_c q_j[c] min_c + FP16-tier part,
//   [B] online softmax over the page (one CTA max per q-head), then the B
//       row of PV for token t: 23-bit fixed point p_tj * vscale_t, 3 limbs.
//   PV = Vcodes^T . B  (4 x M128 N32 K32 MMAs)
//   [C] o_j = o_j alpha_j + 2^Ev_j (acc0 + 256 acc1 + 65536 acc2).
// The Value-min term sum_t p_tj vmin_t and the normaliser are per-thread
// partial sums reduced once per work item.
//
// The integer products are exact; the fixed-point rounding is 2^-22 (QK) and
// 2^-23 (PV) of the per-page block maximum (tests/kernel_model.py models it).
// Every mbarrier wait is bounded (2 s): on expiry the CTA sets
// LF_ERR_DEVICE_TIMEOUT in the status word, drains its own copies and MMAs,
// frees its TMEM and returns.
#include <atomic>

#include "lf_decode_common.cuh"
#include "lf_tcgen05.cuh"

namespace lf {
namespace tc {

using namespace sm100;

constexpr int kP = 128, kD = 128;
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr uint32_t kIdescQK = idesc_u8(128, 32, false, true);  // A: TMEM (K-major), B: MN-major
constexpr uint32_t kIdescPV = idesc_u8(128, 32, true, true);   // A, B: MN-major smem
constexpr uint32_t kM2 = 0x03030303u, kM4 = 0x0F0F0F0Fu;

struct TcSmem {
  int bars, red, kpos, esc, qs, q16, stage0, stage1, meta, apv, bqk, bpv, total;
  int kpad, a_col, tm_qk, tm_pv, tm_cols, bqk_sbo;
};

__host__ __device__ inline int n_slots_of(const lf_layout& L) {
  return 16 * L.words[0] + 8 * L.words[1] + 4 * L.words[2];
}

__host__ __device__ inline TcSmem tc_smem(const lf_layout& L, int pps) {
  TcSmem s;
  const int ns = n_slots_of(L);
  s.kpad = ns == 0 ? 32 : (ns + 31) / 32 * 32;
  s.a_col = 0;
  const int a_cols = s.kpad / 4;
  s.tm_qk = (a_cols + 31) / 32 * 32;
  s.tm_pv = s.tm_qk + 32;
  int need = s.tm_pv + 32, cols = 32;
  while (cols < need) cols *= 2;
  s.tm_cols = cols;
  s.bqk_sbo = s.kpad * 16;
  int off = 0;
  s.bars = off; off += 64;
  s.red = off; off += 256 * 4;
  s.kpos = off; off += s.kpad * 4;
  s.esc = off; off += ((pps + 3) / 4 * 4) * 4;
  s.qs = off; off += kGQ * kD * 4;
  s.q16 = off; off += (L.width[3] > 0 ? L.width[3] : 1) * kGQ * 4;
  off = (off + 127) / 128 * 128;
  s.stage0 = off; off += kP * L.row_words * 4;
  s.stage1 = off; off += kP * L.row_words * 4;
  s.meta = off; off += (pps * L.meta_halves * 2 + 15) / 16 * 16;
  off = (off + 1023) / 1024 * 1024;
  s.apv = off; off += kP * kD;
  s.bqk = off; off += s.kpad * 32;
  s.bpv = off; off += kP * 32;
  // The residual split reuses the region from stage0 for fp32 K/V rows.
  const int resid_end = s.stage0 + resid_smem(kD).total;
  if (resid_end > off) off = resid_end;
  s.total = (off + 1023) / 1024 * 1024;
  return s;
}

// Tier slot held by MMA K position pp, in the order the unpacked u8 codes take:
// an INT2 word w yields 4 columns (w >> 2k) & 0x03030303, i.e. slots
// 16w + k + 4i at byte i; an INT4 word 2 columns (slots 8w + k + 2i); an INT8
// word 1 column (slots 4w + i).  Returns channel | tier << 16 | slot << 18,
// or -1 for a padding position.
__device__ __forceinline__ int kpos_entry(const lf_layout& L, const int32_t* slot_chan, int h, int pp) {
  const int n0 = 16 * L.words[0], n1 = 8 * L.words[1], n2 = 4 * L.words[2];
  int tier, slot;
  if (pp < n0) {
    const int w = pp >> 4, r = pp & 15;
    tier = 0;
    slot = 16 * w + (r >> 2) + 4 * (r & 3);
  } else if (pp < n0 + n1) {
    const int q = pp - n0, w = q >> 3, r = q & 7;
    tier = 1;
    slot = 8 * w + (r >> 2) + 2 * (r & 3);
  } else if (pp < n0 + n1 + n2) {
    tier = 2;
    slot = pp - n0 - n1;
  } else {
    return -1;
  }
  if (slot >= L.width[tier]) return -1;
  const int ch = slot_chan[(tier * L.kv_heads + h) * L.head_dim + slot];
  return ch < 0 ? -1 : (ch | (tier << 16) | (slot << 18));
}

// Pack bytes 0..2 of U[0..7] into MN-major limb rows:
// c0 = {byte0 of U0..U7, byte1 of U0..U7}, c1 = {byte2 of U0..U7, w3, 0}.
__device__ __forceinline__ void pack_limbs(const uint32_t (&U)[kGQ], uint4& c0, uint4& c1, uint32_t w3) {
  uint32_t b0[2], b1[2], b2[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t t01 = __byte_perm(U[4 * h + 0], U[4 * h + 1], 0x5140);
    const uint32_t t23 = __byte_perm(U[4 * h + 2], U[4 * h + 3], 0x5140);
    const uint32_t s01 = __byte_perm(U[4 * h + 0], U[4 * h + 1], 0x7362);
    const uint32_t s23 = __byte_perm(U[4 * h + 2], U[4 * h + 3], 0x7362);
    b0[h] = __byte_perm(t01, t23, 0x5410);
    b1[h] = __byte_perm(t01, t23, 0x7632);
    b2[h] = __byte_perm(s01, s23, 0x5410);
  }
  c0 = make_uint4(b0[0], b0[1], b1[0], b1[1]);
  c1 = make_uint4(b2[0], b2[1], w3, 0u);
}

// Warp reduce-scatter of 8 sums: returns the warp total of v[j] for
// j = 4*bit4(lane) + 2*bit3(lane) + bit2(lane).
__device__ __forceinline__ float warp_sum8_scatter(const float (&v)[kGQ], int lane) {
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
  float k4[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float keep = b4 ? v[4 + k] : v[k];
    const float send = b4 ? v[k] : v[4 + k];
    k4[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
  float k2[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const float keep = b3 ? k4[2 + k] : k4[k];
    const float send = b3 ? k4[k] : k4[2 + k];
    k2[k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  const float keep = b2 ? k2[1] : k2[0];
  const float send = b2 ? k2[0] : k2[1];
  float x = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  return x;
}

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float order_key_to_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}
// Smallest e with x <= 2^e for finite x > 0 (x = 1.f * 2^e' -> e' or e'+1);
// 0 for x <= 0.  Subnormal x count as 2^-126.
__device__ __forceinline__ int exp2_ceil(float x) {
  if (!(x > 0.f)) return 0;
  const uint32_t u = __float_as_uint(x);
  const int e = static_cast<int>(u >> 23) - 127;
  if (e < -126) return -126;
  return (u & 0x7FFFFFu) ? e + 1 : e;
}
// 2^e as a float, e in [-126, 127].
__device__ __forceinline__ float exp2i(int e) { return __int_as_float((e + 127) << 23); }

template <typename RT, typename QT>
__global__ void __launch_bounds__(kDecThreads, 3) decode_partial_tc(DecodeParams p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const lf_layout& L = p.L;
  const TcSmem S = tc_smem(L, p.pps);
  const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int H = L.kv_heads, R = L.row_words, M = L.meta_halves, GQ = p.gq;
  const int pages = p.hist_tokens[b] / kP;
  const int n_page_splits = (pages + p.pps - 1) / p.pps;
  if (s >= n_page_splits + residual_splits(kP)) return;

  float* q_s = reinterpret_cast<float*>(smem + S.qs);
  float* red = reinterpret_cast<float*>(smem + S.red);
  float m[kGQ], o[kGQ], lt[kGQ], lvt[kGQ];
#pragma unroll
  for (int j = 0; j < kGQ; ++j) {
    m[j] = -INFINITY;
    o[j] = 0.f;
    lt[j] = 0.f;
    lvt[j] = 0.f;
  }
  load_query_group<QT>(p, b, h, q_s);

  if (s >= n_page_splits) {  // residual splits: tail rows + new token, fp32
    residual_chunk<RT>(p, b, h, s - n_page_splits, q_s, smem + S.stage0, m, o, lt);
    write_partial(p, b, h, s, tid, o, m, lt, lvt, red);
    return;
  }

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S.bars);  // full[0], full[1], qk, pv
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S.bars + 32);
  volatile int* abort_s = reinterpret_cast<volatile int*>(smem + S.bars + 36);
  int* kpos_s = reinterpret_cast<int*>(smem + S.kpos);
  int* esc_s = reinterpret_cast<int*>(smem + S.esc);
  float* q16_s = reinterpret_cast<float*>(smem + S.q16);
  uint32_t* const stage0 = reinterpret_cast<uint32_t*>(smem + S.stage0);
  const int stage_words = kP * L.row_words;  // stage1 follows stage0
  const uint16_t* meta_s = reinterpret_cast<const uint16_t*>(smem + S.meta);
  unsigned char* apv = smem + S.apv;
  unsigned char* bqk = smem + S.bqk;
  unsigned char* bpv = smem + S.bpv;
  float* red_b = red;            // [4 warps][8] bias partials
  uint32_t* red_m = reinterpret_cast<uint32_t*>(red + 64);  // [4 warps][16] max keys

  const int pg0 = s * p.pps;
  const int npg = min(pages, pg0 + p.pps) - pg0;
  const int64_t head_row = (static_cast<int64_t>(b) * H + h) * L.row_cap;
  const int64_t head_meta = (static_cast<int64_t>(b) * H + h) * L.group_cap;
  const uint32_t row_bytes = kP * R * 4;
  const uint32_t meta_bytes = static_cast<uint32_t>(npg * M * 2);

  if (tid == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) mbar_init(&bars[i], 1);
    *abort_s = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, S.tm_cols);
    tmem_relinquish();
  }
  for (int pp = tid; pp < S.kpad; pp += kDecThreads) kpos_s[pp] = kpos_entry(L, p.slot_chan, h, pp);
  for (int q = tid; q < npg; q += kDecThreads) esc_s[q] = 0;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;

  // Kick off the item's Key meta rows and the first two pages.
  if (tid == 0) {
    mbar_arrive_expect_tx(&bars[0], row_bytes + meta_bytes);
    if (meta_bytes) bulk_g2s(smem + S.meta, p.kmeta + (head_meta + pg0) * M, meta_bytes, &bars[0]);
    bulk_g2s(stage0, p.rows + (head_row + static_cast<int64_t>(pg0) * kP) * R, row_bytes, &bars[0]);
    if (npg > 1) {
      mbar_arrive_expect_tx(&bars[1], row_bytes);
      bulk_g2s(stage0 + stage_words, p.rows + (head_row + static_cast<int64_t>(pg0 + 1) * kP) * R, row_bytes, &bars[1]);
    }
  }

  // Per-q-head block exponent of the query: max_c |q_j[c]| <= 2^eq_j.
  int eq[kGQ];
  {
#pragma unroll
    for (int j = 0; j < kGQ; ++j) {
      const uint32_t a = __float_as_uint(fabsf(q_s[j * kD + tid]));
      const uint32_t mx = __reduce_max_sync(0xffffffffu, a);
      if (lane == 0) red_m[warp * 16 + j] = mx;
    }
    for (int i = tid; i < L.width[3] * kGQ; i += kDecThreads) {
      const int ii = i / kGQ, j = i % kGQ;
      const int ch = p.slot_chan[(3 * H + h) * kD + ii];
      q16_s[i] = ch < 0 ? 0.f : q_s[j * kD + ch];
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kGQ; ++j) {
      uint32_t mx = red_m[j];
#pragma unroll
      for (int w = 1; w < 4; ++w) mx = max(mx, red_m[w * 16 + j]);
      eq[j] = exp2_ceil(__uint_as_float(mx));
    }
  }
  // This thread's QK B rows: K positions tid, tid+128, tid+256.
  float qq[3][kGQ];
  int soff[3], moff[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const int pp = tid + k * kDecThreads;
    const int e = pp < S.kpad ? kpos_s[pp] : -1;
    soff[k] = moff[k] = -1;
    if (e >= 0) {
      const int ch = e & 0xFFFF, tier = (e >> 16) & 3, slot = e >> 18;
      soff[k] = L.scale_off[tier] + slot;
      moff[k] = L.min_off[tier] + slot;
    }
#pragma unroll
    for (int j = 0; j < kGQ; ++j) qq[k][j] = e >= 0 ? q_s[j * kD + (e & 0xFFFF)] * exp2i(22 - eq[j]) : 0.f;
  }
  // A columns past the packed slots stay zero for the whole item.
  for (int c = n_slots_of(L) / 4; c < S.kpad / 4; ++c) tmem_st_x1(tmem + lane_base + S.a_col + c, 0u);

  const float c2 = p.scaling * kLog2e;
  bool ok = true;
  int issued[2] = {1, npg > 1 ? 1 : 0}, waited[2] = {0, 0};
  int mma_open = 0;  // committed-but-unwaited MMA barriers: bit0 qk, bit1 pv
  int i = 0;
  for (; i < npg; ++i) {
    const int st = i & 1;
    if (!mbar_wait_bounded(&bars[st], (i >> 1) & 1, kWaitLimitNs)) { *abort_s = 1; ok = false; }
    else ++waited[st];
    if (i == 0) {
      // Per-page block exponent of the Key scales, from the item's meta rows:
      // max over this thread's slots, warp max, then one shared atomic per warp.
      for (int q = 0; q < npg; ++q) {
        float mx = 0.f;
#pragma unroll
        for (int k = 0; k < 3; ++k)
          if (soff[k] >= 0) mx = fmaxf(mx, half_bits_to_float(meta_s[q * M + soff[k]]));
        const uint32_t wmax = __reduce_max_sync(0xffffffffu, __float_as_uint(mx));
        if (lane == 0) atomicMax(reinterpret_cast<unsigned int*>(esc_s) + q, wmax);
      }
      __syncthreads();
      for (int q = tid; q < npg; q += kDecThreads) esc_s[q] = exp2_ceil(__uint_as_float(esc_s[q]));
      __syncthreads();
    }
    const uint32_t* rowp = stage0 + st * stage_words + tid * R;
    const uint16_t* row16 = reinterpret_cast<const uint16_t*>(rowp);
    // [A1] Key codes -> TMEM (this thread's lane), u8 per slot.
    {
      uint32_t col = tmem + lane_base + S.a_col;
      for (int w = 0; w < L.words[0]; ++w, col += 4) {
        const uint32_t x = rowp[L.code_off[0] + w];
        tmem_st_x4(col, x & kM2, (x >> 2) & kM2, (x >> 4) & kM2, (x >> 6) & kM2);
      }
      for (int w = 0; w < L.words[1]; ++w, col += 2) {
        const uint32_t x = rowp[L.code_off[1] + w];
        tmem_st_x2(col, x & kM4, (x >> 4) & kM4);
      }
      for (int w = 0; w < L.words[2]; ++w, col += 1) tmem_st_x1(col, rowp[L.code_off[2] + w]);
    }
    // [A2] Value codes -> A operand of PV (MN-major: 16 channels x 8 tokens cores).
    {
      unsigned char* dst = apv + (tid & 7) * 16 + (tid >> 3) * 128;
#pragma unroll
      for (int w = 0; w < kD / 16; ++w) {
        const uint32_t x = rowp[L.vcode_off + w];
        *reinterpret_cast<uint4*>(dst + w * 2048) =
            make_uint4(x & kM2, (x >> 2) & kM2, (x >> 4) & kM2, (x >> 6) & kM2);
      }
    }
    // [A3] FP16 Key tier on the CUDA cores; Value scale / min of the token.
    float s16[kGQ];
#pragma unroll
    for (int j = 0; j < kGQ; ++j) s16[j] = 0.f;
    const int h0 = 2 * L.half_off;
    for (int c = 0; c < L.width[3]; ++c) {
      const float kv = half_bits_to_float(row16[h0 + c]);
      const float4 a = *reinterpret_cast<const float4*>(q16_s + c * kGQ);
      const float4 bq = *reinterpret_cast<const float4*>(q16_s + c * kGQ + 4);
      s16[0] = fmaf(a.x, kv, s16[0]);
      s16[1] = fmaf(a.y, kv, s16[1]);
      s16[2] = fmaf(a.z, kv, s16[2]);
      s16[3] = fmaf(a.w, kv, s16[3]);
      s16[4] = fmaf(bq.x, kv, s16[4]);
      s16[5] = fmaf(bq.y, kv, s16[5]);
      s16[6] = fmaf(bq.z, kv, s16[6]);
      s16[7] = fmaf(bq.w, kv, s16[7]);
    }
    const float vs = half_bits_to_float(row16[h0 + L.width[3]]);
    const float vm = half_bits_to_float(row16[h0 + L.width[3] + 1]);
    // [A4] B rows of QK for this thread's slots; bias partials sum_c q_c min_c.
    float bias[kGQ];
#pragma unroll
    for (int j = 0; j < kGQ; ++j) bias[j] = 0.f;
    {
      const float fsc = exp2i(-esc_s[i]);
      const uint16_t* mrow = meta_s + i * M;
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        const int pp = tid + k * kDecThreads;
        if (pp >= S.kpad) break;
        uint4 c0 = make_uint4(0u, 0u, 0u, 0u), c1 = c0;
        if (soff[k] >= 0) {
          const float sc = half_bits_to_float(mrow[soff[k]]) * fsc;
          const float mn = half_bits_to_float(mrow[moff[k]]);
          uint32_t U[kGQ];
#pragma unroll
          for (int j = 0; j < kGQ; ++j) {
            // rint(qq * sc) + 2^23 via the fp32 magic constant 1.5 * 2^23.
            U[j] = __float_as_uint(fmaf(qq[k][j], sc, 12582912.0f)) - 0x4AC00000u;
            bias[j] = fmaf(qq[k][j], mn, bias[j]);
          }
          pack_limbs(U, c0, c1, 1u);
        }
        unsigned char* dst = bqk + (pp & 7) * 16 + (pp >> 3) * 128;
        *reinterpret_cast<uint4*>(dst) = c0;
        *reinterpret_cast<uint4*>(dst + S.bqk_sbo) = c1;
      }
    }
    {
      const float part = warp_sum8_scatter(bias, lane);
      if ((lane & 3) == 0) red_b[warp * kGQ + (((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1))] = part;
    }
    tmem_wait_st();
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (*abort_s) break;
    if (tid == 0) {
      tc_fence_after();
      for (int ks = 0; ks < S.kpad / 32; ++ks)
        mma_u8_ts(tmem + S.tm_qk, tmem + S.a_col + 8 * ks, smem_desc(bqk + 512 * ks, 128, S.bqk_sbo), kIdescQK,
                  ks > 0 ? 1u : 0u);
      mma_commit(&bars[2]);
      if (i + 2 < npg) {  // the stage just consumed takes page i+2
        mbar_arrive_expect_tx(&bars[st], row_bytes);
        bulk_g2s(stage0 + st * stage_words, p.rows + (head_row + static_cast<int64_t>(pg0 + i + 2) * kP) * R, row_bytes,
                 &bars[st]);
        ++issued[st];
      }
    }
    mma_open |= 1;

    // [B] scores, page max, probabilities and the PV B rows.
    if (!mbar_wait_bounded(&bars[2], i & 1, kWaitLimitNs)) { *abort_s = 1; ok = false; }
    else mma_open &= ~1;
    tc_fence_after();
    uint32_t acc[32];
    tmem_ld_x32(tmem + lane_base + S.tm_qk, acc);
    tmem_wait_ld();
    float sc[kGQ];
    {
      const int esc = esc_s[i];
      const int ones = static_cast<int>(acc[24]);
#pragma unroll
      for (int j = 0; j < kGQ; ++j) {
        const float bsum = (red_b[j] + red_b[kGQ + j]) + (red_b[2 * kGQ + j] + red_b[3 * kGQ + j]);
        const float sint = static_cast<float>(static_cast<int>(acc[j])) +
                           256.f * static_cast<float>(static_cast<int>(acc[8 + j])) +
                           65536.f * static_cast<float>(static_cast<int>(acc[16 + j]) - 128 * ones);
        const float val = sint * (c2 * exp2i(eq[j] + esc - 22)) + (bsum * exp2i(eq[j] - 22) + s16[j]) * c2;
        sc[j] = j < GQ ? val : -INFINITY;
        const uint32_t key = __reduce_max_sync(0xffffffffu, order_key(sc[j]));
        if (lane == 0) red_m[warp * 16 + j] = key;
      }
      const uint32_t vkey = __reduce_max_sync(0xffffffffu, __float_as_uint(vs));
      if (lane == 0) red_m[warp * 16 + 8] = vkey;
    }
    __syncthreads();
    float alpha[kGQ];
    int ev[kGQ];
    {
      uint32_t vk = red_m[8];
#pragma unroll
      for (int w = 1; w < 4; ++w) vk = max(vk, red_m[w * 16 + 8]);
      const float vsmax = __uint_as_float(vk);
      uint32_t U[kGQ];
#pragma unroll
      for (int j = 0; j < kGQ; ++j) {
        uint32_t key = red_m[j];
#pragma unroll
        for (int w = 1; w < 4; ++w) key = max(key, red_m[w * 16 + j]);
        const float pm = order_key_to_float(key);
        float pj = 0.f;
        if (j < GQ) {
          const float mnew = fmaxf(m[j], pm);
          alpha[j] = m[j] == -INFINITY ? 0.f : ex2(m[j] - mnew);
          m[j] = mnew;
          pj = ex2(sc[j] - mnew);
          ev[j] = exp2_ceil(ex2(pm - mnew) * vsmax);
        } else {
          alpha[j] = 1.f;
          ev[j] = 0;
        }
        lt[j] = fmaf(lt[j], alpha[j], pj);
        lvt[j] = fmaf(lvt[j], alpha[j], pj * vm);
        // rint(p * vs * 2^(23 - ev)) via the fp32 magic constant 2^23.
        U[j] = __float_as_uint(fmaf(pj, vs * exp2i(23 - ev[j]), 8388608.0f)) - 0x4B000000u;
      }
      uint4 c0, c1;
      pack_limbs(U, c0, c1, 0u);
      unsigned char* dst = bpv + (tid & 7) * 16 + (tid >> 3) * 128;
      *reinterpret_cast<uint4*>(dst) = c0;
      *reinterpret_cast<uint4*>(dst + 2048) = c1;
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (*abort_s) break;
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < kP / 32; ++ks)
        mma_u8_ss(tmem + S.tm_pv, smem_desc(apv + 512 * ks, 128, 2048), smem_desc(bpv + 512 * ks, 128, 2048),
                  kIdescPV, ks > 0 ? 1u : 0u);
      mma_commit(&bars[3]);
    }
    mma_open |= 2;
    // [C] accumulate this thread's head-dim position.
    if (!mbar_wait_bounded(&bars[3], i & 1, kWaitLimitNs)) { *abort_s = 1; ok = false; }
    else mma_open &= ~2;
    tc_fence_after();
    tmem_ld_x32(tmem + lane_base + S.tm_pv, acc);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < kGQ; ++j) {
      const float v = static_cast<float>(static_cast<int>(acc[j])) +
                      256.f * static_cast<float>(static_cast<int>(acc[8 + j])) +
                      65536.f * static_cast<float>(static_cast<int>(acc[16 + j]));
      o[j] = fmaf(o[j], alpha[j], v * exp2i(ev[j] - 23));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_s) {
    // Drain this CTA's own copies and MMAs (bounded), record the failure.
    if (tid == 0) {
      for (int st = 0; st < 2; ++st)
        while (waited[st] < issued[st]) {
          mbar_wait_bounded(&bars[st], waited[st] & 1, kWaitLimitNs);
          ++waited[st];
        }
      if (p.status != nullptr) atomicExch(p.status, LF_ERR_DEVICE_TIMEOUT);
    }
    if (mma_open & 1) mbar_wait_bounded(&bars[2], i & 1, kWaitLimitNs);
    if (mma_open & 2) mbar_wait_bounded(&bars[3], i & 1, kWaitLimitNs);
    __syncthreads();
  }
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, S.tm_cols);
  (void)ok;
#pragma unroll
  for (int j = 0; j < kGQ; ++j) m[j] *= kLn2;  // log2 units -> natural-log units
  // PV row t holds head-dim channel d(t): t = 16w + 4k + i  <->  d = 16w + k + 4i.
  const int d = (tid & ~15) + ((tid & 15) >> 2) + 4 * (tid & 3);
  write_partial(p, b, h, s, d, o, m, lt, lvt, red + 128);
}

}  // namespace tc

bool tc_supported(const lf_layout& L, int gq, int pps) {
  if (L.head_dim != tc::kD || L.page_size != tc::kP || L.k_group != tc::kP || L.v_group != tc::kD) return false;
  if (L.bit_v != 2 || gq > kGQ || gq < 1) return false;
  if (tc::n_slots_of(L) > 384) return false;
  return tc::tc_smem(L, pps).total <= 227 * 1024;
}

template <typename RT, typename QT>
static int launch_tc_typed(const DecodeParams& p, cudaStream_t stream) {
  const tc::TcSmem S = tc::tc_smem(p.L, p.pps);
  auto kern = tc::decode_partial_tc<RT, QT>;
  static std::atomic<int> configured{48 * 1024};
  if (S.total > configured.load()) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S.total);
    if (e != cudaSuccess) {
      set_error("lf_decode_partial (tcgen05): shared memory %d B: %s", S.total, cudaGetErrorString(e));
      return LF_ERR_UNSUPPORTED;
    }
    configured.store(S.total);
  }
  dim3 grid(p.max_splits, p.L.kv_heads, p.batch);
  kern<<<grid, kDecThreads, S.total, stream>>>(p);
  return launch_status("lf_decode_partial (tcgen05)");
}

int occupancy_tc(const lf_layout& L, int pps) {
  const tc::TcSmem S = tc::tc_smem(L, pps);
  if (S.total > 227 * 1024) return 0;
  cudaFuncSetAttribute(tc::decode_partial_tc<__nv_bfloat16, __nv_bfloat16>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, S.total);
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, tc::decode_partial_tc<__nv_bfloat16, __nv_bfloat16>,
                                                    kDecThreads, S.total) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  const int by_tmem = 512 / S.tm_cols;
  return blocks < by_tmem ? blocks : by_tmem;
}

int launch_partial_tc(const DecodeParams& p, int resid_dtype, int q_dtype, cudaStream_t stream) {
#define LF_TC_Q(RT)                                                        \
  switch (q_dtype) {                                                       \
    case LF_F32: return launch_tc_typed<RT, float>(p, stream);             \
    case LF_F16: return launch_tc_typed<RT, __half>(p, stream);            \
    case LF_BF16: return launch_tc_typed<RT, __nv_bfloat16>(p, stream);    \
  }                                                                        \
  break;
  switch (resid_dtype) {
    case LF_F32: LF_TC_Q(float)
    case LF_F16: LF_TC_Q(__half)
    case LF_BF16: LF_TC_Q(__nv_bfloat16)
  }
#undef LF_TC_Q
  set_error("lf_decode_partial: dtype residual %d / query %d", resid_dtype, q_dtype);
  return LF_ERR_INVALID_ARGUMENT;
}

}  // namespace lf
