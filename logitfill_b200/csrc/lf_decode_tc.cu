// K2 on the 5th-generation tensor cores (sm_100a, tcgen05.mma kind::i8).
//
// Geometry: head_dim 128, page 128 = Key group 128, Value group 128, bit_v 2
// (the LogitFill defaults, deepseek_qwen.py:24-46).  One CTA per (split, KV
// head, sequence) work item: four compute warps (thread t owns token t of the
// current page, TMEM lane t and head-dim position t of the PV result) and one
// control warp that issues the 1-D bulk copies of the page row blocks and the
// tensor-core MMAs.
//
// Per page (128 tokens) of packed history, with X = 24-bit fixed point:
//   U_K  Key codes -> u8 in TMEM (A of QK, K-major); the B row of QK for the
//        thread's tier slots: X(q_j[c] * scale_c) + 2^23 as three unsigned
//        limbs plus a column of ones; FP16-tier partial scores (CUDA cores).
//   QK   5 x M128 N32 K32:  acc0 + 256 acc1 + 65536 (acc2 - 128 ones)
//        = sum_c code_tc X_jc, exact in int32.
//   S    scores (+ sum_c q_j[c] min_c + FP16 part), page max per q-head over
//        the four compute warps, online-softmax update, B row of PV for token
//        t: 23-bit X(p_tj * vscale_t), three limbs.
//   U_V  Value codes -> u8 in shared memory (A of PV, MN-major).
//   PV   4 x M128 N32 K32;  C: o_j = o_j alpha_j + 2^Ev_j (acc0 + 256 acc1 + 65536 acc2).
// Compute warps run S(i), U_K(i+1), C(i), U_V(i+1): PV(i) overlaps U_K(i+1)
// and QK(i+1) overlaps C(i) and U_V(i+1).  The Value-min term sum_t p_tj
// vmin_t and the normaliser are per-thread partial sums reduced per item.
//
// The integer products are exact; the fixed-point rounding is 2^-22 (QK) and
// 2^-23 (PV) of the per-page block maximum (tests/kernel_model.py models it).
// Every mbarrier wait is bounded (2 s).  On expiry the CTA records
// LF_ERR_DEVICE_TIMEOUT, stops waiting (every warp still passes the same
// barriers, so nothing deadlocks), drains its own copies and MMAs, frees its
// TMEM and returns.
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

constexpr int kStages = 2;
constexpr int kThreads = kDecThreads + 32;  // 4 compute warps + 1 control warp
constexpr int kMaxPagesPerItem = 16;        // bounds the per-item meta buffer

struct TcSmem {
  int bars, red, kpos, esc, q16, stage0, meta, apv, qs, bqk, bpv, total;
  int kpad, a_col, tm_qk, tm_pv, tm_cols, bqk_sbo, stage_bytes;
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
  s.stage_bytes = kP * L.row_words * 4;
  int off = 0;
  s.bars = off; off += 128;
  s.red = off; off += 320 * 4;
  s.kpos = off; off += s.kpad * 4;
  s.esc = off; off += ((pps + 3) / 4 * 4) * 4;
  s.q16 = off; off += (L.width[3] > 0 ? L.width[3] : 1) * kGQ * 4;
  off = (off + 127) / 128 * 128;
  s.stage0 = off; off += kStages * s.stage_bytes;
  s.meta = off; off += (pps * L.meta_halves * 2 + 15) / 16 * 16;
  off = (off + 1023) / 1024 * 1024;
  s.apv = off; off += 2 * kP * kD;   // two Value tiles (page parity)
  s.qs = s.apv + kP * kD;           // the query group aliases the second tile in the prologue
  s.bqk = off; off += s.kpad * 32;
  s.bpv = off; off += kP * 32;
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

// Barrier slots in shared memory.
enum { kBarFull = 0, kBarKReady = kStages, kBarVReady, kBarQK, kBarPV, kNumBars };

template <int GQ>
__global__ void __launch_bounds__(kThreads, 3) decode_partial_tc(DecodeParams p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const lf_layout& L = p.L;
  const TcSmem S = tc_smem(L, p.pps);
  const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int H = L.kv_heads, R = L.row_words, M = L.meta_halves;
  const int pages = p.hist_tokens[b] / kP;
  const int n_page_splits = (pages + p.pps - 1) / p.pps;
  if (s >= n_page_splits + residual_splits(kP)) return;

  float* q_s = reinterpret_cast<float*>(smem + S.qs);
  float* red = reinterpret_cast<float*>(smem + S.red);

  if (s >= n_page_splits) {  // residual splits: tail rows + new token, fp32 (compute warps)
    if (warp >= 4) return;
    float m[kGQ], o[kGQ], lt[kGQ], lvt[kGQ];
#pragma unroll
    for (int j = 0; j < kGQ; ++j) {
      m[j] = -INFINITY;
      o[j] = lt[j] = lvt[j] = 0.f;
    }
    load_query_group_rt(p, b, h, q_s, kDecThreads);
    const int c = s - n_page_splits;
    unsigned char* region = smem + S.stage0;
    residual_chunk(p, b, h, c, q_s, region, m, o, lt);
    write_partial_group<kGQ>(p, b, h, s, tid, o, m, lt, lvt, red, 1);
    return;
  }

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S.bars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S.bars + 8 * kNumBars);
  volatile int* abort_s = reinterpret_cast<volatile int*>(smem + S.bars + 8 * kNumBars + 4);
  int* kpos_s = reinterpret_cast<int*>(smem + S.kpos);
  int* esc_s = reinterpret_cast<int*>(smem + S.esc);
  float* q16_s = reinterpret_cast<float*>(smem + S.q16);
  unsigned char* stage0 = smem + S.stage0;
  const uint16_t* meta_s = reinterpret_cast<const uint16_t*>(smem + S.meta);
  unsigned char* apv = smem + S.apv;
  unsigned char* bqk = smem + S.bqk;
  unsigned char* bpv = smem + S.bpv;
  float* red_b = red;                                         // [2][4 warps][8] bias partials
  uint32_t* red_m = reinterpret_cast<uint32_t*>(red + 64);    // [2][4 warps][16] max keys
  float* red_w = red + 192;                                   // item-end reductions

  const int pg0 = s * p.pps;
  const int npg = min(pages, pg0 + p.pps) - pg0;
  const int64_t head_row = (static_cast<int64_t>(b) * H + h) * L.row_cap;
  const int64_t head_meta = (static_cast<int64_t>(b) * H + h) * L.group_cap;
  const uint32_t row_bytes = static_cast<uint32_t>(S.stage_bytes);
  const uint32_t meta_bytes = static_cast<uint32_t>(npg * M * 2);

  if (tid == kDecThreads) {
#pragma unroll
    for (int i = 0; i < kStages; ++i) mbar_init(&bars[kBarFull + i], 1);
    mbar_init(&bars[kBarKReady], kDecThreads);
    mbar_init(&bars[kBarVReady], kDecThreads);
    mbar_init(&bars[kBarQK], 1);
    mbar_init(&bars[kBarPV], 1);
    *abort_s = 0;
    fence_mbar_init();
  }
  if (warp == 4) {
    tmem_alloc(tmem_slot, S.tm_cols);
    tmem_relinquish();
  }
  if (tid < kDecThreads) {
    load_query_group_rt(p, b, h, q_s, kDecThreads);
    for (int pp = tid; pp < S.kpad; pp += kDecThreads) kpos_s[pp] = kpos_entry(L, p.slot_chan, h, pp);
    for (int q = tid; q < npg; q += kDecThreads) esc_s[q] = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // ------------------------------------------------------------ control warp
  if (warp == 4) {
    if (lane == 0) {
      const uint64_t kLimit = kWaitLimitNs;
      int issued[kStages] = {0, 0};
      for (int i = 0; i < kStages && i < npg; ++i) {
        uint64_t* full = &bars[kBarFull + i];
        mbar_arrive_expect_tx(full, row_bytes + (i == 0 ? meta_bytes : 0u));
        if (i == 0 && meta_bytes) bulk_g2s(smem + S.meta, p.kmeta + (head_meta + pg0) * M, meta_bytes, full);
        bulk_g2s(stage0 + i * S.stage_bytes, p.rows + (head_row + static_cast<int64_t>(pg0 + i) * kP) * R,
                 row_bytes, full);
        ++issued[i];
      }
      // Descriptors: QK B per K step, PV A/B per K step and Value-tile parity.
      const uint32_t n_ks = static_cast<uint32_t>(S.kpad / 32);
      const uint64_t bqk_desc0 = smem_desc(bqk, 128, S.bqk_sbo);
      const uint64_t apv_desc0 = smem_desc(apv, 128, 2048);
      const uint64_t bpv_desc0 = smem_desc(bpv, 128, 2048);
      int qk_open = 0, pv_open = 0;
      for (int i = 0; i < npg; ++i) {
        if (!*abort_s && !mbar_wait_bounded(&bars[kBarKReady], i & 1, kLimit)) *abort_s = 1;
        tc_fence_after();
        for (uint32_t ks = 0; ks < n_ks; ++ks)  // +512 B per K step = +32 in descriptor units
          mma_u8_ts(tmem + S.tm_qk, tmem + S.a_col + 8 * ks, bqk_desc0 + 32 * ks, kIdescQK, ks > 0 ? 1u : 0u);
        mma_commit(&bars[kBarQK]);
        qk_open = i + 1;
        if (!*abort_s && !mbar_wait_bounded(&bars[kBarVReady], i & 1, kLimit)) *abort_s = 1;
        tc_fence_after();
        const uint64_t a_tile = apv_desc0 + static_cast<uint64_t>((i & 1) * (kP * kD / 16));
#pragma unroll
        for (int ks = 0; ks < kP / 32; ++ks)
          mma_u8_ss(tmem + S.tm_pv, a_tile + 32 * ks, bpv_desc0 + 32 * ks, kIdescPV, ks > 0 ? 1u : 0u);
        mma_commit(&bars[kBarPV]);
        pv_open = i + 1;
        // Stage i % kStages has been read by U(i) and S(i): it takes page i + kStages.
        if (i + kStages < npg && !*abort_s) {
          const int st = i % kStages;
          uint64_t* full = &bars[kBarFull + st];
          mbar_arrive_expect_tx(full, row_bytes);
          bulk_g2s(stage0 + st * S.stage_bytes,
                   p.rows + (head_row + static_cast<int64_t>(pg0 + i + kStages) * kP) * R, row_bytes, full);
          ++issued[st];
        }
      }
      if (*abort_s) {
        // Drain this CTA's copies and MMAs before its shared memory and TMEM go away.
        for (int st = 0; st < kStages; ++st)
          if (issued[st]) mbar_wait_bounded(&bars[kBarFull + st], (issued[st] - 1) & 1, kLimit);
        if (qk_open) mbar_wait_bounded(&bars[kBarQK], (qk_open - 1) & 1, kLimit);
        if (pv_open) mbar_wait_bounded(&bars[kBarPV], (pv_open - 1) & 1, kLimit);
        if (p.status != nullptr) atomicExch(p.status, LF_ERR_DEVICE_TIMEOUT);
      }
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();  // compute warps finished (their partial is written)
    tc_fence_after();
    tmem_dealloc(tmem, S.tm_cols);
    return;
  }

  // ----------------------------------------------------------- compute warps
  float mg[GQ], og[GQ], ltg[GQ], lvtg[GQ];
#pragma unroll
  for (int j = 0; j < GQ; ++j) {
    mg[j] = -INFINITY;
    og[j] = ltg[j] = lvtg[j] = 0.f;
  }
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  const uint64_t kLimit = kWaitLimitNs;
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if (*abort_s) return;
    if (!mbar_wait_bounded(bar, parity, kLimit)) *abort_s = 1;
  };

  // Per-q-head block exponent of the query: max_c |q_j[c]| <= 2^eq_j.
  int eq[GQ];
#pragma unroll
  for (int j = 0; j < GQ; ++j) {
    const uint32_t mx = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(q_s[j * kD + tid])));
    if (lane == 0) red_m[warp * 16 + j] = mx;
  }
  for (int i = tid; i < L.width[3] * kGQ; i += kDecThreads) {
    const int ii = i / kGQ, j = i % kGQ;
    const int ch = p.slot_chan[(3 * H + h) * kD + ii];
    q16_s[i] = ch < 0 ? 0.f : q_s[j * kD + ch];
  }
  named_sync(1, kDecThreads);
#pragma unroll
  for (int j = 0; j < GQ; ++j) {
    const uint32_t mx = max(max(red_m[j], red_m[16 + j]), max(red_m[32 + j], red_m[48 + j]));
    eq[j] = max(-60, min(60, exp2_ceil(__uint_as_float(mx))));
  }
  // This thread's QK B rows: K positions tid and tid+128 (scaled query values).
  float qq[2][GQ];
  int soff[2], moff[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int pp = tid + k * kDecThreads;
    const int e = pp < S.kpad ? kpos_s[pp] : -1;
    soff[k] = moff[k] = -1;
    if (e >= 0) {
      const int tier = (e >> 16) & 3, slot = e >> 18;
      soff[k] = L.scale_off[tier] + slot;
      moff[k] = L.min_off[tier] + slot;
    }
#pragma unroll
    for (int j = 0; j < GQ; ++j) qq[k][j] = e >= 0 ? q_s[j * kD + (e & 0xFFFF)] * exp2i(22 - eq[j]) : 0.f;
  }
  // A columns past the packed slots stay zero for the whole item.
  for (int c = n_slots_of(L) / 4; c < S.kpad / 4; ++c) tmem_st_x1(tmem + lane_base + S.a_col + c, 0u);
  const float c2 = p.scaling * kLog2e;

  // Page-0 data (with the item's meta rows) -> per-page Key-scale exponents.
  wait(&bars[kBarFull + 0], 0);
  for (int q = 0; q < npg; ++q) {
    float mx = 0.f;
#pragma unroll
    for (int k = 0; k < 2; ++k)
      if (soff[k] >= 0) mx = fmaxf(mx, half_bits_to_float(meta_s[q * M + soff[k]]));
    const uint32_t wmax = __reduce_max_sync(0xffffffffu, __float_as_uint(mx));
    if (lane == 0) atomicMax(reinterpret_cast<unsigned int*>(esc_s) + q, wmax);
  }
  named_sync(1, kDecThreads);  // also: every read of the query staging (second Value tile) is done
  for (int q = tid; q < npg; q += kDecThreads) esc_s[q] = max(-60, min(60, exp2_ceil(__uint_as_float(esc_s[q]))));
  named_sync(1, kDecThreads);

  // U(i): one pass over the token's row -- Key codes -> TMEM, Value codes ->
  // Value tile (i & 1), QK B rows for this thread's slots, bias partials.
  auto unpack = [&](int i) {
    const uint32_t* rowp = reinterpret_cast<const uint32_t*>(stage0 + (i % kStages) * S.stage_bytes) + tid * R;
    uint32_t vw[kD / 16];
#pragma unroll
    for (int w = 0; w < kD / 16; ++w) vw[w] = rowp[L.vcode_off + w];
    const uint16_t* mrow = meta_s + i * M;
    float msc[2], mmn[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      msc[k] = soff[k] >= 0 ? half_bits_to_float(mrow[soff[k]]) : 0.f;
      mmn[k] = soff[k] >= 0 ? half_bits_to_float(mrow[moff[k]]) : 0.f;
    }
    uint32_t col = tmem + lane_base + S.a_col;
    {
      const uint32_t* src = rowp + L.code_off[0];
#pragma unroll 4
      for (int w = 0; w < L.words[0]; ++w) {
        const uint32_t x = src[w];
        tmem_st_x4(col + 4 * w, x & kM2, (x >> 2) & kM2, (x >> 4) & kM2, (x >> 6) & kM2);
      }
      col += 4 * L.words[0];
    }
    {
      const uint32_t* src = rowp + L.code_off[1];
#pragma unroll 4
      for (int w = 0; w < L.words[1]; ++w) {
        const uint32_t x = src[w];
        tmem_st_x2(col + 2 * w, x & kM4, (x >> 4) & kM4);
      }
      col += 2 * L.words[1];
    }
    {
      const uint32_t* src = rowp + L.code_off[2];
#pragma unroll 4
      for (int w = 0; w < L.words[2]; ++w) tmem_st_x1(col + w, src[w]);
    }
    {
      unsigned char* dst = apv + (i & 1) * (kP * kD) + (tid & 7) * 16 + (tid >> 3) * 128;
#pragma unroll
      for (int w = 0; w < kD / 16; ++w) {
        const uint32_t x = vw[w];
        *reinterpret_cast<uint4*>(dst + w * 2048) = make_uint4(x & kM2, (x >> 2) & kM2, (x >> 4) & kM2, (x >> 6) & kM2);
      }
    }
    float bias[kGQ];
#pragma unroll
    for (int j = 0; j < kGQ; ++j) bias[j] = 0.f;
    const float fsc = exp2i(-esc_s[i]);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int pp = tid + k * kDecThreads;
      if (pp >= S.kpad) break;
      uint4 c0 = make_uint4(0u, 0u, 0u, 0u), c1 = c0;
      if (soff[k] >= 0) {
        const float sc = msc[k] * fsc;
        uint32_t U[kGQ];
#pragma unroll
        for (int j = 0; j < kGQ; ++j) {
          if (j < GQ) {
            // rint(qq * sc) + 2^23 via the fp32 magic constant 1.5 * 2^23.
            U[j] = __float_as_uint(fmaf(qq[k][j], sc, 12582912.0f)) - 0x4AC00000u;
            bias[j] = fmaf(qq[k][j], mmn[k], bias[j]);
          } else {
            U[j] = 0x800000u;  // X = 0
          }
        }
        pack_limbs(U, c0, c1, 1u);
      }
      unsigned char* dst = bqk + (pp & 7) * 16 + (pp >> 3) * 128;
      *reinterpret_cast<uint4*>(dst) = c0;
      *reinterpret_cast<uint4*>(dst + S.bqk_sbo) = c1;
    }
    const float part = warp_sum8_scatter(bias, lane);
    if ((lane & 3) == 0)
      red_b[(i & 1) * 32 + warp * kGQ + (((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1))] = part;
    tmem_wait_st();
    fence_proxy_async_smem();
    tc_fence_before();
    mbar_arrive(&bars[kBarKReady]);
  };

  float alpha[GQ];
  int ev[GQ];
  // Iteration i runs S(i), U(i+1), C(i); iteration -1 only U(0).
  for (int i = -1; i < npg; ++i) {
    if (i < 0) {
      unpack(0);
      continue;
    }
    // S(i): scores, page max, online softmax, PV B rows.  The FP16 Key tier
    // (CUDA cores) and the token's Value scale / min come from the page's
    // stage, resident until this page's V-ready arrive.
    const uint16_t* row16 =
        reinterpret_cast<const uint16_t*>(stage0 + (i % kStages) * S.stage_bytes) + 2 * tid * R + 2 * L.half_off;
    float s16[GQ];
#pragma unroll
    for (int j = 0; j < GQ; ++j) s16[j] = 0.f;
#pragma unroll 4
    for (int c = 0; c < L.width[3]; ++c) {
      const float kv = half_bits_to_float(row16[c]);
      const float4 qa = *reinterpret_cast<const float4*>(q16_s + c * kGQ);
      const float4 qb = *reinterpret_cast<const float4*>(q16_s + c * kGQ + 4);
      const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
      for (int j = 0; j < GQ; ++j) s16[j] = fmaf(qv[j], kv, s16[j]);
    }
    const float vs_i = half_bits_to_float(row16[L.width[3]]);
    const float vm_i = half_bits_to_float(row16[L.width[3] + 1]);
    const int esc = esc_s[i];
    wait(&bars[kBarQK], i & 1);
    tc_fence_after();
    uint32_t acc[32];
    tmem_ld_x32_sync(tmem + lane_base + S.tm_qk, acc);
    const int ones = static_cast<int>(acc[24]);
    float x[GQ];
    uint32_t* rm = red_m + (i & 1) * 64;
    uint32_t keys[12];
#pragma unroll
    for (int j = 0; j < 12; ++j) keys[j] = 0u;
#pragma unroll
    for (int j = 0; j < GQ; ++j) {
      const int lo = static_cast<int>(acc[j]) + (static_cast<int>(acc[8 + j]) << 8);
      const float sint = fmaf(static_cast<float>(static_cast<int>(acc[16 + j]) - 128 * ones), 65536.f,
                              static_cast<float>(lo));
      x[j] = fmaf(sint, c2 * exp2i(eq[j] + esc - 22), s16[j] * c2);
      keys[j] = order_key(x[j]);
    }
    keys[8] = __float_as_uint(vs_i);
#pragma unroll
    for (int j = 0; j < GQ; ++j) keys[j] = __reduce_max_sync(0xffffffffu, keys[j]);
    keys[8] = __reduce_max_sync(0xffffffffu, keys[8]);
    if (lane == 0) {
      *reinterpret_cast<uint4*>(rm + warp * 16) = make_uint4(keys[0], keys[1], keys[2], keys[3]);
      *reinterpret_cast<uint4*>(rm + warp * 16 + 4) = make_uint4(keys[4], keys[5], keys[6], keys[7]);
      *reinterpret_cast<uint4*>(rm + warp * 16 + 8) = make_uint4(keys[8], 0u, 0u, 0u);
    }
    named_sync(1, kDecThreads);
    uint32_t U[kGQ];
    {
      uint32_t km[12];
      float bs[8];
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const uint4 k0 = *reinterpret_cast<const uint4*>(rm + w * 16);
        const uint4 k1 = *reinterpret_cast<const uint4*>(rm + w * 16 + 4);
        const uint4 k2 = *reinterpret_cast<const uint4*>(rm + w * 16 + 8);
        const float4 b0 = *reinterpret_cast<const float4*>(red_b + (i & 1) * 32 + w * 8);
        const float4 b1 = *reinterpret_cast<const float4*>(red_b + (i & 1) * 32 + w * 8 + 4);
        const uint32_t kk[12] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w, k2.x, k2.y, k2.z, k2.w};
        const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
        for (int e = 0; e < 9; ++e) km[e] = w == 0 ? kk[e] : max(km[e], kk[e]);
#pragma unroll
        for (int e = 0; e < 8; ++e) bs[e] = w == 0 ? bb[e] : bs[e] + bb[e];
      }
      const int ev_vs = max(-60, min(60, exp2_ceil(__uint_as_float(km[8]))));
#pragma unroll
      for (int j = 0; j < kGQ; ++j) {
        if (j < GQ) {
          const float bias = bs[j] * (c2 * exp2i(eq[j] - 22));
          const float pm = order_key_to_float(km[j]) + bias;
          const float mnew = fmaxf(mg[j], pm);
          alpha[j] = mg[j] == -INFINITY ? 0.f : ex2(mg[j] - mnew);
          mg[j] = mnew;
          const float pj = ex2(x[j] + bias - mnew);
          // Bound on p * vscale over the page: 2^(pm - mnew) * max vscale.
          ev[j] = ev_vs + max(-60, static_cast<int>(ceilf(pm - mnew)));
          ltg[j] = fmaf(ltg[j], alpha[j], pj);
          lvtg[j] = fmaf(lvtg[j], alpha[j], pj * vm_i);
          // rint(p * vs * 2^(23 - ev)) via the fp32 magic constant 2^23.
          U[j] = __float_as_uint(fmaf(pj, vs_i * exp2i(23 - ev[j]), 8388608.0f)) - 0x4B000000u;
        } else {
          U[j] = 0u;
        }
      }
    }
    {
      uint4 c0, c1;
      pack_limbs(U, c0, c1, 0u);
      unsigned char* dst = bpv + (tid & 7) * 16 + (tid >> 3) * 128;
      *reinterpret_cast<uint4*>(dst) = c0;
      *reinterpret_cast<uint4*>(dst + 2048) = c1;
    }
    fence_proxy_async_smem();
    tc_fence_before();
    mbar_arrive(&bars[kBarVReady]);
    // U(i+1) while PV(i) runs.
    if (i + 1 < npg) {
      wait(&bars[kBarFull + (i + 1) % kStages], ((i + 1) / kStages) & 1);
      unpack(i + 1);
    }
    // C(i): accumulate this thread's head-dim position.
    wait(&bars[kBarPV], i & 1);
    tc_fence_after();
    tmem_ld_x32_sync(tmem + lane_base + S.tm_pv, acc);
#pragma unroll
    for (int j = 0; j < GQ; ++j) {
      const int lo = static_cast<int>(acc[j]) + (static_cast<int>(acc[8 + j]) << 8);
      const float v = fmaf(static_cast<float>(static_cast<int>(acc[16 + j])), 65536.f, static_cast<float>(lo));
      og[j] = fmaf(og[j], alpha[j], v * exp2i(ev[j] - 23));
    }
  }

#pragma unroll
  for (int j = 0; j < GQ; ++j) mg[j] *= kLn2;  // log2 units -> natural-log units
  // PV row t holds head-dim channel d(t): t = 16w + 4k + i  <->  d = 16w + k + 4i.
  const int d = (tid & ~15) + ((tid & 15) >> 2) + 4 * (tid & 3);
  write_partial_group<GQ>(p, b, h, s, d, og, mg, ltg, lvtg, red_w, 1);
  tc_fence_before();
  __syncthreads();
}

}  // namespace tc

bool tc_supported(const lf_layout& L, int gq, int pps) {
  if (L.head_dim != tc::kD || L.page_size != tc::kP || L.k_group != tc::kP || L.v_group != tc::kD) return false;
  if (L.bit_v != 2 || gq > kGQ || gq < 1) return false;
  if (tc::n_slots_of(L) > 2 * kDecThreads) return false;  // two K positions per compute thread
  if (pps > tc::kMaxPagesPerItem) return false;
  const tc::TcSmem S = tc::tc_smem(L, pps);
  // The residual split's fp32 rows must end before the query staging.
  if (S.stage0 + resid_smem(tc::kD).total > S.qs) return false;
  return S.total <= 227 * 1024;
}

template <int GQ>
static void* tc_kernel_ptr() {
  return reinterpret_cast<void*>(tc::decode_partial_tc<GQ>);
}
static void* tc_kernel_for(int gq) {
  switch (gq) {
    case 1: return tc_kernel_ptr<1>();
    case 2: return tc_kernel_ptr<2>();
    case 3: return tc_kernel_ptr<3>();
    case 4: return tc_kernel_ptr<4>();
    case 5: return tc_kernel_ptr<5>();
    case 6: return tc_kernel_ptr<6>();
    case 7: return tc_kernel_ptr<7>();
    default: return tc_kernel_ptr<8>();
  }
}

int occupancy_tc(const lf_layout& L, int gq, int pps) {
  const tc::TcSmem S = tc::tc_smem(L, pps);
  if (S.total > 227 * 1024) return 0;
  void* kern = tc_kernel_for(gq);
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S.total);
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kern, tc::kThreads, S.total) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  const int by_tmem = 512 / S.tm_cols;
  return blocks < by_tmem ? blocks : by_tmem;
}

int launch_partial_tc(const DecodeParams& p, int resid_dtype, int q_dtype, cudaStream_t stream) {
  DecodeParams q = p;
  q.resid_dtype = resid_dtype;
  q.q_dtype = q_dtype;
  const tc::TcSmem S = tc::tc_smem(q.L, q.pps);
  void* kern = tc_kernel_for(q.gq);
  static std::atomic<int> configured[kGQ + 1];
  if (S.total > 48 * 1024 && S.total > configured[q.gq].load()) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S.total);
    if (e != cudaSuccess) {
      set_error("lf_decode_partial (tcgen05): shared memory %d B: %s", S.total, cudaGetErrorString(e));
      return LF_ERR_UNSUPPORTED;
    }
    configured[q.gq].store(S.total);
  }
  dim3 grid(q.max_splits, q.L.kv_heads, q.batch);
  void* args[] = {&q};
  cudaError_t e = cudaLaunchKernel(kern, grid, dim3(tc::kThreads), args, S.total, stream);
  if (e != cudaSuccess) {
    set_error("lf_decode_partial (tcgen05): %s", cudaGetErrorString(e));
    return LF_ERR_LAUNCH;
  }
  return launch_status("lf_decode_partial (tcgen05)");
}

}  // namespace lf
