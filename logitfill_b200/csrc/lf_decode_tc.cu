// K2 on the 5th-generation tensor cores (sm_100a, tcgen05.mma kind::i8).
//
// Geometry: head_dim 128, page 128 = Key group 128, Value group 128, bit_v 2
// (the LogitFill defaults, deepseek_qwen.py:24-46).  One CTA per (split, KV
// head, sequence) work item: four compute warps (thread t owns token t of the
// current page, TMEM lane t and row t of the PV result) and one control warp.
//
// Control warp: waits on the barriers with all lanes converged; one elected
// lane issues the 1-D bulk copies (a page's row block and meta row per stage)
// and the MMAs, and nothing else, so that each MMA starts as soon as its
// operands are ready.  Issuing from the converged warp keeps the MMA operands
// (TMEM base, descriptors) in uniform registers.
// Compute warps, per page i:
//   U_K  Key codes -> u8 in TMEM (A of QK, K-major), masked in place (INT2
//        slot k of a byte as code * 4^k, INT4 as code * 16^k); the B row of QK
//        for K position t (tier slot c, code weight w_c): for each q-head j the
//        fixed point X = rint(q_j[c] scale_c 2^(29-Eq-Es) / w_c), offset by 2^30: its four
//        bytes are the unsigned limbs, column 4 j + l of the row; K positions 128 and up (wide layouts)
//        take four lanes each, two q-heads per lane; Es is the page's Key-scale exponent, from
//        the largest scale the packer stores in the meta row; partial sums of
//        the Key-min bias sum_c q_j[c] min_c; the token's code sum n_t (the
//        byte sum of its code words, which is the sum of its A row).
//   S    score_tj = 2^(Eq+Es-29) (acc0 + 2^8 acc1 + 2^16 (acc2 + 2^8 (acc3 - 64 n_t)))
//        + FP16-tier part + bias_j; page max per q-head; online softmax with
//        the per-q-head statistics held by lane j of every warp; the B row of
//        PV for token t: rint(p_tj vscale_t 2^(23-Ev)) in three limbs, Ev the
//        page's Value-scale exponent (p <= 1 after the max update).
//   C    o_j += 2^(Ev-23) 4^-k(t) (acc0 + 256 acc1 + 65536 acc2).
//   U_V  Value codes -> u8 in shared memory (A of PV, MN-major), each 2-bit
//        code masked in place, so row t holds code * 4^k(t), k(t) = (t>>2)&3;
//        C removes the power of two exactly.
// Order: S(i), U_K(i+1), C(i), U_V(i+1).  QK(i+1) overlaps C(i) and U_V(i+1),
// PV(i) overlaps U_K(i+1).  Stage i % 2 takes page i + 2 as soon as S(i) has
// read its FP16 tier (the stage's last reader), before S(i)'s softmax.
//
// The integer products are exact; the fixed-point rounding is 2^-29 w_c (QK,
// w_c <= 64) and 2^-23 (PV) of the block maxima (tests/kernel_model.py models
// it).  Every
// mbarrier wait is bounded (2 s).  On expiry the CTA records
// LF_ERR_DEVICE_TIMEOUT, stops waiting (every warp still passes the same
// barriers, so nothing deadlocks), drains its own copies and MMAs, frees its
// TMEM and returns.
#include <algorithm>

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
constexpr int kMaxPagesPerItem = 64;

constexpr int kNumBarsMax = 7;

struct TcSmem {
  int bars, red, redb, redw, q16, qhi, posoff, stage0, bqk, bpv, apv, qs, total;
  int kpad, a_cols, tm_qk, tm_pv, tm_cols, bqk_sbo, rows_bytes, meta_bytes, stage_bytes;
};

__host__ __device__ inline int n_slots_of(const lf_layout& L) {
  return 16 * L.words[0] + 8 * L.words[1] + 4 * L.words[2];
}

__host__ __device__ inline TcSmem tc_smem(const lf_layout& L) {
  TcSmem s;
  const int ns = n_slots_of(L);
  s.kpad = ns == 0 ? 32 : (ns + 31) / 32 * 32;
  s.a_cols = s.kpad / 4;
  s.tm_qk = (s.a_cols + 31) / 32 * 32;
  s.tm_pv = s.tm_qk + 32;
  int need = s.tm_pv + 32, cols = 32;
  while (cols < need) cols *= 2;
  s.tm_cols = cols;
  s.bqk_sbo = s.kpad * 16;
  s.rows_bytes = kP * L.row_words * 4;
  s.meta_bytes = L.meta_halves * 2;
  s.stage_bytes = (s.rows_bytes + s.meta_bytes + 15) / 16 * 16;
  // Four CTAs share an SM up to 57 344 B each (228 KB per SM, 1 KB reserved
  // per CTA); a 160-position layout with 29-word rows needs exactly that.
  int off = 0;
  s.bars = off; off += 8 * kNumBarsMax + 8;  // mbarriers, TMEM address, abort flag
  s.red = off; off += 2 * 4 * 12 * 4;   // page maxima [stage][warp][12]: 8 score maxima, Value-scale bits
  s.redw = s.red;                        // item-end sums (after the page loop, in place of the page maxima)
  s.redb = off; off += 2 * 4 * kGQ * 4;  // bias partials [stage][compute warp][8]
  s.q16 = off; off += ((L.width[3] > 0 ? L.width[3] : 1) * kGQ * 4 + 15) / 16 * 16;
  // K positions 128..159 live in registers; 160.. (K up to 256) here.
  const int hi = s.kpad > kDecThreads + 32 ? s.kpad - kDecThreads - 32 : 0;
  s.qhi = off; off += hi * kGQ * 4;
  s.posoff = off; off += hi * 4;
  off = (off + 127) / 128 * 128;
  s.stage0 = off; off += kStages * s.stage_bytes;
  s.bqk = off; off += s.kpad * 32;
  s.bpv = off; off += kP * 32;
  s.apv = off; off += kP * kD;
  // The query staging (prologue only) takes the end of the Value tile, or
  // more room after it when the residual split's rows reach further.
  const int resid_end = s.stage0 + resid_smem(kD).total;
  s.qs = (s.apv + kP * kD - kGQ * kD * 4);
  if (s.qs < resid_end) s.qs = (resid_end + 15) / 16 * 16;
  if (s.qs + kGQ * kD * 4 > off) off = s.qs + kGQ * kD * 4;
  s.total = (off + 127) / 128 * 128;
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

// B rows of both MMAs order their 32 columns (q-head j, limb l) as n = 4 j + l:
// a 32-byte row is the eight 32-bit words U[0..7] as they lie in registers
// (byte l of U[j] is limb l), stored as two 16-byte halves (columns 0-15 and
// 16-31 of the MN-major core matrices, sbo bytes apart).
__device__ __forceinline__ void store_b_row(unsigned char* dst, int sbo, const uint32_t (&U)[kGQ]) {
  *reinterpret_cast<uint4*>(dst) = make_uint4(U[0], U[1], U[2], U[3]);
  *reinterpret_cast<uint4*>(dst + sbo) = make_uint4(U[4], U[5], U[6], U[7]);
}

// Per-q-head float arithmetic two q-heads at a time: pair(j) for heads j,
// j + 1 (packed fp32x2 instructions, sm_100a, each lane rounded as the
// scalar instruction, so the results are bit-identical) and one(N - 1) for
// an odd last head.
template <int N, typename F2, typename F1>
__device__ __forceinline__ void by_pairs(F2 pair, F1 one) {
#pragma unroll
  for (int j = 0; j + 1 < N; j += 2) pair(j);
  if (N & 1) one(N - 1);
}
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

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

// Warp maximum of a float (redux.sync .f32, sm_100a).
__device__ __forceinline__ float warp_max_f32(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
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
enum { kBarFull = 0, kBarKReady = kStages, kBarVReady, kBarQK, kBarPV, kBarFree, kNumBars };
static_assert(kNumBars <= kNumBarsMax, "barrier slots");

// One B row of QK (K position pp; qv = q_j[c] 2^(29-Eq) / w_c, zero for a
// padding position) and its Key-min bias terms.  X = rint(qv * scale) has
// |X| <= 2^29, so U = X + 2^30 is an unsigned 31-bit number: its four bytes
// are the limbs.
template <int GQ>
__device__ __forceinline__ void qk_b_row(unsigned char* bqk, int sbo, int pp, const float (&qv)[kGQ], float sc,
                                         float mn, float (&bias)[kGQ]) {
  uint32_t U[kGQ];
  float y[kGQ];
  by_pairs<GQ>(
      [&](int j) {
        const float2 q2 = f2(qv[j], qv[j + 1]);
        const float2 y2 = __fmul2_rn(q2, f2(sc, sc));
        const float2 b2 = __ffma2_rn(q2, f2(mn, mn), f2(bias[j], bias[j + 1]));
        y[j] = y2.x;
        y[j + 1] = y2.y;
        bias[j] = b2.x;
        bias[j + 1] = b2.y;
      },
      [&](int j) {
        y[j] = qv[j] * sc;
        bias[j] = fmaf(qv[j], mn, bias[j]);
      });
#pragma unroll
  for (int j = 0; j < kGQ; ++j)
    U[j] = j < GQ ? static_cast<uint32_t>(__float2int_rn(y[j]) + (1 << 30)) : 1u << 30;  // X = 0 past GQ
  store_b_row(bqk + (pp & 7) * 16 + (pp >> 3) * 128, sbo, U);
}

// Two q-heads (2 hp, 2 hp + 1) of the B row of QK at K position pp: the
// same words as qk_b_row, one 8-byte store (columns 8 hp .. 8 hp + 7).
__device__ __forceinline__ void hi_b_row_pair(unsigned char* bqk, int sbo, int pp, int hp, float2 qv, float sc) {
  const float2 y = __fmul2_rn(qv, f2(sc, sc));
  const uint32_t ua = static_cast<uint32_t>(__float2int_rn(y.x) + (1 << 30));
  const uint32_t ub = static_cast<uint32_t>(__float2int_rn(y.y) + (1 << 30));
  unsigned char* dst = bqk + (pp & 7) * 16 + (pp >> 3) * 128 + (hp >= 2 ? sbo : 0) + 8 * (hp & 1);
  *reinterpret_cast<uint2*>(dst) = make_uint2(ua, ub);
}

// K position descriptor: meta offsets of the slot's scale and min, and the
// power of two its unpacked code carries.  The Key codes are masked in place
// without shifting, so INT2 slot 4i + k of a word reaches the MMA as
// code * 4^k and INT4 slot 2i + k as code * 16^k; the B row divides by the
// same power of two (exact in fp32) and the min, multiplied back, keeps the
// bias exact.
__device__ __forceinline__ int pos_desc(const lf_layout& L, int e) {
  if (e < 0) return -1;
  const int tier = (e >> 16) & 3, slot = e >> 18;
  const int lg = tier == 0 ? 2 * (slot & 3) : tier == 1 ? 4 * (slot & 1) : 0;
  return (L.scale_off[tier] + slot) | ((L.min_off[tier] + slot) << 13) | (lg << 26);
}
__device__ __forceinline__ int pos_scale(int po) { return po & 0x1FFF; }
__device__ __forceinline__ int pos_min(int po) { return (po >> 13) & 0x1FFF; }
__device__ __forceinline__ int pos_lg(int po) { return (po >> 26) & 7; }

// The page's Key-scale exponent: largest stored INT2/INT4/INT8 scale <= 2^Es.
__device__ __forceinline__ int page_scale_exp(const uint16_t* meta, int kmax_off) {
  return max(-60, min(60, exp2_ceil(half_bits_to_float(meta[kmax_off]))));
}

template <int GQ>
__global__ void __launch_bounds__(kThreads, 4) decode_partial_tc(DecodeParams p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const lf_layout& L = p.L;
  const TcSmem S = tc_smem(L);
  // Grid: x = (sequence, KV head) pair, y = split, z = virtual-head chunk.
  // Blocks launch in x-fastest order, so every pair's first splits start
  // together and the short residual splits (the last y) take the SMs the page
  // splits leave.
  const int s = blockIdx.y, vc = blockIdx.z, tid = threadIdx.x;
  const int h = blockIdx.x % p.L.kv_heads, b = blockIdx.x / p.L.kv_heads;
  const int lane = tid & 31, warp = tid >> 5;
  const int H = L.kv_heads, R = L.row_words, M = L.meta_halves;
  grid_dep_wait();
  grid_dep_trigger();
  const int pages = p.hist_tokens[b] / kP;
  const int n_page_splits = (pages + p.pps - 1) / p.pps;
  if (s >= n_page_splits + residual_splits(kP, p.q_len)) return;

  float* q_s = reinterpret_cast<float*>(smem + S.qs);
  float* red_w = reinterpret_cast<float*>(smem + S.redw);
  if (s >= n_page_splits) {  // residual splits: tail rows + new token, fp32 (compute warps)
    if (warp >= 4) return;
    float m[kGQ], o[kGQ], lt[kGQ];
#pragma unroll
    for (int j = 0; j < kGQ; ++j) {
      m[j] = -INFINITY;
      o[j] = lt[j] = 0.f;
    }
    residual_chunk(p, b, h, vc, s - n_page_splits, q_s, true, smem + S.stage0, m, o, lt);
    write_partial_resid(p, item_index(p, b, h, vc, s), o, m, lt);
    return;
  }

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S.bars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S.bars + 8 * kNumBars);
  volatile int* abort_s = reinterpret_cast<volatile int*>(smem + S.bars + 8 * kNumBars + 4);
  uint32_t* red_m = reinterpret_cast<uint32_t*>(smem + S.red);  // [stage][warp][12]: 8 score maxima (bits), vscale
  float* red_b = reinterpret_cast<float*>(smem + S.redb);        // [stage][4][8] bias partials
  float* q16_s = reinterpret_cast<float*>(smem + S.q16);         // [FP16 slot][kGQ], times scaling*log2(e)
  float* qhi_s = reinterpret_cast<float*>(smem + S.qhi);         // K positions 160..: q_j[c] 2^(29-Eq) / w_c
  int* posoff_s = reinterpret_cast<int*>(smem + S.posoff);       // K positions 160..: pos_desc, or -1
  unsigned char* stage0 = smem + S.stage0;
  unsigned char* bqk = smem + S.bqk;
  unsigned char* bpv = smem + S.bpv;
  unsigned char* apv = smem + S.apv;

  const int pg0 = s * p.pps;
  const int npg = min(pages, pg0 + p.pps) - pg0;
  const int64_t head_row = (static_cast<int64_t>(b) * H + h) * L.row_cap;
  const int64_t head_meta = (static_cast<int64_t>(b) * H + h) * L.group_cap;
  const float c2 = p.scaling * kLog2e;
  const int kmax_off = L.kmax_off;
  const int n_hi = S.kpad > kDecThreads ? (S.kpad - kDecThreads) / 32 : 0;  // K positions 128.. per 4 lanes

  // Page pg of the item -> stage pg % 2 (row block + meta row); one thread.
  auto issue_page = [&](int pg) {
    unsigned char* dst = stage0 + (pg & 1) * S.stage_bytes;
    uint64_t* full = &bars[kBarFull + (pg & 1)];
    mbar_arrive_expect_tx(full, static_cast<uint32_t>(S.rows_bytes + S.meta_bytes));
    bulk_g2s(dst, p.rows + (head_row + static_cast<int64_t>(pg0 + pg) * kP) * R, S.rows_bytes, full);
    bulk_g2s(dst + S.rows_bytes, p.kmeta + (head_meta + pg0 + pg) * M, S.meta_bytes, full);
  };

  if (tid == kDecThreads) {
#pragma unroll
    for (int i = 0; i < kStages; ++i) mbar_init(&bars[kBarFull + i], 1);
    mbar_init(&bars[kBarKReady], kDecThreads);
    mbar_init(&bars[kBarVReady], kDecThreads);
    mbar_init(&bars[kBarQK], 1);
    mbar_init(&bars[kBarPV], 1);
    mbar_init(&bars[kBarFree], kDecThreads);  // the compute warps' last read of a stage
    *abort_s = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
    // The first page loads while the CTA stages its query.
    issue_page(0);
  }
  if (warp == 4) {
    tmem_alloc(tmem_slot, S.tm_cols);
    tmem_relinquish();
  }
  float qq[kGQ];   // compute thread: q_j[c] 2^(29-Eq) / w_c of its K position
  int po = -1;     // compute thread: pos_desc of its K position, or -1
  // Compute thread: q-heads 2 hp, 2 hp + 1 of K position 128 + (tid >> 2)
  // (wide layouts) and that position's pos_desc.
  const int hp = tid & 3;
  float2 qv_hi = make_float2(0.f, 0.f);
  int po_hi = -1;
  int eq = 0;
  if (tid < kDecThreads) {
    // Query group (thread = channel), its block exponent Eq
    // (max_j,c |q_j[c]| <= 2^Eq), and the scaled query of each K position.
    // Every global load of the prologue is issued here, before any use.
    const int e = tid < S.kpad ? kpos_entry(L, p.slot_chan, h, tid) : -1;
    const int e_hi = kDecThreads < S.kpad ? kpos_entry(L, p.slot_chan, h, kDecThreads + (tid >> 2)) : -1;
    const int e2 = kDecThreads + 32 + tid < S.kpad ? kpos_entry(L, p.slot_chan, h, kDecThreads + 32 + tid) : -1;
    const int n16 = L.width[3] * kGQ;
    const int ch16 = tid < n16 ? p.slot_chan[(3 * H + h) * kD + tid / kGQ] : -1;
    float qc[kGQ];
    {
      // Virtual heads vc*GQ + j: q-head jh, query token ii, stepped in order.
      const int v0 = vc * GQ;
      const int jh0 = v0 / p.q_len, ii0 = v0 - jh0 * p.q_len;
      const int64_t qb = b * p.q_seq_stride + static_cast<int64_t>(h) * p.gq * p.q_head_stride + tid;
      auto gather = [&](auto load) {
        int jh = jh0, ii = ii0;
#pragma unroll
        for (int j = 0; j < kGQ; ++j) {
          qc[j] = j < GQ ? load(qb + jh * p.q_head_stride + ii * p.q_tok_stride) : 0.f;
          if (++ii == p.q_len) {
            ii = 0;
            ++jh;
          }
        }
      };
      if (p.q_dtype == LF_F32) {
        const float* qp = static_cast<const float*>(p.q);
        gather([&](int64_t o) { return qp[o]; });
      } else if (p.q_dtype == LF_F16) {
        const __half* qp = static_cast<const __half*>(p.q);
        gather([&](int64_t o) { return __half2float(qp[o]); });
      } else {
        const __nv_bfloat16* qp = static_cast<const __nv_bfloat16*>(p.q);
        gather([&](int64_t o) { return __bfloat162float(qp[o]); });
      }
    }
    float qmax = 0.f;
#pragma unroll
    for (int j = 0; j < kGQ; ++j) {
      q_s[j * kD + tid] = qc[j];
      qmax = fmaxf(qmax, fabsf(qc[j]));
    }
    const uint32_t wmax = __reduce_max_sync(0xffffffffu, __float_as_uint(qmax));
    if (lane == 0) red_m[warp] = wmax;
    named_sync(1, kDecThreads);
    const uint32_t mx = max(max(red_m[0], red_m[1]), max(red_m[2], red_m[3]));
    eq = max(-60, min(60, exp2_ceil(__uint_as_float(mx))));
    const float qscale = exp2i(29 - eq);
    po = pos_desc(L, e);
    const float qs1 = po >= 0 ? qscale * exp2i(-pos_lg(po)) : 0.f;
#pragma unroll
    for (int j = 0; j < kGQ; ++j) qq[j] = e >= 0 ? q_s[j * kD + (e & 0xFFFF)] * qs1 : 0.f;
    // K positions 128.. (wide layouts, K <= 256).
    po_hi = pos_desc(L, e_hi);
    if (e_hi >= 0) {
      const float qsh = qscale * exp2i(-pos_lg(po_hi));
      qv_hi = make_float2(q_s[2 * hp * kD + (e_hi & 0xFFFF)] * qsh, q_s[(2 * hp + 1) * kD + (e_hi & 0xFFFF)] * qsh);
    }
    if (kDecThreads + 32 + tid < S.kpad) {
      const int po2 = pos_desc(L, e2);
      const float qs2 = po2 >= 0 ? qscale * exp2i(-pos_lg(po2)) : 0.f;
#pragma unroll
      for (int j = 0; j < kGQ; ++j) qhi_s[tid * kGQ + j] = e2 >= 0 ? q_s[j * kD + (e2 & 0xFFFF)] * qs2 : 0.f;
      posoff_s[tid] = po2;
    }
    // FP16-tier query values (times scaling * log2 e), slot-major.
    if (tid < n16) q16_s[tid] = ch16 < 0 ? 0.f : q_s[(tid % kGQ) * kD + ch16] * c2;
    for (int i = tid + kDecThreads; i < n16; i += kDecThreads) {
      const int ch = p.slot_chan[(3 * H + h) * kD + i / kGQ];
      q16_s[i] = ch < 0 ? 0.f : q_s[(i % kGQ) * kD + ch] * c2;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Broadcast from lane 0: the compiler then knows the value is the same in
  // every lane and keeps it (and the TMEM addresses built from it) in uniform
  // registers, which tcgen05 operands are read from.
  const uint32_t tmem = __shfl_sync(0xffffffffu, *tmem_slot, 0);
  const uint64_t kLimit = kWaitLimitNs;

  if (warp == 4) {
    // ------------------------------------------------------------ control warp
    int issued0 = 1, issued1 = 0, qk_open = 0, pv_open = 0;
    const uint32_t n_ks = static_cast<uint32_t>(S.kpad / 32);
    const uint64_t bqk_desc0 = smem_desc(bqk, 128, S.bqk_sbo);
    const uint64_t apv_desc0 = smem_desc(apv, 128, 2048);
    const uint64_t bpv_desc0 = smem_desc(bpv, 128, 2048);
    if (npg > 1) {  // every lane keeps the issue counts; lane 0 drains on abort
      if (lane == 0) issue_page(1);
      issued1 = 1;
    }
    auto cwait = [&](uint64_t* bar, uint32_t parity) {
      if (mbar_try_wait(bar, parity)) return;
      if (*abort_s) return;
      if (!mbar_wait_bounded(bar, parity, kLimit)) *abort_s = 1;
    };
    for (int i = 0; i < npg; ++i) {
      cwait(&bars[kBarKReady], i & 1);
      __syncwarp();
      tc_fence_after();
      if (elect_one()) {
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)  // +512 B per K step = +32 in descriptor units
          if (ks < static_cast<int>(n_ks))
            mma_u8_ts(tmem + S.tm_qk, tmem + 8 * ks, bqk_desc0 + 32 * ks, kIdescQK, ks > 0 ? 1u : 0u);
        mma_commit(&bars[kBarQK]);
      }
      __syncwarp();
      qk_open = i + 1;
      // Stage i % 2 has been read by U_K(i), U_V(i) and the FP16 tier of S(i):
      // it takes page i + 2.
      if (i + kStages < npg && !*abort_s) {
        const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(&bars[kBarFree], i & 1, kLimit));
        if (!ok) {
          *abort_s = 1;
        } else {
          if (elect_one()) issue_page(i + kStages);
          if (i & 1) ++issued1; else ++issued0;
        }
      }
      cwait(&bars[kBarVReady], i & 1);
      __syncwarp();
      tc_fence_after();
      if (elect_one()) {
#pragma unroll
        for (int ks = 0; ks < kP / 32; ++ks)
          mma_u8_ss(tmem + S.tm_pv, apv_desc0 + 32 * ks, bpv_desc0 + 32 * ks, kIdescPV, ks > 0 ? 1u : 0u);
        mma_commit(&bars[kBarPV]);
      }
      __syncwarp();
      pv_open = i + 1;
    }
    if (lane == 0 && *abort_s) {
      // Drain this CTA's copies and MMAs before its shared memory and TMEM go away.
      if (issued0) mbar_wait_bounded(&bars[kBarFull], (issued0 - 1) & 1, kLimit);
      if (issued1) mbar_wait_bounded(&bars[kBarFull + 1], (issued1 - 1) & 1, kLimit);
      if (qk_open) mbar_wait_bounded(&bars[kBarQK], (qk_open - 1) & 1, kLimit);
      if (pv_open) mbar_wait_bounded(&bars[kBarPV], (pv_open - 1) & 1, kLimit);
      if (p.status != nullptr) atomicExch(p.status, LF_ERR_DEVICE_TIMEOUT);
    }
    __syncwarp();
  } else {
    // ----------------------------------------------------------- compute warps
    const uint32_t tm_a = tmem + (static_cast<uint32_t>(__shfl_sync(0xffffffffu, warp, 0) * 32) << 16);
    for (int c = n_slots_of(L) / 4; c < S.a_cols; ++c) tmem_st_x1(tm_a + c, 0u);  // A padding columns
    float og[GQ], lt[GQ], lvt[GQ];
#pragma unroll
    for (int j = 0; j < GQ; ++j) og[j] = lt[j] = lvt[j] = 0.f;
    float m_l = -INFINITY;  // running max of q-head (lane & 7), log2 units
    const int l8 = lane & 7;
    // A wait whose phase has completed costs one try_wait; the abort flag is
    // read only on the slow path.
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      if (mbar_try_wait(bar, parity)) return;
      if (*abort_s) return;
      if (!mbar_wait_bounded(bar, parity, kLimit)) *abort_s = 1;
    };
    const int wd0 = L.words[0], wd1 = L.words[1], wd2 = L.words[2], w3 = L.width[3];
    const int co0 = L.code_off[0], co1 = L.code_off[1], co2 = L.code_off[2], vco = L.vcode_off;
    const int row_off = tid * R;
    const int rk = (tid >> 2) & 3;               // PV row t carries code * 4^rk
    const bool has_pos = tid < S.kpad;           // warp-uniform (K padded to 32)
    const int soff = po >= 0 ? pos_scale(po) : 0, moff = po >= 0 ? pos_min(po) : 0;
    const float mmul = po >= 0 ? exp2i(pos_lg(po)) : 0.f;
    const float cf = c2 * exp2i(eq - 29);        // fixed-point unit 2^(Eq-29) -> log2-scaled score
    const int bslot = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);

    // U_K(i): Key codes of the thread's token -> its TMEM lane (A of QK); the
    // B row of K position tid; bias partials; the token's code sum (every bit
    // of a code word lands in exactly one masked byte of A, so the A row sums
    // to the byte sum of the words) into nsum.  Returns the page's Es.
    int nsum = 0;
    auto unpack_k = [&](int i) -> int {
      const unsigned char* stage = stage0 + (i & 1) * S.stage_bytes;
      const uint32_t* rowp = reinterpret_cast<const uint32_t*>(stage) + row_off;
      const uint16_t* meta = reinterpret_cast<const uint16_t*>(stage + S.rows_bytes);
      uint32_t col = tm_a;
      uint32_t ns = 0u;
      {
        // INT2: two words (8 columns) per store.
        const uint32_t* src = rowp + co0;
        int w = 0;
#pragma unroll 1
        for (; w + 2 <= wd0; w += 2) {
          const uint32_t x = src[w], y = src[w + 1];
          tmem_st_x8(col + 4 * w, x & kM2, x & (kM2 << 2), x & (kM2 << 4), x & (kM2 << 6), y & kM2, y & (kM2 << 2),
                     y & (kM2 << 4), y & (kM2 << 6));
          ns = __dp4a(y, 0x01010101u, __dp4a(x, 0x01010101u, ns));
        }
        if (w < wd0) {
          const uint32_t x = src[w];
          tmem_st_x4(col + 4 * w, x & kM2, x & (kM2 << 2), x & (kM2 << 4), x & (kM2 << 6));
          ns = __dp4a(x, 0x01010101u, ns);
        }
        col += 4 * wd0;
      }
      {
        // INT4: four words (8 columns) per store, then pairs, then one.
        const uint32_t* src = rowp + co1;
        int w = 0;
#pragma unroll 1
        for (; w + 4 <= wd1; w += 4) {
          const uint32_t x = src[w], y = src[w + 1], z = src[w + 2], u = src[w + 3];
          tmem_st_x8(col + 2 * w, x & kM4, x & (kM4 << 4), y & kM4, y & (kM4 << 4), z & kM4, z & (kM4 << 4), u & kM4,
                     u & (kM4 << 4));
          ns = __dp4a(u, 0x01010101u, __dp4a(z, 0x01010101u, __dp4a(y, 0x01010101u, __dp4a(x, 0x01010101u, ns))));
        }
#pragma unroll 1
        for (; w < wd1; ++w) {
          const uint32_t x = src[w];
          tmem_st_x2(col + 2 * w, x & kM4, x & (kM4 << 4));
          ns = __dp4a(x, 0x01010101u, ns);
        }
        col += 2 * wd1;
      }
      {
        // INT8: eight words per store, then one at a time.
        const uint32_t* src = rowp + co2;
        int w = 0;
#pragma unroll 1
        for (; w + 8 <= wd2; w += 8) {
          uint32_t x[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            x[k] = src[w + k];
            ns = __dp4a(x[k], 0x01010101u, ns);
          }
          tmem_st_x8(col + w, x[0], x[1], x[2], x[3], x[4], x[5], x[6], x[7]);
        }
#pragma unroll 1
        for (; w < wd2; ++w) {
          const uint32_t x = src[w];
          tmem_st_x1(col + w, x);
          ns = __dp4a(x, 0x01010101u, ns);
        }
      }
      nsum = static_cast<int>(ns);
      const int esc = page_scale_exp(meta, kmax_off);
      const float fsc = exp2i(-esc);
      float bias[kGQ];
#pragma unroll
      for (int j = 0; j < kGQ; ++j) bias[j] = 0.f;
      if (has_pos) {
        const float sc = po >= 0 ? half_bits_to_float(meta[soff]) * fsc : 0.f;
        const float mn = half_bits_to_float(meta[moff]) * mmul;
        qk_b_row<GQ>(bqk, S.bqk_sbo, tid, qq, sc, mn, bias);
        // K positions 128.. (wide layouts): four lanes per position, two
        // q-heads per lane (the query values are zero for the heads >= GQ).
        auto hi_row = [&](int pp, float2 qv, int o) {
          const float sc2 = o >= 0 ? half_bits_to_float(meta[pos_scale(o)]) * fsc : 0.f;
          const float mn2 = o >= 0 ? half_bits_to_float(meta[pos_min(o)]) * exp2i(pos_lg(o)) : 0.f;
          hi_b_row_pair(bqk, S.bqk_sbo, pp, hp, qv, sc2);
          const float2 b01 = __fmul2_rn(qv, f2(mn2, mn2));
          const float b0 = b01.x, b1 = b01.y;
#pragma unroll
          for (int j = 0; j < kGQ; ++j)
            if (j < GQ) bias[j] += (j >> 1) == hp ? ((j & 1) ? b1 : b0) : 0.f;
        };
        if (n_hi > 0) hi_row(kDecThreads + (tid >> 2), qv_hi, po_hi);
#pragma unroll 1
        for (int k = 1; k < n_hi; ++k) {
          const int r = (tid >> 2) + 32 * (k - 1);
          hi_row(kDecThreads + 32 + r, *reinterpret_cast<const float2*>(qhi_s + r * kGQ + 2 * hp), posoff_s[r]);
        }
      }
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars[kBarKReady]);
      // The bias partials are read only by S(i), after its named barrier: the
      // warp reduction runs after the arrive, off the path to the QK issue.
      const float part = warp_sum8_scatter(bias, lane);
      if ((lane & 3) == 0) red_b[(i & 1) * 32 + warp * kGQ + bslot] = part;
      return esc;
    };
    // U_V(i): Value codes of the thread's token -> row t of the Value tile.
    auto unpack_v = [&](int i) {
      const uint32_t* src = reinterpret_cast<const uint32_t*>(stage0 + (i & 1) * S.stage_bytes) + row_off + vco;
      uint32_t vw[kD / 16];
#pragma unroll
      for (int w = 0; w < kD / 16; ++w) vw[w] = src[w];
      unsigned char* dst = apv + (tid & 7) * 16 + (tid >> 3) * 128;
#pragma unroll
      for (int w = 0; w < kD / 16; ++w) {
        const uint32_t x = vw[w];
        *reinterpret_cast<uint4*>(dst + w * 2048) = make_uint4(x & kM2, x & (kM2 << 2), x & (kM2 << 4), x & (kM2 << 6));
      }
    };

    wait(&bars[kBarFull], 0);
    int esc = unpack_k(0);
    unpack_v(0);
    for (int i = 0; i < npg; ++i) {
      const int st = i & 1;
      // S(i).  The FP16 Key tier (CUDA cores) and the token's Value scale /
      // min come from the page's stage, resident until this page's V-ready.
      const uint16_t* row16 =
          reinterpret_cast<const uint16_t*>(stage0 + st * S.stage_bytes) + 2 * (row_off + L.half_off);
      float s16[GQ];
#pragma unroll
      for (int j = 0; j < GQ; ++j) s16[j] = 0.f;
#pragma unroll 2
      for (int c = 0; c < w3; ++c) {
        const float kv = half_bits_to_float(row16[c]);
        const float4 qa = *reinterpret_cast<const float4*>(q16_s + c * kGQ);
        const float4 qb = *reinterpret_cast<const float4*>(q16_s + c * kGQ + 4);
        const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        by_pairs<GQ>(
            [&](int j) {
              const float2 r = __ffma2_rn(f2(qv[j], qv[j + 1]), f2(kv, kv), f2(s16[j], s16[j + 1]));
              s16[j] = r.x;
              s16[j + 1] = r.y;
            },
            [&](int j) { s16[j] = fmaf(qv[j], kv, s16[j]); });
      }
      const float vs = half_bits_to_float(row16[w3]);
      const float vm = half_bits_to_float(row16[w3 + 1]);
      mbar_arrive(&bars[kBarFree]);  // the last read of this page's stage
      const float f = cf * exp2i(esc), f16 = f * 65536.f;
      const int off64 = 64 * nsum;  // offset 2^30 = 64 * 2^24 per unit of code
      wait(&bars[kBarQK], st);
      tc_fence_after();
      uint32_t a[32];
      tmem_ld_x32_sync(tm_a + S.tm_qk, a);
      float x[GQ], xh[GQ];
      float key[GQ];
#pragma unroll
      for (int j = 0; j < GQ; ++j) {
        // acc_l = column 4 j + l; limbs 0-1 and 2-3 joined exactly in 32 bits.
        const uint32_t lo = a[4 * j] + (a[4 * j + 1] << 8);
        const int hi = static_cast<int>(a[4 * j + 2]) + ((static_cast<int>(a[4 * j + 3]) - off64) << 8);
        x[j] = static_cast<float>(lo);
        xh[j] = static_cast<float>(hi);
      }
      // score = hi * 2^16 f + (lo * f + FP16 tier part)
      by_pairs<GQ>(
          [&](int j) {
            const float2 r = __ffma2_rn(f2(xh[j], xh[j + 1]), f2(f16, f16),
                                        __ffma2_rn(f2(x[j], x[j + 1]), f2(f, f), f2(s16[j], s16[j + 1])));
            x[j] = r.x;
            x[j + 1] = r.y;
          },
          [&](int j) { x[j] = fmaf(xh[j], f16, fmaf(x[j], f, s16[j])); });
#pragma unroll
      for (int j = 0; j < GQ; ++j) key[j] = warp_max_f32(x[j]);
      const uint32_t vkey = __reduce_max_sync(0xffffffffu, __float_as_uint(vs));
      uint32_t* rm = red_m + st * 48;
      if (lane == 0) {
#pragma unroll
        for (int j = 0; j < kGQ; ++j) rm[warp * 12 + j] = j < GQ ? __float_as_uint(key[j]) : 0u;
        rm[warp * 12 + 8] = vkey;
      }
      named_sync(1, kDecThreads);
      // Lane j (mod 8): statistics of q-head j.  The bias is the same for
      // every token of the page, so the page max is max(score) + bias.
      const float* rb = red_b + st * 32 + l8;
      const float bias = ((rb[0] + rb[8]) + (rb[16] + rb[24])) * cf;
      const float km = fmaxf(fmaxf(__uint_as_float(rm[l8]), __uint_as_float(rm[12 + l8])),
                             fmaxf(__uint_as_float(rm[24 + l8]), __uint_as_float(rm[36 + l8])));
      const uint32_t vk = max(max(rm[8], rm[20]), max(rm[32], rm[44]));
      const float mnew = fmaxf(m_l, km + bias);
      const float alpha = m_l == -INFINITY ? 0.f : ex2(m_l - mnew);
      m_l = mnew;
      const float off = bias - mnew;
      const int ev = max(-60, min(60, exp2_ceil(__uint_as_float(vk))));
      const float vsc = vs * exp2i(23 - ev);
      uint32_t U[kGQ];
#pragma unroll
      for (int j = 0; j < GQ; ++j) x[j] = ex2(x[j] + __shfl_sync(0xffffffffu, off, j));  // p_tj
      // Y = rint(p * vs * 2^(23 - Ev)) in [0, 2^23]: the low 24 bits of the
      // fp32 sum 2^23 + Y are Y (2^24 itself has low bits 2^23).
      by_pairs<GQ>(
          [&](int j) {
            const float2 r = __ffma2_rn(f2(x[j], x[j + 1]), f2(vsc, vsc), f2(8388608.0f, 8388608.0f));
            U[j] = __float_as_uint(r.x) & 0x00FFFFFFu;
            U[j + 1] = __float_as_uint(r.y) & 0x00FFFFFFu;
          },
          [&](int j) { U[j] = __float_as_uint(fmaf(x[j], vsc, 8388608.0f)) & 0x00FFFFFFu; });
#pragma unroll
      for (int j = GQ; j < kGQ; ++j) U[j] = 0u;
      store_b_row(bpv + (tid & 7) * 16 + (tid >> 3) * 128, 2048, U);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars[kBarVReady]);
      // The running sums are not read by PV: rescaled and extended after the arrive.
      if (__any_sync(0xffffffffu, l8 < GQ && alpha != 1.f)) {
        float al[GQ];
#pragma unroll
        for (int j = 0; j < GQ; ++j) al[j] = __shfl_sync(0xffffffffu, alpha, j);
        by_pairs<GQ>(
            [&](int j) {
              const float2 aj = f2(al[j], al[j + 1]);
              const float2 o2 = __fmul2_rn(f2(og[j], og[j + 1]), aj);
              const float2 t2 = __fmul2_rn(f2(lt[j], lt[j + 1]), aj);
              const float2 v2 = __fmul2_rn(f2(lvt[j], lvt[j + 1]), aj);
              og[j] = o2.x;
              og[j + 1] = o2.y;
              lt[j] = t2.x;
              lt[j + 1] = t2.y;
              lvt[j] = v2.x;
              lvt[j + 1] = v2.y;
            },
            [&](int j) {
              og[j] *= al[j];
              lt[j] *= al[j];
              lvt[j] *= al[j];
            });
      }
      by_pairs<GQ>(
          [&](int j) {
            const float2 p2 = f2(x[j], x[j + 1]);
            const float2 t2 = __fadd2_rn(f2(lt[j], lt[j + 1]), p2);
            const float2 v2 = __ffma2_rn(p2, f2(vm, vm), f2(lvt[j], lvt[j + 1]));
            lt[j] = t2.x;
            lt[j + 1] = t2.y;
            lvt[j] = v2.x;
            lvt[j + 1] = v2.y;
          },
          [&](int j) {
            lt[j] += x[j];
            lvt[j] = fmaf(x[j], vm, lvt[j]);
          });
      // U_K(i+1) while PV(i) runs.
      if (i + 1 < npg) {
        wait(&bars[kBarFull + (st ^ 1)], ((i + 1) >> 1) & 1);
        esc = unpack_k(i + 1);
      }
      // C(i): accumulate PV row t.
      wait(&bars[kBarPV], st);
      tc_fence_after();
      tmem_ld_x32_sync(tm_a + S.tm_pv, a);
      const float sc = exp2i(ev - 23 - 2 * rk);
      {
        float vl[GQ], vh[GQ];
#pragma unroll
        for (int j = 0; j < GQ; ++j) {
          vl[j] = static_cast<float>(a[4 * j] + (a[4 * j + 1] << 8));
          vh[j] = static_cast<float>(a[4 * j + 2]);
        }
        // og += (limb2 * 2^16 + limbs 0-1) * scale
        by_pairs<GQ>(
            [&](int j) {
              const float2 v2 = __ffma2_rn(f2(vh[j], vh[j + 1]), f2(65536.f, 65536.f), f2(vl[j], vl[j + 1]));
              const float2 o2 = __ffma2_rn(v2, f2(sc, sc), f2(og[j], og[j + 1]));
              og[j] = o2.x;
              og[j + 1] = o2.y;
            },
            [&](int j) { og[j] = fmaf(fmaf(vh[j], 65536.f, vl[j]), sc, og[j]); });
      }
      // U_V(i+1): the Value tile is free once PV(i) has completed.
      if (i + 1 < npg) unpack_v(i + 1);
    }

    float mg[GQ];
#pragma unroll
    for (int j = 0; j < GQ; ++j) mg[j] = __shfl_sync(0xffffffffu, m_l, j) * kLn2;  // natural-log units
    // PV row t holds head-dim channel d(t): t = 16w + 4k + i  <->  d = 16w + k + 4i.
    const int d = (tid & ~15) + ((tid & 15) >> 2) + 4 * (tid & 3);
    // (sequence, KV head, chunk) re-read from the block index: nothing of it
    // stays live through the page loop.
    const int64_t item = (static_cast<int64_t>(blockIdx.x) * p.n_chunks + blockIdx.z) * p.max_splits + s;
    write_partial_group<GQ>(p, item, d, og, mg, lt, lvt, red_w, 1);
  }
  tc_fence_before();
  __syncthreads();  // compute warps finished (their partial is written); copies and MMAs drained
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, S.tm_cols);
  }
}

}  // namespace tc

bool tc_supported(const lf_layout& L, int gq, int pps) {
  if (L.head_dim != tc::kD || L.page_size != tc::kP || L.k_group != tc::kP || L.v_group != tc::kD) return false;
  if (L.bit_v != 2 || gq > kGQ || gq < 1) return false;
  if (tc::n_slots_of(L) > 2 * kDecThreads) return false;  // two K positions per compute thread
  if (pps > tc::kMaxPagesPerItem) return false;
  const tc::TcSmem S = tc::tc_smem(L);
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

// Dynamic shared-memory limit of the GQ-head kernel raised to at least
// smem_bytes, with the full shared-memory carveout so several CTAs fit on
// one SM (the occupancy computation assumes both).
static cudaError_t configure_tc(int gq, int smem_bytes) {
  return raise_smem_limit(tc_kernel_for(gq), smem_bytes, true);
}

// Resident CTAs per SM from the kernel's own limits: registers, shared memory
// (with the per-block reservation), threads and TMEM columns.  The runtime's
// occupancy query answers 1 for this kernel while the hardware runs four of
// its CTAs on one SM (observed with per-CTA SM ids and timestamps), so it is
// not used.
int occupancy_tc(const lf_layout& L, int gq, int pps) {
  (void)pps;  // the stage holds one page's meta row: shared memory does not depend on pps
  const tc::TcSmem S = tc::tc_smem(L);
  if (S.total > 227 * 1024) return 0;
  void* kern = tc_kernel_for(gq);
  cudaFuncAttributes fa;
  int dev = 0, smem_sm = 0, reserved = 0, regs_sm = 0, threads_sm = 0;
  if (configure_tc(gq, S.total) != cudaSuccess || cudaFuncGetAttributes(&fa, kern) != cudaSuccess ||
      cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&threads_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  const int warps = tc::kThreads / 32;
  const int regs_warp = (fa.numRegs * 32 + 255) / 256 * 256;  // allocated per warp in units of 256
  int blocks = regs_sm / (warps * regs_warp);
  blocks = std::min(blocks, smem_sm / (S.total + reserved));
  blocks = std::min(blocks, threads_sm / tc::kThreads);
  blocks = std::min(blocks, 512 / S.tm_cols);
  return std::max(blocks, 0);
}

int launch_partial_tc(const DecodeParams& p, int resid_dtype, int q_dtype, cudaStream_t stream) {
  DecodeParams q = p;
  q.resid_dtype = resid_dtype;
  q.q_dtype = q_dtype;
  const tc::TcSmem S = tc::tc_smem(q.L);
  void* kern = tc_kernel_for(q.cg);
  {
    cudaError_t e = configure_tc(q.cg, S.total);
    if (e != cudaSuccess) {
      set_error("lf_decode_partial (tcgen05): shared memory %d B: %s", S.total, cudaGetErrorString(e));
      return LF_ERR_UNSUPPORTED;
    }
  }
  dim3 grid(q.L.kv_heads * q.batch, q.max_splits, q.n_chunks);
  void* args[] = {&q};
  cudaError_t e = launch_programmatic(kern, grid, dim3(tc::kThreads), S.total, stream, args);
  if (e != cudaSuccess) {
    set_error("lf_decode_partial (tcgen05): %s", cudaGetErrorString(e));
    return LF_ERR_LAUNCH;
  }
  return launch_status("lf_decode_partial (tcgen05)");
}

}  // namespace lf
