// Shared device helpers of the logitfill_b200 kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "logitfill_b200.h"

namespace lf {

// Per-thread error text for lf_last_error().
void set_error(const char* fmt, ...);
int launch_status(const char* what);
// Raise kern's dynamic shared-memory limit on the current device to at least
// `bytes` (optionally with the full shared-memory carveout).  The limit only
// grows: launches and occupancy queries for different layouts share one
// kernel, and lowering it for a small layout would fail a larger one later.
cudaError_t raise_smem_limit(const void* kern, int bytes, bool max_carveout);

template <typename T> struct Scalar;
template <> struct Scalar<float> {
  static __device__ __forceinline__ float load(const float* p) { return *p; }
  static __device__ __forceinline__ void store(float* p, float v) { *p = v; }
};
template <> struct Scalar<__half> {
  static __device__ __forceinline__ float load(const __half* p) { return __half2float(*p); }
  static __device__ __forceinline__ void store(__half* p, float v) { *p = __float2half_rn(v); }
};
template <> struct Scalar<__nv_bfloat16> {
  static __device__ __forceinline__ float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
};

__device__ __forceinline__ float half_bits_to_float(uint16_t bits) {
  return __half2float(__ushort_as_half(bits));
}
__device__ __forceinline__ uint16_t float_to_half_bits(float v) {
  return __half_as_ushort(__float2half_rn(v));
}

// Reference asymmetric min-max step (layout.py:12-18), bit-exact with torch
// CPU fp32: IEEE subtract and divide, clamp to [1e-5, 1e5].
__device__ __forceinline__ float asym_scale(float hi, float lo, int bits) {
  const float qmax = static_cast<float>((1 << bits) - 1);
  float s = __fdiv_rn(__fsub_rn(hi, lo), qmax);
  s = fmaxf(s, 1e-5f);
  s = fminf(s, 1e5f);
  return s;
}
// Code of x: clamp(round_half_even((x - lo) / scale), 0, 2^bits - 1)
// (layout.py:12-18), with the division done by Markstein's method (P. Markstein,
// "Computation of elementary functions on the IBM RISC System/6000
// processor", IBM J. Res. Develop. 34(1), 1990): with rcp = RN(1/scale) and
// q0 = RN(d * rcp) within one ulp of d / scale, the residual d - q0 * scale is
// exact in an FMA and RN(q0 + residual * rcp) is the correctly rounded
// quotient, i.e. the same value as the IEEE division, for the normal-range
// operands here (scale in [1e-5, 1e5]; a quotient too small to be normal
// rounds to code 0 either way).  Three floating-point operations instead of a
// division per element; tests/test_pack_gpu.py checks it against the IEEE
// division bit for bit.
__device__ __forceinline__ float asym_quotient_rcp(float d, float scale, float rcp) {
  const float q0 = __fmul_rn(d, rcp);
  const float r = __fmaf_rn(-q0, scale, d);
  return __fmaf_rn(r, rcp, q0);
}
__device__ __forceinline__ uint32_t asym_code_rcp(float x, float lo, float scale, float rcp, int bits) {
  float c = rintf(asym_quotient_rcp(__fsub_rn(x, lo), scale, rcp));  // round half to even
  const float qmax = static_cast<float>((1 << bits) - 1);
  // Upper clamp first: an infinite x - lo leaves the Markstein residual NaN,
  // and fminf(NaN, qmax) = qmax is the code the IEEE quotient +inf gets.
  c = fminf(c, qmax);
  c = fmaxf(c, 0.0f);
  return static_cast<uint32_t>(c);
}

// Code of x as asym_code_rcp computes it (K1 uses this form), for x - lo >= 0 or
// NaN, which the packer always has (lo is the group's minimum, so x - lo is a
// non-negative number, +inf, or NaN).  For 0 <= q < 2^22 the float sum
// RN(q + 1.5 * 2^23) holds round_half_even(q) in the low bits of its
// significand; a larger, infinite or NaN quotient gives a bit pattern above
// every code, which the unsigned min turns into qmax: the reference's clamp.
__device__ __forceinline__ uint32_t pack_code(float x, float lo, float scale, float rcp, uint32_t qmax) {
  const float q = asym_quotient_rcp(__fsub_rn(x, lo), scale, rcp);
  const uint32_t r = __float_as_uint(__fadd_rn(q, 12582912.0f)) - 0x4B400000u;
  return min(r, qmax);
}

constexpr uint32_t kMagicBits = 0x4B400000u;  // bit pattern of 1.5 * 2^23

// Two codes, each as pack_code forms it, with packed fp32x2 arithmetic
// (sm_100a): every lane of {sub, mul, fma, add}.rn.f32x2 rounds as the scalar
// instruction does.  Takes nscale = -scale: the residual fma(q0, -scale, d)
// equals fma(-q0, scale, d).  Returns each lane's magic-number sum bit pattern
// clamped to kMagicBits + qmax, i.e. code + kMagicBits; a caller that adds
// several shifted codes takes the shifted kMagicBits off once.
__device__ __forceinline__ uint2 pack_bits2(float2 x, float2 lo, float2 nscale, float2 rcp, uint32_t qmax) {
  uint32_t a, b;
  asm("{\n\t.reg .b64 X, L, N, C, M, D, Q, R;\n\t"
      "mov.b64 X, {%2, %3};\n\t"
      "mov.b64 L, {%4, %5};\n\t"
      "mov.b64 N, {%6, %7};\n\t"
      "mov.b64 C, {%8, %9};\n\t"
      "mov.b64 M, {%10, %10};\n\t"
      "sub.rn.f32x2 D, X, L;\n\t"
      "mul.rn.f32x2 Q, D, C;\n\t"
      "fma.rn.f32x2 R, Q, N, D;\n\t"
      "fma.rn.f32x2 Q, R, C, Q;\n\t"
      "add.rn.f32x2 Q, Q, M;\n\t"
      "mov.b64 {%0, %1}, Q;\n\t}"
      : "=r"(a), "=r"(b)
      : "r"(__float_as_uint(x.x)), "r"(__float_as_uint(x.y)), "r"(__float_as_uint(lo.x)),
        "r"(__float_as_uint(lo.y)), "r"(__float_as_uint(nscale.x)), "r"(__float_as_uint(nscale.y)),
        "r"(__float_as_uint(rcp.x)), "r"(__float_as_uint(rcp.y)), "r"(kMagicBits));
  return make_uint2(min(a, kMagicBits + qmax), min(b, kMagicBits + qmax));
}
__device__ __forceinline__ uint2 pack_code2(float2 x, float2 lo, float2 nscale, float2 rcp, uint32_t qmax) {
  const uint2 r = pack_bits2(x, lo, nscale, rcp, qmax);
  return make_uint2(r.x - kMagicBits, r.y - kMagicBits);
}

// (x, y) = (fma(w, v.x, x), fma(w, v.y, y)) as one packed fp32x2 FMA; each
// lane rounds as fmaf does, so the sums equal the scalar ones bit for bit.
__device__ __forceinline__ void fma2_acc(float w, float2 v, float& x, float& y) {
  const float2 r = __ffma2_rn(make_float2(w, w), v, make_float2(x, y));
  x = r.x;
  y = r.y;
}

template <typename F>
__device__ __forceinline__ void dispatch_noop(F) {}

// Programmatic dependent launch.  K2 and K3 are launched with programmatic
// stream serialization, so a grid may begin launching while the kernel before
// it in the stream drains.  grid_dep_wait() returns once that kernel has
// completed and its memory operations are visible (at once for a grid launched
// without the attribute); every kernel here calls it before its first global
// access.  grid_dep_trigger() lets the next programmatic launch begin: it runs
// only after every CTA of this grid has started (or triggered), so the CTAs of
// the dependent grid never hold an SM a CTA of this grid still needs.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// cudaLaunchKernelExC with programmatic stream serialization.
cudaError_t launch_programmatic(const void* kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                void** args);

}  // namespace lf

#define LF_CHECK_ARG(cond, ...)                 \
  do {                                          \
    if (!(cond)) {                              \
      lf::set_error(__VA_ARGS__);               \
      return LF_ERR_INVALID_ARGUMENT;           \
    }                                           \
  } while (0)

#define LF_CHECK_SUPPORTED(cond, ...)           \
  do {                                          \
    if (!(cond)) {                              \
      lf::set_error(__VA_ARGS__);               \
      return LF_ERR_UNSUPPORTED;                \
    }                                           \
  } while (0)
