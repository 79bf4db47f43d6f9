// Self-test of the bounded device-side wait that every tensor-core decode
// kernel uses on its mbarriers.  One thread initialises an mbarrier with one
// expected arrival, arrives on it or not, and waits for the phase with the
// given limit.  Without the arrival the wait runs out, the kernel records
// LF_ERR_DEVICE_TIMEOUT in the status word and returns: the failure path is
// exercised with no fault, trap or hang, and the context stays usable.
#include "lf_common.cuh"
#include "lf_tcgen05.cuh"

namespace lf {

__global__ void selftest_wait_kernel(int32_t* status, uint64_t limit_ns, int arrive) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  sm100::mbar_init(&bar, 1);
  sm100::fence_mbar_init();
  if (arrive) sm100::mbar_arrive(&bar);
  const bool done = sm100::mbar_wait_bounded(&bar, 0, limit_ns);
  *status = done ? LF_OK : LF_ERR_DEVICE_TIMEOUT;
}

}  // namespace lf

extern "C" int lf_selftest_wait(int32_t* status, int64_t limit_ns, int arrive, lf_stream_t stream) {
  LF_CHECK_ARG(status != nullptr, "lf_selftest_wait: null status");
  LF_CHECK_ARG(limit_ns > 0 && limit_ns <= 10000000000LL, "lf_selftest_wait: limit %lld ns out of (0, 10 s]",
               static_cast<long long>(limit_ns));
  lf::selftest_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      status, static_cast<uint64_t>(limit_ns), arrive);
  return lf::launch_status("lf_selftest_wait");
}

// Self-test of K1's per-element division: for each (x, lo, scale) triple the
// quotient (x - lo) / scale and the code exactly as pack_pages_kernel forms
// them (IEEE subtract, Markstein division with rcp = RN(1 / scale), round
// half to even by the magic-number add, clamp to [0, 2^bits - 1]).  The code
// is formed both ways K1 forms codes, one element (pack_code) and a pair of
// elements in packed fp32x2 arithmetic (pack_code2, element i with its
// neighbour i ^ 1 in the other lane); an element whose two codes differ gets
// the code 0xFFFFFFFF, which no reference code equals.
namespace lf {

__global__ void selftest_divide_kernel(const float* __restrict__ x, const float* __restrict__ lo,
                                       const float* __restrict__ scale, int64_t n, int bits,
                                       float* __restrict__ quot, uint32_t* __restrict__ code) {
  const uint32_t qmax = (1u << bits) - 1u;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t j = (i ^ 1) < n ? (i ^ 1) : i;
    const float s = scale[i], rcp = __frcp_rn(s);
    const float sj = scale[j], rcpj = __frcp_rn(sj);
    quot[i] = asym_quotient_rcp(__fsub_rn(x[i], lo[i]), s, rcp);
    const uint32_t ci = pack_code(x[i], lo[i], s, rcp, qmax);
    const uint32_t cj = pack_code(x[j], lo[j], sj, rcpj, qmax);
    const uint2 c2 = pack_code2(make_float2(x[i], x[j]), make_float2(lo[i], lo[j]), make_float2(-s, -sj),
                                make_float2(rcp, rcpj), qmax);
    code[i] = (c2.x == ci && c2.y == cj) ? ci : 0xFFFFFFFFu;
  }
}

}  // namespace lf

extern "C" int lf_selftest_divide(const float* x, const float* lo, const float* scale, int64_t n, int bits,
                                  float* quotient, uint32_t* code, lf_stream_t stream) {
  LF_CHECK_ARG(x && lo && scale && quotient && code, "lf_selftest_divide: null pointer");
  LF_CHECK_ARG(n >= 0, "lf_selftest_divide: n %lld", static_cast<long long>(n));
  LF_CHECK_ARG(bits == 2 || bits == 4 || bits == 8, "lf_selftest_divide: bits %d", bits);
  if (n == 0) return LF_OK;
  const int64_t blocks64 = (n + 255) / 256;
  const int blocks = static_cast<int>(blocks64 < 148 * 32 ? blocks64 : 148 * 32);
  lf::selftest_divide_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(x, lo, scale, n, bits,
                                                                                         quotient, code);
  return lf::launch_status("lf_selftest_divide");
}
