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
