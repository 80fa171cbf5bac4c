// pf_selftest.cu -- pf_selftest_bounded_wait: exercises the bounded mbarrier wait that every
// pipelined kernel of the library uses, without any fault: one thread waits on an mbarrier that
// nothing arrives on; the wait gives up after the given limit, sets bit 0 of the device status
// word and the kernel returns, so the context stays usable and the host reads the status.

#include "pf_common.cuh"
#include "pf_prof.h"
#include "pf_sm100.cuh"
#include "pf_tmap.h"

namespace pf {
namespace {
using namespace sm100;

__global__ void k_selftest_wait(unsigned int* status, unsigned long long limit_ns) {
  __shared__ __align__(8) unsigned long long bar;
  if (threadIdx.x != 0) return;
  const uint32_t b = smem_u32(&bar);
  mbar_init(b, 1);
  fence_barrier_init();
  mbar_wait(b, 0, status, limit_ns);  // nothing arrives: gives up after limit_ns
}

}  // namespace
}  // namespace pf

using namespace pf;

extern "C" PF_API int pf_selftest_bounded_wait(int64_t limit_ns, void* stream) {
  if (limit_ns < 1000000 || limit_ns > 10000000000ll)
    return fail(PF_EINVAL_ARG, "limit_ns %lld outside [1 ms, 10 s]", (long long)limit_ns);
  unsigned int* status;
  PF_TRY(device_status_ptr(&status));
  cudaStream_t st = (cudaStream_t)stream;
  {
    PF_LAUNCH_SCOPE(st, "k_selftest_wait");
    k_selftest_wait<<<1, 32, 0, st>>>(status, (unsigned long long)limit_ns);
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}
