// zb_wait_probe: runs one of the library's two bounded device-side waits on its own, so that a test
// can make it run out and check what the host sees.
//
// Every kernel here that waits for another CTA (the chained hand-off flag) or for its own bulk
// copies (an mbarrier phase) gives up after about one second: it records ZB_ERR_TIMEOUT in the
// device status word and returns instead of spinning on.  This entry point launches one thread
// that calls the same wait functions the scan and layer kernels call, on a flag or an mbarrier
// that the caller arranges never to complete, and reports what the wait returned and how long it
// took.  Nothing faults: the wait is expected to end, and the context stays usable.
#include "ssd_kernels.h"
#include "umma.cuh"

namespace zb {
namespace {

// which = 0: wait_flag on `flag` (result[0]: kFlagReady 1 or kFlagAbort 2)
// which = 1: mbar_wait on a fresh shared-memory mbarrier that expects one arrival and gets none
//            (result[0]: 1 completed, 0 gave up)
// result[1]: microseconds spent in the wait (globaltimer)
__global__ void wait_probe_kernel(const int* flag, int32_t* status, int32_t* result, int which) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  if (which == 1) {
    umma::mbar_init(&bar, 1);
    umma::mbar_fence_init();
  }
  const uint64_t t0 = globaltimer();
  result[0] = which == 0 ? wait_flag(flag, status) : (umma::mbar_wait(&bar, 0, status) ? 1 : 0);
  result[1] = (int32_t)((globaltimer() - t0) / 1000);
}

}  // namespace
}  // namespace zb

extern "C" ZB_API int zb_wait_probe(const int* flag, int32_t* status, int32_t* result, int which, void* stream) {
  if (!status || !result || (which == 0 && !flag)) return ZB_ERR_LAYOUT;
  if (which != 0 && which != 1) return ZB_ERR_UNSUPPORTED;
  zb::wait_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flag, status, result, which);
  zb::note_launches(1);
  return cudaGetLastError() == cudaSuccess ? ZB_OK : ZB_ERR_CUDA;
}
