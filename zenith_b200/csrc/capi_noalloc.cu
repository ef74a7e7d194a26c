// zb_ssd_fwd_noalloc: the forward scan for callers that cannot allocate device memory.
//
// Some callers cannot hand the library a workspace: a serving runtime that reserved all
// device memory at start-up and gives out no scratch, or a foreign-language binding that can
// pass the tensors it was given but has no CUDA allocator.  This entry point takes its scratch
// (the chained-scan ticket, flags and state hand-off slots) from one fixed device array
// declared below, so a call allocates nothing.  Limits and sharing rules are in zb_ssd.h.
#include <mutex>

#include "ssd_kernels.h"

namespace {

// The scratch array.  In host code `g_noalloc_scratch` names a host-side stand-in, not device
// memory: never pass it to a kernel.  Its device address comes from cudaGetSymbolAddress,
// looked up once per device with that device current.
static __device__ __align__(256) unsigned char g_noalloc_scratch[ZB_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (first call per device: lookup).
int scratch_for_current_device(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return ZB_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return ZB_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return ZB_ERR_CUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return ZB_OK;
}

}  // namespace

extern "C" int zb_ssd_fwd_noalloc(const zb_ssd_args* args, void* stream) {
  if (!args) return ZB_ERR_LAYOUT;
  const size_t need = zb_ssd_workspace_bytes(args, 0);
  if (need == 0) return ZB_ERR_SHAPE;  // invalid sizes (same check as zb_ssd_workspace_bytes)
  if (need > (size_t)ZB_NOALLOC_SCRATCH_BYTES) return ZB_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != ZB_OK) return rc;
  zb_ssd_args a = *args;
  a.workspace = scratch;
  a.workspace_bytes = ZB_NOALLOC_SCRATCH_BYTES;
  // zb_ssd_fwd clears the ticket/flag region of the scratch before its kernel runs; every
  // state slot is written before it is read, so leftovers of an earlier call do no harm.
  return zb_ssd_fwd(&a, stream);
}
