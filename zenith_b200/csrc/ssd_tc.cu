// Tensor-core path (tcgen05) of the SSD chunked scan: not enabled yet.
#include "ssd_tc.h"

namespace zb {

bool tc_supported(const zb_ssd_args*) { return false; }
int tc_chunk() { return 64; }
size_t tc_states_bytes(const zb_ssd_args*) { return 0; }
size_t tc_workspace_bytes(const zb_ssd_args*, bool) { return 0; }
int tc_fwd(const zb_ssd_args*, ChainSync, void*, void*, cudaStream_t) { return ZB_ERR_UNSUPPORTED; }
int tc_bwd(const zb_ssd_args*, ChainSync, void*, cudaStream_t) { return ZB_ERR_UNSUPPORTED; }

}  // namespace zb
