// Launch interface of the tensor-core (tcgen05) path, see ssd_tc.cu.
#pragma once

#include "common.cuh"

namespace zb {

// True when the tcgen05 kernels handle these arguments (bf16 vectors, P and N they are built for).
bool tc_supported(const zb_ssd_args* a);
// True when the tensor-core backward exists for these arguments (else saved states use the SIMT layout).
bool tc_has_backward(const zb_ssd_args* a);
// Internal chunk length of the tensor-core path.
int tc_chunk();
size_t tc_states_bytes(const zb_ssd_args* a);
size_t tc_workspace_bytes(const zb_ssd_args* a, bool backward);
int tc_fwd(const zb_ssd_args* a, ChainSync sync, void* chain, void* ws, cudaStream_t stream);
int tc_bwd(const zb_ssd_args* a, ChainSync sync, void* ws, cudaStream_t stream);

}  // namespace zb
