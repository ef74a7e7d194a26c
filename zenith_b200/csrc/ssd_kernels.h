// Internal launch interface between the C ABI (capi.cu) and the kernel files.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "common.cuh"

namespace zb {

constexpr size_t kSimtMaxSmem = 220 * 1024;

struct SimtParams {
  int64_t B, T, H, G, P, N;
  int L, nc;  // internal chunk length and count (ceil(T / L))
  int flags;
  View x, q, k, kp, xp, adt, gamma, beta;
  View y;
  const void* init;
  void* fin;
  void* chain;  // [B*H][nc+1][P][N] in the accumulator type: slot j = state entering chunk j
  ChainSync sync;
  int32_t* status;
  View dy;
  const void* dfin;
  View dx, dq, dk, dkp, dxp, dadt, dgamma, dbeta;
  void* dinit;
  void* gchain;  // [B*H][nc+1][P][N]: slot j = gradient w.r.t. the state entering chunk j
  void* grp;     // [B,T,H,3,N] per-head q/k/kp gradients (accumulator type) when G < H
};

// Largest internal chunk (<= 32) whose forward and backward tiles fit in shared memory; 0 if none.
int simt_pick_chunk(int P, int N, bool f64);
int simt_launch(const SimtParams& p, int dtype, int sdtype, bool backward, cudaStream_t stream);

// Count kernel launches for zb_launch_count().
void note_launches(int n);
// Raise a kernel's dynamic shared-memory limit to `bytes` (once per kernel, device and size).
int dyn_smem(const void* fn, int bytes);

}  // namespace zb
