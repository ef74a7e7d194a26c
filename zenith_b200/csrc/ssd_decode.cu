// Recurrent (decode) form of the SSD scan: for each token in order,
//     h = e^{adt} h + gamma x k^T + beta xp kp^T ,   y = h q
// the per-token recurrence of the reference's test (tests/test_mamba3.py:10-21), started from a
// carried state (e.g. the final state of a chunked forward over the prompt) and advanced in
// place.  Memory-bound on the state: one CTA per (batch, head) keeps its [P, N] state in
// registers for all the call's tokens, reading and writing it once.
//
// 256 threads: warp w owns state rows p = w, w+8, ...; lane l owns columns 4l..4l+3.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "ssd_kernels.h"

namespace zb {
namespace {

constexpr int kDecThreads = 256;
constexpr int kDecMaxRows = 16;  // P <= 128 rows over 8 warps

template <typename TV>
__device__ __forceinline__ float4 ld4f(const TV* p, int n0, int N) {
  float4 v;
  v.x = n0 < N ? ldv<float>(p + n0) : 0.f;
  v.y = n0 + 1 < N ? ldv<float>(p + n0 + 1) : 0.f;
  v.z = n0 + 2 < N ? ldv<float>(p + n0 + 2) : 0.f;
  v.w = n0 + 3 < N ? ldv<float>(p + n0 + 3) : 0.f;
  return v;
}

struct DecParams {
  int64_t B, T, H, G, P, N;
  View x, q, k, kp, xp, adt, gamma, beta, y;
  const float* init;  // [B, H, P, N] or nullptr (zero state)
  float* fin;         // [B, H, P, N] (may equal init)
};

template <typename TV, typename TS>
__global__ void __launch_bounds__(kDecThreads) ssd_decode_kernel(const DecParams p) {
  const int bh = blockIdx.x;
  const int b = bh / (int)p.H, h = bh % (int)p.H;
  const int g = h / (int)(p.H / p.G);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = (int)p.P, N = (int)p.N, n0 = 4 * lane;
  const int64_t PN = (int64_t)P * N;
  float4 s[kDecMaxRows];
  const int rows = (P - warp + 7) / 8;  // rows p = warp + 8 r, r < rows
#pragma unroll
  for (int r = 0; r < kDecMaxRows; ++r) {
    s[r] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < rows && p.init && n0 < N) {
      const float* src = p.init + bh * PN + (int64_t)(warp + 8 * r) * N + n0;
      s[r] = ld4f(src, 0, N - n0);
    }
  }
  for (int64_t t = 0; t < p.T; ++t) {
    const float a = xexp<float>(ldv<float>(p.adt.row<TS>(b, t, h)));
    const float gm = ldv<float>(p.gamma.row<TS>(b, t, h)), bt = ldv<float>(p.beta.row<TS>(b, t, h));
    const float4 qv = ld4f(p.q.row<TV>(b, t, g), n0, N);
    const float4 kv = ld4f(p.k.row<TV>(b, t, g), n0, N);
    const float4 kpv = ld4f(p.kp.row<TV>(b, t, g), n0, N);
    const TV* xr = p.x.row<TV>(b, t, h);
    const TV* xpr = p.xp.row<TV>(b, t, h);
    TV* yr = p.y.wrow<TV>(b, t, h);
#pragma unroll
    for (int r = 0; r < kDecMaxRows; ++r) {
      if (r >= rows) break;
      const int pp = warp + 8 * r;
      const float gx = gm * ldv<float>(xr + pp), bx = bt * ldv<float>(xpr + pp);
      s[r].x = a * s[r].x + gx * kv.x + bx * kpv.x;
      s[r].y = a * s[r].y + gx * kv.y + bx * kpv.y;
      s[r].z = a * s[r].z + gx * kv.z + bx * kpv.z;
      s[r].w = a * s[r].w + gx * kv.w + bx * kpv.w;
      const float yv = warp_sum(s[r].x * qv.x + s[r].y * qv.y + s[r].z * qv.z + s[r].w * qv.w);
      if (lane == 0) stv<float>(yr + pp, yv);
    }
  }
#pragma unroll
  for (int r = 0; r < kDecMaxRows; ++r) {
    if (r < rows && n0 < N) {
      float* dst = p.fin + bh * PN + (int64_t)(warp + 8 * r) * N + n0;
      dst[0] = s[r].x;
      if (n0 + 1 < N) dst[1] = s[r].y;
      if (n0 + 2 < N) dst[2] = s[r].z;
      if (n0 + 3 < N) dst[3] = s[r].w;
    }
  }
}

View as_view(const zb_view& v) { return View{v.ptr, v.sb, v.st, v.sh}; }

}  // namespace
}  // namespace zb

using namespace zb;

extern "C" ZB_API int zb_ssd_decode(const zb_ssd_args* a, void* stream) {
  if (!a) return ZB_ERR_LAYOUT;
  if (a->B <= 0 || a->T <= 0 || a->H <= 0 || a->G <= 0 || a->P <= 0 || a->N <= 0 || a->H % a->G != 0)
    return ZB_ERR_SHAPE;
  if (a->P > 8 * kDecMaxRows || a->N > 128) return ZB_ERR_UNSUPPORTED;
  if (a->scalar_dtype != ZB_F32 || a->dtype == ZB_F64) return ZB_ERR_DTYPE;
  if (!a->x.ptr || !a->q.ptr || !a->k.ptr || !a->kp.ptr || !a->xp.ptr || !a->adt.ptr || !a->gamma.ptr ||
      !a->beta.ptr || !a->y.ptr || !a->final_state)
    return ZB_ERR_LAYOUT;
  DecParams p;
  p.B = a->B; p.T = a->T; p.H = a->H; p.G = a->G; p.P = a->P; p.N = a->N;
  p.x = as_view(a->x); p.q = as_view(a->q); p.k = as_view(a->k); p.kp = as_view(a->kp); p.xp = as_view(a->xp);
  p.adt = as_view(a->adt); p.gamma = as_view(a->gamma); p.beta = as_view(a->beta); p.y = as_view(a->y);
  p.init = static_cast<const float*>(a->initial_state);
  p.fin = static_cast<float*>(a->final_state);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)(a->B * a->H));
  switch (a->dtype) {
    case ZB_F32: ssd_decode_kernel<float, float><<<grid, kDecThreads, 0, s>>>(p); break;
    case ZB_BF16: ssd_decode_kernel<__nv_bfloat16, float><<<grid, kDecThreads, 0, s>>>(p); break;
    case ZB_F16: ssd_decode_kernel<__half, float><<<grid, kDecThreads, 0, s>>>(p); break;
    default: return ZB_ERR_DTYPE;
  }
  note_launches(1);
  return cudaPeekAtLastError() == cudaSuccess ? ZB_OK : ZB_ERR_CUDA;
}
