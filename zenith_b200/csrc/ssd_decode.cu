// Recurrent (decode) form of the SSD scan: for each token in order,
//     h = e^{adt} h + gamma x k^T + beta xp kp^T ,   y = h q
// the per-token recurrence of the reference's test (tests/test_mamba3.py:10-21), started from a
// carried state (e.g. the final state of a chunked forward over the prompt) and advanced in
// place.  Memory-bound on the state: one CTA per (batch, head) keeps its [P, N] state in
// registers for all the call's tokens, reading and writing it once.
//
// 256 threads.  A state row of N columns is held by R = N/4 lanes (rounded up to a power of two),
// four columns per lane, so a warp holds 32/R rows at once (N = 64: two rows per warp, every lane
// busy); the 8 warps cover the P rows in passes.  Per token every load (the scalars, q / k / kp for
// the lane's columns, x / xp for its rows) is issued before any arithmetic, and the state moves as
// 16-byte words: the call is one round trip for the state in, one per token, one for the state out.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "ssd_kernels.h"

namespace zb {
namespace {

constexpr int kDecThreads = 256;
constexpr int kDecMaxPasses = 16;  // P <= 128 rows: at most 16 passes of 8 rows (N > 64)
// The kernel is compiled for at most MP passes (MP = 2, 4, 8, 16): the state of MP passes lives in
// registers, so a smaller MP keeps more CTAs per SM.

// four consecutive elements n0..n0+3 of a row (zero past N) as floats
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
  int lpr;            // lanes per state row (power of two, 4 columns each)
  bool vec;           // N % 4 == 0 and the states 16-byte aligned: 16-byte state accesses
};

template <typename TV, typename TS, int MP>
__global__ void __launch_bounds__(kDecThreads) ssd_decode_kernel(const DecParams p) {
  const int bh = blockIdx.x;
  const int b = bh / (int)p.H, h = bh % (int)p.H;
  const int g = h / (int)(p.H / p.G);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = (int)p.P, N = (int)p.N, lpr = p.lpr;
  const int rpw = 32 / lpr;               // rows per warp and pass
  const int sub = lane / lpr;             // this lane's row within the warp's group
  const int n0 = 4 * (lane % lpr);        // this lane's first column
  const int rows_per_pass = 8 * rpw;
  const int passes = (P + rows_per_pass - 1) / rows_per_pass;
  const int64_t PN = (int64_t)P * N;
  auto row_of = [&](int r) { return r * rows_per_pass + warp * rpw + sub; };
  float4 s[MP];
#pragma unroll
  for (int r = 0; r < MP; ++r) {
    s[r] = make_float4(0.f, 0.f, 0.f, 0.f);
    const int pp = row_of(r);
    if (r < passes && pp < P && p.init && n0 < N) {
      const float* src = p.init + bh * PN + (int64_t)pp * N + n0;
      s[r] = p.vec ? *reinterpret_cast<const float4*>(src) : ld4f(src, 0, N - n0);
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
    float xv[MP], xpv[MP];
#pragma unroll
    for (int r = 0; r < MP; ++r) {
      const int pp = row_of(r);
      const bool in = r < passes && pp < P;
      xv[r] = in ? ldv<float>(xr + pp) : 0.f;
      xpv[r] = in ? ldv<float>(xpr + pp) : 0.f;
    }
    TV* yr = p.y.wrow<TV>(b, t, h);
#pragma unroll
    for (int r = 0; r < MP; ++r) {
      if (r >= passes) break;
      const float gx = gm * xv[r], bx = bt * xpv[r];
      s[r].x = a * s[r].x + gx * kv.x + bx * kpv.x;
      s[r].y = a * s[r].y + gx * kv.y + bx * kpv.y;
      s[r].z = a * s[r].z + gx * kv.z + bx * kpv.z;
      s[r].w = a * s[r].w + gx * kv.w + bx * kpv.w;
      float yv = s[r].x * qv.x + s[r].y * qv.y + s[r].z * qv.z + s[r].w * qv.w;
      for (int o = lpr >> 1; o > 0; o >>= 1) yv += __shfl_xor_sync(0xffffffffu, yv, o);
      const int pp = row_of(r);
      if (lane % lpr == 0 && pp < P) stv<float>(yr + pp, yv);
    }
  }
#pragma unroll
  for (int r = 0; r < MP; ++r) {
    const int pp = row_of(r);
    if (r < passes && pp < P && n0 < N) {
      float* dst = p.fin + bh * PN + (int64_t)pp * N + n0;
      if (p.vec) {
        *reinterpret_cast<float4*>(dst) = s[r];
      } else {
        dst[0] = s[r].x;
        if (n0 + 1 < N) dst[1] = s[r].y;
        if (n0 + 2 < N) dst[2] = s[r].z;
        if (n0 + 3 < N) dst[3] = s[r].w;
      }
    }
  }
}

// Shared-memory variant (N % 4 == 0, 16-byte aligned states, state tile <= 48 KB): the state is
// copied into shared memory by 16-byte asynchronous copies, which hold no registers while in
// flight, so the state bytes in flight per SM are bounded by shared memory (about 200 KB) instead
// of by the registers that would hold them.  128 threads, rows in passes of 4 warps as above, one
// pass at a time; the token's x / xp are staged in shared memory; the last token writes the state
// straight back to global memory.
constexpr int kDecSmemThreads = 128;
constexpr int kDecSmemMaxBytes = 48 << 10;

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src)
               : "memory");
}

template <typename TV, typename TS>
__global__ void __launch_bounds__(kDecSmemThreads) ssd_decode_smem_kernel(const DecParams p) {
  extern __shared__ __align__(16) float s_st[];  // [P][N] state, then x [P] and xp [P] of the token
  const int bh = blockIdx.x;
  const int b = bh / (int)p.H, h = bh % (int)p.H;
  const int g = h / (int)(p.H / p.G);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int P = (int)p.P, N = (int)p.N, lpr = p.lpr;
  const int rpw = 32 / lpr, sub = lane / lpr, n0 = 4 * (lane % lpr);
  const int rows_per_pass = (kDecSmemThreads / 32) * rpw;
  const int passes = (P + rows_per_pass - 1) / rows_per_pass;
  const int PN = P * N;
  float* s_x = s_st + PN;
  float* s_xp = s_x + P;
  if (p.init) {
    const float* src = p.init + (int64_t)bh * PN;
    for (int i = 4 * tid; i < PN; i += 4 * kDecSmemThreads) cp_async16(s_st + i, src + i);
    asm volatile("cp.async.commit_group;" ::: "memory");
  } else {
    for (int i = tid; i < PN; i += kDecSmemThreads) s_st[i] = 0.f;
  }
  float* dst = p.fin + (int64_t)bh * PN;
  for (int64_t t = 0; t < p.T; ++t) {
    const float a = xexp<float>(ldv<float>(p.adt.row<TS>(b, t, h)));
    const float gm = ldv<float>(p.gamma.row<TS>(b, t, h)), bt = ldv<float>(p.beta.row<TS>(b, t, h));
    const float4 qv = ld4f(p.q.row<TV>(b, t, g), n0, N);
    const float4 kv = ld4f(p.k.row<TV>(b, t, g), n0, N);
    const float4 kpv = ld4f(p.kp.row<TV>(b, t, g), n0, N);
    const TV* xr = p.x.row<TV>(b, t, h);
    const TV* xpr = p.xp.row<TV>(b, t, h);
    for (int i = tid; i < P; i += kDecSmemThreads) {
      s_x[i] = ldv<float>(xr + i);
      s_xp[i] = ldv<float>(xpr + i);
    }
    if (t == 0) asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    TV* yr = p.y.wrow<TV>(b, t, h);
    const bool last = (t == p.T - 1);
    for (int r = 0; r < passes; ++r) {
      const int pp = r * rows_per_pass + warp * rpw + sub;
      const bool in = pp < P && n0 < N;
      float4 sv = in ? *reinterpret_cast<const float4*>(s_st + pp * N + n0) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float gx = in ? gm * s_x[pp] : 0.f, bx = in ? bt * s_xp[pp] : 0.f;
      sv.x = a * sv.x + gx * kv.x + bx * kpv.x;
      sv.y = a * sv.y + gx * kv.y + bx * kpv.y;
      sv.z = a * sv.z + gx * kv.z + bx * kpv.z;
      sv.w = a * sv.w + gx * kv.w + bx * kpv.w;
      float yv = sv.x * qv.x + sv.y * qv.y + sv.z * qv.z + sv.w * qv.w;
      for (int o = lpr >> 1; o > 0; o >>= 1) yv += __shfl_xor_sync(0xffffffffu, yv, o);
      if (lane % lpr == 0 && pp < P) stv<float>(yr + pp, yv);
      if (in) *reinterpret_cast<float4*>((last ? dst : s_st) + pp * N + n0) = sv;
    }
    __syncthreads();  // the next token overwrites x / xp
  }
}

View as_view(const zb_view& v) { return View{v.ptr, v.sb, v.st, v.sh}; }

template <typename TV>
int launch_decode(const DecParams& p, int64_t passes, dim3 grid, cudaStream_t s) {
  const int64_t smem = (p.P * p.N + 2 * p.P) * (int64_t)sizeof(float);
  if (p.vec && smem <= kDecSmemMaxBytes) {
    ssd_decode_smem_kernel<TV, float><<<grid, kDecSmemThreads, (size_t)smem, s>>>(p);
    return ZB_OK;
  }
  if (passes <= 2) ssd_decode_kernel<TV, float, 2><<<grid, kDecThreads, 0, s>>>(p);
  else if (passes <= 4) ssd_decode_kernel<TV, float, 4><<<grid, kDecThreads, 0, s>>>(p);
  else if (passes <= 8) ssd_decode_kernel<TV, float, 8><<<grid, kDecThreads, 0, s>>>(p);
  else if (passes <= kDecMaxPasses) ssd_decode_kernel<TV, float, kDecMaxPasses><<<grid, kDecThreads, 0, s>>>(p);
  else return ZB_ERR_UNSUPPORTED;
  return ZB_OK;
}

}  // namespace
}  // namespace zb

using namespace zb;

extern "C" ZB_API int zb_ssd_decode(const zb_ssd_args* a, void* stream) {
  if (!a) return ZB_ERR_LAYOUT;
  if (a->B <= 0 || a->T <= 0 || a->H <= 0 || a->G <= 0 || a->P <= 0 || a->N <= 0 || a->H % a->G != 0)
    return ZB_ERR_SHAPE;
  if (a->P > 8 * kDecMaxPasses || a->N > 128) return ZB_ERR_UNSUPPORTED;
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
  p.lpr = 1;
  while (p.lpr < 32 && 4 * p.lpr < a->N) p.lpr *= 2;
  p.vec = a->N % 4 == 0 && reinterpret_cast<uintptr_t>(a->final_state) % 16 == 0 &&
          reinterpret_cast<uintptr_t>(a->initial_state) % 16 == 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)(a->B * a->H));
  const int64_t rows_per_pass = 8 * (32 / p.lpr), passes = (a->P + rows_per_pass - 1) / rows_per_pass;
  int rc = ZB_ERR_DTYPE;
  switch (a->dtype) {
    case ZB_F32: rc = launch_decode<float>(p, passes, grid, s); break;
    case ZB_BF16: rc = launch_decode<__nv_bfloat16>(p, passes, grid, s); break;
    case ZB_F16: rc = launch_decode<__half>(p, passes, grid, s); break;
    default: break;
  }
  if (rc != ZB_OK) return rc;
  note_launches(1);
  return cudaPeekAtLastError() == cudaSuccess ? ZB_OK : ZB_ERR_CUDA;
}
