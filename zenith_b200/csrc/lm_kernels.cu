// Language-model kernels around the Mamba-3 layers (zenith/model.py:42-99): the residual add
// fused with the RMSNorm that reads it, and the next-token cross-entropy with its logit gradient
// in one pass over the logits.  Both are HBM-bound row kernels: 16-byte accesses, one warp per
// row (RMSNorm) or one CTA per row (cross-entropy), fixed-order reductions.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>

#include "common.cuh"
#include "ssd_kernels.h"
#include "zb_lm.h"

namespace zb {
namespace {

// ---------------------------------------------------------------------------------------------
// residual add + RMSNorm (mamba3.py:8-15; model.py:48-49,87,93)

constexpr int kNormWarps = 8;     // rows in flight per CTA, one warp each
constexpr int kNormGrid = 1024;   // CTAs at most: a fixed grid fixes the order of the dw sums
constexpr int kNormMaxD = 8192;
constexpr int kRowMaxThreads = 256;  // row kernels: D <= 8 x 256 (the registers of a row pair fit)

struct NormP {
  int64_t M, D;
  float eps;
  bool vec;   // D % 8 == 0 and every row pointer 16-byte aligned: 8-element accesses
  bool rows;  // vec and D <= 8 kRowMaxThreads: one CTA per row (the row kernels)
  const void *a, *b;
  void* s;
  const float* w;
  void* u;
  float* r;
  const void *du, *ds;
  void *dsum, *dsum_b;
  float* dw;
  float* part;  // [grid][D] per-CTA dw sums
};

// v rounded to the storage type T
template <typename T> __device__ __forceinline__ float round_to(float v);
template <> __device__ __forceinline__ float round_to<__nv_bfloat16>(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}
template <> __device__ __forceinline__ float round_to<float>(float v) { return v; }

// s = a + b (stored, then read back as stored), r = rsqrt(mean(s^2) + eps), u = (s r) w
template <typename TX, typename TB, typename TU>
__global__ void __launch_bounds__(32 * kNormWarps) rmsnorm_fwd_kernel(const NormP p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, D = (int)p.D;
  const TX* __restrict__ A = static_cast<const TX*>(p.a);
  const TB* __restrict__ Bv = static_cast<const TB*>(p.b);
  TX* __restrict__ S = static_cast<TX*>(p.s);
  TU* __restrict__ U = static_cast<TU*>(p.u);
  for (int64_t row = (int64_t)blockIdx.x * kNormWarps + warp; row < p.M; row += (int64_t)gridDim.x * kNormWarps) {
    const int64_t o = row * D;
    float ss = 0.f;
    if (p.vec) {
      for (int n = 8 * lane; n < D; n += 256) {
        float v[8];
        Vec8<TX>::ld(A + o + n, v);
        if (Bv) {
          float c[8];
          Vec8<TB>::ld(Bv + o + n, c);
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = round_to<TX>(v[e] + c[e]);
          Vec8<TX>::st(S + o + n, v);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += v[e] * v[e];
      }
    } else {
      for (int n = lane; n < D; n += 32) {
        float v = ldv<float>(A + o + n);
        if (Bv) {
          v = round_to<TX>(v + ldv<float>(Bv + o + n));
          stv<float>(S + o + n, v);
        }
        ss += v * v;
      }
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / D + p.eps);
    if (p.r && lane == 0) p.r[row] = r;
    const TX* __restrict__ src = Bv ? S : A;  // the lane re-reads only what it wrote itself
    if (p.vec) {
      for (int n = 8 * lane; n < D; n += 256) {
        float v[8], w[8];
        Vec8<TX>::ld(src + o + n, v);
        Vec8<float>::ld(p.w + n, w);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = v[e] * r * w[e];
        Vec8<TU>::st(U + o + n, v);
      }
    } else {
      for (int n = lane; n < D; n += 32) stv<float>(U + o + n, ldv<float>(src + o + n) * r * p.w[n]);
    }
  }
}

// dsum = ds + r w du - s r^3 / D sum(du w s) (also as TB in dsum_b); per-CTA dw sums of du s r
// (per warp in shared memory, then over the warps in order)
template <typename TX, typename TB, typename TU>
__global__ void __launch_bounds__(32 * kNormWarps) rmsnorm_bwd_kernel(const NormP p) {
  extern __shared__ float sdw[];  // [kNormWarps][D]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, D = (int)p.D;
  float* myw = sdw + warp * D;
  for (int n = lane; n < D; n += 32) myw[n] = 0.f;
  const TX* __restrict__ S = static_cast<const TX*>(p.b ? p.s : p.a);
  const TU* __restrict__ dU = static_cast<const TU*>(p.du);
  const TX* __restrict__ dS = static_cast<const TX*>(p.ds);
  TX* __restrict__ G = static_cast<TX*>(p.dsum);
  TB* __restrict__ GB = static_cast<TB*>(p.dsum_b);
  for (int64_t row = (int64_t)blockIdx.x * kNormWarps + warp; row < p.M; row += (int64_t)gridDim.x * kNormWarps) {
    const int64_t o = row * D;
    const float r = p.r[row];
    float dot = 0.f;
    if (p.vec) {
      for (int n = 8 * lane; n < D; n += 256) {
        float g[8], x[8], w[8];
        Vec8<TU>::ld(dU + o + n, g);
        Vec8<TX>::ld(S + o + n, x);
        Vec8<float>::ld(p.w + n, w);
#pragma unroll
        for (int e = 0; e < 8; ++e) dot += g[e] * w[e] * x[e];
      }
    } else {
      for (int n = lane; n < D; n += 32) dot += ldv<float>(dU + o + n) * p.w[n] * ldv<float>(S + o + n);
    }
    const float k3 = r * r * r / D * warp_sum(dot);
    if (p.vec) {
      for (int n = 8 * lane; n < D; n += 256) {
        float g[8], x[8], w[8], out[8];
        Vec8<TU>::ld(dU + o + n, g);
        Vec8<TX>::ld(S + o + n, x);
        Vec8<float>::ld(p.w + n, w);
        if (dS) Vec8<TX>::ld(dS + o + n, out);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          out[e] = (dS ? out[e] : 0.f) + r * w[e] * g[e] - x[e] * k3;
          myw[n + e] += g[e] * x[e] * r;
        }
        Vec8<TX>::st(G + o + n, out);
        if (GB) Vec8<TB>::st(GB + o + n, out);
      }
    } else {
      for (int n = lane; n < D; n += 32) {
        const float g = ldv<float>(dU + o + n), x = ldv<float>(S + o + n);
        const float v = (dS ? ldv<float>(dS + o + n) : 0.f) + r * p.w[n] * g - x * k3;
        stv<float>(G + o + n, v);
        if (GB) stv<float>(GB + o + n, v);
        myw[n] += g * x * r;
      }
    }
  }
  __syncthreads();
  for (int n = threadIdx.x; n < D; n += blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < kNormWarps; ++k) s += sdw[k * D + n];
    p.part[(int64_t)blockIdx.x * D + n] = s;
  }
}

// ---- one CTA per row, the row in registers (D % 8 == 0, 16-byte aligned rows): thread i owns
// features 8i .. 8i+7, so every element is read once and the dw sums stay in registers

// sum over the CTA, every thread gets the total (warp sums, then the warps' sums in order)
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int k = 0; k < nw; ++k) t += red[k];
  __syncthreads();  // red is reused by the next row
  return t;
}

template <typename TX, typename TB, typename TU>
__global__ void __launch_bounds__(kRowMaxThreads) rmsnorm_fwd_row_kernel(const NormP p) {
  __shared__ float red[32];
  const int D = (int)p.D, n = 8 * threadIdx.x;
  const bool on = n < D;
  const TX* __restrict__ A = static_cast<const TX*>(p.a);
  const TB* __restrict__ Bv = static_cast<const TB*>(p.b);
  TX* __restrict__ S = static_cast<TX*>(p.s);
  TU* __restrict__ U = static_cast<TU*>(p.u);
  float w[8];
  if (on) Vec8<float>::ld(p.w + n, w);
  for (int64_t row = blockIdx.x; row < p.M; row += gridDim.x) {
    const int64_t o = row * D + n;
    float v[8], ss = 0.f;
    if (on) {
      Vec8<TX>::ld(A + o, v);
      if (Bv) {
        float c[8];
        Vec8<TB>::ld(Bv + o, c);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = round_to<TX>(v[e] + c[e]);
        Vec8<TX>::st(S + o, v);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[e] * v[e];
    }
    const float r = rsqrtf(block_sum(ss, red) / D + p.eps);
    if (p.r && threadIdx.x == 0) p.r[row] = r;
    if (on) {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = v[e] * r * w[e];
      Vec8<TU>::st(U + o, v);
    }
  }
}

template <typename TX, typename TB, typename TU>
__global__ void __launch_bounds__(kRowMaxThreads) rmsnorm_bwd_row_kernel(const NormP p) {
  __shared__ float red[32];
  const int D = (int)p.D, n = 8 * threadIdx.x;
  const bool on = n < D;
  const TX* __restrict__ S = static_cast<const TX*>(p.b ? p.s : p.a);
  const TU* __restrict__ dU = static_cast<const TU*>(p.du);
  const TX* __restrict__ dS = static_cast<const TX*>(p.ds);
  TX* __restrict__ G = static_cast<TX*>(p.dsum);
  TB* __restrict__ GB = static_cast<TB*>(p.dsum_b);
  float w[8], dw[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (on) Vec8<float>::ld(p.w + n, w);
  // the next row's loads are issued before this row's reduction and stores
  Pack8<TU> gn;
  Pack8<TX> xn, dn;
  float rn = 0.f;
  int64_t row = blockIdx.x;
  if (row < p.M) {
    rn = p.r[row];
    if (on) {
      gn.ld(dU + row * D + n);
      xn.ld(S + row * D + n);
      if (dS) dn.ld(dS + row * D + n);
    }
  }
  for (; row < p.M; row += gridDim.x) {
    const int64_t o = row * D + n;
    const float r = rn;
    const Pack8<TU> gc = gn;
    const Pack8<TX> xc = xn, dc = dn;
    if (row + gridDim.x < p.M) {
      const int64_t o2 = o + (int64_t)gridDim.x * D;
      rn = p.r[row + gridDim.x];
      if (on) {
        gn.ld(dU + o2);
        xn.ld(S + o2);
        if (dS) dn.ld(dS + o2);
      }
    }
    float g[8], x[8], dot = 0.f;
    if (on) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        g[e] = gc.get(e);
        x[e] = xc.get(e);
        dot += g[e] * w[e] * x[e];
      }
    }
    const float k3 = r * r * r / D * block_sum(dot, red);
    if (on) {
      float out[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        out[e] = (dS ? dc.get(e) : 0.f) + r * w[e] * g[e] - x[e] * k3;
        dw[e] += g[e] * x[e] * r;
      }
      Vec8<TX>::st(G + o, out);
      if (GB) Vec8<TB>::st(GB + o, out);
    }
  }
  if (on) Vec8<float>::st(p.part + (int64_t)blockIdx.x * D + n, dw);
}

// dw[n] = sum over the CTAs' partials in CTA order: 32 features per CTA, the partials split over
// 8 warps (coalesced rows), then the warps' sums in order
__global__ void __launch_bounds__(256) rmsnorm_dw_kernel(const NormP p, int nblocks) {
  __shared__ float sm[8][33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * 32 + lane;
  float s = 0.f;
  if (n < p.D)
    for (int k = warp; k < nblocks; k += 8) s += p.part[(int64_t)k * p.D + n];
  sm[warp][lane] = s;
  __syncthreads();
  if (warp == 0 && n < p.D) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += sm[k][lane];
    p.dw[n] = t;
  }
}

// warp-per-row kernels: M / 8 CTAs up to kNormGrid; row kernels: M CTAs up to kNormGrid
int norm_grid_warp(int64_t M) { return (int)((M + kNormWarps - 1) / kNormWarps < kNormGrid ? (M + kNormWarps - 1) / kNormWarps : kNormGrid); }
int row_grid(int64_t M) { return (int)(M < kNormGrid ? M : kNormGrid); }
int row_threads(int64_t D) { return (int)((D / 8 + 31) / 32 * 32); }


bool aligned16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; }

int norm_check(const zb_rmsnorm_args* a) {
  if (!a) return ZB_ERR_LAYOUT;
  if (a->M <= 0 || a->D <= 0) return ZB_ERR_SHAPE;
  if (a->D > kNormMaxD) return ZB_ERR_UNSUPPORTED;
  for (int32_t d : {a->x_dtype, a->b_dtype, a->u_dtype})
    if (d != ZB_F32 && d != ZB_BF16) return ZB_ERR_DTYPE;
  if (!a->a || !a->w) return ZB_ERR_LAYOUT;
  return ZB_OK;
}

NormP make_norm(const zb_rmsnorm_args* a, bool bwd) {
  NormP p;
  p.M = a->M; p.D = a->D; p.eps = a->eps;
  p.a = a->a; p.b = a->b; p.s = a->s; p.w = a->w; p.u = a->u; p.r = a->r;
  p.du = a->du; p.ds = a->ds; p.dsum = a->dsum; p.dsum_b = a->dsum_b; p.dw = a->dw;
  p.part = static_cast<float*>(a->workspace);
  const void* ptrs_f[] = {a->a, a->b, a->s, a->w, a->u};
  const void* ptrs_b[] = {a->a, a->b, a->s, a->w, a->du, a->ds, a->dsum, a->dsum_b};
  bool ok = a->D % 8 == 0;
  if (bwd) { for (const void* q : ptrs_b) ok = ok && aligned16(q); }
  else { for (const void* q : ptrs_f) ok = ok && aligned16(q); }
  p.vec = ok;
  p.rows = ok && a->D <= 8 * kRowMaxThreads;
  return p;
}

// call f with a value of the element type that a zb_dtype code names (float or bf16)
template <typename F> int with_type(int32_t code, F&& f) {
  switch (code) {
    case ZB_F32: return f(float{});
    case ZB_BF16: return f(__nv_bfloat16{});
    default: return ZB_ERR_DTYPE;
  }
}

// ---------------------------------------------------------------------------------------------
// cross-entropy (model.py:95-97): one CTA per row

constexpr int kXentThreads = 512;

struct XentP {
  int64_t M, V, ld, ignore;
  bool write_grad;
  void* logits;
  const int64_t* labels;
  float* loss;
  float* lse;
  int32_t* status;
};

// max and sum of exp over the CTA: warp shuffles, then the warps' pairs in order
__device__ __forceinline__ void block_max_sum(float& m, float& s, float* sm, float* ss) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float M = fmaxf(m, m2);
    s = (M == -INFINITY) ? 0.f : s * expf(m - M) + s2 * expf(m2 - M);
    m = M;
  }
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
  }
  __syncthreads();
  float M = -INFINITY;
  for (int k = 0; k < nw; ++k) M = fmaxf(M, sm[k]);
  float S = 0.f;
  if (M != -INFINITY)
    for (int k = 0; k < nw; ++k) S += ss[k] * expf(sm[k] - M);
  m = M;
  s = S;
}

constexpr float kLog2e = 1.4426950408889634f;

// kPer > 0: the row is held in registers (packed), kPer 8-element units per thread (V % 8 == 0,
// aligned rows); kPer == 0: any V, the row is read twice.  Exponentials are base 2 of the logits
// scaled by log2(e) (one multiply-add and exp2f per element).
template <typename T, int kPer>
__global__ void __launch_bounds__(kXentThreads) xent_kernel(const XentP p) {
  __shared__ float sm[kXentThreads / 32], ss[kXentThreads / 32];
  const int64_t row = blockIdx.x;
  T* __restrict__ L = static_cast<T*>(p.logits) + row * p.ld;
  const int V = (int)p.V;
  const int64_t lab = p.labels[row];
  bool valid = lab != p.ignore;
  if (valid && (lab < 0 || lab >= p.V)) {
    if (threadIdx.x == 0) atomicCAS(p.status, 0, (int32_t)ZB_ERR_INDEX);
    valid = false;
  }
  const float xl = (valid && threadIdx.x == 0) ? ldv<float>(L + lab) : 0.f;  // before any thread writes
  float m = -INFINITY, s = 0.f;
  Pack8<T> v[kPer > 0 ? kPer : 1];
  if constexpr (kPer > 0) {
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int n = (i * kXentThreads + threadIdx.x) * 8;
      if (n < V) v[i].ld(L + n);
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int n = (i * kXentThreads + threadIdx.x) * 8;
      if (n < V)
#pragma unroll
        for (int e = 0; e < 8; ++e) m = fmaxf(m, v[i].get(e));
    }
    if (m != -INFINITY) {
      const float ml = m * kLog2e;
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int n = (i * kXentThreads + threadIdx.x) * 8;
        if (n < V)
#pragma unroll
          for (int e = 0; e < 8; ++e) s += exp2f(fmaf(v[i].get(e), kLog2e, -ml));
      }
    }
  } else {
    for (int n = threadIdx.x; n < V; n += kXentThreads) {
      const float x = ldv<float>(L + n);
      if (x > m) {
        s = s * expf(m - x) + 1.f;
        m = x;
      } else {
        s += expf(x - m);
      }
    }
  }
  block_max_sum(m, s, sm, ss);
  const float lse = m + logf(s);
  if (threadIdx.x == 0) {
    p.loss[row] = valid ? lse - xl : 0.f;
    if (p.lse) p.lse[row] = lse;
  }
  if (!p.write_grad) return;
  if constexpr (kPer > 0) {
    const float ll = lse * kLog2e;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int n = (i * kXentThreads + threadIdx.x) * 8;
      if (n < V) {
        float g[8];
#pragma unroll
        for (int e = 0; e < 8; ++e)
          g[e] = valid ? exp2f(fmaf(v[i].get(e), kLog2e, -ll)) - (n + e == lab ? 1.f : 0.f) : 0.f;
        Vec8<T>::st(L + n, g);
      }
    }
  } else {
    for (int n = threadIdx.x; n < V; n += kXentThreads) {
      const float x = ldv<float>(L + n);
      stv<float>(L + n, valid ? expf(x - lse) - (n == lab ? 1.f : 0.f) : 0.f);
    }
  }
}

template <typename T> int launch_xent(const XentP& p, bool vec, cudaStream_t st) {
  const dim3 grid((unsigned)p.M);
  const int64_t unit = (int64_t)kXentThreads * 8;
  if (vec && p.V <= unit) xent_kernel<T, 1><<<grid, kXentThreads, 0, st>>>(p);
  else if (vec && p.V <= 2 * unit) xent_kernel<T, 2><<<grid, kXentThreads, 0, st>>>(p);
  else if (vec && p.V <= 4 * unit) xent_kernel<T, 4><<<grid, kXentThreads, 0, st>>>(p);
  else if (vec && p.V <= 8 * unit) xent_kernel<T, 8><<<grid, kXentThreads, 0, st>>>(p);
  else xent_kernel<T, 0><<<grid, kXentThreads, 0, st>>>(p);
  return ZB_OK;
}

int finish_lm(int n) {
  note_launches(n);
  return cudaPeekAtLastError() == cudaSuccess ? ZB_OK : ZB_ERR_CUDA;
}

}  // namespace
}  // namespace zb

using namespace zb;

extern "C" ZB_API uint64_t zb_rmsnorm_workspace_bytes(const zb_rmsnorm_args* a) {
  if (!a || a->M <= 0 || a->D <= 0) return 0;
  return align_up((size_t)row_grid(a->M) * a->D * sizeof(float), 256);  // row_grid >= norm_grid_warp
}

extern "C" ZB_API int zb_rmsnorm_fwd(const zb_rmsnorm_args* a, void* stream) {
  int rc = norm_check(a);
  if (rc) return rc;
  if (!a->u || (a->b && !a->s)) return ZB_ERR_LAYOUT;
  const NormP p = make_norm(a, false);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = with_type(a->x_dtype, [&](auto tx) {
    return with_type(a->b_dtype, [&](auto tb) {
      return with_type(a->u_dtype, [&](auto tu) {
        using TX = decltype(tx);
        using TB = decltype(tb);
        using TU = decltype(tu);
        if (p.rows) rmsnorm_fwd_row_kernel<TX, TB, TU><<<row_grid(a->M), row_threads(a->D), 0, st>>>(p);
        else rmsnorm_fwd_kernel<TX, TB, TU><<<norm_grid_warp(a->M), 32 * kNormWarps, 0, st>>>(p);
        return (int)ZB_OK;
      });
    });
  });
  return rc ? rc : finish_lm(1);
}

extern "C" ZB_API int zb_rmsnorm_bwd(const zb_rmsnorm_args* a, void* stream) {
  int rc = norm_check(a);
  if (rc) return rc;
  if (!a->du || !a->dsum || !a->dw || !a->r || (a->b && !a->s)) return ZB_ERR_LAYOUT;
  if (!a->workspace || a->workspace_bytes < zb_rmsnorm_workspace_bytes(a) ||
      (reinterpret_cast<uintptr_t>(a->workspace) & 255))
    return ZB_ERR_WORKSPACE;
  const NormP p = make_norm(a, true);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = p.rows ? row_grid(a->M) : norm_grid_warp(a->M);
  const int smem = (int)(kNormWarps * a->D * sizeof(float));
  rc = with_type(a->x_dtype, [&](auto tx) {
    return with_type(a->b_dtype, [&](auto tb) {
      return with_type(a->u_dtype, [&](auto tu) {
        using TX = decltype(tx);
        using TB = decltype(tb);
        using TU = decltype(tu);
        if (p.rows) {
          rmsnorm_bwd_row_kernel<TX, TB, TU><<<grid, row_threads(a->D), 0, st>>>(p);
          return (int)ZB_OK;
        }
        auto k = rmsnorm_bwd_kernel<TX, TB, TU>;
        if (dyn_smem(reinterpret_cast<const void*>(k), smem) != ZB_OK)
          return (int)ZB_ERR_CUDA;
        k<<<grid, 32 * kNormWarps, smem, st>>>(p);
        return (int)ZB_OK;
      });
    });
  });
  if (rc) return rc;
  rmsnorm_dw_kernel<<<(unsigned)((a->D + 31) / 32), 256, 0, st>>>(p, grid);
  return finish_lm(2);
}

extern "C" ZB_API int zb_xent(const zb_xent_args* a, void* stream) {
  if (!a) return ZB_ERR_LAYOUT;
  if (a->M <= 0 || a->V <= 0 || a->ld < a->V || a->M > 0x7fffffff || a->V > 0x7fffffff) return ZB_ERR_SHAPE;
  if (!a->logits || !a->labels || !a->loss || !a->status) return ZB_ERR_LAYOUT;
  XentP p;
  p.M = a->M; p.V = a->V; p.ld = a->ld; p.ignore = a->ignore_index;
  p.write_grad = a->write_grad != 0;
  p.logits = a->logits; p.labels = a->labels; p.loss = a->loss; p.lse = a->lse; p.status = a->status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t es = a->dtype == ZB_F32 ? 4 : 2;
  const bool vec = a->V % 8 == 0 && (a->ld * es) % 16 == 0 && aligned16(a->logits);
  switch (a->dtype) {
    case ZB_F32: launch_xent<float>(p, vec, st); break;
    case ZB_BF16: launch_xent<__nv_bfloat16>(p, vec, st); break;
    default: return ZB_ERR_DTYPE;
  }
  return finish_lm(1);
}
