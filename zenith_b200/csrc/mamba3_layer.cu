// Mamba-3 layer body around the SSD scan (zenith/mamba3.py:96-119), forward and backward:
// the prologue that turns the in_proj split into the scan operands (discretisation, RMSNorm,
// RoPE, one-token shift) and the epilogue (D skip, silu gate).
//
// One CTA per (batch, 64-token segment, head group), one warp per head of the group (at most 29
// heads a group; H <= 31 is one group).  Per-token RMSNorm and
// RoPE run lane-parallel over the state features: lane i owns RoPE pair i (features 2i, 2i+1)
// and the pass-through pair (2A+2i, 2A+2i+1), A = N/4 angles.  theta = cumsum_t(DT ang) spans
// the whole sequence; it crosses segments through per-segment sums (forward) and per-segment
// totals of its gradient (backward).  Reductions over heads and over (batch, token) run in a
// fixed order, so results are bitwise reproducible.  With several head groups the backward's sums
// over heads are summed per group, then over the groups by a per-token kernel.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"
#include "ssd_kernels.h"
#include "umma.cuh"
#include "zb_mamba3.h"

namespace zb {
namespace {

constexpr int kSeg = 64;  // tokens per segment
// row kernels run one warp per head, up to 32 heads: 1024 threads, at most 64 registers each

struct M3 {
  int64_t B, T, H, P, N;
  int NA, nseg;
  int hg, nhg;  // heads per group, head groups: CTA (b, seg, g) owns heads g hg .. min(H, (g + 1) hg) - 1
  bool pairs;  // B / C rows and their gradients allow 2-element accesses (checked on the host)
  bool vec8;   // x, z, out, dout, dx, dz allow 16-byte accesses of 8 elements (checked on the host)
  bool rows8;  // Bm, Cm rows allow 16-byte accesses of 8 elements (checked on the host)
  float A_floor, eps;
  View x, z, Bm, Cm, dd_dt, dd_A, trap, ang;
  const float *dt_bias, *B_bias, *C_bias, *B_norm_w, *C_norm_w, *D;
  void *q, *k_ext, *xp;
  float *adt, *gamma, *beta, *theta;
  const void* y;
  View out, dout;
  void* dy;
  const void *dxs, *dxp, *dq, *dk, *dkp;
  const float *dadt, *dgamma, *dbeta;
  View dx, dz, dBm, dCm, ddd_dt, ddd_A, dtrap, dang;
  float *ddt_bias, *dB_bias, *dC_bias, *dB_norm_w, *dC_norm_w, *dD;
  int32_t* status;  // device word: a bounded wait that gave up records ZB_ERR_TIMEOUT
  const float* theta0;  // [B][H][NA] theta before the first token, or null (0)
  const void* kp0;      // [B][H][N] k of the token before the first (k_ext row 0), or null (0)
  // scratch
  float* segsum;  // [B][H][nseg][NA]   theta segment sums (forward) / theta-gradient segment totals (backward)
  float* dDTl;    // [B][T][H]          backward: DT gradient through theta, within-segment part
  float* dangl;   // [nhg][B][T][NA]    backward: ang gradient, within-segment part (per head group)
  float* duC;     // [nhg][B][T][N]     backward, nhg > 1: C row gradient before the RMSNorm, per head group
  float* duB;     // [nhg][B][T][N]     backward, nhg > 1: B row gradient before the RMSNorm, per head group
  float* pbias;   // [2][B][nseg][H][N] backward: B_bias, C_bias partial sums
  float* pnorm;   // [2][B][nseg][N]    backward: B_norm_w, C_norm_w partial sums
  float* pdt;     // [B][nseg][H]       backward: dt_bias partial sums
  float* pD;      // [B][nseg][H]       backward: D partial sums
};

// ---------------------------------------------------------------------------------------------
// per-token discretisation (mamba3.py:105-110)

__device__ __forceinline__ float softplus20(float v) { return v > 20.f ? v : log1pf(expf(v)); }
__device__ __forceinline__ float sigmoidf_(float v) { return 1.f / (1.f + expf(-v)); }
// The silu gate's sigmoid, evaluated per output element: the hardware exponential and a fast
// reciprocal (relative error about 1e-6 for |v| < 10; 0 once 1 + e^-v passes 2^126, where the
// sigmoid is below 1e-38 anyway).
__device__ __forceinline__ float gate_sigmoid(float v) { return __fdividef(1.f, 1.f + __expf(-v)); }

// sin and cos of a RoPE angle theta (a running sum over the sequence, so it grows without bound).
// Cody-Waite reduction by 2 pi (Cody and Waite, "Software Manual for the Elementary Functions",
// 1980): theta - k 2pi with k the nearest integer and 2pi split into its float value plus the
// remainder, each product folded in by one fma; then the hardware approximation on [-pi, pi],
// whose absolute error there is below 5e-7.  For |theta| up to 1e5 the reduction adds under 1e-7.
__device__ __forceinline__ void sincos_angle(float theta, float* sn, float* cs) {
  constexpr float kTwoPiHi = 6.28318548202514648f;  // 2 pi rounded to float
  constexpr float kTwoPiLo = -1.74845553e-7f;       // 2 pi - kTwoPiHi
  const float k = rintf(theta * 0.159154943091895336f);
  const float r = fmaf(-k, kTwoPiLo, fmaf(-k, kTwoPiHi, theta));
  __sincosf(r, sn, cs);
}

struct Disc {
  float DT, A, adt, tr, gamma, beta, ea, ht, xs;
};
__device__ __forceinline__ Disc discretise(float dd_dt, float dd_A, float trap, float dt_bias, float A_floor) {
  Disc d;
  d.ht = fmaxf(dd_A, 0.f) + 1.f / (1.f - fminf(dd_A, 0.f));  // heavy_tail (mamba3.py:18-19)
  d.A = -fminf(d.ht, -A_floor);                                 // -heavy_tail(dd_A).clamp(max=-A_floor)
  d.xs = dd_dt + dt_bias;
  d.DT = softplus20(d.xs);
  d.adt = d.A * d.DT;
  d.tr = sigmoidf_(trap);
  d.gamma = d.tr * d.DT;
  d.ea = expf(d.adt);
  d.beta = (1.f - d.tr) * d.DT * d.ea;
  return d;
}

// the four features lane owns: f[0], f[0]+1 rotated by theta_lane, f[2], f[2]+1 passed through
struct Feat {
  int f0, f2;
  bool on;
};
__device__ __forceinline__ Feat feat(int lane, int NA) { return {2 * lane, 2 * NA + 2 * lane, lane < NA}; }

// two adjacent elements (an even feature index) as one access
template <typename T> struct Pair;
template <> struct Pair<float> {
  static __device__ __forceinline__ float2 ld(const float* p) { return *reinterpret_cast<const float2*>(p); }
  static __device__ __forceinline__ void st(float* p, float a, float b) { *reinterpret_cast<float2*>(p) = make_float2(a, b); }
};
template <> struct Pair<__nv_bfloat16> {
  static __device__ __forceinline__ float2 ld(const __nv_bfloat16* p) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
  }
  static __device__ __forceinline__ void st(__nv_bfloat16* p, float a, float b) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
  }
};

// the lane's four features of a row; pairs = the row allows 2-element accesses
template <typename T> __device__ __forceinline__ void ld4(const T* row, Feat f, float (&v)[4], bool pairs = true) {
  if (pairs) {
    const float2 a = Pair<T>::ld(row + f.f0), c = Pair<T>::ld(row + f.f2);
    v[0] = a.x; v[1] = a.y; v[2] = c.x; v[3] = c.y;
  } else {
    v[0] = ldv<float>(row + f.f0);
    v[1] = ldv<float>(row + f.f0 + 1);
    v[2] = ldv<float>(row + f.f2);
    v[3] = ldv<float>(row + f.f2 + 1);
  }
}
template <typename T> __device__ __forceinline__ void st4(T* row, Feat f, const float (&v)[4], bool pairs = true) {
  if (pairs) {
    Pair<T>::st(row + f.f0, v[0], v[1]);
    Pair<T>::st(row + f.f2, v[2], v[3]);
  } else {
    stv<float>(row + f.f0, v[0]);
    stv<float>(row + f.f0 + 1, v[1]);
    stv<float>(row + f.f2, v[2]);
    stv<float>(row + f.f2 + 1, v[3]);
  }
}

// the lane's four features of an fp32 row (8-byte aligned pairs: two 2-float loads)
__device__ __forceinline__ void ldp4(const float* row, Feat f, float (&v)[4]) {
  const float2 a = *reinterpret_cast<const float2*>(row + f.f0), c = *reinterpret_cast<const float2*>(row + f.f2);
  v[0] = a.x;
  v[1] = a.y;
  v[2] = c.x;
  v[3] = c.y;
}

// rope(rmsnorm(c) + bias): u = c r w + bias (mamba3.py:13-15,113-114), then rotate the first pair
__device__ __forceinline__ void norm_bias_rope(const float (&c)[4], float r, const float (&w)[4], const float (&bias)[4],
                                               float sn, float cs, float (&u)[4], float (&o)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) u[j] = c[j] * r * w[j] + bias[j];
  o[0] = u[0] * cs - u[1] * sn;  // rope (mamba3.py:22-27)
  o[1] = u[0] * sn + u[1] * cs;
  o[2] = u[2];
  o[3] = u[3];
}

// the CTA's (batch, segment, head group): blockIdx.x = (b nseg + seg) nhg + g, heads h0 .. h0 + hc - 1
struct Blk {
  int b, seg, g, h0, hc;
};
__device__ __forceinline__ Blk blk(const M3& p) {
  Blk k;
  k.g = blockIdx.x % p.nhg;
  const int bs = blockIdx.x / p.nhg;
  k.b = bs / p.nseg;
  k.seg = bs % p.nseg;
  k.h0 = k.g * p.hg;
  k.hc = min(p.hg, (int)p.H - k.h0);
  return k;
}

// ---------------------------------------------------------------------------------------------
// forward
//
// Every row kernel stages its segment's per-token inputs (B / C rows, angles, scalars) in shared
// memory with coalesced loads first, so the per-head walks over the segment read shared memory
// only; theta's running sum is the one serial dependency.

// shared layout of a forward segment: C rows, B rows (both scaled by their RMSNorm factor),
// angles, DT per head of the group
struct FwdSeg {
  float *c, *bm, *ang, *dt;
  __device__ FwdSeg(float* s, int N, int NA)
      : c(s), bm(s + kSeg * N), ang(s + 2 * kSeg * N), dt(s + 2 * kSeg * N + kSeg * NA) {}
};

// stage the segment's C / B rows and angles; optionally scale the rows by their RMSNorm factor.
// One warp per token: it copies the token's rows (16-byte vectors when the views allow), then sums
// their squares from its own copy, so no block barrier separates the two.
template <typename TI>
__device__ __forceinline__ void stage_rows(const M3& p, int b, int64_t t0, int nt, float* c, float* bm, float* ang,
                                           float* rfac) {
  const int N = (int)p.N, NA = p.NA;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  for (int t = warp; t < nt; t += nwarps) {
    const TI* cr = p.Cm.row<TI>(b, t0 + t, 0);
    const TI* br = p.Bm.row<TI>(b, t0 + t, 0);
    const TI* ar = p.ang.row<TI>(b, t0 + t, 0);
    float* cs = c + t * N;
    float* bs = bm + t * N;
    if (p.rows8) {
      for (int n = 8 * lane; n < N; n += 256) {
        float v[8];
        Vec8<TI>::ld(cr + n, v);
#pragma unroll
        for (int e = 0; e < 8; ++e) cs[n + e] = v[e];
        Vec8<TI>::ld(br + n, v);
#pragma unroll
        for (int e = 0; e < 8; ++e) bs[n + e] = v[e];
      }
    } else {
      for (int n = lane; n < N; n += 32) {
        cs[n] = ldv<float>(cr + n);
        bs[n] = ldv<float>(br + n);
      }
    }
    for (int i = lane; i < NA; i += 32) ang[t * NA + i] = ldv<float>(ar + i);
    __syncwarp();
    // RMSNorm factors r = rsqrt(mean(x^2) + eps)
    float sc = 0.f, sb = 0.f;
    for (int n = lane; n < N; n += 32) {
      sc += cs[n] * cs[n];
      sb += bs[n] * bs[n];
    }
    sc = warp_sum(sc);
    sb = warp_sum(sb);
    const float rc = rsqrtf(sc / N + p.eps), rb = rsqrtf(sb / N + p.eps);
    if (rfac) {
      if (lane == 0) {
        rfac[2 * t] = rc;
        rfac[2 * t + 1] = rb;
      }
    } else {
      for (int n = lane; n < N; n += 32) {
        cs[n] *= rc;
        bs[n] *= rb;
      }
    }
  }
  __syncthreads();
}

// theta segment sums: segsum[b][h][seg][i] = sum over the segment's tokens of DT * ang_i
template <typename TI>
__global__ void __launch_bounds__(1024) m3_segsum_kernel(const M3 p) {
  extern __shared__ float smem[];
  const Blk k = blk(p);
  const int b = k.b, seg = k.seg, hc = k.hc;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = (int)p.H, NA = p.NA;
  const int64_t t0 = (int64_t)seg * kSeg;
  const int nt = (int)min((int64_t)kSeg, p.T - t0);
  float* sA = smem;              // [kSeg][NA]
  float* sDT = smem + kSeg * NA;  // [kSeg][hc]
  for (int idx = threadIdx.x; idx < nt * NA; idx += blockDim.x)
    sA[idx] = ldv<float>(p.ang.row<TI>(b, t0 + idx / NA, 0) + idx % NA);
  for (int idx = threadIdx.x; idx < nt * hc; idx += blockDim.x) {
    const int t = idx / hc, hh = k.h0 + idx % hc;
    sDT[idx] = softplus20(ldv<float>(p.dd_dt.row<TI>(b, t0 + t, hh)) + p.dt_bias[hh]);
  }
  __syncthreads();
  if (w < hc && lane < NA) {
    float acc = 0.f;
    for (int t = 0; t < nt; ++t) acc += sDT[t * hc + w] * sA[t * NA + lane];
    p.segsum[((b * H + k.h0 + w) * p.nseg + seg) * NA + lane] = acc;
  }
}

// q, k (into k_ext rows t+1), xp, adt, gamma, beta and theta for one segment of one batch, the
// heads of one group
template <typename TI, typename TO>
__global__ void __launch_bounds__(1024) m3_prologue_fwd_kernel(const M3 p) {
  extern __shared__ float smem[];
  const Blk k = blk(p);
  const int b = k.b, seg = k.seg, hc = k.hc;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, h = k.h0 + w;
  const int NA = p.NA, N = (int)p.N, P = (int)p.P, H = (int)p.H;
  const int64_t t0 = (int64_t)seg * kSeg;
  const int nt = (int)min((int64_t)kSeg, p.T - t0);
  FwdSeg S(smem, N, NA);
  // per (token, head) discretisation: scan scalars out, DT kept for theta
  for (int idx = threadIdx.x; idx < nt * hc; idx += blockDim.x) {
    const int t = idx / hc, hl = idx % hc, hh = k.h0 + hl;
    const Disc d = discretise(ldv<float>(p.dd_dt.row<TI>(b, t0 + t, hh)), ldv<float>(p.dd_A.row<TI>(b, t0 + t, hh)),
                              ldv<float>(p.trap.row<TI>(b, t0 + t, hh)), p.dt_bias[hh], p.A_floor);
    const int64_t bth = (b * p.T + t0 + t) * H + hh;
    p.adt[bth] = d.adt;
    p.gamma[bth] = d.gamma;
    p.beta[bth] = d.beta;
    S.dt[t * hc + hl] = d.DT;
  }
  stage_rows<TI>(p, b, t0, nt, S.c, S.bm, S.ang, nullptr);  // rows scaled by their RMSNorm factor
  TO* __restrict__ q = static_cast<TO*>(p.q);
  TO* __restrict__ kx = static_cast<TO*>(p.k_ext);
  const int64_t HN = (int64_t)H * N;
  const Feat f = feat(lane, NA);
  if (w < hc && f.on) {
    float th = p.theta0 ? p.theta0[(int64_t)(b * H + h) * NA + lane] : 0.f;  // theta at the end of the previous segment
    const float* __restrict__ ss = p.segsum + (int64_t)(b * H + h) * p.nseg * NA + lane;
#pragma unroll 8
    for (int s = 0; s < seg; ++s) th += __ldg(ss + (int64_t)s * NA);
    float wc[4], wb[4], cb[4], bb[4];
    ldp4(p.C_norm_w, f, wc);
    ldp4(p.B_norm_w, f, wb);
    ldp4(p.C_bias + h * N, f, cb);
    ldp4(p.B_bias + h * N, f, bb);
    if (seg == 0) {  // k_ext row 0 = kp of token 0: the previous token's k, or 0 at the sequence start
      float k0[4] = {0.f, 0.f, 0.f, 0.f};
      if (p.kp0) ld4(static_cast<const TO*>(p.kp0) + (int64_t)(b * H + h) * N, f, k0);
      st4(kx + (int64_t)b * (p.T + 1) * HN + h * N, f, k0);
    }
    // two tokens per pass: their shared-memory reads come before the global stores (which may
    // alias them for the compiler), so the two sincos / RoPE chains overlap
    for (int t = 0; t < nt; t += 2) {
      const int nu = t + 1 < nt ? 2 : 1;
      float th2[2], c[2][4], bm[2][4];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (u < nu) {
          th += S.dt[(t + u) * hc + w] * S.ang[(t + u) * NA + lane];  // theta = cumsum_t(DT ang) (mamba3.py:111)
          ldp4(S.c + (t + u) * N, f, c[u]);
          ldp4(S.bm + (t + u) * N, f, bm[u]);
        }
        th2[u] = th;
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (u >= nu) continue;
        const int64_t bth = (b * p.T + t0 + t + u) * H + h;
        p.theta[bth * NA + lane] = th2[u];
        float sn, cs, uu[4], o[4];
        sincos_angle(th2[u], &sn, &cs);
        const float one = 1.f;
        norm_bias_rope(c[u], one, wc, cb, sn, cs, uu, o);
        st4(q + bth * N, f, o);
        norm_bias_rope(bm[u], one, wb, bb, sn, cs, uu, o);
        st4(kx + (b * (p.T + 1) + t0 + t + u + 1) * HN + h * N, f, o);
      }
    }
  }
  // xp = x one token later (mamba3.py:115), all threads over (token, group head, feature); not
  // needed (NULL) when the scan reads x one token earlier itself (ZB_FLAG_SHIFTED)
  TO* __restrict__ xp = static_cast<TO*>(p.xp);
  const int HP = H * P, GP = hc * P;
  if (!xp) return;
  if (p.vec8) {
    const int GP8 = GP / 8, P8 = P / 8;
    for (int idx = threadIdx.x; idx < nt * GP8; idx += blockDim.x) {
      const int t = idx / GP8, r8 = idx % GP8, hh = k.h0 + r8 / P8, pp = (r8 % P8) * 8;
      const int64_t tt = t0 + t;
      float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (tt > 0) Vec8<TI>::ld(p.x.row<TI>(b, tt - 1, hh) + pp, v);
      Vec8<TO>::st(xp + (b * p.T + tt) * HP + hh * P + pp, v);
    }
  } else {
    for (int idx = threadIdx.x; idx < nt * GP; idx += blockDim.x) {
      const int t = idx / GP, r = k.h0 * P + idx % GP, hh = r / P, pp = r % P;
      const int64_t tt = t0 + t;
      stv<float>(xp + (b * p.T + tt) * HP + r, tt > 0 ? ldv<float>(p.x.row<TI>(b, tt - 1, hh) + pp) : 0.f);
    }
  }
}

// out = (y + D x) * silu(z)   (mamba3.py:119); 256 threads over (token, head, feature)
template <typename TI, typename TO>
__global__ void __launch_bounds__(256) m3_epilogue_fwd_kernel(const M3 p) {
  const int b = blockIdx.x / p.nseg, seg = blockIdx.x % p.nseg;
  const int P = (int)p.P, HP = (int)(p.H * P);
  const int64_t t0 = (int64_t)seg * kSeg;
  const int nt = (int)min((int64_t)kSeg, p.T - t0);
  const TO* __restrict__ y = static_cast<const TO*>(p.y);
#pragma unroll 4
  for (int idx = threadIdx.x; idx < nt * HP; idx += blockDim.x) {
    const int t = idx / HP, r = idx % HP, hh = r / P, pp = r % P;
    const int64_t tt = t0 + t;
    float v = ldv<float>(y + (b * p.T + tt) * HP + r) + p.D[hh] * ldv<float>(p.x.row<TI>(b, tt, hh) + pp);
    if (p.z.ptr) {
      const float zz = ldv<float>(p.z.row<TI>(b, tt, hh) + pp);
      v *= zz * gate_sigmoid(zz);
    }
    stv<float>(p.out.wrow<TI>(b, tt, hh) + pp, v);
  }
}

// ---------------------------------------------------------------------------------------------
// backward

// dy = dout silu(z) for the scan; dz = dout (y + D x) silu'(z); D partial sums of dy . x.
// 256 threads; thread tid keeps features r = tid + 256 k of every token, so its sums have a fixed head.
template <typename TI, typename TO>
__global__ void __launch_bounds__(256) m3_epilogue_bwd_kernel(const M3 p) {
  extern __shared__ float sacc[];  // [H * P] per-feature sums
  const int b = blockIdx.x / p.nseg, seg = blockIdx.x % p.nseg;
  const int P = (int)p.P, H = (int)p.H, HP = H * P;
  const int64_t t0 = (int64_t)seg * kSeg;
  const int nt = (int)min((int64_t)kSeg, p.T - t0);
  const TO* __restrict__ y = static_cast<const TO*>(p.y);
  TO* __restrict__ dy = static_cast<TO*>(p.dy);
  constexpr int kSlots = 32;  // HP <= 32 * 256 features per token
  float acc[kSlots];
#pragma unroll
  for (int s = 0; s < kSlots; ++s) acc[s] = 0.f;
  for (int t = 0; t < nt; ++t) {
    const int64_t tt = t0 + t;
#pragma unroll
    for (int s = 0; s < kSlots; ++s) {
      const int r = threadIdx.x + 256 * s;
      if (r >= HP) break;
      const int hh = r / P, pp = r % P;
      const float go = ldv<float>(p.dout.row<TI>(b, tt, hh) + pp);
      const float xv = ldv<float>(p.x.row<TI>(b, tt, hh) + pp);
      float g = go;
      if (p.z.ptr) {
        const float zz = ldv<float>(p.z.row<TI>(b, tt, hh) + pp), sg = gate_sigmoid(zz);
        g = go * zz * sg;
        const float v = ldv<float>(y + (b * p.T + tt) * HP + r) + p.D[hh] * xv;
        stv<float>(p.dz.wrow<TI>(b, tt, hh) + pp, go * v * sg * (1.f + zz * (1.f - sg)));
      }
      stv<float>(dy + (b * p.T + tt) * HP + r, g);
      acc[s] += g * xv;
    }
  }
  // per head: features h*P .. h*P+P-1 summed in feature order
#pragma unroll
  for (int s = 0; s < kSlots; ++s) {
    const int r = threadIdx.x + 256 * s;
    if (r >= HP) break;
    sacc[r] = acc[s];
  }
  __syncthreads();
  for (int hh = threadIdx.x; hh < H; hh += blockDim.x) {
    float s = 0.f;
    for (int pp = 0; pp < P; ++pp) s += sacc[hh * P + pp];
    p.pD[(b * p.nseg + seg) * H + hh] = s;
  }
}

// dx = scan dx + dxp of the next token (xp[t+1] = x[t]) + D dy, with dy = dout silu(z) as the
// epilogue backward stored it for the scan   (mamba3.py:115,119)
template <typename TI, typename TO>
__global__ void __launch_bounds__(256) m3_dx_kernel(const M3 p) {
  const int b = blockIdx.x / p.nseg, seg = blockIdx.x % p.nseg;
  const int P = (int)p.P, HP = (int)(p.H * P);
  const int64_t t0 = (int64_t)seg * kSeg;
  const int nt = (int)min((int64_t)kSeg, p.T - t0);
  const TO* __restrict__ dxs = static_cast<const TO*>(p.dxs);
  const TO* __restrict__ dxp = static_cast<const TO*>(p.dxp);
  const TO* __restrict__ dy = static_cast<const TO*>(p.dy);
#pragma unroll 4
  for (int idx = threadIdx.x; idx < nt * HP; idx += blockDim.x) {
    const int t = idx / HP, r = idx % HP, hh = r / P, pp = r % P;
    const int64_t tt = t0 + t, o = (b * p.T + tt) * HP + r;
    float g = ldv<float>(dxs + o);
    if (tt + 1 < p.T) g += ldv<float>(dxp + o + HP);
    stv<float>(p.dx.wrow<TI>(b, tt, hh) + pp, g + p.D[hh] * ldv<float>(dy + o));
  }
}

// the lane's four features of the per-head rows src [H][N], summed in head order
__device__ __forceinline__ void sum_heads(const float* src, int H, int N, Feat f, float (&du)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) du[j] = 0.f;
  if (f.on)
#pragma unroll 4
    for (int hh = 0; hh < H; ++hh) {
      float v[4];
      ldp4(src + hh * N, f, v);
#pragma unroll
      for (int j = 0; j < 4; ++j) du[j] += v[j];
    }
}

// RMSNorm backward of one token (mamba3.py:13-15), given du, the gradient of its normalised
// output summed over heads (u = x r w + bias_h for every head h): dx = r w du - x r^3 / N
// sum(du w x); dw accumulates du x r.  Lanes past the RoPE angles hold zeros, so the warp-wide sum
// sees every lane.
__device__ __forceinline__ void rms_bwd_du(const float (&du)[4], int N, const float (&xv)[4], const float (&wv)[4],
                                           float rr, float (&gw)[4], float (&gx)[4]) {
  float dl = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) dl += du[j] * wv[j] * xv[j];
  const float k3 = rr * rr * rr / N * warp_sum(dl);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    gw[j] += du[j] * xv[j] * rr;
    gx[j] = rr * wv[j] * du[j] - xv[j] * k3;
  }
}

// Per-token rows that the reverse walk needs from global memory, for all heads of the group at
// once: dq, dk, dkp of the next token (kp[t+1] = k[t]) and theta.  For one token and a run of
// consecutive heads each is one contiguous block ([B, T, H, N] layout), so one thread moves a
// token with four bulk copies (cp.async.bulk, completion on the slot's mbarrier) into a ring of
// kRing slots, kRing - 1 tokens ahead of their use.  Slot layout: dq [hc][N] | dk [hc][N] |
// dkp [hc][N] (op dtype) | theta [hc][NA] (fp32).
template <int kRing> constexpr int kRingBars = (kRing + 1) / 2 * 2;  // barriers, padded to 16 bytes

struct RowRing {
  unsigned char* base;
  uint64_t* bars;
  int slot_bytes, row_bytes;  // row_bytes: one [hc][N] block
};

template <typename TO>
__device__ __forceinline__ void ring_issue_token(const M3& p, const RowRing& R, int slot, int b, int64_t tt, int h0, int hc) {
  const int64_t bth = (b * p.T + tt) * p.H + h0;
  const bool has_next = tt + 1 < p.T;
  const uint32_t th_bytes = (uint32_t)(hc * p.NA * 4);
  const uint32_t bytes = (uint32_t)R.row_bytes * (has_next ? 3u : 2u) + th_bytes;
  unsigned char* dst = R.base + (size_t)slot * R.slot_bytes;
  uint64_t* bar = R.bars + slot;
  umma::fence_proxy_async_smem();  // the slot's previous contents were read through the generic proxy
  umma::mbar_arrive_expect_tx(bar, bytes);
  umma::bulk_load(dst, static_cast<const TO*>(p.dq) + bth * p.N, R.row_bytes, bar);
  umma::bulk_load(dst + R.row_bytes, static_cast<const TO*>(p.dk) + bth * p.N, R.row_bytes, bar);
  if (has_next) umma::bulk_load(dst + 2 * R.row_bytes, static_cast<const TO*>(p.dkp) + (bth + p.H) * p.N, R.row_bytes, bar);
  umma::bulk_load(dst + 3 * R.row_bytes, p.theta + bth * p.NA, th_bytes, bar);
}

// Reverse walk over one segment: RoPE and RMSNorm backward, bias / norm-weight partial sums,
// the within-segment suffix of the theta gradient, and the per-token sums over heads (dCm, dBm,
// the ang and DT gradients' within-segment parts) through shared memory.  Warps 0..hc-1 own a
// head each; warps hc, hc+1, hc+2 only reduce over heads (C rows, B rows, angles), one token
// behind the head warps, so the two kinds of work overlap.  Thread 0 feeds the row ring.
// kRing: ring slots (tokens in flight); kGrouped: several head groups (p.nhg > 1)
template <typename TI, typename TO, int kRing, bool kGrouped>
__global__ void __launch_bounds__(1024) m3_prologue_bwd_kernel(const M3 p) {
  extern __shared__ __align__(16) float smem[];
  const int NA = p.NA, N = (int)p.N, H = (int)p.H;
  Blk k;
  if (kGrouped) {
    k = blk(p);
  } else {  // one group: blockIdx.x = b nseg + seg
    k.b = blockIdx.x / p.nseg;
    k.seg = blockIdx.x % p.nseg;
    k.g = 0;
    k.h0 = 0;
    k.hc = H;
  }
  const int b = k.b, seg = k.seg, hc = k.hc;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, h = k.h0 + w;  // h: global head of a head warp
  const int64_t t0 = (int64_t)seg * kSeg;
  const int nt = (int)min((int64_t)kSeg, p.T - t0);
  // shared: ring slots and their mbarriers, then C rows, B rows, angles, RMSNorm factors
  // [kSeg][2], DT [kSeg][hc], then two staging buffers of (dvq, dvk: hc x N; theta-gradient
  // suffix sums: hc x (NA + 1))
  const int es = (int)sizeof(TO);
  RowRing R;
  R.row_bytes = hc * N * es;
  R.slot_bytes = 3 * R.row_bytes + hc * NA * 4;
  R.base = reinterpret_cast<unsigned char*>(smem);
  R.bars = reinterpret_cast<uint64_t*>(R.base + (size_t)kRing * R.slot_bytes);
  float* sC = reinterpret_cast<float*>(R.bars + kRingBars<kRing>);
  float* sB = sC + kSeg * N;
  float* sA = sB + kSeg * N;
  float* sR = sA + kSeg * NA;
  float* sDT = sR + 2 * kSeg;
  float* stage = sDT + kSeg * hc;
  const int NA1 = NA + 1;  // padded: lane h reads head h's row without bank conflicts
  const int buf_floats = (hc * (2 * N + NA1) + 3) & ~3;  // keeps both buffers 16-byte aligned
  int uses[kRing] = {};  // thread 0: copies issued into each slot so far
  if (threadIdx.x == 0) {  // ring barriers, then the first kRing - 1 tokens (nt-1, nt-2, ...)
    for (int i = 0; i < kRing; ++i) umma::mbar_init(R.bars + i, 1);
    umma::mbar_fence_init();
#pragma unroll
    for (int i = 0; i < kRing - 1; ++i)
      if (nt - 1 - i >= 0) {
        ring_issue_token<TO>(p, R, i, b, t0 + nt - 1 - i, k.h0, hc);
        ++uses[i];
      }
  }
  for (int idx = threadIdx.x; idx < nt * hc; idx += blockDim.x) {
    const int t = idx / hc, hh = k.h0 + idx % hc;
    sDT[idx] = softplus20(ldv<float>(p.dd_dt.row<TI>(b, t0 + t, hh)) + p.dt_bias[hh]);
  }
  stage_rows<TI>(p, b, t0, nt, sC, sB, sA, sR);  // ends with a block barrier
  const Feat f = feat(lane, NA);
  float wc[4] = {}, wb[4] = {}, cb[4] = {}, bb[4] = {};
  if (f.on) {
    ldp4(p.C_norm_w, f, wc);
    ldp4(p.B_norm_w, f, wb);
    if (w < hc) {
      ldp4(p.C_bias + h * N, f, cb);
      ldp4(p.B_bias + h * N, f, bb);
    }
  }
  const int64_t GN = (int64_t)hc * N;
  // reduction roles on the R = min(3, 32 - hc) warps after the group's heads
  const int Rw = (int)(blockDim.x >> 5) - hc;
  const bool head = w < hc;
  const bool wC = (w == hc), wB = (w == hc + (Rw >= 2 ? 1 : 0)), wA = (w == hc + (Rw >= 3 ? 2 : Rw - 1));
  // several groups: the sums over the group's heads go to global memory, m3_rms_bwd_kernel finishes
  float gcb[4] = {}, gbb[4] = {}, gwc[4] = {}, gwb[4] = {};
  float sfx = 0.f;  // theta gradient summed over this segment's tokens >= t
  bool ok = true, aborted = false;
  // head warps compute token nt-1-step at step `step`; reduction warps reduce the token staged
  // at the previous step (one extra step at the end)
  for (int step = 0; step <= nt; ++step) {
    if (threadIdx.x == 0 && step < nt) {  // keep kRing - 1 tokens in flight (the slot was freed by the last barrier)
      const int ti = nt - 1 - step - (kRing - 1);
      if (ti >= 0) {
        const int sl = (step + kRing - 1) % kRing;
        ring_issue_token<TO>(p, R, sl, b, t0 + ti, k.h0, hc);
#pragma unroll
        for (int i = 0; i < kRing; ++i) uses[i] += (i == sl);
      }
    }
    if (head && step < nt) {
      const int t = nt - 1 - step;
      ok = umma::mbar_wait(R.bars + step % kRing, (uint32_t)((step / kRing) & 1), p.status);
      const unsigned char* slot = R.base + (size_t)(step % kRing) * R.slot_bytes;
      float* buf = stage + (step & 1) * buf_floats;
      float c[4] = {}, bm[4] = {};
      const float rc = sR[2 * t], rb = sR[2 * t + 1];
      if (f.on && ok) {
        ldp4(sC + t * N, f, c);
        ldp4(sB + t * N, f, bm);
        float sn, cs;
        sincos_angle(reinterpret_cast<const float*>(slot + 3 * R.row_bytes)[w * NA + lane], &sn, &cs);
        float uq[4], oq[4], uk[4], ok4[4];
        norm_bias_rope(c, rc, wc, cb, sn, cs, uq, oq);
        norm_bias_rope(bm, rb, wb, bb, sn, cs, uk, ok4);
        float gq[4], gk[4], gkp[4] = {0.f, 0.f, 0.f, 0.f};
        ld4(reinterpret_cast<const TO*>(slot) + w * N, f, gq);
        ld4(reinterpret_cast<const TO*>(slot + R.row_bytes) + w * N, f, gk);
        if (t0 + t + 1 < p.T) ld4(reinterpret_cast<const TO*>(slot + 2 * R.row_bytes) + w * N, f, gkp);
#pragma unroll
        for (int j = 0; j < 4; ++j) gk[j] += gkp[j];
        // rope backward: rotate the gradient back; d theta from the rotated outputs
        const float dvq[4] = {gq[0] * cs + gq[1] * sn, -gq[0] * sn + gq[1] * cs, gq[2], gq[3]};
        const float dvk[4] = {gk[0] * cs + gk[1] * sn, -gk[0] * sn + gk[1] * cs, gk[2], gk[3]};
        sfx += (gq[1] * oq[0] - gq[0] * oq[1]) + (gk[1] * ok4[0] - gk[0] * ok4[1]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          gcb[j] += dvq[j];
          gbb[j] += dvk[j];
        }
        float* bq = buf + w * N;
        float* bk = buf + GN + w * N;
        *reinterpret_cast<float2*>(bq + f.f0) = make_float2(dvq[0], dvq[1]);
        *reinterpret_cast<float2*>(bq + f.f2) = make_float2(dvq[2], dvq[3]);
        *reinterpret_cast<float2*>(bk + f.f0) = make_float2(dvk[0], dvk[1]);
        *reinterpret_cast<float2*>(bk + f.f2) = make_float2(dvk[2], dvk[3]);
        buf[2 * GN + w * NA1 + lane] = sfx;
      }
    } else if (!head && step > 0) {
      // per-token sums over heads in head order, then the RMSNorm backward of Cm / Bm
      const int t = nt - step;  // the token the head warps staged at step - 1
      const float* buf = stage + ((step - 1) & 1) * buf_floats;
      const int64_t gbt = ((int64_t)k.g * p.B + b) * p.T + t0 + t;  // (group, batch, token) row
      if (wC) {
        float du[4], x4[4] = {}, gx[4];
        sum_heads(buf, hc, N, f, du);
        if (kGrouped) {
          if (f.on) st4(p.duC + gbt * N, f, du);
        } else {
          if (f.on) ldp4(sC + t * N, f, x4);
          rms_bwd_du(du, N, x4, wc, sR[2 * t], gwc, gx);
          if (f.on) st4(p.dCm.wrow<TI>(b, t0 + t, 0), f, gx, p.pairs);
        }
      }
      if (wB) {
        float du[4], x4[4] = {}, gx[4];
        sum_heads(buf + GN, hc, N, f, du);
        if (kGrouped) {
          if (f.on) st4(p.duB + gbt * N, f, du);
        } else {
          if (f.on) ldp4(sB + t * N, f, x4);
          rms_bwd_du(du, N, x4, wb, sR[2 * t + 1], gwb, gx);
          if (f.on) st4(p.dBm.wrow<TI>(b, t0 + t, 0), f, gx, p.pairs);
        }
      }
      if (wA) {
        const float* sf = buf + 2 * GN;  // [hc][NA1] theta-gradient suffix sums
        if (lane < NA) {  // ang gradient, within-segment part: sum_h DT[t][h] sfx[h][i]
          float s = 0.f;
          for (int hh = 0; hh < hc; ++hh) s += sDT[t * hc + hh] * sf[hh * NA1 + lane];
          p.dangl[gbt * NA + lane] = s;
        }
        if (lane < hc) {  // DT gradient through theta, within-segment part: sum_i sfx[h][i] ang[t][i]
          float s = 0.f;
          for (int i = 0; i < NA; ++i) s += sf[lane * NA1 + i] * sA[t * NA + i];
          p.dDTl[(b * p.T + t0 + t) * H + k.h0 + lane] = s;
        }
      }
    }
    if (__syncthreads_or(!ok)) {  // a ring wait gave up (status recorded): stop every warp
      aborted = true;
      break;
    }
  }
  if (aborted) {  // let the copies in flight land (bounded waits on each slot's last use), then leave
    if (threadIdx.x == 0)
#pragma unroll
      for (int i = 0; i < kRing; ++i)
        if (uses[i] > 0) umma::mbar_wait(R.bars + i, (uint32_t)((uses[i] - 1) & 1), p.status);
    return;
  }
  if (head && f.on) {
    p.segsum[((b * H + h) * p.nseg + seg) * NA + lane] = sfx;
    const int64_t pb = ((int64_t)(b * p.nseg + seg) * H + h) * N;
    const int64_t part1 = (int64_t)p.B * p.nseg * H * N;
    float* pB = p.pbias + pb;
    float* pC = p.pbias + part1 + pb;
    pB[f.f0] = gbb[0]; pB[f.f0 + 1] = gbb[1]; pB[f.f2] = gbb[2]; pB[f.f2 + 1] = gbb[3];
    pC[f.f0] = gcb[0]; pC[f.f0 + 1] = gcb[1]; pC[f.f2] = gcb[2]; pC[f.f2 + 1] = gcb[3];
  }
  const int64_t pn = (int64_t)(b * p.nseg + seg) * N;
  if (kGrouped) return;  // the norm-weight partials come from m3_rms_bwd_kernel
  if (wB && f.on) {
    float* o = p.pnorm + pn;
    o[f.f0] = gwb[0]; o[f.f0 + 1] = gwb[1]; o[f.f2] = gwb[2]; o[f.f2 + 1] = gwb[3];
  }
  if (wC && f.on) {
    float* o = p.pnorm + (int64_t)p.B * p.nseg * N + pn;
    o[f.f0] = gwc[0]; o[f.f0 + 1] = gwc[1]; o[f.f2] = gwc[2]; o[f.f2 + 1] = gwc[3];
  }
}

// Several head groups: the C / B row gradients summed over the groups in group order, then the
// RMSNorm backward per token (one warp per token) and the norm-weight partial sums of the segment
// (per warp, then over the warps in order).
template <typename TI>
__global__ void __launch_bounds__(256) m3_rms_bwd_kernel(const M3 p) {
  __shared__ float sw[2][8][128];  // [B, C][warp][feature]
  const int b = blockIdx.x / p.nseg, seg = blockIdx.x % p.nseg;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int N = (int)p.N, NA = p.NA;
  const int64_t t0 = (int64_t)seg * kSeg;
  const int nt = (int)min((int64_t)kSeg, p.T - t0);
  const int64_t gstride = p.B * p.T * N;
  const Feat f = feat(lane, NA);
  float wc[4] = {}, wb[4] = {};
  if (f.on) {
    ldp4(p.C_norm_w, f, wc);
    ldp4(p.B_norm_w, f, wb);
  }
  float gwc[4] = {}, gwb[4] = {};
  for (int t = w; t < nt; t += 8) {
    const int64_t tt = t0 + t, row = (b * p.T + tt) * N;
    float c4[4] = {}, b4[4] = {}, duc[4] = {}, dub[4] = {};
    if (f.on) {
      ld4(p.Cm.row<TI>(b, tt, 0), f, c4, p.pairs);
      ld4(p.Bm.row<TI>(b, tt, 0), f, b4, p.pairs);
      for (int g = 0; g < p.nhg; ++g) {
        float v[4];
        ldp4(p.duC + g * gstride + row, f, v);
#pragma unroll
        for (int j = 0; j < 4; ++j) duc[j] += v[j];
        ldp4(p.duB + g * gstride + row, f, v);
#pragma unroll
        for (int j = 0; j < 4; ++j) dub[j] += v[j];
      }
    }
    float sc = 0.f, sb = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      sc += c4[j] * c4[j];
      sb += b4[j] * b4[j];
    }
    sc = warp_sum(sc);
    sb = warp_sum(sb);
    const float rc = rsqrtf(sc / N + p.eps), rb = rsqrtf(sb / N + p.eps);
    float gx[4];
    rms_bwd_du(duc, N, c4, wc, rc, gwc, gx);
    if (f.on) st4(p.dCm.wrow<TI>(b, tt, 0), f, gx, p.pairs);
    rms_bwd_du(dub, N, b4, wb, rb, gwb, gx);
    if (f.on) st4(p.dBm.wrow<TI>(b, tt, 0), f, gx, p.pairs);
  }
  if (f.on) {
    st4(&sw[0][w][0], f, gwb);
    st4(&sw[1][w][0], f, gwc);
  }
  __syncthreads();
  const int64_t pn = (int64_t)(b * p.nseg + seg) * N;
  for (int i = threadIdx.x; i < 2 * N; i += blockDim.x) {
    const int part = i / N, n = i % N;
    float s = 0.f;
    for (int k = 0; k < 8; ++k) s += sw[part][k][n];
    p.pnorm[part * p.B * p.nseg * N + pn + n] = s;
  }
}

// The theta-gradient carry from later segments, then the discretisation backward per (token,
// head) (mamba3.py:105-111) and the ang gradient.  Thread tid keeps head tid % H (blockDim is a
// multiple of H), so its dt_bias partial sum has a fixed head.
template <typename TI>
__global__ void __launch_bounds__(1024) m3_scalars_bwd_kernel(const M3 p) {
  extern __shared__ float smem[];  // sA [kSeg][NA] | sC [H][NA + 1] | sDT [kSeg][H] | sacc [blockDim]
  const int b = blockIdx.x / p.nseg, seg = blockIdx.x % p.nseg;
  const int NA = p.NA, H = (int)p.H;
  const int64_t t0 = (int64_t)seg * kSeg;
  const int nt = (int)min((int64_t)kSeg, p.T - t0);
  const int NA1 = NA + 1;  // padded rows: the (token, head) walk below reads them without bank conflicts
  float* sA = smem;
  float* sC = sA + kSeg * NA;
  float* sDT = sC + H * NA1;
  float* sacc = sDT + kSeg * H;
  for (int idx = threadIdx.x; idx < H * NA; idx += blockDim.x) {  // theta gradient over all later segments
    const int hh = idx / NA, i = idx % NA;
    const float* __restrict__ src = p.segsum + (int64_t)(b * H + hh) * p.nseg * NA + i;
    float C = 0.f;
#pragma unroll 8
    for (int s = seg + 1; s < p.nseg; ++s) C += __ldg(src + (int64_t)s * NA);
    sC[hh * NA1 + i] = C;
  }
  for (int idx = threadIdx.x; idx < nt * NA; idx += blockDim.x)
    sA[idx] = ldv<float>(p.ang.row<TI>(b, t0 + idx / NA, 0) + idx % NA);
  __syncthreads();
  float acc_dt = 0.f;
  for (int idx = threadIdx.x; idx < nt * H; idx += blockDim.x) {
    const int t = idx / H, hh = idx % H;
    const int64_t tt = t0 + t, bth = (b * p.T + tt) * H + hh;
    const float ddA = ldv<float>(p.dd_A.row<TI>(b, tt, hh));
    const Disc d = discretise(ldv<float>(p.dd_dt.row<TI>(b, tt, hh)), ddA, ldv<float>(p.trap.row<TI>(b, tt, hh)),
                              p.dt_bias[hh], p.A_floor);
    float carry = 0.f;
    for (int i = 0; i < NA; ++i) carry += sC[hh * NA1 + i] * sA[t * NA + i];
    sDT[t * H + hh] = d.DT;
    const float ga = p.dadt[bth], gg = p.dgamma[bth], gb = p.dbeta[bth];
    const float g_adt = ga + gb * d.beta;  // beta = (1 - tr) DT e^{adt}
    const float g_DT = g_adt * d.A + gg * d.tr + gb * (1.f - d.tr) * d.ea + p.dDTl[bth] + carry;
    const float g_A = g_adt * d.DT;
    const float g_tr = gg * d.DT - gb * d.DT * d.ea;
    const float g_xs = g_DT * (d.xs > 20.f ? 1.f : sigmoidf_(d.xs));  // softplus'
    // clamp(max=-A_floor) passes the gradient where heavy_tail <= -A_floor; heavy_tail's two
    // clamps pass it at x >= 0 and x <= 0 respectively (torch.clamp's masks)
    const float dht = (ddA >= 0.f ? 1.f : 0.f) + (ddA <= 0.f ? 1.f / ((1.f - ddA) * (1.f - ddA)) : 0.f);
    const float g_ddA = d.ht <= -p.A_floor ? -g_A * dht : 0.f;
    stv<float>(p.ddd_dt.wrow<TI>(b, tt, hh), g_xs);
    stv<float>(p.ddd_A.wrow<TI>(b, tt, hh), g_ddA);
    stv<float>(p.dtrap.wrow<TI>(b, tt, hh), g_tr * d.tr * (1.f - d.tr));
    acc_dt += g_xs;
  }
  sacc[threadIdx.x] = acc_dt;
  __syncthreads();
  for (int hh = threadIdx.x; hh < H; hh += blockDim.x) {  // dt_bias partial: threads of head hh in order
    float s = 0.f;
    for (int k = hh; k < (int)blockDim.x; k += H) s += sacc[k];
    p.pdt[(b * p.nseg + seg) * H + hh] = s;
  }
  // ang gradient: the within-segment part (per head group) plus sum_h DT[t][h] * carry[h][i]
  const int64_t gstride = p.B * p.T * NA;
  for (int idx = threadIdx.x; idx < nt * NA; idx += blockDim.x) {
    const int t = idx / NA, i = idx % NA;
    float s = p.dangl[(b * p.T + t0 + t) * NA + i];
    for (int g = 1; g < p.nhg; ++g) s += p.dangl[g * gstride + (b * p.T + t0 + t) * NA + i];
    for (int hh = 0; hh < H; ++hh) s += sDT[t * H + hh] * sC[hh * NA1 + i];
    stv<float>(p.dang.wrow<TI>(b, t0 + t, 0) + i, s);
  }
}

// ---------------------------------------------------------------------------------------------
// elementwise kernels, 16-byte vectors: blockDim = slots x groups, slots = H P / 8 (head,
// 8-feature slot) and up to 4 groups; group g walks the segment's tokens g, g + groups, ...
// (P % 8 == 0 and 16-byte-aligned views; the kernels above are the fallback)

template <typename TI, typename TO>
__global__ void __launch_bounds__(1024) m3_epilogue_fwd_vec_kernel(const M3 p) {
  const int b = blockIdx.x / p.nseg, seg = blockIdx.x % p.nseg;
  const int P = (int)p.P, P8 = P / 8, HP = (int)p.H * P;
  const int slots = (int)p.H * P8, grp = threadIdx.x / slots, ngrp = blockDim.x / slots, sl = threadIdx.x % slots;
  const int hh = sl / P8, pp = (sl % P8) * 8, r = hh * P + pp;
  const int64_t t0 = (int64_t)seg * kSeg;
  const int nt = (int)min((int64_t)kSeg, p.T - t0);
  const float Dh = p.D[hh];
  const TO* __restrict__ y = static_cast<const TO*>(p.y) + (int64_t)b * p.T * HP + r;
  // two tokens per pass, all loads before either store (as in m3_dx_vec_kernel)
  for (int t = grp; t < nt; t += 2 * ngrp) {
    Pack8<TO> yv[2];
    Pack8<TI> xv[2], zv[2];
    bool on[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int64_t tt = t0 + t + u * ngrp;
      on[u] = t + u * ngrp < nt;
      if (on[u]) {
        yv[u].ld(y + tt * HP);
        xv[u].ld(p.x.row<TI>(b, tt, hh) + pp);
        if (p.z.ptr) zv[u].ld(p.z.row<TI>(b, tt, hh) + pp);
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (!on[u]) continue;
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        o[e] = yv[u].get(e) + Dh * xv[u].get(e);
        if (p.z.ptr) {
          const float zz = zv[u].get(e);
          o[e] *= zz * gate_sigmoid(zz);
        }
      }
      Vec8<TI>::st(p.out.wrow<TI>(b, t0 + t + u * ngrp, hh) + pp, o);
    }
  }
}

template <typename TI, typename TO>
__global__ void __launch_bounds__(1024) m3_epilogue_bwd_vec_kernel(const M3 p) {
  extern __shared__ float sacc[];  // [H * P / 8] per-slot sums
  const int b = blockIdx.x / p.nseg, seg = blockIdx.x % p.nseg;
  const int P = (int)p.P, P8 = P / 8, H = (int)p.H, HP = H * P;
  const int slots = (int)p.H * P8, grp = threadIdx.x / slots, ngrp = blockDim.x / slots, sl = threadIdx.x % slots;
  const int hh = sl / P8, pp = (sl % P8) * 8, r = hh * P + pp;
  const int64_t t0 = (int64_t)seg * kSeg;
  const int nt = (int)min((int64_t)kSeg, p.T - t0);
  const float Dh = p.D[hh];
  const TO* __restrict__ y = static_cast<const TO*>(p.y) + (int64_t)b * p.T * HP + r;
  TO* __restrict__ dy = static_cast<TO*>(p.dy) + (int64_t)b * p.T * HP + r;
  float acc = 0.f;
  // two tokens per pass, all loads before any store (as in m3_dx_vec_kernel)
  for (int t = grp; t < nt; t += 2 * ngrp) {
    Pack8<TI> go[2], xv[2], zv[2];
    Pack8<TO> yv[2];
    bool on[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int64_t tt = t0 + t + u * ngrp;
      on[u] = t + u * ngrp < nt;
      if (on[u]) {
        go[u].ld(p.dout.row<TI>(b, tt, hh) + pp);
        xv[u].ld(p.x.row<TI>(b, tt, hh) + pp);
        if (p.z.ptr) {
          zv[u].ld(p.z.row<TI>(b, tt, hh) + pp);
          yv[u].ld(y + tt * HP);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (!on[u]) continue;
      const int64_t tt = t0 + t + u * ngrp;
      float g[8];
      if (p.z.ptr) {
        float dz[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float zz = zv[u].get(e), o = go[u].get(e), sg = gate_sigmoid(zz);
          g[e] = o * zz * sg;
          dz[e] = o * (yv[u].get(e) + Dh * xv[u].get(e)) * sg * (1.f + zz * (1.f - sg));
        }
        Vec8<TI>::st(p.dz.wrow<TI>(b, tt, hh) + pp, dz);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) g[e] = go[u].get(e);
      }
      Vec8<TO>::st(dy + tt * HP, g);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc += g[e] * xv[u].get(e);
    }
  }
  sacc[threadIdx.x] = acc;
  __syncthreads();
  for (int h2 = threadIdx.x; h2 < H; h2 += blockDim.x) {  // per head: groups, then slots in feature order
    float s = 0.f;
    for (int g = 0; g < ngrp; ++g)
      for (int k = 0; k < P8; ++k) s += sacc[g * slots + h2 * P8 + k];
    p.pD[(b * p.nseg + seg) * H + h2] = s;
  }
}

template <typename TI, typename TO>
__global__ void __launch_bounds__(1024) m3_dx_vec_kernel(const M3 p) {
  const int b = blockIdx.x / p.nseg, seg = blockIdx.x % p.nseg;
  const int P = (int)p.P, P8 = P / 8, HP = (int)p.H * P;
  const int slots = (int)p.H * P8, grp = threadIdx.x / slots, ngrp = blockDim.x / slots, sl = threadIdx.x % slots;
  const int hh = sl / P8, pp = (sl % P8) * 8, r = hh * P + pp;
  const int64_t t0 = (int64_t)seg * kSeg;
  const int nt = (int)min((int64_t)kSeg, p.T - t0);
  const float Dh = p.D[hh];
  const TO* __restrict__ dxs = static_cast<const TO*>(p.dxs) + (int64_t)b * p.T * HP + r;
  const TO* __restrict__ dxp = static_cast<const TO*>(p.dxp) + (int64_t)b * p.T * HP + r;
  const TO* __restrict__ dy = static_cast<const TO*>(p.dy) + (int64_t)b * p.T * HP + r;
  // two tokens per pass, all their loads issued before either store (the store through a view may
  // alias the loads as far as the compiler knows, so it would not hoist them itself)
  for (int t = grp; t < nt; t += 2 * ngrp) {
    Pack8<TO> ga[2], gy[2], gp[2];  // dout silu(z) is dy, as stored for the scan
    bool on[2], nx[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int64_t tt = t0 + t + u * ngrp;
      on[u] = t + u * ngrp < nt;
      nx[u] = on[u] && tt + 1 < p.T;  // xp[t+1] = x[t]
      if (on[u]) {
        ga[u].ld(dxs + tt * HP);
        gy[u].ld(dy + tt * HP);
      }
      if (nx[u]) gp[u].ld(dxp + (tt + 1) * HP);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (!on[u]) continue;
      float g[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) g[e] = ga[u].get(e) + (nx[u] ? gp[u].get(e) : 0.f) + Dh * gy[u].get(e);
      Vec8<TI>::st(p.dx.wrow<TI>(b, t0 + t + u * ngrp, hh) + pp, g);
    }
  }
}

// parameter gradients: fixed-order sums of the per-(batch, segment) partials.  One warp lane per
// output over 32 consecutive outputs, the partials split over the 8 warps of the CTA (coalesced
// rows), then the warps' sums in order.
__global__ void __launch_bounds__(256) m3_param_reduce_kernel(const M3 p) {
  __shared__ float sm[8][33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t H = p.H, N = p.N, BS = p.B * p.nseg;
  const int64_t n_bias = H * N;
  const int64_t total = 2 * n_bias + 2 * N + 2 * H;
  const int64_t i = (int64_t)blockIdx.x * 32 + lane;
  const float* src = nullptr;
  int64_t stride = 0;
  float* dst = nullptr;
  if (i < 2 * n_bias) {  // B_bias then C_bias
    const int64_t part = i / n_bias, j = i % n_bias;
    src = p.pbias + part * BS * n_bias + j;
    stride = n_bias;
    dst = (part ? p.dC_bias : p.dB_bias) + j;
  } else if (i < 2 * n_bias + 2 * N) {  // B_norm_w then C_norm_w
    const int64_t r = i - 2 * n_bias, part = r / N, j = r % N;
    src = p.pnorm + part * BS * N + j;
    stride = N;
    dst = (part ? p.dC_norm_w : p.dB_norm_w) + j;
  } else if (i < total) {  // dt_bias then D
    const int64_t r = i - 2 * n_bias - 2 * N, part = r / H, j = r % H;
    src = (part ? p.pD : p.pdt) + j;
    stride = H;
    dst = (part ? p.dD : p.ddt_bias) + j;
  }
  float s = 0.f;
  if (src)
    for (int64_t k = warp; k < BS; k += 8) s += src[k * stride];
  sm[warp][lane] = s;
  __syncthreads();
  if (warp == 0 && dst) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += sm[k][lane];
    *dst = t;
  }
}

// ---------------------------------------------------------------------------------------------
// host

View view_of(const zb_view& v) { return View{v.ptr, v.sb, v.st, v.sh}; }

// head groups: up to 31 heads in one group; more heads split evenly into groups of at most 28
void head_groups(int64_t H, int* hg, int* nhg) {
  *nhg = H <= 31 ? 1 : (int)((H + 27) / 28);
  *hg = (int)((H + *nhg - 1) / *nhg);
}

struct WsLayout {
  size_t segsum, dDTl, dangl, duC, duB, pbias, pnorm, pdt, pD, total;
};
WsLayout ws_layout(const zb_m3_args* a) {
  const int64_t nseg = (a->T + kSeg - 1) / kSeg, NA = a->N / 4;
  int hg, nhg;
  head_groups(a->H, &hg, &nhg);
  const size_t ng = nhg > 1 ? (size_t)nhg : 0;
  WsLayout L;
  size_t off = 0;
  auto take = [&](size_t floats) {
    const size_t o = off;
    off = align_up(off + floats * sizeof(float), 256);
    return o;
  };
  L.segsum = take((size_t)a->B * a->H * nseg * NA);
  L.dDTl = take((size_t)a->B * a->T * a->H);
  L.dangl = take((size_t)nhg * a->B * a->T * NA);
  L.duC = take(ng * a->B * a->T * a->N);
  L.duB = take(ng * a->B * a->T * a->N);
  L.pbias = take((size_t)2 * a->B * nseg * a->H * a->N);
  L.pnorm = take((size_t)2 * a->B * nseg * a->N);
  L.pdt = take((size_t)a->B * nseg * a->H);
  L.pD = take((size_t)a->B * nseg * a->H);
  L.total = off;
  return L;
}

int check(const zb_m3_args* a) {
  if (!a) return ZB_ERR_LAYOUT;
  if (a->B <= 0 || a->T <= 0 || a->H <= 0 || a->P <= 0 || a->N <= 0) return ZB_ERR_SHAPE;
  if (a->H > 128 || a->H * a->P > 8192 || a->N % 16 != 0 || a->N > 128 || a->P > 256) return ZB_ERR_UNSUPPORTED;
  if ((double)a->B * (double)(a->T + 1) * (double)a->H * (double)(a->N > a->P ? a->N : a->P) > 9.0e15)
    return ZB_ERR_SHAPE;
  if ((a->io_dtype != ZB_F32 && a->io_dtype != ZB_BF16) || (a->op_dtype != ZB_F32 && a->op_dtype != ZB_BF16))
    return ZB_ERR_DTYPE;
  if (!a->x.ptr || !a->dt_bias || !a->B_bias || !a->C_bias || !a->B_norm_w || !a->C_norm_w || !a->D)
    return ZB_ERR_LAYOUT;
  if (!a->workspace || a->workspace_bytes < ws_layout(a).total || (reinterpret_cast<uintptr_t>(a->workspace) & 255))
    return ZB_ERR_WORKSPACE;
  const void* contiguous[] = {a->q, a->k_ext, a->xp, a->theta, a->y, a->dy, a->dxs, a->dxp, a->dq, a->dk, a->dkp};
  for (const void* c : contiguous)
    if (reinterpret_cast<uintptr_t>(c) & 15) return ZB_ERR_LAYOUT;
  return ZB_OK;
}

// a view allows aligned accesses of `elems` elements: base and (b, t, h) strides all multiples
bool view_aligned(const zb_view& v, int64_t elems, size_t esize) {
  if (!v.ptr) return true;
  const uint64_t bytes = (uint64_t)elems * esize;
  return reinterpret_cast<uintptr_t>(v.ptr) % bytes == 0 && (v.sb * (int64_t)esize) % bytes == 0 &&
         (v.st * (int64_t)esize) % bytes == 0 && (v.sh * (int64_t)esize) % bytes == 0;
}

M3 make_m3(const zb_m3_args* a) {
  M3 p;
  memset(&p, 0, sizeof(p));
  const size_t es = a->io_dtype == ZB_F32 ? 4 : 2;
  p.pairs = view_aligned(a->Bm, 2, es) && view_aligned(a->Cm, 2, es) && view_aligned(a->dBm, 2, es) &&
            view_aligned(a->dCm, 2, es);
  p.rows8 = a->N % 8 == 0 && view_aligned(a->Bm, 8, es) && view_aligned(a->Cm, 8, es);
  p.vec8 = a->P % 8 == 0 && view_aligned(a->x, 8, es) && view_aligned(a->z, 8, es) && view_aligned(a->out, 8, es) &&
           view_aligned(a->dout, 8, es) && view_aligned(a->dx, 8, es) && view_aligned(a->dz, 8, es);
  p.B = a->B; p.T = a->T; p.H = a->H; p.P = a->P; p.N = a->N;
  p.NA = (int)(a->N / 4);
  p.nseg = (int)((a->T + kSeg - 1) / kSeg);
  head_groups(a->H, &p.hg, &p.nhg);
  p.A_floor = a->A_floor; p.eps = a->eps;
  p.x = view_of(a->x); p.z = view_of(a->z); p.Bm = view_of(a->Bm); p.Cm = view_of(a->Cm);
  p.dd_dt = view_of(a->dd_dt); p.dd_A = view_of(a->dd_A); p.trap = view_of(a->trap); p.ang = view_of(a->ang);
  p.dt_bias = a->dt_bias; p.B_bias = a->B_bias; p.C_bias = a->C_bias;
  p.B_norm_w = a->B_norm_w; p.C_norm_w = a->C_norm_w; p.D = a->D;
  p.q = a->q; p.k_ext = a->k_ext; p.xp = a->xp;
  p.adt = a->adt; p.gamma = a->gamma; p.beta = a->beta; p.theta = a->theta;
  p.y = a->y; p.out = view_of(a->out); p.dout = view_of(a->dout); p.dy = a->dy;
  p.dxs = a->dxs; p.dxp = a->dxp; p.dq = a->dq; p.dk = a->dk; p.dkp = a->dkp;
  p.dadt = a->dadt; p.dgamma = a->dgamma; p.dbeta = a->dbeta;
  p.dx = view_of(a->dx); p.dz = view_of(a->dz); p.dBm = view_of(a->dBm); p.dCm = view_of(a->dCm);
  p.ddd_dt = view_of(a->ddd_dt); p.ddd_A = view_of(a->ddd_A); p.dtrap = view_of(a->dtrap); p.dang = view_of(a->dang);
  p.ddt_bias = a->ddt_bias; p.dB_bias = a->dB_bias; p.dC_bias = a->dC_bias;
  p.dB_norm_w = a->dB_norm_w; p.dC_norm_w = a->dC_norm_w; p.dD = a->dD;
  p.status = a->status;
  p.theta0 = a->theta0;
  p.kp0 = a->kp0;
  const WsLayout L = ws_layout(a);
  unsigned char* ws = static_cast<unsigned char*>(a->workspace);
  p.segsum = reinterpret_cast<float*>(ws + L.segsum);
  p.dDTl = reinterpret_cast<float*>(ws + L.dDTl);
  p.dangl = reinterpret_cast<float*>(ws + L.dangl);
  p.duC = reinterpret_cast<float*>(ws + L.duC);
  p.duB = reinterpret_cast<float*>(ws + L.duB);
  p.pbias = reinterpret_cast<float*>(ws + L.pbias);
  p.pnorm = reinterpret_cast<float*>(ws + L.pnorm);
  p.pdt = reinterpret_cast<float*>(ws + L.pdt);
  p.pD = reinterpret_cast<float*>(ws + L.pD);
  return p;
}

// dispatch a (io type, op type) kernel template on the argument dtypes
#define ZB_M3_DISPATCH(IO, OP, ...)                                                                    \
  do {                                                                                                 \
    if ((IO) == ZB_F32 && (OP) == ZB_F32) { using TI = float; using TO = float; __VA_ARGS__ }           \
    else if ((IO) == ZB_F32) { using TI = float; using TO = __nv_bfloat16; __VA_ARGS__ }                \
    else if ((OP) == ZB_F32) { using TI = __nv_bfloat16; using TO = float; __VA_ARGS__ }                \
    else { using TI = __nv_bfloat16; using TO = __nv_bfloat16; __VA_ARGS__ }                            \
  } while (0)

int finish(int n_launches) {
  note_launches(n_launches);
  return cudaPeekAtLastError() == cudaSuccess ? ZB_OK : ZB_ERR_CUDA;
}

}  // namespace
}  // namespace zb

using namespace zb;

extern "C" ZB_API uint64_t zb_m3_workspace_bytes(const zb_m3_args* a) { return a ? ws_layout(a).total : 0; }

extern "C" ZB_API int zb_m3_prologue_fwd(const zb_m3_args* a, void* stream) {
  int rc = check(a);
  if (rc) return rc;
  if (!a->q || !a->k_ext || !a->adt || !a->gamma || !a->beta || !a->theta || !a->Bm.ptr || !a->Cm.ptr ||
      !a->dd_dt.ptr || !a->dd_A.ptr || !a->trap.ptr || !a->ang.ptr)
    return ZB_ERR_LAYOUT;
  const M3 p = make_m3(a);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)(p.B * p.nseg * p.nhg)), block((unsigned)(32 * p.hg));
  const int smem0 = (int)(kSeg * (p.NA + p.hg) * sizeof(float));
  const int smem1 = (int)(kSeg * (2 * p.N + p.NA + p.hg) * sizeof(float));
  ZB_M3_DISPATCH(a->io_dtype, a->op_dtype, {
    auto k1 = m3_prologue_fwd_kernel<TI, TO>;
    if (dyn_smem(reinterpret_cast<const void*>(k1), smem1) != ZB_OK) return ZB_ERR_CUDA;
    m3_segsum_kernel<TI><<<grid, block, smem0, s>>>(p);
    k1<<<grid, block, smem1, s>>>(p);
  });
  return finish(2);
}

extern "C" ZB_API int zb_m3_epilogue_fwd(const zb_m3_args* a, void* stream) {
  int rc = check(a);
  if (rc) return rc;
  if (!a->y || !a->out.ptr) return ZB_ERR_LAYOUT;
  const M3 p = make_m3(a);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)(p.B * p.nseg));
  const unsigned slots = (unsigned)(p.H * p.P / 8), vthreads = slots * (slots >= 256 ? 1024 / slots : 4);
  ZB_M3_DISPATCH(a->io_dtype, a->op_dtype, {
    if (p.vec8) m3_epilogue_fwd_vec_kernel<TI, TO><<<grid, vthreads, 0, s>>>(p);
    else m3_epilogue_fwd_kernel<TI, TO><<<grid, 256, 0, s>>>(p);
  });
  return finish(1);
}

extern "C" ZB_API int zb_m3_epilogue_bwd(const zb_m3_args* a, void* stream) {
  int rc = check(a);
  if (rc) return rc;
  if (!a->y || !a->dout.ptr || !a->dy || (a->z.ptr && !a->dz.ptr)) return ZB_ERR_LAYOUT;
  const M3 p = make_m3(a);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)(p.B * p.nseg));
  const int smem = (int)(p.H * p.P * sizeof(float));
  const unsigned slots = (unsigned)(p.H * p.P / 8), vthreads = slots * (slots >= 256 ? 1024 / slots : 4);
  ZB_M3_DISPATCH(a->io_dtype, a->op_dtype, {
    if (p.vec8) m3_epilogue_bwd_vec_kernel<TI, TO><<<grid, vthreads, vthreads * sizeof(float), s>>>(p);
    else m3_epilogue_bwd_kernel<TI, TO><<<grid, 256, smem, s>>>(p);
  });
  return finish(1);
}

extern "C" ZB_API int zb_m3_prologue_bwd(const zb_m3_args* a, void* stream) {
  int rc = check(a);
  if (rc) return rc;
  if (!a->theta || !a->dout.ptr || !a->dy || !a->dxs || !a->dxp || !a->dq || !a->dk || !a->dkp || !a->dadt || !a->dgamma ||
      !a->dbeta || !a->dx.ptr || !a->dBm.ptr || !a->dCm.ptr || !a->ddd_dt.ptr || !a->ddd_A.ptr || !a->dtrap.ptr ||
      !a->dang.ptr || !a->ddt_bias || !a->dB_bias || !a->dC_bias || !a->dB_norm_w || !a->dC_norm_w || !a->dD ||
      !a->status)
    return ZB_ERR_LAYOUT;
  const M3 p = make_m3(a);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)(p.B * p.nseg)), ggrid((unsigned)(p.B * p.nseg * p.nhg));
  // staged rows (C, B: N each; angles; RMSNorm factors; DT per group head) for kSeg tokens, then
  // two staging buffers of (dvq, dvk: hg x N; DT * theta-gradient: hg x NA)
  // plus the per-warp row rings: as many slots (4, 2 or 1) as shared memory allows
  // ring slots: as many (4, 2 or 1) as shared memory allows
  const int op_es = a->op_dtype == ZB_F32 ? 4 : 2;
  const size_t buf_floats = (p.hg * (2 * p.N + p.NA + 1) + 3) & ~(size_t)3;
  const size_t base1 = (kSeg * (2 * p.N + p.NA + 2 + p.hg) + 2 * buf_floats) * sizeof(float);
  const size_t ring1 = (size_t)p.hg * (3 * p.N * op_es + p.NA * 4);
  const size_t kMaxSmem = 227 * 1024;
  auto need = [&](int r) { return base1 + r * ring1 + 8 * ((r + 1) / 2 * 2); };
  const int ring = need(4) <= kMaxSmem ? 4 : need(2) <= kMaxSmem ? 2 : 1;
  const int smem1 = (int)need(ring);
  if ((size_t)smem1 > kMaxSmem) return ZB_ERR_UNSUPPORTED;
  // scalars kernel: thread tid keeps head tid % H, so blockDim is a multiple of H
  const int sthreads = (int)(p.H * (p.H <= 32 ? 32 : 1024 / p.H));
  const int smem2 = (int)((kSeg * p.NA + p.H * (p.NA + 1) + kSeg * p.H + sthreads) * sizeof(float));
  ZB_M3_DISPATCH(a->io_dtype, a->op_dtype, {
    auto k1 = p.nhg > 1 ? (ring == 4   ? m3_prologue_bwd_kernel<TI, TO, 4, true>
                           : ring == 2 ? m3_prologue_bwd_kernel<TI, TO, 2, true>
                                       : m3_prologue_bwd_kernel<TI, TO, 1, true>)
                        : (ring == 4   ? m3_prologue_bwd_kernel<TI, TO, 4, false>
                           : ring == 2 ? m3_prologue_bwd_kernel<TI, TO, 2, false>
                                       : m3_prologue_bwd_kernel<TI, TO, 1, false>);
    if (dyn_smem(reinterpret_cast<const void*>(k1), smem1) != ZB_OK) return ZB_ERR_CUDA;
    if (p.vec8) {
      const unsigned slots = (unsigned)(p.H * p.P / 8), vthreads = slots * (slots >= 256 ? 1024 / slots : 4);
      m3_dx_vec_kernel<TI, TO><<<grid, vthreads, 0, s>>>(p);
    }
    else m3_dx_kernel<TI, TO><<<grid, 256, 0, s>>>(p);
    k1<<<ggrid, (unsigned)(32 * (p.hg + (p.hg <= 29 ? 3 : 32 - p.hg))), smem1, s>>>(p);  // heads + reduction warps
    if (p.nhg > 1) m3_rms_bwd_kernel<TI><<<grid, 256, 0, s>>>(p);
    m3_scalars_bwd_kernel<TI><<<grid, (unsigned)sthreads, smem2, s>>>(p);
  });
  const int64_t n_params = 2 * p.H * p.N + 2 * p.N + 2 * p.H;
  m3_param_reduce_kernel<<<(unsigned)((n_params + 31) / 32), 256, 0, s>>>(p);
  return finish(p.nhg > 1 ? 5 : 4);
}
