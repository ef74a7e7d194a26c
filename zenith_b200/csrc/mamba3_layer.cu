// Mamba-3 layer body around the SSD scan (zenith/mamba3.py:96-119), forward and backward:
// the prologue that turns the in_proj split into the scan operands (discretisation, RMSNorm,
// RoPE, one-token shift) and the epilogue (D skip, silu gate).
//
// One CTA per (batch, 64-token segment), one warp per head (H <= 32).  Per-token RMSNorm and
// RoPE run lane-parallel over the state features: lane i owns RoPE pair i (features 2i, 2i+1)
// and the pass-through pair (2A+2i, 2A+2i+1), A = N/4 angles.  theta = cumsum_t(DT ang) spans
// the whole sequence; it crosses segments through per-segment sums (forward) and per-segment
// totals of its gradient (backward).  Reductions over heads and over (batch, token) run in a
// fixed order, so results are bitwise reproducible.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"
#include "ssd_kernels.h"
#include "zb_mamba3.h"

namespace zb {
namespace {

constexpr int kSeg = 64;  // tokens per segment
// row kernels run one warp per head, up to 32 heads: 1024 threads, at most 64 registers each

struct M3 {
  int64_t B, T, H, P, N;
  int NA, nseg;
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
  // scratch
  float* segsum;  // [B][H][nseg][NA]   theta segment sums (forward) / theta-gradient segment totals (backward)
  float* dDTl;    // [B][T][H]          backward: DT gradient through theta, within-segment part
  float* dangl;   // [B][T][NA]         backward: ang gradient, within-segment part
  float* pbias;   // [2][B][nseg][H][N] backward: B_bias, C_bias partial sums
  float* pnorm;   // [2][B][nseg][N]    backward: B_norm_w, C_norm_w partial sums
  float* pdt;     // [B][nseg][H]       backward: dt_bias partial sums
  float* pD;      // [B][nseg][H]       backward: D partial sums
};

// ---------------------------------------------------------------------------------------------
// per-token discretisation (mamba3.py:105-110)

__device__ __forceinline__ float softplus20(float v) { return v > 20.f ? v : log1pf(expf(v)); }
__device__ __forceinline__ float sigmoidf_(float v) { return 1.f / (1.f + expf(-v)); }

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

template <typename T> __device__ __forceinline__ void ld4(const T* row, Feat f, float (&v)[4]) {
  v[0] = ldv<float>(row + f.f0);
  v[1] = ldv<float>(row + f.f0 + 1);
  v[2] = ldv<float>(row + f.f2);
  v[3] = ldv<float>(row + f.f2 + 1);
}
template <typename T> __device__ __forceinline__ void st4(T* row, Feat f, const float (&v)[4]) {
  stv<float>(row + f.f0, v[0]);
  stv<float>(row + f.f0 + 1, v[1]);
  stv<float>(row + f.f2, v[2]);
  stv<float>(row + f.f2 + 1, v[3]);
}
__device__ __forceinline__ void ldp4(const float* row, Feat f, float (&v)[4]) {
  v[0] = row[f.f0];
  v[1] = row[f.f0 + 1];
  v[2] = row[f.f2];
  v[3] = row[f.f2 + 1];
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

// ---------------------------------------------------------------------------------------------
// forward

// theta segment sums: segsum[b][h][seg][i] = sum over the segment's tokens of DT * ang_i
template <typename TI>
__global__ void __launch_bounds__(1024) m3_segsum_kernel(const M3 p) {
  const int b = blockIdx.x / p.nseg, seg = blockIdx.x % p.nseg;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t0 = (int64_t)seg * kSeg, t1 = min(p.T, t0 + kSeg);
  const float dtb = p.dt_bias[h];
  float acc = 0.f;
  for (int64_t t = t0; t < t1; ++t) {
    const float DT = softplus20(ldv<float>(p.dd_dt.row<TI>(b, t, h)) + dtb);
    if (lane < p.NA) acc += DT * ldv<float>(p.ang.row<TI>(b, t, 0) + lane);
  }
  if (lane < p.NA) p.segsum[((b * p.H + h) * p.nseg + seg) * p.NA + lane] = acc;
}

// q, k (into k_ext rows t+1), xp, adt, gamma, beta and theta for one segment of one batch
template <typename TI, typename TO>
__global__ void __launch_bounds__(1024) m3_prologue_fwd_kernel(const M3 p) {
  const int b = blockIdx.x / p.nseg, seg = blockIdx.x % p.nseg;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NA = p.NA, N = (int)p.N, P = (int)p.P, H = (int)p.H;
  const Feat f = feat(lane, NA);
  float th = 0.f;  // theta at the end of the previous segment
  if (f.on)
    for (int s = 0; s < seg; ++s) th += p.segsum[((b * H + h) * p.nseg + s) * NA + lane];
  float wc[4] = {}, wb[4] = {}, cb[4] = {}, bb[4] = {};
  if (f.on) {
    ldp4(p.C_norm_w, f, wc);
    ldp4(p.B_norm_w, f, wb);
    ldp4(p.C_bias + h * N, f, cb);
    ldp4(p.B_bias + h * N, f, bb);
  }
  const float dtb = p.dt_bias[h];
  const int64_t t0 = (int64_t)seg * kSeg, t1 = min(p.T, t0 + kSeg);
  TO* q = static_cast<TO*>(p.q);
  TO* kx = static_cast<TO*>(p.k_ext);
  TO* xp = static_cast<TO*>(p.xp);
  const int64_t HN = (int64_t)H * N, HP = (int64_t)H * P;
  if (seg == 0 && f.on) {  // k_ext row 0 = kp of token 0 = 0
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
    st4(kx + (int64_t)b * (p.T + 1) * HN + h * N, f, zero);
  }
  for (int64_t t = t0; t < t1; ++t) {
    const Disc d = discretise(ldv<float>(p.dd_dt.row<TI>(b, t, h)), ldv<float>(p.dd_A.row<TI>(b, t, h)),
                              ldv<float>(p.trap.row<TI>(b, t, h)), dtb, p.A_floor);
    const int64_t bth = (b * p.T + t) * H + h;
    if (lane == 0) {
      p.adt[bth] = d.adt;
      p.gamma[bth] = d.gamma;
      p.beta[bth] = d.beta;
    }
    float c[4] = {}, bm[4] = {};
    if (f.on) {
      th += d.DT * ldv<float>(p.ang.row<TI>(b, t, 0) + lane);  // theta = cumsum_t(DT ang) (mamba3.py:111)
      p.theta[bth * NA + lane] = th;
      ld4(p.Cm.row<TI>(b, t, 0), f, c);
      ld4(p.Bm.row<TI>(b, t, 0), f, bm);
    }
    const float sc = warp_sum(c[0] * c[0] + c[1] * c[1] + c[2] * c[2] + c[3] * c[3]);
    const float sb = warp_sum(bm[0] * bm[0] + bm[1] * bm[1] + bm[2] * bm[2] + bm[3] * bm[3]);
    if (f.on) {
      const float rc = rsqrtf(sc / N + p.eps), rb = rsqrtf(sb / N + p.eps);
      float sn, cs;
      sincosf(th, &sn, &cs);
      float u[4], o[4];
      norm_bias_rope(c, rc, wc, cb, sn, cs, u, o);
      st4(q + (b * p.T + t) * HN + h * N, f, o);
      norm_bias_rope(bm, rb, wb, bb, sn, cs, u, o);
      st4(kx + (b * (p.T + 1) + t + 1) * HN + h * N, f, o);
    }
    for (int pp = lane; pp < P; pp += 32)  // xp = x one token later (mamba3.py:115)
      stv<float>(xp + (b * p.T + t) * HP + h * P + pp, t > 0 ? ldv<float>(p.x.row<TI>(b, t - 1, h) + pp) : 0.f);
  }
}

// out = (y + D x) * silu(z)   (mamba3.py:119)
template <typename TI, typename TO>
__global__ void __launch_bounds__(1024) m3_epilogue_fwd_kernel(const M3 p) {
  const int b = blockIdx.x / p.nseg, seg = blockIdx.x % p.nseg;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = (int)p.P;
  const int64_t HP = p.H * P;
  const float Dh = p.D[h];
  const TO* y = static_cast<const TO*>(p.y);
  const int64_t t0 = (int64_t)seg * kSeg, t1 = min(p.T, t0 + kSeg);
  for (int64_t t = t0; t < t1; ++t)
    for (int pp = lane; pp < P; pp += 32) {
      float v = ldv<float>(y + (b * p.T + t) * HP + h * P + pp) + Dh * ldv<float>(p.x.row<TI>(b, t, h) + pp);
      if (p.z.ptr) {
        const float zz = ldv<float>(p.z.row<TI>(b, t, h) + pp);
        v *= zz * sigmoidf_(zz);
      }
      stv<float>(p.out.wrow<TI>(b, t, h) + pp, v);
    }
}

// ---------------------------------------------------------------------------------------------
// backward

// dy = dout silu(z) for the scan; dz = dout (y + D x) silu'(z); D partial sums of dy . x
template <typename TI, typename TO>
__global__ void __launch_bounds__(1024) m3_epilogue_bwd_kernel(const M3 p) {
  const int b = blockIdx.x / p.nseg, seg = blockIdx.x % p.nseg;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = (int)p.P;
  const int64_t HP = p.H * P;
  const float Dh = p.D[h];
  const TO* y = static_cast<const TO*>(p.y);
  TO* dy = static_cast<TO*>(p.dy);
  const int64_t t0 = (int64_t)seg * kSeg, t1 = min(p.T, t0 + kSeg);
  float acc = 0.f;
  for (int64_t t = t0; t < t1; ++t)
    for (int pp = lane; pp < P; pp += 32) {
      const float go = ldv<float>(p.dout.row<TI>(b, t, h) + pp);
      const float xv = ldv<float>(p.x.row<TI>(b, t, h) + pp);
      float g = go;
      if (p.z.ptr) {
        const float zz = ldv<float>(p.z.row<TI>(b, t, h) + pp), s = sigmoidf_(zz);
        g = go * zz * s;
        const float v = ldv<float>(y + (b * p.T + t) * HP + h * P + pp) + Dh * xv;
        stv<float>(p.dz.wrow<TI>(b, t, h) + pp, go * v * s * (1.f + zz * (1.f - s)));
      }
      stv<float>(dy + (b * p.T + t) * HP + h * P + pp, g);
      acc += g * xv;
    }
  acc = warp_sum(acc);
  if (lane == 0) p.pD[(b * p.nseg + seg) * p.H + h] = acc;
}

// RMSNorm backward of one token (mamba3.py:13-15), given the per-head gradients of its
// normalised output staged in src [H][N]: they are summed in head order (u = x r w + bias_h for
// every head h), then dx = r w du - x r^3 / N sum(du w x); dw accumulates du x r.  Lanes past
// the RoPE angles hold zeros, so the warp-wide sum sees every lane.
__device__ __forceinline__ void rms_bwd_token(const float* src, int H, int N, Feat f, const float (&xv)[4],
                                              const float (&wv)[4], float rr, float (&gw)[4], float (&gx)[4]) {
  float du[4] = {0.f, 0.f, 0.f, 0.f};
  if (f.on)
    for (int hh = 0; hh < H; ++hh) {
      const float* r = src + hh * N;
      du[0] += r[f.f0];
      du[1] += r[f.f0 + 1];
      du[2] += r[f.f2];
      du[3] += r[f.f2 + 1];
    }
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

// Reverse walk over one segment: RoPE and RMSNorm backward, bias / norm-weight partial sums,
// dx (scan dx + shifted dxp + D skip), the within-segment suffix of the theta gradient, and the
// per-token sums over heads (dCm, dBm, ang gradient part) through shared memory.
template <typename TI, typename TO>
__global__ void __launch_bounds__(1024) m3_prologue_bwd_kernel(const M3 p) {
  extern __shared__ float smem[];  // [2 buffers][dvq H*N | dvk H*N | DT*sfx H*NA]
  const int b = blockIdx.x / p.nseg, seg = blockIdx.x % p.nseg;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NA = p.NA, N = (int)p.N, P = (int)p.P, H = (int)p.H;
  const int buf_floats = H * (2 * N + NA);
  const Feat f = feat(lane, NA);
  float wc[4] = {}, wb[4] = {}, cb[4] = {}, bb[4] = {};
  if (f.on) {
    ldp4(p.C_norm_w, f, wc);
    ldp4(p.B_norm_w, f, wb);
    ldp4(p.C_bias + h * N, f, cb);
    ldp4(p.B_bias + h * N, f, bb);
  }
  const float dtb = p.dt_bias[h], Dh = p.D[h];
  const int64_t t0 = (int64_t)seg * kSeg, t1 = min(p.T, t0 + kSeg);
  const int64_t HN = (int64_t)H * N, HP = (int64_t)H * P;
  const TO* dq = static_cast<const TO*>(p.dq);
  const TO* dk = static_cast<const TO*>(p.dk);
  const TO* dkp = static_cast<const TO*>(p.dkp);
  const TO* dxs = static_cast<const TO*>(p.dxs);
  const TO* dxp = static_cast<const TO*>(p.dxp);
  const bool wC = (h == 0), wB = (h == 1 % H), wA = (h == 2 % H);
  float gcb[4] = {}, gbb[4] = {}, gwc[4] = {}, gwb[4] = {};
  float sfx = 0.f;  // theta gradient summed over this segment's tokens >= t
  int step = 0;
  for (int64_t t = t1 - 1; t >= t0; --t, ++step) {
    float* buf = smem + (step & 1) * buf_floats;
    const int64_t bth = (b * p.T + t) * H + h;
    const float DT = softplus20(ldv<float>(p.dd_dt.row<TI>(b, t, h)) + dtb);
    float c[4] = {}, bm[4] = {};
    if (f.on) {
      ld4(p.Cm.row<TI>(b, t, 0), f, c);
      ld4(p.Bm.row<TI>(b, t, 0), f, bm);
    }
    const float sc = warp_sum(c[0] * c[0] + c[1] * c[1] + c[2] * c[2] + c[3] * c[3]);
    const float sb = warp_sum(bm[0] * bm[0] + bm[1] * bm[1] + bm[2] * bm[2] + bm[3] * bm[3]);
    const float rc = rsqrtf(sc / N + p.eps), rb = rsqrtf(sb / N + p.eps);
    float part = 0.f;
    if (f.on) {
      const float th = p.theta[bth * NA + lane];
      float sn, cs;
      sincosf(th, &sn, &cs);
      float uq[4], oq[4], uk[4], ok[4];
      norm_bias_rope(c, rc, wc, cb, sn, cs, uq, oq);
      norm_bias_rope(bm, rb, wb, bb, sn, cs, uk, ok);
      float gq[4], gk[4], gkp[4] = {};
      ld4(dq + (b * p.T + t) * HN + h * N, f, gq);
      ld4(dk + (b * p.T + t) * HN + h * N, f, gk);
      if (t + 1 < p.T) ld4(dkp + (b * p.T + t + 1) * HN + h * N, f, gkp);  // kp[t+1] = k[t]
#pragma unroll
      for (int j = 0; j < 4; ++j) gk[j] += gkp[j];
      // rope backward: rotate the gradient back; d theta from the rotated outputs
      const float dvq[4] = {gq[0] * cs + gq[1] * sn, -gq[0] * sn + gq[1] * cs, gq[2], gq[3]};
      const float dvk[4] = {gk[0] * cs + gk[1] * sn, -gk[0] * sn + gk[1] * cs, gk[2], gk[3]};
      sfx += (gq[1] * oq[0] - gq[0] * oq[1]) + (gk[1] * ok[0] - gk[0] * ok[1]);
      part = sfx * ldv<float>(p.ang.row<TI>(b, t, 0) + lane);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        gcb[j] += dvq[j];
        gbb[j] += dvk[j];
      }
      float* bq = buf + h * N;
      float* bk = buf + HN + h * N;
      bq[f.f0] = dvq[0]; bq[f.f0 + 1] = dvq[1]; bq[f.f2] = dvq[2]; bq[f.f2 + 1] = dvq[3];
      bk[f.f0] = dvk[0]; bk[f.f0 + 1] = dvk[1]; bk[f.f2] = dvk[2]; bk[f.f2 + 1] = dvk[3];
      buf[2 * HN + h * NA + lane] = DT * sfx;
    }
    part = warp_sum(part);
    if (lane == 0) p.dDTl[bth] = part;
    // dx = scan dx + dxp of the next token (xp[t+1] = x[t]) + D dout silu(z)
    for (int pp = lane; pp < P; pp += 32) {
      float g = ldv<float>(dxs + (b * p.T + t) * HP + h * P + pp);
      if (t + 1 < p.T) g += ldv<float>(dxp + (b * p.T + t + 1) * HP + h * P + pp);
      float go = ldv<float>(p.dout.row<TI>(b, t, h) + pp);
      if (p.z.ptr) {
        const float zz = ldv<float>(p.z.row<TI>(b, t, h) + pp);
        go *= zz * sigmoidf_(zz);
      }
      stv<float>(p.dx.wrow<TI>(b, t, h) + pp, g + Dh * go);
    }
    __syncthreads();
    // per-token sums over heads in head order, then the RMSNorm backward of Cm / Bm
    if (wC) {
      float gx[4];
      rms_bwd_token(buf, H, N, f, c, wc, rc, gwc, gx);
      if (f.on) st4(p.dCm.wrow<TI>(b, t, 0), f, gx);
    }
    if (wB) {
      float gx[4];
      rms_bwd_token(buf + HN, H, N, f, bm, wb, rb, gwb, gx);
      if (f.on) st4(p.dBm.wrow<TI>(b, t, 0), f, gx);
    }
    if (wA && lane < NA) {
      float s = 0.f;
      for (int hh = 0; hh < H; ++hh) s += buf[2 * HN + hh * NA + lane];
      p.dangl[(b * p.T + t) * NA + lane] = s;
    }
  }
  if (f.on) {
    p.segsum[((b * H + h) * p.nseg + seg) * NA + lane] = sfx;
    const int64_t pb = ((int64_t)(b * p.nseg + seg) * H + h) * N;
    const int64_t part1 = (int64_t)p.B * p.nseg * HN;
    float* pB = p.pbias + pb;
    float* pC = p.pbias + part1 + pb;
    pB[f.f0] = gbb[0]; pB[f.f0 + 1] = gbb[1]; pB[f.f2] = gbb[2]; pB[f.f2 + 1] = gbb[3];
    pC[f.f0] = gcb[0]; pC[f.f0 + 1] = gcb[1]; pC[f.f2] = gcb[2]; pC[f.f2 + 1] = gcb[3];
    const int64_t pn = (int64_t)(b * p.nseg + seg) * N;
    if (wB) {
      float* o = p.pnorm + pn;
      o[f.f0] = gwb[0]; o[f.f0 + 1] = gwb[1]; o[f.f2] = gwb[2]; o[f.f2 + 1] = gwb[3];
    }
    if (wC) {
      float* o = p.pnorm + (int64_t)p.B * p.nseg * N + pn;
      o[f.f0] = gwc[0]; o[f.f0 + 1] = gwc[1]; o[f.f2] = gwc[2]; o[f.f2 + 1] = gwc[3];
    }
  }
}

// The theta-gradient carry from later segments, then the discretisation backward per token
// (mamba3.py:105-111) and the ang gradient.
template <typename TI>
__global__ void __launch_bounds__(1024) m3_scalars_bwd_kernel(const M3 p) {
  extern __shared__ float smem[];  // sDT [kSeg][H] | sC [H][NA]
  const int b = blockIdx.x / p.nseg, seg = blockIdx.x % p.nseg;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NA = p.NA, H = (int)p.H;
  float* sDT = smem;
  float* sC = smem + kSeg * H;
  float C = 0.f;  // theta gradient summed over all later tokens (later segments)
  if (lane < NA) {
    for (int s = seg + 1; s < p.nseg; ++s) C += p.segsum[((b * H + h) * p.nseg + s) * NA + lane];
    sC[h * NA + lane] = C;
  }
  const float dtb = p.dt_bias[h];
  const int64_t t0 = (int64_t)seg * kSeg, t1 = min(p.T, t0 + kSeg);
  float acc_dt = 0.f;
  for (int64_t t = t0; t < t1; ++t) {
    const int64_t bth = (b * p.T + t) * H + h;
    const Disc d = discretise(ldv<float>(p.dd_dt.row<TI>(b, t, h)), ldv<float>(p.dd_A.row<TI>(b, t, h)),
                              ldv<float>(p.trap.row<TI>(b, t, h)), dtb, p.A_floor);
    const float carry = warp_sum(lane < NA ? C * ldv<float>(p.ang.row<TI>(b, t, 0) + lane) : 0.f);
    if (lane == 0) {
      sDT[(t - t0) * H + h] = d.DT;
      const float ga = p.dadt[bth], gg = p.dgamma[bth], gb = p.dbeta[bth];
      const float g_adt = ga + gb * d.beta;  // beta = (1 - tr) DT e^{adt}
      const float g_DT = g_adt * d.A + gg * d.tr + gb * (1.f - d.tr) * d.ea + p.dDTl[bth] + carry;
      const float g_A = g_adt * d.DT;
      const float g_tr = gg * d.DT - gb * d.DT * d.ea;
      const float g_xs = g_DT * (d.xs > 20.f ? 1.f : sigmoidf_(d.xs));  // softplus'
      const float ddA = ldv<float>(p.dd_A.row<TI>(b, t, h));
      // clamp(max=-A_floor) passes the gradient where heavy_tail <= -A_floor; heavy_tail's two
      // clamps pass it at x >= 0 and x <= 0 respectively (torch.clamp's masks)
      const float dht = (ddA >= 0.f ? 1.f : 0.f) + (ddA <= 0.f ? 1.f / ((1.f - ddA) * (1.f - ddA)) : 0.f);
      const float g_ddA = d.ht <= -p.A_floor ? -g_A * dht : 0.f;
      stv<float>(p.ddd_dt.wrow<TI>(b, t, h), g_xs);
      stv<float>(p.ddd_A.wrow<TI>(b, t, h), g_ddA);
      stv<float>(p.dtrap.wrow<TI>(b, t, h), g_tr * d.tr * (1.f - d.tr));
      acc_dt += g_xs;
    }
  }
  if (lane == 0) p.pdt[(b * p.nseg + seg) * H + h] = acc_dt;
  __syncthreads();
  // ang gradient: the within-segment part plus sum_h DT[t][h] * carry[h][i]
  const int n = (int)(t1 - t0) * NA;
  for (int idx = threadIdx.x; idx < n; idx += blockDim.x) {
    const int tt = idx / NA, i = idx % NA;
    float s = p.dangl[(b * p.T + t0 + tt) * NA + i];
    for (int hh = 0; hh < H; ++hh) s += sDT[tt * H + hh] * sC[hh * NA + i];
    stv<float>(p.dang.wrow<TI>(b, t0 + tt, 0) + i, s);
  }
}

// parameter gradients: fixed-order sums of the per-(batch, segment) partials
__global__ void m3_param_reduce_kernel(const M3 p) {
  const int64_t H = p.H, N = p.N, BS = p.B * p.nseg;
  const int64_t n_bias = H * N;
  const int64_t total = 2 * n_bias + 2 * N + 2 * H;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    if (i < 2 * n_bias) {  // B_bias then C_bias
      const int64_t part = i / n_bias, j = i % n_bias;
      const float* src = p.pbias + part * BS * n_bias + j;
      for (int64_t k = 0; k < BS; ++k) s += src[k * n_bias];
      (part ? p.dC_bias : p.dB_bias)[j] = s;
    } else if (i < 2 * n_bias + 2 * N) {  // B_norm_w then C_norm_w
      const int64_t r = i - 2 * n_bias, part = r / N, j = r % N;
      const float* src = p.pnorm + part * BS * N + j;
      for (int64_t k = 0; k < BS; ++k) s += src[k * N];
      (part ? p.dC_norm_w : p.dB_norm_w)[j] = s;
    } else {  // dt_bias then D
      const int64_t r = i - 2 * n_bias - 2 * N, part = r / H, j = r % H;
      const float* src = (part ? p.pD : p.pdt) + j;
      for (int64_t k = 0; k < BS; ++k) s += src[k * H];
      (part ? p.dD : p.ddt_bias)[j] = s;
    }
  }
}

// ---------------------------------------------------------------------------------------------
// host

View view_of(const zb_view& v) { return View{v.ptr, v.sb, v.st, v.sh}; }

struct WsLayout {
  size_t segsum, dDTl, dangl, pbias, pnorm, pdt, pD, total;
};
WsLayout ws_layout(const zb_m3_args* a) {
  const int64_t nseg = (a->T + kSeg - 1) / kSeg, NA = a->N / 4;
  WsLayout L;
  size_t off = 0;
  auto take = [&](size_t floats) {
    const size_t o = off;
    off = align_up(off + floats * sizeof(float), 256);
    return o;
  };
  L.segsum = take((size_t)a->B * a->H * nseg * NA);
  L.dDTl = take((size_t)a->B * a->T * a->H);
  L.dangl = take((size_t)a->B * a->T * NA);
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
  if (a->H > 32 || a->N % 4 != 0 || a->N > 128) return ZB_ERR_UNSUPPORTED;
  if ((double)a->B * (double)(a->T + 1) * (double)a->H * (double)(a->N > a->P ? a->N : a->P) > 9.0e15)
    return ZB_ERR_SHAPE;
  if ((a->io_dtype != ZB_F32 && a->io_dtype != ZB_BF16) || (a->op_dtype != ZB_F32 && a->op_dtype != ZB_BF16))
    return ZB_ERR_DTYPE;
  if (!a->x.ptr || !a->dt_bias || !a->B_bias || !a->C_bias || !a->B_norm_w || !a->C_norm_w || !a->D)
    return ZB_ERR_LAYOUT;
  if (!a->workspace || a->workspace_bytes < ws_layout(a).total || (reinterpret_cast<uintptr_t>(a->workspace) & 255))
    return ZB_ERR_WORKSPACE;
  return ZB_OK;
}

M3 make_m3(const zb_m3_args* a) {
  M3 p;
  memset(&p, 0, sizeof(p));
  p.B = a->B; p.T = a->T; p.H = a->H; p.P = a->P; p.N = a->N;
  p.NA = (int)(a->N / 4);
  p.nseg = (int)((a->T + kSeg - 1) / kSeg);
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
  const WsLayout L = ws_layout(a);
  unsigned char* ws = static_cast<unsigned char*>(a->workspace);
  p.segsum = reinterpret_cast<float*>(ws + L.segsum);
  p.dDTl = reinterpret_cast<float*>(ws + L.dDTl);
  p.dangl = reinterpret_cast<float*>(ws + L.dangl);
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
  if (!a->q || !a->k_ext || !a->xp || !a->adt || !a->gamma || !a->beta || !a->theta || !a->Bm.ptr || !a->Cm.ptr ||
      !a->dd_dt.ptr || !a->dd_A.ptr || !a->trap.ptr || !a->ang.ptr)
    return ZB_ERR_LAYOUT;
  const M3 p = make_m3(a);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)(p.B * p.nseg)), block((unsigned)(32 * p.H));
  ZB_M3_DISPATCH(a->io_dtype, a->op_dtype, {
    m3_segsum_kernel<TI><<<grid, block, 0, s>>>(p);
    m3_prologue_fwd_kernel<TI, TO><<<grid, block, 0, s>>>(p);
  });
  return finish(2);
}

extern "C" ZB_API int zb_m3_epilogue_fwd(const zb_m3_args* a, void* stream) {
  int rc = check(a);
  if (rc) return rc;
  if (!a->y || !a->out.ptr) return ZB_ERR_LAYOUT;
  const M3 p = make_m3(a);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)(p.B * p.nseg)), block((unsigned)(32 * p.H));
  ZB_M3_DISPATCH(a->io_dtype, a->op_dtype, { m3_epilogue_fwd_kernel<TI, TO><<<grid, block, 0, s>>>(p); });
  return finish(1);
}

extern "C" ZB_API int zb_m3_epilogue_bwd(const zb_m3_args* a, void* stream) {
  int rc = check(a);
  if (rc) return rc;
  if (!a->y || !a->dout.ptr || !a->dy || (a->z.ptr && !a->dz.ptr)) return ZB_ERR_LAYOUT;
  const M3 p = make_m3(a);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)(p.B * p.nseg)), block((unsigned)(32 * p.H));
  ZB_M3_DISPATCH(a->io_dtype, a->op_dtype, { m3_epilogue_bwd_kernel<TI, TO><<<grid, block, 0, s>>>(p); });
  return finish(1);
}

extern "C" ZB_API int zb_m3_prologue_bwd(const zb_m3_args* a, void* stream) {
  int rc = check(a);
  if (rc) return rc;
  if (!a->theta || !a->dout.ptr || !a->dxs || !a->dxp || !a->dq || !a->dk || !a->dkp || !a->dadt || !a->dgamma ||
      !a->dbeta || !a->dx.ptr || !a->dBm.ptr || !a->dCm.ptr || !a->ddd_dt.ptr || !a->ddd_A.ptr || !a->dtrap.ptr ||
      !a->dang.ptr || !a->ddt_bias || !a->dB_bias || !a->dC_bias || !a->dB_norm_w || !a->dC_norm_w || !a->dD)
    return ZB_ERR_LAYOUT;
  const M3 p = make_m3(a);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)(p.B * p.nseg)), block((unsigned)(32 * p.H));
  // two staging buffers of (dvq, dvk: H x N; DT * theta-gradient: H x NA)
  const int smem1 = (int)(2 * (p.H * (2 * p.N + p.NA)) * sizeof(float));
  const int smem2 = (int)((kSeg * p.H + p.H * p.NA) * sizeof(float));
  ZB_M3_DISPATCH(a->io_dtype, a->op_dtype, {
    auto k1 = m3_prologue_bwd_kernel<TI, TO>;
    if (cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, smem1) != cudaSuccess) return ZB_ERR_CUDA;
    k1<<<grid, block, smem1, s>>>(p);
    m3_scalars_bwd_kernel<TI><<<grid, block, smem2, s>>>(p);
  });
  m3_param_reduce_kernel<<<64, 256, 0, s>>>(p);
  return finish(3);
}
