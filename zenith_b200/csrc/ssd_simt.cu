// Generic SIMT path of the SSD chunked scan (any dtype incl. fp64, any P/N that fits shared
// memory).  One CTA per (batch, head, chunk); CTAs take chunks in ticket order and hand the
// running state to the CTA of the next chunk through global memory (chained scan), so the
// reference's serial Python loop over chunks (zenith/mamba3.py:51-53) disappears into one
// launch.  The backward runs the same chain in reverse for the state gradient.
//
// This path computes in the accumulator type TA (fp32, or fp64 for fp64 inputs) with plain
// FMAs.  It is the accurate path for fp32/fp64 inputs; bf16 inputs with P=64 take the
// tensor-core path in ssd_tc.cu.
#include "common.cuh"
#include "ssd_kernels.h"

namespace zb {

namespace {

constexpr int kThreads = 256;

template <typename TA> __device__ __forceinline__ TA ldcg_t(const TA* p) { return __ldcg(p); }

template <typename TA>
struct SmemLayout {
  int L, P, N, N1, P1, L1;
  __host__ __device__ SmemLayout(int L_, int P_, int N_) : L(L_), P(P_), N(N_), N1(N_ + 1), P1(P_ + 1), L1(L_ + 1) {}
  // forward: 5 scalars/token, q k kp [L][N1], x xp [L][P1], Sg Sb [L][L1], S [P][N1]
  __host__ __device__ size_t fwd_elems() const {
    return 5 * (size_t)L + 3 * (size_t)L * N1 + 2 * (size_t)L * P1 + 2 * (size_t)L * L1 + (size_t)P * N1;
  }
  // backward: 10 scalars/token, q k kp [L][N1], x xp dy [L][P1], A Ap E Ep Z Zg Zb [L][L1],
  // S G [P][N1], 64 scratch
  __host__ __device__ size_t bwd_elems() const {
    return 10 * (size_t)L + 3 * (size_t)L * N1 + 3 * (size_t)L * P1 + 7 * (size_t)L * L1 + 2 * (size_t)P * N1 + 64;
  }
};

// ---------------------------------------------------------------------------------------------
// forward
template <typename TI, typename TS, typename TA>
__global__ void __launch_bounds__(kThreads) ssd_fwd_simt_kernel(const SimtParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TA* sm = reinterpret_cast<TA*>(smem_raw);
  const int L = p.L, P = (int)p.P, N = (int)p.N;
  const int N1 = N + 1, P1 = P + 1, L1 = L + 1;
  TA* s_c = sm;
  TA* s_ec = s_c + L;
  TA* s_w = s_ec + L;
  TA* s_g = s_w + L;
  TA* s_b = s_g + L;
  TA* s_q = s_b + L;
  TA* s_k = s_q + L * N1;
  TA* s_kp = s_k + L * N1;
  TA* s_x = s_kp + L * N1;
  TA* s_xp = s_x + L * P1;
  TA* s_Sg = s_xp + L * P1;
  TA* s_Sb = s_Sg + L * L1;
  TA* s_S = s_Sb + L * L1;
  __shared__ int s_ticket, s_ready;

  const int tid = threadIdx.x;
  const bool state_only = (p.flags & ZB_FLAG_STATE_ONLY) != 0;
  if (tid == 0) s_ticket = (int)atomicAdd(p.sync.ticket, 1u);
  __syncthreads();
  const UnitIdx u = decode_ticket((uint32_t)s_ticket, p.B, p.H, p.G);
  const int j = u.chunk;
  const int64_t bh = u.bh, b = u.b, h = u.h, g = u.g;
  const int64_t t0 = (int64_t)j * L;
  const int sh = (p.flags & ZB_FLAG_SHIFTED) ? 1 : 0;  // xp / kp = x / k one token later
  const int Lc = (int)min((int64_t)L, p.T - t0);
  int* flags = p.sync.flags + bh * (p.nc + 1);

  if (tid < 32) {
    TA a = 0, gm = 0, bt = 0;
    if (tid < Lc) {
      a = ldv<TA>(p.adt.row<TS>(b, t0 + tid, h));
      gm = ldv<TA>(p.gamma.row<TS>(b, t0 + tid, h));
      bt = ldv<TA>(p.beta.row<TS>(b, t0 + tid, h));
    }
    const TA c = warp_incl_scan(a, tid);
    if (tid < L) {
      s_c[tid] = c;
      s_g[tid] = gm;
      s_b[tid] = bt;
    }
  }
  for (int i = tid; i < L * N; i += kThreads) {
    const int t = i / N, n = i % N;
    const bool v = t < Lc;
    s_k[t * N1 + n] = v ? ldv<TA>(p.k.row<TI>(b, t0 + t, g) + n) : TA(0);
    s_kp[t * N1 + n] = v && t0 + t >= sh ? ldv<TA>(p.kp.row<TI>(b, t0 + t - sh, g) + n) : TA(0);
    if (!state_only) s_q[t * N1 + n] = v ? ldv<TA>(p.q.row<TI>(b, t0 + t, g) + n) : TA(0);
  }
  for (int i = tid; i < L * P; i += kThreads) {
    const int t = i / P, pp = i % P;
    const bool v = t < Lc;
    s_x[t * P1 + pp] = v ? ldv<TA>(p.x.row<TI>(b, t0 + t, h) + pp) : TA(0);
    s_xp[t * P1 + pp] = v && t0 + t >= sh ? ldv<TA>(p.xp.row<TI>(b, t0 + t - sh, h) + pp) : TA(0);
  }
  __syncthreads();
  const TA cl = s_c[Lc - 1];
  if (tid < L) {
    s_ec[tid] = xexp(s_c[tid]);
    s_w[tid] = xexp(cl - s_c[tid]);
  }
  __syncthreads();
  const TA a_chunk = xexp(cl);

  const int64_t PN = (int64_t)P * N;
  TA* chain_bh = reinterpret_cast<TA*>(p.chain) + bh * (int64_t)(p.nc + 1) * PN;
  TA* slot_in = chain_bh + (int64_t)j * PN;
  TA* slot_out = chain_bh + (int64_t)(j + 1) * PN;

  // chunk-local state S_loc (mamba3.py:46-47), parked in the outgoing slot until the
  // incoming state is known (each thread re-reads only what it wrote itself)
  for (int i = tid; i < P * N; i += kThreads) {
    const int pp = i / N, n = i % N;
    TA acc = 0;
    for (int s = 0; s < Lc; ++s)
      acc += s_w[s] * (s_g[s] * s_x[s * P1 + pp] * s_k[s * N1 + n] + s_b[s] * s_xp[s * P1 + pp] * s_kp[s * N1 + n]);
    slot_out[i] = acc;
  }
  // masked intra-chunk scores (mamba3.py:41-44)
  if (!state_only) {
    for (int i = tid; i < L * L; i += kThreads) {
      const int t = i / L, s = i % L;
      TA vg = 0, vb = 0;
      if (s <= t && t < Lc) {
        TA dk = 0, dkp = 0;
        for (int n = 0; n < N; ++n) {
          const TA qv = s_q[t * N1 + n];
          dk += qv * s_k[s * N1 + n];
          dkp += qv * s_kp[s * N1 + n];
        }
        const TA m = xexp(s_c[t] - s_c[s]);
        vg = dk * s_g[s] * m;
        vb = dkp * s_b[s] * m;
      }
      s_Sg[t * L1 + s] = vg;
      s_Sb[t * L1 + s] = vb;
    }
  }
  __syncthreads();
  if (tid == 0) s_ready = (j == 0) ? kFlagReady : wait_flag(&flags[j], p.status);
  __syncthreads();
  if (s_ready != kFlagReady) {
    if (tid == 0) st_release(&flags[j + 1], kFlagAbort);
    return;
  }
  for (int i = tid; i < P * N; i += kThreads) {
    TA v;
    if (j == 0) {
      v = p.init ? reinterpret_cast<const TA*>(p.init)[bh * PN + i] : TA(0);
      slot_in[i] = v;
    } else {
      v = ldcg_t(slot_in + i);
    }
    s_S[(i / N) * N1 + i % N] = v;
  }
  __syncthreads();
  // S_in[j+1] = e^{c_L} S_in[j] + S_loc[j]   (mamba3.py:52)
  const bool last = (j == p.nc - 1);
  for (int i = tid; i < P * N; i += kThreads) {
    const TA v = a_chunk * s_S[(i / N) * N1 + i % N] + slot_out[i];
    slot_out[i] = v;
    if (last && p.fin) reinterpret_cast<TA*>(p.fin)[bh * PN + i] = v;
  }
  // the barrier orders every thread's ring writes before thread 0's release (cumulative)
  __syncthreads();
  if (tid == 0) st_release(&flags[j + 1], kFlagReady);
  if (state_only) return;

  // y = y_intra + e^{c} (q S_in^T)   (mamba3.py:45,55)
  for (int i = tid; i < Lc * P; i += kThreads) {
    const int t = i / P, pp = i % P;
    TA acc = 0;
    for (int s = 0; s <= t; ++s) acc += s_Sg[t * L1 + s] * s_x[s * P1 + pp] + s_Sb[t * L1 + s] * s_xp[s * P1 + pp];
    TA ai = 0;
    for (int n = 0; n < N; ++n) ai += s_q[t * N1 + n] * s_S[pp * N1 + n];
    acc += s_ec[t] * ai;
    stv<TA>(p.y.wrow<TI>(b, t0 + t, h) + pp, acc);
  }
}

// ---------------------------------------------------------------------------------------------
// backward (reverse chain)
template <typename TI, typename TS, typename TA>
__global__ void __launch_bounds__(kThreads) ssd_bwd_simt_kernel(const SimtParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TA* sm = reinterpret_cast<TA*>(smem_raw);
  const int L = p.L, P = (int)p.P, N = (int)p.N;
  const int N1 = N + 1, P1 = P + 1, L1 = L + 1;
  TA* s_c = sm;
  TA* s_ec = s_c + L;
  TA* s_w = s_ec + L;
  TA* s_g = s_w + L;
  TA* s_b = s_g + L;
  TA* s_dc = s_b + L;     // dL/dc_t
  TA* s_dg = s_dc + L;    // dL/dgamma_s
  TA* s_db = s_dg + L;    // dL/dbeta_s
  TA* s_xu = s_db + L;    // x_s . (Gn k_s)
  TA* s_xpu = s_xu + L;   // xp_s . (Gn kp_s)
  TA* s_q = s_xpu + L;
  TA* s_k = s_q + L * N1;
  TA* s_kp = s_k + L * N1;
  TA* s_x = s_kp + L * N1;
  TA* s_xp = s_x + L * P1;
  TA* s_dy = s_xp + L * P1;
  TA* s_A = s_dy + L * P1;
  TA* s_Ap = s_A + L * L1;
  TA* s_E = s_Ap + L * L1;
  TA* s_Ep = s_E + L * L1;
  TA* s_Z = s_Ep + L * L1;  // dA.A + dAp.Ap   (row sums - column sums -> dc)
  TA* s_Zg = s_Z + L * L1;  // E (q.k)         (column sums -> dgamma)
  TA* s_Zb = s_Zg + L * L1; // Ep (q.kp)       (column sums -> dbeta)
  TA* s_S = s_Zb + L * L1;  // S_in [P][N1]
  TA* s_G = s_S + P * N1;   // Gn   [P][N1]
  TA* s_red = s_G + P * N1; // 64 scratch
  __shared__ int s_ticket, s_ready;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool state_only = (p.flags & ZB_FLAG_STATE_ONLY) != 0;
  if (tid == 0) s_ticket = (int)atomicAdd(p.sync.ticket, 1u);
  __syncthreads();
  const UnitIdx u = decode_ticket((uint32_t)s_ticket, p.B, p.H, p.G);
  const int j = p.nc - 1 - u.chunk;
  const int64_t bh = u.bh, b = u.b, h = u.h, g = u.g;
  const int64_t t0 = (int64_t)j * L;
  const int sh = (p.flags & ZB_FLAG_SHIFTED) ? 1 : 0;  // xp / kp = x / k one token later
  const int Lc = (int)min((int64_t)L, p.T - t0);
  int* flags = p.sync.flags + bh * (p.nc + 1);
  const int64_t PN = (int64_t)P * N;

  if (tid < 32) {
    TA a = 0, gm = 0, bt = 0;
    if (tid < Lc) {
      a = ldv<TA>(p.adt.row<TS>(b, t0 + tid, h));
      gm = ldv<TA>(p.gamma.row<TS>(b, t0 + tid, h));
      bt = ldv<TA>(p.beta.row<TS>(b, t0 + tid, h));
    }
    const TA c = warp_incl_scan(a, tid);
    if (tid < L) {
      s_c[tid] = c;
      s_g[tid] = gm;
      s_b[tid] = bt;
      s_dc[tid] = 0;
      s_dg[tid] = 0;
      s_db[tid] = 0;
      s_xu[tid] = 0;
      s_xpu[tid] = 0;
    }
  }
  for (int i = tid; i < L * N; i += kThreads) {
    const int t = i / N, n = i % N;
    const bool v = t < Lc;
    s_q[t * N1 + n] = v ? ldv<TA>(p.q.row<TI>(b, t0 + t, g) + n) : TA(0);
    if (!state_only) {
      s_k[t * N1 + n] = v ? ldv<TA>(p.k.row<TI>(b, t0 + t, g) + n) : TA(0);
      s_kp[t * N1 + n] = v && t0 + t >= sh ? ldv<TA>(p.kp.row<TI>(b, t0 + t - sh, g) + n) : TA(0);
    }
  }
  for (int i = tid; i < L * P; i += kThreads) {
    const int t = i / P, pp = i % P;
    const bool v = t < Lc;
    s_dy[t * P1 + pp] = v ? ldv<TA>(p.dy.row<TI>(b, t0 + t, h) + pp) : TA(0);
    if (!state_only) {
      s_x[t * P1 + pp] = v ? ldv<TA>(p.x.row<TI>(b, t0 + t, h) + pp) : TA(0);
      s_xp[t * P1 + pp] = v && t0 + t >= sh ? ldv<TA>(p.xp.row<TI>(b, t0 + t - sh, h) + pp) : TA(0);
    }
  }
  const TA* states_bh = reinterpret_cast<const TA*>(p.chain) + bh * (int64_t)(p.nc + 1) * PN;
  if (!state_only) {
    for (int i = tid; i < P * N; i += kThreads) s_S[(i / N) * N1 + i % N] = ldcg_t(states_bh + (int64_t)j * PN + i);
  }
  __syncthreads();
  const TA cl = s_c[Lc - 1];
  if (tid < L) {
    s_ec[tid] = xexp(s_c[tid]);
    s_w[tid] = xexp(cl - s_c[tid]);
  }
  __syncthreads();
  const TA a_chunk = xexp(cl);

  // intra-chunk score gradients: A = (q.k) g M, dA = dy.x, E = dA M, ...  All reductions
  // below run in a fixed order (no atomics), so results are bitwise reproducible.
  if (!state_only) {
    for (int i = tid; i < L * L; i += kThreads) {
      const int t = i / L, s = i % L;
      TA vA = 0, vAp = 0, vE = 0, vEp = 0, z = 0, zg = 0, zb = 0;
      if (s <= t && t < Lc) {
        TA qk = 0, qkp = 0, da = 0, dap = 0;
        for (int n = 0; n < N; ++n) {
          const TA qv = s_q[t * N1 + n];
          qk += qv * s_k[s * N1 + n];
          qkp += qv * s_kp[s * N1 + n];
        }
        for (int pp = 0; pp < P; ++pp) {
          const TA d = s_dy[t * P1 + pp];
          da += d * s_x[s * P1 + pp];
          dap += d * s_xp[s * P1 + pp];
        }
        const TA m = xexp(s_c[t] - s_c[s]);
        vA = qk * s_g[s] * m;
        vAp = qkp * s_b[s] * m;
        vE = da * m;
        vEp = dap * m;
        z = da * vA + dap * vAp;
        zg = vE * qk;
        zb = vEp * qkp;
      }
      s_A[t * L1 + s] = vA;
      s_Ap[t * L1 + s] = vAp;
      s_E[t * L1 + s] = vE;
      s_Ep[t * L1 + s] = vEp;
      s_Z[t * L1 + s] = z;
      s_Zg[t * L1 + s] = zg;
      s_Zb[t * L1 + s] = zb;
    }
    __syncthreads();
    // one warp per token u: dc_u = sum_s Z[u][s] - sum_t Z[t][u]; dgamma_u, dbeta_u = column sums
    for (int u = warp; u < L; u += kThreads / 32) {
      TA dc = 0, dg = 0, db = 0;
      if (lane < L) {
        dc = s_Z[u * L1 + lane] - s_Z[lane * L1 + u];
        dg = s_Zg[lane * L1 + u];
        db = s_Zb[lane * L1 + u];
      }
      dc = warp_sum(dc);
      dg = warp_sum(dg);
      db = warp_sum(db);
      if (lane == 0) {
        s_dc[u] = dc;
        s_dg[u] = dg;
        s_db[u] = db;
      }
    }
  }
  // dS_in_loc = sum_t e^{c_t} dy_t q_t^T, parked in this chunk's outgoing gradient slot
  TA* gchain_bh = reinterpret_cast<TA*>(p.gchain) + bh * (int64_t)(p.nc + 1) * PN;
  TA* gslot_out = gchain_bh + (int64_t)j * PN;
  const TA* gslot_in = gchain_bh + (int64_t)(j + 1) * PN;
  for (int i = tid; i < P * N; i += kThreads) {
    const int pp = i / N, n = i % N;
    TA acc = 0;
    for (int t = 0; t < Lc; ++t) acc += s_ec[t] * s_dy[t * P1 + pp] * s_q[t * N1 + n];
    gslot_out[i] = acc;
  }
  __syncthreads();
  const bool last = (j == p.nc - 1);
  if (tid == 0) s_ready = last ? kFlagReady : wait_flag(&flags[j + 1], p.status);
  __syncthreads();
  if (s_ready != kFlagReady) {
    if (tid == 0) st_release(&flags[j], kFlagAbort);
    return;
  }
  for (int i = tid; i < P * N; i += kThreads) {
    TA v;
    if (last) v = p.dfin ? reinterpret_cast<const TA*>(p.dfin)[bh * PN + i] : TA(0);
    else v = ldcg_t(gslot_in + i);
    s_G[(i / N) * N1 + i % N] = v;
  }
  __syncthreads();
  // G[j] = dS_in_loc + e^{c_L} Gn ;  da = <Gn, S_in>
  TA da_part = 0;
  for (int i = tid; i < P * N; i += kThreads) {
    const TA gn = s_G[(i / N) * N1 + i % N];
    const TA v = gslot_out[i] + a_chunk * gn;
    gslot_out[i] = v;
    if (j == 0 && p.dinit) reinterpret_cast<TA*>(p.dinit)[bh * PN + i] = v;
    if (!state_only) da_part += gn * s_S[(i / N) * N1 + i % N];
  }
  // the barrier orders every thread's ring writes before thread 0's release (cumulative)
  __syncthreads();
  if (tid == 0) st_release(&flags[j], kFlagReady);
  if (state_only) return;
  da_part = warp_sum(da_part);
  if (lane == 0) s_red[warp] = da_part;
  __syncthreads();

  // dx, dxp and the state-term dot products: one warp per token s, lanes over p
  for (int s = warp; s < Lc; s += kThreads / 32) {
    TA xu = 0, xpu = 0;
    for (int pp = lane; pp < P; pp += 32) {
      TA u = 0, up = 0;
      for (int n = 0; n < N; ++n) {
        const TA gn = s_G[pp * N1 + n];
        u += gn * s_k[s * N1 + n];
        up += gn * s_kp[s * N1 + n];
      }
      TA vx = 0, vxp = 0;
      for (int t = s; t < Lc; ++t) {
        const TA d = s_dy[t * P1 + pp];
        vx += s_A[t * L1 + s] * d;
        vxp += s_Ap[t * L1 + s] * d;
      }
      vx += s_w[s] * s_g[s] * u;
      vxp += s_w[s] * s_b[s] * up;
      stv<TA>(p.dx.wrow<TI>(b, t0 + s, h) + pp, vx);
      stv<TA>(p.dxp.wrow<TI>(b, t0 + s, h) + pp, vxp);
      xu += s_x[s * P1 + pp] * u;
      xpu += s_xp[s * P1 + pp] * up;
    }
    xu = warp_sum(xu);
    xpu = warp_sum(xpu);
    if (lane == 0) {
      s_xu[s] = xu;
      s_xpu[s] = xpu;
    }
  }
  const bool grouped = p.G != p.H;
  // dq (intra + inter) and its contribution to dc: one warp per token t, lanes over n
  for (int t = warp; t < Lc; t += kThreads / 32) {
    TA dct = 0;
    for (int n = lane; n < N; n += 32) {
      TA acc = 0;
      for (int s = 0; s <= t; ++s) acc += s_E[t * L1 + s] * s_g[s] * s_k[s * N1 + n] + s_Ep[t * L1 + s] * s_b[s] * s_kp[s * N1 + n];
      TA r = 0;
      for (int pp = 0; pp < P; ++pp) r += s_S[pp * N1 + n] * s_dy[t * P1 + pp];
      acc += s_ec[t] * r;
      dct += s_ec[t] * s_q[t * N1 + n] * r;
      if (grouped) reinterpret_cast<TA*>(p.grp)[((b * p.T + t0 + t) * p.H + h) * 3 * N + n] = acc;
      else stv<TA>(p.dq.wrow<TI>(b, t0 + t, h) + n, acc);
    }
    dct = warp_sum(dct);
    if (lane == 0) s_dc[t] += dct;
  }
  // dk, dkp
  for (int i = tid; i < Lc * N; i += kThreads) {
    const int s = i / N, n = i % N;
    TA e = 0, ep = 0;
    for (int t = s; t < Lc; ++t) {
      const TA qv = s_q[t * N1 + n];
      e += s_E[t * L1 + s] * qv;
      ep += s_Ep[t * L1 + s] * qv;
    }
    TA gx = 0, gxp = 0;
    for (int pp = 0; pp < P; ++pp) {
      const TA gn = s_G[pp * N1 + n];
      gx += gn * s_x[s * P1 + pp];
      gxp += gn * s_xp[s * P1 + pp];
    }
    const TA vk = s_g[s] * (e + s_w[s] * gx);
    const TA vkp = s_b[s] * (ep + s_w[s] * gxp);
    if (grouped) {
      TA* gp = reinterpret_cast<TA*>(p.grp) + ((b * p.T + t0 + s) * p.H + h) * 3 * N;
      gp[N + n] = vk;
      gp[2 * N + n] = vkp;
    } else {
      stv<TA>(p.dk.wrow<TI>(b, t0 + s, h) + n, vk);
      stv<TA>(p.dkp.wrow<TI>(b, t0 + s, h) + n, vkp);
    }
  }
  __syncthreads();
  // per-token scalar gradients; warp 0 owns the chunk's tokens (L <= 32)
  if (warp == 0) {
    TA da = 0;
    for (int wi = 0; wi < kThreads / 32; ++wi) da += s_red[wi];
    TA dcv = 0, wdw = 0, dgv = 0, dbv = 0;
    if (lane < Lc) {
      const TA w = s_w[lane];
      const TA dw = s_g[lane] * s_xu[lane] + s_b[lane] * s_xpu[lane];
      dgv = s_dg[lane] + w * s_xu[lane];
      dbv = s_db[lane] + w * s_xpu[lane];
      dcv = s_dc[lane] - w * dw;
      wdw = w * dw;
    }
    wdw = warp_sum(wdw);
    if (lane == Lc - 1) dcv += a_chunk * da + wdw;
    // dadt_u = sum_{t >= u} dc_t  (reverse cumulative sum: c = cumsum(adt))
    const TA total = warp_sum(dcv);
    const TA incl = warp_incl_scan(dcv, lane);
    const TA dadt = total - incl + dcv;
    if (lane < Lc) {
      stv<TA>(p.dadt.wrow<TS>(b, t0 + lane, h), dadt);
      stv<TA>(p.dgamma.wrow<TS>(b, t0 + lane, h), dgv);
      stv<TA>(p.dbeta.wrow<TS>(b, t0 + lane, h), dbv);
    }
  }
}

// sum the per-head q/k/kp gradients of each group: grp [B,T,H,3,N] (TA) -> dq/dk/dkp [B,T,G,N]
template <typename TI, typename TA>
__global__ void group_reduce_kernel(const SimtParams p) {
  const int64_t N = p.N, r = p.H / p.G;
  const int64_t total = p.B * p.T * p.G * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i % N, g = (i / N) % p.G, t = (i / (N * p.G)) % p.T, b = i / (N * p.G * p.T);
    TA acc[3] = {0, 0, 0};
    for (int64_t u = 0; u < r; ++u) {
      const TA* gp = reinterpret_cast<const TA*>(p.grp) + ((b * p.T + t) * p.H + g * r + u) * 3 * N;
      acc[0] += gp[n];
      acc[1] += gp[N + n];
      acc[2] += gp[2 * N + n];
    }
    stv<TA>(p.dq.wrow<TI>(b, t, g) + n, acc[0]);
    stv<TA>(p.dk.wrow<TI>(b, t, g) + n, acc[1]);
    stv<TA>(p.dkp.wrow<TI>(b, t, g) + n, acc[2]);
  }
}

}  // namespace

int simt_pick_chunk(int P, int N, bool f64) {
  const size_t esz = f64 ? 8 : 4;
  for (int L : {32, 16, 8, 4}) {
    SmemLayout<float> lay(L, P, N);
    if (lay.bwd_elems() * esz <= kSimtMaxSmem && lay.fwd_elems() * esz <= kSimtMaxSmem) return L;
  }
  return 0;
}

template <typename TI, typename TS, typename TA>
static int launch_simt(const SimtParams& p, bool backward, cudaStream_t stream) {
  SmemLayout<TA> lay(p.L, (int)p.P, (int)p.N);
  const size_t smem = (backward ? lay.bwd_elems() : lay.fwd_elems()) * sizeof(TA);
  const dim3 grid((unsigned)(p.B * p.H * p.nc)), block(kThreads);
  if (!backward) {
    auto k = ssd_fwd_simt_kernel<TI, TS, TA>;
    if (dyn_smem(reinterpret_cast<const void*>(k), (int)smem) != ZB_OK) return ZB_ERR_CUDA;
    k<<<grid, block, smem, stream>>>(p);
    note_launches(1);
  } else {
    auto k = ssd_bwd_simt_kernel<TI, TS, TA>;
    if (dyn_smem(reinterpret_cast<const void*>(k), (int)smem) != ZB_OK) return ZB_ERR_CUDA;
    k<<<grid, block, smem, stream>>>(p);
    note_launches(1);
    if (p.G != p.H && !(p.flags & ZB_FLAG_STATE_ONLY)) {
      const int64_t total = p.B * p.T * p.G * p.N;
      const unsigned nb = (unsigned)std::min<int64_t>((total + 255) / 256, 148 * 16);
      group_reduce_kernel<TI, TA><<<nb, 256, 0, stream>>>(p);
      note_launches(1);
    }
  }
  return cudaPeekAtLastError() == cudaSuccess ? ZB_OK : ZB_ERR_CUDA;
}

int simt_launch(const SimtParams& p, int dtype, int sdtype, bool backward, cudaStream_t stream) {
  if (dtype == ZB_F64 && sdtype == ZB_F64) return launch_simt<double, double, double>(p, backward, stream);
  if (dtype == ZB_F32 && sdtype == ZB_F32) return launch_simt<float, float, float>(p, backward, stream);
  if (dtype == ZB_BF16 && sdtype == ZB_F32) return launch_simt<__nv_bfloat16, float, float>(p, backward, stream);
  if (dtype == ZB_BF16 && sdtype == ZB_BF16) return launch_simt<__nv_bfloat16, __nv_bfloat16, float>(p, backward, stream);
  if (dtype == ZB_F16 && sdtype == ZB_F32) return launch_simt<__half, float, float>(p, backward, stream);
  if (dtype == ZB_F16 && sdtype == ZB_F16) return launch_simt<__half, __half, float>(p, backward, stream);
  return ZB_ERR_DTYPE;
}

}  // namespace zb
