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
// Register-tiled products over the shared-memory tiles, used when P <= 64 and N <= 128 (the model
// shapes); other sizes take the one-output-per-thread loops.  A warp owns RM consecutive output
// rows (all its lanes read the same element of the row operand: a broadcast) and the columns
// lane + 32 j, j < RN (consecutive lanes read consecutive elements of the column operand; the rows
// of every tile are padded to an odd length, so strided column reads do not collide in a bank
// either).  Each product accumulates over k in increasing order: results are reproducible.
// Out-of-range rows and columns read a clamped index and are never stored.
constexpr int kTiledMaxP = 64, kTiledMaxN = 128;

template <int RM, int RN>
struct Tile {
  int m0, n0;        // first row of the warp; first column of this lane
  int m[RM], n[RN];  // clamped row / column indices
  __device__ __forceinline__ bool ok(int i, int j, int M, int Nn) const { return m0 + i < M && n0 + 32 * j < Nn; }
};

template <int RM, int RN, int NT = kThreads, class F>
__device__ __forceinline__ void for_tiles(int M, int Nn, F&& f) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mb = (M + RM - 1) / RM, nb = (Nn + 32 * RN - 1) / (32 * RN);
  for (int task = warp; task < mb * nb; task += NT / 32) {
    Tile<RM, RN> tl;
    tl.m0 = (task / nb) * RM;
    tl.n0 = (task % nb) * 32 * RN + lane;
#pragma unroll
    for (int i = 0; i < RM; ++i) tl.m[i] = min(tl.m0 + i, M - 1);
#pragma unroll
    for (int j = 0; j < RN; ++j) tl.n[j] = min(tl.n0 + 32 * j, Nn - 1);
    f(tl);
  }
}

// acc[i][j] += sum_{k < K} a[i][k as] * b[j][k bs] * scale(k)
template <int RM, int RN, typename TA, class FS>
__device__ __forceinline__ void tile_mm(TA (&acc)[RM][RN], const TA* const (&a)[RM], int as, const TA* const (&b)[RN],
                                        int bs, int K, FS scale) {
  for (int k = 0; k < K; ++k) {
    const TA sc = scale(k);
    TA av[RM], bv[RN];
#pragma unroll
    for (int i = 0; i < RM; ++i) av[i] = a[i][k * as];
#pragma unroll
    for (int j = 0; j < RN; ++j) bv[j] = b[j][k * bs] * sc;
#pragma unroll
    for (int i = 0; i < RM; ++i)
#pragma unroll
      for (int j = 0; j < RN; ++j) acc[i][j] += av[i] * bv[j];
  }
}
// two row operands against one column operand: acc1 += a1 b, acc2 += a2 b
template <int RM, int RN, typename TA>
__device__ __forceinline__ void tile_mm_2a(TA (&acc1)[RM][RN], TA (&acc2)[RM][RN], const TA* const (&a1)[RM],
                                           const TA* const (&a2)[RM], int as, const TA* const (&b)[RN], int bs, int K) {
  for (int k = 0; k < K; ++k) {
    TA av1[RM], av2[RM], bv[RN];
#pragma unroll
    for (int i = 0; i < RM; ++i) {
      av1[i] = a1[i][k * as];
      av2[i] = a2[i][k * as];
    }
#pragma unroll
    for (int j = 0; j < RN; ++j) bv[j] = b[j][k * bs];
#pragma unroll
    for (int i = 0; i < RM; ++i)
#pragma unroll
      for (int j = 0; j < RN; ++j) {
        acc1[i][j] += av1[i] * bv[j];
        acc2[i][j] += av2[i] * bv[j];
      }
  }
}
// one row operand against two column operands: acc1 += a b1, acc2 += a b2
template <int RM, int RN, typename TA>
__device__ __forceinline__ void tile_mm_2b(TA (&acc1)[RM][RN], TA (&acc2)[RM][RN], const TA* const (&a)[RM], int as,
                                           const TA* const (&b1)[RN], const TA* const (&b2)[RN], int bs, int K) {
  for (int k = 0; k < K; ++k) {
    TA av[RM], bv1[RN], bv2[RN];
#pragma unroll
    for (int i = 0; i < RM; ++i) av[i] = a[i][k * as];
#pragma unroll
    for (int j = 0; j < RN; ++j) {
      bv1[j] = b1[j][k * bs];
      bv2[j] = b2[j][k * bs];
    }
#pragma unroll
    for (int i = 0; i < RM; ++i)
#pragma unroll
      for (int j = 0; j < RN; ++j) {
        acc1[i][j] += av[i] * bv1[j];
        acc2[i][j] += av[i] * bv2[j];
      }
  }
}
template <typename TA>
struct Unscaled {
  __device__ __forceinline__ TA operator()(int) const { return TA(1); }
};

// The copy loops issue kLoadBatch global loads per thread before any of their shared-memory stores:
// a store between two loads would make the second wait for the first (the compiler cannot prove
// that a generic pointer does not alias shared memory), one memory round trip per element.
constexpr int kLoadBatch = 8;

// rows [0, L) of a [B, T, H, D] view (tokens t0 + t - sh, head hh) -> shared tile [L][D1]; rows
// t >= Lc and tokens before the start of the sequence read as zero
template <typename TA, typename TI, int NT = kThreads>
__device__ __forceinline__ void load_tile(TA* dst, int D1, const View& v, int64_t b, int64_t t0, int sh, int64_t hh,
                                          int L, int D, int Lc) {
  const int total = L * D;
  for (int base = threadIdx.x; base < total; base += NT * kLoadBatch) {
    TA val[kLoadBatch];
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int i = base + u * NT, t = i / D, d = i - t * D;
      val[u] = (i < total && t < Lc && t0 + t >= sh) ? ldv<TA>(v.row<TI>(b, t0 + t - sh, hh) + d) : TA(0);
    }
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int i = base + u * NT, t = i / D, d = i - t * D;
      if (i < total) dst[t * D1 + d] = val[u];
    }
  }
}

// a [P][N] state in global memory (read through L2; zero when src is null) -> shared [P][N1]
template <typename TA, int NT = kThreads>
__device__ __forceinline__ void load_state(TA* dst, int N1, const TA* src, int P, int N) {
  const int total = P * N;
  for (int base = threadIdx.x; base < total; base += NT * kLoadBatch) {
    TA val[kLoadBatch];
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int i = base + u * NT;
      val[u] = (src && i < total) ? ldcg_t(src + i) : TA(0);
    }
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int i = base + u * NT;
      if (i < total) dst[(i / N) * N1 + i % N] = val[u];
    }
  }
}

// the chain update out[i] = a * s[i] + out[i] for a [P][N] state (s in shared memory [P][N1]),
// also written to `copy` when given; returns sum_i s[i] * dot[i] over this thread's elements when
// `dot` (shared [P][N1]) is given
template <typename TA, int NT = kThreads>
__device__ __forceinline__ TA chain_update(TA* out, const TA* s, TA a, int N1, int P, int N, TA* copy, const TA* dot) {
  const int total = P * N;
  TA acc = 0;
  for (int base = threadIdx.x; base < total; base += NT * kLoadBatch) {
    TA val[kLoadBatch];
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int i = base + u * NT;
      val[u] = i < total ? out[i] : TA(0);
    }
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int i = base + u * NT;
      if (i < total) {
        const int si = (i / N) * N1 + i % N;
        const TA v = val[u] + a * s[si];
        out[i] = v;
        if (copy) copy[i] = v;
        if (dot) acc += s[si] * dot[si];
      }
    }
  }
  return acc;
}

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
  const bool tiled = P <= kTiledMaxP && N <= kTiledMaxN;
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
  load_tile<TA, TI>(s_k, N1, p.k, b, t0, 0, g, L, N, Lc);
  load_tile<TA, TI>(s_kp, N1, p.kp, b, t0, sh, g, L, N, Lc);
  if (!state_only) load_tile<TA, TI>(s_q, N1, p.q, b, t0, 0, g, L, N, Lc);
  load_tile<TA, TI>(s_x, P1, p.x, b, t0, 0, h, L, P, Lc);
  load_tile<TA, TI>(s_xp, P1, p.xp, b, t0, sh, h, L, P, Lc);
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
  if (tiled) {
    // rows p, columns n: sum_s x_sp (w_s g_s k_sn) + xp_sp (w_s b_s kp_sn)
    for_tiles<8, 4>(P, N, [&](const Tile<8, 4>& tl) {
      TA acc[8][4] = {};
      const TA* a[8];
      const TA* bb[4];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = s_x + tl.m[i];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) bb[jj] = s_k + tl.n[jj];
      tile_mm(acc, a, P1, bb, N1, Lc, [&](int s) { return s_w[s] * s_g[s]; });
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = s_xp + tl.m[i];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) bb[jj] = s_kp + tl.n[jj];
      tile_mm(acc, a, P1, bb, N1, Lc, [&](int s) { return s_w[s] * s_b[s]; });
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
          if (tl.ok(i, jj, P, N)) slot_out[(tl.m0 + i) * N + tl.n0 + 32 * jj] = acc[i][jj];
    });
  } else {
    for (int i = tid; i < P * N; i += kThreads) {
      const int pp = i / N, n = i % N;
      TA acc = 0;
      for (int s = 0; s < Lc; ++s)
        acc += s_w[s] * (s_g[s] * s_x[s * P1 + pp] * s_k[s * N1 + n] + s_b[s] * s_xp[s * P1 + pp] * s_kp[s * N1 + n]);
      slot_out[i] = acc;
    }
  }
  // masked intra-chunk scores (mamba3.py:41-44)
  if (!state_only && tiled) {
    // rows t, columns s: q_t . k_s and q_t . kp_s
    for_tiles<4, 1>(L, L, [&](const Tile<4, 1>& tl) {
      TA dk[4][1] = {}, dkp[4][1] = {};
      const TA* a[4];
      const TA* b1[1] = {s_k + tl.n[0] * N1};
      const TA* b2[1] = {s_kp + tl.n[0] * N1};
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = s_q + tl.m[i] * N1;
      tile_mm_2b(dk, dkp, a, 1, b1, b2, 1, N);
      const int s = tl.n0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int t = tl.m0 + i;
        if (!tl.ok(i, 0, L, L)) continue;
        TA vg = 0, vb = 0;
        if (s <= t && t < Lc) {
          const TA m = xexp(s_c[t] - s_c[s]);
          vg = dk[i][0] * s_g[s] * m;
          vb = dkp[i][0] * s_b[s] * m;
        }
        s_Sg[t * L1 + s] = vg;
        s_Sb[t * L1 + s] = vb;
      }
    });
  } else if (!state_only) {
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
  if (j == 0) {
    for (int i = tid; i < P * N; i += kThreads) {
      const TA v = p.init ? reinterpret_cast<const TA*>(p.init)[bh * PN + i] : TA(0);
      slot_in[i] = v;
      s_S[(i / N) * N1 + i % N] = v;
    }
  } else {
    load_state(s_S, N1, slot_in, P, N);
  }
  __syncthreads();
  // S_in[j+1] = e^{c_L} S_in[j] + S_loc[j]   (mamba3.py:52)
  const bool last = (j == p.nc - 1);
  chain_update<TA>(slot_out, s_S, a_chunk, N1, P, N, (last && p.fin) ? reinterpret_cast<TA*>(p.fin) + bh * PN : nullptr,
                   nullptr);
  // the barrier orders every thread's ring writes before thread 0's release (cumulative)
  __syncthreads();
  if (tid == 0) st_release(&flags[j + 1], kFlagReady);
  if (state_only) return;

  // y = y_intra + e^{c} (q S_in^T)   (mamba3.py:45,55)
  if (tiled) {
    // rows t, columns p; the scores are zero above the diagonal
    for_tiles<4, 2>(Lc, P, [&](const Tile<4, 2>& tl) {
      TA yi[4][2] = {}, yr[4][2] = {};
      const TA* a[4];
      const TA* bb[2];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = s_Sg + tl.m[i] * L1;
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) bb[jj] = s_x + tl.n[jj];
      tile_mm(yi, a, 1, bb, P1, Lc, Unscaled<TA>());
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = s_Sb + tl.m[i] * L1;
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) bb[jj] = s_xp + tl.n[jj];
      tile_mm(yi, a, 1, bb, P1, Lc, Unscaled<TA>());
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = s_q + tl.m[i] * N1;
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) bb[jj] = s_S + tl.n[jj] * N1;
      tile_mm(yr, a, 1, bb, 1, N, Unscaled<TA>());
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int jj = 0; jj < 2; ++jj)
          if (tl.ok(i, jj, Lc, P)) {
            const int t = tl.m0 + i;
            stv<TA>(p.y.wrow<TI>(b, t0 + t, h) + tl.n0 + 32 * jj, yi[i][jj] + s_ec[t] * yr[i][jj]);
          }
    });
  } else {
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
}

// ---------------------------------------------------------------------------------------------
// backward (reverse chain)
template <typename TI, typename TS, typename TA, int NT>
__global__ void __launch_bounds__(NT) ssd_bwd_simt_kernel(const SimtParams p) {
  // row blocks of the register tiles: twice as many warps take half as many rows each
  constexpr int R4 = NT >= 512 ? 2 : 4, R8 = 2 * R4;
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
  const bool tiled = P <= kTiledMaxP && N <= kTiledMaxN;
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
  load_tile<TA, TI, NT>(s_q, N1, p.q, b, t0, 0, g, L, N, Lc);
  load_tile<TA, TI, NT>(s_dy, P1, p.dy, b, t0, 0, h, L, P, Lc);
  const TA* states_bh = reinterpret_cast<const TA*>(p.chain) + bh * (int64_t)(p.nc + 1) * PN;
  if (!state_only) {
    load_tile<TA, TI, NT>(s_k, N1, p.k, b, t0, 0, g, L, N, Lc);
    load_tile<TA, TI, NT>(s_kp, N1, p.kp, b, t0, sh, g, L, N, Lc);
    load_tile<TA, TI, NT>(s_x, P1, p.x, b, t0, 0, h, L, P, Lc);
    load_tile<TA, TI, NT>(s_xp, P1, p.xp, b, t0, sh, h, L, P, Lc);
    load_state<TA, NT>(s_S, N1, states_bh + (int64_t)j * PN, P, N);
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
  // score-gradient terms of one (t, s): A, Ap, E, Ep and the products whose sums give dc, dgamma, dbeta
  auto score_terms = [&](int t, int s, TA qk, TA qkp, TA da, TA dap) {
    TA vA = 0, vAp = 0, vE = 0, vEp = 0, z = 0, zg = 0, zb = 0;
    if (s <= t && t < Lc) {
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
  };
  if (!state_only && tiled) {
    // rows t, columns s: q_t . k_s, q_t . kp_s, dy_t . x_s, dy_t . xp_s
    for_tiles<R4, 1, NT>(L, L, [&](const Tile<R4, 1>& tl) {
      TA qk[R4][1] = {}, qkp[R4][1] = {}, da[R4][1] = {}, dap[R4][1] = {};
      const TA* a[R4];
      const TA* b1[1] = {s_k + tl.n[0] * N1};
      const TA* b2[1] = {s_kp + tl.n[0] * N1};
#pragma unroll
      for (int i = 0; i < R4; ++i) a[i] = s_q + tl.m[i] * N1;
      tile_mm_2b(qk, qkp, a, 1, b1, b2, 1, N);
      const TA* c1[1] = {s_x + tl.n[0] * P1};
      const TA* c2[1] = {s_xp + tl.n[0] * P1};
#pragma unroll
      for (int i = 0; i < R4; ++i) a[i] = s_dy + tl.m[i] * P1;
      tile_mm_2b(da, dap, a, 1, c1, c2, 1, P);
#pragma unroll
      for (int i = 0; i < R4; ++i)
        if (tl.ok(i, 0, L, L)) score_terms(tl.m0 + i, tl.n0, qk[i][0], qkp[i][0], da[i][0], dap[i][0]);
    });
  }
  if (!state_only) {
    for (int i = tid; !tiled && i < L * L; i += NT) {
      const int t = i / L, s = i % L;
      TA qk = 0, qkp = 0, da = 0, dap = 0;
      if (s <= t && t < Lc) {
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
      }
      score_terms(t, s, qk, qkp, da, dap);
    }
    __syncthreads();
    // one warp per token u: dc_u = sum_s Z[u][s] - sum_t Z[t][u]; dgamma_u, dbeta_u = column sums
    for (int u = warp; u < L; u += NT / 32) {
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
  if (tiled) {
    // rows p, columns n: sum_t dy_tp (e^{c_t} q_tn)
    for_tiles<R8, 4, NT>(P, N, [&](const Tile<R8, 4>& tl) {
      TA acc[R8][4] = {};
      const TA* a[R8];
      const TA* bb[4];
#pragma unroll
      for (int i = 0; i < R8; ++i) a[i] = s_dy + tl.m[i];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) bb[jj] = s_q + tl.n[jj];
      tile_mm(acc, a, P1, bb, N1, Lc, [&](int t) { return s_ec[t]; });
#pragma unroll
      for (int i = 0; i < R8; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
          if (tl.ok(i, jj, P, N)) gslot_out[(tl.m0 + i) * N + tl.n0 + 32 * jj] = acc[i][jj];
    });
  } else {
    for (int i = tid; i < P * N; i += NT) {
      const int pp = i / N, n = i % N;
      TA acc = 0;
      for (int t = 0; t < Lc; ++t) acc += s_ec[t] * s_dy[t * P1 + pp] * s_q[t * N1 + n];
      gslot_out[i] = acc;
    }
  }
  __syncthreads();
  const bool last = (j == p.nc - 1);
  if (tid == 0) s_ready = last ? kFlagReady : wait_flag(&flags[j + 1], p.status);
  __syncthreads();
  if (s_ready != kFlagReady) {
    if (tid == 0) st_release(&flags[j], kFlagAbort);
    return;
  }
  load_state<TA, NT>(s_G, N1, last ? (p.dfin ? reinterpret_cast<const TA*>(p.dfin) + bh * PN : nullptr) : gslot_in, P, N);
  __syncthreads();
  // G[j] = dS_in_loc + e^{c_L} Gn ;  da = <Gn, S_in>
  TA da_part = chain_update<TA, NT>(gslot_out, s_G, a_chunk, N1, P, N,
                                (j == 0 && p.dinit) ? reinterpret_cast<TA*>(p.dinit) + bh * PN : nullptr,
                                state_only ? nullptr : s_S);
  // the barrier orders every thread's ring writes before thread 0's release (cumulative)
  __syncthreads();
  if (tid == 0) st_release(&flags[j], kFlagReady);
  if (state_only) return;
  da_part = warp_sum(da_part);
  if (lane == 0) s_red[warp] = da_part;
  __syncthreads();

  // dx, dxp and the state-term dot products x_s . u_s, xp_s . up_s (u_s = Gn k_s, up_s = Gn kp_s)
  if (tiled) {
    // rows s, columns p (one warp covers all P <= 64 columns of its rows)
    for_tiles<R4, 2, NT>(Lc, P, [&](const Tile<R4, 2>& tl) {
      TA vx[R4][2] = {}, vxp[R4][2] = {}, uu[R4][2] = {}, up[R4][2] = {};
      const TA* a1[R4];
      const TA* a2[R4];
      const TA* bb[2];
#pragma unroll
      for (int i = 0; i < R4; ++i) {
        a1[i] = s_A + tl.m[i];
        a2[i] = s_Ap + tl.m[i];
      }
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) bb[jj] = s_dy + tl.n[jj];
      tile_mm_2a(vx, vxp, a1, a2, L1, bb, P1, Lc);  // sum_t A[t][s] dy_tp (zero for t < s)
#pragma unroll
      for (int i = 0; i < R4; ++i) {
        a1[i] = s_k + tl.m[i] * N1;
        a2[i] = s_kp + tl.m[i] * N1;
      }
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) bb[jj] = s_G + tl.n[jj] * N1;
      tile_mm_2a(uu, up, a1, a2, 1, bb, 1, N);
#pragma unroll
      for (int i = 0; i < R4; ++i) {
        const int sr = tl.m0 + i;
        const int sc = tl.m[i];
        TA xu = 0, xpu = 0;
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          if (!tl.ok(i, jj, Lc, P)) continue;
          const int pp = tl.n0 + 32 * jj;
          stv<TA>(p.dx.wrow<TI>(b, t0 + sr, h) + pp, vx[i][jj] + s_w[sc] * s_g[sc] * uu[i][jj]);
          stv<TA>(p.dxp.wrow<TI>(b, t0 + sr, h) + pp, vxp[i][jj] + s_w[sc] * s_b[sc] * up[i][jj]);
          xu += s_x[sc * P1 + pp] * uu[i][jj];
          xpu += s_xp[sc * P1 + pp] * up[i][jj];
        }
        xu = warp_sum(xu);
        xpu = warp_sum(xpu);
        if (lane == 0 && sr < Lc) {
          s_xu[sr] = xu;
          s_xpu[sr] = xpu;
        }
      }
    });
  } else {
    for (int s = warp; s < Lc; s += NT / 32) {
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
  }
  const bool grouped = p.G != p.H;
  auto store_dq = [&](int t, int n, TA v) {
    if (grouped) reinterpret_cast<TA*>(p.grp)[((b * p.T + t0 + t) * p.H + h) * 3 * N + n] = v;
    else stv<TA>(p.dq.wrow<TI>(b, t0 + t, h) + n, v);
  };
  auto store_dk = [&](int s, int n, TA vk, TA vkp) {
    if (grouped) {
      TA* gp = reinterpret_cast<TA*>(p.grp) + ((b * p.T + t0 + s) * p.H + h) * 3 * N;
      gp[N + n] = vk;
      gp[2 * N + n] = vkp;
    } else {
      stv<TA>(p.dk.wrow<TI>(b, t0 + s, h) + n, vk);
      stv<TA>(p.dkp.wrow<TI>(b, t0 + s, h) + n, vkp);
    }
  };
  if (tiled) {
    // dq: rows t, columns n (one warp covers all N <= 128 columns of its rows):
    // sum_s E[t][s] (g_s k_sn) + Ep[t][s] (b_s kp_sn) + e^{c_t} r_tn, r_tn = sum_p dy_tp S_pn;
    // dc_t += e^{c_t} q_t . r_t
    for_tiles<R4, 4, NT>(Lc, N, [&](const Tile<R4, 4>& tl) {
      TA acc[R4][4] = {}, r[R4][4] = {};
      const TA* a[R4];
      const TA* bb[4];
#pragma unroll
      for (int i = 0; i < R4; ++i) a[i] = s_E + tl.m[i] * L1;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) bb[jj] = s_k + tl.n[jj];
      tile_mm(acc, a, 1, bb, N1, Lc, [&](int sv) { return s_g[sv]; });
#pragma unroll
      for (int i = 0; i < R4; ++i) a[i] = s_Ep + tl.m[i] * L1;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) bb[jj] = s_kp + tl.n[jj];
      tile_mm(acc, a, 1, bb, N1, Lc, [&](int sv) { return s_b[sv]; });
#pragma unroll
      for (int i = 0; i < R4; ++i) a[i] = s_dy + tl.m[i] * P1;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) bb[jj] = s_S + tl.n[jj];
      tile_mm(r, a, 1, bb, N1, P, Unscaled<TA>());
#pragma unroll
      for (int i = 0; i < R4; ++i) {
        const int t = tl.m0 + i;
        const TA ect = s_ec[tl.m[i]];
        TA dct = 0;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          if (!tl.ok(i, jj, Lc, N)) continue;
          const int n = tl.n0 + 32 * jj;
          store_dq(t, n, acc[i][jj] + ect * r[i][jj]);
          dct += ect * s_q[t * N1 + n] * r[i][jj];
        }
        dct = warp_sum(dct);
        if (lane == 0 && t < Lc) s_dc[t] += dct;
      }
    });
    // dk, dkp: rows s, columns n: g_s (sum_t E[t][s] q_tn + w_s sum_p x_sp Gn_pn), likewise with Ep, xp, b
    for_tiles<R4, 4, NT>(Lc, N, [&](const Tile<R4, 4>& tl) {
      TA e[R4][4] = {}, ep[R4][4] = {}, gx[R4][4] = {}, gxp[R4][4] = {};
      const TA* a1[R4];
      const TA* a2[R4];
      const TA* bb[4];
#pragma unroll
      for (int i = 0; i < R4; ++i) {
        a1[i] = s_E + tl.m[i];
        a2[i] = s_Ep + tl.m[i];
      }
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) bb[jj] = s_q + tl.n[jj];
      tile_mm_2a(e, ep, a1, a2, L1, bb, N1, Lc);  // zero for t < s
#pragma unroll
      for (int i = 0; i < R4; ++i) {
        a1[i] = s_x + tl.m[i] * P1;
        a2[i] = s_xp + tl.m[i] * P1;
      }
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) bb[jj] = s_G + tl.n[jj];
      tile_mm_2a(gx, gxp, a1, a2, 1, bb, N1, P);
#pragma unroll
      for (int i = 0; i < R4; ++i) {
        const int sc = tl.m[i];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
          if (tl.ok(i, jj, Lc, N))
            store_dk(tl.m0 + i, tl.n0 + 32 * jj, s_g[sc] * (e[i][jj] + s_w[sc] * gx[i][jj]),
                     s_b[sc] * (ep[i][jj] + s_w[sc] * gxp[i][jj]));
      }
    });
  } else {
    // dq (intra + inter) and its contribution to dc: one warp per token t, lanes over n
    for (int t = warp; t < Lc; t += NT / 32) {
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
    for (int i = tid; i < Lc * N; i += NT) {
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
  }
  __syncthreads();
  // per-token scalar gradients; warp 0 owns the chunk's tokens (L <= 32)
  if (warp == 0) {
    TA da = 0;
    for (int wi = 0; wi < NT / 32; ++wi) da += s_red[wi];
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
    // the backward holds one CTA per SM (its tiles fill shared memory): fp32 accumulation runs it with
    // 512 threads so that twice the warps hide the latencies; fp64 keeps 256 (register file)
    constexpr int kBwdNT = sizeof(TA) == 4 ? 2 * kThreads : kThreads;
    auto k = ssd_bwd_simt_kernel<TI, TS, TA, kBwdNT>;
    if (dyn_smem(reinterpret_cast<const void*>(k), (int)smem) != ZB_OK) return ZB_ERR_CUDA;
    k<<<grid, dim3(kBwdNT), smem, stream>>>(p);
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
