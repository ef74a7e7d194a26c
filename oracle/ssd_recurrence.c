/*
 * Oracle for long sequences: TEST INFRASTRUCTURE ONLY (never linked into libzenith_ssd.so; only
 * the tests and __graft_entry__.smoke() load it, as a checker of the CUDA kernels).
 *
 * The SSD scan of zenith/mamba3.py:30-56 in its per-token (recurrent) form, in double precision,
 * with the adjoint of that recurrence for all eight input gradients.  It needs O(P N) memory per
 * head and a checkpoint of the state every CKPT tokens, so it checks sequences the chunked
 * float64 oracle (and the reference's autograd, O(T * chunk) memory) cannot hold.
 *
 * Forward, per (batch b, head h); head h reads q / k / kp of group h / (H / G)
 * (the reference test's naive recurrence, tests/test_mamba3.py:10-21):
 *     h_t = e^{adt_t} h_{t-1} + gamma_t x_t k_t^T + beta_t xp_t kp_t^T        (P x N)
 *     y_t = h_t q_t                                                           h_{-1} = initial state
 * Backward: the adjoint lam_t = dL/dh_t runs from the last token to the first (the formulation
 * of mojo/ssd_bwd.mojo:98-144, extended to kp / xp, the initial and the final state):
 *     lam_{T-1} = dy_{T-1} q_{T-1}^T + dfinal,   lam_t = dy_t q_t^T + e^{adt_{t+1}} lam_{t+1}
 *     dx_t = gamma_t lam_t k_t        dxp_t = beta_t lam_t kp_t
 *     dk_t = gamma_t lam_t^T x_t      dkp_t = beta_t lam_t^T xp_t      dq_t = h_t^T dy_t
 *     dgamma_t = x_t . lam_t k_t      dbeta_t = xp_t . lam_t kp_t
 *     dadt_t = e^{adt_t} <lam_t, h_{t-1}>                              dinit = e^{adt_0} lam_0
 * dq / dk / dkp are summed over the heads of a group.
 *
 * Every row p of the state evolves on its own, so both directions run the rows in parallel
 * (OpenMP).  The backward walks one head at a time and, per block of CKPT tokens, sums the rows'
 * contributions to dq / dk / dkp / dgamma / dbeta / dadt in row order (deterministic).
 *
 * Layouts (contiguous, double): x, xp, y, dy, dx, dxp [B, T, H, P]; q, k, kp, dq, dk, dkp
 * [B, T, G, N]; adt, gamma, beta and their gradients [B, T, H]; states [B, H, P, N].
 * Returns 0, or -1 on bad sizes / a failed allocation.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define CKPT 64

typedef struct {
  int64_t B, T, H, G, P, N;
} dims_t;

static int dims_ok(const dims_t* d) {
  return d->B > 0 && d->T > 0 && d->H > 0 && d->G > 0 && d->P > 0 && d->N > 0 && d->H % d->G == 0;
}

/* one step of a state row: row = a row + g xv k + b xpv kp; returns row . q (q may be NULL) */
static inline double step_row(double* row, int64_t N, double a, double gx, const double* k, double bx,
                              const double* kp, const double* q) {
  double acc = 0.0;
  for (int64_t n = 0; n < N; ++n) {
    const double v = a * row[n] + gx * k[n] + bx * kp[n];
    row[n] = v;
    if (q) acc += v * q[n];
  }
  return acc;
}

int zb_oracle_recurrence_fwd(int64_t B, int64_t T, int64_t H, int64_t G, int64_t P, int64_t N, const double* x,
                             const double* q, const double* k, const double* kp, const double* xp, const double* adt,
                             const double* gamma, const double* beta, const double* init, double* y, double* fin) {
  const dims_t d = {B, T, H, G, P, N};
  if (!dims_ok(&d) || !x || !q || !k || !kp || !xp || !adt || !gamma || !beta || !y) return -1;
  const int64_t r = H / G;
  int failed = 0;
#pragma omp parallel for collapse(3) schedule(dynamic, 4)
  for (int64_t b = 0; b < B; ++b) {
    for (int64_t h = 0; h < H; ++h) {
      for (int64_t p = 0; p < P; ++p) { /* every state row evolves on its own */
        double* row = (double*)malloc(sizeof(double) * N);
        if (!row) {
#pragma omp atomic write
          failed = 1;
          continue;
        }
        const int64_t g = h / r;
        if (init)
          memcpy(row, init + ((b * H + h) * P + p) * N, sizeof(double) * N);
        else
          memset(row, 0, sizeof(double) * N);
        for (int64_t t = 0; t < T; ++t) {
          const int64_t bt = b * T + t, ih = bt * H + h, ig = (bt * G + g) * N, iv = ih * P + p;
          y[iv] = step_row(row, N, exp(adt[ih]), gamma[ih] * x[iv], k + ig, beta[ih] * xp[iv], kp + ig, q + ig);
        }
        if (fin) memcpy(fin + ((b * H + h) * P + p) * N, row, sizeof(double) * N);
        free(row);
      }
    }
  }
  return failed ? -1 : 0;
}

int zb_oracle_recurrence_bwd(int64_t B, int64_t T, int64_t H, int64_t G, int64_t P, int64_t N, const double* x,
                             const double* q, const double* k, const double* kp, const double* xp, const double* adt,
                             const double* gamma, const double* beta, const double* init, const double* dy,
                             const double* dfinal, double* dx, double* dq, double* dk, double* dkp, double* dxp,
                             double* dadt, double* dgamma, double* dbeta, double* dinit) {
  const dims_t d = {B, T, H, G, P, N};
  if (!dims_ok(&d) || !x || !q || !k || !kp || !xp || !adt || !gamma || !beta || !dy) return -1;
  if (!dx || !dq || !dk || !dkp || !dxp || !dadt || !dgamma || !dbeta) return -1;
  const int64_t r = H / G;
  const int64_t nblk = (T + CKPT - 1) / CKPT;
  memset(dq, 0, sizeof(double) * B * T * G * N);
  memset(dk, 0, sizeof(double) * B * T * G * N);
  memset(dkp, 0, sizeof(double) * B * T * G * N);
  /* per head, per row p: checkpoints (the state entering each block of CKPT tokens), the states
     inside the current block, the adjoint row, and the row's contributions to the sums over p
     for the current block (dk, dkp, dq rows and dgamma, dbeta, dadt) */
  double* ck = (double*)malloc(sizeof(double) * P * nblk * N);
  double* hs = (double*)malloc(sizeof(double) * P * (CKPT + 1) * N);
  double* lam = (double*)malloc(sizeof(double) * P * N);
  double* part = (double*)malloc(sizeof(double) * P * CKPT * (3 * N + 3));
  if (!ck || !hs || !lam || !part) {
    free(ck);
    free(hs);
    free(lam);
    free(part);
    return -1;
  }
  const int64_t pstride = CKPT * (3 * N + 3); /* one row's block of partial sums */
  for (int64_t b = 0; b < B; ++b) {
    for (int64_t h = 0; h < H; ++h) {
      const int64_t g = h / r;
      /* forward sweep, rows in parallel: checkpoints */
#pragma omp parallel for schedule(static)
      for (int64_t p = 0; p < P; ++p) {
        double* row = hs + p * (CKPT + 1) * N;
        if (init)
          memcpy(row, init + ((b * H + h) * P + p) * N, sizeof(double) * N);
        else
          memset(row, 0, sizeof(double) * N);
        for (int64_t t = 0; t < T; ++t) {
          if (t % CKPT == 0) memcpy(ck + (p * nblk + t / CKPT) * N, row, sizeof(double) * N);
          const int64_t bt = b * T + t, ih = bt * H + h, ig = (bt * G + g) * N, iv = ih * P + p;
          step_row(row, N, exp(adt[ih]), gamma[ih] * x[iv], k + ig, beta[ih] * xp[iv], kp + ig, NULL);
        }
        if (dfinal)
          memcpy(lam + p * N, dfinal + ((b * H + h) * P + p) * N, sizeof(double) * N);
        else
          memset(lam + p * N, 0, sizeof(double) * N);
      }
      /* reverse sweep, one block at a time: each row recomputes the block's states and runs its
         adjoint; then the row contributions are summed over p in row order */
      for (int64_t blk = nblk - 1; blk >= 0; --blk) {
        const int64_t t0 = blk * CKPT, t1 = (t0 + CKPT < T) ? t0 + CKPT : T;
#pragma omp parallel for schedule(static)
        for (int64_t p = 0; p < P; ++p) {
          double* hp = hs + p * (CKPT + 1) * N; /* hp[0] = h_{t0-1} */
          double* lp = lam + p * N;
          double* pp = part + p * pstride;
          memcpy(hp, ck + (p * nblk + blk) * N, sizeof(double) * N);
          for (int64_t t = t0; t < t1; ++t) {
            const int64_t bt = b * T + t, ih = bt * H + h, ig = (bt * G + g) * N, iv = ih * P + p;
            double* nx = hp + (t - t0 + 1) * N;
            memcpy(nx, hp + (t - t0) * N, sizeof(double) * N);
            step_row(nx, N, exp(adt[ih]), gamma[ih] * x[iv], k + ig, beta[ih] * xp[iv], kp + ig, NULL);
          }
          for (int64_t t = t1 - 1; t >= t0; --t) {
            const int64_t bt = b * T + t, ih = bt * H + h, ig = (bt * G + g) * N, iv = ih * P + p;
            /* e^{adt_{t+1}}, or 1 at the last token, where lam holds dfinal */
            const double a_next = (t == T - 1) ? 1.0 : exp(adt[ih + H]);
            const double* ht = hp + (t - t0 + 1) * N;
            const double* hprev = hp + (t - t0) * N;
            const double dyv = dy[iv], xv = x[iv], xpv = xp[iv], gm = gamma[ih], bt_ = beta[ih];
            const double* qt = q + ig;
            const double* kt = k + ig;
            const double* kpt = kp + ig;
            double* pk = pp + (t - t0) * (3 * N + 3);
            double* pkp = pk + N;
            double* pq = pk + 2 * N;
            double lk = 0.0, lkp = 0.0, lh = 0.0;
            for (int64_t n = 0; n < N; ++n) {
              const double l = dyv * qt[n] + a_next * lp[n];
              lp[n] = l;
              lk += l * kt[n];
              lkp += l * kpt[n];
              lh += l * hprev[n];
              pk[n] = gm * xv * l;
              pkp[n] = bt_ * xpv * l;
              pq[n] = dyv * ht[n];
            }
            dx[iv] = gm * lk;
            dxp[iv] = bt_ * lkp;
            pk[3 * N] = xv * lk;                 /* dgamma */
            pk[3 * N + 1] = xpv * lkp;           /* dbeta */
            pk[3 * N + 2] = exp(adt[ih]) * lh;   /* dadt */
          }
        }
#pragma omp parallel for schedule(static)
        for (int64_t t = t0; t < t1; ++t) {
          const int64_t bt = b * T + t, ih = bt * H + h, ig = (bt * G + g) * N;
          double sg = 0.0, sb = 0.0, sa = 0.0;
          for (int64_t p = 0; p < P; ++p) {
            const double* pk = part + p * pstride + (t - t0) * (3 * N + 3);
            for (int64_t n = 0; n < N; ++n) {
              dk[ig + n] += pk[n];
              dkp[ig + n] += pk[N + n];
              dq[ig + n] += pk[2 * N + n];
            }
            sg += pk[3 * N];
            sb += pk[3 * N + 1];
            sa += pk[3 * N + 2];
          }
          dgamma[ih] = sg;
          dbeta[ih] = sb;
          dadt[ih] = sa;
        }
      }
      if (dinit) {
        const double a0 = exp(adt[(b * T) * H + h]);
        for (int64_t p = 0; p < P; ++p)
          for (int64_t n = 0; n < N; ++n) dinit[((b * H + h) * P + p) * N + n] = a0 * lam[p * N + n];
      }
    }
  }
  free(ck);
  free(hs);
  free(lam);
  free(part);
  return 0;
}
