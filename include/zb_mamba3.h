/*
 * zb_mamba3.h — C ABI of the Mamba-3 layer body around the SSD scan (libzenith_ssd.so).
 *
 * Replaces the part of the reference's Mamba3.forward between the in_proj split and out_proj
 * (zenith/mamba3.py:96-119) except the scan itself, which is zb_ssd_fwd / zb_ssd_bwd:
 *   prologue  (mamba3.py:105-116): A = -min(heavy_tail(dd_A), -A_floor); DT = softplus(dd_dt + dt_bias);
 *             adt = A DT; tr = sigmoid(trap); gamma = tr DT; beta = (1-tr) DT e^{adt};
 *             theta = cumsum_t(DT ang); q = rope(rmsnorm(Cm) + C_bias, theta);
 *             k = rope(rmsnorm(Bm) + B_bias, theta); kp, xp = k, x one token later (zero first)
 *   epilogue  (mamba3.py:119): out = (y + D x) * silu(z)
 * A layer step is: zb_m3_prologue_fwd -> zb_ssd_fwd -> zb_m3_epilogue_fwd, and backward
 * zb_m3_epilogue_bwd -> zb_ssd_bwd -> zb_m3_prologue_bwd.
 *
 * Sizes: H <= 128 heads with H P <= 8192 (more than 31 heads run in groups of at most 28),
 * N % 16 == 0 and N <= 128 (N/4 RoPE angles rotate the first N/2 features), P <= 256.  Layer inputs may be strided views (the in_proj split); scan operands and
 * scan gradients are contiguous and 16-byte aligned.  All kernels are deterministic (fixed-order reductions).
 */
#ifndef ZB_MAMBA3_H
#define ZB_MAMBA3_H

#include "zb_ssd.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
  int64_t B, T, H, P, N;
  float A_floor, eps;  /* Mamba3.A_floor (mamba3.py:73), RMSNorm eps (mamba3.py:9)                   */
  int32_t io_dtype;    /* ZB_F32 / ZB_BF16: x, z, Bm, Cm, dd_dt, dd_A, trap, ang, out, dout, gradients */
  int32_t op_dtype;    /* ZB_F32 / ZB_BF16: scan operands q, k_ext, xp, scan output y, dy, scan grads  */
  /* layer inputs: x, z [B,T,H,P] (z may be NULL: no gate); Bm, Cm [B,T,N] and ang [B,T,N/4]
     (sh unused); dd_dt, dd_A, trap [B,T,H] */
  zb_view x, z, Bm, Cm, dd_dt, dd_A, trap, ang;
  /* parameters, contiguous fp32: dt_bias [H], B_bias [H,N], C_bias [H,N], B_norm_w [N],
     C_norm_w [N], D [H] */
  const float *dt_bias, *B_bias, *C_bias, *B_norm_w, *C_norm_w, *D;
  /* scan operands written by the prologue, contiguous: q [B,T,H,N]; k_ext [B,T+1,H,N] (rows
     1..T are k, rows 0..T-1 are kp); xp [B,T,H,P], or NULL when the scan reads x one token
     earlier itself (ZB_FLAG_SHIFTED); adt, gamma, beta fp32 [B,T,H]; theta fp32 [B,T,H,N/4]
     (kept for the backward) */
  void *q, *k_ext, *xp;
  float *adt, *gamma, *beta, *theta;
  /* scan output y (contiguous [B,T,H,P]) and the layer output out [B,T,H,P] (view) */
  const void* y;
  zb_view out;
  /* backward: dout [B,T,H,P] (view); dy written for the scan backward (contiguous); the scan's
     gradients (contiguous): dxs, dxp [B,T,H,P], dq, dk, dkp [B,T,H,N], dadt, dgamma, dbeta fp32 */
  zb_view dout;
  void* dy;
  const void *dxs, *dxp, *dq, *dk, *dkp;
  const float *dadt, *dgamma, *dbeta;
  /* layer gradients: views shaped like the inputs (dz unused without z); parameter gradients
     contiguous fp32, overwritten */
  zb_view dx, dz, dBm, dCm, ddd_dt, ddd_A, dtrap, dang;
  float *ddt_bias, *dB_bias, *dC_bias, *dB_norm_w, *dC_norm_w, *dD;
  /* scratch (from zb_m3_workspace_bytes), 256-byte aligned; the same buffer must be passed to
     zb_m3_epilogue_bwd and the zb_m3_prologue_bwd that follows it */
  void* workspace;
  uint64_t workspace_bytes;
  /* device int32 status word (zb_m3_prologue_bwd): a bounded wait on its row copies that gives up
     after about a second records ZB_ERR_TIMEOUT there and the kernel returns */
  int32_t* status;
  /* continuing a sequence (zb_m3_prologue_fwd; decode): theta0 [B,H,N/4] fp32, theta after the
     tokens before this call (NULL: zero); kp0 [B,H,N] op dtype, k of the token before this call,
     written to k_ext row 0 (NULL: zeros, the sequence start) */
  const float* theta0;
  const void* kp0;
} zb_m3_args;

/* scratch bytes the four calls need (the maximum over them) */
ZB_API uint64_t zb_m3_workspace_bytes(const zb_m3_args* args);
/* q, k_ext, xp, adt, gamma, beta, theta from the layer inputs     (replaces mamba3.py:105-116) */
ZB_API int zb_m3_prologue_fwd(const zb_m3_args* args, void* stream);
/* out = (y + D x) * silu(z)                                        (replaces mamba3.py:119)     */
ZB_API int zb_m3_epilogue_fwd(const zb_m3_args* args, void* stream);
/* from dout: dy for the scan backward, dz, and the D gradient's partial sums (in workspace)   */
ZB_API int zb_m3_epilogue_bwd(const zb_m3_args* args, void* stream);
/* from the scan's gradients and dy (as zb_m3_epilogue_bwd wrote it): dx, dBm, dCm, ddd_dt,
   ddd_A, dtrap, dang and all parameter grads */
ZB_API int zb_m3_prologue_bwd(const zb_m3_args* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ZB_MAMBA3_H */
