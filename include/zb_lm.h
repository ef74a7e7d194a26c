/*
 * zb_lm.h — C ABI of the language-model kernels around the Mamba-3 layers (libzenith_ssd.so).
 *
 * They replace, in the reference's ZenithForCausalLM (zenith/model.py:42-99):
 *   zb_rmsnorm_fwd / zb_rmsnorm_bwd   the residual add and the RMSNorm that reads it:
 *       Layer.forward  x + mixer(norm(x))          (model.py:48-49)
 *       recurrent_norm(s + x), norm(s)             (model.py:87,93)
 *       RMSNorm        x rsqrt(mean(x^2) + eps) w  (zenith/mamba3.py:8-15)
 *     as one pass: s = a + b (b optional), u = s r w with r = rsqrt(mean(s^2) + eps), and back:
 *     dsum = ds + r w du - s r^3 / D sum(du w s)  (the gradient of both a and b), dw = sum du s r.
 *   zb_xent                           the next-token cross-entropy over the LM head's logits,
 *       F.cross_entropy(logits[:, :-1].float(), labels[:, 1:])   (model.py:95-97)
 *     per row: loss = logsumexp(l) - l[label], and (optionally) the row's logit gradient
 *     softmax(l) - onehot(label), written over the logits in the same pass.
 *
 * Tensors are dense row-major [M, D] / [M, V] (row strides as given), no torch types cross the
 * boundary, every entry point returns a zb_status code and launches on `stream`.  Results are
 * bitwise reproducible (fixed-order reductions; the dw partials use a fixed grid).
 */
#ifndef ZB_LM_H
#define ZB_LM_H

#include "zb_ssd.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
  int64_t M, D;       /* rows, features (D <= 8192) */
  float eps;          /* RMSNorm eps (mamba3.py:9) */
  int32_t x_dtype;    /* ZB_F32 / ZB_BF16: a, s, ds, dsum (the residual stream) */
  int32_t b_dtype;    /* ZB_F32 / ZB_BF16: b, dsum_b (the layer output added to it) */
  int32_t u_dtype;    /* ZB_F32 / ZB_BF16: u, du (the normalised output) */
  /* forward */
  const void* a;      /* [M, D] */
  const void* b;      /* [M, D] or NULL */
  void* s;            /* [M, D]: a + b, written when b != NULL (NULL allowed when b == NULL) */
  const float* w;     /* [D] */
  void* u;            /* [M, D] */
  float* r;           /* [M] the RMSNorm factor, kept for the backward (may be NULL in the forward) */
  /* backward (s = the forward's sum, or a when there was no b) */
  const void* du;     /* [M, D] */
  const void* ds;     /* [M, D] gradient reaching s from its other uses (the residual), or NULL */
  void* dsum;         /* [M, D] */
  void* dsum_b;       /* [M, D] dsum in b_dtype (b's gradient), or NULL */
  float* dw;          /* [D], overwritten */
  void* workspace;    /* zb_rmsnorm_workspace_bytes(), 256-byte aligned */
  uint64_t workspace_bytes;
} zb_rmsnorm_args;

ZB_API uint64_t zb_rmsnorm_workspace_bytes(const zb_rmsnorm_args* args);
/* s = a + b (if b), u = s r w, r saved                       (replaces model.py:48-49,87,93 + mamba3.py:14-15) */
ZB_API int zb_rmsnorm_fwd(const zb_rmsnorm_args* args, void* stream);
/* dsum = ds + RMSNorm backward of du; dw                     (the autograd backward of the same) */
ZB_API int zb_rmsnorm_bwd(const zb_rmsnorm_args* args, void* stream);

typedef struct {
  int64_t M, V;          /* rows (tokens), vocabulary */
  int64_t ld;            /* row stride of logits, in elements (>= V) */
  int32_t dtype;         /* ZB_BF16 / ZB_F32 logits */
  int32_t write_grad;    /* nonzero: overwrite each row with softmax - onehot (zeros for ignored rows) */
  int64_t ignore_index;  /* rows with this label contribute nothing (F.cross_entropy's -100) */
  void* logits;          /* [M, ld] */
  const int64_t* labels; /* [M] */
  float* loss;           /* [M]: logsumexp - logit[label]; 0 for ignored rows */
  float* lse;            /* [M] logsumexp, or NULL */
  int32_t* status;       /* device word: a label outside [0, V) (not ignore_index) sets ZB_ERR_INDEX there
                            and the row is treated as ignored */
} zb_xent_args;

/* per-row cross-entropy and logit gradient in one pass        (replaces model.py:95-97) */
ZB_API int zb_xent(const zb_xent_args* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ZB_LM_H */
