"""CPU oracle for the fused Mamba-3 SSD layer body: TEST INFRASTRUCTURE ONLY.

Restates in float64 PyTorch the part of the reference's ``Mamba3.forward`` between the
``in_proj`` split and ``out_proj`` (zenith/mamba3.py:96-119), with its helpers ``RMSNorm``
(:8-15), ``heavy_tail`` (:18-19) and ``rope`` (:22-27), around the SSD scan of
``oracle.ssd_oracle``.  It checks the CUDA prologue / epilogue kernels of ``zenith_b200``;
only the tests may import it.  Gradients come from PyTorch autograd through this
restatement, with the scan's backward written out in ``oracle.ssd_oracle``.

Pinning: ``tests/test_oracle.py`` checks it against golden vectors that
``tests/golden/make_golden.py`` writes by running the reference ``Mamba3`` module itself
(``in_proj`` / ``out_proj`` replaced by identities, autograd; the module runs in float32, as
its forward upcasts to it).

Per token t, head h (B, C are the per-token state projections, shared by all heads):
    A     = -min(heavy_tail(dd_A), -A_floor)         (mamba3.py:105; = A_floor when A_floor > 0)
    DT    = softplus(dd_dt + dt_bias_h)              (:106)
    adt   = A DT;  tr = sigmoid(trap)                (:107-108)
    gamma = tr DT;  beta = (1 - tr) DT e^{adt}       (:109-110)
    theta = cumsum_t(DT * ang)                       (:111, over the whole sequence)
    q     = rope(rmsnorm(C) + C_bias_h, theta)       (:113)
    k     = rope(rmsnorm(B) + B_bias_h, theta)       (:114)
    xp, kp = x, k shifted one token later, zero at t = 0   (:115-116)
    out   = (ssd(x, q, k, kp, xp, adt, gamma, beta) + D_h x) * silu(z)   (:118-119)
"""

from __future__ import annotations

import torch

from oracle import ssd_oracle

F64 = torch.float64


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def heavy_tail(x: torch.Tensor) -> torch.Tensor:
    return x.clamp(min=0) + 1.0 / (1.0 - x.clamp(max=0))


def softplus(x: torch.Tensor) -> torch.Tensor:
    """log(1 + e^x), and x itself above 20 (torch.nn.functional.softplus's threshold)."""
    return torch.where(x > 20, x, torch.log1p(torch.exp(x.clamp(max=20))))


def rope(v: torch.Tensor, theta: torch.Tensor) -> torch.Tensor:
    """Rotate pairs (2i, 2i+1) of the first 2 * theta.shape[-1] features by theta_i."""
    R = 2 * theta.shape[-1]
    a, b = v[..., 0:R:2], v[..., 1:R:2]
    c, s = torch.cos(theta), torch.sin(theta)
    rot = torch.stack((a * c - b * s, a * s + b * c), dim=-1).flatten(-2)
    return torch.cat((rot, v[..., R:]), dim=-1)


def shift(t: torch.Tensor) -> torch.Tensor:
    """Token t takes token t-1's value; token 0 takes zeros."""
    return torch.cat((torch.zeros_like(t[:, :1]), t[:, :-1]), dim=1)


def prologue(x, Bm, Cm, dd_dt, dd_A, trap, ang, dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, A_floor, eps=1e-5):
    """The scan operands (q, k, kp, xp, adt, gamma, beta) of one layer."""
    A = -torch.minimum(heavy_tail(dd_A), torch.full_like(dd_A, -A_floor))
    DT = softplus(dd_dt + dt_bias)
    adt = A * DT
    tr = torch.sigmoid(trap)
    gamma = tr * DT
    beta = (1 - tr) * DT * torch.exp(adt)
    theta = torch.cumsum(DT.unsqueeze(-1) * ang.unsqueeze(2), dim=1)          # [B, T, H, N/4]
    q = rope(rmsnorm(Cm, C_norm_w, eps).unsqueeze(2) + C_bias, theta)
    k = rope(rmsnorm(Bm, B_norm_w, eps).unsqueeze(2) + B_bias, theta)
    return q, k, shift(k), shift(x), adt, gamma, beta


class _Scan(torch.autograd.Function):
    """The float64 scan oracle with its written-out backward."""

    @staticmethod
    def forward(ctx, chunk, x, q, k, kp, xp, adt, gamma, beta):
        ctx.chunk = chunk
        ctx.save_for_backward(x, q, k, kp, xp, adt, gamma, beta)
        return ssd_oracle.ssd_forward(x, q, k, kp, xp, adt, gamma, beta, chunk)[0]

    @staticmethod
    def backward(ctx, dy):
        g = ssd_oracle.ssd_backward(dy, *ctx.saved_tensors, ctx.chunk)
        return (None, *(g[n] for n in ("dx", "dq", "dk", "dkp", "dxp", "dadt", "dgamma", "dbeta")))


def _round(t: torch.Tensor, dtype) -> torch.Tensor:
    """Round to ``dtype`` and back; the gradient passes through unchanged."""
    return t if dtype is None else t + (t.to(dtype).to(t.dtype) - t).detach()


def forward(x, z, Bm, Cm, dd_dt, dd_A, trap, ang, dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D, A_floor, chunk,
            eps=1e-5, scan_operand_dtype=None):
    """(ssd(...) + D x) * silu(z): the layer body between the in_proj split and out_proj.
    ``scan_operand_dtype`` rounds the scan's vector operands (x, q, k, kp, xp) to that dtype, as a
    16-bit scan reads them; the D skip keeps the unrounded x."""
    q, k, kp, xp, adt, gamma, beta = prologue(x, Bm, Cm, dd_dt, dd_A, trap, ang, dt_bias, B_bias, C_bias, B_norm_w,
                                              C_norm_w, A_floor, eps)
    r = scan_operand_dtype
    y = _Scan.apply(chunk, _round(x, r), _round(q, r), _round(k, r), _round(kp, r), _round(xp, r), adt, gamma, beta)
    y = y + D[:, None] * x
    return y if z is None else y * torch.nn.functional.silu(z)


INPUTS = ("x", "z", "Bm", "Cm", "dd_dt", "dd_A", "trap", "ang")
PARAMS = ("dt_bias", "B_bias", "C_bias", "B_norm_w", "C_norm_w", "D")


def forward_backward(tensors: dict, dout: torch.Tensor, A_floor: float, chunk: int, eps: float = 1e-5,
                     scan_operand_dtype=None):
    """Output and the gradients of every input and parameter (float64, autograd)."""
    leaves = {n: tensors[n].detach().to(F64).clone().requires_grad_(True) for n in INPUTS + PARAMS
              if tensors.get(n) is not None}
    out = forward(*(leaves.get(n) for n in INPUTS + PARAMS), A_floor, chunk, eps, scan_operand_dtype)
    out.backward(dout.to(F64))
    grads = {"d" + n: leaves[n].grad for n in leaves}
    return out.detach(), grads
