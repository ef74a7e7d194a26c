"""CPU oracle for the SSD chunked scan: TEST INFRASTRUCTURE ONLY.

This module restates, in float64 PyTorch on the CPU, the algorithm of the reference's
``ssd(x, q, k, kp, xp, adt, gamma, beta, chunk_size)`` (zenith/mamba3.py:30-56) and its
gradient.  It is the checker for the CUDA kernels in ``zenith_b200``; only the tests,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs of
``bench.py`` may import it.  The product path never calls it.

Pinning: ``tests/test_oracle.py`` checks these functions against golden vectors written by
``tests/golden/make_golden.py``, which runs the reference's own ``ssd`` (forward) and
PyTorch autograd through it (all eight gradients) on seeded inputs, and against the
reference test's per-token recurrence (tests/test_mamba3.py:10-21).

Notation (one batch element b, one head h, chunk j of L tokens, local t, s):
    c_t  = sum_{u<=t} adt_u                  (zenith/mamba3.py:40)
    M_ts = exp(c_t - c_s) [s <= t]           (zenith/mamba3.py:41-42)
    y_t  = sum_s M_ts (q_t.k_s) g_s x_s + M_ts (q_t.kp_s) b_s xp_s + e^{c_t} S_in q_t
    S_loc = sum_s e^{c_L - c_s} (g_s x_s k_s^T + b_s xp_s kp_s^T)     (mamba3.py:46-47)
    S_in[j+1] = e^{c_L} S_in[j] + S_loc[j]                            (mamba3.py:48-54)
The reference starts from a zero state and drops the final state; ``initial_state`` and the
returned final state are extensions (used for context parallelism and decode hand-off).
"""

from __future__ import annotations

import torch

F64 = torch.float64


def _split_chunks(t: torch.Tensor, L: int) -> torch.Tensor:
    """[B, T, H, ...] -> [B, H, nc, L, ...] (zenith/mamba3.py:36-39)."""
    B, T, H = t.shape[:3]
    return t.movedim(1, 2).reshape(B, H, T // L, L, *t.shape[3:])


def _expand_groups(t: torch.Tensor, H: int) -> torch.Tensor:
    """q/k/kp given per group [B, T, G, N] -> per head [B, T, H, N] (head h uses group h // (H/G))."""
    G = t.shape[2]
    if G == H:
        return t
    assert H % G == 0
    return t.repeat_interleave(H // G, dim=2)


def _sum_groups(t: torch.Tensor, G: int) -> torch.Tensor:
    B, T, H, N = t.shape
    if G == H:
        return t
    return t.reshape(B, T, G, H // G, N).sum(3)


def ssd_forward(x, q, k, kp, xp, adt, gamma, beta, chunk_size, initial_state=None, dtype=F64):
    """Chunked SSD forward, computed in ``dtype`` (float64 by default; the CPU baseline of the
    benchmark runs it in float32 under autograd, the same work the reference does on a CPU).

    Returns ``(y [B,T,H,P], final_state [B,H,P,N], chunk_states [B,H,nc,P,N])`` where
    ``chunk_states[:, :, j]`` is the state entering chunk j.
    Follows zenith/mamba3.py:30-56 (same chunked algorithm).
    """
    B, T, H, P = x.shape
    N = q.shape[-1]
    assert T % chunk_size == 0, "sequence length must be a multiple of chunk_size"
    L = chunk_size
    nc = T // L
    q, k, kp = (_expand_groups(t.to(dtype), H) for t in (q, k, kp))
    xc, xpc = _split_chunks(x.to(dtype), L), _split_chunks(xp.to(dtype), L)
    qc, kc, kpc = _split_chunks(q, L), _split_chunks(k, L), _split_chunks(kp, L)
    ac, gc, bc = (_split_chunks(t.to(dtype), L) for t in (adt, gamma, beta))

    c = torch.cumsum(ac, dim=-1)                                   # [B,H,nc,L]
    diff = c[..., :, None] - c[..., None, :]                        # c_t - c_s
    lower = torch.ones(L, L, dtype=torch.bool).tril()
    M = torch.where(lower, torch.exp(torch.where(lower, diff, torch.zeros((), dtype=dtype))), torch.zeros((), dtype=dtype))
    Sg = torch.einsum("bhjtn,bhjsn->bhjts", qc, kc) * gc[..., None, :] * M
    Sb = torch.einsum("bhjtn,bhjsn->bhjts", qc, kpc) * bc[..., None, :] * M
    y_intra = torch.einsum("bhjts,bhjsp->bhjtp", Sg, xc) + torch.einsum("bhjts,bhjsp->bhjtp", Sb, xpc)

    w = torch.exp(c[..., -1:] - c)                                  # [B,H,nc,L]
    S_loc = torch.einsum("bhjs,bhjsp,bhjsn->bhjpn", w * gc, xc, kc) + \
        torch.einsum("bhjs,bhjsp,bhjsn->bhjpn", w * bc, xpc, kpc)
    a = torch.exp(c[..., -1])                                       # [B,H,nc]

    S = torch.zeros(B, H, P, N, dtype=dtype) if initial_state is None else initial_state.to(dtype).clone()
    s_in = []
    for j in range(nc):
        s_in.append(S)
        S = a[:, :, j, None, None] * S + S_loc[:, :, j]
    s_in = torch.stack(s_in, dim=2)
    y = y_intra + torch.exp(c)[..., None] * torch.einsum("bhjtn,bhjpn->bhjtp", qc, s_in)
    return y.reshape(B, H, T, P).movedim(2, 1), S, s_in


def ssd_backward(dy, x, q, k, kp, xp, adt, gamma, beta, chunk_size, initial_state=None, dfinal=None):
    """Explicit float64 gradient of :func:`ssd_forward` (adjoint of zenith/mamba3.py:30-56).

    Returns a dict with dx, dq, dk, dkp, dxp, dadt, dgamma, dbeta (shaped like the inputs;
    dq/dk/dkp summed over the heads of a group when G < H) and dinitial_state [B,H,P,N].
    ``dfinal`` is the gradient flowing into the returned final state (zero when None).
    """
    B, T, H, P = x.shape
    G = q.shape[2]
    N = q.shape[-1]
    L = chunk_size
    assert T % L == 0, "sequence length must be a multiple of chunk_size"
    nc = T // L
    _, _, s_in = ssd_forward(x, q, k, kp, xp, adt, gamma, beta, L, initial_state)
    q, k, kp = (_expand_groups(t.to(F64), H) for t in (q, k, kp))
    xc, xpc, dyc = (_split_chunks(t.to(F64), L) for t in (x, xp, dy))
    qc, kc, kpc = _split_chunks(q, L), _split_chunks(k, L), _split_chunks(kp, L)
    ac, gc, bc = (_split_chunks(t.to(F64), L) for t in (adt, gamma, beta))

    c = torch.cumsum(ac, dim=-1)
    diff = c[..., :, None] - c[..., None, :]
    lower = torch.ones(L, L, dtype=torch.bool).tril()
    M = torch.where(lower, torch.exp(torch.where(lower, diff, torch.zeros(()))), torch.zeros((), dtype=F64))
    ec = torch.exp(c)
    w = torch.exp(c[..., -1:] - c)
    a = torch.exp(c[..., -1])

    QK = torch.einsum("bhjtn,bhjsn->bhjts", qc, kc)
    QKp = torch.einsum("bhjtn,bhjsn->bhjts", qc, kpc)
    A = QK * gc[..., None, :] * M
    Ap = QKp * bc[..., None, :] * M
    dA = torch.einsum("bhjtp,bhjsp->bhjts", dyc, xc)
    dAp = torch.einsum("bhjtp,bhjsp->bhjts", dyc, xpc)
    E, Ep = dA * M, dAp * M

    # intra-chunk terms
    dx = torch.einsum("bhjts,bhjtp->bhjsp", A, dyc)
    dxp = torch.einsum("bhjts,bhjtp->bhjsp", Ap, dyc)
    dq = torch.einsum("bhjts,bhjs,bhjsn->bhjtn", E, gc, kc) + torch.einsum("bhjts,bhjs,bhjsn->bhjtn", Ep, bc, kpc)
    dk = gc[..., None] * torch.einsum("bhjts,bhjtn->bhjsn", E, qc)
    dkp = bc[..., None] * torch.einsum("bhjts,bhjtn->bhjsn", Ep, qc)
    dg = (E * QK).sum(-2)
    db = (Ep * QKp).sum(-2)
    Z = dA * A + dAp * Ap
    dc = Z.sum(-1) - Z.sum(-2)

    # inter-chunk output term  y_t += e^{c_t} S_in q_t
    r = torch.einsum("bhjpn,bhjtp->bhjtn", s_in, dyc)               # S_in^T dy_t
    dq = dq + ec[..., None] * r
    dc = dc + ec * (qc * r).sum(-1)
    dS_in_loc = torch.einsum("bhjt,bhjtp,bhjtn->bhjpn", ec, dyc, qc)

    # reverse state chain: Gn[j] = gradient w.r.t. the state leaving chunk j
    Gcur = torch.zeros(B, H, P, N, dtype=F64) if dfinal is None else dfinal.to(F64).clone()
    Gn = [None] * nc
    for j in reversed(range(nc)):
        Gn[j] = Gcur
        Gcur = dS_in_loc[:, :, j] + a[:, :, j, None, None] * Gcur
    dinit = Gcur
    Gn = torch.stack(Gn, dim=2)                                      # [B,H,nc,P,N]

    da = (Gn * s_in).sum((-1, -2))                                   # [B,H,nc]
    u = torch.einsum("bhjpn,bhjsn->bhjsp", Gn, kc)
    up = torch.einsum("bhjpn,bhjsn->bhjsp", Gn, kpc)
    xu = (xc * u).sum(-1)
    xpu = (xpc * up).sum(-1)
    dx = dx + (w * gc)[..., None] * u
    dxp = dxp + (w * bc)[..., None] * up
    dk = dk + (w * gc)[..., None] * torch.einsum("bhjpn,bhjsp->bhjsn", Gn, xc)
    dkp = dkp + (w * bc)[..., None] * torch.einsum("bhjpn,bhjsp->bhjsn", Gn, xpc)
    dg = dg + w * xu
    db = db + w * xpu
    dw = gc * xu + bc * xpu
    dc = dc - w * dw
    dc[..., -1] += a * da + (w * dw).sum(-1)

    # adt enters only through c = cumsum(adt): reverse cumulative sum inside each chunk
    dadt = torch.flip(torch.cumsum(torch.flip(dc, [-1]), -1), [-1])

    def unchunk(t):
        return t.reshape(B, H, T, *t.shape[4:]).movedim(2, 1)

    out = {
        "dx": unchunk(dx), "dxp": unchunk(dxp),
        "dq": _sum_groups(unchunk(dq), G), "dk": _sum_groups(unchunk(dk), G), "dkp": _sum_groups(unchunk(dkp), G),
        "dadt": unchunk(dadt), "dgamma": unchunk(dg), "dbeta": unchunk(db),
        "dinitial_state": dinit,
    }
    return out


def naive_recurrence(x, q, k, kp, xp, adt, gamma, beta, initial_state=None):
    """Per-token recurrence in float64 (restates tests/test_mamba3.py:10-21; Mojo ssd_fwd_cpu,
    mojo/ssd_fwd.mojo:40-56):  h_t = e^{adt_t} h_{t-1} + g_t x_t k_t^T + b_t xp_t kp_t^T,  y_t = h_t q_t.
    Returns (y, final_state)."""
    B, T, H, P = x.shape
    q, k, kp = (_expand_groups(t.to(F64), H) for t in (q, k, kp))
    x, xp, adt, gamma, beta = (t.to(F64) for t in (x, xp, adt, gamma, beta))
    N = q.shape[-1]
    h = torch.zeros(B, H, P, N, dtype=F64) if initial_state is None else initial_state.to(F64).clone()
    ys = []
    for t in range(T):
        h = torch.exp(adt[:, t])[..., None, None] * h \
            + gamma[:, t][..., None, None] * x[:, t][..., :, None] * k[:, t][..., None, :] \
            + beta[:, t][..., None, None] * xp[:, t][..., :, None] * kp[:, t][..., None, :]
        ys.append(torch.einsum("bhpn,bhn->bhp", h, q[:, t]))
    return torch.stack(ys, 1), h


def max_rel_err(out: torch.Tensor, ref: torch.Tensor) -> float:
    """max|out - ref| / max|ref| (per-tensor, max-normalised; elementwise relative error is
    unbounded near zeros)."""
    out = out.detach().to(F64).cpu()
    ref = ref.detach().to(F64).cpu()
    denom = ref.abs().max().item()
    if denom == 0.0:
        return out.abs().max().item()
    return (out - ref).abs().max().item() / denom


def flops_per_token_head(P: int, N: int, L: int, ratio: int = 1) -> int:
    """Algorithmic forward flops per token per head: 4 L N / r + 4 L P + 6 N P."""
    return 4 * L * N // ratio + 4 * L * P + 6 * N * P


__all__ = ["ssd_forward", "ssd_backward", "naive_recurrence", "max_rel_err", "flops_per_token_head"]
