"""CPU baseline of the SSD scan: TEST AND BENCHMARK INFRASTRUCTURE ONLY.

The reference's chunked scan (zenith/mamba3.py:30-56) restated with the same sequence of tensor
operations: chunk relayout by transpose + reshape, in-chunk cumsum, the decay mask as exp of a
masked segment sum, score matmuls scaled by gamma / beta, the intra-chunk output, chunk-local
states, a Python loop over chunks for the state recurrence with a stack of the entering states,
and the inter-chunk output.  The reference itself cannot be imported where the benchmark runs, so
``bench.py``'s ``cpu_baseline`` / ``--impl reference`` time this restatement: same operations, same
shapes, same autograd graph, hence the reference's cost on a CPU (checked against the reference in
the container that has it: within a few percent).  ``oracle/ssd_oracle.py`` remains the checker.
"""

from __future__ import annotations

import torch


def ssd_reference_ops(x, q, k, kp, xp, adt, gamma, beta, chunk_size):
    """y [B, T, H, P] of the SSD scan, computed with the reference's operation sequence."""
    Bsz, T, H, P = x.shape
    N = q.shape[-1]
    assert T % chunk_size == 0, "sequence length must be a multiple of chunk_size"
    L = chunk_size
    nc = T // L

    def split(t):  # [B, T, H, ...] -> [B, H, nc, L, ...]
        return t.transpose(1, 2).reshape(Bsz, H, nc, L, *t.shape[3:])

    xs, qs, ks, kps, xps, a, g, bt = (split(t) for t in (x, q, k, kp, xp, adt, gamma, beta))
    c = a.cumsum(-1)
    lower = torch.ones(L, L, dtype=torch.bool, device=x.device).tril()
    mask = torch.exp((c.unsqueeze(-1) - c.unsqueeze(-2)).masked_fill(~lower, float("-inf")))
    s_g = (qs @ ks.transpose(-1, -2)) * g.unsqueeze(-2)
    s_b = (qs @ kps.transpose(-1, -2)) * bt.unsqueeze(-2)
    y_intra = (mask * s_g) @ xs + (mask * s_b) @ xps
    w = torch.exp(c[..., -1:] - c)
    local = ((w * g).unsqueeze(-1) * xs).transpose(-1, -2) @ ks + ((w * bt).unsqueeze(-1) * xps).transpose(-1, -2) @ kps
    decay = torch.exp(c[..., -1])
    entering = []
    state = xs.new_zeros(Bsz, H, P, N)
    for j in range(nc):
        entering.append(state)
        state = decay[:, :, j, None, None] * state + local[:, :, j]
    s_in = torch.stack(entering, dim=2)
    y = y_intra + torch.exp(c).unsqueeze(-1) * (qs @ s_in.transpose(-1, -2))
    return y.reshape(Bsz, H, T, P).transpose(1, 2)


__all__ = ["ssd_reference_ops"]
