"""Seeded synthetic SSD inputs with the value distributions of the Mamba-3 block.

The SSD boundary tensors are built the way ``Mamba3.forward`` builds them
(zenith/mamba3.py:105-116), from randomly drawn per-token/per-head quantities:

* x ~ N(0, 1)                                      [B, T, H, P]
* dt = softplus(N(0, 1) + bias_h), where softplus(bias_h) is log-uniform in [1e-3, 1e-1]
  (the dt_bias initialisation of zenith/mamba3.py:87-89)
* A_h = -exp(U(log 1, log 16))                     (per head)
* B, C ~ N(0, 1) / sqrt(N)                         [B, T, G, N]
* trapezoid weight 0.5:  gamma = 0.5 dt,  beta = 0.5 dt e^{A dt}   (mamba3.py:108-110)
* adt = A dt;  k = B;  q = C;  kp, xp = one-token shift with a zero row at t = 0
  (mamba3.py:115-116)
* dy ~ N(0, 1) (upstream gradient)

Everything is drawn in float32 on the CPU from ``torch.Generator().manual_seed(seed)`` so the
same seed gives the same tensors on every machine; the caller casts and moves them.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class SsdShape:
    B: int
    T: int
    H: int
    P: int
    N: int
    G: int
    chunk: int
    name: str = ""

    @property
    def tokens(self) -> int:
        return self.B * self.T


# Workloads of the SSD benchmark suite (batch, seqlen, heads, head dim P, state N, groups G, chunk).
SHAPES = {
    "tiny": SsdShape(2, 256, 4, 32, 16, 4, 64, "tiny fp32 (B2 T256 H4 P32 N16 L64)"),
    "layer": SsdShape(8, 2048, 24, 64, 128, 24, 64, "model-scale layer (B8 T2048 H24 P64 N128 L64)"),
    "long": SsdShape(1, 131072, 24, 64, 128, 24, 128, "long context (B1 T131072 H24 P64 N128 L128)"),
    "infer": SsdShape(64, 512, 32, 64, 64, 4, 64, "inference fwd (B64 T512 H32 P64 N64 G4 L64)"),
}


def _shift(t: torch.Tensor) -> torch.Tensor:
    out = torch.zeros_like(t)
    out[:, 1:] = t[:, :-1]
    return out


def make_inputs(shape: SsdShape, seed: int = 0, trap: float = 0.5):
    """Return a dict of float32 CPU tensors x, q, k, kp, xp, adt, gamma, beta, dy, D."""
    g = torch.Generator().manual_seed(seed)
    B, T, H, P, N, G = shape.B, shape.T, shape.H, shape.P, shape.N, shape.G
    x = torch.randn(B, T, H, P, generator=g)
    dt0 = torch.exp(torch.rand(H, generator=g) * (math.log(1e-1) - math.log(1e-3)) + math.log(1e-3))
    bias = dt0 + torch.log(-torch.expm1(-dt0))                 # inverse softplus
    dt = torch.nn.functional.softplus(torch.randn(B, T, H, generator=g) + bias)
    A = -torch.exp(torch.rand(H, generator=g) * math.log(16.0))
    Bm = torch.randn(B, T, G, N, generator=g) / math.sqrt(N)
    Cm = torch.randn(B, T, G, N, generator=g) / math.sqrt(N)
    D = torch.randn(H, generator=g)
    dy = torch.randn(B, T, H, P, generator=g)
    adt = A * dt
    gamma = trap * dt
    beta = (1.0 - trap) * dt * torch.exp(adt)
    return {
        "x": x, "q": Cm, "k": Bm, "kp": _shift(Bm), "xp": _shift(x),
        "adt": adt, "gamma": gamma, "beta": beta, "dy": dy, "D": D,
    }


ARG_ORDER = ("x", "q", "k", "kp", "xp", "adt", "gamma", "beta")
