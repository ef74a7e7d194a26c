"""CPU oracle for the Mamba-3 language model: TEST INFRASTRUCTURE ONLY.

Restates in float64 PyTorch the reference's looped causal LM, ``ZenithForCausalLM.forward``
(zenith/model.py:79-99), over a parameter dict keyed like the reference's ``state_dict``:

    x = embed(ids)                                         (model.py:81)
    x = layer(x) for the input layers                      (:82-83)
    s = x; repeat `loops` times (all but the last without autograd, :85-86):
        h = recurrent_norm(s + x); h = layer(h) for the recurrent layers; s = h   (:87-90)
    s = layer(s) for the output layers                     (:91-92)
    logits = norm(s) @ embed^T   (lm_head tied to embed)   (:93, _tied_weights_keys :54)
    loss = cross_entropy(logits[:, :-1], ids[:, 1:])       (:95-97)
    layer(x) = x + mixer(norm(x))                          (Layer.forward, :48-49)
    mixer = Mamba3.forward (zenith/mamba3.py:96-120): in_proj, split, the layer body of
            oracle.mamba3_oracle, out_proj

Only the tests and the benchmark's CPU baseline may import it.  Pinning: tests/test_oracle.py
checks it against golden vectors that tests/golden/make_golden.py writes by running the
reference model itself (float32, autograd).
"""

from __future__ import annotations

from contextlib import nullcontext

import torch
import torch.nn.functional as F

from oracle import mamba3_oracle as M

A_FLOOR = 1e-4   # Mamba3.A_floor default (mamba3.py:68)
EPS = 1e-5       # RMSNorm eps default (mamba3.py:9)


def dims(cfg: dict):
    d_inner = cfg["expand"] * cfg["d_model"]
    H = d_inner // cfg["headdim"]
    N = cfg["d_state"]
    return d_inner, H, cfg["headdim"], N, N // 4


def in_proj_sizes(cfg: dict):
    """The in_proj split [z, x, B, C, dd_dt, dd_A, trap, angles] (mamba3.py:81,98-100)."""
    d_inner, H, _, N, NA = dims(cfg)
    return [d_inner, d_inner, N, N, H, H, H, NA]


def mixer(p: dict, pre: str, u: torch.Tensor, cfg: dict) -> torch.Tensor:
    """Mamba3.forward (mamba3.py:96-120) with the layer body of oracle.mamba3_oracle."""
    Bsz, T, _ = u.shape
    d_inner, H, P, N, NA = dims(cfg)
    z, x, Bm, Cm, dd_dt, dd_A, trap, ang = torch.split(u @ p[pre + "in_proj.weight"].T, in_proj_sizes(cfg), dim=-1)
    y = M.forward(x.reshape(Bsz, T, H, P), z.reshape(Bsz, T, H, P), Bm, Cm, dd_dt, dd_A, trap, ang,
                  p[pre + "dt_bias"], p[pre + "B_bias"], p[pre + "C_bias"], p[pre + "B_norm.weight"],
                  p[pre + "C_norm.weight"], p[pre + "D"], A_FLOOR, cfg["chunk_size"], EPS)
    return y.to(u.dtype).reshape(Bsz, T, d_inner) @ p[pre + "out_proj.weight"].T


def layer(p: dict, pre: str, x: torch.Tensor, cfg: dict) -> torch.Tensor:
    return x + mixer(p, pre + "mixer.", M.rmsnorm(x, p[pre + "norm.weight"], EPS), cfg)


def forward(p: dict, cfg: dict, ids: torch.Tensor, labels: torch.Tensor | None = None, loops: int | None = None):
    """(logits, loss); loss is None without labels."""
    loops = loops or cfg["max_loops"]
    x = p["embed.weight"][ids]
    for i in range(cfg["n_input"]):
        x = layer(p, f"input_layers.{i}.", x, cfg)
    s = x
    for t in range(loops):
        with torch.no_grad() if t < loops - 1 else nullcontext():
            h = M.rmsnorm(s + x, p["recurrent_norm.weight"], EPS)
            for i in range(cfg["n_recurrent"]):
                h = layer(p, f"recurrent_layers.{i}.", h, cfg)
            s = h
    for i in range(cfg["n_output"]):
        s = layer(p, f"output_layers.{i}.", s, cfg)
    logits = M.rmsnorm(s, p["norm.weight"], EPS) @ p["embed.weight"].T
    loss = None
    if labels is not None:
        V = logits.shape[-1]
        loss = F.cross_entropy(logits[:, :-1].reshape(-1, V), labels[:, 1:].reshape(-1))
    return logits, loss


def forward_backward(params: dict, cfg: dict, ids: torch.Tensor, loops: int | None = None):
    """Logits, loss and the gradient of the loss for every parameter (float64 autograd)."""
    leaves = {n: t.detach().to(torch.float64).clone().requires_grad_(True) for n, t in params.items()}
    logits, loss = forward(leaves, cfg, ids, ids, loops)
    loss.backward()
    return logits.detach(), loss.detach(), {n: leaves[n].grad for n in leaves}
