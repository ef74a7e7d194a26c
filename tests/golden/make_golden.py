"""Write the golden vectors in tests/golden/ by running the reference's own SSD path.

Run in a container that has the reference checked out (read-only is fine):

    python tests/golden/make_golden.py --reference <checkout of the reference project>
    (or set ZENITH_REFERENCE to that directory)

For every case it imports ``zenith.mamba3.ssd`` (zenith/mamba3.py:30-56) from the reference,
runs it in float64 with PyTorch autograd on seeded inputs, and stores the inputs, the output
``y``, the upstream gradient ``dy`` and all eight input gradients.  Cases with G < H feed the
reference ``repeat_interleave``d q/k/kp (the reference has no groups), so autograd sums the
per-head gradients over each group.  The final state comes from the reference test's
per-token recurrence (tests/test_mamba3.py:10-21), imported from the reference's tests.

It also runs the reference ``Mamba3`` module (zenith/mamba3.py:58-119) with its input and
output projections replaced by identities, for the fused layer body (prologue, scan, D skip,
silu gate): the split tensors, the parameters, the output and every gradient; and the reference
language model ``ZenithForCausalLM`` (zenith/model.py:42-99) at a small configuration: token
ids, parameters, logits, loss and every parameter gradient (``--only lm`` writes just that).

The fixtures are consumed by tests/test_oracle.py (CPU) and the GPU parity tests; nothing at
run time reads the reference.
"""

from __future__ import annotations

import argparse
import os
import importlib.util
import pathlib
import sys

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from zenith_b200.synthetic import SHAPES, SsdShape, make_inputs  # noqa: E402

NAMES = ("x", "q", "k", "kp", "xp", "adt", "gamma", "beta")


def _random_case(B, T, H, P, N, G, seed):
    """Inputs drawn like the reference's own tests (tests/test_mamba3.py:24-33)."""
    g = torch.Generator().manual_seed(seed)
    x, xp = torch.randn(2, B, T, H, P, generator=g, dtype=torch.float64)
    q, k, kp = torch.randn(3, B, T, G, N, generator=g, dtype=torch.float64)
    adt = -torch.rand(B, T, H, generator=g, dtype=torch.float64)
    gamma, beta = torch.rand(2, B, T, H, generator=g, dtype=torch.float64)
    dy = torch.randn(B, T, H, P, generator=g, dtype=torch.float64)
    return dict(x=x, q=q, k=k, kp=kp, xp=xp, adt=adt, gamma=gamma, beta=beta, dy=dy)


def _run_reference(ssd, naive, inp, chunk):
    H = inp["x"].shape[2]
    leaves = {n: inp[n].detach().to(torch.float64).clone().requires_grad_(True) for n in NAMES}
    args = []
    for n in NAMES:
        t = leaves[n]
        if n in ("q", "k", "kp") and t.shape[2] != H:
            t = t.repeat_interleave(H // t.shape[2], dim=2)
        args.append(t)
    y = ssd(*args, chunk)
    y.backward(inp["dy"].to(torch.float64))
    with torch.no_grad():
        h = naive_final_state(naive, *[a.detach() for a in args])
    out = {"y": y.detach()}
    for n in NAMES:
        out["d" + n] = leaves[n].grad.detach()
    out["final_state"] = h
    return out


def naive_final_state(naive, x, q, k, kp, xp, adt, gamma, beta):
    """Read the final state h_T out of the reference test's recurrence, which returns only y:
    append one token with adt = 0, gamma = beta = 0 (so h is unchanged) and q = e_n; its output
    is column n of h_T.  All N columns run at once as N copies of the batch."""
    B, T, H, P = x.shape
    N = q.shape[-1]

    def ext(t, last):
        return torch.cat([t.repeat(N, *([1] * (t.dim() - 1))), last], dim=1)

    eye = torch.eye(N, dtype=x.dtype)                               # copy n reads column n
    q_last = eye[:, None, None, :].expand(N, B, H, N).reshape(N * B, 1, H, N)
    zP = torch.zeros(N * B, 1, H, P, dtype=x.dtype)
    zN = torch.zeros(N * B, 1, H, N, dtype=x.dtype)
    zS = torch.zeros(N * B, 1, H, dtype=x.dtype)
    y = naive(ext(x, zP), ext(q, q_last), ext(k, zN), ext(kp, zN), ext(xp, zP), ext(adt, zS), ext(gamma, zS), ext(beta, zS))
    return y[:, -1].reshape(N, B, H, P).permute(1, 2, 3, 0).contiguous()   # [B,H,P,N]


def mamba3_case(Mamba3, B, T, H, P, N, chunk, A_floor, seed):
    """The layer body of the reference ``Mamba3`` module (zenith/mamba3.py:96-119) between the
    ``in_proj`` split and ``out_proj``: both projections are replaced by identities, so the
    module's input is the concatenation of the split tensors and its output is the gated y.
    autograd; parameters are perturbed away from their initial values so that every
    parameter gradient is generic.  The reference forward upcasts to float32 (``x.float()``,
    mamba3.py:102), so the module runs in float32: the fixtures carry float32 precision."""
    torch.manual_seed(seed)
    m = Mamba3(d_model=H * P // 2, d_state=N, expand=2, headdim=P, chunk_size=chunk, A_floor=A_floor)
    m.in_proj = torch.nn.Identity()
    m.out_proj = torch.nn.Identity()
    g = torch.Generator().manual_seed(seed + 100)
    with torch.no_grad():
        m.B_bias.add_(0.3 * torch.randn(m.B_bias.shape, generator=g))
        m.C_bias.add_(0.3 * torch.randn(m.C_bias.shape, generator=g))
        m.B_norm.weight.add_(0.2 * torch.randn(N, generator=g))
        m.C_norm.weight.add_(0.2 * torch.randn(N, generator=g))
        m.D.add_(0.5 * torch.randn(H, generator=g))
    NA = N // 4
    sizes = [H * P, H * P, N, N, H, H, H, NA]
    names = ("z", "x", "Bm", "Cm", "dd_dt", "dd_A", "trap", "ang")
    u = torch.randn(B, T, sum(sizes), generator=g).requires_grad_(True)
    out = m(u)
    dout = torch.randn(out.shape, generator=g)
    out.backward(dout)
    blob = {"chunk_size": np.array(chunk), "A_floor": np.array(A_floor), "eps": np.array(m.B_norm.eps)}
    shapes = {"z": (B, T, H, P), "x": (B, T, H, P), "Bm": (B, T, N), "Cm": (B, T, N), "dd_dt": (B, T, H),
              "dd_A": (B, T, H), "trap": (B, T, H), "ang": (B, T, NA)}
    for n, piece, gpiece in zip(names, torch.split(u.detach(), sizes, dim=-1), torch.split(u.grad, sizes, dim=-1)):
        blob["in_" + n] = piece.reshape(shapes[n]).numpy()
        blob["out_d" + n] = gpiece.reshape(shapes[n]).numpy()
    params = {"dt_bias": m.dt_bias, "B_bias": m.B_bias, "C_bias": m.C_bias, "B_norm_w": m.B_norm.weight,
              "C_norm_w": m.C_norm.weight, "D": m.D}
    for n, prm in params.items():
        blob["in_" + n] = prm.detach().numpy()
        blob["out_d" + n] = prm.grad.numpy()
    blob["in_dout"] = dout.reshape(B, T, H, P).numpy()
    blob["out_out"] = out.detach().reshape(B, T, H, P).numpy()
    return blob


LM_CONFIG = dict(vocab_size=256, d_model=64, d_state=16, expand=2, headdim=16, chunk_size=32, n_input=1,
                 n_recurrent=1, n_output=1, max_loops=2, tie_word_embeddings=True)  # as configs/*/config.json


def lm_case(cfg, B, T, loops, seed):
    """The reference language model (zenith/model.py:42-99) at a small configuration: one training
    forward (``model(ids, labels=ids, loops=loops)``, loops > 1 so the no-autograd loops run
    too) and its backward, in float32.  Norm weights, biases and D are perturbed away from their
    initial values so every parameter gradient is generic.  Stores the configuration, the token
    ids, every parameter (``lm_head.weight`` is ``embed.weight``), the logits, the loss and every
    parameter gradient."""
    from zenith import ZenithConfig, ZenithForCausalLM

    torch.manual_seed(seed)
    model = ZenithForCausalLM(ZenithConfig(**cfg))
    g = torch.Generator().manual_seed(seed + 100)
    with torch.no_grad():
        for n, prm in model.named_parameters():
            if n.endswith(("norm.weight", "B_bias", "C_bias", ".D")):
                prm.add_(0.2 * torch.randn(prm.shape, generator=g))
    ids = torch.randint(0, cfg["vocab_size"], (B, T), generator=g)
    out = model(ids, labels=ids, loops=loops)
    out.loss.backward()
    blob = {"config_keys": np.array(list(cfg)), "config_vals": np.array(list(cfg.values())),
            "ids": ids.numpy(), "loops": np.array(loops), "out_logits": out.logits.detach().numpy(),
            "out_loss": out.loss.detach().numpy()}
    for n, prm in model.named_parameters():   # tied lm_head.weight is listed once, as embed.weight
        blob["in_" + n] = prm.detach().numpy()
        blob["grad_" + n] = prm.grad.numpy()
    return blob


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ZENITH_REFERENCE"),
                    help="directory of the reference project (the one holding zenith/); default $ZENITH_REFERENCE")
    ap.add_argument("--only", choices=("ssd", "mamba3", "lm"), help="write one group of fixtures")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set ZENITH_REFERENCE")
    sys.path.insert(0, args.reference)
    from zenith.mamba3 import ssd  # the reference's own chunked scan

    if args.only == "lm":
        return write_lm()

    spec = importlib.util.spec_from_file_location("ref_test_mamba3", pathlib.Path(args.reference) / "tests" / "test_mamba3.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    naive = mod.naive

    cases = {}
    # 1. the tiny fp32 workload (B2 T256 H4 P32 N16 L64) with the Mamba-3 value distributions;
    #    stored as float32 to keep the fixture small.
    s = SHAPES["tiny"]
    inp = make_inputs(s, seed=0)
    cases["tiny_f32"] = (inp, s.chunk, np.float32)
    # 2. small float64 cases with odd sizes, drawn like the reference's tests.
    cases["small_f64"] = (_random_case(2, 64, 3, 5, 7, 3, seed=1), 16, np.float64)
    cases["ragged_f64"] = (_random_case(1, 48, 2, 3, 5, 2, seed=2), 16, np.float64)
    cases["onechunk_f64"] = (_random_case(1, 32, 1, 8, 4, 1, seed=3), 32, np.float64)
    cases["groups_f64"] = (_random_case(2, 64, 4, 8, 16, 2, seed=4), 16, np.float64)
    cases["chunk1_f64"] = (_random_case(1, 20, 2, 4, 6, 2, seed=5), 1, np.float64)

    for name, (inp, chunk, dt) in cases.items():
        out = _run_reference(ssd, naive, inp, chunk)
        # cross-check the closed-form final state against the reference test's recurrence y
        ref_args = []
        H = inp["x"].shape[2]
        for n in NAMES:
            t = inp[n].to(torch.float64)
            if n in ("q", "k", "kp") and t.shape[2] != H:
                t = t.repeat_interleave(H // t.shape[2], dim=2)
            ref_args.append(t)
        y_naive = naive(*ref_args)
        err = (y_naive - out["y"]).abs().max().item() / out["y"].abs().max().item()
        assert err < 1e-9, (name, err)
        blob = {"chunk_size": np.array(chunk)}
        for n in NAMES + ("dy",):
            blob["in_" + n] = inp[n].numpy().astype(dt)
        for n, v in out.items():
            blob["out_" + n] = v.numpy().astype(dt)
        path = HERE / f"{name}.npz"
        np.savez_compressed(path, **blob)
        print(f"{name}: chunk {chunk}, naive-vs-chunked {err:.2e}, {path.stat().st_size / 1e3:.0f} kB")

    # 3. the Mamba-3 layer body around the scan (prologue: discretisation, RMSNorm, RoPE, shift;
    #    epilogue: D skip and silu gate), from the reference module itself (float32, as it runs).
    from zenith.mamba3 import Mamba3
    m3 = {
        "mamba3_small_f32": (2, 128, 4, 16, 16, 32, 1e-4, 11),
        "mamba3_wide_f32": (1, 96, 3, 8, 32, 16, 1e-4, 12),
        "mamba3_floor_f32": (2, 64, 2, 8, 16, 16, -0.5, 13),   # negative floor: the clamp lets A vary
    }
    for name, (B, T, H, P, N, chunk, A_floor, seed) in m3.items():
        blob = mamba3_case(Mamba3, B, T, H, P, N, chunk, A_floor, seed)
        path = HERE / f"{name}.npz"
        np.savez_compressed(path, **blob)
        print(f"{name}: B{B} T{T} H{H} P{P} N{N} chunk {chunk}, {path.stat().st_size / 1e3:.0f} kB")
    # 4. the language model around the layers
    write_lm()


def write_lm():
    path = HERE / "lm_small_f32.npz"
    np.savez_compressed(path, **lm_case(LM_CONFIG, 2, 64, 2, 21))
    print(f"lm_small_f32: {LM_CONFIG}, {path.stat().st_size / 1e3:.0f} kB")


if __name__ == "__main__":
    main()
