"""Write the golden vectors in tests/golden/ by running the reference's own SSD path.

Run in a container that has the reference checked out (read-only is fine):

    python tests/golden/make_golden.py --reference /root/reference

For every case it imports ``zenith.mamba3.ssd`` (zenith/mamba3.py:30-56) from the reference,
runs it in float64 with PyTorch autograd on seeded inputs, and stores the inputs, the output
``y``, the upstream gradient ``dy`` and all eight input gradients.  Cases with G < H feed the
reference ``repeat_interleave``d q/k/kp (the reference has no groups), so autograd sums the
per-head gradients over each group.  The final state comes from the reference test's
per-token recurrence (tests/test_mamba3.py:10-21), imported from the reference's tests.

The fixtures are consumed by tests/test_oracle.py (CPU) and the GPU parity tests; nothing at
run time reads the reference.
"""

from __future__ import annotations

import argparse
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from zenith.mamba3 import ssd  # the reference's own chunked scan

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


if __name__ == "__main__":
    main()
