"""Small fixed workloads for profiler captures (ncu).

    python -m zenith_b200.profile_case [--batch 2] [--iters 3] [--dtype bf16|fp32]
        a few forward (saving states) + backward calls of the scan on B sequences of the layer
        shape (T2048 H24 P64 N128, chunk 64); bf16 runs the tensor-core kernels, fp32 the SIMT ones
    python -m zenith_b200.profile_case --workload infer [--batch 64] [--iters 3]
        a few inference forwards (final state out, no saved states) on B sequences of the inference
        shape (T512 H32 P64 N64, 4 q/k groups, chunk 64): the tensor-core forward at N = 64
    python -m zenith_b200.profile_case --workload rows [--batch 2] [--heads 48] [--iters 2]
        the row kernels around it, once per iteration each: the fused Mamba-3 layer body (fwd + bwd,
        bf16, P64 N128) on B sequences of 2048 tokens, the residual add + RMSNorm (d_model 1536) and
        the LM head's cross-entropy (vocabulary 32000) on the same B x 2048 tokens
"""
from __future__ import annotations

import argparse

import torch

import zenith_b200
from zenith_b200.ssd import prepare_inputs, ssd_bwd_op, ssd_fwd_op
from zenith_b200.synthetic import SsdShape, make_inputs

NAMES = ("x", "q", "k", "kp", "xp", "adt", "gamma", "beta")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=2)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--seqlen", type=int, default=2048)
    ap.add_argument("--workload", choices=("scan", "infer", "rows"), default="scan")
    ap.add_argument("--heads", type=int, default=48)
    ap.add_argument("--dtype", choices=("bf16", "fp32"), default="bf16")
    args = ap.parse_args()
    if args.workload == "rows":
        return rows(args)
    if args.workload == "infer":
        return infer(args)
    s = SsdShape(args.batch, args.seqlen, 24, 64, 128, 24, 64)
    inp = make_inputs(s, seed=0)
    dev = torch.device("cuda")
    vdt = torch.float32 if args.dtype == "fp32" else torch.bfloat16
    a = prepare_inputs(*((inp[n].to(vdt) if n in ("x", "q", "k", "kp", "xp") else inp[n]).to(dev) for n in NAMES))
    dy = inp["dy"].to(vdt).to(dev)
    for _ in range(args.iters):
        _, _, st = ssd_fwd_op(*a, s.chunk, None, True, False)
        ssd_bwd_op(dy, *a, st, s.chunk, None, None, False)
    torch.cuda.synchronize()
    zenith_b200.check_status()
    print("ok")


def infer(args):
    s = SsdShape(args.batch, 512, 32, 64, 64, 4, 64)
    inp = make_inputs(s, seed=0)
    dev = torch.device("cuda")
    a = prepare_inputs(*((inp[n].to(torch.bfloat16) if n in ("x", "q", "k", "kp", "xp") else inp[n]).to(dev)
                         for n in NAMES))
    for _ in range(args.iters):
        ssd_fwd_op(*a, s.chunk, None, False, False)
    torch.cuda.synchronize()
    zenith_b200.check_status()
    print("ok")


def rows(args):
    from zenith_b200 import lm

    dev = torch.device("cuda")
    B, T, H, P, N, D, V = args.batch, args.seqlen, args.heads, 64, 128, 1536, 32000
    g = torch.Generator().manual_seed(0)
    mk = lambda *sh: torch.randn(*sh, generator=g)  # noqa: E731
    n_in = 2 * H * P + 2 * N + 3 * H + N // 4
    zxbc = mk(B, T, n_in).to(dev, torch.bfloat16).requires_grad_()
    prm = [(torch.rand(H, generator=g) * -4.0 - 3.0), torch.ones(H, N), torch.ones(H, N), torch.ones(N), torch.ones(N),
           torch.ones(H)]
    prm = [t.to(dev).requires_grad_() for t in prm]
    dout = mk(B, T, H, P).to(dev, torch.bfloat16)
    resid = mk(B * T, D).to(dev).requires_grad_()
    delta = mk(B * T, D).to(dev, torch.bfloat16).requires_grad_()
    w = torch.ones(D, device=dev, requires_grad=True)
    h = mk(B * T, D).to(dev, torch.bfloat16).requires_grad_()
    W = (0.02 * mk(V, D)).to(dev, torch.bfloat16).requires_grad_()
    labels = torch.randint(0, V, (B * T,), generator=g).to(dev)
    for _ in range(args.iters):
        out = zenith_b200.mamba3_layer_packed(zxbc, *prm, H, P, N, 1e-4, 64, 1e-5, torch.bfloat16)
        out.backward(dout)
        s_, u = lm.add_rmsnorm(resid, delta, w, 1e-5, torch.bfloat16)
        (u.float().sum() + s_.sum()).backward()
        lm.linear_cross_entropy(h, W, labels, compute_dtype=torch.bfloat16).backward()
    torch.cuda.synchronize()
    zenith_b200.check_status()
    print("ok")


if __name__ == "__main__":
    main()
