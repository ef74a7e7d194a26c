"""Small fixed workload for profiler captures (ncu): a few forward (saving states) + backward
calls of the bf16 scan on B sequences of the layer shape (T2048 H24 P64 N128, chunk 64).

    python -m zenith_b200.profile_case [--batch 2] [--iters 3]
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
    args = ap.parse_args()
    s = SsdShape(args.batch, args.seqlen, 24, 64, 128, 24, 64)
    inp = make_inputs(s, seed=0)
    dev = torch.device("cuda")
    a = prepare_inputs(*((inp[n].to(torch.bfloat16) if n in ("x", "q", "k", "kp", "xp") else inp[n]).to(dev)
                         for n in NAMES))
    dy = inp["dy"].to(torch.bfloat16).to(dev)
    for _ in range(args.iters):
        _, _, st = ssd_fwd_op(*a, s.chunk, None, True, False)
        ssd_bwd_op(dy, *a, st, s.chunk, None, None, False)
    torch.cuda.synchronize()
    zenith_b200.check_status()
    print("ok")


if __name__ == "__main__":
    main()
