"""Host-side logic of bench.py: the reference arm's scan against the goldens, and the split of one
job's (batch, head) chains over ranks."""
import pytest
import torch

import bench
from oracle.ssd_oracle import max_rel_err
from tests.golden_io import CASES, NAMES, load
from zenith_b200.synthetic import SHAPES


@pytest.mark.parametrize("case", [c for c in CASES if "group" not in c])
def test_reference_arm_scan_matches_reference_golden(case):
    """Whichever scan the reference arm times (the installed reference, else its restatement)
    reproduces the reference's goldens, forward and autograd backward."""
    fn, kind, _ = bench.reference_ssd()
    assert kind in ("reference", "port")
    inp, out, L = load(case)
    leaves = [inp[n].clone().requires_grad_() for n in NAMES]
    y = fn(*leaves, L)
    y.backward(inp["dy"])
    tol = 1e-11 if out["y"].dtype == torch.float64 else 1e-6
    assert max_rel_err(y, out["y"]) < tol
    for n, t in zip(NAMES, leaves):
        assert max_rel_err(t.grad, out["d" + n]) < tol, n


@pytest.mark.parametrize("workload", ["layer", "infer", "long"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shards_cover_every_chain_once(workload, world):
    shape = SHAPES[workload]
    seen = torch.zeros(shape.B, shape.H, dtype=torch.int64)
    for r in range(world):
        local, bs, hs = bench.shard_of(shape, r, world)
        part = seen[bs, hs]
        assert part.shape == (local.B, local.H)
        assert local.T == shape.T and local.H // local.G == shape.H // shape.G  # whole q/k groups
        seen[bs, hs] += 1
    assert bool((seen == 1).all())
