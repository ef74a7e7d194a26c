"""Context parallelism on CPU ranks (gloo): the exchange logic of zenith_b200.parallel with the
oracle as the per-rank scan, against the oracle on the whole sequence."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from oracle.ssd_oracle import max_rel_err, ssd_backward, ssd_forward
import time

from tests.cp_workers import (NAMES, cp_delay_worker, cp_failure_worker, cp_initial_state_worker, cp_mismatch_worker,
                             cp_parity_worker, shape_for)
from zenith_b200.synthetic import make_inputs


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_context_parallel_matches_whole_sequence(world, tmp_path):
    mp.start_processes(cp_parity_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    s = shape_for(world)
    inp = make_inputs(s, seed=11)
    args = [inp[n].double() for n in NAMES]
    y, _, _ = ssd_forward(*args, s.chunk)
    g = ssd_backward(inp["dy"].double(), *args, s.chunk)
    parts = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    assert max_rel_err(torch.cat([p["y"] for p in parts], 1), y) < 1e-12
    for n in NAMES:
        got = torch.cat([p["d" + n] for p in parts], 1)
        assert max_rel_err(got, g["d" + n]) < 1e-11, n


def test_context_parallel_initial_state_and_its_gradient_on_rank_zero(tmp_path):
    """initial_state starts the whole sequence (rank 0's is used, the others' ignored) and rank 0
    gets its gradient; the other ranks' initial states get none."""
    world = 3
    mp.start_processes(cp_initial_state_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    s = shape_for(world)
    inp = make_inputs(s, seed=12)
    s0 = torch.randn(s.B, s.H, s.P, s.N, generator=torch.Generator().manual_seed(5), dtype=torch.float64)
    args = [inp[n].double() for n in NAMES]
    y, _, _ = ssd_forward(*args, s.chunk, initial_state=s0)
    g = ssd_backward(inp["dy"].double(), *args, s.chunk, initial_state=s0)
    parts = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    assert max_rel_err(torch.cat([p["y"] for p in parts], 1), y) < 1e-12
    for n in NAMES:
        assert max_rel_err(torch.cat([p["d" + n] for p in parts], 1), g["d" + n]) < 1e-11, n
    assert max_rel_err(parts[0]["dinitial_state"], g["dinitial_state"]) < 1e-11
    assert all(p["dinitial_state"] is None for p in parts[1:])


def test_context_parallel_rank_failure_ends_in_an_error_not_a_hang(tmp_path):
    ctx = mp.start_processes(cp_failure_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    try:
        while not ctx.join(timeout=90):
            pass
    except mp.ProcessRaisedException as e:
        assert "injected failure on rank 1" in str(e)
    for p in ctx.processes:
        if p.is_alive():
            p.join(timeout=60)
        assert not p.is_alive(), "a rank hung"
    msg = (tmp_path / "rank0.txt").read_text() if (tmp_path / "rank0.txt").exists() else "rank 0 died"
    assert msg.startswith("error") or msg == "rank 0 died", msg


def _run_pair(worker, tmp_path, bound_s):
    """Start two ranks of `worker`; both must exit within `bound_s` seconds; returns what each
    recorded."""
    t0 = time.monotonic()
    ctx = mp.start_processes(worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=False, start_method="spawn")
    while not ctx.join(timeout=5):
        assert time.monotonic() - t0 < bound_s, "a rank hung"
    return [(tmp_path / f"rank{r}.txt").read_text() for r in range(2)]


def test_context_parallel_shape_mismatch_raises_on_every_rank(tmp_path):
    """A rank whose local range has another state size: ValueError on both ranks, before any
    send / recv of a state."""
    res = _run_pair(cp_mismatch_worker, tmp_path, 120)
    for r in res:
        assert r.startswith("error: ValueError: cp_ssd: the ranks' local ranges differ"), r


def test_context_parallel_stalled_rank_ends_in_a_timeout_not_a_hang(tmp_path):
    """Rank 1 sleeps past the 4 s process-group timeout before the exchange: rank 0's first
    collective ends with an error; rank 1, arriving late, ends with one too."""
    res = _run_pair(cp_delay_worker, tmp_path, 120)
    assert res[0].startswith("error: ") and "Timed out" in res[0], res[0]
    assert res[1].startswith("error: "), res[1]
