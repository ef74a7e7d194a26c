"""Worker functions for the multi-process (gloo, CPU) context-parallel tests.  The local scan is
the CPU oracle, injected through zenith_b200.parallel.LocalScan, so these tests check the
exchange logic (chain order, state combine, gradient hand-back) without a GPU."""
import datetime
import os
import time

import torch
import torch.distributed as dist

from oracle.ssd_oracle import ssd_backward, ssd_forward
from zenith_b200.parallel import LocalScan, cp_ssd
from zenith_b200.synthetic import SsdShape, make_inputs

NAMES = ("x", "q", "k", "kp", "xp", "adt", "gamma", "beta")


def oracle_scan() -> LocalScan:
    def final_state(inp, chunk, init):
        return ssd_forward(*inp, chunk, initial_state=init)[1]

    def forward(inp, chunk, init):
        y, _, _ = ssd_forward(*inp, chunk, initial_state=init)
        return y, None

    def dinitial(dy, inp, chunk):
        return ssd_backward(dy, *inp, chunk)["dinitial_state"]

    def backward(dy, inp, saved, chunk, init, dfinal):
        g = ssd_backward(dy, *inp, chunk, initial_state=init, dfinal=dfinal)
        return tuple(g["d" + n] for n in NAMES + ("initial_state",))

    def total_decay(adt):
        return torch.exp(adt.sum(1))

    def combine(s_prev, d, f):
        return d[..., None, None] * s_prev + f

    return LocalScan(final_state, forward, dinitial, backward, total_decay, combine)


def _init(rank, world, port, timeout_s=20):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def shape_for(world):
    return SsdShape(2, 64 * world, 3, 6, 5, 3, 16)


def cp_parity_worker(rank, world, port, outdir):
    _init(rank, world, port)
    s = shape_for(world)
    inp = make_inputs(s, seed=11)
    Tl = s.T // world
    sl = slice(rank * Tl, (rank + 1) * Tl)
    leaves = [inp[n][:, sl].double().clone().requires_grad_() for n in NAMES]
    y = cp_ssd(*leaves, s.chunk, impl=oracle_scan())
    y.backward(inp["dy"][:, sl].double())
    out = {"y": y.detach()}
    for n, t in zip(NAMES, leaves):
        out["d" + n] = t.grad.detach()
    torch.save(out, os.path.join(outdir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def cp_initial_state_worker(rank, world, port, outdir):
    """An initial state on rank 0 (the other ranks pass one too, which they must ignore): outputs,
    input gradients and rank 0's initial-state gradient."""
    _init(rank, world, port)
    s = shape_for(world)
    inp = make_inputs(s, seed=12)
    s0 = torch.randn(s.B, s.H, s.P, s.N, generator=torch.Generator().manual_seed(5), dtype=torch.float64)
    Tl = s.T // world
    sl = slice(rank * Tl, (rank + 1) * Tl)
    leaves = [inp[n][:, sl].double().clone().requires_grad_() for n in NAMES]
    init = (s0 if rank == 0 else torch.zeros_like(s0)).clone().requires_grad_()
    y = cp_ssd(*leaves, s.chunk, impl=oracle_scan(), initial_state=init)
    y.backward(inp["dy"][:, sl].double())
    out = {"y": y.detach(), "dinitial_state": init.grad}
    for n, t in zip(NAMES, leaves):
        out["d" + n] = t.grad.detach()
    torch.save(out, os.path.join(outdir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def cp_failure_worker(rank, world, port, outdir):
    """Rank 1 fails before the exchange; rank 0 must end with an error, not hang."""
    _init(rank, world, port)
    s = shape_for(world)
    inp = make_inputs(s, seed=11)
    Tl = s.T // world
    sl = slice(rank * Tl, (rank + 1) * Tl)
    if rank == 1:
        raise RuntimeError("injected failure on rank 1")
    leaves = [inp[n][:, sl].double() for n in NAMES]
    try:
        # rank 0 waits in the exchange's all_gather for rank 1, which never arrives
        y = cp_ssd(*(t.requires_grad_() for t in leaves), s.chunk, impl=oracle_scan())
        y.sum().backward()
        result = "no error"
    except Exception as e:  # noqa: BLE001 - any error is the expected outcome
        result = "error: " + type(e).__name__
    with open(os.path.join(outdir, f"rank{rank}.txt"), "w") as f:
        f.write(result)


def _run_and_record(rank, outdir, s, sl):
    inp = make_inputs(s, seed=11)
    leaves = [inp[n][:, sl].double().requires_grad_() for n in NAMES]
    try:
        y = cp_ssd(*leaves, s.chunk, impl=oracle_scan())
        y.sum().backward()
        result = "no error"
    except Exception as e:  # noqa: BLE001 - the test checks which error
        result = "error: " + type(e).__name__ + ": " + str(e).splitlines()[0][:200]
    with open(os.path.join(outdir, f"rank{rank}.txt"), "w") as f:
        f.write(result)


def cp_mismatch_worker(rank, world, port, outdir):
    """Rank 1 passes a local range with a larger head dimension P (a state of another size): every
    rank must raise ValueError before any state is sent."""
    _init(rank, world, port)
    s = shape_for(world)
    if rank == 1:
        s = SsdShape(s.B, s.T, s.H, s.P + 1, s.N, s.G, s.chunk)
    Tl = s.T // world
    _run_and_record(rank, outdir, s, slice(rank * Tl, (rank + 1) * Tl))


def cp_delay_worker(rank, world, port, outdir):
    """Rank 1 stalls past the process group's timeout before the exchange: rank 0 must end with an
    error (the timeout), not wait for it."""
    _init(rank, world, port, timeout_s=4)
    s = shape_for(world)
    if rank == 1:
        time.sleep(10)
    Tl = s.T // world
    _run_and_record(rank, outdir, s, slice(rank * Tl, (rank + 1) * Tl))
