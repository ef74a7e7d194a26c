"""Context parallelism on 2 GPUs over NCCL: cp_ssd on the two halves of a chunk-128 sequence
(bf16), its output and all eight gradients against the float64 recurrence oracle on the whole
sequence (max|out - ref| / max|ref| < 2e-2, the bf16 contract), and the graph-replayed step
(CpGraphedStep) against cp_ssd, bit for bit."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

NAMES = ("x", "q", "k", "kp", "xp", "adt", "gamma", "beta")


def _shape():
    from zenith_b200.synthetic import SsdShape

    return SsdShape(1, 16384, 4, 64, 128, 4, 128)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir):
    import datetime

    import torch.distributed as dist

    import zenith_b200
    from zenith_b200.parallel import CpGraphedStep, cp_ssd
    from zenith_b200.synthetic import make_inputs

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    s = _shape()
    inp = make_inputs(s, seed=2)
    Tl = s.T // world
    sl = slice(rank * Tl, (rank + 1) * Tl)
    leaves = [(inp[n].to(torch.bfloat16) if n in ("x", "q", "k", "kp", "xp") else inp[n])[:, sl].to(dev).contiguous()
              .requires_grad_() for n in NAMES]
    dy = inp["dy"][:, sl].to(torch.bfloat16).to(dev)
    y = cp_ssd(*leaves, s.chunk)
    y.backward(dy)
    zenith_b200.check_status(dev)
    out = {"y": y.detach().float().cpu()}
    for n, t in zip(NAMES, leaves):
        out["d" + n] = t.grad.detach().float().cpu()
    # the same step with the local work replayed from CUDA graphs, called twice
    step = CpGraphedStep(*(t.detach() for t in leaves), dy, s.chunk)
    for _ in range(2):
        gy, grads = step()
    torch.cuda.synchronize()
    zenith_b200.check_status(dev)
    out["graphed_y"] = gy.float().cpu()
    for n, t in zip(NAMES, grads):
        out["graphed_d" + n] = t.float().cpu()
    del step
    torch.save(out, os.path.join(outdir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_context_parallel_two_gpus_matches_oracle(tmp_path):
    from oracle.recurrence import recurrence_backward, recurrence_forward
    from oracle.ssd_oracle import max_rel_err
    from zenith_b200.synthetic import make_inputs

    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    s = _shape()
    inp = make_inputs(s, seed=2)
    rounded = {n: (inp[n].to(torch.bfloat16) if n in ("x", "q", "k", "kp", "xp") else inp[n]) for n in NAMES}
    dy = inp["dy"].to(torch.bfloat16)
    args = [rounded[n] for n in NAMES]
    ref_y, _ = recurrence_forward(*args)
    ref = recurrence_backward(dy, *args)
    parts = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    errs = {"y": max_rel_err(torch.cat([p["y"] for p in parts], 1), ref_y)}
    errs.update({"d" + n: max_rel_err(torch.cat([p["d" + n] for p in parts], 1), ref["d" + n]) for n in NAMES})
    assert all(v < 2e-2 for v in errs.values()), errs
    # the graph-replayed step runs the same kernels in the same order: identical results
    for p in parts:
        for key in ["y"] + ["d" + n for n in NAMES]:
            assert torch.equal(p["graphed_" + key], p[key]), key
