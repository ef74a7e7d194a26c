#!/usr/bin/env python
"""SSD chunked-scan forward + backward benchmark on B200 (rewrite of the reference's
scripts/bench_ssd.py, which timed zenith.mamba3.ssd fwd+bwd on Apple MPS).

One step = one forward and one backward of the SSD scan over one batch of the model-scale
layer workload (B8 T2048 H24 P64 N128, chunk 64, bf16 vectors with fp32 per-token scalars,
synthetic inputs with the Mamba-3 value distributions).  Multi-GPU: one process per GPU
(torchrun); the (batch, head) chains of the one job are independent, so rank r runs its 1/N
share of them (by batch, else by heads; no collective on the data path; ``--replicate`` gives
every rank a whole job instead); the timed region is bracketed by barriers and the slowest
rank's CUDA-event time is reported.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  ``--impl reference`` times the reference on the host CPU cores
instead (rank 0 only): its own ``zenith.mamba3.ssd`` (or ``ZenithForCausalLM`` for the LM step)
in fp32 under PyTorch autograd when the reference package is installed under baseline/_ref, else
the restatement of zenith/mamba3.py:30-56 with the same tensor operations.
"""
from __future__ import annotations

import argparse
import csv
import datetime
import io
import json
import os
import pathlib
import statistics
import subprocess
import sys
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "SSD fwd+bwd tokens/s"
METRIC_FWD = "SSD fwd tokens/s"  # --workload infer: forward with the final state, no saved states
UNIT = "tokens/s"
NAMES = ("x", "q", "k", "kp", "xp", "adt", "gamma", "beta")
VEC = ("x", "q", "k", "kp", "xp")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default="layer")
    ap.add_argument("--replicate", action="store_true",
                    help="N > 1: every rank runs a whole job of its own (weak scaling) instead of 1/N of one job")
    ap.add_argument("--eager", action="store_true", help="time eager launches instead of CUDA-graph replays")
    ap.add_argument("--dtype", choices=("bf16", "fp32"), default="bf16",
                    help="vector dtype (fp32: the drop-in's fp32 path, Mamba3.forward without autocast)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="budget of the CPU baseline sample")
    return ap.parse_args()


def algorithmic_bytes(shape, e_in=2, e_sc=4):
    """Per token per head (each input read once per pass, each output written once):
    fwd = e(2P + 3N/r) + 3 e_s + e P ;  bwd = e(2P + 3N/r) + 3 e_s + e P (dy) + e(2P + 3N/r) + 3 e_s."""
    r = shape.H // shape.G
    vin = e_in * (2 * shape.P + 3 * shape.N / r) + 3 * e_sc
    fwd = vin + e_in * shape.P
    bwd = vin + e_in * shape.P + vin
    return fwd, bwd


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


FP32_FMA_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12  # nominal B200 CUDA-core fp32: SMs x lanes x FMA x max clock


def flop_roofline(shape, th, dom, dms, fwd_only, dtype="bf16"):
    """The flop side of the dominant kernel: algorithmic flops per token-head (forward
    4 L N / r + 4 L P + 6 N P, backward twice that) over its time, against the measured
    burst bf16 tensor peak (bf16, tensor-core kernels) or the nominal fp32 FMA peak (fp32, SIMT)."""
    L, r = 64, shape.H // shape.G
    f = 4 * L * shape.N // r + 4 * L * shape.P + 6 * shape.N * shape.P
    flops = (f if dom == "fwd" else 2 * f) * th
    if dtype == "fp32":
        peak, kind = FP32_FMA_TFLOPS, "nominal fp32 FMA (CUDA cores)"
    else:
        p = ROOT / "MEASURED_PEAKS.json"
        peak, kind = ((float(json.loads(p.read_text())["bf16_tflops"]), "measured bf16 tensor") if p.exists()
                      else (1590.0, "fallback bf16 tensor"))
    achieved = flops / (dms / 1e3) / 1e12
    return {"kernel": "ssd_" + dom, "achieved_tflops": achieved, "peak_tflops": peak, "peak_kind": kind,
            "frac": achieved / peak, "flops_per_launch": flops, "algorithmic_chunk": L}


def traffic_from_profile(kernel: str):
    """DRAM bytes per launch from the committed ncu summary (profiles/traffic.json), if any."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    v = d.get(kernel)
    return None if v is None else float(v)


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling while the timed region runs."""

    FIELDS = ("clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.active",
              "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
              "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        import threading

        self.proc = None
        self.lines: list[str] = []
        self.error = ""
        self.first = threading.Event()
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            if not uuid.startswith("GPU-"):
                uuid = "GPU-" + uuid
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={uuid}", "--query-gpu=" + ",".join(self.FIELDS), "--format=csv,noheader,nounits",
                 "-lms", "10"], stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
        except Exception as e:  # no nvidia-smi: report it in the line
            self.error = repr(e)
            return

        def reader():
            for line in self.proc.stdout:
                self.lines.append(line)
                self.first.set()
            self.first.set()

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()
        self.first.wait(timeout=10.0)  # nvidia-smi takes a moment to start: sample before timing

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "error": self.error}
        n_before = len(self.lines)
        self.proc.terminate()
        try:
            _, err = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            _, err = self.proc.communicate()
        self.thread.join(timeout=5)
        out = "".join(self.lines[:max(n_before, 1)])
        rows = [r for r in csv.reader(io.StringIO(out)) if len(r) >= len(self.FIELDS)]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "error": (err or "")[-200:]}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        sm = [num(r[0]) for r in rows if num(r[0]) is not None]
        mx = [num(r[1]) for r in rows if num(r[1]) is not None]
        reasons = set()
        for r in rows:
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), r[4:8]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def make_device_inputs(shape, rank, dev):
    from zenith_b200.synthetic import make_inputs

    inp = make_inputs(shape, seed=rank)
    out = {}
    for n in NAMES + ("dy",):
        t = inp[n].to(torch.bfloat16) if (n in VEC or n == "dy") else inp[n]
        out[n] = t.to(dev).contiguous()
    return out


# ------------------------------------------------------------------------------------------------
# CPU baseline / reference arm


def reference_package():
    """The reference package as installed under baseline/_ref (``pip install --target``), or None
    with the reason it is not there or does not import."""
    path = ROOT / "baseline" / "_ref"
    if not (path / "zenith" / "mamba3.py").exists():
        return None, "no reference installed under baseline/_ref"
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))
    try:
        import zenith
        import zenith.mamba3  # noqa: F401
    except Exception as e:  # noqa: BLE001 - any import failure falls back to the restatement
        return None, f"the installed reference does not import ({type(e).__name__}: {str(e)[:120]})"
    return zenith, ""


def reference_ssd():
    """(ssd function, kind, description): the reference's own ``zenith.mamba3.ssd`` when installed,
    else its restatement with the same tensor operations (oracle/ssd_reference_ops.py)."""
    ref, why = reference_package()
    if ref is not None:
        return ref.mamba3.ssd, "reference", "reference zenith.mamba3.ssd (installed under baseline/_ref)"
    from oracle.ssd_reference_ops import ssd_reference_ops

    return (ssd_reference_ops, "port",
            f"reference ssd (zenith/mamba3.py:30-56) restated with its tensor-op sequence [{why}]")


def cpu_reference_sample(shape, seconds: float, max_reps: int | None = None, fwd_only: bool = False):
    """Time the reference's scan on the host CPU (``reference_ssd``), fp32, forward plus PyTorch
    autograd backward, on a one-sequence slice of the workload; returns (tokens/s, cores, reps,
    sample string, kind)."""
    from zenith_b200.synthetic import SsdShape, make_inputs

    ssd_fn, kind, origin = reference_ssd()

    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    # one sequence of the workload; for long contexts an 8192-token slice (the scan is linear in T,
    # so tokens/s of a slice stands for the whole sequence)
    sl = SsdShape(1, min(shape.T, 8192), shape.H, shape.P, shape.N, shape.G, shape.chunk)
    inp = make_inputs(sl, seed=0)
    if sl.G != sl.H:  # the reference has one q/k per head: grouped q/k/kp are expanded to the heads
        for n in ("q", "k", "kp"):
            inp[n] = inp[n].repeat_interleave(sl.H // sl.G, dim=2)
    leaves = [(inp[n].to(torch.bfloat16).float() if n in VEC else inp[n]).requires_grad_() for n in NAMES]
    dy = inp["dy"].to(torch.bfloat16).float()

    def once():
        if fwd_only:
            with torch.no_grad():
                ssd_fn(*leaves, sl.chunk)
            return
        y = ssd_fn(*leaves, sl.chunk)
        y.backward(dy)
        for t in leaves:
            t.grad = None

    once()  # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        once()
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds or (max_reps is not None and reps >= max_reps):
            break
    tok_s = reps * sl.B * sl.T / el
    what = "forward" if fwd_only else "fp32 forward + autograd backward"
    sample = (f"{origin}, {what} on host CPU, "
              f"1 sequence (T{sl.T} H{sl.H} P{sl.P} N{sl.N} G{sl.G} chunk {sl.chunk}) of the B{shape.B} workload, "
              f"{reps} reps in {el:.1f} s, {cores} threads")
    return tok_s, cores, reps, sample, kind


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from zenith_b200.synthetic import SHAPES

    shape = SHAPES[args.workload]
    seconds = max(3.0, min(120.0, 2.0 * (args.steps + args.warmup)))
    fwd_only = args.workload == "infer"
    tok_s, cores, reps, sample, kind = cpu_reference_sample(shape, seconds, fwd_only=fwd_only)
    ms = shape.B * shape.T / tok_s * 1e3
    line = {
        "impl": "reference", "metric": METRIC_FWD if fwd_only else METRIC, "value": tok_s, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": shape.name, "B": shape.B, "T": shape.T, "H": shape.H, "P": shape.P, "N": shape.N,
                   "chunk": shape.chunk, "device": "host cpu"},
        "cpu_baseline": {"value": tok_s, "unit": UNIT, "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": tok_s, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------------------------
# our arm


L2_BYTES = 126 << 20  # B200 L2


def shard_of(shape, rank, world):
    """Rank r's part of one job: contiguous ranges of the B*H independent (batch, head) chains,
    by batch when the ranks divide B (every rank keeps whole sequences), else by heads (whole
    q/k groups).  Returns (local shape, batch slice, head slice)."""
    from zenith_b200.synthetic import SsdShape

    if shape.B % world == 0:
        bl = shape.B // world
        return (SsdShape(bl, shape.T, shape.H, shape.P, shape.N, shape.G, shape.chunk, shape.name),
                slice(rank * bl, (rank + 1) * bl), slice(None))
    if shape.H % world == 0 and shape.G % world == 0:
        hl, gl = shape.H // world, shape.G // world
        return (SsdShape(shape.B, shape.T, hl, shape.P, shape.N, gl, shape.chunk, shape.name),
                slice(None), slice(rank * hl, (rank + 1) * hl))
    raise SystemExit(f"{world} ranks do not divide the batch ({shape.B}) or the q/k groups ({shape.G})")


def run_ours(args):
    import torch.distributed as dist

    import zenith_b200
    from zenith_b200 import _lib
    from zenith_b200.ssd import ssd_bwd_op, ssd_fwd_op
    from zenith_b200.synthetic import SHAPES, SsdShape, make_inputs

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    shape = SHAPES[args.workload]
    # Long-context workload on N > 1 GPUs: context parallelism (each rank owns T/N tokens of the
    # sequence; the boundary states move by one NCCL all_gather per direction).  Otherwise the B*H
    # independent (batch, head) chains of ONE job are split over the ranks (no collective on the
    # data path), or with --replicate every rank runs a whole job of its own (weak scaling).
    cp = args.workload == "long" and world > 1
    fwd_only = args.workload == "infer"  # C4: inference forward returning the final state (decode hand-off)
    replicate = args.replicate and not cp
    if cp:
        # each rank draws only its own range of the sequence (the whole one is 7 GB of host memory)
        local_shape = SsdShape(shape.B, shape.T // world, shape.H, shape.P, shape.N, shape.G, shape.chunk)
        full = make_inputs(local_shape, seed=rank)
        part = {n: v for n, v in full.items() if n != "D"}
    elif replicate or world == 1:
        full = make_inputs(shape, seed=rank)
        local_shape = shape
        part = {n: v for n, v in full.items() if n != "D"}
    else:
        full = make_inputs(shape, seed=0)
        local_shape, sl_b, sl_h = shard_of(shape, rank, world)
        r = shape.H // shape.G
        sl_g = sl_h if sl_h == slice(None) else slice(sl_h.start // r, sl_h.stop // r)
        part = {n: (v[sl_b, :, sl_g] if n in ("q", "k", "kp") else v[sl_b, :, sl_h]) for n, v in full.items() if n != "D"}
    vdt = torch.float32 if args.dtype == "fp32" else torch.bfloat16
    inp = {n: (t.to(vdt) if (n in VEC or n == "dy") else t).to(dev).contiguous() for n, t in part.items()}
    del full, part
    chunk = shape.chunk
    fwd_b, bwd_b = algorithmic_bytes(shape, e_in=vdt.itemsize)
    if fwd_only:
        bwd_b = 0
    th = local_shape.B * local_shape.T * local_shape.H
    step_bytes = (fwd_b + bwd_b) * th
    tokens_per_step = shape.B * shape.T * (world if replicate else 1)

    # Rotating copies of the inputs, so that a step's inputs were last touched at least two steps
    # earlier and at least twice the L2 has been streamed since (a step reads and writes
    # step_bytes): each step starts from HBM, not from a warm L2.
    n_sets = 1 if step_bytes >= 2 * L2_BYTES else int(-(-2 * L2_BYTES // step_bytes)) + 1
    sets = [inp] + [{n: t.clone() for n, t in inp.items()} for _ in range(n_sets - 1)]

    if cp:
        from zenith_b200.parallel import _check_local_shapes, cp_ssd

        _check_local_shapes(sets[0]["x"], sets[0]["q"], None)  # once: every step has the same shapes

        def step(st, ev=None):
            leaves = [st[n].detach().requires_grad_() for n in NAMES]
            if ev is not None:
                ev[0].record()
            y = cp_ssd(*leaves, chunk, check_shapes=False)
            if ev is not None:
                ev[1].record()
            y.backward(st["dy"])
            if ev is not None:
                ev[2].record()
            return y
    elif fwd_only:
        def step(st, ev=None):
            a = [st[n] for n in NAMES]
            if ev is not None:
                ev[0].record()
            y, fin, _ = ssd_fwd_op(*a, chunk, None, False, False)
            if ev is not None:
                ev[1].record()
                ev[2].record()
            return y, fin
    else:
        def step(st, ev=None):
            a = [st[n] for n in NAMES]
            if ev is not None:
                ev[0].record()
            y, fin, states = ssd_fwd_op(*a, chunk, None, True, False)
            if ev is not None:
                ev[1].record()
            g = ssd_bwd_op(st["dy"], *a, states, chunk, None, None, False)
            if ev is not None:
                ev[2].record()
            return y, g

    def barrier():
        if world > 1:
            dist.barrier()

    for i in range(max(args.warmup, 3)):
        step(sets[i % n_sets])
    torch.cuda.synchronize()
    zenith_b200.check_status(dev)

    # The step's launches are captured once per buffer set in a CUDA graph and replayed: the
    # same kernels on the same data each step, without the host's per-launch cost (which
    # would set the pace once a rank's share of the job takes ~100 us).  Context parallelism
    # replays its local work from graphs with the two NCCL all_gathers issued between them
    # (zenith_b200.parallel.CpGraphedStep; collectives stay outside the graphs).
    graphs = []
    cp_steps = []
    if cp and not args.eager:
        from zenith_b200.parallel import CpGraphedStep

        cp_steps = [CpGraphedStep(*(st[n] for n in NAMES), st["dy"], chunk) for st in sets]
        for c in cp_steps:  # one untimed call of each
            c()
        torch.cuda.synchronize()
        zenith_b200.check_status(dev)
    if not cp and not args.eager:
        keep = []
        for st in sets:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                keep.append(step(st))
            graphs.append(g)
        for g in graphs:  # one untimed replay of each
            g.replay()
        torch.cuda.synchronize()
        zenith_b200.check_status(dev)

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    launches0 = _lib.launch_count()
    start.record()
    for i in range(args.steps):
        if graphs:
            graphs[i % n_sets].replay()
        elif cp_steps:
            cp_steps[i % n_sets]()
        else:
            step(sets[i % n_sets])
    end.record()
    torch.cuda.synchronize()
    launches = _lib.launch_count() - launches0
    if graphs or cp_steps:  # replays launch without the host library: count the captured step's launches
        c0 = _lib.launch_count()
        step(sets[0])
        torch.cuda.synchronize()
        launches = (_lib.launch_count() - c0) * args.steps
    barrier()
    clocks = sampler.stop()
    zenith_b200.check_status(dev)
    elapsed_ms = start.elapsed_time(end)

    # per-kernel durations of the forward and backward launches (events around each op on the
    # launching stream, eager, over the same number of steps and the same buffer rotation)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        if cp_steps:
            cp_steps[i % n_sets](evs[i])
        else:
            step(sets[i % n_sets], evs[i])
    torch.cuda.synchronize()
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    bwd_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    del graphs, cp_steps
    t = torch.tensor([elapsed_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms = float(t.item())
    ms_per_step = elapsed_ms / args.steps
    value = tokens_per_step / (ms_per_step / 1e3)

    # End-to-end through the public API with host buffers (pinned).  Every step copies its inputs and
    # dy in (host -> device) and y plus all eight gradients out (device -> host) inside the timed
    # region.  Copies run on their own streams with two device buffer sets, so step i+1's inputs
    # and step i-1's outputs cross PCIe while step i computes, as a data pipeline would.
    # (--workload infer: inputs in, y and the final state out, no backward)
    in_names = NAMES if fwd_only else NAMES + ("dy",)
    host = {n: inp[n].cpu().pin_memory() for n in in_names}
    B_, T_, H_, P_ = inp["x"].shape
    out_shapes = ({"y": (inp["x"].shape, inp["x"].dtype), "final": ((B_, H_, P_, inp["q"].shape[3]), torch.float32)}
                  if fwd_only else {n: (host["x" if n == "y" else n].shape, host["x" if n == "y" else n].dtype)
                                    for n in ("y",) + NAMES})
    outs = [{n: torch.empty(sh, dtype=dt).pin_memory() for n, (sh, dt) in out_shapes.items()} for _ in range(2)]
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = sum(v.numel() * v.element_size() for v in outs[0].values())
    cur = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    dbuf = [{n: torch.empty_like(inp[n]) for n in in_names} for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_free = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    for e in ev_free:
        e.record(cur)

    def issue_h2d(i):
        k = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_free[k])  # step i-2 has finished with buffer set k
            for n in in_names:
                dbuf[k][n].copy_(host[n], non_blocking=True)
            ev_in[k].record(s_in)

    def compute_and_d2h(i):
        k = i % 2
        cur.wait_event(ev_in[k])
        if fwd_only:
            with torch.no_grad():
                y, fin = zenith_b200.ssd(*(dbuf[k][n] for n in NAMES), chunk, return_final_state=True)
            ev_free[k].record(cur)
            ev_done[k].record(cur)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_done[k])
                for n, t in (("y", y), ("final", fin)):
                    outs[k][n].copy_(t, non_blocking=True)
                    t.record_stream(s_out)
            return
        leaves = [dbuf[k][n].detach().requires_grad_() for n in NAMES]
        y = zenith_b200.parallel.cp_ssd(*leaves, chunk) if cp else zenith_b200.ssd(*leaves, chunk)
        y.backward(dbuf[k]["dy"])
        ev_free[k].record(cur)
        ev_done[k].record(cur)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_done[k])
            outs[k]["y"].copy_(y.detach(), non_blocking=True)
            y.record_stream(s_out)
            for n, lf in zip(NAMES, leaves):
                outs[k][n].copy_(lf.grad, non_blocking=True)
                lf.grad.record_stream(s_out)

    def e2e_run(steps):
        issue_h2d(0)
        for i in range(steps):
            if i + 1 < steps:
                issue_h2d(i + 1)
            compute_and_d2h(i)
        cur.wait_stream(s_out)

    e2e_steps = max(3, args.steps)
    e2e_run(2)
    torch.cuda.synchronize()
    barrier()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(cur)
    s_in.wait_event(s2)
    e2e_run(e2e_steps)
    e2.record(cur)
    torch.cuda.synchronize()
    zenith_b200.check_status(dev)
    t2 = torch.tensor([s2.elapsed_time(e2)], device=dev)
    if world > 1:
        dist.all_reduce(t2, op=dist.ReduceOp.MAX)
    e2e_value = tokens_per_step / (float(t2.item()) / e2e_steps / 1e3)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tok_s, cores, reps, sample, kind = cpu_reference_sample(shape, args.cpu_seconds, fwd_only=fwd_only)
        cpu = {"value": tok_s, "unit": UNIT, "cores": cores, "kind": kind, "sample": sample}

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    peak, peak_kind = peaks()
    if fwd_only:
        bwd_b = 0
    kern = {"fwd": (fwd_ms, fwd_b * th, "ssd_fwd"), "bwd": (bwd_ms, bwd_b * th, "ssd_bwd")}
    dom = "fwd" if fwd_only else max(kern, key=lambda k: kern[k][0])
    dms, dbytes, dname = kern[dom]
    achieved = dbytes / (dms / 1e3) / 1e9
    step_gbs = (fwd_b + bwd_b) * th / (ms_per_step / 1e3) / 1e9
    if cp:
        par = f"context-parallel x{world} (T/{world} per rank, boundary states by one NCCL all_gather per direction)"
    elif replicate:
        par = f"replicated x{world} (each rank a whole B{shape.B} job of its own)"
    else:
        par = (f"batch x heads sharded x{world}: (batch, head) chains {local_shape.B * local_shape.H} of "
               f"{shape.B * shape.H} per rank, no collective on the data path")
    line = {
        "metric": METRIC_FWD if fwd_only else METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak" if replicate else "strong",
        "vs_baseline": None, "dtype": args.dtype, "data": "synthetic",
        "config": {"workload": shape.name, "B": shape.B, "T": shape.T, "H": shape.H, "P": shape.P,
                   "N": shape.N, "G": shape.G, "chunk": shape.chunk, "vector_dtype": args.dtype, "scalar_dtype": "fp32",
                   "kernels": "SIMT (fp32 FMA)" if args.dtype == "fp32" else "tensor-core (tcgen05)",
                   "parallelism": par, "B_per_rank": local_shape.B, "H_per_rank": local_shape.H,
                   "tokens_per_rank": local_shape.B * local_shape.T,
                   "timed_launch": ("eager" if args.eager else
                                    "CUDA graphs of the local work replayed, the NCCL all_gathers issued between them"
                                    if cp else "CUDA graph of one step, replayed"),
                   "l2": (f"inputs larger than L2: {step_bytes / 1e9:.3f} GB read+written per step per rank, "
                          f"{n_sets} rotating input set(s) so each step starts from HBM")},
        "roofline": {"bound": "hbm", "kernel": dname, "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "traffic": (traffic_from_profile(dname if args.workload == "layer" else dname + "_infer")
                                 if args.workload in ("layer", "infer") and args.dtype == "bf16" else None),
                     "algorithmic_bytes_per_launch": dbytes, "launch_ms": dms},
        "step_roofline": {"achieved_gbs": step_gbs, "frac": step_gbs / peak,
                          "algorithmic_bytes_per_token_head": fwd_b + bwd_b, "fwd_ms": fwd_ms, "bwd_ms": bwd_ms},
        "flop_roofline": flop_roofline(shape, th, dom, dms, fwd_only, args.dtype),
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------------------------
# --workload mamba3: the fused Mamba-3 layer body (prologue, scan, epilogue; mamba3.py:96-119)

LAYER_METRIC = "Mamba-3 layer body fwd+bwd tokens/s"


def layer_inputs(B, T, H, P, N, dev, dtype, seed=0):
    """The in_proj split and the layer parameters, with the reference module's scales."""
    g = torch.Generator().manual_seed(seed)
    mk = lambda *sh: torch.randn(*sh, generator=g)  # noqa: E731
    t = {"x": mk(B, T, H, P), "z": mk(B, T, H, P), "Bm": mk(B, T, N), "Cm": mk(B, T, N), "dd_dt": mk(B, T, H),
         "dd_A": mk(B, T, H), "trap": mk(B, T, H), "ang": mk(B, T, N // 4)}
    dt = torch.exp(torch.rand(H, generator=g) * (torch.log(torch.tensor(0.1)) - torch.log(torch.tensor(1e-3)))
                   + torch.log(torch.tensor(1e-3)))
    prm = {"dt_bias": dt + torch.log(-torch.expm1(-dt)), "B_bias": torch.ones(H, N), "C_bias": torch.ones(H, N),
           "B_norm_w": torch.ones(N), "C_norm_w": torch.ones(N), "D": torch.ones(H)}
    dout = mk(B, T, H, P)
    return ({n: v.to(dev, dtype) for n, v in t.items()}, {n: v.to(dev) for n, v in prm.items()}, dout.to(dev, dtype))


def layer_bytes(H, P, N, e=2):
    """Per token per head: the layer inputs read and outputs written once (B / C / ang rows are per
    token, shared by the heads).  fwd: x, z, B, C, ang, 3 scalars in; out.  bwd: x, z, dout, B, C,
    ang, 3 scalars in; dx, dz, dB, dC, dang, 3 scalar gradients out."""
    rows = e * (2 * N + N // 4) / H
    fwd = e * 2 * P + rows + 3 * e + e * P
    bwd = (e * 3 * P + rows + 3 * e) + (e * 2 * P + rows + 3 * e)
    return fwd, bwd


def run_layer(args):
    import zenith_b200
    from zenith_b200 import _lib

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, T, H, P, N = 8, 2048, 24, 64, 128
    t, prm, dout = layer_inputs(B, T, H, P, N, dev, torch.bfloat16)
    names = ("x", "z", "Bm", "Cm", "dd_dt", "dd_A", "trap", "ang")
    leaves = [t[n].requires_grad_() for n in names] + [prm[n].requires_grad_() for n in prm]

    def step():
        out = zenith_b200.mamba3_ssd_fused(*leaves, chunk_size=64, scan_dtype=torch.bfloat16)
        out.backward(dout)
        for lf in leaves:
            lf.grad = None

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    zenith_b200.check_status(dev)
    sampler = ClockSampler(0)
    launches0 = _lib.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    zenith_b200.check_status(dev)
    ms = e0.elapsed_time(e1) / args.steps
    fwd_b, bwd_b = layer_bytes(H, P, N)
    peak, peak_kind = peaks()
    gbs = (fwd_b + bwd_b) * B * T * H / (ms / 1e3) / 1e9
    line = {
        "metric": LAYER_METRIC, "value": B * T / (ms / 1e3), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"Mamba-3 layer body B{B} T{T} H{H} P{P} N{N} chunk 64 (in_proj split -> gated y)",
                   "io_dtype": "bf16", "scan_dtype": "bf16", "l2": "inputs larger than L2"},
        "roofline": {"bound": "hbm", "kernel": "layer step", "achieved": gbs, "peak": peak, "unit": "GB/s",
                     "frac": gbs / peak, "peak_kind": peak_kind, "traffic": None,
                     "algorithmic_bytes_per_token_head": fwd_b + bwd_b},
        "gpu_launches": _lib.launch_count() - launches0,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------------------------
# --workload decode: the recurrent (decode) step that continues the inference prefill (scope row f3):
# one token for each of B64 sequences x H32 heads (P64 N64, 4 q/k groups); the fp32 states are
# advanced in place (zb_ssd_decode).  The reference has no decode path (its generation re-runs the
# chunked scan over the whole prefix, zenith/model.py:79-99); the CPU baseline is the per-token
# recurrence of the reference's test (tests/test_mamba3.py:10-21) in fp32 torch on the host.

DECODE_METRIC = "SSD decode tokens/s"
DECODE_SHAPE = dict(B=64, H=32, P=64, N=64, G=4)


def decode_bytes(B, H, P, N, G):
    """Algorithmic bytes of one decode step: the fp32 state read and written once, the token's bf16
    vectors (x, xp [H, P]; q, k, kp [G, N]) and fp32 scalars read, y written (bf16)."""
    return B * (2 * H * P * N * 4 + 2 * (2 * H * P + 3 * G * N) + 3 * H * 4 + 2 * H * P)


def decode_tokens(B, H, P, N, G, n_tok, dev, dtype=torch.bfloat16):
    """n_tok single-token inputs (T = 1 views) with the Mamba-3 value distributions."""
    from zenith_b200.synthetic import SsdShape, make_inputs

    inp = make_inputs(SsdShape(B, 64, H, P, N, G, 64), seed=7)
    out = []
    for t in range(n_tok):
        out.append({n: (inp[n][:, t:t + 1].to(dtype) if n in VEC else inp[n][:, t:t + 1]).to(dev).contiguous()
                    for n in NAMES})
    return out


def cpu_decode_sample(seconds: float):
    """The per-token recurrence h = e^{adt} h + g x k^T + b xp kp^T, y = h q in fp32 torch on the host
    cores for the whole decode batch; returns (tokens/s, cores, sample string)."""
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    B, H, P, N, G = (DECODE_SHAPE[k] for k in ("B", "H", "P", "N", "G"))
    tok = decode_tokens(B, H, P, N, G, 4, torch.device("cpu"), torch.float32)
    h = torch.zeros(B, H, P, N)
    r = H // G

    def once(tk):
        nonlocal h
        q, k, kp = (tk[n][:, 0].repeat_interleave(r, dim=1) for n in ("q", "k", "kp"))
        x, xp = tk["x"][:, 0], tk["xp"][:, 0]
        a, g, b = (tk[n][:, 0] for n in ("adt", "gamma", "beta"))
        h = torch.exp(a)[..., None, None] * h + (g[..., None, None] * x[..., :, None]) * k[..., None, :] \
            + (b[..., None, None] * xp[..., :, None]) * kp[..., None, :]
        return torch.einsum("bhpn,bhn->bhp", h, q)

    once(tok[0])
    reps, t0 = 0, time.perf_counter()
    while True:
        once(tok[reps % 4])
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    sample = (f"per-token recurrence (tests/test_mamba3.py:10-21) in fp32 torch on host CPU, the whole B{B} x H{H} "
              f"decode batch, {reps} steps in {el:.1f} s, {cores} threads")
    return reps * B / el, cores, sample


def run_decode(args):
    import zenith_b200
    from zenith_b200 import _lib

    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return 0
        seconds = max(3.0, min(60.0, 0.5 * (args.steps + args.warmup)))
        tok_s, cores, sample = cpu_decode_sample(seconds)
        B = DECODE_SHAPE["B"]
        print(json.dumps({
            "impl": "reference", "metric": DECODE_METRIC, "value": tok_s, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": B / tok_s * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": {"workload": "decode step", **DECODE_SHAPE, "device": "host cpu"},
            "cpu_baseline": {"value": tok_s, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": tok_s, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}), flush=True)
        return 0
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, H, P, N, G = (DECODE_SHAPE[k] for k in ("B", "H", "P", "N", "G"))
    step_bytes = decode_bytes(B, H, P, N, G)
    # rotating state sets (each one decode batch's states), together more than twice the L2, so every
    # step reads its states from HBM
    state_bytes = B * H * P * N * 4
    n_sets = int(-(-2 * L2_BYTES // state_bytes)) + 1
    g = torch.Generator().manual_seed(3)
    states = [(0.1 * torch.randn(B, H, P, N, generator=g)).to(dev) for _ in range(n_sets)]
    toks = decode_tokens(B, H, P, N, G, n_sets, dev)

    def step(i):
        tk = toks[i]
        return zenith_b200.ssd_decode(*(tk[n] for n in NAMES), state=states[i])

    for i in range(n_sets):
        step(i)
    torch.cuda.synchronize()
    graphs, keep = [], []
    c0 = _lib.launch_count()
    for i in range(n_sets):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            keep.append(step(i))
        graphs.append(gr)
    per_step = (_lib.launch_count() - c0) // n_sets  # kernels captured per step
    for i in range(max(args.warmup, 3)):
        graphs[i % n_sets].replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(0)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        graphs[i % n_sets].replay()
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    launches = per_step * args.steps
    ms = e0.elapsed_time(e1) / args.steps
    # end to end through the public API: the token's inputs from pinned host memory, y back to the host
    host = [{n: t.cpu().pin_memory() for n, t in tk.items()} for tk in toks]
    y_host = torch.empty(B, 1, H, P, dtype=torch.bfloat16).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host[0].values())
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(args.steps):
        tk = {n: t.to(dev, non_blocking=True) for n, t in host[i % n_sets].items()}
        y = zenith_b200.ssd_decode(*(tk[n] for n in NAMES), state=states[i % n_sets])
        y_host.copy_(y, non_blocking=True)
    torch.cuda.synchronize()
    e2e_ms = (time.perf_counter() - t0) * 1e3 / args.steps
    zenith_b200.check_status(dev)
    cpu = None
    if not args.no_cpu_baseline:
        tok_s, cores, sample = cpu_decode_sample(min(args.cpu_seconds, 10.0))
        cpu = {"value": tok_s, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}
    peak, peak_kind = peaks()
    gbs = step_bytes / (ms / 1e3) / 1e9
    print(json.dumps({
        "metric": DECODE_METRIC, "value": B / (ms / 1e3), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"decode step B{B} H{H} P{P} N{N} G{G} (one token per sequence, fp32 states in place)",
                   "timed_launch": "CUDA graph of one step, replayed",
                   "l2": f"{n_sets} rotating state sets of {state_bytes / 1e6:.1f} MB, more than twice the L2"},
        "roofline": {"bound": "hbm", "kernel": "ssd_decode", "achieved": gbs, "peak": peak, "unit": "GB/s",
                     "frac": gbs / peak, "peak_kind": peak_kind, "traffic": None,
                     "algorithmic_bytes_per_launch": step_bytes},
        "cpu_baseline": cpu,
        "e2e": {"value": B / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": y_host.numel() * y_host.element_size()},
        "gpu_launches": launches,
        "clocks": clocks,
    }), flush=True)
    return 0


# ------------------------------------------------------------------------------------------------
# --workload lm: one data-parallel training step of the Mamba-3 LM (zenith/model.py:42-99,
# zenith/train.py:99-111): d_model 1536, expand 2, headdim 64 (48 heads), N 128, 24 layers
# (4 input, 16 recurrent, 4 output, one loop), vocab 32000 tied, micro-batch 8 x 2048 per GPU.

LM_METRIC = "Mamba-3 LM training step tokens/s"
LM_CONFIG = dict(vocab_size=32000, d_model=1536, d_state=128, expand=2, headdim=64, chunk_size=64, n_input=4,
                 n_recurrent=16, n_output=4, max_loops=1, tie_word_embeddings=True)
LM_BATCH, LM_SEQ = 8, 2048


def lm_flops_per_token(cfg):
    """Algorithmic FLOPs per token of one training step (forward + backward = 3x forward): the
    in_proj / out_proj / LM-head GEMMs (2 flops per weight per token, forward) and the SSD scan
    (fwd F = 4 L N + 4 L P + 6 N P per head, chunk L)."""
    d, V = cfg["d_model"], cfg["vocab_size"]
    d_inner = cfg["expand"] * d
    H, P, N, Lc = d_inner // cfg["headdim"], cfg["headdim"], cfg["d_state"], cfg["chunk_size"]
    n_in = 2 * d_inner + 2 * N + 3 * H + N // 4
    layers = cfg["n_input"] + cfg["n_recurrent"] * cfg["max_loops"] + cfg["n_output"]
    gemm = 2 * (d * n_in + d_inner * d) * layers + 2 * d * V
    scan = (4 * Lc * N + 4 * Lc * P + 6 * N * P) * H * layers
    return 3 * (gemm + scan)


def cpu_lm_sample(cfg, seconds: float, T: int = 128):
    """The reference LM's forward + backward (float32, autograd) on the host CPU for one sequence of
    T tokens: the reference's own ``ZenithForCausalLM`` when installed under baseline/_ref, else the
    oracle restatement of zenith/model.py:79-99.  The optimiser step (one per 16,384 tokens on the
    GPU) is left out of the sample.  Returns (tokens/s, cores, sample string, kind)."""
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    torch.manual_seed(0)
    ids = torch.randint(0, cfg["vocab_size"], (1, T))
    ref, why = reference_package()
    if ref is not None:
        model = ref.ZenithForCausalLM(ref.ZenithConfig(**cfg))
        model.train()
        kind, origin = "reference", "reference ZenithForCausalLM (installed under baseline/_ref)"

        def once():
            model(ids, labels=ids, loops=cfg["max_loops"]).loss.backward()
            model.zero_grad(set_to_none=True)
    else:
        from oracle import lm_oracle

        with torch.device("cpu"):
            from zenith_b200.lm import ZenithForCausalLM

            model = ZenithForCausalLM(cfg)          # initialisation only; the step below is the oracle's
        params = {n: t.detach().clone().requires_grad_(True) for n, t in model.named_parameters()}
        kind, origin = "port", f"reference LM (zenith/model.py:79-99) restated [{why}]"

        def once():
            _, loss = lm_oracle.forward(params, cfg, ids, ids, loops=cfg["max_loops"])
            loss.backward()
            for t in params.values():
                t.grad = None

    once()
    reps, t0 = 0, time.perf_counter()
    while True:
        once()
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    tok_s = reps * T / el
    sample = (f"{origin}: float32 forward + autograd backward on host CPU, 1 sequence of {T} tokens of the full "
              f"model (no optimiser step), {reps} reps in {el:.1f} s, {cores} threads")
    return tok_s, cores, sample, kind


def run_lm_reference(args):
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    seconds = max(5.0, min(120.0, 2.0 * (args.steps + args.warmup)))
    tok_s, cores, sample, kind = cpu_lm_sample(LM_CONFIG, seconds)
    line = {
        "impl": "reference", "metric": LM_METRIC, "value": tok_s, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": LM_BATCH * LM_SEQ / tok_s * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": "Mamba-3 LM training step", **LM_CONFIG, "micro_batch": LM_BATCH, "seq_len": LM_SEQ,
                   "device": "host cpu"},
        "cpu_baseline": {"value": tok_s, "unit": UNIT, "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": tok_s, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_lm(args):
    import torch.distributed as dist

    import zenith_b200
    from zenith_b200 import _lib, lm

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    torch.manual_seed(0)                                  # identical replicas
    model = lm.ZenithForCausalLM(LM_CONFIG).to(dev)
    net = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local], bucket_cap_mb=100,
                                                    gradient_as_bucket_view=True) if world > 1 else model
    opt = lm.make_optimizer(model)
    g = torch.Generator().manual_seed(1000 + rank)        # every rank its own micro-batch
    n_batches = 4
    host_ids = [torch.randint(0, LM_CONFIG["vocab_size"], (LM_BATCH, LM_SEQ), generator=g).pin_memory()
                for _ in range(n_batches)]
    dev_ids = [t.to(dev) for t in host_ids]

    def barrier():
        if world > 1:
            dist.barrier()

    for i in range(max(args.warmup, 3)):
        lm.train_step(net, opt, dev_ids[i % n_batches], loops=1)
    torch.cuda.synchronize()
    zenith_b200.check_status(dev)

    sampler = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    launches0 = _lib.launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(args.steps):
        lm.train_step(net, opt, dev_ids[i % n_batches], loops=1)
    end.record()
    torch.cuda.synchronize()
    launches = _lib.launch_count() - launches0
    barrier()
    clocks = sampler.stop()
    zenith_b200.check_status(dev)
    t = torch.tensor([start.elapsed_time(end)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item()) / args.steps
    tokens = LM_BATCH * LM_SEQ * world
    value = tokens / (ms / 1e3)

    # end to end: token ids from pinned host memory every step, the loss read back every step
    e2e_steps = max(3, args.steps)
    ids_buf = torch.empty(LM_BATCH, LM_SEQ, dtype=torch.int64, device=dev)
    barrier()
    torch.cuda.synchronize()
    start.record()
    for i in range(e2e_steps):
        ids_buf.copy_(host_ids[i % n_batches], non_blocking=True)
        loss = lm.train_step(net, opt, ids_buf, loops=1)
        loss.item()
    end.record()
    torch.cuda.synchronize()
    t = torch.tensor([start.elapsed_time(end)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item()) / e2e_steps
    zenith_b200.check_status(dev)

    line = None
    if rank == 0:
        flops = lm_flops_per_token(LM_CONFIG) * LM_BATCH * LM_SEQ
        pk = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
        peak, kind = (float(pk["bf16_tflops_sustained"]), "measured sustained") if pk else (1400.0, "fallback")
        achieved = flops / (ms / 1e3) / 1e12
        cpu = None
        if not args.no_cpu_baseline:
            tok_s, cores, sample, kind = cpu_lm_sample(LM_CONFIG, args.cpu_seconds)
            cpu = {"value": tok_s, "unit": UNIT, "cores": cores, "kind": kind, "sample": sample}
        line = {
            "metric": LM_METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "Mamba-3 LM training step (AdamW, grad clip, DDP all-reduce over NCCL)",
                       **LM_CONFIG, "micro_batch": LM_BATCH, "seq_len": LM_SEQ, "global_batch": LM_BATCH * world,
                       "parallelism": f"dp{world}", "params": sum(p.numel() for p in model.parameters()),
                       "l2": "activations far larger than L2"},
            "roofline": {"bound": "tensor", "kernel": "training step (GEMMs + SSD scan), model FLOPs",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                         "peak_kind": kind, "traffic": None, "flops_per_step": flops},
            "cpu_baseline": cpu,
            "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": LM_BATCH * LM_SEQ * 8,
                    "d2h_bytes_per_step": 4},
            "gpu_launches": launches,
            "clocks": clocks,
        }
    if world > 1:
        del net
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    if args.workload == "lm":
        return run_lm_reference(args) if args.impl == "reference" else run_lm(args)
    if args.workload == "decode":
        return run_decode(args)
    if args.workload == "mamba3":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "metric": LAYER_METRIC,
                              "unavailable": "the layer-body workload has no separate reference arm; the scan "
                                             "workloads time the reference algorithm"}), flush=True)
            return 0
        return run_layer(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
