"""Context parallelism for long sequences: each rank owns a contiguous range of the sequence.

The reference runs one sequence on one device (zenith/mamba3.py:30-56).  Because the SSD state
recurrence is linear, S_out = D S_in + F with D = exp(sum adt) over a range and F that range's final
state from a zero start, a sequence split over ranks needs only the boundary states:

forward
  1. every rank: F_r = final state of its range from zero (rank 0: from the initial state),
     D_r = exp(sum_t adt) per (b, h)  (state-only pass: reads x, xp, k, kp and the scalars)
  2. one all_gather of every rank's [D_r | F_r] (fp32, [B, H] + [B, H, P, N]); each rank forms its
     own entering state locally, S_0 = 0, S_{i+1} = D_i S_i + F_i for i < r
  3. every rank: the full local scan with initial_state = S_r (saving chunk states)
backward
  1. every rank: G_r = gradient w.r.t. its initial state from its own dy alone (state-only pass)
  2. one all_gather of [D_r | G_r]; each rank forms E_r, the gradient w.r.t. the state leaving it:
     E_{R-1} = 0, E_{i-1} = D_i E_i + G_i for i > r
  3. every rank: the full local backward with dfinal = E_r; rank 0's initial-state gradient is the
     one that backward returns.
One collective per direction, so the exchange costs one all_gather latency at any rank count
instead of R - 1 dependent send / recv hops.

Ranks hold data in the caller's layout ([B, T_local, H, ...]).  The exchange is collective: every
rank of the group must call with equally shaped local ranges (checked first, by one small all_gather:
a mismatch raises ValueError on every rank).
"""

from __future__ import annotations

import datetime
from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import _lib as L
from .ssd import _stream, prepare_inputs, ssd_bwd_op, ssd_fwd_op

NAMES = ("x", "q", "k", "kp", "xp", "adt", "gamma", "beta")


# ------------------------------------------------------------------------------------------------
# local scan implementation (injectable: the default is the CUDA library)


@dataclass
class LocalScan:
    """The per-rank operations context parallelism needs."""

    final_state: Callable    # (inputs, chunk, init) -> F [B,H,P,N]
    forward: Callable        # (inputs, chunk, init) -> (y, saved)
    dinitial: Callable       # (dy, inputs, chunk) -> G [B,H,P,N]   (dfinal = 0)
    backward: Callable       # (dy, inputs, saved, chunk, init, dfinal) -> 8 grads + d(initial state)
    total_decay: Callable    # (adt) -> D [B,H] fp32
    combine: Callable        # (s_prev, d, f) -> d * s_prev + f


def _cuda_final_state(inp, chunk, init):
    return ssd_fwd_op(*inp, int(chunk), init, False, True)[1]


def _cuda_forward(inp, chunk, init):
    y, fin, states = ssd_fwd_op(*inp, int(chunk), init, True, False)
    return y, (states, fin)


def _cuda_dinitial(dy, inp, chunk):
    empty = torch.empty(0, dtype=torch.uint8, device=dy.device)
    out = ssd_bwd_op(dy, *inp, empty, int(chunk), None, None, True)
    return out[-1]


def _cuda_backward(dy, inp, saved, chunk, init, dfinal):
    states, _ = saved
    out = ssd_bwd_op(dy, *inp, states, int(chunk), init, dfinal, False)
    return out[:9]


def _cuda_total_decay(adt):
    B, T, H = adt.shape
    out = torch.empty(B * H, dtype=torch.float32, device=adt.device)
    a = L.Args()
    a.B, a.T, a.H = B, T, H
    a.scalar_dtype = L.DTYPE_CODE[adt.dtype]
    a.adt = L.view(adt)
    with L.device_guard(adt.device):
        L.check(L.lib().zb_ssd_total_decay(ctypes_byref(a), out.data_ptr(), _stream(adt.device)), "zb_ssd_total_decay")
    return out.view(B, H)


def _cuda_combine(s_prev, d, f):
    s_prev, d, f = (t.contiguous() for t in (s_prev, d, f))  # read as flat arrays
    out = torch.empty_like(f)
    BH = d.numel()
    with L.device_guard(f.device):
        L.check(L.lib().zb_ssd_state_combine(s_prev.data_ptr(), d.data_ptr(), f.data_ptr(), out.data_ptr(), BH,
                                             f.numel() // BH, _stream(f.device)), "zb_ssd_state_combine")
    return out


def ctypes_byref(a):
    import ctypes

    return ctypes.byref(a)


CUDA_SCAN = LocalScan(_cuda_final_state, _cuda_forward, _cuda_dinitial, _cuda_backward, _cuda_total_decay, _cuda_combine)


# ------------------------------------------------------------------------------------------------
# the exchange


def _gather(X, D, group):
    """Every rank's (X_r, D_r), in rank order: one all_gather of [D_r | X_r] packed in X's dtype."""
    world = dist.get_world_size(group)
    packed = torch.cat([D.reshape(-1).to(X.dtype), X.reshape(-1)]).contiguous()
    parts = [torch.empty_like(packed) for _ in range(world)]
    dist.all_gather(parts, packed, group=group)
    nd = D.numel()
    return [(p[nd:].view_as(X), p[:nd].view(D.shape).to(D.dtype).contiguous()) for p in parts]


def _entering_state(F, D, group, impl: LocalScan):
    """S_r, the state entering this rank's range: S_0 = 0, S_{i+1} = D_i S_i + F_i (rank 0's F
    already starts from the initial state)."""
    rank = dist.get_rank(group)
    S = torch.zeros_like(F)
    for Fi, Di in _gather(F, D, group)[:rank]:
        S = impl.combine(S, Di, Fi)
    return S


def _leaving_gradient(G, D, group, impl: LocalScan):
    """E_r, the gradient w.r.t. the state leaving this rank's range: E_{R-1} = 0,
    E_{i-1} = D_i E_i + G_i."""
    rank = dist.get_rank(group)
    E = torch.zeros_like(G)
    for Gi, Di in reversed(_gather(G, D, group)[rank + 1:]):
        E = impl.combine(E, Di, Gi)
    return E


def _check_local_shapes(x, q, group):
    """Every rank must pass an equally shaped local range: the exchanged state is [B, H, P, N], and
    an all_gather of different sizes is undefined under NCCL.  One all_gather of each rank's
    (B, T_local, H, P, N, G) makes a mismatch raise the same ValueError on every rank."""
    sig = torch.tensor([x.shape[0], x.shape[1], x.shape[2], x.shape[3], q.shape[3], q.shape[2]], dtype=torch.int64,
                       device=x.device)
    parts = [torch.empty_like(sig) for _ in range(dist.get_world_size(group))]
    dist.all_gather(parts, sig, group=group)
    sigs = [tuple(t.tolist()) for t in parts]
    if any(t != sigs[0] for t in sigs):
        raise ValueError("cp_ssd: the ranks' local ranges differ in shape (B, T_local, H, P, N, G by rank): "
                         + str(sigs))


class _CpScan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, chunk, group, impl, init, x, q, k, kp, xp, adt, gamma, beta):
        inp = (x, q, k, kp, xp, adt, gamma, beta)
        rank = dist.get_rank(group)
        if rank != 0:
            init = None  # only the first range starts from the caller's initial state
        F = impl.final_state(inp, chunk, init)
        D = impl.total_decay(adt)
        S = _entering_state(F, D, group, impl)  # every rank takes part in the all_gather
        if init is not None:
            S = init.to(F.dtype).contiguous()
        y, saved = impl.forward(inp, chunk, S)
        ctx.chunk, ctx.group, ctx.impl = chunk, group, impl
        ctx.saved = saved
        ctx.has_init = init is not None
        ctx.save_for_backward(S, D, *inp)
        return y

    @staticmethod
    def backward(ctx, dy):
        S, D, *inp = ctx.saved_tensors
        dy = dy.to(inp[0].dtype).contiguous()
        G = ctx.impl.dinitial(dy, tuple(inp), ctx.chunk)
        E = _leaving_gradient(G, D, ctx.group, ctx.impl)
        out = ctx.impl.backward(dy, tuple(inp), ctx.saved, ctx.chunk, S, E)
        grads, dinit = out[:8], out[8]
        return (None, None, None, dinit if ctx.has_init else None, *grads)


def cp_ssd(x, q, k, kp, xp, adt, gamma, beta, chunk_size, *, group=None, initial_state=None,
           impl: Optional[LocalScan] = None, check_shapes: bool = True):
    """Context-parallel SSD scan over the ranks of ``group`` (default: the world).

    Each rank passes its contiguous range of the sequence ([B, T_local, H, ...], rank r holding
    tokens [r T_local, (r+1) T_local)); returns this rank's y.  Same arithmetic as
    ``zenith_b200.ssd`` on the whole sequence, differentiable w.r.t. all eight inputs.
    ``initial_state`` [B, H, P, N] (read on rank 0 only; the other ranks ignore theirs) starts the
    sequence from a given state and is differentiable on rank 0.
    ``check_shapes=False`` skips the first all_gather of every rank's local shape, which reads the
    result back on the host: for calls captured in a CUDA graph, after a checked call with the same
    shapes on every rank.
    """
    assert x.shape[1] % chunk_size == 0, "sequence length must be a multiple of chunk_size"
    if check_shapes:
        _check_local_shapes(x, q, group)
    impl = impl or CUDA_SCAN
    if impl is CUDA_SCAN:
        args = prepare_inputs(x, q, k, kp, xp, adt, gamma, beta)
    else:
        args = (x, q, k, kp, xp, adt, gamma, beta)
    y = _CpScan.apply(int(chunk_size), group, impl, initial_state, *args)
    return y.to(x.dtype) if y.dtype != x.dtype else y


class CpGraphedStep:
    """One context-parallel forward + backward over fixed tensors, with the local work replayed from
    CUDA graphs and the two exchanges issued eagerly between them (the collectives stay outside the
    graphs): per call, the host launches four graph replays and two all_gathers instead of the eager
    step's few dozen kernels and Python steps.

    Construct it on every rank of ``group`` with this rank's local range ([B, T_local, H, ...], as
    ``cp_ssd``) and the gradient of its output ``dy``; the construction is collective (one shape
    check, one eager warm-up step).  Each call reads the input tensors given here and returns
    ``(y, grads)``: this rank's output and the gradients of the eight inputs, tensors that the next
    call overwrites.  Inputs already in the kernels' dtypes (one vector dtype, fp32 scalars) with a
    contiguous innermost dimension are read in place, so updating them between calls updates the
    step; others are converted once, here.  No initial state."""

    def __init__(self, x, q, k, kp, xp, adt, gamma, beta, dy, chunk_size, *, group=None,
                 impl: Optional[LocalScan] = None):
        assert x.shape[1] % chunk_size == 0, "sequence length must be a multiple of chunk_size"
        _check_local_shapes(x, q, group)
        self.impl = impl or CUDA_SCAN
        self.group, self.chunk = group, int(chunk_size)
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.inp = tuple(prepare_inputs(x, q, k, kp, xp, adt, gamma, beta)) if self.impl is CUDA_SCAN else \
            (x, q, k, kp, xp, adt, gamma, beta)
        self.dy = dy.to(self.inp[0].dtype).contiguous()
        # one eager step first: every lazy initialisation happens outside the graphs
        self._pre_forward()
        self.recv1 = torch.empty(self.world, self.send1.numel(), dtype=self.send1.dtype, device=self.send1.device)
        dist.all_gather_into_tensor(self.recv1, self.send1, group=group)
        self._main_forward()
        self._pre_backward()
        self.recv2 = torch.empty_like(self.recv1)
        dist.all_gather_into_tensor(self.recv2, self.send2, group=group)
        self._main_backward()
        torch.cuda.synchronize()
        self.graphs = []
        pool = None
        for piece in (self._pre_forward, self._main_forward, self._pre_backward, self._main_backward):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=pool):
                piece()
            pool = g.pool()
            self.graphs.append(g)
        torch.cuda.synchronize()

    # the four pieces (captured once; their outputs are attributes, at fixed addresses)
    def _pre_forward(self):
        self.F = self.impl.final_state(self.inp, self.chunk, None)
        self.D = self.impl.total_decay(self.inp[5])
        self.send1 = torch.cat([self.D.reshape(-1).to(self.F.dtype), self.F.reshape(-1)])

    def _parts(self, recv):
        nd = self.D.numel()
        return [(recv[i, nd:].view_as(self.F), recv[i, :nd].view(self.D.shape).to(self.D.dtype))
                for i in range(self.world)]

    def _main_forward(self):
        S = torch.zeros_like(self.F)
        for Fi, Di in self._parts(self.recv1)[:self.rank]:
            S = self.impl.combine(S, Di, Fi)
        self.S = S
        self.y, self.saved = self.impl.forward(self.inp, self.chunk, S)

    def _pre_backward(self):
        self.G = self.impl.dinitial(self.dy, self.inp, self.chunk)
        self.send2 = torch.cat([self.D.reshape(-1).to(self.G.dtype), self.G.reshape(-1)])

    def _main_backward(self):
        E = torch.zeros_like(self.G)
        for Gi, Di in reversed(self._parts(self.recv2)[self.rank + 1:]):
            E = self.impl.combine(E, Di, Gi)
        self.grads = self.impl.backward(self.dy, self.inp, self.saved, self.chunk, self.S, E)[:8]

    def __call__(self, events=None):
        """One step; ``events`` (three CUDA events, optional) are recorded before it, after the
        forward and after the backward."""
        g1, g2, g3, g4 = self.graphs
        if events is not None:
            events[0].record()
        g1.replay()
        dist.all_gather_into_tensor(self.recv1, self.send1, group=self.group)
        g2.replay()
        if events is not None:
            events[1].record()
        g3.replay()
        dist.all_gather_into_tensor(self.recv2, self.send2, group=self.group)
        g4.replay()
        if events is not None:
            events[2].record()
        return self.y, self.grads


def init_process_group_from_env(backend: str, timeout_s: float = 120.0, device_id=None):
    """Initialise torch.distributed from RANK / WORLD_SIZE / MASTER_ADDR / MASTER_PORT with a
    short timeout, so that ranks waiting for a failed peer end with an error instead of hanging."""
    kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device_id is not None:
        kw["device_id"] = device_id
    dist.init_process_group(backend, **kw)
