"""Drop-in SSD chunked scan: ``ssd(x, q, k, kp, xp, adt, gamma, beta, chunk_size)``.

Same signature, layouts, return value and error behaviour as the reference's
``zenith.mamba3.ssd`` (zenith/mamba3.py:30-56), which ``Mamba3.forward`` calls through its
``scan`` attribute as ``self.scan(x, q, k, kp, xp, ADT, gamma, beta, self.chunk_size)``
(zenith/mamba3.py:77,118).  Forward and backward run in libzenith_ssd.so (sm_100a CUDA
kernels) behind two ``torch.library`` custom ops with a registered autograd formula and fake
(meta) implementations, so the op also works under ``torch.compile`` (the reference's
``--compile_scan``, zenith/train.py:75-79).

Extensions with no reference counterpart (the reference always starts from a zero state and
drops the final state, zenith/mamba3.py:50-54):
``initial_state=[B,H,P,N]`` and ``return_final_state=True`` (both differentiable).

Precision: fp32/fp64 inputs are computed in fp32/fp64.  bf16/fp16 inputs are read as stored,
multiplied with fp32 accumulation; scans, decays and states stay fp32.  Under CUDA autocast
with a 16-bit dtype, fp32 vector inputs are cast to that dtype first, as the reference's
matmuls are under autocast; y is returned in the caller's dtype.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch
from torch import Tensor

from . import _lib as L

_VEC = ("x", "q", "k", "kp", "xp")
_SCA = ("adt", "gamma", "beta")


def _acc_dtype(vdt: torch.dtype) -> torch.dtype:
    return torch.float64 if vdt == torch.float64 else torch.float32


# Stand-in data address for sizing calls made without data (fake tensors under torch.compile):
# 4 KiB aligned, like every allocation.  The kernel family, and with it the saved-state size, depends
# on the inputs' alignment; the real ops re-align a misaligned input (_realign) so that they always
# agree with a sizing call.
_SIZING_ADDR = 1 << 12


def _build_args(x, q, k, kp, xp, adt, gamma, beta, chunk_size, flags=0, sizing_only=False) -> L.Args:
    B, T, H, P = x.shape
    G, N = q.shape[2], q.shape[3]
    a = L.Args()
    a.B, a.T, a.H, a.G, a.P, a.N, a.chunk_size = B, T, H, G, P, N, chunk_size
    a.dtype = L.DTYPE_CODE[x.dtype]
    a.scalar_dtype = L.DTYPE_CODE[adt.dtype]
    a.flags = flags
    for n, t in zip(_VEC + _SCA, (x, q, k, kp, xp, adt, gamma, beta)):
        setattr(a, n, L.view(t, _SIZING_ADDR if sizing_only else None))
    return a


def _realign(t: Tensor) -> Tensor:
    """``t`` itself, or a copy with the same strides at a 16-byte aligned address when its data
    address is not (a view at an odd element offset): see _SIZING_ADDR."""
    if t.data_ptr() % 16 == 0:
        return t
    return torch.empty_strided(t.size(), t.stride(), dtype=t.dtype, device=t.device).copy_(t)


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def kernel_family(x, q, k, kp, xp, adt, gamma, beta, chunk_size, *, states_saved=True) -> str:
    """'tensor-core' or 'simt': which kernels the library runs for these (prepared) inputs."""
    a = _build_args(x, q, k, kp, xp, adt, gamma, beta, chunk_size)
    a.y = L.view(x)  # an output with the input's layout (only its alignment matters here)
    fam = L.lib().zb_ssd_kernel_family(ctypes.byref(a), 1 if states_saved else 0)
    return {1: "tensor-core", 0: "simt"}.get(fam, "invalid")


def states_nbytes(x, q, k, kp, xp, adt, gamma, beta, chunk_size) -> int:
    """Bytes of the saved chunk states, from shapes, strides and dtypes only (no data access)."""
    a = _build_args(x, q, k, kp, xp, adt, gamma, beta, chunk_size, sizing_only=True)
    return int(L.lib().zb_ssd_states_bytes(ctypes.byref(a)))


# ------------------------------------------------------------------------------------------------
# custom ops


@torch.library.custom_op("zenith_b200::ssd_fwd", mutates_args=(), device_types="cuda")
def ssd_fwd_op(x: Tensor, q: Tensor, k: Tensor, kp: Tensor, xp: Tensor, adt: Tensor, gamma: Tensor, beta: Tensor,
               chunk_size: int, initial_state: Optional[Tensor], save_states: bool,
               state_only: bool) -> tuple[Tensor, Tensor, Tensor]:
    with L.device_guard(x.device):
        return _ssd_fwd_impl(x, q, k, kp, xp, adt, gamma, beta, chunk_size, initial_state, save_states, state_only)


def _ssd_fwd_impl(x, q, k, kp, xp, adt, gamma, beta, chunk_size, initial_state, save_states, state_only):
    B, T, H, P = x.shape
    N = q.shape[3]
    dev = x.device
    x, q, k, kp, xp = (_realign(t) for t in (x, q, k, kp, xp))
    a = _build_args(x, q, k, kp, xp, adt, gamma, beta, chunk_size, L.ZB_FLAG_STATE_ONLY if state_only else 0)
    lib = L.lib()
    y = torch.empty((0,) if state_only else (B, T, H, P), dtype=x.dtype, device=dev)
    final = torch.empty((B, H, P, N), dtype=_acc_dtype(x.dtype), device=dev)
    states = torch.empty(lib.zb_ssd_states_bytes(ctypes.byref(a)) if save_states else 0, dtype=torch.uint8, device=dev)
    ws_bytes = lib.zb_ssd_workspace_bytes(ctypes.byref(a), 0)
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=dev)
    if not state_only:
        a.y = L.view(y)
    a.initial_state = L.ptr(initial_state)
    a.final_state = final.data_ptr()
    a.states = L.ptr(states)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    a.status = L.status_word(dev).data_ptr()
    L.check(lib.zb_ssd_fwd(ctypes.byref(a), _stream(dev)), "zb_ssd_fwd")
    return y, final, states


@ssd_fwd_op.register_fake
def _(x, q, k, kp, xp, adt, gamma, beta, chunk_size, initial_state, save_states, state_only):
    B, T, H, P = x.shape
    N = q.shape[3]
    nbytes = states_nbytes(x, q, k, kp, xp, adt, gamma, beta, chunk_size) if save_states else 0
    y = x.new_empty((0,) if state_only else (B, T, H, P))
    return y, x.new_empty((B, H, P, N), dtype=_acc_dtype(x.dtype)), x.new_empty((nbytes,), dtype=torch.uint8)


@torch.library.custom_op("zenith_b200::ssd_bwd", mutates_args=(), device_types="cuda")
def ssd_bwd_op(dy: Tensor, x: Tensor, q: Tensor, k: Tensor, kp: Tensor, xp: Tensor, adt: Tensor, gamma: Tensor,
               beta: Tensor, states: Tensor, chunk_size: int, initial_state: Optional[Tensor],
               dfinal: Optional[Tensor], state_only: bool) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    with L.device_guard(x.device):
        return _ssd_bwd_impl(dy, x, q, k, kp, xp, adt, gamma, beta, states, chunk_size, initial_state, dfinal, state_only)


def _ssd_bwd_impl(dy, x, q, k, kp, xp, adt, gamma, beta, states, chunk_size, initial_state, dfinal, state_only):
    B, T, H, P = x.shape
    dev = x.device
    lib = L.lib()
    dy, x, q, k, kp, xp = (_realign(t) for t in (dy, x, q, k, kp, xp))
    a = _build_args(x, q, k, kp, xp, adt, gamma, beta, chunk_size, L.ZB_FLAG_STATE_ONLY if state_only else 0)
    if state_only:
        grads = [torch.empty(0, dtype=t.dtype, device=dev) for t in (x, q, k, kp, xp, adt, gamma, beta)]
    else:
        grads = [torch.empty(t.shape, dtype=t.dtype, device=dev) for t in (x, q, k, kp, xp, adt, gamma, beta)]
        for n, g in zip(L._VIEWS_BWD, grads):
            setattr(a, n, L.view(g))
    dinit = torch.empty((B, H, P, q.shape[3]), dtype=_acc_dtype(x.dtype), device=dev)
    ws_bytes = lib.zb_ssd_workspace_bytes(ctypes.byref(a), 1)
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=dev)
    a.dy = L.view(dy)
    a.initial_state = L.ptr(initial_state)
    a.dfinal_state = L.ptr(dfinal)
    a.states = L.ptr(states)
    a.dinitial_state = dinit.data_ptr()
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    a.status = L.status_word(dev).data_ptr()
    L.check(lib.zb_ssd_bwd(ctypes.byref(a), _stream(dev)), "zb_ssd_bwd")
    # order of grads: x, q, k, kp, xp, adt, gamma, beta
    return (*grads, dinit)


@ssd_bwd_op.register_fake
def _(dy, x, q, k, kp, xp, adt, gamma, beta, states, chunk_size, initial_state, dfinal, state_only):
    B, T, H, P = x.shape
    if state_only:
        grads = [t.new_empty((0,)) for t in (x, q, k, kp, xp, adt, gamma, beta)]
    else:
        grads = [torch.empty_like(t, memory_format=torch.contiguous_format) for t in (x, q, k, kp, xp, adt, gamma, beta)]
    return (*grads, x.new_empty((B, H, P, q.shape[3]), dtype=_acc_dtype(x.dtype)))


def _setup_context(ctx, inputs, output):
    x, q, k, kp, xp, adt, gamma, beta, chunk_size, initial_state, save_states, state_only = inputs
    _, _, states = output
    ctx.chunk_size = chunk_size
    ctx.has_init = initial_state is not None
    ctx.state_only = state_only
    # gradients of unused outputs (the final state, the saved-state bytes) arrive as None rather
    # than as zero-filled tensors; the backward treats None as zero
    ctx.set_materialize_grads(False)
    saved = [x, q, k, kp, xp, adt, gamma, beta, states]
    if initial_state is not None:
        saved.append(initial_state)
    ctx.save_for_backward(*saved)


def _backward(ctx, dy, dfinal, _dstates):
    saved = ctx.saved_tensors
    x, q, k, kp, xp, adt, gamma, beta, states = saved[:9]
    init = saved[9] if ctx.has_init else None
    if states.numel() == 0:
        raise RuntimeError("zenith_b200.ssd: backward needs the forward to save its chunk states")
    if ctx.state_only or dy is None or dy.numel() == 0:
        dy = torch.zeros(x.shape, dtype=x.dtype, device=x.device)
    dy = dy.to(x.dtype)
    if dy.stride(-1) != 1:
        dy = dy.contiguous()
    if dfinal is not None:
        dfinal = dfinal.to(_acc_dtype(x.dtype)).contiguous()
    out = ssd_bwd_op(dy, x, q, k, kp, xp, adt, gamma, beta, states, ctx.chunk_size, init, dfinal, False)
    L.poll_status(x)
    dx, dq, dk, dkp, dxp, dadt, dgamma, dbeta, dinit = out
    return dx, dq, dk, dkp, dxp, dadt, dgamma, dbeta, None, (dinit if ctx.has_init else None), None, None


torch.library.register_autograd("zenith_b200::ssd_fwd", _backward, setup_context=_setup_context)


# ------------------------------------------------------------------------------------------------
# public entry point


def _inner_contig(t: Tensor) -> Tensor:
    return t if t.stride(-1) == 1 or t.shape[-1] == 1 else t.contiguous()


def _check_scan_shapes(what, x, q, k, kp, xp, adt, gamma, beta):
    """x, xp [B, T, H, P]; q, k, kp [B, T, G, N]; adt, gamma, beta [B, T, H] (the reference's
    layouts, zenith/mamba3.py:30-39, with G = H or G dividing H)."""
    if x.dim() != 4 or q.dim() != 4:
        raise ValueError(f"{what}: x [B, T, H, P] and q [B, T, G, N] must be 4-D, got {tuple(x.shape)}, {tuple(q.shape)}")
    B, T, H, P = x.shape
    G, N = q.shape[2], q.shape[3]
    L.check_shapes(what, q=(q, (B, T, G, N)), k=(k, (B, T, G, N)), kp=(kp, (B, T, G, N)), xp=(xp, (B, T, H, P)),
                   adt=(adt, (B, T, H)), gamma=(gamma, (B, T, H)), beta=(beta, (B, T, H)))


def prepare_inputs(x, q, k, kp, xp, adt, gamma, beta):
    """Unify dtypes (one for the five vectors, one for the three per-token scalars) and make the
    innermost dimension contiguous.  Under CUDA autocast with a 16-bit dtype, fp32 vectors are
    cast to that dtype (the reference's matmuls run in it under autocast)."""
    L.check_same_device(x.device, "zenith_b200.ssd", q=q, k=k, kp=kp, xp=xp, adt=adt, gamma=gamma, beta=beta)
    _check_scan_shapes("zenith_b200.ssd", x, q, k, kp, xp, adt, gamma, beta)
    vec = [x, q, k, kp, xp]
    sca = [adt, gamma, beta]
    vdt = vec[0].dtype
    for t in vec[1:]:
        vdt = torch.promote_types(vdt, t.dtype)
    sdt = sca[0].dtype
    for t in sca[1:]:
        sdt = torch.promote_types(sdt, t.dtype)
    if x.is_cuda and torch.is_autocast_enabled("cuda") and vdt == torch.float32:
        vdt = torch.get_autocast_dtype("cuda")
    if vdt not in L.DTYPE_CODE:
        raise TypeError(f"zenith_b200.ssd: unsupported dtype {vdt}")
    if vdt == torch.float64:
        sdt = torch.float64
    elif sdt == torch.float64 or sdt not in L.DTYPE_CODE:
        sdt = torch.float32
    vec = [_inner_contig(t.to(vdt)) for t in vec]
    sca = [t.to(sdt) for t in sca]
    return (*vec, *sca)


def _empty_scan(x, q, k, kp, xp, adt, gamma, beta, initial_state, return_final_state):
    """An empty batch, head, feature or state dimension (T > 0): there is nothing to compute and no
    kernel runs.  y is all zeros, as the reference's matmuls over empty dimensions give (empty
    unless only N is 0), and every input gradient is zero; the final state is empty."""
    L.check_same_device(x.device, "zenith_b200.ssd", q=q, k=k, kp=kp, xp=xp, adt=adt, gamma=gamma, beta=beta,
                        initial_state=initial_state)
    _check_scan_shapes("zenith_b200.ssd", x, q, k, kp, xp, adt, gamma, beta)
    Bsz, T, H, P = x.shape
    N = q.shape[-1]
    y = torch.zeros((Bsz, T, H, P), dtype=x.dtype, device=x.device)
    final = torch.zeros((Bsz, H, P, N), dtype=_acc_dtype(x.dtype), device=x.device)
    leaves = [t for t in (x, q, k, kp, xp, adt, gamma, beta, initial_state) if t is not None and t.requires_grad]
    if torch.is_grad_enabled() and leaves:
        anchor = sum(t.sum() for t in leaves) * 0  # zero gradients of the inputs' shapes
        y = y + anchor.to(y.dtype)
        final = final + anchor.to(final.dtype)
    return (y, final) if return_final_state else y


def ssd(x, q, k, kp, xp, adt, gamma, beta, chunk_size, *, initial_state=None, return_final_state=False):
    """SSD chunked scan on the GPU; drop-in for ``zenith.mamba3.ssd`` (zenith/mamba3.py:30-56).

    x, xp: [B, T, H, P]; q, k, kp: [B, T, G, N] (G == H, or G dividing H with head h reading
    group h // (H // G)); adt, gamma, beta: [B, T, H].  Returns y [B, T, H, P] in x's dtype, or
    ``(y, final_state)`` with ``return_final_state=True`` (final_state [B, H, P, N] fp32, fp64
    for fp64 inputs).  Raises AssertionError("sequence length must be a multiple of
    chunk_size") like the reference.  A kernel error recorded on the device by an earlier call
    (a timed-out wait) raises ``SsdError`` here once it is visible, without a synchronisation.
    """
    Bsz, T, H, P = x.shape
    N = q.shape[-1]
    assert T % chunk_size == 0, "sequence length must be a multiple of chunk_size"
    if T > 0 and (x.numel() == 0 or q.numel() == 0):
        return _empty_scan(x, q, k, kp, xp, adt, gamma, beta, initial_state, return_final_state)
    if not x.is_cuda:
        raise RuntimeError("zenith_b200.ssd runs on CUDA tensors only (no CPU path)")
    out_dtype = x.dtype
    args = prepare_inputs(x, q, k, kp, xp, adt, gamma, beta)
    if initial_state is not None:
        L.check_same_device(x.device, "zenith_b200.ssd", initial_state=initial_state)
        if tuple(initial_state.shape) != (Bsz, H, P, N):
            raise ValueError(f"initial_state must be [B, H, P, N] = {(Bsz, H, P, N)}")
        initial_state = initial_state.to(_acc_dtype(args[0].dtype)).contiguous()
    need_grad = torch.is_grad_enabled() and any(
        t.requires_grad for t in (x, q, k, kp, xp, adt, gamma, beta, initial_state) if t is not None)
    y, final, _ = torch.ops.zenith_b200.ssd_fwd(*args, int(chunk_size), initial_state, need_grad, False)
    L.poll_status(x)
    if y.dtype != out_dtype:
        y = y.to(out_dtype)
    if return_final_state:
        return y, final
    return y


def ssd_final_state(x, q, k, kp, xp, adt, gamma, beta, chunk_size, *, initial_state=None):
    """Forward without outputs: only the final state [B, H, P, N] (not differentiable).
    Used by the context-parallel pre-pass."""
    args = prepare_inputs(x, q, k, kp, xp, adt, gamma, beta)
    with torch.no_grad():
        _, final, _ = torch.ops.zenith_b200.ssd_fwd(*args, int(chunk_size), initial_state, False, True)
    return final


def ssd_dinitial_state(dy, x, q, k, kp, xp, adt, gamma, beta, chunk_size, *, dfinal=None):
    """Backward state chain only: the gradient w.r.t. the initial state of a range given dy on
    its outputs (and dfinal on its final state); not differentiable.  Used by the
    context-parallel pre-pass of the backward."""
    args = prepare_inputs(x, q, k, kp, xp, adt, gamma, beta)
    with torch.no_grad():
        states = torch.empty(0, dtype=torch.uint8, device=x.device)
        dy = _inner_contig(dy.to(args[0].dtype))
        if dfinal is not None:
            dfinal = dfinal.to(_acc_dtype(args[0].dtype)).contiguous()
        out = torch.ops.zenith_b200.ssd_bwd(dy, *args, states, int(chunk_size), None, dfinal, True)
    return out[-1]


def ssd_decode(x, q, k, kp, xp, adt, gamma, beta, state: Tensor) -> Tensor:
    """Recurrent (decode) form: for each of the T tokens in order,
    ``h = e^{adt} h + gamma x k^T + beta xp kp^T``, ``y = h q`` (the reference test's per-token
    recurrence, tests/test_mamba3.py:10-21), starting from ``state`` and updating it in place.

    Shapes as ``ssd`` (x, xp ``[B,T,H,P]``, q, k, kp ``[B,T,G,N]``, scalars ``[B,T,H]``; T is
    typically 1); ``state`` is a contiguous fp32 ``[B,H,P,N]`` tensor, e.g. the final state of
    a chunked forward over the prompt (``ssd(..., return_final_state=True)``).  Returns y
    ``[B,T,H,P]`` in x's dtype.  Inference only (no autograd)."""
    B, T, H, P = x.shape
    N = q.shape[3]
    L.check_same_device(x.device, "ssd_decode", q=q, k=k, kp=kp, xp=xp, adt=adt, gamma=gamma, beta=beta, state=state)
    _check_scan_shapes("ssd_decode", x, q, k, kp, xp, adt, gamma, beta)
    if state.dtype != torch.float32 or tuple(state.shape) != (B, H, P, N) or not state.is_contiguous():
        raise ValueError("ssd_decode: state must be a contiguous float32 [B, H, P, N] tensor")
    L.require_cuda(x.device, "ssd_decode")
    if any(t.dtype != x.dtype for t in (q, k, kp, xp)):
        raise ValueError("ssd_decode: x, q, k, kp and xp must share one dtype, got "
                         + ", ".join(str(t.dtype) for t in (x, q, k, kp, xp)))
    dev = x.device
    scal = [t if t.dtype == torch.float32 else t.float() for t in (adt, gamma, beta)]
    vec = [t if t.stride(-1) == 1 else t.contiguous() for t in (x, q, k, kp, xp)]
    a = _build_args(*vec, *scal, 1)
    y = torch.empty(B, T, H, P, dtype=x.dtype, device=dev)
    a.y = L.view(y)
    a.initial_state = state.data_ptr()
    a.final_state = state.data_ptr()
    with L.device_guard(dev):
        L.check(L.lib().zb_ssd_decode(ctypes.byref(a), _stream(dev)), "zb_ssd_decode")
    return y


def use_b200_scan(model: torch.nn.Module) -> int:
    """Install :func:`ssd` as the scan of every Mamba-3 block (``module.scan``, the reference's
    injection point, zenith/mamba3.py:77).  Returns the number of blocks patched."""
    n = 0
    for m in model.modules():
        if type(m).__name__ == "Mamba3" and hasattr(m, "scan"):
            m.scan = ssd
            n += 1
    return n
