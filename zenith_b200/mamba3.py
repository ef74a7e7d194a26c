"""Fused Mamba-3 layer body on B200: ``mamba3_ssd_fused(...)``.

Replaces the part of the reference's ``Mamba3.forward`` between the ``in_proj`` split and
``out_proj`` (zenith/mamba3.py:96-119): the discretisation (A from ``heavy_tail``, softplus DT,
trapezoid gamma / beta), theta = cumsum(DT * ang), RMSNorm + bias + RoPE of the B / C
projections, the one-token shift of x and k, the SSD scan, and ``(y + D x) * silu(z)``.  The
prologue and epilogue run as CUDA kernels of libzenith_ssd.so (``include/zb_mamba3.h``), the
scan as the library's SSD kernels; gradients reach every input and parameter (dt_bias,
B_bias, C_bias, the two RMSNorm weights, D).

``use_b200_layer(module)`` makes a reference-style ``Mamba3`` module (same attribute names)
run its forward through this op.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch
from torch import Tensor

from . import _lib as L
from .ssd import _build_args


class M3Args(ctypes.Structure):
    """ctypes mirror of ``zb_m3_args`` (include/zb_mamba3.h)."""

    _fields_ = (
        [(n, ctypes.c_int64) for n in ("B", "T", "H", "P", "N")]
        + [("A_floor", ctypes.c_float), ("eps", ctypes.c_float), ("io_dtype", ctypes.c_int32), ("op_dtype", ctypes.c_int32)]
        + [(n, L.View) for n in ("x", "z", "Bm", "Cm", "dd_dt", "dd_A", "trap", "ang")]
        + [(n, ctypes.c_void_p) for n in ("dt_bias", "B_bias", "C_bias", "B_norm_w", "C_norm_w", "D")]
        + [(n, ctypes.c_void_p) for n in ("q", "k_ext", "xp", "adt", "gamma", "beta", "theta", "y")]
        + [("out", L.View), ("dout", L.View), ("dy", ctypes.c_void_p)]
        + [(n, ctypes.c_void_p) for n in ("dxs", "dxp", "dq", "dk", "dkp", "dadt", "dgamma", "dbeta")]
        + [(n, L.View) for n in ("dx", "dz", "dBm", "dCm", "ddd_dt", "ddd_A", "dtrap", "dang")]
        + [(n, ctypes.c_void_p) for n in ("ddt_bias", "dB_bias", "dC_bias", "dB_norm_w", "dC_norm_w", "dD")]
        + [("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_uint64), ("status", ctypes.c_void_p)]
        + [("theta0", ctypes.c_void_p), ("kp0", ctypes.c_void_p)]
    )


_FNS = ("zb_m3_prologue_fwd", "zb_m3_epilogue_fwd", "zb_m3_epilogue_bwd", "zb_m3_prologue_bwd")


def _lib():
    lib = L.lib()
    if not getattr(lib, "_m3_typed", False):
        lib.zb_m3_workspace_bytes.restype = ctypes.c_uint64
        lib.zb_m3_workspace_bytes.argtypes = [ctypes.POINTER(M3Args)]
        for fn in _FNS:
            getattr(lib, fn).restype = ctypes.c_int
            getattr(lib, fn).argtypes = [ctypes.POINTER(M3Args), ctypes.c_void_p]
        lib._m3_typed = True
    return lib


def _v(t: Optional[Tensor]) -> L.View:
    """A [B,T,H,D] tensor as (ptr, sb, st, sh); the innermost dimension must be contiguous."""
    if t is None:
        return L.View(0, 0, 0, 0)
    if t.stride(-1) != 1:
        raise ValueError("innermost dimension must be contiguous")
    return L.View(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))


def _scalar_view(t: Tensor) -> L.View:
    """[B,T,H] per-token scalars: element (b, t, h) at b*sb + t*st + h*sh."""
    return L.View(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))


def _row_view(t: Tensor) -> L.View:
    """[B,T,D] per-token rows: the kernels index (b, t, 0) + d (innermost contiguous)."""
    if t.stride(-1) != 1:
        raise ValueError("innermost dimension must be contiguous")
    return L.View(t.data_ptr(), t.stride(0), t.stride(1), 0)


def _base_args(x, z, Bm, Cm, dd_dt, dd_A, trap, ang, params, A_floor, eps, op_dtype) -> M3Args:
    B, T, H, P = x.shape
    N = Bm.shape[-1]
    a = M3Args()
    a.B, a.T, a.H, a.P, a.N = B, T, H, P, N
    a.A_floor, a.eps = float(A_floor), float(eps)
    a.io_dtype = L.DTYPE_CODE[x.dtype]
    a.op_dtype = L.DTYPE_CODE[op_dtype]
    a.x, a.z = _v(x), _v(z)
    a.Bm, a.Cm, a.ang = _row_view(Bm), _row_view(Cm), _row_view(ang)
    a.dd_dt, a.dd_A, a.trap = _scalar_view(dd_dt), _scalar_view(dd_A), _scalar_view(trap)
    for n, t in zip(("dt_bias", "B_bias", "C_bias", "B_norm_w", "C_norm_w", "D"), params):
        setattr(a, n, t.data_ptr())
    a.status = L.status_word(x.device).data_ptr()
    return a


def _check(rc: int, what: str):
    L.check(rc, what)


def _scan_fwd(xs, q, k, adt, gamma, beta, chunk_size, save_states):
    """The scan with kp / xp read as k / x one token earlier (ZB_FLAG_SHIFTED): no xp tensor.
    Returns y, the saved states (empty without ``save_states``) and the final state."""
    B, T, H, P = xs.shape
    N = q.shape[3]
    dev = xs.device
    lib = L.lib()
    a = _build_args(xs, q, k, k, xs, adt, gamma, beta, chunk_size, L.ZB_FLAG_SHIFTED)
    y = torch.empty(B, T, H, P, dtype=xs.dtype, device=dev)
    final = torch.empty(B, H, P, N, dtype=torch.float32, device=dev)
    states = torch.empty(lib.zb_ssd_states_bytes(ctypes.byref(a)) if save_states else 0, dtype=torch.uint8, device=dev)
    ws = torch.empty(max(int(lib.zb_ssd_workspace_bytes(ctypes.byref(a), 0)), 256), dtype=torch.uint8, device=dev)
    a.y = L.view(y)
    a.final_state = final.data_ptr()
    a.states = L.ptr(states)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    a.status = L.status_word(dev).data_ptr()
    _check(lib.zb_ssd_fwd(ctypes.byref(a), torch.cuda.current_stream(dev).cuda_stream), "zb_ssd_fwd")
    return y, states, final


def _scan_bwd(dy, xs, q, k, adt, gamma, beta, states, chunk_size):
    """Backward of ``_scan_fwd``: dx, dq, dk, dkp, dxp, dadt, dgamma, dbeta (kp / xp gradients per token)."""
    dev = xs.device
    lib = L.lib()
    a = _build_args(xs, q, k, k, xs, adt, gamma, beta, chunk_size, L.ZB_FLAG_SHIFTED)
    grads = [torch.empty(t.shape, dtype=t.dtype, device=dev) for t in (xs, q, k, k, xs, adt, gamma, beta)]
    for n, g in zip(L._VIEWS_BWD, grads):
        setattr(a, n, L.view(g))
    dinit = torch.empty(xs.shape[0], xs.shape[2], xs.shape[3], q.shape[3], dtype=torch.float32, device=dev)
    ws = torch.empty(max(int(lib.zb_ssd_workspace_bytes(ctypes.byref(a), 1)), 256), dtype=torch.uint8, device=dev)
    a.dy = L.view(dy)
    a.states = L.ptr(states)
    a.dinitial_state = dinit.data_ptr()
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    a.status = L.status_word(dev).data_ptr()
    _check(lib.zb_ssd_bwd(ctypes.byref(a), torch.cuda.current_stream(dev).cuda_stream), "zb_ssd_bwd")
    return grads


def _layer_fwd(x, z, Bm, Cm, dd_dt, dd_A, trap, ang, params, A_floor, chunk_size, eps, op_dtype, save_states=True):
    """Prologue -> scan -> epilogue.  Returns the output and the tensors the backward needs."""
    B, T, H, P = x.shape
    N = Bm.shape[-1]
    if T % chunk_size != 0:
        raise AssertionError("sequence length must be a multiple of chunk_size")  # mamba3.py:33
    dev = x.device
    lib = _lib()
    a = _base_args(x, z, Bm, Cm, dd_dt, dd_A, trap, ang, params, A_floor, eps, op_dtype)
    ws = torch.empty(max(int(lib.zb_m3_workspace_bytes(ctypes.byref(a))), 256), dtype=torch.uint8, device=dev)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    q = torch.empty(B, T, H, N, dtype=op_dtype, device=dev)
    k_ext = torch.empty(B, T + 1, H, N, dtype=op_dtype, device=dev)
    adt, gamma, beta = (torch.empty(B, T, H, dtype=torch.float32, device=dev) for _ in range(3))
    theta = torch.empty(B, T, H, N // 4, dtype=torch.float32, device=dev)
    for n, t in (("q", q), ("k_ext", k_ext), ("adt", adt), ("gamma", gamma), ("beta", beta), ("theta", theta)):
        setattr(a, n, t.data_ptr())
    stream = torch.cuda.current_stream(dev).cuda_stream
    _check(lib.zb_m3_prologue_fwd(ctypes.byref(a), stream), "zb_m3_prologue_fwd")
    xs = x if x.dtype == op_dtype else x.to(op_dtype)
    y, states, _ = _scan_fwd(xs, q, k_ext[:, 1:], adt, gamma, beta, chunk_size, save_states)
    out = torch.empty(B, T, H, P, dtype=x.dtype, device=dev)
    a.y, a.out = y.data_ptr(), _v(out)
    _check(lib.zb_m3_epilogue_fwd(ctypes.byref(a), stream), "zb_m3_epilogue_fwd")
    return out, (xs, q, k_ext, adt, gamma, beta, theta, y, states)


def _layer_bwd(x, z, Bm, Cm, dd_dt, dd_A, trap, ang, params, scan_saved, A_floor, chunk_size, eps, op_dtype, dout,
               grads_in):
    """Epilogue backward -> scan backward -> prologue backward.  ``grads_in`` maps dx, dz, dBm,
    dCm, ddd_dt, ddd_A, dtrap, dang to the tensors (or views) to write; returns the parameter
    gradients (fp32, in the order of ``params``)."""
    xs, q, k_ext, adt, gamma, beta, theta, y, states = scan_saved
    B, T, H, P = x.shape
    dev = x.device
    dout = dout.to(x.dtype)
    if dout.stride(-1) != 1:
        dout = dout.contiguous()
    lib = _lib()
    a = _base_args(x, z, Bm, Cm, dd_dt, dd_A, trap, ang, params, A_floor, eps, op_dtype)
    ws = torch.empty(max(int(lib.zb_m3_workspace_bytes(ctypes.byref(a))), 256), dtype=torch.uint8, device=dev)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    for n, t in (("q", q), ("k_ext", k_ext), ("adt", adt), ("gamma", gamma), ("beta", beta), ("theta", theta),
                 ("y", y)):
        setattr(a, n, t.data_ptr())
    a.dout = _v(dout)
    dy = torch.empty(B, T, H, P, dtype=op_dtype, device=dev)
    a.dy, a.dz = dy.data_ptr(), _v(grads_in["dz"] if z is not None else None)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _check(lib.zb_m3_epilogue_bwd(ctypes.byref(a), stream), "zb_m3_epilogue_bwd")
    dxs, dq, dk, dkp, dxp, dadt, dgamma, dbeta = _scan_bwd(dy, xs, q, k_ext[:, 1:], adt, gamma, beta, states,
                                                           chunk_size)
    for n, t in (("dxs", dxs), ("dxp", dxp), ("dq", dq), ("dk", dk), ("dkp", dkp), ("dadt", dadt),
                 ("dgamma", dgamma), ("dbeta", dbeta)):
        setattr(a, n, t.data_ptr())
    a.dx = _v(grads_in["dx"])
    a.dBm, a.dCm, a.dang = (_row_view(grads_in[n]) for n in ("dBm", "dCm", "dang"))
    a.ddd_dt, a.ddd_A, a.dtrap = (_scalar_view(grads_in[n]) for n in ("ddd_dt", "ddd_A", "dtrap"))
    gp = [torch.empty(prm.shape, dtype=torch.float32, device=dev) for prm in params]
    for n, t in zip(("ddt_bias", "dB_bias", "dC_bias", "dB_norm_w", "dC_norm_w", "dD"), gp):
        setattr(a, n, t.data_ptr())
    _check(lib.zb_m3_prologue_bwd(ctypes.byref(a), stream), "zb_m3_prologue_bwd")
    return gp


def _fp32_params(ps):
    return [prm.detach().float().contiguous() for prm in ps]


class _Mamba3Fused(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, z, Bm, Cm, dd_dt, dd_A, trap, ang, dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D, A_floor,
                chunk_size, eps, op_dtype):
        params = _fp32_params((dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D))
        out, saved = _layer_fwd(x, z, Bm, Cm, dd_dt, dd_A, trap, ang, params, A_floor, chunk_size, eps, op_dtype)
        ctx.save_for_backward(x, z if z is not None else torch.empty(0, device=x.device), Bm, Cm, dd_dt, dd_A, trap,
                              ang, *params, *saved)
        ctx.has_z = z is not None
        ctx.meta = (float(A_floor), int(chunk_size), float(eps), op_dtype)
        ctx.param_dtypes = [prm.dtype for prm in (dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D)]
        L.poll_status(x)
        return out

    @staticmethod
    def backward(ctx, dout):
        t = ctx.saved_tensors
        x, z, Bm, Cm, dd_dt, dd_A, trap, ang = t[:8]
        params, saved = t[8:14], t[14:]
        z = z if ctx.has_z else None
        A_floor, chunk_size, eps, op_dtype = ctx.meta
        grads_in = {n: torch.empty(v.shape, dtype=v.dtype, device=x.device)
                    for n, v in (("dx", x), ("dBm", Bm), ("dCm", Cm), ("ddd_dt", dd_dt), ("ddd_A", dd_A),
                                 ("dtrap", trap), ("dang", ang))}
        grads_in["dz"] = torch.empty(z.shape, dtype=z.dtype, device=x.device) if z is not None else None
        gp = _layer_bwd(x, z, Bm, Cm, dd_dt, dd_A, trap, ang, params, saved, A_floor, chunk_size, eps, op_dtype, dout,
                        grads_in)
        gp = [g.to(dt) for g, dt in zip(gp, ctx.param_dtypes)]
        L.poll_status(x)
        return (grads_in["dx"], grads_in["dz"], grads_in["dBm"], grads_in["dCm"], grads_in["ddd_dt"],
                grads_in["ddd_A"], grads_in["dtrap"], grads_in["dang"], *gp, None, None, None, None)


def split_in_proj(zxbc: Tensor, H: int, P: int, N: int):
    """The in_proj output [B, T, 2 H P + 2 N + 3 H + N/4] split as Mamba3.forward does
    (mamba3.py:98-103), as views: z, x [B,T,H,P]; Bm, Cm [B,T,N]; dd_dt, dd_A, trap [B,T,H]; ang [B,T,N/4]."""
    Bsz, T, _ = zxbc.shape
    z, x, Bm, Cm, dd_dt, dd_A, trap, ang = torch.split(zxbc, [H * P, H * P, N, N, H, H, H, N // 4], dim=-1)
    return x.view(Bsz, T, H, P), z.view(Bsz, T, H, P), Bm, Cm, dd_dt, dd_A, trap, ang


class _Mamba3Packed(torch.autograd.Function):
    """The layer body on the packed in_proj output: the split pieces are views, and the backward
    writes every piece's gradient straight into one packed gradient tensor (no concatenation)."""

    @staticmethod
    def forward(ctx, zxbc, dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D, H, P, N, A_floor, chunk_size, eps,
                op_dtype, grad):
        params = _fp32_params((dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D))
        x, z, *rest = split_in_proj(zxbc, H, P, N)
        out, saved = _layer_fwd(x, z, *rest, params, A_floor, chunk_size, eps, op_dtype, save_states=grad)
        if grad:
            ctx.save_for_backward(zxbc, *params, *saved)
        ctx.meta = (H, P, N, float(A_floor), int(chunk_size), float(eps), op_dtype)
        ctx.param_dtypes = [prm.dtype for prm in (dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D)]
        return out

    @staticmethod
    def backward(ctx, dout):
        t = ctx.saved_tensors
        zxbc, params, saved = t[0], t[1:7], t[7:]
        H, P, N, A_floor, chunk_size, eps, op_dtype = ctx.meta
        x, z, Bm, Cm, dd_dt, dd_A, trap, ang = split_in_proj(zxbc, H, P, N)
        dzxbc = torch.empty_like(zxbc, memory_format=torch.contiguous_format)
        gx, gz, gBm, gCm, gdt, gdA, gtr, gang = split_in_proj(dzxbc, H, P, N)
        grads_in = {"dx": gx, "dz": gz, "dBm": gBm, "dCm": gCm, "ddd_dt": gdt, "ddd_A": gdA, "dtrap": gtr,
                    "dang": gang}
        gp = _layer_bwd(x, z, Bm, Cm, dd_dt, dd_A, trap, ang, params, saved, A_floor, chunk_size, eps, op_dtype, dout,
                        grads_in)
        gp = [g.to(dt) for g, dt in zip(gp, ctx.param_dtypes)]
        return (dzxbc, *gp, None, None, None, None, None, None, None, None)


def _check_params(what, H, N, dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D):
    """The layer parameters' shapes (zenith/mamba3.py:89-93) and contiguity (the kernels read them
    as plain arrays)."""
    L.check_shapes(what, dt_bias=(dt_bias, (H,)), B_bias=(B_bias, (H, N)), C_bias=(C_bias, (H, N)),
                   B_norm_w=(B_norm_w, (N,)), C_norm_w=(C_norm_w, (N,)), D=(D, (H,)))
    L.check_contiguous(what, dt_bias=dt_bias, B_bias=B_bias, C_bias=C_bias, B_norm_w=B_norm_w, C_norm_w=C_norm_w, D=D)


def mamba3_layer_packed(zxbc: Tensor, dt_bias: Tensor, B_bias: Tensor, C_bias: Tensor, B_norm_w: Tensor,
                        C_norm_w: Tensor, D: Tensor, H: int, P: int, N: int, A_floor: float = 1e-4,
                        chunk_size: int = 64, eps: float = 1e-5, scan_dtype: Optional[torch.dtype] = None) -> Tensor:
    """``mamba3_ssd_fused`` on the packed in_proj output ``zxbc`` ``[B, T, 2HP + 2N + 3H + N/4]``
    (float32 or bfloat16, innermost dimension contiguous), split as Mamba3.forward splits it
    (mamba3.py:98-100).  Returns ``[B, T, H, P]`` in zxbc's dtype; the gradient of zxbc is
    written as one tensor."""
    if zxbc.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("mamba3_layer_packed: float32 or bfloat16 input")
    L.check_same_device(zxbc.device, "mamba3_layer_packed", dt_bias=dt_bias, B_bias=B_bias, C_bias=C_bias,
                        B_norm_w=B_norm_w, C_norm_w=C_norm_w, D=D)
    if zxbc.dim() != 3 or zxbc.shape[-1] != 2 * H * P + 2 * N + 3 * H + N // 4:
        raise ValueError(f"mamba3_layer_packed: zxbc must be [B, T, 2HP + 2N + 3H + N/4] = [B, T, "
                         f"{2 * H * P + 2 * N + 3 * H + N // 4}], got {tuple(zxbc.shape)}")
    _check_params("mamba3_layer_packed", H, N, dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D)
    L.require_cuda(zxbc.device, "mamba3_layer_packed")
    if zxbc.stride(-1) != 1:
        zxbc = zxbc.contiguous()
    op_dtype = _scan_dtype(zxbc, scan_dtype)
    # no backward (the reference's non-final loops run under no_grad): no saved states
    grad = torch.is_grad_enabled() and any(t.requires_grad for t in (zxbc, dt_bias, B_bias, C_bias, B_norm_w,
                                                                      C_norm_w, D))
    with L.device_guard(zxbc.device):
        return _Mamba3Packed.apply(zxbc, dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D, H, P, N, A_floor, chunk_size,
                                   eps, op_dtype, grad)


def _scan_dtype(x: Tensor, scan_dtype: Optional[torch.dtype]) -> torch.dtype:
    if scan_dtype is not None:
        return scan_dtype
    if x.dtype == torch.float32 and torch.is_autocast_enabled("cuda") and \
            torch.get_autocast_dtype("cuda") == torch.bfloat16:
        return torch.bfloat16  # the reference's matmuls run in bf16 under autocast
    return x.dtype


def mamba3_ssd_fused(x: Tensor, z: Optional[Tensor], Bm: Tensor, Cm: Tensor, dd_dt: Tensor, dd_A: Tensor,
                     trap: Tensor, ang: Tensor, dt_bias: Tensor, B_bias: Tensor, C_bias: Tensor, B_norm_w: Tensor,
                     C_norm_w: Tensor, D: Tensor, A_floor: float = 1e-4, chunk_size: int = 64, eps: float = 1e-5,
                     scan_dtype: Optional[torch.dtype] = None) -> Tensor:
    """``(ssd(x, q, k, kp, xp, adt, gamma, beta) + D x) * silu(z)`` with the scan operands built
    from the in_proj split as ``Mamba3.forward`` does (zenith/mamba3.py:96-119).

    Shapes: x, z ``[B,T,H,P]``; Bm, Cm ``[B,T,N]``; dd_dt, dd_A, trap ``[B,T,H]``; ang
    ``[B,T,N/4]``; dt_bias, D ``[H]``; B_bias, C_bias ``[H,N]``; B_norm_w, C_norm_w ``[N]``.
    The layer inputs share one dtype (float32 or bfloat16) and may be strided views with a
    contiguous innermost dimension.  ``z=None`` skips the gate.  ``scan_dtype`` picks the scan's
    operand precision: float32 (exact, SIMT kernels) or bfloat16 (tensor-core kernels); by
    default the inputs' dtype, or bfloat16 under CUDA bf16 autocast.  Returns ``[B,T,H,P]`` in
    the inputs' dtype.
    """
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("mamba3_ssd_fused: float32 or bfloat16 layer inputs")
    L.check_same_device(x.device, "mamba3_ssd_fused", z=z, Bm=Bm, Cm=Cm, dd_dt=dd_dt, dd_A=dd_A, trap=trap, ang=ang,
                        dt_bias=dt_bias, B_bias=B_bias, C_bias=C_bias, B_norm_w=B_norm_w, C_norm_w=C_norm_w, D=D)
    if x.dim() != 4 or Bm.dim() != 3:
        raise ValueError(f"mamba3_ssd_fused: x [B, T, H, P] and Bm [B, T, N], got {tuple(x.shape)}, {tuple(Bm.shape)}")
    B_, T_, H_, P_ = x.shape
    N_ = Bm.shape[-1]
    L.check_shapes("mamba3_ssd_fused", z=(z, (B_, T_, H_, P_)), Bm=(Bm, (B_, T_, N_)), Cm=(Cm, (B_, T_, N_)),
                   dd_dt=(dd_dt, (B_, T_, H_)), dd_A=(dd_A, (B_, T_, H_)), trap=(trap, (B_, T_, H_)),
                   ang=(ang, (B_, T_, N_ // 4)))
    _check_params("mamba3_ssd_fused", H_, N_, dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D)
    L.require_cuda(x.device, "mamba3_ssd_fused")
    dt = x.dtype
    vals = [t.to(dt) if t.dtype != dt else t for t in (Bm, Cm, dd_dt, dd_A, trap, ang)]
    z = z.to(dt) if z is not None and z.dtype != dt else z
    op_dtype = _scan_dtype(x, scan_dtype)
    with L.device_guard(x.device):
        return _Mamba3Fused.apply(x, z, *vals, dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D, A_floor, chunk_size,
                                  eps, op_dtype)


def layer_forward(module, u: Tensor, scan_dtype: Optional[torch.dtype] = None) -> Tensor:
    """``Mamba3.forward`` (zenith/mamba3.py:96-120) with the layer body fused: in_proj, the
    packed layer body (``mamba3_layer_packed``), out_proj.  ``module`` has the reference's
    attributes.  A bfloat16 in_proj output (autocast) feeds the kernels as it is; they compute in
    float32, as the reference's ``.float()`` upcasts do."""
    Bsz, T, _ = u.shape
    zxbc = module.in_proj(u)
    if zxbc.dtype not in (torch.float32, torch.bfloat16):
        zxbc = zxbc.float()
    y = mamba3_layer_packed(zxbc, module.dt_bias, module.B_bias, module.C_bias, module.B_norm.weight,
                            module.C_norm.weight, module.D, module.nheads, module.headdim, module.d_state,
                            module.A_floor, module.chunk_size, module.B_norm.eps, scan_dtype)
    return module.out_proj(y.reshape(Bsz, T, module.d_inner).to(u.dtype))


def use_b200_layer(module, scan_dtype: Optional[torch.dtype] = None):
    """Route a reference-style ``Mamba3`` module's forward through the fused layer body."""
    module.forward = lambda u: layer_forward(module, u, scan_dtype)
    return module


# ---------------------------------------------------------------------------------------------
# decode: the layer body one token at a time from a carried cache (inference only)

class LayerCache:
    """What one Mamba-3 layer carries from token to token: the scan state ``[B,H,P,N]`` fp32,
    theta ``[B,H,N/4]`` fp32 (the running ``cumsum(DT ang)``, mamba3.py:111) and the previous
    token's k ``[B,H,N]`` and x ``[B,H,P]`` (kp and xp of the next token, mamba3.py:115-116)."""

    def __init__(self, state: Tensor, theta: Tensor, k_prev: Tensor, x_prev: Tensor):
        self.state, self.theta, self.k_prev, self.x_prev = state, theta, k_prev, x_prev


def _prologue(zxbc, params, H, P, N, A_floor, eps, op_dtype, cache: Optional[LayerCache]):
    x, z, Bm, Cm, dd_dt, dd_A, trap, ang = split_in_proj(zxbc, H, P, N)
    B, T = x.shape[:2]
    dev = x.device
    lib = _lib()
    a = _base_args(x, z, Bm, Cm, dd_dt, dd_A, trap, ang, params, A_floor, eps, op_dtype)
    ws = torch.empty(max(int(lib.zb_m3_workspace_bytes(ctypes.byref(a))), 256), dtype=torch.uint8, device=dev)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    q = torch.empty(B, T, H, N, dtype=op_dtype, device=dev)
    k_ext = torch.empty(B, T + 1, H, N, dtype=op_dtype, device=dev)
    adt, gamma, beta = (torch.empty(B, T, H, dtype=torch.float32, device=dev) for _ in range(3))
    theta = torch.empty(B, T, H, N // 4, dtype=torch.float32, device=dev)
    for n, t in (("q", q), ("k_ext", k_ext), ("adt", adt), ("gamma", gamma), ("beta", beta), ("theta", theta)):
        setattr(a, n, t.data_ptr())
    if cache is not None:
        a.theta0, a.kp0 = cache.theta.data_ptr(), cache.k_prev.data_ptr()
    stream = torch.cuda.current_stream(dev).cuda_stream
    _check(lib.zb_m3_prologue_fwd(ctypes.byref(a), stream), "zb_m3_prologue_fwd")
    return a, (x, z), q, k_ext, adt, gamma, beta, theta, stream


@torch.no_grad()
def mamba3_layer_prefill(zxbc: Tensor, dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D, H: int, P: int, N: int,
                         A_floor: float = 1e-4, chunk_size: int = 64, eps: float = 1e-5,
                         scan_dtype: Optional[torch.dtype] = None):
    """``mamba3_layer_packed`` over a prompt (T a multiple of chunk_size) without autograd, also
    returning the ``LayerCache`` that continues it with ``mamba3_layer_step``."""
    if zxbc.stride(-1) != 1:
        zxbc = zxbc.contiguous()
    op_dtype = _scan_dtype(zxbc, scan_dtype)
    params = _fp32_params((dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D))
    T = zxbc.shape[1]
    if T % chunk_size != 0:
        raise AssertionError("sequence length must be a multiple of chunk_size")  # mamba3.py:33
    a, (x, z), q, k_ext, adt, gamma, beta, theta, stream = _prologue(zxbc, params, H, P, N, A_floor, eps, op_dtype,
                                                                     None)
    xs = x if x.dtype == op_dtype else x.to(op_dtype)
    y, _, final = _scan_fwd(xs, q, k_ext[:, 1:], adt, gamma, beta, chunk_size, False)
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    a.y, a.out = y.data_ptr(), _v(out)
    _check(_lib().zb_m3_epilogue_fwd(ctypes.byref(a), stream), "zb_m3_epilogue_fwd")
    cache = LayerCache(final, theta[:, -1].contiguous(), k_ext[:, -1].contiguous(), xs[:, -1].contiguous())
    return out, cache


@torch.no_grad()
def mamba3_layer_step(zxbc: Tensor, dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D, H: int, P: int, N: int,
                      cache: LayerCache, A_floor: float = 1e-4, eps: float = 1e-5) -> Tensor:
    """The layer body for the next token(s) ``zxbc [B, T, n_in]`` (T usually 1) from ``cache``,
    which it advances in place: the prologue continues theta and the k shift from the cache, the
    scan runs in its recurrent form from the cached state (``zb_ssd_decode``), then the gate."""
    if zxbc.stride(-1) != 1:
        zxbc = zxbc.contiguous()
    op_dtype = cache.k_prev.dtype
    params = _fp32_params((dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D))
    a, (x, z), q, k_ext, adt, gamma, beta, theta, stream = _prologue(zxbc, params, H, P, N, A_floor, eps, op_dtype,
                                                                     cache)
    xs = x if x.dtype == op_dtype else x.to(op_dtype)
    xp = torch.cat((cache.x_prev[:, None], xs[:, :-1]), dim=1)
    from .ssd import ssd_decode

    y = ssd_decode(xs, q, k_ext[:, 1:], k_ext[:, :-1], xp, adt, gamma, beta, cache.state)
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    a.y, a.out = y.data_ptr(), _v(out)
    _check(_lib().zb_m3_epilogue_fwd(ctypes.byref(a), stream), "zb_m3_epilogue_fwd")
    cache.theta.copy_(theta[:, -1])
    cache.k_prev.copy_(k_ext[:, -1])
    cache.x_prev.copy_(xs[:, -1])
    return out

