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
from .ssd import ssd_bwd_op, ssd_fwd_op


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
        + [("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_uint64)]
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
    return a


def _check(rc: int, what: str):
    L.check(rc, what)


class _Mamba3Fused(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, z, Bm, Cm, dd_dt, dd_A, trap, ang, dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D, A_floor,
                chunk_size, eps, op_dtype):
        B, T, H, P = x.shape
        N = Bm.shape[-1]
        if T % chunk_size != 0:
            raise AssertionError("sequence length must be a multiple of chunk_size")  # mamba3.py:33
        dev = x.device
        params = [p.detach().float().contiguous() for p in (dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D)]
        lib = _lib()
        a = _base_args(x, z, Bm, Cm, dd_dt, dd_A, trap, ang, params, A_floor, eps, op_dtype)
        ws = torch.empty(max(int(lib.zb_m3_workspace_bytes(ctypes.byref(a))), 256), dtype=torch.uint8, device=dev)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        q = torch.empty(B, T, H, N, dtype=op_dtype, device=dev)
        k_ext = torch.empty(B, T + 1, H, N, dtype=op_dtype, device=dev)
        xp = torch.empty(B, T, H, P, dtype=op_dtype, device=dev)
        adt, gamma, beta = (torch.empty(B, T, H, dtype=torch.float32, device=dev) for _ in range(3))
        theta = torch.empty(B, T, H, N // 4, dtype=torch.float32, device=dev)
        for n, t in (("q", q), ("k_ext", k_ext), ("xp", xp), ("adt", adt), ("gamma", gamma), ("beta", beta),
                     ("theta", theta)):
            setattr(a, n, t.data_ptr())
        stream = torch.cuda.current_stream(dev).cuda_stream
        _check(lib.zb_m3_prologue_fwd(ctypes.byref(a), stream), "zb_m3_prologue_fwd")
        xs = x if x.dtype == op_dtype else x.to(op_dtype)
        k, kp = k_ext[:, 1:], k_ext[:, :-1]
        y, _, states = ssd_fwd_op(xs, q, k, kp, xp, adt, gamma, beta, chunk_size, None, True, False)
        out = torch.empty(B, T, H, P, dtype=x.dtype, device=dev)
        a.y, a.out = y.data_ptr(), _v(out)
        _check(lib.zb_m3_epilogue_fwd(ctypes.byref(a), stream), "zb_m3_epilogue_fwd")
        ctx.save_for_backward(x, z if z is not None else torch.empty(0, device=dev), Bm, Cm, dd_dt, dd_A, trap, ang,
                              *params, xs, q, k_ext, xp, adt, gamma, beta, theta, y, states)
        ctx.has_z = z is not None
        ctx.meta = (float(A_floor), int(chunk_size), float(eps), op_dtype)
        ctx.param_dtypes = [p.dtype for p in (dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D)]
        return out

    @staticmethod
    def backward(ctx, dout):
        (x, z, Bm, Cm, dd_dt, dd_A, trap, ang, dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D, xs, q, k_ext, xp, adt,
         gamma, beta, theta, y, states) = ctx.saved_tensors
        z = z if ctx.has_z else None
        A_floor, chunk_size, eps, op_dtype = ctx.meta
        B, T, H, P = x.shape
        N = Bm.shape[-1]
        dev = x.device
        dout = dout.to(x.dtype)
        if dout.stride(-1) != 1:
            dout = dout.contiguous()
        lib = _lib()
        params = (dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D)
        a = _base_args(x, z, Bm, Cm, dd_dt, dd_A, trap, ang, params, A_floor, eps, op_dtype)
        ws = torch.empty(max(int(lib.zb_m3_workspace_bytes(ctypes.byref(a))), 256), dtype=torch.uint8, device=dev)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        for n, t in (("q", q), ("k_ext", k_ext), ("xp", xp), ("adt", adt), ("gamma", gamma), ("beta", beta),
                     ("theta", theta), ("y", y)):
            setattr(a, n, t.data_ptr())
        a.dout = _v(dout)
        dy = torch.empty(B, T, H, P, dtype=op_dtype, device=dev)
        dz = torch.empty_like(z, memory_format=torch.contiguous_format) if z is not None else None
        a.dy, a.dz = dy.data_ptr(), _v(dz)
        stream = torch.cuda.current_stream(dev).cuda_stream
        _check(lib.zb_m3_epilogue_bwd(ctypes.byref(a), stream), "zb_m3_epilogue_bwd")
        k, kp = k_ext[:, 1:], k_ext[:, :-1]
        dxs, dq, dk, dkp, dxp, dadt, dgamma, dbeta, _ = ssd_bwd_op(dy, xs, q, k, kp, xp, adt, gamma, beta, states,
                                                                  chunk_size, None, None, False)
        for n, t in (("dxs", dxs), ("dxp", dxp), ("dq", dq), ("dk", dk), ("dkp", dkp), ("dadt", dadt),
                     ("dgamma", dgamma), ("dbeta", dbeta)):
            setattr(a, n, t.data_ptr())
        grads_in = {n: torch.empty(t.shape, dtype=t.dtype, device=dev)
                    for n, t in (("dx", x), ("dBm", Bm), ("dCm", Cm), ("ddd_dt", dd_dt), ("ddd_A", dd_A),
                                 ("dtrap", trap), ("dang", ang))}
        for n in ("dx",):
            setattr(a, n, _v(grads_in[n]))
        a.dBm, a.dCm, a.dang = _row_view(grads_in["dBm"]), _row_view(grads_in["dCm"]), _row_view(grads_in["dang"])
        a.ddd_dt, a.ddd_A, a.dtrap = (_scalar_view(grads_in[n]) for n in ("ddd_dt", "ddd_A", "dtrap"))
        gp = [torch.empty_like(p) for p in params]
        for n, t in zip(("ddt_bias", "dB_bias", "dC_bias", "dB_norm_w", "dC_norm_w", "dD"), gp):
            setattr(a, n, t.data_ptr())
        _check(lib.zb_m3_prologue_bwd(ctypes.byref(a), stream), "zb_m3_prologue_bwd")
        gp = [g.to(dt) for g, dt in zip(gp, ctx.param_dtypes)]
        return (grads_in["dx"], dz, grads_in["dBm"], grads_in["dCm"], grads_in["ddd_dt"], grads_in["ddd_A"],
                grads_in["dtrap"], grads_in["dang"], *gp, None, None, None, None)


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
    dt = x.dtype
    vals = [t.to(dt) if t.dtype != dt else t for t in (Bm, Cm, dd_dt, dd_A, trap, ang)]
    z = z.to(dt) if z is not None and z.dtype != dt else z
    op_dtype = _scan_dtype(x, scan_dtype)
    return _Mamba3Fused.apply(x, z, *vals, dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, D, A_floor, chunk_size, eps,
                              op_dtype)


def layer_forward(module, u: Tensor, scan_dtype: Optional[torch.dtype] = None) -> Tensor:
    """``Mamba3.forward`` (zenith/mamba3.py:96-119) with the layer body fused: in_proj, the split,
    ``mamba3_ssd_fused``, out_proj.  ``module`` has the reference's attributes."""
    Bsz, T, _ = u.shape
    H, P, N = module.nheads, module.headdim, module.d_state
    z, x, Bm, Cm, dd_dt, dd_A, trap, ang = torch.split(
        module.in_proj(u), [module.d_inner, module.d_inner, N, N, H, H, H, module.num_angles], dim=-1)
    x = x.float().view(Bsz, T, H, P) if x.dtype != torch.bfloat16 else x.reshape(Bsz, T, H, P)
    z = z.float().view(Bsz, T, H, P) if z.dtype != torch.bfloat16 else z.reshape(Bsz, T, H, P)
    y = mamba3_ssd_fused(x, z, Bm, Cm, dd_dt, dd_A, trap, ang, module.dt_bias, module.B_bias, module.C_bias,
                         module.B_norm.weight, module.C_norm.weight, module.D, module.A_floor, module.chunk_size,
                         module.B_norm.eps, scan_dtype)
    return module.out_proj(y.reshape(Bsz, T, module.d_inner).to(u.dtype))


def use_b200_layer(module, scan_dtype: Optional[torch.dtype] = None):
    """Route a reference-style ``Mamba3`` module's forward through the fused layer body."""
    module.forward = lambda u: layer_forward(module, u, scan_dtype)
    return module
