"""Long-sequence oracle: TEST INFRASTRUCTURE ONLY.

ctypes binding of ``oracle/libssd_recurrence.so`` (``oracle/ssd_recurrence.c``, built by
``oracle/Makefile``): the SSD scan of zenith/mamba3.py:30-56 as its per-token recurrence
(tests/test_mamba3.py:10-21) and the adjoint of that recurrence (mojo/ssd_bwd.mojo:98-144),
in float64 on the host cores, with O(P N) memory per head.  It checks the CUDA kernels at
sequence lengths the chunked oracle cannot hold (long-context workloads, context-parallel
splits).  Only the tests and ``__graft_entry__.smoke()`` may import it.

Pinned in ``tests/test_oracle.py`` against the golden vectors of the reference's own ``ssd``
(forward and autograd) and against the chunked oracle.
"""

from __future__ import annotations

import ctypes
import pathlib

import torch

LIB = pathlib.Path(__file__).resolve().parent / "libssd_recurrence.so"
_lib = None

F64 = torch.float64
_P = ctypes.c_void_p
_I = ctypes.c_int64


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            raise RuntimeError(f"{LIB} is missing: build it with `make -C oracle`")
        L = ctypes.CDLL(str(LIB))
        L.zb_oracle_recurrence_fwd.restype = ctypes.c_int
        L.zb_oracle_recurrence_fwd.argtypes = [_I] * 6 + [_P] * 11
        L.zb_oracle_recurrence_bwd.restype = ctypes.c_int
        L.zb_oracle_recurrence_bwd.argtypes = [_I] * 6 + [_P] * 20
        _lib = L
    return _lib


def _c(t):
    return None if t is None else t.detach().to("cpu", F64).contiguous()


def _p(t):
    return None if t is None else t.data_ptr()


def recurrence_forward(x, q, k, kp, xp, adt, gamma, beta, initial_state=None):
    """y [B, T, H, P] and the final state [B, H, P, N] (float64, CPU)."""
    B, T, H, P = x.shape
    G, N = q.shape[2], q.shape[3]
    ins = [_c(t) for t in (x, q, k, kp, xp, adt, gamma, beta)]
    init = _c(initial_state)
    y = torch.empty(B, T, H, P, dtype=F64)
    fin = torch.empty(B, H, P, N, dtype=F64)
    rc = lib().zb_oracle_recurrence_fwd(B, T, H, G, P, N, *map(_p, ins), _p(init), _p(y), _p(fin))
    if rc != 0:
        raise RuntimeError("oracle recurrence forward failed")
    return y, fin


def recurrence_backward(dy, x, q, k, kp, xp, adt, gamma, beta, initial_state=None, dfinal=None):
    """All eight input gradients (dq / dk / dkp summed over the heads of a group) and the
    initial-state gradient, as a dict keyed like ``oracle.ssd_oracle.ssd_backward``."""
    B, T, H, P = x.shape
    G, N = q.shape[2], q.shape[3]
    ins = [_c(t) for t in (x, q, k, kp, xp, adt, gamma, beta)]
    outs = {n: torch.empty_like(t) for n, t in zip(("dx", "dq", "dk", "dkp", "dxp", "dadt", "dgamma", "dbeta"), ins)}
    dinit = torch.empty(B, H, P, N, dtype=F64)
    init, dyc, dfin = _c(initial_state), _c(dy), _c(dfinal)  # held until the call returns
    rc = lib().zb_oracle_recurrence_bwd(B, T, H, G, P, N, *map(_p, ins), _p(init), _p(dyc), _p(dfin),
                                        *(_p(outs[n]) for n in outs), _p(dinit))
    if rc != 0:
        raise RuntimeError("oracle recurrence backward failed")
    outs["dinitial_state"] = dinit
    return outs


__all__ = ["recurrence_forward", "recurrence_backward"]
