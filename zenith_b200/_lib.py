"""ctypes binding of libzenith_ssd.so (the C ABI declared in include/zb_ssd.h).

The shared library is built in-tree by ``zenith_b200.build`` (nvcc, sm_100a).  There is no
fallback: if the library is missing or fails to load, every op raises.
"""

from __future__ import annotations

import contextlib
import ctypes
import pathlib
import threading

import torch

LIB_PATH = pathlib.Path(__file__).resolve().parent / "libzenith_ssd.so"

ZB_F32, ZB_BF16, ZB_F16, ZB_F64 = 0, 1, 2, 3
ZB_FLAG_STATE_ONLY = 1
ZB_FLAG_SHIFTED = 2  # xp / kp are x / k one token later: the kernels read x / k at t - 1
ZB_ERR_SHAPE, ZB_ERR_TIMEOUT, ZB_ERR_SCRATCH_LIMIT = 1, 5, 8
ZB_NOALLOC_SCRATCH_BYTES = 32 << 20

DTYPE_CODE = {torch.float32: ZB_F32, torch.bfloat16: ZB_BF16, torch.float16: ZB_F16, torch.float64: ZB_F64}


class View(ctypes.Structure):
    _fields_ = [("ptr", ctypes.c_void_p), ("sb", ctypes.c_int64), ("st", ctypes.c_int64), ("sh", ctypes.c_int64)]


_VIEWS_FWD = ("x", "q", "k", "kp", "xp", "adt", "gamma", "beta")
_VIEWS_BWD = ("dx", "dq", "dk", "dkp", "dxp", "dadt", "dgamma", "dbeta")


class Args(ctypes.Structure):
    _fields_ = (
        [(n, ctypes.c_int64) for n in ("B", "T", "H", "G", "P", "N", "chunk_size")]
        + [(n, ctypes.c_int32) for n in ("dtype", "scalar_dtype", "flags", "reserved")]
        + [(n, View) for n in _VIEWS_FWD]
        + [("y", View), ("initial_state", ctypes.c_void_p), ("final_state", ctypes.c_void_p), ("states", ctypes.c_void_p)]
        + [("dy", View), ("dfinal_state", ctypes.c_void_p)]
        + [(n, View) for n in _VIEWS_BWD]
        + [("dinitial_state", ctypes.c_void_p), ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
           ("status", ctypes.c_void_p)]
    )


EXPORTS = (
    "zb_version", "zb_strerror", "zb_last_cuda_error", "zb_ssd_states_bytes", "zb_ssd_workspace_bytes",
    "zb_ssd_fwd", "zb_ssd_bwd", "zb_ssd_state_combine", "zb_ssd_total_decay", "zb_ssd_check_status",
    "zb_launch_count", "zb_ssd_decode",
)

_lib = None
_lock = threading.Lock()


class SsdError(RuntimeError):
    def __init__(self, code: int, what: str):
        self.code = code
        super().__init__(f"{what}: zenith_b200 status {code} ({strerror(code)})")


def lib() -> ctypes.CDLL:
    """Load the library once; raise if it is missing (no CPU fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m zenith_b200.build`")
        L = ctypes.CDLL(str(LIB_PATH))
        L.zb_version.restype = ctypes.c_int
        L.zb_strerror.restype = ctypes.c_char_p
        L.zb_strerror.argtypes = [ctypes.c_int]
        L.zb_last_cuda_error.restype = ctypes.c_char_p
        for fn in ("zb_ssd_states_bytes", "zb_ssd_workspace_bytes"):
            getattr(L, fn).restype = ctypes.c_size_t
        L.zb_ssd_states_bytes.argtypes = [ctypes.POINTER(Args)]
        L.zb_ssd_workspace_bytes.argtypes = [ctypes.POINTER(Args), ctypes.c_int]
        for fn in ("zb_ssd_fwd", "zb_ssd_bwd", "zb_ssd_decode"):
            getattr(L, fn).restype = ctypes.c_int
            getattr(L, fn).argtypes = [ctypes.POINTER(Args), ctypes.c_void_p]
        L.zb_ssd_state_combine.restype = ctypes.c_int
        L.zb_ssd_state_combine.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]
        L.zb_ssd_total_decay.restype = ctypes.c_int
        L.zb_ssd_total_decay.argtypes = [ctypes.POINTER(Args), ctypes.c_void_p, ctypes.c_void_p]
        L.zb_ssd_check_status.restype = ctypes.c_int
        L.zb_ssd_check_status.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        L.zb_launch_count.restype = ctypes.c_uint64
        L.zb_ssd_kernel_family.restype = ctypes.c_int
        L.zb_ssd_kernel_family.argtypes = [ctypes.POINTER(Args), ctypes.c_int]
        L.zb_ssd_fwd_noalloc.restype = ctypes.c_int
        L.zb_ssd_fwd_noalloc.argtypes = [ctypes.POINTER(Args), ctypes.c_void_p]
        _lib = L
    return _lib


def launch_count() -> int:
    """Kernels launched by the library so far in this process."""
    return int(lib().zb_launch_count())


def strerror(code: int) -> str:
    try:
        return lib().zb_strerror(code).decode()
    except Exception:  # pragma: no cover - only when the library itself is broken
        return "?"


def check(code: int, what: str) -> None:
    if code != 0:
        extra = lib().zb_last_cuda_error().decode()
        err = SsdError(code, what)
        if extra:
            err.args = (err.args[0] + f" [{extra}]",)
        raise err


def view(t: torch.Tensor | None, ptr: int | None = None) -> View:
    """[B, T, H, D] (or [B, T, H]) tensor -> View; the innermost dimension must be contiguous.
    ``ptr`` replaces the data address (sizing calls that have no data, e.g. fake tensors)."""
    if t is None:
        return View(None, 0, 0, 0)
    if t.dim() == 4:
        assert t.stride(-1) == 1 or t.shape[-1] == 1, "innermost dimension must be contiguous"
    return View(t.data_ptr() if ptr is None else ptr, t.stride(0), t.stride(1), t.stride(2))


def ptr(t: torch.Tensor | None):
    return None if t is None or t.numel() == 0 else t.data_ptr()


def check_same_device(device: torch.device, what: str, **tensors) -> None:
    """Raise ValueError unless every given tensor (None is skipped) lives on ``device``.  The
    library receives raw data addresses: a tensor on another device (or in host memory) would
    otherwise reach a kernel as a pointer it cannot use, where PyTorch's own operators raise."""
    bad = {n: str(t.device) for n, t in tensors.items() if t is not None and t.device != device}
    if bad:
        raise ValueError(f"{what}: expected all tensors on {device}, got "
                         + ", ".join(f"{n} on {d}" for n, d in bad.items()))


def check_shapes(what: str, **named) -> None:
    """Raise ValueError unless each ``name=(tensor, shape)`` tensor (None is skipped) has that
    shape.  The library sizes every operand from a few dimensions of the leading tensors; an
    operand of another shape would be read past its end, where PyTorch's operators raise."""
    bad = [f"{n} {tuple(t.shape)} (expected {tuple(e)})" for n, (t, e) in named.items()
           if t is not None and tuple(t.shape) != tuple(e)]
    if bad:
        raise ValueError(f"{what}: wrong shape: " + ", ".join(bad))


def check_contiguous(what: str, **named) -> None:
    """Raise ValueError unless each tensor (None is skipped) is contiguous (parameters that the
    kernels read as plain arrays)."""
    bad = [n for n, t in named.items() if t is not None and not t.is_contiguous()]
    if bad:
        raise ValueError(f"{what}: expected contiguous tensors: " + ", ".join(bad))


def require_cuda(device: torch.device, what: str) -> None:
    """Raise RuntimeError unless ``device`` is a CUDA device: there is no CPU path, and a host
    address handed to a kernel would fault the GPU instead of raising."""
    if device.type != "cuda":
        raise RuntimeError(f"{what} runs on CUDA tensors only (no CPU path), got {device}")


def device_guard(device: torch.device):
    """Make ``device`` the current CUDA device for a library call (the library launches on the
    current device, on the stream it is given); no CUDA call when it is current already."""
    if device.type != "cuda" or device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device.index)


_status: dict[int, torch.Tensor] = {}


def status_word(device: torch.device) -> torch.Tensor:
    """One int32 status word per device (0 = fine), shared by all calls."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = t
    return t


class StatusPoll:
    """Deferred, non-blocking check of one device's status word.

    ``poll()`` first looks at the asynchronous copy of the word that the previous ``poll()``
    queued (into pinned host memory, behind that call's launches): if the copy has landed and the
    word was nonzero, the word is cleared and ``SsdError`` is raised.  Then it queues a new copy
    behind the launches made so far.  It never waits for the GPU, so an error surfaces at the
    first call after the faulty kernel has finished, usually the next step."""

    def __init__(self, word: torch.Tensor, host: torch.Tensor, make_event):
        self.word, self.host, self.make_event = word, host, make_event
        self.event = None

    def poll(self) -> None:
        if self.event is not None and self.event.query():
            self.event = None
            code = int(self.host[0])
            if code != 0:
                self.word.zero_()
                self.host.zero_()
                check(code, "kernel status (an earlier call)")
        if self.event is None:
            self.host.copy_(self.word, non_blocking=True)
            self.event = self.make_event()
            self.event.record()


_polls: dict[int, StatusPoll] = {}


def _tracing(t: torch.Tensor) -> bool:
    """True while torch.compile / AOT autograd traces the caller with fake tensors."""
    if torch.compiler.is_compiling():
        return True
    from torch._subclasses.fake_tensor import is_fake

    return bool(is_fake(t))


def poll_status(t: torch.Tensor) -> None:
    """Raise ``SsdError`` if an earlier kernel on ``t``'s device has recorded an error (a timed-out
    wait, a label out of range), without synchronising; see ``StatusPoll``.  Does nothing for
    tensors that are not on a GPU, while the call is being traced (torch.compile) and while the
    current stream is being captured into a CUDA graph."""
    if not t.is_cuda or _tracing(t) or torch.cuda.is_current_stream_capturing():
        return
    device = t.device
    idx = device.index if device.index is not None else torch.cuda.current_device()
    p = _polls.get(idx)
    if p is None:
        p = StatusPoll(status_word(torch.device("cuda", idx)), torch.zeros(1, dtype=torch.int32).pin_memory(),
                       torch.cuda.Event)
        _polls[idx] = p
    p.poll()


def check_status(device: torch.device | None = None, reset: bool = True) -> None:
    """Synchronise and raise if a kernel on ``device`` recorded an error (e.g. a timed-out wait)."""
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    st = status_word(dev)
    code = lib().zb_ssd_check_status(st.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    if code != 0:
        if reset:
            st.zero_()
        check(code, "kernel status")
