"""Host-side input checks of the Python entry points (CPU).

The library receives raw data addresses and sizes every operand from a few leading dimensions,
so the Python layer must refuse what PyTorch's own operators refuse: tensors on different
devices or in host memory, operands of the wrong shape, and parameters that are not contiguous
raise an error before any library call, instead of reaching a kernel as addresses the GPU
cannot use or as buffers it would read past their end.  A call on a CUDA device that is not the
current one runs with that device made current for the call.
"""
import contextlib

import pytest
import torch

import zenith_b200
from zenith_b200 import _lib as L
from zenith_b200 import lm
from zenith_b200.synthetic import SsdShape, make_inputs

NAMES = ("x", "q", "k", "kp", "xp", "adt", "gamma", "beta")


def test_check_same_device_names_the_tensors_on_another_device():
    cpu = torch.device("cpu")
    a, m = torch.zeros(2), torch.zeros(2, device="meta")
    L.check_same_device(cpu, "f", a=a, b=None)
    with pytest.raises(ValueError, match=r"f: expected all tensors on cpu, got b on meta"):
        L.check_same_device(cpu, "f", a=a, b=m)


def test_prepare_inputs_refuses_mixed_devices():
    inp = make_inputs(SsdShape(1, 64, 2, 8, 4, 2, 32))
    args = [inp[n] for n in NAMES]
    args[5] = args[5].to("meta")
    with pytest.raises(ValueError, match="adt on meta"):
        zenith_b200.prepare_inputs(*args)


def _host_calls():
    inp = make_inputs(SsdShape(1, 64, 2, 8, 4, 2, 32))
    args = [inp[n] for n in NAMES]
    B, T, H, P, N = 1, 64, 2, 8, 4
    g = torch.Generator().manual_seed(0)
    layer = dict(x=torch.randn(B, T, H, P, generator=g), z=torch.randn(B, T, H, P, generator=g),
                 Bm=torch.randn(B, T, N, generator=g), Cm=torch.randn(B, T, N, generator=g),
                 dd_dt=torch.randn(B, T, H, generator=g), dd_A=torch.randn(B, T, H, generator=g),
                 trap=torch.randn(B, T, H, generator=g), ang=torch.randn(B, T, N // 4, generator=g),
                 dt_bias=torch.zeros(H), B_bias=torch.ones(H, N), C_bias=torch.ones(H, N), B_norm_w=torch.ones(N),
                 C_norm_w=torch.ones(N), D=torch.ones(H))
    zxbc = torch.randn(B, T, 2 * H * P + 2 * N + 3 * H + N // 4, generator=g)
    prm = (layer["dt_bias"], layer["B_bias"], layer["C_bias"], layer["B_norm_w"], layer["C_norm_w"], layer["D"])
    return {
        "ssd": lambda: zenith_b200.ssd(*args, 32),
        "ssd_decode": lambda: zenith_b200.ssd_decode(*(t[:, :1] for t in args), state=torch.zeros(B, H, P, N)),
        "mamba3_ssd_fused": lambda: zenith_b200.mamba3_ssd_fused(**layer, chunk_size=32),
        "mamba3_layer_packed": lambda: zenith_b200.mamba3_layer_packed(zxbc, *prm, H, P, N),
        "add_rmsnorm": lambda: lm.add_rmsnorm(torch.randn(4, 16), torch.randn(4, 16), torch.ones(16)),
        "linear_cross_entropy": lambda: lm.linear_cross_entropy(torch.randn(4, 16), torch.randn(32, 16),
                                                                torch.zeros(4, dtype=torch.int64)),
    }


@pytest.mark.parametrize("name", list(_host_calls()))
def test_entry_points_refuse_host_tensors_before_any_launch(name):
    before = L.launch_count()
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        _host_calls()[name]()
    assert L.launch_count() == before


def test_device_guard_makes_the_tensors_device_current_only_when_it_is_not(monkeypatch):
    monkeypatch.setattr(torch.cuda, "current_device", lambda: 0)
    assert isinstance(L.device_guard(torch.device("cpu")), contextlib.nullcontext)
    assert isinstance(L.device_guard(torch.device("cuda", 0)), contextlib.nullcontext)
    g = L.device_guard(torch.device("cuda", 1))
    assert isinstance(g, torch.cuda.device) and g.idx == 1


def _shape_errors():
    """(name, call, message) for calls with one operand of the wrong shape (or layout)."""
    inp = make_inputs(SsdShape(1, 64, 2, 8, 4, 2, 32))
    args = [inp[n] for n in NAMES]
    short_k = list(args)
    short_k[2] = args[2][:, :32]
    wide_adt = list(args)
    wide_adt[5] = torch.zeros(1, 64, 3)
    dec = [t[:, :1] for t in args]
    dec[2] = torch.zeros(1, 1, 2, 8)
    B, T, H, P, N = 1, 64, 2, 8, 4
    g = torch.Generator().manual_seed(0)
    layer = dict(x=torch.randn(B, T, H, P, generator=g), z=torch.randn(B, T, H, P, generator=g),
                 Bm=torch.randn(B, T, N, generator=g), Cm=torch.randn(B, T, N, generator=g),
                 dd_dt=torch.randn(B, T, H, generator=g), dd_A=torch.randn(B, T, H, generator=g),
                 trap=torch.randn(B, T, H, generator=g), ang=torch.randn(B, T, 2, generator=g),
                 dt_bias=torch.zeros(H), B_bias=torch.ones(H, N), C_bias=torch.ones(H, N), B_norm_w=torch.ones(N),
                 C_norm_w=torch.ones(N), D=torch.ones(H))
    strided = dict(layer, ang=torch.randn(B, T, N // 4, generator=g), B_bias=torch.ones(H, 2 * N)[:, ::2])
    prm = (layer["dt_bias"], layer["B_bias"], layer["C_bias"], layer["B_norm_w"], layer["C_norm_w"], layer["D"])
    zxbc = torch.randn(B, T, 2 * H * P + 2 * N + 3 * H + N // 4 + 1, generator=g)
    return [
        ("ssd k", lambda: zenith_b200.prepare_inputs(*short_k), r"k \(1, 32, 2, 4\) \(expected \(1, 64, 2, 4\)\)"),
        ("ssd adt", lambda: zenith_b200.prepare_inputs(*wide_adt), r"adt \(1, 64, 3\)"),
        ("ssd_decode k", lambda: zenith_b200.ssd_decode(*dec, state=torch.zeros(B, H, P, N)),
         r"k \(1, 1, 2, 8\) \(expected \(1, 1, 2, 4\)\)"),
        ("fused ang", lambda: zenith_b200.mamba3_ssd_fused(**layer, chunk_size=32), r"ang \(1, 64, 2\)"),
        ("fused strided bias", lambda: zenith_b200.mamba3_ssd_fused(**strided, chunk_size=32), "contiguous tensors: B_bias"),
        ("packed width", lambda: zenith_b200.mamba3_layer_packed(zxbc, *prm, H, P, N), "zxbc must be"),
        ("rmsnorm b", lambda: lm.add_rmsnorm(torch.randn(4, 16), torch.randn(4, 8), torch.ones(16)), r"b \(4, 8\)"),
        ("rmsnorm weight", lambda: lm.add_rmsnorm(torch.randn(4, 16), None, torch.ones(8)), r"weight \(8,\)"),
        ("xent labels", lambda: lm.linear_cross_entropy(torch.randn(4, 16), torch.randn(32, 16),
                                                        torch.zeros(5, dtype=torch.int64)), r"labels \(5,\)"),
        ("xent weight", lambda: lm.linear_cross_entropy(torch.randn(4, 16), torch.randn(32, 8),
                                                        torch.zeros(4, dtype=torch.int64)), r"weight \(32, 8\)"),
    ]


@pytest.mark.parametrize("case", range(len(_shape_errors())), ids=[c[0] for c in _shape_errors()])
def test_entry_points_refuse_wrong_shapes_before_any_launch(case):
    _, call, message = _shape_errors()[case]
    before = L.launch_count()
    with pytest.raises(ValueError, match=message):
        call()
    assert L.launch_count() == before


@pytest.mark.parametrize("empty", ["B", "H", "P", "N"])
def test_empty_dimensions_give_the_references_zeros_without_a_launch(empty):
    """B, H, P or N of size zero (T > 0): y is all zeros (empty unless only N is 0) and every
    gradient is zero, as the reference's matmuls over empty dimensions give; no kernel runs.
    Checked against the installed reference's own ssd when it is there."""
    import pathlib
    import sys

    sizes = dict(B=2, H=3, P=4, N=8)
    sizes[empty] = 0
    B, H, P, N, T = sizes["B"], sizes["H"], sizes["P"], sizes["N"], 128
    g = torch.Generator().manual_seed(1)
    shapes = [(B, T, H, P), (B, T, H, N), (B, T, H, N), (B, T, H, N), (B, T, H, P), (B, T, H), (B, T, H), (B, T, H)]
    ours = [torch.randn(*s, generator=g).requires_grad_() for s in shapes]
    before = L.launch_count()
    y, fin = zenith_b200.ssd(*ours, 64, return_final_state=True)
    assert L.launch_count() == before
    assert tuple(y.shape) == (B, T, H, P) and not y.any()
    assert tuple(fin.shape) == (B, H, P, N)
    y.sum().backward()
    for t in ours:
        assert t.grad is not None and tuple(t.grad.shape) == tuple(t.shape) and not t.grad.any()
    path = pathlib.Path(__file__).resolve().parent.parent / "baseline" / "_ref"
    if (path / "zenith" / "mamba3.py").exists():
        if str(path) not in sys.path:
            sys.path.insert(0, str(path))
        import zenith.mamba3

        ref = zenith.mamba3.ssd(*(t.detach() for t in ours), 64)
        assert ref.shape == y.shape and torch.equal(ref, y)


def test_empty_sequence_raises_like_the_reference():
    """T = 0: the reference fails (torch.stack of no chunks, a RuntimeError); so does this library."""
    shapes = [(1, 0, 2, 4), (1, 0, 2, 8), (1, 0, 2, 8), (1, 0, 2, 8), (1, 0, 2, 4), (1, 0, 2), (1, 0, 2), (1, 0, 2)]
    with pytest.raises(RuntimeError):
        zenith_b200.ssd(*(torch.zeros(*s) for s in shapes), 64)
