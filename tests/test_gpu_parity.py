"""GPU parity: the CUDA scan (through the C ABI) against the CPU oracle and the reference's golden
vectors.  Tolerances (max|out - ref| / max|ref| per tensor):
  fp64 inputs: 1e-10;  fp32 inputs: 1e-4;  bf16 inputs: 2e-2 against the fp64 oracle applied to
  the bf16-rounded inputs (the reference computed in bf16 end to end is itself off by up to 1e-1).
"""
import pytest
import torch
import torch.nn.functional as F

import zenith_b200
from oracle.ssd_oracle import max_rel_err, ssd_backward, ssd_forward
from tests.golden_io import CASES, NAMES, load
from zenith_b200.ssd import kernel_family
from zenith_b200.synthetic import SHAPES, SsdShape, make_inputs

pytestmark = pytest.mark.gpu

TOL = {torch.float64: 1e-10, torch.float32: 1e-4, torch.bfloat16: 2e-2, torch.float16: 5e-3}
VEC = ("x", "q", "k", "kp", "xp")


def _cast(inp, dtype, sdtype):
    return {n: inp[n].to(dtype if n in VEC or n == "dy" else sdtype) for n in NAMES + ("dy",)}


def run_cuda(inp, chunk, init=None, dfinal=None, grad=True):
    dev = torch.device("cuda")
    leaves = {n: inp[n].to(dev).clone().requires_grad_(grad) for n in NAMES}
    init_d = None if init is None else init.to(dev).clone().requires_grad_(grad)
    y, fin = zenith_b200.ssd(*(leaves[n] for n in NAMES), chunk, initial_state=init_d, return_final_state=True)
    out = {"y": y.detach(), "final_state": fin.detach()}
    if grad:
        loss = (y.double() * inp["dy"].to(dev).double()).sum()
        if dfinal is not None:
            loss = loss + (fin.double() * dfinal.to(dev).double()).sum()
        loss.backward()
        for n in NAMES:
            out["d" + n] = leaves[n].grad
        if init_d is not None:
            out["dinitial_state"] = init_d.grad
    zenith_b200.check_status()
    return out


def oracle(inp, chunk, init=None, dfinal=None):
    args = [inp[n].double() for n in NAMES]
    y, fin, _ = ssd_forward(*args, chunk, initial_state=init)
    g = ssd_backward(inp["dy"].double(), *args, chunk, initial_state=init, dfinal=dfinal)
    return {"y": y, "final_state": fin, **g}


def compare(got, ref, tol, keys=None):
    keys = keys or [k for k in got if k in ref]
    errs = {k: max_rel_err(got[k], ref[k]) for k in keys}
    bad = {k: v for k, v in errs.items() if not v < tol}
    assert not bad, f"tolerance {tol}: {bad} (all: {errs})"
    return errs


@pytest.mark.parametrize("case", [c for c in CASES if c.endswith("f64")])
def test_fp64_matches_reference_golden(case):
    inp, ref, chunk = load(case)
    got = run_cuda(inp, chunk)
    compare(got, ref, TOL[torch.float64])


@pytest.mark.parametrize("case", CASES)
def test_fp32_matches_reference_golden(case):
    inp, ref, chunk = load(case)
    got = run_cuda(_cast(inp, torch.float32, torch.float32), chunk)
    compare(got, ref, TOL[torch.float32])


@pytest.mark.parametrize("sdtype", [torch.float32, torch.bfloat16])
def test_bf16_tiny_config_matches_oracle_on_rounded_inputs(sdtype):
    inp, _, chunk = load("tiny_f32")
    inp = _cast(inp, torch.bfloat16, sdtype)
    compare(run_cuda(inp, chunk), oracle(inp, chunk), TOL[torch.bfloat16])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [SsdShape(2, 512, 4, 64, 128, 4, 64), SsdShape(1, 384, 3, 64, 128, 3, 128),
                                   SsdShape(2, 256, 8, 64, 64, 2, 64)], ids=["model", "chunk128", "groups"])
def test_model_shapes_match_oracle(dtype, shape):
    inp = make_inputs(shape, seed=3)
    inp = _cast(inp, dtype, torch.float32)
    fam = kernel_family(*zenith_b200.prepare_inputs(*(inp[n].cuda() for n in NAMES)), shape.chunk)
    # bf16 with one q/k group per head runs the tcgen05 forward and backward; the rest SIMT
    assert fam == ("tensor-core" if dtype == torch.bfloat16 and shape.G == shape.H else "simt")
    compare(run_cuda(inp, shape.chunk), oracle(inp, shape.chunk), TOL[dtype])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_initial_state_and_final_state_gradients(dtype):
    shape = SsdShape(2, 192, 3, 64, 128, 3, 64)
    inp = _cast(make_inputs(shape, seed=5), dtype, torch.float32)
    g = torch.Generator().manual_seed(11)
    init = torch.randn(2, 3, 64, 128, generator=g)
    dfinal = torch.randn(2, 3, 64, 128, generator=g)
    got = run_cuda(inp, shape.chunk, init=init, dfinal=dfinal)
    ref = oracle(inp, shape.chunk, init=init.double(), dfinal=dfinal.double())
    compare(got, ref, TOL[dtype])


@pytest.mark.parametrize("T,chunk", [(48, 16), (16, 8), (8, 1), (96, 32), (160, 32)])
def test_ragged_lengths_and_small_chunks(T, chunk):
    inp = _cast(make_inputs(SsdShape(2, T, 2, 16, 32, 2, chunk), seed=T), torch.float32, torch.float32)
    compare(run_cuda(inp, chunk), oracle(inp, chunk), TOL[torch.float32])


def test_noncontiguous_views_like_mamba3_split():
    # Mamba3.forward passes split/pad views (zenith/mamba3.py:99-102,115-116)
    B, T, H, P, N, L = 2, 128, 4, 16, 32, 32
    g = torch.Generator().manual_seed(2)
    proj = torch.randn(B, T, 2 * H * P + 3 * H * N + 7, generator=g, device="cpu")
    x = proj[..., : H * P].view(B, T, H, P)
    k = proj[..., 2 * H * P: 2 * H * P + H * N].view(B, T, H, N)
    q = proj[..., 2 * H * P + H * N: 2 * H * P + 2 * H * N].view(B, T, H, N)
    xp = F.pad(x, (0, 0, 0, 0, 1, 0))[:, :-1]
    kp = F.pad(k, (0, 0, 0, 0, 1, 0))[:, :-1]
    adt = -torch.rand(B, T, H, generator=g) * 0.3
    gm, bt = torch.rand(2, B, T, H, generator=g) * 0.1
    dy = torch.randn(B, T, H, P, generator=g)
    dev = "cuda"
    big = proj.to(dev)
    xd = big[..., : H * P].view(B, T, H, P).requires_grad_(False)
    leaves = [t.to(dev) for t in (x, q, k, kp, xp, adt, gm, bt)]
    # rebuild the views on the device so strides match the model's
    leaves[0] = xd
    leaves[1] = big[..., 2 * H * P + H * N: 2 * H * P + 2 * H * N].view(B, T, H, N)
    leaves[2] = big[..., 2 * H * P: 2 * H * P + H * N].view(B, T, H, N)
    leaves[3] = F.pad(leaves[2], (0, 0, 0, 0, 1, 0))[:, :-1]
    leaves[4] = F.pad(xd, (0, 0, 0, 0, 1, 0))[:, :-1]
    assert not leaves[0].is_contiguous() and not leaves[3].is_contiguous()
    y = zenith_b200.ssd(*leaves, L)
    zenith_b200.check_status()
    ref, _, _ = ssd_forward(x, q, k, kp, xp, adt, gm, bt, L)
    assert max_rel_err(y, ref) < TOL[torch.float32]
    _ = dy


def test_autocast_casts_like_the_reference_and_returns_input_dtype():
    inp, _, chunk = load("tiny_f32")
    dev = "cuda"
    args = [inp[n].to(dev) for n in NAMES]
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = zenith_b200.ssd(*args, chunk)
    assert y.dtype == torch.float32
    rounded = _cast(inp, torch.bfloat16, torch.float32)
    ref, _, _ = ssd_forward(*(rounded[n].double() for n in NAMES), chunk)
    assert max_rel_err(y, ref) < TOL[torch.bfloat16]


def test_no_grad_forward_matches():
    inp, ref, chunk = load("tiny_f32")
    with torch.no_grad():
        y = zenith_b200.ssd(*(inp[n].cuda() for n in NAMES), chunk)
    zenith_b200.check_status()
    assert max_rel_err(y, ref["y"]) < TOL[torch.float32]


@pytest.mark.parametrize("shape", [SsdShape(2, 256, 4, 64, 128, 4, 64), SsdShape(2, 192, 8, 64, 64, 2, 64),
                                   SsdShape(1, 512, 3, 64, 128, 1, 128), SsdShape(3, 64, 2, 64, 128, 2, 64)],
                         ids=["n128", "n64-groups", "g1-chunk128", "one-chunk"])
def test_tensor_core_forward_matches_oracle(shape):
    """bf16 forward without saved states (the tcgen05 kernel), with initial and final state."""
    inp = _cast(make_inputs(shape, seed=21), torch.bfloat16, torch.float32)
    g = torch.Generator().manual_seed(5)
    init = torch.randn(shape.B, shape.H, shape.P, shape.N, generator=g)
    dev = "cuda"
    prepared = zenith_b200.prepare_inputs(*(inp[n].to(dev) for n in NAMES))
    assert kernel_family(*prepared, shape.chunk, states_saved=False) == "tensor-core"
    with torch.no_grad():
        y, fin = zenith_b200.ssd(*(inp[n].to(dev) for n in NAMES), shape.chunk, initial_state=init.to(dev),
                                 return_final_state=True)
    zenith_b200.check_status()
    ref = oracle(inp, shape.chunk, init=init.double())
    assert max_rel_err(y, ref["y"]) < TOL[torch.bfloat16]
    assert max_rel_err(fin, ref["final_state"]) < TOL[torch.bfloat16]


@pytest.mark.parametrize("shape", [SsdShape(24, 128, 24, 64, 128, 24, 64), SsdShape(40, 128, 32, 64, 64, 4, 64)],
                         ids=["n128-576-chains", "n64-1280-chains-groups"])
def test_tensor_core_forward_banded_ticket_order_matches_oracle(shape):
    """More (batch, head) chains than one band of the forward's ticket order (512 chains at N = 128,
    1024 at N = 64; the last band partial): y, the final state and, through the saved states, the
    gradients still match."""
    inp = _cast(make_inputs(shape, seed=23), torch.bfloat16, torch.float32)
    g = torch.Generator().manual_seed(6)
    init = torch.randn(shape.B, shape.H, shape.P, shape.N, generator=g)
    if shape.G == shape.H:  # the tensor-core backward (one q/k group per head) reads the saved states
        got = run_cuda(inp, shape.chunk, init=init)
        compare(got, oracle(inp, shape.chunk, init=init.double()), TOL[torch.bfloat16])
        return
    with torch.no_grad():
        y, fin = zenith_b200.ssd(*(inp[n].to("cuda") for n in NAMES), shape.chunk, initial_state=init.to("cuda"),
                                 return_final_state=True)
    zenith_b200.check_status()
    yr, fr, _ = ssd_forward(*(inp[n].double() for n in NAMES), shape.chunk, initial_state=init.double())
    assert max_rel_err(y, yr) < TOL[torch.bfloat16]
    assert max_rel_err(fin, fr) < TOL[torch.bfloat16]


@pytest.mark.parametrize("shape", [SsdShape(1, 8192, 2, 64, 128, 2, 128), SsdShape(2, 4096, 3, 64, 64, 3, 64)],
                         ids=["B1-T8192-H2", "B2-T4096-H3-N64"])
def test_long_sequences_with_few_heads_match_oracle(shape):
    """Few (batch, head) chains and many chunks: the library splits each sequence into segments
    joined by a state-only pass and a combine step; all outputs, gradients and the boundary
    states must still match the oracle."""
    inp = _cast(make_inputs(shape, seed=31), torch.bfloat16, torch.float32)
    g = torch.Generator().manual_seed(13)
    init = torch.randn(shape.B, shape.H, shape.P, shape.N, generator=g)
    dfinal = torch.randn(shape.B, shape.H, shape.P, shape.N, generator=g)
    got = run_cuda(inp, shape.chunk, init=init, dfinal=dfinal)
    ref = oracle(inp, shape.chunk, init=init.double(), dfinal=dfinal.double())
    compare(got, ref, TOL[torch.bfloat16])
    # the state-only passes (context-parallel pre-passes) take the same segmented route
    dev = "cuda"
    args = [inp[n].to(dev) for n in NAMES]
    fin = zenith_b200.ssd_final_state(*args, shape.chunk, initial_state=init.to(dev))
    dinit = zenith_b200.ssd_dinitial_state(inp["dy"].to(dev), *args, shape.chunk, dfinal=dfinal.to(dev))
    zenith_b200.check_status()
    assert max_rel_err(fin, ref["final_state"]) < TOL[torch.bfloat16]
    assert max_rel_err(dinit, ref["dinitial_state"]) < TOL[torch.bfloat16]


@pytest.mark.parametrize("adt_range", [(-1.0, 0.0), (-12.0, -5.0), (-0.2, 0.1)], ids=["mild", "steep", "mixed-sign"])
def test_tensor_core_decay_paths_match_oracle(adt_range):
    """The tensor-core kernels factorise the decay mask per 8-token block when every adt of a chunk
    lies in [-8, 0], and take a per-element exponential otherwise: chunks of either kind (steep
    decays beyond -8, positive adt) against the oracle, forward and all eight gradients."""
    s = SsdShape(2, 256, 4, 64, 128, 4, 64)
    inp = _cast(make_inputs(s, seed=41), torch.bfloat16, torch.float32)
    lo, hi = adt_range
    inp["adt"] = lo + (hi - lo) * torch.rand(s.B, s.T, s.H, generator=torch.Generator().manual_seed(3))
    compare(run_cuda(inp, s.chunk), oracle(inp, s.chunk), TOL[torch.bfloat16])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_runs_are_bitwise_deterministic(dtype):
    inp = _cast(make_inputs(SsdShape(2, 256, 4, 64, 128, 4, 64), seed=9), dtype, torch.float32)
    a = run_cuda(inp, 64)
    b = run_cuda(inp, 64)
    for k in a:
        assert torch.equal(a[k], b[k]), k


def test_state_only_passes_match_oracle():
    shape = SsdShape(2, 256, 3, 64, 128, 3, 64)
    inp = _cast(make_inputs(shape, seed=4), torch.float32, torch.float32)
    dev = "cuda"
    args = [inp[n].to(dev) for n in NAMES]
    g = torch.Generator().manual_seed(3)
    init = torch.randn(2, 3, 64, 128, generator=g)
    dfin = torch.randn(2, 3, 64, 128, generator=g)
    fin = zenith_b200.ssd_final_state(*args, 64, initial_state=init.to(dev))
    dinit = zenith_b200.ssd_dinitial_state(inp["dy"].to(dev), *args, 64, dfinal=dfin.to(dev))
    zenith_b200.check_status()
    ref = oracle(inp, 64, init=init.double(), dfinal=dfin.double())
    assert max_rel_err(fin, ref["final_state"]) < TOL[torch.float32]
    ref0 = oracle(inp, 64, init=None, dfinal=dfin.double())
    assert max_rel_err(dinit, ref0["dinitial_state"]) < TOL[torch.float32]


def test_full_size_layer_workload_slice_parity_and_state_split():
    """B8 T2048 H24 P64 N128 (bf16, chunk 64).  Heads are independent, so a two-head slice of the
    full run must match the oracle on that slice; and running the two halves of the sequence
    with the first half's final state handed to the second must reproduce the full run."""
    s = SHAPES["layer"]
    inp = _cast(make_inputs(s, seed=0), torch.bfloat16, torch.float32)
    got = run_cuda(inp, s.chunk)
    sl = {n: inp[n][:1, :, :2] for n in NAMES + ("dy",)}
    ref = oracle(sl, s.chunk)
    got_sl = {k: (v[:1, :2] if k == "final_state" else v[:1, :, :2]) for k, v in got.items()}
    compare(got_sl, ref, TOL[torch.bfloat16])
    dev = "cuda"
    h = s.T // 2
    with torch.no_grad():
        args = [inp[n].to(dev) for n in NAMES]
        first = [a[:, :h] for a in args]
        second = [a[:, h:] for a in args]
        y1, f1 = zenith_b200.ssd(*first, s.chunk, return_final_state=True)
        y2, f2 = zenith_b200.ssd(*second, s.chunk, initial_state=f1, return_final_state=True)
    zenith_b200.check_status()
    assert max_rel_err(torch.cat([y1, y2], 1), got["y"]) < 1e-2
    assert max_rel_err(f2, got["final_state"]) < 1e-3


# ------------------------------------------------------------------------------------------------
# recurrent (decode) form


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,tol,P,N", [(torch.float32, 1e-5, 64, 128), (torch.bfloat16, 2e-2, 64, 128),
                                           (torch.bfloat16, 2e-2, 64, 64), (torch.float32, 1e-5, 128, 128),
                                           (torch.float32, 1e-5, 48, 20), (torch.float32, 1e-5, 3, 5)],
                         ids=["f32-p64-n128", "bf16-p64-n128", "bf16-p64-n64", "f32-p128-n128", "f32-p48-n20",
                              "f32-p3-n5"])
def test_decode_matches_per_token_recurrence(dtype, tol, P, N):
    """zb_ssd_decode against the reference test's per-token recurrence (float64 oracle), from a
    random initial state, several tokens in one call and one token per call; the shapes cover each
    row-pass count the kernel is compiled for, rows held by 32 / 16 / 8 / 2 lanes, N not a multiple of 4
    (element-wise state accesses) and P not a multiple of the rows per pass."""
    import zenith_b200
    from oracle.ssd_oracle import naive_recurrence

    g = torch.Generator().manual_seed(7)
    B, T, H, G = 2, 6, 4, 2
    x, xp = torch.randn(2, B, T, H, P, generator=g)
    q, k, kp = torch.randn(3, B, T, G, N, generator=g) / N ** 0.5
    adt = -torch.rand(B, T, H, generator=g)
    gamma, beta = torch.rand(2, B, T, H, generator=g)
    s0 = torch.randn(B, H, P, N, generator=g)
    vec = [t.to(dtype) for t in (x, q, k, kp, xp)]
    ref_y, ref_s = naive_recurrence(*[t.double() for t in vec], adt, gamma, beta, initial_state=s0)
    dev = torch.device("cuda")
    dvec = [t.to(dev) for t in vec]
    dsc = [t.to(dev) for t in (adt, gamma, beta)]
    state = s0.to(dev).contiguous()
    y = zenith_b200.ssd_decode(*dvec, *dsc, state)
    zenith_b200.check_status(dev)
    assert max_rel_err(y, ref_y) < tol
    assert max_rel_err(state, ref_s) < (1e-6 if dtype == torch.float32 else 1e-5)
    state = s0.to(dev).contiguous()  # one token per call (decode)
    ys = [zenith_b200.ssd_decode(*[t[:, i:i + 1] for t in dvec], *[t[:, i:i + 1] for t in dsc], state) for i in range(T)]
    assert max_rel_err(torch.cat(ys, 1), ref_y) < tol
    assert max_rel_err(state, ref_s) < (1e-6 if dtype == torch.float32 else 1e-5)


@pytest.mark.gpu
def test_decode_continues_a_chunked_prefill():
    """Prefill with the chunked tensor-core scan (final state out), then decode the next tokens
    one by one from that state: the decode outputs equal the chunked scan over the whole sequence."""
    import zenith_b200
    from zenith_b200.synthetic import SsdShape, make_inputs

    s = SsdShape(2, 256, 4, 64, 128, 4, 64)
    inp = make_inputs(s, seed=3)
    dev = torch.device("cuda")
    t = {n: (inp[n].to(torch.bfloat16) if n in ("x", "q", "k", "kp", "xp") else inp[n]).to(dev) for n in NAMES}
    y_full = zenith_b200.ssd(*(t[n] for n in NAMES), s.chunk)
    pre = 192
    _, state = zenith_b200.ssd(*(t[n][:, :pre] for n in NAMES), s.chunk, return_final_state=True)
    state = state.contiguous()
    ys = [zenith_b200.ssd_decode(*(t[n][:, i:i + 1] for n in NAMES), state) for i in range(pre, s.T)]
    zenith_b200.check_status(dev)
    assert max_rel_err(torch.cat(ys, 1).float(), y_full[:, pre:].float()) < 2e-2
