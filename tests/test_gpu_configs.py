"""GPU parity at the benchmark configurations' own shapes, and under torch.compile.

* Inference forward (B64 T512 H32 P64 N64, 4 q/k groups, chunk 64, bf16): y and the final state
  (the decode hand-off) against the float64 recurrence oracle at the exact shape.
* Long context, chunk 128 (bf16): T = 32768 forward and all eight gradients with an initial state
  and a final-state gradient; and the full B1 T131072 H24 sequence, forward for every head and the
  backward of two heads, against the recurrence oracle (oracle/ssd_recurrence.c, O(P N) memory).
* torch.compile of the drop-in (the reference's --compile_scan, zenith/train.py:75-79) and
  torch.library.opcheck of both custom ops.

Tolerance (max|out - ref| / max|ref| per tensor): 2e-2 for bf16 inputs against the float64
oracle on the bf16-rounded inputs; compiled against eager: bitwise.
"""
import pytest
import torch

import zenith_b200
from oracle.recurrence import recurrence_backward, recurrence_forward
from oracle.ssd_oracle import max_rel_err
from zenith_b200.ssd import kernel_family, ssd_bwd_op, ssd_fwd_op
from zenith_b200.synthetic import SHAPES, SsdShape, make_inputs

pytestmark = pytest.mark.gpu

NAMES = ("x", "q", "k", "kp", "xp", "adt", "gamma", "beta")
VEC = ("x", "q", "k", "kp", "xp")
BF16_TOL = 2e-2


def _bf16_inputs(shape, seed):
    inp = make_inputs(shape, seed=seed)
    return {n: (inp[n].to(torch.bfloat16) if n in VEC or n == "dy" else inp[n]) for n in NAMES + ("dy",)}


def _dev(inp, names=NAMES):
    return [inp[n].cuda() for n in names]


def test_inference_forward_at_its_exact_shape_matches_recurrence_oracle():
    s = SHAPES["infer"]  # B64 T512 H32 P64 N64 G4 chunk 64
    inp = _bf16_inputs(s, seed=0)
    args = _dev(inp)
    assert kernel_family(*args, s.chunk, states_saved=False) == "tensor-core"
    with torch.no_grad():
        y, fin = zenith_b200.ssd(*args, s.chunk, return_final_state=True)
    zenith_b200.check_status()
    ref_y, ref_fin = recurrence_forward(*(inp[n] for n in NAMES))
    assert max_rel_err(y, ref_y) < BF16_TOL
    assert max_rel_err(fin, ref_fin) < BF16_TOL


def test_chunk128_long_sequence_forward_backward_matches_recurrence_oracle():
    """T = 32768 at chunk 128 on four heads: few (batch, head) chains, so the library takes its
    segmented route (state-only pass, combine, full pass) in both directions."""
    s = SsdShape(1, 32768, 4, 64, 128, 4, 128)
    inp = _bf16_inputs(s, seed=5)
    g = torch.Generator().manual_seed(17)
    init = torch.randn(s.B, s.H, s.P, s.N, generator=g)
    dfin = torch.randn(s.B, s.H, s.P, s.N, generator=g)
    leaves = [t.requires_grad_() for t in _dev(inp)]
    init_d = init.cuda().requires_grad_()
    y, fin = zenith_b200.ssd(*leaves, s.chunk, initial_state=init_d, return_final_state=True)
    ((y.double() * inp["dy"].cuda().double()).sum() + (fin.double() * dfin.cuda().double()).sum()).backward()
    zenith_b200.check_status()
    args = [inp[n] for n in NAMES]
    ref_y, ref_fin = recurrence_forward(*args, initial_state=init)
    ref = recurrence_backward(inp["dy"], *args, initial_state=init, dfinal=dfin)
    errs = {"y": max_rel_err(y, ref_y), "final_state": max_rel_err(fin, ref_fin),
            "dinitial_state": max_rel_err(init_d.grad, ref["dinitial_state"])}
    errs.update({"d" + n: max_rel_err(t.grad, ref["d" + n]) for n, t in zip(NAMES, leaves)})
    assert all(v < BF16_TOL for v in errs.values()), errs


def test_full_long_context_sequence_matches_recurrence_oracle():
    """B1 T131072 H24 P64 N128 chunk 128: y and the final state of every head, and all eight
    gradients of two heads (heads are independent, so a head's gradients do not depend on the
    others), against the recurrence oracle."""
    s = SHAPES["long"]
    inp = _bf16_inputs(s, seed=0)
    leaves = [t.requires_grad_() for t in _dev(inp)]
    y, fin = zenith_b200.ssd(*leaves, s.chunk, return_final_state=True)
    y.backward(inp["dy"].cuda())
    zenith_b200.check_status()
    ref_y, ref_fin = recurrence_forward(*(inp[n] for n in NAMES))
    assert max_rel_err(y, ref_y) < BF16_TOL
    assert max_rel_err(fin, ref_fin) < BF16_TOL
    heads = [0, s.H - 1]
    sl = {n: inp[n][:, :, heads] for n in NAMES + ("dy",)}
    ref = recurrence_backward(sl["dy"], *(sl[n] for n in NAMES))
    errs = {"d" + n: max_rel_err(t.grad[:, :, heads], ref["d" + n]) for n, t in zip(NAMES, leaves)}
    assert all(v < BF16_TOL for v in errs.values()), errs


def test_compiled_drop_in_matches_eager_bitwise():
    """torch.compile(ssd), as the reference's trainer wraps its scan (zenith/train.py:75-79):
    forward and all eight gradients equal the eager call bit for bit (same kernels)."""
    s = SsdShape(2, 256, 4, 64, 128, 4, 64)
    inp = _bf16_inputs(s, seed=8)
    compiled = torch.compile(zenith_b200.ssd, fullgraph=True)
    outs = []
    for fn in (zenith_b200.ssd, compiled):
        leaves = [t.requires_grad_() for t in _dev(inp)]
        y = fn(*leaves, s.chunk)
        y.backward(inp["dy"].cuda())
        outs.append([y.detach()] + [t.grad for t in leaves])
    zenith_b200.check_status()
    for a, b in zip(*outs):
        assert torch.equal(a, b)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_custom_ops_pass_opcheck(dtype):
    """torch.library.opcheck: schema, fake (meta) implementation, autograd registration and AOT
    dispatch of zenith_b200::ssd_fwd and zenith_b200::ssd_bwd."""
    s = SsdShape(1, 128, 2, 64, 128, 2, 64)
    inp = make_inputs(s, seed=2)
    args = [(inp[n].to(dtype) if n in VEC else inp[n]).cuda().requires_grad_() for n in NAMES]
    torch.library.opcheck(ssd_fwd_op, (*args, s.chunk, None, True, False))
    with torch.no_grad():
        _, _, states = ssd_fwd_op(*args, s.chunk, None, True, False)
    dy = inp["dy"].to(dtype).cuda()
    plain = [a.detach() for a in args]
    torch.library.opcheck(ssd_bwd_op, (dy, *plain, states, s.chunk, None, None, False))
