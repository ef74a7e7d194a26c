"""The CPU oracle against the reference's golden vectors and the reference tests' properties."""
import pytest
import torch

from oracle.ssd_oracle import max_rel_err, naive_recurrence, ssd_backward, ssd_forward
from oracle import lm_oracle, mamba3_oracle
from tests.golden_io import CASES, LM_CASES, MAMBA3_CASES, NAMES, load, load_lm, load_mamba3


@pytest.mark.parametrize("case", CASES)
def test_oracle_forward_matches_reference_golden(case):
    inp, out, L = load(case)
    y, final, _ = ssd_forward(*(inp[n] for n in NAMES), L)
    tol = 1e-12 if out["y"].dtype == torch.float64 else 1e-6
    assert max_rel_err(y, out["y"]) < tol
    assert max_rel_err(final, out["final_state"]) < tol


@pytest.mark.parametrize("case", CASES)
def test_oracle_backward_matches_reference_autograd(case):
    inp, out, L = load(case)
    g = ssd_backward(inp["dy"], *(inp[n] for n in NAMES), L)
    tol = 1e-11 if out["y"].dtype == torch.float64 else 1e-6
    for n in NAMES:
        assert max_rel_err(g["d" + n], out["d" + n]) < tol, n


@pytest.mark.parametrize("chunk", [1, 4, 16, 64])
def test_oracle_is_independent_of_chunk_size(chunk):
    # property of the reference (tests/test_mamba3.py:46-54), extended to the backward
    g = torch.Generator().manual_seed(1)
    B, T, H, P, N = 1, 64, 2, 3, 5
    x, xp = torch.randn(2, B, T, H, P, generator=g, dtype=torch.float64)
    q, k, kp = torch.randn(3, B, T, H, N, generator=g, dtype=torch.float64)
    adt = -torch.rand(B, T, H, generator=g, dtype=torch.float64)
    ga, be = torch.rand(2, B, T, H, generator=g, dtype=torch.float64)
    dy = torch.randn(B, T, H, P, generator=g, dtype=torch.float64)
    args = (x, q, k, kp, xp, adt, ga, be)
    y, fin, _ = ssd_forward(*args, chunk)
    yn, hn = naive_recurrence(*args)
    assert max_rel_err(y, yn) < 1e-12 and max_rel_err(fin, hn) < 1e-12
    g1 = ssd_backward(dy, *args, chunk)
    g64 = ssd_backward(dy, *args, 64)
    for n in NAMES:
        assert max_rel_err(g1["d" + n], g64["d" + n]) < 1e-11


def test_oracle_initial_state_and_final_state_gradients_match_autograd():
    g = torch.Generator().manual_seed(7)
    B, T, H, P, N, L = 2, 32, 2, 4, 6, 8
    ts = [torch.randn(B, T, H, P, generator=g, dtype=torch.float64) for _ in range(2)]
    qs = [torch.randn(B, T, H, N, generator=g, dtype=torch.float64) for _ in range(3)]
    adt = -torch.rand(B, T, H, generator=g, dtype=torch.float64)
    ga, be = torch.rand(2, B, T, H, generator=g, dtype=torch.float64)
    s0 = torch.randn(B, H, P, N, generator=g, dtype=torch.float64)
    dy = torch.randn(B, T, H, P, generator=g, dtype=torch.float64)
    dfin = torch.randn(B, H, P, N, generator=g, dtype=torch.float64)
    leaves = [t.clone().requires_grad_() for t in (ts[0], qs[0], qs[1], qs[2], ts[1], adt, ga, be, s0)]
    y, fin = naive_recurrence(*leaves[:8], initial_state=leaves[8])
    (y * dy).sum().add_((fin * dfin).sum()).backward()
    got = ssd_backward(dy, *[t.detach() for t in leaves[:8]], L, initial_state=s0, dfinal=dfin)
    for n, leaf in zip(NAMES + ("initial_state",), leaves):
        assert max_rel_err(got["d" + n], leaf.grad) < 1e-11, n


def test_oracle_rejects_length_not_multiple_of_chunk():
    t = torch.zeros(1, 10, 1, 2, dtype=torch.float64)
    n = torch.zeros(1, 10, 1, 3, dtype=torch.float64)
    a = torch.zeros(1, 10, 1, dtype=torch.float64)
    with pytest.raises(AssertionError, match="multiple of chunk_size"):
        ssd_forward(t, n, n, n, t, a, a, a, 4)


@pytest.mark.parametrize("case", MAMBA3_CASES)
def test_mamba3_oracle_matches_reference_module(case):
    """The layer-body oracle (prologue, scan, D skip, silu gate) against the reference Mamba3
    module run in float32 with autograd: the output and every input / parameter gradient."""
    tensors, dout, ref, meta = load_mamba3(case)
    out, grads = mamba3_oracle.forward_backward(tensors, dout, meta["A_floor"], meta["chunk"], meta["eps"])
    assert max_rel_err(out, ref["out"].double()) < 2e-6
    for n in mamba3_oracle.INPUTS + mamba3_oracle.PARAMS:
        r = ref["d" + n].double()
        if r.abs().max() == 0:   # dd_A: the A_floor clamp is saturated (mamba3.py:105)
            assert grads["d" + n].abs().max() == 0, n
        else:
            assert max_rel_err(grads["d" + n], r) < 2e-6, n


@pytest.mark.parametrize("case", LM_CASES)
def test_lm_oracle_matches_reference_model(case):
    """The language-model oracle (embedding, input / looped recurrent / output layers, tied LM
    head, next-token cross-entropy) against the reference ZenithForCausalLM run in float32:
    logits, loss and the gradient of every parameter."""
    cfg, ids, loops, params, logits, loss, grads = load_lm(case)
    o_logits, o_loss, o_grads = lm_oracle.forward_backward(params, cfg, ids, loops)
    assert max_rel_err(o_logits, logits.double()) < 2e-5
    assert abs(o_loss.item() - loss.item()) < 2e-5 * abs(loss.item())
    assert set(o_grads) == set(grads)
    for n, g in grads.items():
        if g.abs().max() == 0:   # dd_A rows of in_proj can be saturated by the A_floor clamp
            assert o_grads[n].abs().max() < 1e-12, n
        else:
            assert max_rel_err(o_grads[n], g.double()) < 5e-5, (n, max_rel_err(o_grads[n], g.double()))



# ------------------------------------------------------------------------------------------------
# the long-sequence C oracle (per-token recurrence and its adjoint, oracle/ssd_recurrence.c)

from oracle.recurrence import recurrence_backward, recurrence_forward  # noqa: E402


@pytest.mark.parametrize("case", CASES)
def test_recurrence_oracle_matches_reference_golden(case):
    """Forward, final state and all eight gradients of the recurrence oracle against the
    reference's own ssd and its autograd (goldens)."""
    inp, out, L = load(case)
    args = [inp[n] for n in NAMES]
    y, fin = recurrence_forward(*args)
    tol = 1e-11 if out["y"].dtype == torch.float64 else 1e-6
    assert max_rel_err(y, out["y"]) < tol
    assert max_rel_err(fin, out["final_state"]) < tol
    g = recurrence_backward(inp["dy"], *args)
    for n in NAMES:
        assert max_rel_err(g["d" + n], out["d" + n]) < tol, n


def test_recurrence_oracle_matches_chunked_oracle_with_states_and_groups():
    """Initial state, final-state gradient, grouped q/k and a length that is not a multiple of the
    checkpoint interval: the recurrence oracle against the chunked oracle."""
    g = torch.Generator().manual_seed(11)
    B, T, H, G, P, N = 2, 200, 4, 2, 5, 7
    x, xp = torch.randn(2, B, T, H, P, generator=g, dtype=torch.float64)
    q, k, kp = torch.randn(3, B, T, G, N, generator=g, dtype=torch.float64)
    adt = -0.3 * torch.rand(B, T, H, generator=g, dtype=torch.float64)
    ga, be = torch.rand(2, B, T, H, generator=g, dtype=torch.float64)
    s0 = torch.randn(B, H, P, N, generator=g, dtype=torch.float64)
    dy = torch.randn(B, T, H, P, generator=g, dtype=torch.float64)
    dfin = torch.randn(B, H, P, N, generator=g, dtype=torch.float64)
    args = (x, q, k, kp, xp, adt, ga, be)
    y, fin = recurrence_forward(*args, initial_state=s0)
    yr, finr, _ = ssd_forward(*args, 8, initial_state=s0)
    assert max_rel_err(y, yr) < 1e-12 and max_rel_err(fin, finr) < 1e-12
    got = recurrence_backward(dy, *args, initial_state=s0, dfinal=dfin)
    ref = ssd_backward(dy, *args, 8, initial_state=s0, dfinal=dfin)
    for n in NAMES + ("initial_state",):
        assert max_rel_err(got["d" + n], ref["d" + n]) < 1e-11, n


# ------------------------------------------------------------------------------------------------
# the CPU baseline's restatement of the reference's operation sequence (oracle/ssd_reference_ops.py)

from oracle.ssd_reference_ops import ssd_reference_ops  # noqa: E402


@pytest.mark.parametrize("case", [c for c in CASES if not c.startswith("groups")])
def test_reference_ops_restatement_matches_reference_golden(case):
    """Forward and autograd backward of the restatement the benchmark's CPU baseline times, against
    the reference's own ssd (goldens); one q/k group per head, as in the reference."""
    inp, out, L = load(case)
    leaves = [inp[n].clone().requires_grad_() for n in NAMES]
    y = ssd_reference_ops(*leaves, L)
    y.backward(inp["dy"])
    tol = 1e-11 if out["y"].dtype == torch.float64 else 1e-6
    assert max_rel_err(y, out["y"]) < tol
    for n, t in zip(NAMES, leaves):
        assert max_rel_err(t.grad, out["d" + n]) < tol, n


# ------------------------------------------------------------------------------------------------
# the oracle against the reference itself, live, when it is installed (baseline/_ref)


def _installed_reference_ssd():
    import pathlib
    import sys

    path = pathlib.Path(__file__).resolve().parent.parent / "baseline" / "_ref"
    if not (path / "zenith" / "mamba3.py").exists():
        pytest.skip("the reference is not installed under baseline/_ref")
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))
    import zenith.mamba3

    return zenith.mamba3.ssd


@pytest.mark.parametrize("B,T,H,P,N,chunk,seed", [(2, 192, 3, 8, 12, 64, 11), (1, 96, 2, 5, 7, 32, 12),
                                                  (3, 64, 1, 16, 4, 16, 13), (1, 40, 4, 3, 9, 8, 14)])
def test_oracle_matches_the_installed_reference_live(B, T, H, P, N, chunk, seed):
    """Forward and autograd backward of the installed reference's own ``ssd`` in float64 on fresh
    random inputs (shapes and seeds the goldens do not hold), against the oracle's forward and its
    explicit backward."""
    ref_ssd = _installed_reference_ssd()
    g = torch.Generator().manual_seed(seed)
    f64 = torch.float64
    x, xp = torch.randn(2, B, T, H, P, generator=g, dtype=f64)
    q, k, kp = torch.randn(3, B, T, H, N, generator=g, dtype=f64)
    adt = -2.0 * torch.rand(B, T, H, generator=g, dtype=f64)
    ga, be = torch.rand(2, B, T, H, generator=g, dtype=f64)
    dy = torch.randn(B, T, H, P, generator=g, dtype=f64)
    args = (x, q, k, kp, xp, adt, ga, be)
    leaves = [t.clone().requires_grad_() for t in args]
    y_ref = ref_ssd(*leaves, chunk)
    y_ref.backward(dy)
    y, _, _ = ssd_forward(*args, chunk)
    grads = ssd_backward(dy, *args, chunk)
    assert max_rel_err(y, y_ref) < 1e-12
    for n, t in zip(NAMES, leaves):
        assert max_rel_err(grads["d" + n], t.grad) < 1e-11, n
