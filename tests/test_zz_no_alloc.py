"""zb_ssd_fwd_noalloc: the forward scan for callers that cannot allocate device memory.

Some callers of this library cannot obtain device memory for a call (a serving runtime that
reserved every byte up front, a foreign-language binding without a CUDA allocator).  For
them the library has one extra C entry point whose scratch lives in a fixed device array
inside the library; the caller passes only its inputs and outputs.  This file checks it
through the C ABI against the regular entry point (zb_ssd_fwd, behind zenith_b200.ssd) and
against the float64 oracle, on two calls in a row with different inputs, since every call
reuses the same array; and once with a saved-states buffer, whose states a regular backward
then reads.  The file is named to run last.
"""
import ctypes

import pytest
import torch

import zenith_b200
from oracle.ssd_oracle import max_rel_err, ssd_backward, ssd_forward
from zenith_b200 import _lib as L
from zenith_b200.ssd import _build_args, prepare_inputs
from zenith_b200.synthetic import SsdShape, make_inputs

NAMES = ("x", "q", "k", "kp", "xp", "adt", "gamma", "beta")
TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}


def _inputs(shape, seed, dtype, dev):
    inp = make_inputs(shape, seed=seed)
    return prepare_inputs(*((inp[n].to(dtype) if n in ("x", "q", "k", "kp", "xp") else inp[n]).to(dev) for n in NAMES))


def _noalloc_forward(args, chunk, states=None):
    """Call the C entry point directly; the test (the caller) owns y, the final state and the
    optional saved-states buffer."""
    x = args[0]
    B, T, H, P = x.shape
    N = args[1].shape[-1]
    y = torch.empty(B, T, H, P, dtype=x.dtype, device=x.device)
    fin = torch.empty(B, H, P, N, dtype=torch.float32, device=x.device)
    a = _build_args(*args, chunk)
    a.y = L.view(y)
    a.final_state = fin.data_ptr()
    a.states = L.ptr(states)
    a.status = L.status_word(x.device).data_ptr()
    rc = L.lib().zb_ssd_fwd_noalloc(ctypes.byref(a), torch.cuda.current_stream(x.device).cuda_stream)
    L.check(rc, "zb_ssd_fwd_noalloc")
    return y, fin


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_forward_matches_regular_entry_point_twice_in_a_row(dtype):
    dev = torch.device("cuda")
    shape = SsdShape(2, 256, 4, 64, 128, 4, 64)
    for seed in (1, 2):  # the second call runs on scratch left over from the first
        args = _inputs(shape, seed, dtype, dev)
        with torch.no_grad():
            y_ref, fin_ref = zenith_b200.ssd(*args, shape.chunk, return_final_state=True)
        y, fin = _noalloc_forward(args, shape.chunk)
        zenith_b200.check_status(dev)
        assert max_rel_err(y, y_ref) < TOL[dtype], seed
        assert max_rel_err(fin, fin_ref) < TOL[dtype], seed
        # and against the float64 oracle on the same (rounded) inputs
        o_y, o_fin, _ = ssd_forward(*(t.double().cpu() for t in args), shape.chunk)
        assert max_rel_err(y, o_y) < TOL[dtype], seed
        assert max_rel_err(fin, o_fin) < TOL[dtype], seed


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_forward_saves_states_that_a_regular_backward_reads(dtype):
    """With a saved-states buffer (the caller's memory) the no-alloc forward writes the chunk
    states a training step's backward needs; the regular backward on them gives the oracle's
    gradients."""
    from zenith_b200.ssd import ssd_bwd_op, states_nbytes

    dev = torch.device("cuda")
    shape = SsdShape(2, 256, 4, 64, 128, 4, 64)
    args = _inputs(shape, 3, dtype, dev)
    states = torch.empty(states_nbytes(*args, shape.chunk), dtype=torch.uint8, device=dev)
    y, fin = _noalloc_forward(args, shape.chunk, states)
    dy = make_inputs(shape, seed=3)["dy"].to(dtype).to(dev)
    grads = ssd_bwd_op(dy, *args, states, shape.chunk, None, None, False)
    zenith_b200.check_status(dev)
    ref_in = [t.double().cpu() for t in args]
    o_y, o_fin, _ = ssd_forward(*ref_in, shape.chunk)
    ref = ssd_backward(dy.double().cpu(), *ref_in, shape.chunk)
    assert max_rel_err(y, o_y) < TOL[dtype]
    assert max_rel_err(fin, o_fin) < TOL[dtype]
    for n, g in zip(NAMES, grads[:8]):
        assert max_rel_err(g, ref["d" + n]) < TOL[dtype], n


def test_noalloc_rejects_calls_beyond_the_fixed_scratch_before_touching_the_gpu():
    big = SsdShape(64, 8192, 32, 64, 128, 32, 64)
    x = torch.empty(0)
    a = L.Args()
    a.B, a.T, a.H, a.G, a.P, a.N, a.chunk_size = big.B, big.T, big.H, big.G, big.P, big.N, big.chunk
    a.dtype = a.scalar_dtype = L.ZB_F32
    assert L.lib().zb_ssd_workspace_bytes(ctypes.byref(a), 0) > L.ZB_NOALLOC_SCRATCH_BYTES
    assert L.lib().zb_ssd_fwd_noalloc(ctypes.byref(a), None) == L.ZB_ERR_SCRATCH_LIMIT
    assert "no-alloc" in L.strerror(L.ZB_ERR_SCRATCH_LIMIT)
    del x
