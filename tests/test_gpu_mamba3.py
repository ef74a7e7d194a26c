"""GPU parity of the fused Mamba-3 layer body (``zenith_b200.mamba3_ssd_fused``): the prologue /
epilogue CUDA kernels around the scan, against golden vectors from the reference ``Mamba3``
module and against the float64 oracle (``oracle/mamba3_oracle.py``).  Error metric: max |out -
ref| / max |ref| per tensor."""
import pytest
import torch

from oracle import mamba3_oracle as M
from oracle.ssd_oracle import max_rel_err
from tests.golden_io import MAMBA3_CASES, load_mamba3

pytestmark = pytest.mark.gpu

ALL = M.INPUTS + M.PARAMS


def _run(tensors, dout, meta, scan_dtype=None, io_dtype=torch.float32):
    import zenith_b200

    dev = torch.device("cuda")
    leaves = {}
    for n in ALL:
        t = tensors[n]
        dt = io_dtype if n in M.INPUTS else torch.float32
        leaves[n] = t.to(dev, dt).clone().requires_grad_(True)
    out = zenith_b200.mamba3_ssd_fused(*(leaves[n] for n in ALL), A_floor=meta["A_floor"], chunk_size=meta["chunk"],
                                       eps=meta["eps"], scan_dtype=scan_dtype)
    out.backward(dout.to(dev, out.dtype))
    torch.cuda.synchronize()
    zenith_b200.check_status()
    return out.detach().double().cpu(), {"d" + n: leaves[n].grad.double().cpu() for n in ALL}


def _synthetic(B, T, H, P, N, seed, A_floor=1e-4):
    """Layer-body inputs with the reference module's scales: dt_bias from its dt init
    (mamba3.py:87-89), biases and norm weights near their initial ones."""
    g = torch.Generator().manual_seed(seed)
    t = {
        "x": torch.randn(B, T, H, P, generator=g), "z": torch.randn(B, T, H, P, generator=g),
        "Bm": torch.randn(B, T, N, generator=g), "Cm": torch.randn(B, T, N, generator=g),
        "dd_dt": torch.randn(B, T, H, generator=g), "dd_A": torch.randn(B, T, H, generator=g),
        "trap": torch.randn(B, T, H, generator=g), "ang": torch.randn(B, T, N // 4, generator=g),
    }
    dt = torch.exp(torch.rand(H, generator=g) * (torch.log(torch.tensor(0.1)) - torch.log(torch.tensor(1e-3)))
                   + torch.log(torch.tensor(1e-3)))
    t["dt_bias"] = dt + torch.log(-torch.expm1(-dt))
    t["B_bias"] = 1 + 0.3 * torch.randn(H, N, generator=g)
    t["C_bias"] = 1 + 0.3 * torch.randn(H, N, generator=g)
    t["B_norm_w"] = 1 + 0.2 * torch.randn(N, generator=g)
    t["C_norm_w"] = 1 + 0.2 * torch.randn(N, generator=g)
    t["D"] = 1 + 0.5 * torch.randn(H, generator=g)
    dout = torch.randn(B, T, H, P, generator=g)
    return t, dout, {"A_floor": A_floor, "chunk": 64, "eps": 1e-5}


@pytest.mark.parametrize("case", MAMBA3_CASES)
def test_fused_layer_fp32_matches_reference_module(case):
    """fp32 scan operands: the layer output and every input / parameter gradient match the
    reference Mamba3 module (float32 goldens) to 1e-4."""
    tensors, dout, ref, meta = load_mamba3(case)
    out, grads = _run(tensors, dout, meta, scan_dtype=torch.float32)
    assert max_rel_err(out, ref["out"].double()) < 1e-4
    for n in ALL:
        r = ref["d" + n].double()
        if r.abs().max() == 0:
            assert grads["d" + n].abs().max() == 0, n
        else:
            assert max_rel_err(grads["d" + n], r) < 1e-4, (n, max_rel_err(grads["d" + n], r))


def test_fused_layer_bf16_scan_matches_oracle():
    """bf16 scan operands (tensor-core scan kernels, P64 N128) against the float64 oracle with the
    same operand rounding, to 2e-2."""
    import zenith_b200
    from zenith_b200.ssd import kernel_family

    tensors, dout, meta = _synthetic(2, 256, 4, 64, 128, seed=21)
    out, grads = _run(tensors, dout, meta, scan_dtype=torch.bfloat16)
    ref_out, ref = M.forward_backward(tensors, dout, meta["A_floor"], meta["chunk"], meta["eps"],
                                      scan_operand_dtype=torch.bfloat16)
    assert max_rel_err(out, ref_out) < 2e-2
    for n in ALL:
        if ref["d" + n].abs().max() == 0:
            assert grads["d" + n].abs().max() < 1e-6, n
        else:
            assert max_rel_err(grads["d" + n], ref["d" + n]) < 2e-2, (n, max_rel_err(grads["d" + n], ref["d" + n]))
    # the scan operands the fused op builds take the tensor-core kernels
    dev = torch.device("cuda")
    B, T, H, P, N = 2, 256, 4, 64, 128
    q = torch.empty(B, T, H, N, dtype=torch.bfloat16, device=dev)
    k_ext = torch.empty(B, T + 1, H, N, dtype=torch.bfloat16, device=dev)
    xb = torch.empty(B, T, H, P, dtype=torch.bfloat16, device=dev)
    s = torch.empty(B, T, H, device=dev)
    assert kernel_family(xb, q, k_ext[:, 1:], k_ext[:, :-1], xb, s, s, s, 64) == "tensor-core"
    del zenith_b200


def test_fused_layer_bf16_inputs_and_long_theta():
    """bf16 layer inputs (the in_proj split under autocast) and a sequence of many theta segments:
    against the oracle on the bf16-rounded inputs."""
    tensors, dout, meta = _synthetic(1, 1024, 3, 64, 64, seed=22)
    for n in M.INPUTS:
        tensors[n] = tensors[n].to(torch.bfloat16).float()
    out, grads = _run(tensors, dout, meta, scan_dtype=torch.bfloat16, io_dtype=torch.bfloat16)
    ref_out, ref = M.forward_backward(tensors, dout, meta["A_floor"], meta["chunk"], meta["eps"],
                                      scan_operand_dtype=torch.bfloat16)
    assert max_rel_err(out, ref_out) < 3e-2
    for n in ALL:
        if ref["d" + n].abs().max() > 0:
            assert max_rel_err(grads["d" + n], ref["d" + n]) < 3e-2, (n, max_rel_err(grads["d" + n], ref["d" + n]))


def test_fused_layer_is_deterministic_and_runs_without_gate():
    tensors, dout, meta = _synthetic(2, 192, 5, 32, 32, seed=23, A_floor=-0.5)
    a = _run(tensors, dout, meta, scan_dtype=torch.float32)
    b = _run(tensors, dout, meta, scan_dtype=torch.float32)
    assert torch.equal(a[0], b[0])
    for n in a[1]:
        assert torch.equal(a[1][n], b[1][n]), n
    # no gate: out = ssd(...) + D x
    t2 = dict(tensors)
    t2["z"] = None
    import zenith_b200

    dev = torch.device("cuda")
    args = [None if t2[n] is None else t2[n].to(dev) for n in ALL]
    out = zenith_b200.mamba3_ssd_fused(*args, A_floor=-0.5, chunk_size=64, scan_dtype=torch.float32)
    ref = M.forward(*(None if t2[n] is None else t2[n].double() for n in ALL), -0.5, 64)
    assert max_rel_err(out.double().cpu(), ref) < 1e-4


def test_fused_layer_rejects_length_not_multiple_of_chunk():
    import zenith_b200

    tensors, dout, meta = _synthetic(1, 96, 2, 16, 16, seed=24)
    dev = torch.device("cuda")
    with pytest.raises(AssertionError, match="sequence length must be a multiple of chunk_size"):
        zenith_b200.mamba3_ssd_fused(*(tensors[n].to(dev) for n in ALL), chunk_size=64)


def test_fused_layer_reads_the_in_proj_split_in_place():
    """Layer inputs as views into one [B, T, n_in] projection, as Mamba3.forward's torch.split makes
    them (mamba3.py:98-100), including an odd column offset that rules out vector accesses."""
    import zenith_b200

    B, T, H, P, N = 2, 128, 3, 16, 32
    tensors, dout, meta = _synthetic(B, T, H, P, N, seed=25)
    sizes = [H * P, H * P, N, N, H, H, H, N // 4]
    names = ("z", "x", "Bm", "Cm", "dd_dt", "dd_A", "trap", "ang")
    dev = torch.device("cuda")
    for pad in (0, 1):
        u = torch.zeros(B, T, pad + sum(sizes), device=dev)
        off = pad
        views = {}
        for n, sz in zip(names, sizes):
            u[..., off:off + sz] = tensors[n].to(dev).reshape(B, T, sz)
            views[n] = u[..., off:off + sz]
            off += sz
        u.requires_grad_(True)
        pieces = torch.split(u[..., pad:], sizes, dim=-1)
        v = dict(zip(names, pieces))
        v["x"] = v["x"].view(B, T, H, P)
        v["z"] = v["z"].view(B, T, H, P)
        params = {n: tensors[n].to(dev).requires_grad_(True) for n in M.PARAMS}
        out = zenith_b200.mamba3_ssd_fused(*(v[n] for n in M.INPUTS), *(params[n] for n in M.PARAMS),
                                           A_floor=meta["A_floor"], chunk_size=64, scan_dtype=torch.float32)
        out.backward(dout.to(dev))
        ref_out, ref = M.forward_backward(tensors, dout, meta["A_floor"], 64, meta["eps"])
        assert max_rel_err(out.detach().double().cpu(), ref_out) < 1e-4, pad
        g = u.grad[..., pad:]
        for n, piece in zip(names, torch.split(g, sizes, dim=-1)):
            assert max_rel_err(piece.reshape(ref["d" + n].shape).double().cpu(), ref["d" + n]) < 1e-4, (pad, n)
        for n in M.PARAMS:
            assert max_rel_err(params[n].grad.double().cpu(), ref["d" + n]) < 1e-4, (pad, n)


@pytest.mark.parametrize("H,scan_dtype", [(28, torch.bfloat16), (31, torch.float32)])
def test_fused_layer_many_heads(H, scan_dtype):
    """Many heads at N = 128: the backward's per-warp row ring shrinks to 2 (bf16) and 1 (fp32)
    slots to fit shared memory; results still match the oracle."""
    tensors, dout, meta = _synthetic(1, 128, H, 16, 128, seed=26)
    out, grads = _run(tensors, dout, meta, scan_dtype=scan_dtype)
    rnd = torch.bfloat16 if scan_dtype == torch.bfloat16 else None
    ref_out, ref = M.forward_backward(tensors, dout, meta["A_floor"], meta["chunk"], meta["eps"],
                                      scan_operand_dtype=rnd)
    tol = 2e-2 if rnd is not None else 1e-4
    assert max_rel_err(out, ref_out) < tol
    for n in ALL:
        if ref["d" + n].abs().max() > 0:
            assert max_rel_err(grads["d" + n], ref["d" + n]) < tol, (n, max_rel_err(grads["d" + n], ref["d" + n]))


@pytest.mark.parametrize("H,P,scan_dtype", [(48, 64, torch.bfloat16), (40, 16, torch.float32), (32, 32, torch.float32)])
def test_fused_layer_head_groups(H, P, scan_dtype):
    """More than 31 heads: the row kernels split the heads into groups (48 -> 2 x 24, 40 -> 2 x 20,
    32 -> 2 x 16); the backward sums the B / C row gradients over the groups before the RMSNorm.
    Results match the oracle."""
    tensors, dout, meta = _synthetic(2, 192, H, P, 128, seed=27)
    out, grads = _run(tensors, dout, meta, scan_dtype=scan_dtype)
    rnd = torch.bfloat16 if scan_dtype == torch.bfloat16 else None
    ref_out, ref = M.forward_backward(tensors, dout, meta["A_floor"], meta["chunk"], meta["eps"],
                                      scan_operand_dtype=rnd)
    tol = 2e-2 if rnd is not None else 1e-4
    assert max_rel_err(out, ref_out) < tol
    for n in ALL:
        if ref["d" + n].abs().max() > 0:
            assert max_rel_err(grads["d" + n], ref["d" + n]) < tol, (n, max_rel_err(grads["d" + n], ref["d" + n]))


@pytest.mark.parametrize("dtype,P,N", [(torch.bfloat16, 64, 128), (torch.float32, 16, 32)])
def test_shifted_flag_matches_explicit_shifted_operands(dtype, P, N):
    """ZB_FLAG_SHIFTED (xp / kp read as x / k one token earlier, what the layer body uses) gives
    bitwise the same y and gradients as passing the shifted tensors explicitly, on the tensor-core
    (bf16) and SIMT (fp32) paths."""
    from zenith_b200 import mamba3 as m3
    from zenith_b200.ssd import ssd_bwd_op, ssd_fwd_op

    g = torch.Generator().manual_seed(31)
    B, T, H = 2, 256, 4
    dev = torch.device("cuda")
    x = torch.randn(B, T, H, P, generator=g).to(dev, dtype)
    q = (torch.randn(B, T, H, N, generator=g) / N ** 0.5).to(dev, dtype)
    k = (torch.randn(B, T, H, N, generator=g) / N ** 0.5).to(dev, dtype)
    adt = (-0.1 * torch.rand(B, T, H, generator=g)).to(dev)
    gamma, beta = (0.1 * torch.rand(2, B, T, H, generator=g)).to(dev)
    dy = torch.randn(B, T, H, P, generator=g).to(dev, dtype)
    shift = lambda t: torch.cat((torch.zeros_like(t[:, :1]), t[:, :-1]), dim=1)  # noqa: E731
    y1, st1, _ = m3._scan_fwd(x, q, k, adt, gamma, beta, 64, True)
    y0, _, st0 = ssd_fwd_op(x, q, k, shift(k), shift(x), adt, gamma, beta, 64, None, True, False)
    g1 = m3._scan_bwd(dy, x, q, k, adt, gamma, beta, st1, 64)
    g0 = ssd_bwd_op(dy, x, q, k, shift(k), shift(x), adt, gamma, beta, st0, 64, None, None, False)[:8]
    torch.cuda.synchronize()
    zenith_b200_check()
    assert torch.equal(y1, y0)
    for a, b in zip(g1, g0):
        assert torch.equal(a, b)


def zenith_b200_check():
    import zenith_b200

    zenith_b200.check_status()
