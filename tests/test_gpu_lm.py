"""GPU parity of the language-model kernels and model (zenith_b200.lm): the fused residual-add +
RMSNorm and the one-pass cross-entropy against plain float64 PyTorch restatements, and the whole
looped LM (forward logits, loss, every parameter gradient) against golden vectors from the
reference ZenithForCausalLM (float32) and against the float64 oracle under bf16 autocast.
Error metric: max |out - ref| / max |ref| per tensor."""
import pytest
import torch
import torch.nn.functional as F

from oracle import lm_oracle
from oracle.ssd_oracle import max_rel_err
from tests.golden_io import LM_CASES, load_lm

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def _rmsnorm_ref(s, w, eps):
    return s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + eps) * w


@pytest.mark.parametrize("x_dtype,b_dtype,u_dtype,D", [
    (torch.float32, torch.float32, torch.float32, 256),
    (torch.float32, torch.bfloat16, torch.bfloat16, 1536),
    (torch.bfloat16, torch.bfloat16, torch.bfloat16, 640),
    (torch.float32, None, torch.float32, 100),           # D % 8 != 0: the scalar path
    (torch.float32, torch.float32, torch.bfloat16, 36),
    (torch.float32, torch.bfloat16, torch.bfloat16, 4096),  # D > 2048: one warp per row, 16-byte accesses
])
def test_add_rmsnorm_matches_torch(x_dtype, b_dtype, u_dtype, D):
    from zenith_b200 import lm

    g = torch.Generator().manual_seed(D)
    M = 3 * 333
    a = torch.randn(M, D, generator=g).to(x_dtype)
    b = torch.randn(M, D, generator=g).to(b_dtype) if b_dtype else None
    w = 1 + 0.3 * torch.randn(D, generator=g)
    ds = torch.randn(M, D, generator=g)
    du = torch.randn(M, D, generator=g)
    la, lw = a.to(DEV).requires_grad_(), w.to(DEV).requires_grad_()
    lb = b.to(DEV).requires_grad_() if b is not None else None
    out = lm.add_rmsnorm(la, lb, lw, 1e-5, u_dtype)
    s, u = out if b is not None else (la, out)
    tot = (u.float() * du.to(DEV)).sum() + ((s.float() * ds.to(DEV)).sum() if b is not None else 0)
    tot.backward()
    # reference: float64 on the stored sum (rounded to the residual dtype), as the kernel computes
    ra, rw = a.double().requires_grad_(), w.double().requires_grad_()
    rb = b.double().requires_grad_() if b is not None else None
    rs = (ra + rb) if rb is not None else ra
    rs_st = rs + (rs.to(x_dtype).double() - rs).detach()
    ru = _rmsnorm_ref(rs_st, rw, 1e-5)
    rtot = (ru * du.double()).sum() + ((rs_st * ds.double()).sum() if rb is not None else 0)
    rtot.backward()
    tol_u = 1e-5 if u_dtype == torch.float32 else 8e-3
    tol_g = 1e-5 if (x_dtype == torch.float32 and u_dtype == torch.float32) else 2e-2
    assert max_rel_err(u.double().cpu(), ru.to(u_dtype).double()) < tol_u
    if b is not None:
        assert max_rel_err(s.double().cpu(), rs_st) < 1e-6
        assert max_rel_err(lb.grad.double().cpu(), rb.grad) < tol_g
    assert max_rel_err(la.grad.double().cpu(), ra.grad) < tol_g
    assert max_rel_err(lw.grad.double().cpu(), rw.grad) < tol_g


@pytest.mark.parametrize("dtype,V", [(torch.float32, 1000), (torch.float32, 999), (torch.bfloat16, 32000),
                                     (torch.bfloat16, 50001), (torch.float32, 8)])
@pytest.mark.parametrize("chunk_rows", [None, 64])
def test_linear_cross_entropy_matches_torch(dtype, V, chunk_rows, monkeypatch):
    """One row chunk, or chunks of 64 rows (the last of the 300 ragged) with the weight gradient
    accumulated over them."""
    from zenith_b200 import lm

    if chunk_rows:
        monkeypatch.setattr(lm, "_CE_CHUNK_BYTES", chunk_rows * V * (4 if dtype == torch.float32 else 2))
    g = torch.Generator().manual_seed(V)
    M, d = 300, 64
    h = torch.randn(M, d, generator=g)
    W = 0.3 * torch.randn(V, d, generator=g)
    labels = torch.randint(0, V, (M,), generator=g)
    labels[::7] = -100                                   # ignored rows
    lh, lW = h.to(DEV).requires_grad_(), W.to(DEV).requires_grad_()
    loss = lm.linear_cross_entropy(lh, lW, labels.to(DEV), compute_dtype=dtype)
    loss.backward()
    # float64 reference on the operands and logits as the kernel sees them (rounded to dtype)
    rh, rW = h.double().requires_grad_(), W.double().requires_grad_()
    rnd = lambda t: t + (t.to(dtype).double() - t).detach()
    logits = rnd(rnd(rh) @ rnd(rW).T)
    ref = F.cross_entropy(logits, labels)
    ref.backward()
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert abs(loss.item() - ref.item()) < tol * abs(ref.item())
    assert max_rel_err(lh.grad.double().cpu(), rh.grad) < tol
    assert max_rel_err(lW.grad.double().cpu(), rW.grad) < tol


@pytest.mark.parametrize("x_dtype", [torch.bfloat16, torch.float32])
def test_autocast_projection_matches_float64(x_dtype):
    """The LM's bias-free projection under bf16 autocast: output and input gradient as bf16
    autocast gives them, the float32 weight gradient straight from the GEMM; all against float64
    on the bf16-rounded operands (2e-2, and 1e-5 for the weight gradient, which sees no bf16
    output rounding)."""
    from zenith_b200 import lm

    g = torch.Generator().manual_seed(7)
    x = torch.randn(2, 300, 96, generator=g).to(x_dtype)
    lin = torch.nn.Linear(96, 200, bias=False).to(DEV)
    dy = torch.randn(2, 300, 200, generator=g)
    lx = x.to(DEV).requires_grad_()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = lm._proj(lin, lx)
    assert y.dtype == torch.bfloat16
    y.backward(dy.to(DEV, torch.bfloat16))
    assert lx.grad.dtype == x_dtype and lin.weight.grad.dtype == torch.float32
    rx = x.to(torch.bfloat16).double().requires_grad_()
    rw = lin.weight.detach().cpu().to(torch.bfloat16).double().requires_grad_()
    ry = rx @ rw.T
    ry.backward(dy.to(torch.bfloat16).double())
    assert max_rel_err(y.double().cpu(), ry) < 2e-2
    assert max_rel_err(lx.grad.double().cpu(), rx.grad) < 2e-2
    assert max_rel_err(lin.weight.grad.double().cpu(), rw.grad) < 1e-5


def test_cross_entropy_rejects_out_of_range_labels():
    """A label outside [0, V) sets the device status word (the row is skipped, nothing faults)."""
    import zenith_b200
    from zenith_b200 import lm

    h = torch.randn(4, 16, device=DEV)
    W = torch.randn(32, 16, device=DEV)
    labels = torch.tensor([1, 2, 40, 3], device=DEV)
    lm.linear_cross_entropy(h, W, labels)
    with pytest.raises(zenith_b200.SsdError, match="status 9"):
        zenith_b200.check_status()
    zenith_b200.check_status()   # reset by the failed check


def _model(case):
    from zenith_b200 import lm

    cfg, ids, loops, params, logits, loss, grads = load_lm(case)
    model = lm.ZenithForCausalLM(cfg).to(DEV)
    lm.load_reference_state_dict(model, {n: t.to(DEV) for n, t in params.items()})
    return model, cfg, ids, loops, params, logits, loss, grads


@pytest.mark.parametrize("case", LM_CASES)
def test_lm_fp32_matches_reference_model(case):
    """float32 throughout (exact scan): logits, loss and every parameter gradient of the reference
    ZenithForCausalLM to 1e-4, including the no-autograd recurrent loops."""
    model, cfg, ids, loops, params, logits, loss, grads = _model(case)
    out = model(ids.to(DEV), labels=ids.to(DEV), loops=loops, return_logits=True)
    out.loss.backward()
    torch.cuda.synchronize()
    assert max_rel_err(out.logits.double().cpu(), logits.double()) < 1e-4
    assert abs(out.loss.item() - loss.item()) < 1e-4 * abs(loss.item())
    named = dict(model.named_parameters())
    for n, g in grads.items():
        assert max_rel_err(named[n].grad.double().cpu(), g.double()) < 1e-4, (n, max_rel_err(named[n].grad.double().cpu(), g.double()))


@pytest.mark.parametrize("case", LM_CASES)
def test_lm_bf16_autocast_matches_oracle(case):
    """bf16 autocast (bf16 GEMMs, bf16 in_proj output into the layer kernels, tensor-core scan)
    against the float64 oracle: loss to 1e-2, logits and parameter gradients to 5e-2 (bf16
    rounding of the GEMM operands through five layers)."""
    model, cfg, ids, loops, params, logits, loss, grads = _model(case)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = model(ids.to(DEV), labels=ids.to(DEV), loops=loops, return_logits=True)
    out.loss.backward()
    o_logits, o_loss, o_grads = lm_oracle.forward_backward(params, cfg, ids, loops)
    assert abs(out.loss.item() - o_loss.item()) < 1e-2 * abs(o_loss.item())
    assert max_rel_err(out.logits.double().cpu(), o_logits) < 5e-2
    named = dict(model.named_parameters())
    errs = {n: max_rel_err(named[n].grad.double().cpu(), g) for n, g in o_grads.items() if g.abs().max() > 0}
    bad = {n: e for n, e in errs.items() if not e < 5e-2}
    assert not bad, bad


def test_train_step_reduces_loss():
    """A few AdamW steps on one fixed batch of the small configuration lower its loss."""
    from zenith_b200 import lm

    cfg = dict(vocab_size=256, d_model=64, d_state=16, expand=2, headdim=16, chunk_size=32, n_input=1,
               n_recurrent=1, n_output=1, max_loops=2)
    torch.manual_seed(0)
    model = lm.ZenithForCausalLM(cfg).to(DEV)
    opt = lm.make_optimizer(model, lr=3e-3)
    ids = torch.randint(0, 256, (2, 64), device=DEV)
    losses = [lm.train_step(model, opt, ids, loops=2).item() for _ in range(8)]
    assert losses[-1] < losses[0] - 0.1, losses


def test_train_step_raises_on_a_label_outside_the_vocabulary():
    """The reference's F.cross_entropy raises on a label outside the vocabulary.  Here the loss
    kernel records it in the device status word (nothing faults, the row is skipped) and the
    training loop raises SsdError from train_step once that is visible, without a sync of its
    own: at the latest in the step after the faulty one has finished on the GPU."""
    import zenith_b200
    from zenith_b200 import lm

    cfg = dict(vocab_size=256, d_model=64, d_state=16, expand=2, headdim=16, chunk_size=32, n_input=1,
               n_recurrent=1, n_output=1, max_loops=1)
    torch.manual_seed(0)
    model = lm.ZenithForCausalLM(cfg).to(DEV)
    opt = lm.make_optimizer(model)
    good = torch.randint(0, 256, (2, 64), device=DEV)
    bad = good.clone()
    bad[1, 5] = 300                      # a label outside [0, 256); the input ids stay in range (an
                                         # id outside the table would fault in the embedding gather)
    lm.train_step(model, opt, good)
    lm.train_step(model, opt, good, labels=bad)  # queued; the error is recorded on the device
    torch.cuda.synchronize()             # (the faulty step has finished by the next call)
    with pytest.raises(zenith_b200.SsdError, match="status 9"):
        lm.train_step(model, opt, good)
    lm.train_step(model, opt, good)      # the word was cleared: training goes on
    zenith_b200.check_status()


# behaviour of the model, as the reference's own model tests check it (tests/test_model.py)

TINY = dict(vocab_size=1024, d_model=128, d_state=32, expand=2, headdim=32, chunk_size=32, n_input=1, n_recurrent=2,
            n_output=1, max_loops=4)


def _tiny():
    from zenith_b200 import lm

    torch.manual_seed(0)
    return lm.ZenithForCausalLM(TINY).to(DEV)


def test_loss_is_finite_for_each_loop_count_and_none_without_labels():
    model = _tiny()
    ids = torch.randint(0, 1024, (2, 64), device=DEV)
    for k in range(1, 5):
        out = model(ids, labels=ids, loops=k, return_logits=True)
        assert out.logits.shape == (2, 64, 1024)
        assert torch.isfinite(out.loss)
    assert model(ids[:1, :32]).loss is None


def test_more_loops_change_output_and_default_is_max_loops():
    model = _tiny()
    ids = torch.randint(0, 1024, (1, 64), device=DEV)
    with torch.no_grad():
        l1, l2 = model(ids, loops=1).logits, model(ids, loops=2).logits
        assert not torch.allclose(l1, l2)
        assert torch.equal(model(ids).logits, model(ids, loops=TINY["max_loops"]).logits)


def test_only_last_loop_is_tracked_by_autograd():
    model = _tiny()
    seen = {}
    for i, layer in enumerate(model.recurrent_layers):
        layer.mixer.register_forward_hook(lambda m, inp, out, i=i: seen.setdefault(i, []).append(out.requires_grad))
    ids = torch.randint(0, 1024, (1, 64), device=DEV)
    model(ids, labels=ids, loops=3).loss.backward()
    assert all(flags == [False, False, True] for flags in seen.values())


def test_loss_matches_manual_next_token_cross_entropy():
    model = _tiny()
    ids = torch.randint(0, 1024, (2, 64), device=DEV)
    out = model(ids, labels=ids, loops=2, return_logits=True)
    expected = F.cross_entropy(out.logits[:, :-1].reshape(-1, 1024).double(), ids[:, 1:].reshape(-1))
    assert abs(out.loss.item() - expected.item()) < 1e-5 * abs(expected.item())


def test_lm_head_is_tied_and_layer_is_identity_when_mixer_output_is_zero():
    from zenith_b200 import lm

    model = _tiny()
    assert model.lm_head.weight is model.embed.weight
    layer = lm.Layer(lm.ZenithConfig.from_dict(TINY)).to(DEV)
    torch.nn.init.zeros_(layer.mixer.out_proj.weight)
    x = torch.randn(1, 64, 128, device=DEV)
    assert torch.allclose(layer(x), x)


def test_use_b200_layer_matches_oracle_mixer():
    """``use_b200_layer`` on a module with the reference Mamba3's attributes (in_proj, the packed
    layer body, out_proj), float32: output and the gradients of both projections and every layer
    parameter against the oracle's ``Mamba3.forward`` restatement, to 1e-4."""
    import zenith_b200
    from zenith_b200 import lm

    torch.manual_seed(5)
    cfg = dict(d_model=64, d_state=32, expand=2, headdim=16, chunk_size=32)
    m = lm.Mamba3(64, 32, 2, 16, 32).to(DEV)
    with torch.no_grad():
        for prm in (m.B_bias, m.C_bias, m.B_norm.weight, m.C_norm.weight, m.D):
            prm.add_(0.2 * torch.randn_like(prm))
    zenith_b200.use_b200_layer(m, scan_dtype=torch.float32)
    u = torch.randn(2, 96, 64, device=DEV)
    dout = torch.randn(2, 96, 64, device=DEV)
    out = m(u)
    out.backward(dout)
    params = {"mixer." + n: t.detach().cpu() for n, t in m.named_parameters()}
    leaves = {n: t.double().requires_grad_(True) for n, t in params.items()}
    ref = lm_oracle.mixer(leaves, "mixer.", u.cpu().double(), dict(cfg, vocab_size=0))
    ref.backward(dout.cpu().double())
    assert max_rel_err(out.double().cpu(), ref.detach()) < 1e-4
    for n, prm in m.named_parameters():
        g = leaves["mixer." + n].grad
        assert max_rel_err(prm.grad.double().cpu(), g) < 1e-4, n


def test_train_step_folds_clipping_into_fused_adamw():
    """The fused path (the clip scale passed to the fused AdamW kernel as its gradient divisor) makes
    the same update as clip_grad_norm_ followed by a plain AdamW step, with clipping active."""
    from zenith_b200 import lm

    cfg = dict(vocab_size=256, d_model=64, d_state=16, expand=2, headdim=16, chunk_size=32, n_input=1,
               n_recurrent=1, n_output=1, max_loops=1)
    torch.manual_seed(0)
    a = lm.ZenithForCausalLM(cfg).to(DEV)
    b = lm.ZenithForCausalLM(cfg).to(DEV)
    b.load_state_dict(a.state_dict())
    opt_a = lm.make_optimizer(a, lr=1e-3)
    opt_b = torch.optim.AdamW(b.parameters(), lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, foreach=False)
    ids = torch.randint(0, 256, (2, 64), device=DEV)
    for _ in range(2):
        lm.train_step(a, opt_a, ids, loops=1, grad_clip=0.05, amp=False)
        lm.train_step(b, opt_b, ids, loops=1, grad_clip=0.05, amp=False)
    for (n, pa), (_, pb) in zip(a.named_parameters(), b.named_parameters()):
        assert torch.allclose(pa, pb, rtol=1e-5, atol=1e-7), n


# token-by-token inference from the layer caches (prefill + recurrent scan)

def test_stream_logits_match_the_full_forward():
    """A chunked prefill of 64 tokens then 32 tokens one at a time (layer caches: scan state,
    theta, previous k and x, per recurrent loop pass) reproduce the full forward's logits at
    every position, float32, to 1e-4; likewise with no prefill at all."""
    model = _tiny()
    ids = torch.randint(0, 1024, (2, 96), device=DEV)
    with torch.no_grad():
        full = model(ids, loops=2).logits
    stream = model.stream_logits(ids, prefill_len=64, loops=2)
    assert max_rel_err(stream.double().cpu(), full.double().cpu()) < 1e-4
    short = model.stream_logits(ids[:, :5], prefill_len=0, loops=2)
    assert max_rel_err(short.double().cpu(), full[:, :5].double().cpu()) < 1e-4


def test_generate_is_greedy_on_the_full_forward():
    """Each generated token is the argmax of the full forward's logits at the previous position
    (the prompt is 40 tokens: a 32-token prefill, then 8 prompt tokens one at a time)."""
    model = _tiny()
    prompt = torch.randint(0, 1024, (2, 40), device=DEV)
    out = model.generate(prompt, 12, loops=2)
    assert out.shape == (2, 52) and torch.equal(out[:, :40], prompt)
    padded = torch.cat((out, torch.zeros(2, 12, dtype=out.dtype, device=DEV)), dim=1)   # 64 tokens
    with torch.no_grad():
        logits = model(padded, loops=2).logits
    assert torch.equal(logits[:, 39:51].argmax(-1), out[:, 40:52])


def test_generate_with_a_cuda_graph_matches_eager():
    """The CUDA-graph single-token step gives the same tokens as the eager steps (fp32 and bf16
    autocast), with a prompt that leaves tokens to step through after the prefill."""
    model = _tiny()
    prompt = torch.randint(0, 1024, (3, 45), device=DEV)
    for amp in (False, True):
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=amp):
            eager = model.generate(prompt, 10, loops=2, cuda_graph=False)
            graphed = model.generate(prompt, 10, loops=2, cuda_graph=True)
        assert torch.equal(eager, graphed), amp
