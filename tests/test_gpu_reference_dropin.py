"""The drop-in against the reference's own code, run live beside it on the GPU.

When the reference package is installed under baseline/_ref (``pip install --target``, the same
install the benchmark's reference arm times), these tests run the reference's functions and
modules on the GPU next to this library, on identical inputs, in float32 with TF32 off:

- the reference's ``ssd`` (zenith/mamba3.py:30-56) under autograd against ``zenith_b200.ssd`` on
  the whole model-scale layer workload (B8 T2048 H24 P64 N128, chunk 64), which the CPU oracle
  cannot finish in seconds: y and all eight input gradients, bf16 vectors against the reference
  in float32 on the same bf16-rounded values (2e-2) and float32 vectors (1e-4);
- the same at chunk 128 on a long sequence (T 16384), the chunk size of the long-context
  workload;
- the reference's ``Mamba3`` block (zenith/mamba3.py:59-119) with its scan hook set by
  ``use_b200_scan``, and with its forward routed through the fused layer body by
  ``use_b200_layer``, against the untouched block: output, input gradient and every parameter
  gradient (1e-4);
- the reference's ``ZenithForCausalLM`` (zenith/model.py:52-99) with ``use_b200_scan``, and this
  library's ``ZenithForCausalLM`` loading the reference model's state_dict, against the untouched
  reference model: loss, logits and every parameter gradient (1e-4).

Error metric: max |out - ref| / max |ref| per tensor.  Skipped when the reference is not installed.
"""
import copy
import pathlib
import sys

import pytest
import torch

import zenith_b200
from zenith_b200.synthetic import SHAPES, SsdShape, make_inputs

pytestmark = pytest.mark.gpu

ROOT = pathlib.Path(__file__).resolve().parent.parent
NAMES = ("x", "q", "k", "kp", "xp", "adt", "gamma", "beta")
VEC = ("x", "q", "k", "kp", "xp")


def _reference():
    """The installed reference package (``zenith`` with ``mamba3`` and ``model``)."""
    path = ROOT / "baseline" / "_ref"
    if not (path / "zenith" / "mamba3.py").exists():
        pytest.skip("the reference is not installed under baseline/_ref")
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))
    import zenith
    import zenith.mamba3  # noqa: F401
    import zenith.model  # noqa: F401

    return zenith


@pytest.fixture(autouse=True)
def _full_fp32_matmuls():
    """The reference runs as the float32 reference: no TF32 in its matmuls."""
    saved = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32, torch.get_float32_matmul_precision())
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = saved[0], saved[1]
    torch.set_float32_matmul_precision(saved[2])


def _rel(out: torch.Tensor, ref: torch.Tensor) -> float:
    """max |out - ref| / max |ref| in float64 on the device (max |out| where ref is all zeros)."""
    out, ref = out.detach().double(), ref.detach().to(out.device).double()
    denom = ref.abs().max().item()
    num = (out - ref).abs().max().item()
    return num / denom if denom > 0 else num


def _scan_against_reference(ref, shape: SsdShape, dtype: torch.dtype, tol: float):
    dev = torch.device("cuda")
    inp = make_inputs(shape, seed=0)
    ours = [(inp[n].to(dtype) if n in VEC else inp[n]).to(dev).requires_grad_() for n in NAMES]
    dy = inp["dy"].to(dtype).to(dev)
    del inp
    y = zenith_b200.ssd(*ours, shape.chunk)
    y.backward(dy)
    zenith_b200.check_status(dev)
    # the reference in float32 on the same (rounded) values
    theirs = [t.detach().float().requires_grad_() for t in ours]
    y_ref = ref.mamba3.ssd(*theirs, shape.chunk)
    y_ref.backward(dy.float())
    errs = {"y": _rel(y, y_ref)}
    errs.update({"d" + n: _rel(a.grad, b.grad) for n, a, b in zip(NAMES, ours, theirs)})
    bad = {k: v for k, v in errs.items() if not v < tol}
    assert not bad, f"{shape} {dtype}: {bad} (all: {errs})"


@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 2e-2), (torch.float32, 1e-4)], ids=["bf16", "fp32"])
def test_whole_layer_workload_matches_the_reference_ssd(dtype, tol):
    _scan_against_reference(_reference(), SHAPES["layer"], dtype, tol)


def test_chunk128_long_sequence_matches_the_reference_ssd():
    _scan_against_reference(_reference(), SsdShape(1, 16384, 4, 64, 128, 4, 128), torch.bfloat16, 2e-2)


def _grads(module: torch.nn.Module, extra: dict) -> dict:
    out = dict(extra)
    out.update({n: p.grad for n, p in module.named_parameters() if p.grad is not None})
    return out


def _compare(ours: dict, theirs: dict, tol: float, what: str):
    assert set(ours) == set(theirs), (what, sorted(set(ours) ^ set(theirs)))
    errs = {k: _rel(ours[k], v) for k, v in theirs.items()}
    bad = {k: v for k, v in errs.items() if not v < tol}
    assert not bad, f"{what}: {bad}"


@pytest.mark.parametrize("route", ["scan_hook", "fused_layer_body"])
def test_reference_mamba3_block_on_the_b200_path(route):
    ref = _reference()
    from zenith_b200.mamba3 import use_b200_layer

    dev = torch.device("cuda")
    torch.manual_seed(0)
    block = ref.mamba3.Mamba3(768, d_state=128, expand=2, headdim=64, chunk_size=64).to(dev)
    ours = copy.deepcopy(block)
    if route == "scan_hook":
        assert zenith_b200.use_b200_scan(ours) == 1
    else:
        use_b200_layer(ours, torch.float32)
    g = torch.Generator().manual_seed(1)
    u = torch.randn(2, 512, 768, generator=g).to(dev)
    gout = torch.randn(2, 512, 768, generator=g).to(dev)
    res = []
    for m in (block, ours):
        uu = u.clone().requires_grad_()
        out = m(uu)
        out.backward(gout)
        res.append((out.detach(), _grads(m, {"u": uu.grad})))
    zenith_b200.check_status(dev)
    assert _rel(res[1][0], res[0][0]) < 1e-4
    _compare(res[1][1], res[0][1], 1e-4, route)


@pytest.mark.parametrize("tying", ["as_installed", "tied"])
def test_reference_lm_on_the_b200_scan_and_this_librarys_lm_on_its_weights(tying):
    """``as_installed``: the reference model as the installed transformers builds it (transformers
    5.x leaves lm_head untied: the reference's config has no ``tie_word_embeddings``);
    ``tied``: lm_head sharing the embedding, as zenith/model.py declares (``_tied_weights_keys``)."""
    ref = _reference()
    dev = torch.device("cuda")
    cfg = ref.model.ZenithConfig(vocab_size=512, d_model=256, d_state=64, expand=2, headdim=64, chunk_size=64,
                                 n_input=1, n_recurrent=2, n_output=1, max_loops=2)
    torch.manual_seed(0)
    model = ref.model.ZenithForCausalLM(cfg)
    if tying == "tied":
        model.lm_head.weight = model.embed.weight
    tied = model.lm_head.weight is model.embed.weight
    model.to(dev)
    patched = copy.deepcopy(model)
    assert zenith_b200.use_b200_scan(patched) == 4
    lib_lm = zenith_b200.ZenithForCausalLM({**cfg.to_dict(), "tie_word_embeddings": tied})
    from zenith_b200.lm import load_reference_state_dict

    load_reference_state_dict(lib_lm, model.state_dict())
    lib_lm.to(dev)
    ids = torch.randint(0, 512, (2, 256), generator=torch.Generator().manual_seed(2)).to(dev)
    res = {}
    for name, m in (("reference", model), ("scan_hook", patched), ("library_lm", lib_lm)):
        kw = {"return_logits": True} if m is lib_lm else {}
        out = m(ids, labels=ids, loops=2, **kw)
        out.loss.backward()
        res[name] = (out.loss.detach(), out.logits.detach(), _grads(m, {}))
    zenith_b200.check_status(dev)
    loss0, logits0, grads0 = res["reference"]
    for name in ("scan_hook", "library_lm"):
        loss, logits, grads = res[name]
        assert abs(loss.item() - loss0.item()) / abs(loss0.item()) < 1e-5, name
        assert _rel(logits, logits0) < 1e-4, name
        _compare(grads, grads0, 1e-4, name)
