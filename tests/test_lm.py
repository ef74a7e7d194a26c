"""CPU checks of the language-model layer (zenith_b200.lm): the C ABI structs match
include/zb_lm.h, the module tree matches the reference's parameter names and shapes (a reference
state_dict loads as it is), the C2 training configuration has the expected size, and the training
step's gradient all-reduce keeps data-parallel replicas identical (gloo, two ranks).  No kernel runs."""
import os
import pathlib
import re

import pytest
import torch
import torch.multiprocessing as mp

from tests.golden_io import LM_CASES, load_lm
from zenith_b200 import lm

ROOT = pathlib.Path(__file__).resolve().parent.parent


def header_fields(struct: str):
    text = (ROOT / "include" / "zb_lm.h").read_text()
    body = text[: text.index("} " + struct + ";")]
    body = body[body.rindex("typedef struct {") + len("typedef struct {"):]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    names = []
    for line in body.splitlines():
        decl = line.strip().rstrip(";")
        if not decl:
            continue
        decl = re.sub(r"^(const\s+)?\w+\s*\*?", "", decl)
        names += [n.strip().lstrip("*") for n in decl.split(",")]
    return names


@pytest.mark.parametrize("struct,cls", [("zb_rmsnorm_args", lm.NormArgs), ("zb_xent_args", lm.XentArgs)])
def test_ctypes_structs_match_header(struct, cls):
    assert header_fields(struct) == [f[0] for f in cls._fields_]


@pytest.mark.parametrize("case", LM_CASES)
def test_reference_state_dict_loads(case):
    cfg, ids, loops, params, *_ = load_lm(case)
    model = lm.ZenithForCausalLM(cfg)
    ours = dict(model.named_parameters())
    assert set(ours) == set(params)
    for n, t in params.items():
        assert ours[n].shape == t.shape, n
    lm.load_reference_state_dict(model, params)
    for n, t in params.items():
        assert torch.equal(ours[n].detach(), t), n
    assert model.lm_head.weight is model.embed.weight


def test_training_configuration_size():
    """d_model 1536, expand 2, headdim 64 (48 heads), N 128, 24 layers, vocab 32000, tied."""
    cfg = lm.ZenithConfig(vocab_size=32000, d_model=1536, d_state=128, expand=2, headdim=64, chunk_size=64,
                          n_input=4, n_recurrent=16, n_output=4, max_loops=1)
    with torch.device("meta"):
        model = lm.ZenithForCausalLM(cfg)
    n = sum(p.numel() for p in model.parameters())
    # in_proj, out_proj, dt_bias + D, B_bias + C_bias, B_norm + C_norm, the layer norm
    per_layer = 1536 * (2 * 3072 + 2 * 128 + 3 * 48 + 32) + 3072 * 1536 + 2 * 48 + 2 * 48 * 128 + 2 * 128 + 1536
    assert n == 24 * per_layer + 32000 * 1536 + 2 * 1536
    assert 390e6 < n < 420e6
    assert model.input_layers[0].mixer.nheads == 48


class _Tiny(torch.nn.Module):
    """A CPU stand-in with the LM's call signature, for the data-parallel plumbing."""

    def __init__(self):
        super().__init__()
        torch.manual_seed(0)
        self.embed = torch.nn.Embedding(16, 8)
        self.proj = torch.nn.Linear(8, 16, bias=False)

    def forward(self, ids, labels=None, loops=None):
        logits = self.proj(self.embed(ids))
        loss = torch.nn.functional.cross_entropy(logits[:, :-1].reshape(-1, 16), labels[:, 1:].reshape(-1))
        return lm.LMOutput(loss, None)


def _ddp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        model = torch.nn.parallel.DistributedDataParallel(_Tiny())
        opt = torch.optim.AdamW(model.parameters(), lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
        g = torch.Generator().manual_seed(100 + rank)           # different data on every rank
        for _ in range(3):
            ids = torch.randint(0, 16, (2, 12), generator=g)
            lm.train_step(model, opt, ids, loops=1, grad_clip=1.0, amp=False)
        flat = torch.cat([p.detach().reshape(-1) for p in model.parameters()])
        gathered = [torch.empty_like(flat) for _ in range(world)]
        torch.distributed.all_gather(gathered, flat)
        q.put((rank, all(torch.equal(gathered[0], t) for t in gathered), float(flat.abs().sum())))
    finally:
        torch.distributed.destroy_process_group()


def test_train_step_keeps_replicas_identical():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_ddp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(same for _, same, _ in res)
    assert res[0][2] == res[1][2]


def test_lm_c_abi_rejects_bad_arguments_without_launching():
    """The LM entry points validate on the host and return a status (no kernel runs): NULL
    pointers, bad sizes and dtypes, a missing workspace."""
    import ctypes

    from zenith_b200 import _lib as L

    lib = lm._lib()
    a = lm.NormArgs(M=0, D=16, eps=1e-5, x_dtype=0, b_dtype=0, u_dtype=0)
    assert lib.zb_rmsnorm_fwd(ctypes.byref(a), None) == 1          # ZB_ERR_SHAPE
    a = lm.NormArgs(M=4, D=16, eps=1e-5, x_dtype=3, b_dtype=0, u_dtype=0)
    assert lib.zb_rmsnorm_fwd(ctypes.byref(a), None) == 2          # ZB_ERR_DTYPE (fp64)
    a = lm.NormArgs(M=4, D=16, eps=1e-5, x_dtype=0, b_dtype=0, u_dtype=0)
    assert lib.zb_rmsnorm_fwd(ctypes.byref(a), None) == 3          # ZB_ERR_LAYOUT (no a / w)
    a = lm.NormArgs(M=4, D=9000, eps=1e-5, x_dtype=0, b_dtype=0, u_dtype=0)
    assert lib.zb_rmsnorm_fwd(ctypes.byref(a), None) == 7          # ZB_ERR_UNSUPPORTED (D > 8192)
    a = lm.NormArgs(M=4, D=16, eps=1e-5, x_dtype=0, b_dtype=0, u_dtype=0)
    a.a, a.w, a.du, a.dsum, a.dw, a.r = 16, 16, 16, 16, 16, 16     # never dereferenced: the workspace check fails first
    assert lib.zb_rmsnorm_bwd(ctypes.byref(a), None) == 6          # ZB_ERR_WORKSPACE
    assert lib.zb_rmsnorm_workspace_bytes(ctypes.byref(lm.NormArgs(M=10, D=64))) >= 10 * 64 * 4
    x = lm.XentArgs(M=4, V=0, ld=0, dtype=1)
    assert lib.zb_xent(ctypes.byref(x), None) == 1                 # ZB_ERR_SHAPE
    x = lm.XentArgs(M=4, V=8, ld=8, dtype=1)
    assert lib.zb_xent(ctypes.byref(x), None) == 3                 # ZB_ERR_LAYOUT (no pointers)
    assert L.strerror(9).startswith("label outside")
