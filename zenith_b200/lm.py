"""The Mamba-3 language model on the B200 kernels: a drop-in for the reference's looped causal LM
``ZenithForCausalLM`` (zenith/model.py:42-99) and its training step (zenith/train.py:99-111).

Same modules, parameter names and shapes as the reference (a reference ``state_dict`` loads as
it is), same forward semantics: embedding, input layers, ``loops`` passes of the shared
recurrent block of which only the last is tracked by autograd, output layers, final norm, tied
LM head, next-token cross-entropy.  What runs where:

- the residual add and the RMSNorm that reads it, forward and backward: ``zb_rmsnorm_fwd`` /
  ``zb_rmsnorm_bwd`` (one pass each; the layer output is added into the residual stream as it is
  normalised for the next layer);
- the Mamba-3 layer body between in_proj and out_proj: ``mamba3_layer_packed`` (prologue, the
  tcgen05 SSD scan, epilogue), reading the packed in_proj output and writing its gradient as one
  tensor;
- in_proj / out_proj / LM head GEMMs: cuBLAS through torch (bf16 under autocast, as the
  reference's ``train.py`` runs them), the weight gradients written in float32 by the GEMM;
- the next-token cross-entropy: row chunk by row chunk, ``zb_xent`` computes each row's loss and
  overwrites the logits with their gradient in the same pass, and the gradient GEMMs consume the
  chunk at once, so the logits never exist whole and no float32 logits or softmax are stored.

``train_step`` is one optimiser step (autocast forward, backward, gradient clipping, AdamW),
with the gradient all-reduce of ``DistributedDataParallel`` over NCCL when the model is wrapped.
"""

from __future__ import annotations

import ctypes
import dataclasses
import math
from contextlib import nullcontext
from typing import NamedTuple, Optional

import torch
import torch.nn as nn
from torch import Tensor

from . import _lib as L
from .mamba3 import LayerCache, _scan_dtype, mamba3_layer_packed, mamba3_layer_prefill, mamba3_layer_step


# ---------------------------------------------------------------------------------------------
# C ABI (include/zb_lm.h)

class NormArgs(ctypes.Structure):
    """ctypes mirror of ``zb_rmsnorm_args``."""

    _fields_ = (
        [("M", ctypes.c_int64), ("D", ctypes.c_int64), ("eps", ctypes.c_float)]
        + [(n, ctypes.c_int32) for n in ("x_dtype", "b_dtype", "u_dtype")]
        + [(n, ctypes.c_void_p) for n in ("a", "b", "s", "w", "u", "r", "du", "ds", "dsum", "dsum_b", "dw",
                                          "workspace")]
        + [("workspace_bytes", ctypes.c_uint64)]
    )


class XentArgs(ctypes.Structure):
    """ctypes mirror of ``zb_xent_args``."""

    _fields_ = [("M", ctypes.c_int64), ("V", ctypes.c_int64), ("ld", ctypes.c_int64), ("dtype", ctypes.c_int32),
                ("write_grad", ctypes.c_int32), ("ignore_index", ctypes.c_int64), ("logits", ctypes.c_void_p),
                ("labels", ctypes.c_void_p), ("loss", ctypes.c_void_p), ("lse", ctypes.c_void_p),
                ("status", ctypes.c_void_p)]


def _lib():
    lib = L.lib()
    if not getattr(lib, "_lm_typed", False):
        lib.zb_rmsnorm_workspace_bytes.restype = ctypes.c_uint64
        lib.zb_rmsnorm_workspace_bytes.argtypes = [ctypes.POINTER(NormArgs)]
        for fn in ("zb_rmsnorm_fwd", "zb_rmsnorm_bwd"):
            getattr(lib, fn).restype = ctypes.c_int
            getattr(lib, fn).argtypes = [ctypes.POINTER(NormArgs), ctypes.c_void_p]
        lib.zb_xent.restype = ctypes.c_int
        lib.zb_xent.argtypes = [ctypes.POINTER(XentArgs), ctypes.c_void_p]
        lib._lm_typed = True
    return lib


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _code(dt: torch.dtype) -> int:
    if dt not in (torch.float32, torch.bfloat16):
        raise TypeError(f"zenith_b200.lm: float32 or bfloat16 tensors, not {dt}")
    return L.DTYPE_CODE[dt]


# ---------------------------------------------------------------------------------------------
# residual add + RMSNorm

class _AddRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b, weight, eps, u_dtype):
        D = a.shape[-1]
        M = a.numel() // D
        dev = a.device
        w = weight.detach().float().contiguous()
        s = torch.empty_like(a) if b is not None else None
        u = torch.empty(a.shape, dtype=u_dtype, device=dev)
        r = torch.empty(M, dtype=torch.float32, device=dev)
        args = NormArgs(M=M, D=D, eps=float(eps), x_dtype=_code(a.dtype),
                        b_dtype=_code(b.dtype if b is not None else a.dtype), u_dtype=_code(u_dtype))
        args.a, args.b, args.s = a.data_ptr(), L.ptr(b), L.ptr(s)
        args.w, args.u, args.r = w.data_ptr(), u.data_ptr(), r.data_ptr()
        L.check(_lib().zb_rmsnorm_fwd(ctypes.byref(args), _stream(dev)), "zb_rmsnorm_fwd")
        ctx.save_for_backward(s if b is not None else a, w, r)
        ctx.meta = (float(eps), b.dtype if b is not None else None, weight.dtype)
        ctx.set_materialize_grads(False)
        return (s, u) if b is not None else u

    @staticmethod
    def backward(ctx, *grads):
        s, w, r = ctx.saved_tensors
        eps, b_dtype, w_dtype = ctx.meta
        ds, du = grads if b_dtype is not None else (None, grads[0])
        D = s.shape[-1]
        M = s.numel() // D
        dev = s.device
        if du is None:
            du = torch.zeros(s.shape, dtype=s.dtype, device=dev)
        du = du.contiguous()
        ds = ds.contiguous() if ds is not None else None
        dsum = torch.empty_like(s)
        dsum_b = torch.empty(s.shape, dtype=b_dtype, device=dev) if b_dtype not in (None, s.dtype) else None
        dw = torch.empty(D, dtype=torch.float32, device=dev)
        args = NormArgs(M=M, D=D, eps=eps, x_dtype=_code(s.dtype), b_dtype=_code(b_dtype or s.dtype),
                        u_dtype=_code(du.dtype))
        args.a, args.w, args.r = s.data_ptr(), w.data_ptr(), r.data_ptr()
        args.du, args.ds, args.dsum, args.dsum_b, args.dw = du.data_ptr(), L.ptr(ds), dsum.data_ptr(), L.ptr(dsum_b), dw.data_ptr()
        lib = _lib()
        nbytes = int(lib.zb_rmsnorm_workspace_bytes(ctypes.byref(args)))
        ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
        args.workspace, args.workspace_bytes = ws.data_ptr(), ws.numel()
        L.check(lib.zb_rmsnorm_bwd(ctypes.byref(args), _stream(dev)), "zb_rmsnorm_bwd")
        if b_dtype is None:
            return dsum, None, dw.to(w_dtype), None, None
        return dsum, dsum_b if dsum_b is not None else dsum, dw.to(w_dtype), None, None


def add_rmsnorm(a: Tensor, b: Optional[Tensor], weight: Tensor, eps: float = 1e-5,
                out_dtype: Optional[torch.dtype] = None):
    """``s = a + b`` and ``u = RMSNorm(s) = s rsqrt(mean(s^2) + eps) w`` (zenith/mamba3.py:8-15)
    in one pass; returns ``(s, u)``, or ``u`` alone when ``b`` is None.  ``a``: float32 or
    bfloat16 ``[..., D]``; ``b`` may be the other of the two; ``u`` in ``out_dtype`` (default
    ``a``'s).  The backward is one pass too and gives ``a`` and ``b`` the same gradient."""
    L.check_same_device(a.device, "add_rmsnorm", b=b, weight=weight)
    L.check_shapes("add_rmsnorm", b=(b, tuple(a.shape)), weight=(weight, (a.shape[-1],)))
    L.require_cuda(a.device, "add_rmsnorm")
    a = a.contiguous()
    b = b.contiguous() if b is not None else None
    with L.device_guard(a.device):
        return _AddRMSNorm.apply(a, b, weight, eps, out_dtype or a.dtype)


# ---------------------------------------------------------------------------------------------
# LM head + next-token cross-entropy

class _fp32_reductions:
    """cuBLAS may reduce split-K partial sums of a bf16 GEMM in bf16 (torch's default); the LM
    head's GEMMs sum over the vocabulary, so they keep those reductions in fp32."""

    def __enter__(self):
        self.prev = torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction
        torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False

    def __exit__(self, *exc):
        torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = self.prev


_CE_CHUNK_BYTES = 256 << 20  # logits of one row chunk of the fused loss


class _LinearCrossEntropy(torch.autograd.Function):
    """The loss is the graph's last operation, so its gradient with respect to the logits is
    known in the forward: each row chunk's logits are computed, turned into per-row losses and
    ``softmax - onehot`` in place by ``zb_xent``, and (when a gradient is wanted) fed straight to
    the two gradient GEMMs.  Only one chunk of logits exists at a time; the backward scales the
    stored gradients by ``dloss / n_valid``."""

    @staticmethod
    def forward(ctx, h, weight, labels, ignore_index, compute_dtype, need_grad):
        dev = h.device
        hc = h.to(compute_dtype)
        wc = weight.to(compute_dtype)
        M, V = hc.shape[0], wc.shape[0]
        rows = max(1, min(M, _CE_CHUNK_BYTES // (V * hc.element_size())))
        loss_rows = torch.empty(M, dtype=torch.float32, device=dev)
        dh = torch.empty_like(hc) if need_grad else None
        dw = None
        status = L.status_word(dev).data_ptr()
        lib = _lib()
        with _fp32_reductions():
            for r0 in range(0, M, rows):
                r1 = min(M, r0 + rows)
                logits = hc[r0:r1] @ wc.t()                                # [rows, V] (cuBLAS)
                args = XentArgs(M=r1 - r0, V=V, ld=logits.stride(0), dtype=_code(logits.dtype), write_grad=1,
                                ignore_index=int(ignore_index), logits=logits.data_ptr(),
                                labels=labels[r0:r1].data_ptr(), loss=loss_rows[r0:r1].data_ptr(), lse=None,
                                status=status)
                L.check(lib.zb_xent(ctypes.byref(args), _stream(dev)), "zb_xent")
                if not need_grad:
                    continue
                # the logits now hold softmax - onehot: this chunk's share of both gradients, unscaled
                torch.mm(logits, wc, out=dh[r0:r1])
                gt, hr = logits.t(), hc[r0:r1]
                if compute_dtype == torch.float32:
                    dw = gt @ hr if dw is None else dw.addmm_(gt, hr)
                else:   # accumulated in float32 by the GEMM itself
                    dw = (torch.mm(gt, hr, out_dtype=torch.float32) if dw is None
                          else torch.addmm(dw, gt, hr, out_dtype=torch.float32, out=dw))
        n_valid = (labels != ignore_index).sum().clamp_(min=1).to(torch.float32)
        ctx.save_for_backward(dh, dw, n_valid)
        ctx.dtypes = (h.dtype, weight.dtype)
        return loss_rows.sum() / n_valid

    @staticmethod
    def backward(ctx, gl):
        dh, dw, n_valid = ctx.saved_tensors
        scale = gl / n_valid
        gh = dh.float().mul_(scale).to(ctx.dtypes[0]) if ctx.needs_input_grad[0] else None
        gw = (dw * scale).to(ctx.dtypes[1]) if ctx.needs_input_grad[1] else None
        return gh, gw, None, None, None, None


def linear_cross_entropy(h: Tensor, weight: Tensor, labels: Tensor, ignore_index: int = -100,
                         compute_dtype: Optional[torch.dtype] = None) -> Tensor:
    """``F.cross_entropy(h @ weight.T, labels)`` (mean over rows whose label is not
    ``ignore_index``) without storing the logits: row chunk by row chunk (about 256 MB of logits
    each), the logits GEMM runs in ``compute_dtype`` (bf16 under CUDA autocast, else h's dtype),
    ``zb_xent`` turns each row into its loss and its gradient ``softmax - onehot`` in place, and
    the gradient GEMMs consume the chunk at once (the weight gradient accumulated in float32).
    ``h``: ``[M, d]``; ``weight``: ``[V, d]``; ``labels``: ``[M]`` int64."""
    if compute_dtype is None:
        ac = torch.is_autocast_enabled("cuda")
        compute_dtype = torch.get_autocast_dtype("cuda") if ac else h.dtype
    L.check_same_device(h.device, "linear_cross_entropy", weight=weight, labels=labels)
    if h.dim() != 2 or weight.dim() != 2:
        raise ValueError(f"linear_cross_entropy: h [M, d] and weight [V, d], got {tuple(h.shape)}, {tuple(weight.shape)}")
    L.check_shapes("linear_cross_entropy", weight=(weight, (weight.shape[0], h.shape[1])), labels=(labels, (h.shape[0],)))
    L.require_cuda(h.device, "linear_cross_entropy")
    labels = labels.contiguous().to(torch.int64)
    need_grad = torch.is_grad_enabled() and (h.requires_grad or weight.requires_grad)
    with torch.autocast("cuda", enabled=False), L.device_guard(h.device):
        return _LinearCrossEntropy.apply(h.contiguous(), weight, labels, ignore_index, compute_dtype, need_grad)


# ---------------------------------------------------------------------------------------------
# modules (parameter names and shapes of zenith/mamba3.py:58-93 and zenith/model.py:12-77)

@dataclasses.dataclass
class ZenithConfig:
    """The reference's ``ZenithConfig`` fields (zenith/model.py:12-39)."""

    vocab_size: int = 32000
    d_model: int = 640
    d_state: int = 128
    expand: int = 2
    headdim: int = 64
    chunk_size: int = 64
    n_input: int = 4
    n_recurrent: int = 16
    n_output: int = 4
    max_loops: int = 4
    tie_word_embeddings: bool = True

    @classmethod
    def from_dict(cls, d: dict) -> "ZenithConfig":
        names = {f.name for f in dataclasses.fields(cls)}
        return cls(**{k: v for k, v in d.items() if k in names})


class RMSNorm(nn.Module):
    """zenith/mamba3.py:8-15 (weight ``[dim]``, eps 1e-5)."""

    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: Tensor) -> Tensor:
        return add_rmsnorm(x, None, self.weight, self.eps)


class _AutocastLinear(torch.autograd.Function):
    """``x @ w.T`` as bf16 autocast runs it (bf16 operands, bf16 output), except that the weight
    gradient comes out of the GEMM in float32 (cuBLAS with an fp32 output) instead of as a bf16
    tensor cast up to the float32 parameter's dtype in a separate pass."""

    @staticmethod
    def forward(ctx, x, w):
        xb, wb = x.to(torch.bfloat16), w.to(torch.bfloat16)
        ctx.save_for_backward(xb, wb)
        ctx.x_dtype = x.dtype
        return xb @ wb.t()

    @staticmethod
    def backward(ctx, gy):
        xb, wb = ctx.saved_tensors
        g2 = gy.reshape(-1, gy.shape[-1]).to(torch.bfloat16)
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = (g2 @ wb).view(xb.shape).to(ctx.x_dtype)
        if ctx.needs_input_grad[1]:
            dw = torch.mm(g2.t(), xb.reshape(-1, xb.shape[-1]), out_dtype=torch.float32)
        return dx, dw


def _proj(lin: nn.Linear, x: Tensor) -> Tensor:
    """A bias-free projection: ``_AutocastLinear`` for a float32 weight under CUDA bf16 autocast
    with gradients on, else the module itself."""
    w = lin.weight
    if (x.is_cuda and w.dtype == torch.float32 and torch.is_grad_enabled() and torch.is_autocast_enabled("cuda")
            and torch.get_autocast_dtype("cuda") == torch.bfloat16):
        with torch.autocast("cuda", enabled=False):
            return _AutocastLinear.apply(x, w)
    return lin(x)


class Mamba3(nn.Module):
    """The reference ``Mamba3`` mixer (zenith/mamba3.py:58-120) on the fused layer body."""

    def __init__(self, d_model, d_state=128, expand=2, headdim=64, chunk_size=64, dt_min=1e-3, dt_max=1e-1,
                 dt_init_floor=1e-4, A_floor=1e-4):
        super().__init__()
        self.d_state, self.headdim, self.chunk_size, self.A_floor = d_state, headdim, chunk_size, A_floor
        self.d_inner = expand * d_model
        self.nheads = self.d_inner // headdim
        self.num_angles = d_state // 4
        n_in = 2 * self.d_inner + 2 * d_state + 3 * self.nheads + self.num_angles
        self.in_proj = nn.Linear(d_model, n_in, bias=False)
        self.out_proj = nn.Linear(self.d_inner, d_model, bias=False)
        dt = torch.exp(torch.rand(self.nheads) * (math.log(dt_max) - math.log(dt_min)) + math.log(dt_min))
        dt = dt.clamp(min=dt_init_floor)
        self.dt_bias = nn.Parameter(dt + torch.log(-torch.expm1(-dt)))   # inverse softplus (mamba3.py:87-89)
        self.B_bias = nn.Parameter(torch.ones(self.nheads, d_state))
        self.C_bias = nn.Parameter(torch.ones(self.nheads, d_state))
        self.B_norm = RMSNorm(d_state)
        self.C_norm = RMSNorm(d_state)
        self.D = nn.Parameter(torch.ones(self.nheads))

    def forward(self, u: Tensor) -> Tensor:
        Bsz, T, _ = u.shape
        zxbc = _proj(self.in_proj, u)
        if zxbc.dtype not in (torch.float32, torch.bfloat16):
            zxbc = zxbc.float()
        y = mamba3_layer_packed(zxbc, self.dt_bias, self.B_bias, self.C_bias, self.B_norm.weight,
                                self.C_norm.weight, self.D, self.nheads, self.headdim, self.d_state, self.A_floor,
                                self.chunk_size, self.B_norm.eps)
        return _proj(self.out_proj, y.reshape(Bsz, T, self.d_inner))


class Layer(nn.Module):
    """``x + mixer(norm(x))`` (zenith/model.py:42-49)."""

    def __init__(self, cfg: ZenithConfig):
        super().__init__()
        self.norm = RMSNorm(cfg.d_model)
        self.mixer = Mamba3(cfg.d_model, cfg.d_state, cfg.expand, cfg.headdim, cfg.chunk_size)

    def forward(self, x: Tensor) -> Tensor:
        s, delta = run_layers([self], x)
        return s + delta


def _u_dtype(x: Tensor) -> torch.dtype:
    """The in_proj input dtype: the autocast dtype when CUDA autocast is on (in_proj would cast
    to it), else the residual stream's."""
    return torch.get_autocast_dtype("cuda") if torch.is_autocast_enabled("cuda") else x.dtype


def run_layers(layers, x: Tensor, delta: Optional[Tensor] = None):
    """``x = x + layer.mixer(layer.norm(x))`` for each layer, with every residual add fused into
    the RMSNorm of the next layer.  Returns ``(s, delta)`` with the stack's output ``s + delta``
    (the last add is left to the caller, to fuse it with whatever reads it)."""
    for layer in layers:
        if delta is None:
            u = add_rmsnorm(x, None, layer.norm.weight, layer.norm.eps, _u_dtype(x))
        else:
            x, u = add_rmsnorm(x, delta, layer.norm.weight, layer.norm.eps, _u_dtype(x))
        delta = layer.mixer(u)
    return x, delta


class LMOutput(NamedTuple):
    loss: Optional[Tensor]
    logits: Optional[Tensor]


class ZenithForCausalLM(nn.Module):
    """The reference's looped Mamba-3 LM (zenith/model.py:52-99) on the B200 kernels.  With
    labels the loss comes from ``linear_cross_entropy`` and ``logits`` is None unless
    ``return_logits`` (the fused loss never stores them); without labels the logits are
    returned."""

    def __init__(self, config):
        super().__init__()
        cfg = config if isinstance(config, ZenithConfig) else ZenithConfig.from_dict(
            config if isinstance(config, dict) else vars(config))
        self.config = cfg
        self.embed = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.input_layers = nn.ModuleList(Layer(cfg) for _ in range(cfg.n_input))
        self.recurrent_layers = nn.ModuleList(Layer(cfg) for _ in range(cfg.n_recurrent))
        self.output_layers = nn.ModuleList(Layer(cfg) for _ in range(cfg.n_output))
        self.recurrent_norm = RMSNorm(cfg.d_model)
        self.norm = RMSNorm(cfg.d_model)
        self.lm_head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)
        if cfg.tie_word_embeddings:
            self.lm_head.weight = self.embed.weight
        self.reset_parameters()

    def reset_parameters(self, std: float = 0.02):
        """Linear and embedding weights N(0, 0.02), as the reference's post_init leaves them."""
        with torch.no_grad():
            for m in self.modules():
                if isinstance(m, (nn.Linear, nn.Embedding)):
                    m.weight.normal_(0.0, std)

    def get_input_embeddings(self):
        return self.embed

    def get_output_embeddings(self):
        return self.lm_head

    @torch.no_grad()
    def stream_logits(self, input_ids: Tensor, prefill_len: Optional[int] = None,
                      loops: Optional[int] = None) -> Tensor:
        """The logits of every position, computed the way ``generate`` computes them: a chunked
        prefill of the first ``prefill_len`` tokens (a multiple of chunk_size; default the longest
        such prefix), then the remaining tokens one at a time from the layer caches (the scan in its
        recurrent form, ``zb_ssd_decode``)."""
        loops = loops or self.config.max_loops
        T, L = input_ids.shape[1], self.config.chunk_size
        prefill_len = T // L * L if prefill_len is None else prefill_len
        caches: dict = {}
        outs = [_Generation.forward(self, input_ids[:, :prefill_len], caches, loops)] if prefill_len else []
        for t in range(prefill_len, T):
            outs.append(_Generation.forward(self, input_ids[:, t:t + 1], caches, loops))
        return torch.cat(outs, dim=1)

    @torch.no_grad()
    def generate(self, input_ids: Tensor, max_new_tokens: int, loops: Optional[int] = None,
                 cuda_graph: bool = True) -> Tensor:
        """Greedy decoding: the prompt is prefilled (its longest chunk_size-multiple prefix in one
        chunked pass, the rest token by token), then each new token is the argmax of the last
        logits and runs through the layers from their caches.  Returns the prompt followed by the
        new tokens.  The reference has no cache (model.py:79-99); this is the recurrent form of
        its forward.  With ``cuda_graph`` the single-token step (a few hundred launches) is
        captured once in a CUDA graph and replayed per token."""
        loops = loops or self.config.max_loops
        T, L = input_ids.shape[1], self.config.chunk_size
        pre = T // L * L
        caches: dict = {}
        logits = None
        if pre:
            logits = _Generation.forward(self, input_ids[:, :pre], caches, loops)
        for t in range(pre, T):
            logits = _Generation.forward(self, input_ids[:, t:t + 1], caches, loops)
        ids = [input_ids]
        step = None
        for i in range(max_new_tokens):
            nxt = logits[:, -1].argmax(-1, keepdim=True)
            ids.append(nxt)
            if i + 1 == max_new_tokens:
                break
            if cuda_graph and step is None and caches:
                step = _GraphStep(self, caches, loops, nxt)
            logits = step(nxt) if step is not None else _Generation.forward(self, nxt, caches, loops)
        return torch.cat(ids, dim=1)

    def forward(self, input_ids: Tensor, labels: Optional[Tensor] = None, loops: Optional[int] = None,
                return_logits: bool = False) -> LMOutput:
        cfg = self.config
        loops = loops or cfg.max_loops
        x = self.embed(input_ids)
        x, d = run_layers(self.input_layers, x)
        x = x + d if d is not None else x
        s = x
        for t in range(loops):
            with torch.no_grad() if t < loops - 1 else nullcontext():
                h = add_rmsnorm(s, x, self.recurrent_norm.weight, self.recurrent_norm.eps)[1]   # norm(s + x)
                h, d = run_layers(self.recurrent_layers, h)
                s = h + d if d is not None else h
        s, d = run_layers(self.output_layers, s)
        if d is None:
            u = add_rmsnorm(s, None, self.norm.weight, self.norm.eps, _u_dtype(s))
        else:
            u = add_rmsnorm(s, d, self.norm.weight, self.norm.eps, _u_dtype(s))[1]
        loss = logits = None
        if labels is not None:
            Bsz, T = labels.shape
            # next-token targets: position t predicts labels[t + 1]; the last position is ignored
            tgt = torch.cat((labels[:, 1:], torch.full_like(labels[:, :1], -100)), dim=1)
            loss = linear_cross_entropy(u.reshape(Bsz * T, -1), self.lm_head.weight, tgt.reshape(-1))
        if labels is None or return_logits:
            logits = self.lm_head(u)
        return LMOutput(loss, logits)


def _empty_cache(B, H, P, N, dtype, dev) -> LayerCache:
    """The cache before a sequence's first token: zero state, theta, k and x."""
    z = lambda *sh, dt=torch.float32: torch.zeros(*sh, dtype=dt, device=dev)  # noqa: E731
    return LayerCache(z(B, H, P, N), z(B, H, N // 4), z(B, H, N, dt=dtype), z(B, H, P, dt=dtype))


class _Generation:
    """Token-by-token inference for ZenithForCausalLM: the forward (model.py:79-93) on new tokens
    with one layer cache per (stack, layer, loop pass), since every pass of the shared recurrent
    block runs over the sequence with its own scan state."""

    @staticmethod
    def mixer(m: "Mamba3", u: Tensor, caches: dict, key) -> Tensor:
        Bsz, T, _ = u.shape
        zxbc = m.in_proj(u)
        if zxbc.dtype not in (torch.float32, torch.bfloat16):
            zxbc = zxbc.float()
        prm = (m.dt_bias, m.B_bias, m.C_bias, m.B_norm.weight, m.C_norm.weight, m.D)
        H, P, N = m.nheads, m.headdim, m.d_state
        if key not in caches:
            if T % m.chunk_size == 0:  # a chunked prefill
                out, caches[key] = mamba3_layer_prefill(zxbc, *prm, H, P, N, m.A_floor, m.chunk_size, m.B_norm.eps)
                return m.out_proj(out.reshape(Bsz, T, m.d_inner))
            caches[key] = _empty_cache(Bsz, H, P, N, _scan_dtype(zxbc, None), zxbc.device)
        out = mamba3_layer_step(zxbc, *prm, H, P, N, caches[key], m.A_floor, m.B_norm.eps)
        return m.out_proj(out.reshape(Bsz, T, m.d_inner))

    @staticmethod
    def forward(model: "ZenithForCausalLM", input_ids: Tensor, caches: dict, loops: int) -> Tensor:
        """Logits of the new tokens; ``caches`` is advanced."""
        def stack(name, layers, h, loop):
            for i, layer in enumerate(layers):
                u = add_rmsnorm(h, None, layer.norm.weight, layer.norm.eps, _u_dtype(h))
                h = h + _Generation.mixer(layer.mixer, u, caches, (name, i, loop)).to(h.dtype)
            return h

        x = stack("in", model.input_layers, model.embed(input_ids), 0)
        s = x
        for t in range(loops):
            h = add_rmsnorm(s, x, model.recurrent_norm.weight, model.recurrent_norm.eps)[1]
            s = stack("rec", model.recurrent_layers, h, t)
        s = stack("out", model.output_layers, s, 0)
        return model.lm_head(add_rmsnorm(s, None, model.norm.weight, model.norm.eps, _u_dtype(s)))


class _GraphStep:
    """One single-token generation step captured in a CUDA graph: the token goes into a static
    buffer, the replay runs every kernel of the step (advancing the layer caches in place, which
    the graph reads and writes at fixed addresses) and leaves the logits in a static buffer.  The
    eager warm-up that capture needs would advance the caches, so they are restored after it."""

    def __init__(self, model, caches: dict, loops: int, tok: Tensor):
        self.tok = tok.clone()
        saved = {k: (c.state.clone(), c.theta.clone(), c.k_prev.clone(), c.x_prev.clone()) for k, c in caches.items()}
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                _Generation.forward(model, self.tok, caches, loops)
        torch.cuda.current_stream().wait_stream(side)
        for k, c in caches.items():
            for dst, src in zip((c.state, c.theta, c.k_prev, c.x_prev), saved[k]):
                dst.copy_(src)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.logits = _Generation.forward(model, self.tok, caches, loops)

    def __call__(self, tok: Tensor) -> Tensor:
        self.tok.copy_(tok)
        self.graph.replay()
        return self.logits


def load_reference_state_dict(model: ZenithForCausalLM, state_dict: dict):
    """Load a reference ``ZenithForCausalLM`` state_dict (same names; the tied ``lm_head.weight``
    may be present or not)."""
    sd = dict(state_dict)
    if model.config.tie_word_embeddings:
        sd.pop("lm_head.weight", None)
    missing, unexpected = model.load_state_dict(sd, strict=False)
    missing = [m for m in missing if not (m == "lm_head.weight" and model.config.tie_word_embeddings)]
    if missing or unexpected:
        raise KeyError(f"state_dict mismatch: missing {missing}, unexpected {unexpected}")


# ---------------------------------------------------------------------------------------------
# training step (zenith/train.py:99-111)

def train_step(model: nn.Module, opt: torch.optim.Optimizer, ids: Tensor, loops: int = 1, grad_clip: float = 1.0,
               amp: bool = True, labels: Optional[Tensor] = None) -> Tensor:
    """One optimiser step on a batch of token ids: bf16-autocast forward with ``labels=ids`` (or the
    given ``labels``, shifted inside the model like ids),
    backward (under ``DistributedDataParallel`` the gradient all-reduce runs during it), global
    gradient-norm clipping, the optimiser step.  Returns the loss (a device scalar, no sync).
    Raises ``SsdError`` when a kernel of an earlier step recorded an error in the device status
    word (a label outside the vocabulary, a timed-out wait), as soon as that is visible without
    a synchronisation: at the latest, the step after the faulty one has finished on the GPU."""
    L.poll_status(ids)  # an error an earlier step's kernels recorded (e.g. a label out of range)
    ctx = torch.autocast("cuda", dtype=torch.bfloat16) if amp else nullcontext()
    with ctx:
        loss = model(ids, labels=ids if labels is None else labels, loops=loops).loss
    loss.backward()
    fused = all(g.get("fused") for g in opt.param_groups) and isinstance(opt, torch.optim.Adam)
    if fused:
        # clip_grad_norm_'s scale (max_norm / (norm + 1e-6), at most 1) applied inside the fused
        # AdamW kernel, which divides each gradient by `grad_scale` as it reads it: one pass over
        # the gradients fewer than scaling them in place first
        grads = [q.grad for g in opt.param_groups for q in g["params"] if q.grad is not None]
        norm = torch.nn.utils.get_total_norm(grads, 2.0, foreach=True)
        opt.grad_scale = ((norm + 1e-6) / grad_clip).clamp_(min=1.0).to(torch.float32)
        try:
            opt.step()
        finally:
            del opt.grad_scale
    else:
        torch.nn.utils.clip_grad_norm_(model.parameters(), grad_clip, foreach=True)
        opt.step()
    opt.zero_grad(set_to_none=True)
    L.poll_status(ids)
    return loss.detach()


def make_optimizer(model: nn.Module, lr: float = 5e-4, weight_decay: float = 0.1) -> torch.optim.Optimizer:
    """AdamW with the reference's settings (train.py:89: betas (0.9, 0.95), eps 1e-8), fused CUDA."""
    return torch.optim.AdamW(model.parameters(), lr=lr, betas=(0.9, 0.95), eps=1e-8, weight_decay=weight_decay,
                             fused=True)
