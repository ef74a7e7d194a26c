"""Load the golden fixtures written by tests/golden/make_golden.py."""
import pathlib

import numpy as np
import torch

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
NAMES = ("x", "q", "k", "kp", "xp", "adt", "gamma", "beta")
CASES = sorted(p.stem for p in GOLDEN.glob("*.npz") if not p.stem.startswith(("mamba3_", "lm_")))  # scan-boundary cases


def load(name):
    z = np.load(GOLDEN / f"{name}.npz")
    inp = {n: torch.from_numpy(z["in_" + n]) for n in NAMES + ("dy",)}
    out = {k[4:]: torch.from_numpy(z[k]) for k in z.files if k.startswith("out_")}
    return inp, out, int(z["chunk_size"])


MAMBA3_CASES = ("mamba3_small_f32", "mamba3_wide_f32", "mamba3_floor_f32")


def load_mamba3(name):
    """Inputs and parameters, upstream gradient, output and all gradients of one layer-body case
    (written from the reference ``Mamba3`` module by make_golden.py)."""
    z = np.load(GOLDEN / f"{name}.npz")
    tensors = {k[3:]: torch.from_numpy(z[k]) for k in z.files if k.startswith("in_") and k != "in_dout"}
    ref = {k[4:]: torch.from_numpy(z[k]) for k in z.files if k.startswith("out_")}
    meta = {"A_floor": float(z["A_floor"]), "chunk": int(z["chunk_size"]), "eps": float(z["eps"])}
    return tensors, torch.from_numpy(z["in_dout"]), ref, meta


LM_CASES = ("lm_small_f32",)


def load_lm(name):
    """Configuration, token ids, loop count, parameters (state_dict names, lm_head tied to embed),
    logits, loss and parameter gradients of one language-model case (from the reference
    ``ZenithForCausalLM`` by make_golden.py)."""
    z = np.load(GOLDEN / f"{name}.npz")
    cfg = {str(k): int(v) for k, v in zip(z["config_keys"], z["config_vals"])}
    params = {k[3:]: torch.from_numpy(z[k]) for k in z.files if k.startswith("in_")}
    grads = {k[5:]: torch.from_numpy(z[k]) for k in z.files if k.startswith("grad_")}
    return (cfg, torch.from_numpy(z["ids"]), int(z["loops"]), params, torch.from_numpy(z["out_logits"]),
            torch.from_numpy(z["out_loss"]), grads)
