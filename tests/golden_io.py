"""Load the golden fixtures written by tests/golden/make_golden.py."""
import pathlib

import numpy as np
import torch

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
NAMES = ("x", "q", "k", "kp", "xp", "adt", "gamma", "beta")
CASES = sorted(p.stem for p in GOLDEN.glob("*.npz"))


def load(name):
    z = np.load(GOLDEN / f"{name}.npz")
    inp = {n: torch.from_numpy(z["in_" + n]) for n in NAMES + ("dy",)}
    out = {k[4:]: torch.from_numpy(z[k]) for k in z.files if k.startswith("out_")}
    return inp, out, int(z["chunk_size"])
