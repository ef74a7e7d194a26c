"""CPU-only checks of the C ABI: the library loads, exports every symbol include/zb_ssd.h
declares, and its host-side validation/sizing logic behaves (no kernel is launched)."""
import ctypes
import pathlib
import re

import pytest
import torch

from zenith_b200 import _lib as L
from zenith_b200.ssd import _build_args

ROOT = pathlib.Path(__file__).resolve().parent.parent


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        names |= set(re.findall(r"^ZB_API\s+[\w\s\*]+?\b(zb_\w+)\s*\(", h.read_text(), flags=re.M))
    return names


def test_library_loads_and_exports_every_declared_symbol():
    lib = L.lib()
    declared = declared_symbols()
    assert declared, "no ZB_API declarations found"
    for name in declared:
        assert hasattr(lib, name), name
    assert set(L.EXPORTS) <= declared
    assert lib.zb_version() >= 100


def test_ctypes_struct_matches_header_field_order():
    text = (ROOT / "include" / "zb_ssd.h").read_text()
    body = text[text.index("typedef struct {\n  int64_t B"):]
    body = body[: body.index("} zb_ssd_args;")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    fields = []
    for line in body.splitlines():
        line = line.split("/*")[0].strip()
        if not line or line.startswith("typedef"):
            continue
        decl = line.rstrip(";")
        typ, names = decl.split(None, 1) if not decl.startswith("const") else (decl.rsplit(None, 1)[0], decl.rsplit(None, 1)[1])
        for n in names.split(","):
            fields.append(n.strip().lstrip("*"))
    assert fields == [f[0] for f in L.Args._fields_]


def _args(B=2, T=256, H=4, G=4, P=32, N=16, chunk=64, dtype=torch.float32):
    x = torch.zeros(B, T, H, P, dtype=dtype)
    q = torch.zeros(B, T, G, N, dtype=dtype)
    a = torch.zeros(B, T, H, dtype=torch.float64 if dtype == torch.float64 else torch.float32)
    return _build_args(x, q, q, q, x, a, a, a, chunk)


def test_sizing_rejects_length_not_multiple_of_chunk():
    lib = L.lib()
    assert lib.zb_ssd_states_bytes(ctypes.byref(_args(T=250, chunk=64))) == 0
    assert lib.zb_ssd_workspace_bytes(ctypes.byref(_args(T=250, chunk=64)), 0) == 0
    assert lib.zb_ssd_states_bytes(ctypes.byref(_args(H=4, G=3))) == 0


def test_sizing_scales_with_chunks_and_state():
    lib = L.lib()
    s1 = lib.zb_ssd_states_bytes(ctypes.byref(_args(T=256)))
    s2 = lib.zb_ssd_states_bytes(ctypes.byref(_args(T=512)))
    assert s1 > 0 and s2 > s1
    # every saved state holds P*N accumulator elements
    assert s1 % (32 * 16 * 4) == 0 or s1 % 256 == 0
    assert lib.zb_ssd_workspace_bytes(ctypes.byref(_args()), 1) > 0


def test_entry_points_validate_before_touching_the_gpu():
    lib = L.lib()
    a = _args(T=250, chunk=64)
    assert lib.zb_ssd_fwd(ctypes.byref(a), None) == L.ZB_ERR_SHAPE
    a = _args()
    a.status = None
    assert lib.zb_ssd_fwd(ctypes.byref(a), None) != 0
    assert lib.zb_strerror(L.ZB_ERR_TIMEOUT).decode().startswith("timed out")
    # the bounded-wait probe: missing pointers or an unknown wait are refused before any launch
    probe = lib.zb_wait_probe
    probe.restype = ctypes.c_int
    probe.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    assert probe(None, 16, 16, 0, None) == 3     # ZB_ERR_LAYOUT: the flag wait needs a flag
    assert probe(16, None, 16, 0, None) == 3     # no status word
    assert probe(16, 16, None, 1, None) == 3     # no result buffer
    assert probe(16, 16, 16, 2, None) == 7       # ZB_ERR_UNSUPPORTED: no such wait


def test_python_entry_raises_reference_assertion_message():
    from zenith_b200 import ssd

    t = torch.zeros(1, 10, 1, 2)
    n = torch.zeros(1, 10, 1, 3)
    a = torch.zeros(1, 10, 1)
    with pytest.raises(AssertionError, match="multiple of chunk_size"):
        ssd(t, n, n, n, t, a, a, a, 4)


def test_python_entry_has_no_cpu_path():
    from zenith_b200 import ssd

    t = torch.zeros(1, 8, 1, 2)
    n = torch.zeros(1, 8, 1, 3)
    a = torch.zeros(1, 8, 1)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        ssd(t, n, n, n, t, a, a, a, 4)


def test_prepare_inputs_unifies_dtypes_and_inner_contiguity():
    from zenith_b200 import prepare_inputs

    x = torch.zeros(1, 8, 2, 4, dtype=torch.bfloat16)
    q = torch.zeros(1, 8, 2, 6, dtype=torch.float32)
    xt = torch.zeros(1, 8, 4, 2).transpose(2, 3)  # innermost stride 2
    a = torch.zeros(1, 8, 2, dtype=torch.float64)
    out = prepare_inputs(x, q, q, q, xt, a, a, a)
    assert all(t.dtype == torch.float32 for t in out[:5])
    assert all(t.dtype == torch.float32 for t in out[5:])
    assert all(t.stride(-1) == 1 for t in out[:5])
    out = prepare_inputs(*(t.double() for t in (x, q, q, q, xt)), a.float(), a, a)
    assert all(t.dtype == torch.float64 for t in out)
