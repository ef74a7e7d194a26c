"""Failure detection on the GPU without a fault.  The library's bounded device-side waits (the
chained hand-off flag and the mbarrier phase wait, `csrc/common.cuh:wait_flag`,
`csrc/umma.cuh:mbar_wait`) give up after about a second on something that never completes,
record ZB_ERR_TIMEOUT in the device status word and return; the host turns the word into an
exception, and the CUDA context stays usable for the next scan.  `zb_wait_probe` runs each wait
on its own, on a flag nothing sets or an mbarrier nothing arrives on."""
import ctypes

import pytest
import torch

import zenith_b200
from oracle.ssd_oracle import max_rel_err, ssd_forward
from zenith_b200 import _lib as L

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")
FLAG_WAIT, MBAR_WAIT = 0, 1


def _probe(flag, status, which):
    lib = L.lib()
    lib.zb_wait_probe.restype = ctypes.c_int
    lib.zb_wait_probe.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    result = torch.zeros(2, dtype=torch.int32, device=DEV)
    rc = lib.zb_wait_probe(flag.data_ptr() if flag is not None else None, status.data_ptr(), result.data_ptr(),
                           which, torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == 0
    torch.cuda.synchronize(DEV)
    ret, us = result.tolist()
    return ret, us


def _zeros():
    return torch.zeros(1, dtype=torch.int32, device=DEV)


def test_flag_wait_gives_up_and_records_timeout():
    flag, status = _zeros(), _zeros()          # nothing ever sets the flag
    ret, us = _probe(flag, status, FLAG_WAIT)
    assert ret == 2                            # aborted
    assert status.item() == L.ZB_ERR_TIMEOUT
    assert 0.9e6 <= us < 10e6                  # about one second


def test_flag_wait_ends_at_once_on_ready_aborted_or_failed():
    flag, status = _zeros(), _zeros()
    flag.fill_(1)                              # predecessor published
    ret, us = _probe(flag, status, FLAG_WAIT)
    assert (ret, status.item()) == (1, 0) and us < 100_000
    flag.fill_(2)                              # predecessor aborted: pass it on, record nothing new
    ret, us = _probe(flag, status, FLAG_WAIT)
    assert (ret, status.item()) == (2, 0) and us < 100_000
    flag.zero_()
    status.fill_(L.ZB_ERR_TIMEOUT)             # another CTA already failed: stop without waiting it out
    ret, us = _probe(flag, status, FLAG_WAIT)
    assert (ret, status.item()) == (2, L.ZB_ERR_TIMEOUT) and us < 100_000


def test_mbarrier_wait_gives_up_and_records_timeout():
    status = _zeros()
    ret, us = _probe(None, status, MBAR_WAIT)  # one arrival expected, none made
    assert ret == 0
    assert status.item() == L.ZB_ERR_TIMEOUT
    assert 0.9e6 <= us < 10e6


def test_host_raises_on_the_status_word_and_the_context_stays_usable():
    from zenith_b200.synthetic import SsdShape, make_inputs

    _probe(_zeros(), L.status_word(DEV), FLAG_WAIT)   # the library's own status word
    with pytest.raises(zenith_b200.SsdError, match="status 5"):
        zenith_b200.check_status(DEV)
    zenith_b200.check_status(DEV)                      # the failed check reset it
    shape = SsdShape(1, 256, 4, 64, 128, 4, 64)
    inp = make_inputs(shape, seed=3)
    names = ("x", "q", "k", "kp", "xp", "adt", "gamma", "beta")
    args = [(inp[n].to(torch.bfloat16) if n in ("x", "q", "k", "kp", "xp") else inp[n]).to(DEV) for n in names]
    y = zenith_b200.ssd(*args, shape.chunk)
    zenith_b200.check_status(DEV)
    ref, _, _ = ssd_forward(*[t.cpu().double() for t in args], shape.chunk)
    assert max_rel_err(y, ref) < 2e-2
