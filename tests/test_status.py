"""Host logic of the deferred status check (zenith_b200._lib.StatusPoll), on the CPU: a device
error recorded by one call surfaces as SsdError in a later call once the asynchronous copy of the
status word has landed, without waiting for the GPU; the word is then cleared."""
import pytest
import torch

from zenith_b200 import _lib as L


class FakeEvent:
    """Stands in for a CUDA event: 'done' says whether the copy queued before it has landed."""

    done = True

    def record(self):
        pass

    def query(self):
        return FakeEvent.done


def _poll():
    return L.StatusPoll(torch.zeros(1, dtype=torch.int32), torch.zeros(1, dtype=torch.int32), FakeEvent)


def test_error_surfaces_in_the_call_after_its_copy_lands_and_is_cleared():
    FakeEvent.done = True
    p = _poll()
    p.poll()                      # step 1: fine, queues a copy of 0
    p.word[0] = 9                 # a kernel of step 2 records "label out of range"
    p.poll()                      # step 2's poll: the copy of step 1 said 0; queues a copy of 9
    with pytest.raises(L.SsdError, match="status 9"):
        p.poll()                  # step 3: the copy has landed and shows the error
    assert int(p.word[0]) == 0    # cleared, so the next step runs
    p.poll()
    p.poll()


def test_a_copy_still_in_flight_is_not_read_and_not_overwritten():
    FakeEvent.done = False
    p = _poll()
    p.poll()                      # queues a copy; it has not landed
    p.word[0] = 5
    p.poll()                      # must neither read the stale host value nor queue another copy
    assert int(p.host[0]) == 0
    FakeEvent.done = True
    p.poll()                      # the first copy (of 0) has landed: fine; queues a copy of 5
    with pytest.raises(L.SsdError, match="status 5"):
        p.poll()
