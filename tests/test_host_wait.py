"""Host-side accounting of the blocking device-to-host reads (no GPU): the
wrapper's size reads and event waits go through read_back / wait_event, which
add their blocked time and count to ``host_wait`` when the benchmark installs it
and do nothing else otherwise."""

import torch

from gsplat_b200.cuda import _backend as B


class _Event:
    """Stands in for a CUDA event."""

    def __init__(self):
        self.waits = 0

    def synchronize(self):
        self.waits += 1


def test_read_back_and_wait_event_accounting():
    t = torch.tensor([3, -4, 5], dtype=torch.int32)
    assert B.host_wait is None
    assert B.read_back(t) == [3, -4, 5]
    ev = _Event()
    B.wait_event(ev)
    assert ev.waits == 1
    B.host_wait = [0.0, 0]
    try:
        assert B.read_back(t) == [3, -4, 5]
        B.wait_event(ev)
        assert ev.waits == 2
        assert B.host_wait[1] == 2 and B.host_wait[0] >= 0.0
    finally:
        B.host_wait = None
