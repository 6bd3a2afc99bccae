"""dsmoe_clock_probe: two probes around GPU work give every SM's mean clock
over it; the median must be a plausible B200 SM clock."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_clock_probe_brackets_work():
    from dsmoe._lib import ClockProbe

    dev = torch.device("cuda", 0)
    a = torch.randn(4096, 4096, device=dev, dtype=torch.bfloat16)
    probe = ClockProbe(dev)
    probe.start()
    for _ in range(20):
        a = (a @ a).clamp_(-1, 1)
    probe.stop()
    torch.cuda.synchronize()
    mhz = probe.mhz()
    assert mhz is not None and 300.0 < mhz < 2500.0, mhz
    # (nearly) every SM got one of the probe's 4 x n_SM blocks, both times
    assert int((probe.a.view(-1, 2)[:, 1] > 0).sum()) >= 0.9 * probe.n
    assert int((probe.b.view(-1, 2)[:, 1] > 0).sum()) >= 0.9 * probe.n
