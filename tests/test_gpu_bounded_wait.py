"""The streaming kernels' bounded waits give up, report and return.

A test hook (ATTNRES_TEST_WITHHOLD_COPY=<unit>) makes warp 0 of CTA 0 post the
byte count of one unit without issuing its copy, so that unit's mbarrier never
completes. The wait must run out (20 ms under the hook), set the status bit,
let the warp's other copies land, and return: the context stays usable and the
next launch without the hook is exact. Nothing faults or hangs the GPU.
"""
import pytest
import torch

from attnres_b200 import _native

pytestmark = pytest.mark.gpu

FULL_WAIT_TIMEOUT, DRAIN_TIMEOUT = 1, 4


def _read(values, keys, q):
    import attnres_b200

    return attnres_b200.lrid_attention_residual_read(values, keys, q, 1, 0.125, True)


@pytest.mark.parametrize("unit", [0, 3])
def test_withheld_copy_times_out_and_the_next_launch_is_exact(monkeypatch, unit):
    S, N, D, R = 9, 4096, 1024, 64
    torch.manual_seed(5)
    values = [torch.randn(1, N, D, device="cuda", dtype=torch.bfloat16) for _ in range(S)]
    keys = [torch.randn(1, N, R, device="cuda", dtype=torch.bfloat16) for _ in range(S)]
    q = torch.randn(1, R, device="cuda") * 0.02
    monkeypatch.setenv("ATTNRES_B200_PATH", "auto")
    _native.device_status(reset=True)
    ref = _read(values, keys, q)
    torch.cuda.synchronize()
    assert _native.device_status(reset=True) == 0

    monkeypatch.setenv("ATTNRES_TEST_WITHHOLD_COPY", str(unit))
    _read(values, keys, q)
    torch.cuda.synchronize()  # returns: the kernel gave up instead of hanging
    status = _native.device_status(reset=True)
    assert status & FULL_WAIT_TIMEOUT, f"status {status:#x}"
    assert status & DRAIN_TIMEOUT, f"status {status:#x}"  # the withheld stage also fails its drain wait

    monkeypatch.delenv("ATTNRES_TEST_WITHHOLD_COPY")
    again = _read(values, keys, q)
    torch.cuda.synchronize()
    assert _native.device_status(reset=True) == 0
    assert torch.equal(again, ref)
