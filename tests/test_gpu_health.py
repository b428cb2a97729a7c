"""Device-side failure detection: a bounded wait on a flag that nothing sets gives up after its
limit, records the timeout in the device error word and returns; the context stays usable.
(The wait is a global-memory acquire spin with a 0.2 s limit -- no trap, no unbounded loop.)"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_wait_probe_times_out_and_reports():
    from hrm_text_b200._native import cuda
    from hrm_text_b200.utils.errors import DeviceWaitTimeout, check_device_errors
    check_device_errors()  # start clean
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = cuda().wait_flag_probe(flag, 1, 0.2)  # nothing ever sets the flag
    assert int(status.item()) == 1
    with pytest.raises(DeviceWaitTimeout, match="site 99"):
        check_device_errors()
    # the context is still usable
    x = torch.randn(256, 256, device="cuda")
    assert torch.isfinite((x @ x).sum()).item()
    check_device_errors()


def test_wait_probe_sees_set_flag():
    from hrm_text_b200._native import cuda
    from hrm_text_b200.utils.errors import check_device_errors
    flag = torch.ones(1, dtype=torch.int32, device="cuda")
    status = cuda().wait_flag_probe(flag, 1, 0.2)
    assert int(status.item()) == 0
    check_device_errors()
